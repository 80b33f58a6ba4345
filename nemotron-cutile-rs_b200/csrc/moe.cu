// moe.cu — the MoE layer (MoeLayer::forward_into, nemotron-nn/src/moe.rs:154-249)
// as a chain of device kernels on one stream:
//   router GEMM (tcgen05, f32-accurate via a 3-way bf16 split of the weight)
//   -> top-k routing -> expert histogram/permutation -> token gather
//   -> grouped up-projection (+relu2 epilogue) -> grouped down-projection
//   -> shared expert (two dense GEMMs) -> rank-ordered combine.
#include <stdlib.h>

#include "ep.h"
#include "gemm_tc.h"
#include "route.h"

namespace nk {

constexpr int kMoeBN = 256;
constexpr int kRouterMaxSplits = 16;

// Grouped tile lists over row segments: segment s holds seg_rows[s]
// contiguous rows (segments back to back) for expert seg_expert[s] (identity
// when null).  Each segment gets ceil(n_out/fh) feature tiles of fh rows x
// ceil(rows/BN) token tiles, feature-major within the segment.  Block b
// builds list b (n_out[b], tiles[b], count[b]): the up and the down
// projection in one launch.  n_seg <= 1024; after a scan of the per-segment
// tile counts every thread writes tiles, locating its segment by binary search.
struct TileLists {
  int n_out[2];
  TcTile *tiles[2];
  int *count[2];
  // list 1 (the down projection) with seg_yoff: segment s's rows go to rank
  // s / seg_per_rank's buffer from row seg_yoff[s] (expert-parallel return)
  const int32_t *seg_yoff;
  int seg_per_rank;
  // list 1 starts at segment seg_rot and wraps: each rank starts its return
  // at its own rank's rows, so at any time every rank receives from one peer
  int seg_rot;
  // list 0 (the up projection) of an in-kernel pull: the same rotation, and
  // each tile carries its segment (whose rows it waits for)
  int pull;
};

__global__ void __launch_bounds__(1024) build_tiles_kernel(const int32_t *__restrict__ seg_rows,
                                                           const int32_t *__restrict__ seg_expert,
                                                           int n_seg, int bn, int fh,
                                                           TileLists lists) {
  __shared__ int tiles_sc[1024];
  __shared__ int rows_sc[1024];
  const int s = threadIdx.x;
  const int n_out = lists.n_out[blockIdx.x];
  TcTile *tiles = lists.tiles[blockIdx.x];
  const int ft = (n_out + fh - 1) / fh;
  const int rot = n_seg > 0 && (blockIdx.x == 1 || lists.pull) ? lists.seg_rot % n_seg : 0;
  const int c = s < n_seg ? seg_rows[s] : 0;  // rows scan: segment order
  const int ps = s < n_seg ? (s + rot < n_seg ? s + rot : s + rot - n_seg) : 0;
  const int cp = s < n_seg ? seg_rows[ps] : 0;  // tiles scan: list order
  tiles_sc[s] = ft * ((cp + bn - 1) / bn);
  rows_sc[s] = c;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {  // inclusive scans of tiles and rows
    const int v = s >= o ? tiles_sc[s - o] : 0;
    const int r = s >= o ? rows_sc[s - o] : 0;
    __syncthreads();
    tiles_sc[s] += v;
    rows_sc[s] += r;
    __syncthreads();
  }
  const int total = tiles_sc[1023];
  if (s == 0) *lists.count[blockIdx.x] = total;
  for (int j = s; j < total; j += 1024) {
    int lo = 0, hi = n_seg - 1;  // first segment whose inclusive tile sum exceeds j
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (tiles_sc[mid] > j) hi = mid;
      else lo = mid + 1;
    }
    const int seg = lo + rot < n_seg ? lo + rot : lo + rot - n_seg;
    const int rows = seg_rows[seg];
    const int tt = (rows + bn - 1) / bn;
    const int local = j - (tiles_sc[lo] - ft * tt);
    const int f = local / tt, t = local - f * tt;
    const int e = seg_expert ? seg_expert[seg] : seg;
    TcTile tile;
    tile.w_row = e * n_out + f * fh;
    tile.x_row = rows_sc[seg] - rows + t * bn;
    const int fv = n_out - f * fh, tv = rows - t * bn;
    tile.valid = ((fv > fh ? fh : fv) << 16) | (tv > bn ? bn : tv);
    tile.out_col0 = f * fh;
    if (blockIdx.x == 1 && lists.seg_yoff) {
      tile.y_rank = seg / lists.seg_per_rank;
      tile.y_row = lists.seg_yoff[seg] + t * bn;
    }
    if (blockIdx.x == 0 && lists.pull) tile.src = seg;
    tiles[j] = tile;
  }
}

// out[t, c] = 0 (+ shared[t, c]) + Σ_r w[t, r] * y[slot_pos[t*k + r], c], each
// product and sum rounded in f32 in rank order (moe.rs:195-246).  One block per
// token; each thread owns 8 consecutive columns (16-byte loads; H % 8 == 0).
__device__ __forceinline__ void bf16x8_to_f32(const uint4 &v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

template <bool OUT_F32>
__global__ void __launch_bounds__(128) combine_kernel(const __nv_bfloat16 *__restrict__ y,
                                                      const __nv_bfloat16 *__restrict__ shared,
                                                      const float *__restrict__ w,
                                                      const int32_t *__restrict__ slot_pos,
                                                      int64_t H, int top_k, void *__restrict__ out) {
  const int64_t t = blockIdx.x;
  __shared__ int32_t pos[32];
  __shared__ float wt[32];
  if (threadIdx.x < top_k) {
    pos[threadIdx.x] = slot_pos[t * top_k + threadIdx.x];
    wt[threadIdx.x] = w[t * top_k + threadIdx.x];
  }
  __syncthreads();
  const int64_t vecs = H >> 3;
  for (int64_t v = threadIdx.x; v < vecs; v += blockDim.x) {
    // all rows' vectors are requested before the rank-ordered sums use them
    // (up to 8 in flight; larger top_k continues one row at a time)
    uint4 yv[8];
#pragma unroll
    for (int r = 0; r < 8; ++r)
      if (r < top_k) yv[r] = reinterpret_cast<const uint4 *>(y + (int64_t)pos[r] * H)[v];
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = 0.0f;
    if (shared) {
      float sf[8];
      bf16x8_to_f32(reinterpret_cast<const uint4 *>(shared + t * H)[v], sf);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = __fadd_rn(o[i], sf[i]);
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      if (r >= top_k) break;
      float yf[8];
      bf16x8_to_f32(yv[r], yf);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = __fadd_rn(o[i], __fmul_rn(wt[r], yf[i]));
    }
    for (int r = 8; r < top_k; ++r) {
      float yf[8];
      bf16x8_to_f32(reinterpret_cast<const uint4 *>(y + (int64_t)pos[r] * H)[v], yf);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = __fadd_rn(o[i], __fmul_rn(wt[r], yf[i]));
    }
    if (OUT_F32) {
      float4 *dst = reinterpret_cast<float4 *>(reinterpret_cast<float *>(out) + t * H) + 2 * v;
      dst[0] = make_float4(o[0], o[1], o[2], o[3]);
      dst[1] = make_float4(o[4], o[5], o[6], o[7]);
    } else {
      uint32_t pk[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        __nv_bfloat162 b = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
        pk[i] = *reinterpret_cast<uint32_t *>(&b);
      }
      reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(out) + t * H)[v] =
          make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  }
}

namespace {

constexpr int kStages = 7;
struct StageTimer {
  bool enabled = false;
  bool recorded = false;
  cudaEvent_t ev[kStages + 1] = {};
  void mark(int i, cudaStream_t s) {
    if (!enabled) return;
    if (!ev[i]) cudaEventCreate(&ev[i]);
    // Inside a stream capture the record becomes a graph node; "external" makes
    // the event observable after each replay of the graph.
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(s, &cs);
    if (cs == cudaStreamCaptureStatusActive)
      cudaEventRecordWithFlags(ev[i], s, cudaEventRecordExternal);
    else
      cudaEventRecord(ev[i], s);
    if (i == kStages) recorded = true;
  }
};
StageTimer &timer() {
  static thread_local StageTimer t;
  return t;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

struct Carver {
  uint8_t *base;
  size_t off = 0;
  void *take(size_t bytes) {
    void *p = base ? base + off : nullptr;
    off += align256(bytes);
    return p;
  }
};

// Scratch of the dispatch stage (router, routing, plan, gather).
struct DispatchWs {
  float *router_partial;
  void *route_scratch;
};
DispatchWs carve_dispatch(const nk_moe_layer &L, int64_t T, Carver &c) {
  const int64_t E = L.experts;
  DispatchWs w;
  w.router_partial = (float *)c.take(sizeof(float) * T * E * kRouterMaxSplits);
  w.route_scratch = c.take(route_exact_scratch_bytes(T, E, (int)L.top_k));
  return w;
}

// Scratch of the grouped expert stage over R rows in n_seg segments.
struct ExpertsWs {
  TcTile *tiles_up, *tiles_down;
  int *tile_counts;
  uint16_t *hmid;  // [R, I]
};
ExpertsWs carve_experts(const nk_moe_layer &L, int64_t R, int64_t n_seg, Carver &c) {
  ExpertsWs w;
  const int64_t rows = R > 0 ? R : 1;
  w.tiles_up = (TcTile *)c.take(sizeof(TcTile) * ceil_div(L.inter, 128) *
                                (ceil_div(rows, kMoeBN) + n_seg));
  w.tiles_down = (TcTile *)c.take(sizeof(TcTile) * ceil_div(L.hidden, 128) *
                                  (ceil_div(rows, kMoeBN) + n_seg));
  w.tile_counts = (int *)c.take(sizeof(int) * 2);
  w.hmid = (uint16_t *)c.take(2 * rows * L.inter);
  return w;
}

// Everything nk_moe_forward needs.
struct MoeWorkspace {
  DispatchWs d;
  ExpertsWs x;
  int32_t *idx, *counts, *offsets, *slot_pos;
  float *w;
  uint16_t *xp;  // [T*k, H] routed rows in expert order; reused for the expert outputs
  uint16_t *s1;  // [T, Is]
  uint16_t *sh;  // [T, H]
  size_t bytes;
};

MoeWorkspace carve(const nk_moe_layer &L, int64_t T, uint8_t *base) {
  MoeWorkspace ws{};
  Carver c{base};
  const int64_t E = L.experts, S = T * L.top_k, H = L.hidden;
  ws.d = carve_dispatch(L, T, c);
  ws.x = carve_experts(L, S, E, c);
  ws.idx = (int32_t *)c.take(sizeof(int32_t) * S);
  ws.w = (float *)c.take(sizeof(float) * S);
  ws.counts = (int32_t *)c.take(sizeof(int32_t) * E);
  ws.offsets = (int32_t *)c.take(sizeof(int32_t) * (E + 1));
  ws.slot_pos = (int32_t *)c.take(sizeof(int32_t) * S);
  ws.xp = (uint16_t *)c.take(2 * S * H);
  if (L.shared_inter > 0) {
    ws.s1 = (uint16_t *)c.take(2 * T * L.shared_inter);
    ws.sh = (uint16_t *)c.take(2 * T * H);
  }
  ws.bytes = c.off;
  return ws;
}

// INT4 rows of K codes are K/2 bytes, loaded by TMA in 16-byte steps.
nk_status validate_weight_kind(const nk_moe_layer *L) {
  if (L->weight_kind != NK_W_BF16 && L->weight_kind != NK_W_INT8_ROW &&
      L->weight_kind != NK_W_INT4_AFFINE)
    return fail(NK_UNSUPPORTED, "weight_kind");
  if (L->weight_kind == NK_W_INT4_AFFINE &&
      (L->hidden % 32 || L->inter % 32 || L->shared_inter % 32))
    return fail(NK_UNSUPPORTED, "INT4_AFFINE experts need hidden, inter, shared_inter % 32 == 0");
  return NK_OK;
}

nk_status validate(const nk_moe_layer *L) {
  if (!L) return fail(NK_INVALID_SHAPE, "null layer");
  if (L->hidden <= 0 || L->experts <= 0 || L->top_k <= 0 || L->top_k > L->experts ||
      L->inter <= 0 || L->shared_inter < 0)
    return fail(NK_INVALID_SHAPE, "moe shape needs hidden, experts, inter > 0, 0 < top_k <= experts");
  if (L->experts > 1024 || L->top_k > 32)
    return fail(NK_UNSUPPORTED, "experts <= 1024 and top_k <= 32");
  if (L->hidden % 8 || L->inter % 16 || (L->shared_inter % 16))
    return fail(NK_UNSUPPORTED, "hidden % 8 == 0 and inter, shared_inter % 16 == 0 required");
  nk_status st = validate_weight_kind(L);
  if (st != NK_OK) return st;
  if (L->route_mode < NK_ROUTE_SIGMOID || L->route_mode > NK_ROUTE_SIGMOID_RENORM)
    return fail(NK_UNSUPPORTED, "route_mode");
  if (!L->router_w3 || !L->up_w || !L->down_w) return fail(NK_INVALID_PARAMS, "missing weights");
  if (L->weight_kind != NK_W_BF16 && (!L->up_scale || !L->down_scale))
    return fail(NK_INVALID_PARAMS, "quantized expert weights need scales");
  if (L->weight_kind == NK_W_INT4_AFFINE && (!L->up_zero_point || !L->down_zero_point))
    return fail(NK_INVALID_PARAMS, "INT4_AFFINE expert weights need zero points");
  if (L->shared_inter > 0 && (!L->shared_up_w || !L->shared_down_w))
    return fail(NK_INVALID_PARAMS, "missing shared expert weights");
  if (L->shared_inter > 0 && L->weight_kind != NK_W_BF16 &&
      (!L->shared_up_scale || !L->shared_down_scale))
    return fail(NK_INVALID_PARAMS, "quantized shared expert needs scales");
  if (L->shared_inter > 0 && L->weight_kind == NK_W_INT4_AFFINE &&
      (!L->shared_up_zero_point || !L->shared_down_zero_point))
    return fail(NK_INVALID_PARAMS, "INT4_AFFINE shared expert needs zero points");
  return NK_OK;
}

// The grouped expert stage reads only the expert dimensions and weights.
nk_status validate_experts(const nk_moe_layer *L) {
  if (!L) return fail(NK_INVALID_SHAPE, "null layer");
  if (L->hidden <= 0 || L->experts <= 0 || L->inter <= 0)
    return fail(NK_INVALID_SHAPE, "hidden, experts and inter must be positive");
  if (L->hidden % 8 || L->inter % 16)
    return fail(NK_UNSUPPORTED, "hidden % 8 == 0 and inter % 16 == 0 required");
  nk_status st = validate_weight_kind(L);
  if (st != NK_OK) return st;
  if (!L->up_w || !L->down_w) return fail(NK_INVALID_PARAMS, "missing expert weights");
  if (L->weight_kind != NK_W_BF16 && (!L->up_scale || !L->down_scale))
    return fail(NK_INVALID_PARAMS, "quantized expert weights need scales");
  if (L->weight_kind == NK_W_INT4_AFFINE && (!L->up_zero_point || !L->down_zero_point))
    return fail(NK_INVALID_PARAMS, "INT4_AFFINE expert weights need zero points");
  return NK_OK;
}

// One GEMM's weight operand in the layer's kind: tc_gemm kind, row pitch for
// K inputs, and the epilogue / transform parameters (per-row int8 scales, or
// per-expert INT4 scale and zero point for groups of `rows` weight rows).
struct WOp {
  int wk;
  const void *w;
  const float *scale;
  const uint8_t *zp;
};
int moe_wk(const nk_moe_layer &L) {
  return L.weight_kind == NK_W_INT8_ROW ? WK_INT8
                                        : (L.weight_kind == NK_W_INT4_AFFINE ? WK_INT4NK : WK_BF16);
}
int64_t w_pitch(int wk, int64_t k) { return wk == WK_BF16 ? 2 * k : (wk == WK_INT8 ? k : k / 2); }
void apply_wop(TcArgs &a, const WOp &op, int group_rows) {
  if (op.wk == WK_INT8) a.row_scale = op.scale;
  if (op.wk == WK_INT4NK) {
    a.group_scale = op.scale;
    a.group_zp = op.zp;
    a.group_rows = group_rows;
  }
}

TcArgs base_args(int *err) {
  TcArgs a{};
  a.w_scale = 1.0f;
  a.err = err;
  return a;
}

// Dense Y[T, n_out] = act(X[T, k] · W[n_out, k]ᵀ ...) through the tcgen05 kernel.
// Accumulators per CTA for the grouped bf16 expert GEMMs (NK_GROUPED_FA=1
// selects the one-accumulator kernel, for comparison).
int grouped_fa() {
  static const int v = [] {
    const char *e = getenv("NK_GROUPED_FA");
    return e && atoi(e) == 1 ? 1 : 2;
  }();
  return v;
}

// Expert parallel, bf16 experts: NK_EP_PULL=1 has the owners pull routed
// rows inside their up projection; by default the sources push them before it
// (measured faster at two GPUs: 1.06-1.08 ms per step against 1.16).
bool ep_pull_enabled() {
  static const bool v = [] {
    const char *e = getenv("NK_EP_PULL");
    return e && atoi(e) == 1;
  }();
  return v;
}

// CTA pairs for the grouped GEMMs: NK_GROUPED_PAIR=2 selects them (default
// single CTAs).
int grouped_pair() {
  static const int v = [] {
    const char *e = getenv("NK_GROUPED_PAIR");
    return e ? atoi(e) : 0;
  }();
  return v;
}

nk_status dense(const WOp &op, const float *bias, const uint16_t *x, int64_t T, int64_t k,
                int64_t n_out, void *y, bool y_f32, bool relu2, int *err, cudaStream_t s,
                int max_ctas = 0) {
  const int bn = T <= 16 ? 16 : (T <= 64 ? 64 : 256);
  TcArgs a = base_args(err);
  a.f_tiles = (int)ceil_div(n_out, 128);
  a.t_tiles = (int)ceil_div(T, bn);
  a.n_features = (int)n_out;
  a.n_tokens = (int)T;
  a.k_blocks = (int)ceil_div(k, 64);
  a.y = y;
  a.ldy = n_out;
  a.y_f32 = y_f32;
  apply_wop(a, op, (int)n_out);
  a.bias = bias;
  a.relu2 = relu2;
  int64_t tiles = (int64_t)a.f_tiles * a.t_tiles;
  const int ctas = max_ctas > 0 && max_ctas < num_sms() ? max_ctas : num_sms();
  int grid = (int)(tiles < ctas ? tiles : ctas);
  return tc_gemm(op.wk, op.w, n_out, k, w_pitch(op.wk, k), x, T, k, k, bn, a, grid, s);
}

}  // namespace

// Router -> routing -> plan -> gather.  Outputs: indices/weights [T,k], counts [E],
// offsets [E+1], slot_pos [T*k], xp [T*k, H] (routed rows in expert order).
nk_status dispatch_stage(const nk_moe_layer &L, const uint16_t *x, int64_t T, int32_t *idx,
                         float *rw, int32_t *counts, int32_t *offsets, int32_t *slot_pos,
                         uint16_t *xp, const DispatchWs &ws, StageTimer &tm, cudaStream_t s) {
  int *err = device_error_ptr();
  const int64_t E = L.experts, K = L.top_k, H = L.hidden;
  nk_status st;
  tm.mark(0, s);
  // router scores [T, E] f32: x · (hi + mid)ᵀ.  K is split over CTAs into f32
  // partial sums; the routing kernels add them in split order and add the bias
  // after the GEMM as linear.rs:333-339 does.  These scores are approximate
  // (tensor-core f32 accumulation); the routing rescores the experts near each
  // token's top-k boundary exactly, given the accumulation bound c.
  float c_bound = 0.0f;
  int router_splits = 1;
  {
    const int64_t hp = ceil_div(H, 64) * 64;
    const int bn = T <= 16 ? 16 : (T <= 64 ? 64 : 256);
    const int k_blocks = (int)(2 * hp / 64);  // hi and mid parts; lo enters the bound
    TcArgs a = base_args(err);
    a.f_tiles = (int)ceil_div(E, 128);
    a.t_tiles = (int)ceil_div(T, bn);
    const int base_tiles = a.f_tiles * a.t_tiles;
    int want = num_sms() / base_tiles;
    if (want < 1) want = 1;
    if (want > kRouterMaxSplits) want = kRouterMaxSplits;
    if (want > k_blocks) want = k_blocks;
    const int per = (int)ceil_div(k_blocks, want);
    const int splits = (int)ceil_div(k_blocks, per);  // every split gets >= 1 block
    a.n_features = (int)E;
    a.n_tokens = (int)T;
    a.k_blocks = k_blocks;
    a.x_k_period = (int)(hp / 64);
    a.k_splits = splits;
    a.split_stride = T * E;
    a.y = ws.router_partial;
    a.ldy = E;
    a.y_f32 = 1;
    int64_t tiles = (int64_t)base_tiles * splits;
    int grid = (int)(tiles < num_sms() ? tiles : num_sms());
    st = tc_gemm(WK_BF16, L.router_w3, E, 2 * hp, 3 * hp * 2, x, T, H, H, bn, a, grid, s);
    if (st != NK_OK) return st;
    c_bound = (float)((double)(per * 64 + splits + 2) * 0x1p-22);
    router_splits = splits;
  }
  tm.mark(1, s);
  // routes, the expert plan and (xp) the routed rows copied into expert order;
  // without xp the rows are moved elsewhere (expert-parallel dispatch)
  st = launch_route_exact(ws.router_partial, router_splits, x, T, (int)H, L.router_w3,
                          L.router_b, L.router_norms, c_bound, (int)E, (int)K, L.route_mode,
                          ws.route_scratch, idx, rw, counts, offsets, slot_pos, xp, s);
  tm.mark(2, s);
  return st;
}

// Grouped expert MLP over R rows laid out as n_seg back-to-back segments:
// out[r] = relu2(rows[r] · up_eᵀ + b_up) · down_eᵀ + b_down for the segment's
// expert e.  out may alias rows (rows are fully consumed before out is written).
// With y_peers, out is unused: segment s's outputs are stored into rank
// s / seg_per_rank's buffer (y_peers) from row seg_yoff[s] (peer memory).
// With pull (bf16 experts, two-accumulator kernel), the up projection's copy
// warps first bring each source rank's rows into `rows` (the receive buffer).
struct EpPull {
  const uint64_t *src;  // [ranks] send buffers
  const int32_t *tab;   // [segments][3] first send row, first receive row, rows
  int *arrived;         // [segments], zeroed by the plan
};
nk_status experts_stage(const nk_moe_layer &L, const uint16_t *rows, int64_t R,
                        const int32_t *seg_expert, const int32_t *seg_rows, int n_seg,
                        uint16_t *out, const ExpertsWs &ws, StageTimer &tm, cudaStream_t s,
                        int max_ctas = 0, const uint64_t *y_peers = nullptr,
                        const int32_t *seg_yoff = nullptr, int seg_per_rank = 1,
                        int seg_rot = 0, const EpPull *pull = nullptr) {
  const int ctas = max_ctas > 0 && max_ctas < num_sms() ? max_ctas : num_sms();
  int *err = device_error_ptr();
  const int64_t E = L.experts, H = L.hidden, I = L.inter;
  const int wk = moe_wk(L);
  // bf16 experts: 256-feature tiles on single CTAs with two accumulators, so
  // each token tile is loaded once per 256 features.  Quantized experts: one
  // accumulator (their transform warps need the registers).  CTA pairs
  // (NK_GROUPED_PAIR=2) measured 1.5-2.5x slower here.
  const int gp = grouped_pair();
  const int pair = gp == 2 ? 2 : 1;
  const int fa = wk == WK_BF16 && pair == 1 ? grouped_fa() : 1;
  const int gctas = pair == 2 ? (ctas & ~1) : ctas;
  if (pull && fa != 2) return fail(NK_UNSUPPORTED, "in-kernel pull needs the two-accumulator kernel");
  TileLists lists;
  lists.n_out[0] = (int)I;
  lists.n_out[1] = (int)H;
  lists.tiles[0] = ws.tiles_up;
  lists.tiles[1] = ws.tiles_down;
  lists.count[0] = ws.tile_counts;
  lists.count[1] = ws.tile_counts + 1;
  lists.seg_yoff = y_peers ? seg_yoff : nullptr;
  lists.seg_per_rank = seg_per_rank;
  lists.seg_rot = y_peers || pull ? seg_rot : 0;
  lists.pull = pull ? 1 : 0;
  build_tiles_kernel<<<2, 1024, 0, s>>>(seg_rows, seg_expert, n_seg, kMoeBN, 128 * fa * pair,
                                        lists);
  nk_status st = check_launch("build_tiles_kernel");
  if (st != NK_OK) return st;
  if (R == 0) return NK_OK;
  tm.mark(3, s);
  {  // grouped up-projection + relu2
    TcArgs a = base_args(err);
    a.tiles = ws.tiles_up;
    a.tile_count = ws.tile_counts;
    a.k_blocks = (int)ceil_div(H, 64);
    a.y = ws.hmid;
    a.ldy = I;
    apply_wop(a, WOp{wk, L.up_w, L.up_scale, L.up_zero_point}, (int)I);
    a.bias = L.up_b;
    a.relu2 = 1;
    if (pull) {
      a.pull_src = pull->src;
      a.pull_tab = pull->tab;
      a.pull_arrived = pull->arrived;
      a.pull_dst = const_cast<uint16_t *>(rows);
      a.pull_seg_per_rank = seg_per_rank;
      a.pull_segs = n_seg;
      a.pull_rot = seg_rot;
      a.pull_row_vecs = H / 8;
    }
    st = tc_gemm(wk, L.up_w, E * I, H, w_pitch(wk, H), rows, R, H, H, kMoeBN, a, gctas, s, pair,
                 fa);
    if (st != NK_OK) return st;
  }
  tm.mark(4, s);
  {  // grouped down-projection
    TcArgs a = base_args(err);
    a.tiles = ws.tiles_down;
    a.tile_count = ws.tile_counts + 1;
    a.k_blocks = (int)ceil_div(I, 64);
    a.y = out;
    a.ldy = H;
    apply_wop(a, WOp{wk, L.down_w, L.down_scale, L.down_zero_point}, (int)H);
    a.bias = L.down_b;
    a.y_peers = y_peers;
    st = tc_gemm(wk, L.down_w, E * H, I, w_pitch(wk, I), ws.hmid, R, I, I, kMoeBN, a, gctas, s,
                 pair, fa);
  }
  return st;
}

nk_status shared_stage(const nk_moe_layer &L, const uint16_t *x, int64_t T, uint16_t *s1,
                       uint16_t *sh, cudaStream_t s, int max_ctas = 0) {
  int *err = device_error_ptr();
  const int wk = moe_wk(L);
  const int64_t Is = L.shared_inter, H = L.hidden;
  nk_status st = dense(WOp{wk, L.shared_up_w, L.shared_up_scale, L.shared_up_zero_point},
                       L.shared_up_b, x, T, H, Is, s1, false, true, err, s, max_ctas);
  if (st != NK_OK) return st;
  return dense(WOp{wk, L.shared_down_w, L.shared_down_scale, L.shared_down_zero_point},
               L.shared_down_b, s1, T, Is, H, sh, false, false, err, s, max_ctas);
}

nk_status combine_stage(const uint16_t *y, const uint16_t *sh, const float *rw,
                        const int32_t *slot_pos, int64_t T, int64_t H, int K, void *out,
                        int out_dtype, cudaStream_t s) {
  if (T == 0) return NK_OK;
  if (out_dtype == NK_F32)
    combine_kernel<true><<<(unsigned)T, 128, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16 *>(y), reinterpret_cast<const __nv_bfloat16 *>(sh),
        rw, slot_pos, H, K, out);
  else
    combine_kernel<false><<<(unsigned)T, 128, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16 *>(y), reinterpret_cast<const __nv_bfloat16 *>(sh),
        rw, slot_pos, H, K, out);
  return check_launch("combine_kernel");
}

nk_status ws_too_small(size_t need, size_t have) {
  nk_status st = fail(NK_WORKSPACE_TOO_SMALL, "workspace smaller than the *_workspace_bytes query");
  tls_error().expected = need;
  tls_error().actual = have;
  return st;
}

// Side stream and fork/join events of the calling thread (one set per device).
struct SideStream {
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  int device = -1;
};
nk_status side_stream(SideStream **out) {
  static thread_local SideStream ss[64];
  int d = 0;
  NK_CUDA_TRY(cudaGetDevice(&d));
  if (d < 0 || d >= 64) return fail(NK_DEVICE_ERROR, "device ordinal out of range");
  SideStream &s = ss[d];
  if (!s.stream) {
    NK_CUDA_TRY(cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking));
    NK_CUDA_TRY(cudaEventCreateWithFlags(&s.fork, cudaEventDisableTiming));
    NK_CUDA_TRY(cudaEventCreateWithFlags(&s.join, cudaEventDisableTiming));
  }
  *out = &s;
  return NK_OK;
}

// SMs given to the shared expert while the routed experts run beside it:
// 3/4 of its share of the layer's FLOPs (the routed experts are partly
// HBM-bound and keep their throughput on fewer SMs), for batches of at least
// 1024 tokens; smaller batches run it after the routed experts on all SMs.
// NK_SHARED_SMS overrides (0 disables the overlap).  Measured on B200 at
// T = 4096: 28 SMs -> 0.913 ms per layer vs 0.950 ms without overlap.
int shared_expert_sms(const nk_moe_layer &L, int64_t T) {
  static const int env = [] {
    const char *e = getenv("NK_SHARED_SMS");
    return e ? atoi(e) : -1;
  }();
  if (env >= 0) return env;
  if (L.shared_inter <= 0 || T < 1024) return 0;
  const double routed = (double)L.top_k * L.inter, shared = (double)L.shared_inter;
  int v = (int)(0.75 * num_sms() * shared / (routed + shared) + 0.5);
  if (v < 8) v = 8;
  if (v > num_sms() / 2) v = num_sms() / 2;
  return v;
}

nk_status moe_forward(const nk_moe_layer &L, const uint16_t *x, int64_t T, void *out,
                      int out_dtype, int32_t *indices, float *weights, void *workspace,
                      size_t ws_bytes, cudaStream_t s) {
  MoeWorkspace need = carve(L, T, nullptr);
  if (!workspace || ws_bytes < need.bytes) return ws_too_small(need.bytes, ws_bytes);
  MoeWorkspace ws = carve(L, T, reinterpret_cast<uint8_t *>(workspace));
  const int64_t K = L.top_k, S = T * K;
  int32_t *idx = indices ? indices : ws.idx;
  float *rw = weights ? weights : ws.w;
  StageTimer &tm = timer();
  tm.recorded = false;
  nk_status st;
  // The shared expert only needs x: for large batches it starts at once on a
  // side stream, limited to a few SMs, while the routed path runs on the rest.
  const int sh_sms = L.shared_inter > 0 ? shared_expert_sms(L, T) : 0;
  const bool overlap = sh_sms > 0 && sh_sms < num_sms();
  SideStream *side = nullptr;
  if (overlap) {
    st = side_stream(&side);
    if (st != NK_OK) return st;
    NK_CUDA_TRY(cudaEventRecord(side->fork, s));
    NK_CUDA_TRY(cudaStreamWaitEvent(side->stream, side->fork, 0));
    st = shared_stage(L, x, T, ws.s1, ws.sh, side->stream, sh_sms);
    if (st != NK_OK) return st;
    NK_CUDA_TRY(cudaEventRecord(side->join, side->stream));
  }
  st = dispatch_stage(L, x, T, idx, rw, ws.counts, ws.offsets, ws.slot_pos, ws.xp, ws.d, tm, s);
  if (st != NK_OK) return st;
  // experts in expert order: one segment per expert, rows = counts[e]; outputs into xp
  st = experts_stage(L, ws.xp, S, nullptr, ws.counts, (int)L.experts, ws.xp, ws.x, tm, s,
                     overlap ? num_sms() - sh_sms : 0);
  if (st != NK_OK) return st;
  tm.mark(5, s);
  if (L.shared_inter > 0) {
    if (overlap) {
      NK_CUDA_TRY(cudaStreamWaitEvent(s, side->join, 0));
    } else {
      st = shared_stage(L, x, T, ws.s1, ws.sh, s);
      if (st != NK_OK) return st;
    }
  }
  tm.mark(6, s);
  st = combine_stage(ws.xp, ws.sh, rw, ws.slot_pos, T, L.hidden, (int)K, out, out_dtype, s);
  tm.mark(7, s);
  return st;
}

// Scratch of nk_moe_forward_ep.
struct EpWorkspace {
  DispatchWs d;
  ExpertsWs x;
  int32_t *idx, *counts, *offsets, *slot_pos;
  float *w;
  uint16_t *s1, *sh;
  size_t bytes;
};

EpWorkspace carve_ep(const nk_moe_layer &L, const nk_moe_layer &local, const nk_ep_ctx &c,
                     int64_t T, uint8_t *base) {
  EpWorkspace ws{};
  Carver cv{base};
  const int64_t E = L.experts, S = T * L.top_k;
  ws.d = carve_dispatch(L, T, cv);
  ws.x = carve_experts(local, c.capacity_rows, (int64_t)c.ranks * local.experts, cv);
  ws.idx = (int32_t *)cv.take(sizeof(int32_t) * S);
  ws.w = (float *)cv.take(sizeof(float) * S);
  ws.counts = (int32_t *)cv.take(sizeof(int32_t) * E);
  ws.offsets = (int32_t *)cv.take(sizeof(int32_t) * (E + 1));
  ws.slot_pos = (int32_t *)cv.take(sizeof(int32_t) * S);
  if (L.shared_inter > 0) {
    ws.s1 = (uint16_t *)cv.take(2 * T * L.shared_inter);
    ws.sh = (uint16_t *)cv.take(2 * T * L.hidden);
  }
  ws.bytes = cv.off;
  return ws;
}

nk_status validate_ep(const nk_ep_ctx *c, const nk_moe_layer *L, const nk_moe_layer *local,
                      int64_t T) {
  if (!c || !c->connected) return fail(NK_INVALID_PARAMS, "connected nk_ep_ctx required");
  nk_status st = validate(L);
  if (st != NK_OK) return st;
  st = validate_experts(local);
  if (st != NK_OK) return st;
  if (L->experts != c->experts || L->hidden != c->hidden || L->top_k != c->top_k ||
      local->experts * c->ranks != c->experts || local->hidden != c->hidden ||
      local->inter != L->inter || local->weight_kind != L->weight_kind)
    return fail(NK_INVALID_SHAPE, "layer, local experts and context disagree");
  if (T <= 0) return fail(NK_INVALID_ROW_COUNT, "row_count must be non-zero");
  if (T > c->max_tokens) return fail(NK_INVALID_SHAPE, "more tokens than the context holds");
  return NK_OK;
}

// MoeLayer::forward_into (moe.rs:154-249) with the experts spread over ranks:
// route here, exchange counts, send each routed row straight into its
// expert owner's receive buffer, run this rank's experts on what arrived,
// send the results straight back, combine in rank order.  Device barriers in
// peer memory order the phases; no host synchronisation, no collectives.
nk_status moe_forward_ep(nk_ep_ctx *c, const nk_moe_layer &L, const nk_moe_layer &local,
                         const uint16_t *x, int64_t T, void *out, int out_dtype,
                         int32_t *indices, float *weights, void *workspace, size_t ws_bytes,
                         cudaStream_t s) {
  const EpWorkspace need = carve_ep(L, local, *c, T, nullptr);
  if (!workspace || ws_bytes < need.bytes) return ws_too_small(need.bytes, ws_bytes);
  EpWorkspace ws = carve_ep(L, local, *c, T, reinterpret_cast<uint8_t *>(workspace));
  int32_t *idx = indices ? indices : ws.idx;
  float *rw = weights ? weights : ws.w;
  StageTimer &tm = timer();
  tm.recorded = false;
  nk_status st;
  // shared expert beside the exchange (side stream, a share of the SMs)
  const int sh_sms = L.shared_inter > 0 ? shared_expert_sms(L, T) : 0;
  const bool overlap = sh_sms > 0 && sh_sms < num_sms();
  SideStream *side = nullptr;
  if (overlap) {
    st = side_stream(&side);
    if (st != NK_OK) return st;
    NK_CUDA_TRY(cudaEventRecord(side->fork, s));
    NK_CUDA_TRY(cudaStreamWaitEvent(side->stream, side->fork, 0));
    st = shared_stage(L, x, T, ws.s1, ws.sh, side->stream, sh_sms);
    if (st != NK_OK) return st;
    NK_CUDA_TRY(cudaEventRecord(side->join, side->stream));
  }
  // Rows are pushed to their owners before the up projection (ep_dispatch +
  // barrier), or, with NK_EP_PULL=1 and bf16 experts, pulled by the owners'
  // up projection from this rank's send buffer (the routing writes them there
  // in expert order)
  const bool pull = ep_pull_enabled() && moe_wk(local) == WK_BF16 && grouped_pair() == 1 &&
                    grouped_fa() == 2;
  st = dispatch_stage(L, x, T, idx, rw, ws.counts, ws.offsets, ws.slot_pos,
                      pull ? ep_send(c) : nullptr, ws.d, tm, s);
  if (st != NK_OK) return st;
  // also: every peer is done with the last forward, and (pull) every send
  // buffer of this forward is written
  st = ep_exchange_counts(c, ws.counts, s);
  if (st != NK_OK) return st;
  st = ep_plan(c, s, pull);
  if (st != NK_OK) return st;
  if (!pull) {
    st = ep_dispatch(c, x, T, idx, ws.slot_pos, ws.offsets, s);
    if (st != NK_OK) return st;
    st = ep_barrier(c, s);  // every routed row has arrived
    if (st != NK_OK) return st;
  }
  uint16_t *recv = ep_recv(c);
  const EpPull pl{ep_send_table(c), c->pull_tab, c->arrived};
  // the down projection's epilogue stores every result row straight into its
  // source rank's result buffer (the return exchange fused into the GEMM)
  st = experts_stage(local, recv, c->capacity_rows, c->seg_expert, c->seg_rows,
                     c->ranks * (int)local.experts, recv, ws.x, tm, s,
                     overlap ? num_sms() - sh_sms : 0, ep_out_table(c), c->ret_off,
                     (int)local.experts, c->rank * (int)local.experts, pull ? &pl : nullptr);
  if (st != NK_OK) return st;
  st = ep_barrier(c, s);  // every result is back
  if (st != NK_OK) return st;
  tm.mark(5, s);
  if (L.shared_inter > 0) {
    if (overlap) {
      NK_CUDA_TRY(cudaStreamWaitEvent(s, side->join, 0));
    } else {
      st = shared_stage(L, x, T, ws.s1, ws.sh, s);
      if (st != NK_OK) return st;
    }
  }
  tm.mark(6, s);
  st = combine_stage(ep_out(c), ws.sh, rw, ws.slot_pos, T, L.hidden, (int)L.top_k, out,
                     out_dtype, s);
  tm.mark(7, s);
  return st;
}

}  // namespace nk

using namespace nk;

extern "C" {

nk_status nk_moe_workspace_bytes(const nk_moe_layer *layer, int64_t tokens, size_t *bytes) {
  nk_status st = validate(layer);
  if (st != NK_OK) return st;
  if (tokens <= 0) return fail(NK_INVALID_ROW_COUNT, "row_count must be non-zero");
  *bytes = carve(*layer, tokens, nullptr).bytes;
  return ok();
}

nk_status nk_moe_forward(const nk_moe_layer *layer, const uint16_t *x, int64_t tokens,
                         void *out, int32_t out_dtype, int32_t *indices, float *weights,
                         void *workspace, size_t workspace_bytes, void *stream) {
  nk_status st = validate(layer);
  if (st != NK_OK) return st;
  if (tokens <= 0) return fail(NK_INVALID_ROW_COUNT, "row_count must be non-zero");
  if (tokens > (1 << 24)) return fail(NK_UNSUPPORTED, "too many tokens for one call");
  if (out_dtype != NK_F32 && out_dtype != NK_BF16) return fail(NK_UNSUPPORTED, "out_dtype");
  st = moe_forward(*layer, x, tokens, out, out_dtype, indices, weights, workspace,
                   workspace_bytes, as_stream(stream));
  return st == NK_OK ? ok() : st;
}

nk_status nk_moe_dispatch_workspace_bytes(const nk_moe_layer *layer, int64_t tokens,
                                          size_t *bytes) {
  nk_status st = validate(layer);
  if (st != NK_OK) return st;
  if (tokens <= 0) return fail(NK_INVALID_ROW_COUNT, "row_count must be non-zero");
  Carver c{nullptr};
  carve_dispatch(*layer, tokens, c);
  *bytes = c.off;
  return ok();
}

nk_status nk_moe_dispatch(const nk_moe_layer *layer, const uint16_t *x, int64_t tokens,
                          int32_t *indices, float *weights, int32_t *counts, int32_t *offsets,
                          int32_t *slot_pos, uint16_t *routed_rows, void *workspace,
                          size_t workspace_bytes, void *stream) {
  nk_status st = validate(layer);
  if (st != NK_OK) return st;
  if (tokens <= 0) return fail(NK_INVALID_ROW_COUNT, "row_count must be non-zero");
  if (tokens > (1 << 24)) return fail(NK_UNSUPPORTED, "too many tokens for one call");
  Carver c{nullptr};
  carve_dispatch(*layer, tokens, c);
  if (!workspace || workspace_bytes < c.off) return ws_too_small(c.off, workspace_bytes);
  Carver w{reinterpret_cast<uint8_t *>(workspace)};
  DispatchWs ws = carve_dispatch(*layer, tokens, w);
  StageTimer &tm = timer();
  tm.recorded = false;
  st = dispatch_stage(*layer, x, tokens, indices, weights, counts, offsets, slot_pos,
                      routed_rows, ws, tm, as_stream(stream));
  return st == NK_OK ? ok() : st;
}

nk_status nk_moe_experts_workspace_bytes(const nk_moe_layer *layer, int64_t rows,
                                         int32_t n_segments, size_t *bytes) {
  nk_status st = validate_experts(layer);
  if (st != NK_OK) return st;
  if (rows < 0 || n_segments <= 0 || n_segments > 1024)
    return fail(NK_INVALID_SHAPE, "rows >= 0 and 0 < n_segments <= 1024");
  Carver c{nullptr};
  carve_experts(*layer, rows, n_segments, c);
  *bytes = c.off;
  return ok();
}

nk_status nk_moe_experts(const nk_moe_layer *layer, const uint16_t *rows, int64_t n_rows,
                         const int32_t *seg_expert, const int32_t *seg_rows, int32_t n_segments,
                         uint16_t *out, void *workspace, size_t workspace_bytes, void *stream) {
  nk_status st = validate_experts(layer);
  if (st != NK_OK) return st;
  if (n_rows < 0 || n_rows > (1 << 27) || n_segments <= 0 || n_segments > 1024)
    return fail(NK_INVALID_SHAPE, "0 <= rows and 0 < n_segments <= 1024");
  Carver c{nullptr};
  carve_experts(*layer, n_rows, n_segments, c);
  if (!workspace || workspace_bytes < c.off) return ws_too_small(c.off, workspace_bytes);
  Carver w{reinterpret_cast<uint8_t *>(workspace)};
  ExpertsWs ws = carve_experts(*layer, n_rows, n_segments, w);
  StageTimer &tm = timer();
  st = experts_stage(*layer, rows, n_rows, seg_expert, seg_rows, n_segments, out, ws, tm,
                     as_stream(stream));
  return st == NK_OK ? ok() : st;
}

nk_status nk_moe_combine(const uint16_t *expert_rows, const uint16_t *shared, const float *weights,
                         const int32_t *slot_pos, int64_t tokens, int64_t hidden, int64_t top_k,
                         void *out, int32_t out_dtype, void *stream) {
  if (tokens < 0 || hidden <= 0 || top_k <= 0 || top_k > 32 || hidden % 8)
    return fail(NK_INVALID_SHAPE, "tokens >= 0, 0 < top_k <= 32, hidden % 8 == 0");
  if (out_dtype != NK_F32 && out_dtype != NK_BF16) return fail(NK_UNSUPPORTED, "out_dtype");
  nk_status st = combine_stage(expert_rows, shared, weights, slot_pos, tokens, hidden,
                               (int)top_k, out, out_dtype, as_stream(stream));
  return st == NK_OK ? ok() : st;
}

nk_status nk_moe_shared(const nk_moe_layer *layer, const uint16_t *x, int64_t tokens,
                        uint16_t *scratch, uint16_t *out, void *stream) {
  nk_status st = validate(layer);
  if (st != NK_OK) return st;
  if (layer->shared_inter <= 0) return fail(NK_INVALID_PARAMS, "layer has no shared expert");
  if (tokens <= 0) return fail(NK_INVALID_ROW_COUNT, "row_count must be non-zero");
  st = shared_stage(*layer, x, tokens, scratch, out, as_stream(stream));
  return st == NK_OK ? ok() : st;
}

nk_status nk_set_stage_timing(int32_t enable) {
  timer().enabled = enable != 0;
  return ok();
}

nk_status nk_moe_stage_times(float *ms, int32_t capacity, int32_t *count) {
  StageTimer &t = timer();
  if (!t.recorded) return fail(NK_INVALID_PARAMS, "no timed nk_moe_forward on this thread");
  NK_CUDA_TRY(cudaEventSynchronize(t.ev[kStages]));
  int n = capacity < kStages ? capacity : kStages;
  for (int i = 0; i < n; ++i) NK_CUDA_TRY(cudaEventElapsedTime(&ms[i], t.ev[i], t.ev[i + 1]));
  if (count) *count = n;
  return ok();
}


nk_status nk_moe_forward_ep_workspace_bytes(const nk_ep_ctx *ctx, const nk_moe_layer *layer,
                                            const nk_moe_layer *local, int64_t tokens,
                                            size_t *bytes) {
  nk_status st = validate_ep(ctx, layer, local, tokens);
  if (st != NK_OK) return st;
  if (!bytes) return fail(NK_INVALID_PARAMS, "bytes is null");
  *bytes = carve_ep(*layer, *local, *ctx, tokens, nullptr).bytes;
  return ok();
}

nk_status nk_moe_forward_ep(nk_ep_ctx *ctx, const nk_moe_layer *layer, const nk_moe_layer *local,
                            const uint16_t *x, int64_t tokens, void *out, int32_t out_dtype,
                            int32_t *indices, float *weights, void *workspace,
                            size_t workspace_bytes, void *stream) {
  nk_status st = validate_ep(ctx, layer, local, tokens);
  if (st != NK_OK) return st;
  if (out_dtype != NK_F32 && out_dtype != NK_BF16) return fail(NK_UNSUPPORTED, "out_dtype");
  st = moe_forward_ep(ctx, *layer, *local, x, tokens, out, out_dtype, indices, weights,
                      workspace, workspace_bytes, as_stream(stream));
  return st == NK_OK ? ok() : st;
}


nk_status nk_router_norms(const uint16_t *router_w3, int64_t experts, int64_t hidden,
                          float *norms, void *stream) {
  if (experts <= 0 || hidden <= 0) return fail(NK_INVALID_SHAPE, "experts and hidden > 0");
  if (!router_w3 || !norms) return fail(NK_INVALID_PARAMS, "router_w3 and norms");
  nk_status st = launch_router_norms(router_w3, experts, hidden, norms, as_stream(stream));
  return st == NK_OK ? ok() : st;
}

}  // extern "C"
