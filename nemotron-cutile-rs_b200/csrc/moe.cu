// moe.cu — the MoE layer (MoeLayer::forward_into, nemotron-nn/src/moe.rs:154-249)
// as a chain of device kernels on one stream:
//   router GEMM (tcgen05, f32-accurate via a 3-way bf16 split of the weight)
//   -> top-k routing -> expert histogram/permutation -> token gather
//   -> grouped up-projection (+relu2 epilogue) -> grouped down-projection
//   -> shared expert (two dense GEMMs) -> rank-ordered combine.
#include "gemm_tc.h"
#include "route.h"

namespace nk {

constexpr int kMoeBN = 256;
constexpr int kRouterMaxSplits = 16;

// Grouped tile list: for each expert e with c_e routed rows, ceil(n_out/128)
// feature tiles x ceil(c_e/BN) token tiles.  One block; E <= 1024.
__global__ void build_tiles_kernel(const int32_t *__restrict__ counts,
                                   const int32_t *__restrict__ offsets, int E, int n_out,
                                   int bn, TcTile *__restrict__ tiles, int *__restrict__ count) {
  __shared__ int sc[1024];
  const int e = threadIdx.x;
  const int ft = (n_out + 127) / 128;
  int c = e < E ? counts[e] : 0;
  int tt = (c + bn - 1) / bn;
  int mine = ft * tt;
  sc[e] = mine;
  __syncthreads();
  for (int o = 1; o < blockDim.x; o <<= 1) {
    int v = e >= o ? sc[e - o] : 0;
    __syncthreads();
    sc[e] += v;
    __syncthreads();
  }
  int base = sc[e] - mine;
  if (e == blockDim.x - 1) *count = sc[e];
  if (e >= E) return;
  int off = offsets[e];
  for (int f = 0; f < ft; ++f)
    for (int t = 0; t < tt; ++t) {
      TcTile tile;
      tile.w_row = e * n_out + f * 128;
      tile.x_row = off + t * bn;
      int fv = n_out - f * 128, tv = c - t * bn;
      tile.valid = ((fv > 128 ? 128 : fv) << 16) | (tv > bn ? bn : tv);
      tile.out_col0 = f * 128;
      tiles[base + f * tt + t] = tile;
    }
}

// Xp[pos, :] = x[perm[pos] / top_k, :]  (16-byte vectors; H % 8 == 0).
__global__ void gather_rows_kernel(const uint4 *__restrict__ x, const int32_t *__restrict__ perm,
                                   int64_t slots, int top_k, int64_t row_vecs,
                                   uint4 *__restrict__ xp) {
  const int64_t pos = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (pos >= slots) return;
  const int64_t t = perm[pos] / top_k;
  const uint4 *src = x + t * row_vecs;
  uint4 *dst = xp + pos * row_vecs;
  for (int64_t v = threadIdx.x & 31; v < row_vecs; v += 32) dst[v] = src[v];
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
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = 0.0f;
    if (shared) {
      float sf[8];
      bf16x8_to_f32(reinterpret_cast<const uint4 *>(shared + t * H)[v], sf);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = __fadd_rn(o[i], sf[i]);
    }
    for (int r = 0; r < top_k; ++r) {
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

// scores[i] = (Σ_s partial[s][i]) + bias[i % E], partial sums added in split order.
__global__ void router_reduce_kernel(const float *__restrict__ partial, int splits, int64_t n,
                                     int E, const float *__restrict__ bias,
                                     float *__restrict__ scores) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float acc = partial[i];
  for (int s = 1; s < splits; ++s) acc = __fadd_rn(acc, partial[(int64_t)s * n + i]);
  if (bias) acc = __fadd_rn(acc, bias[i % E]);
  scores[i] = acc;
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

struct MoeWorkspace {
  float *scores;
  float *router_partial;  // [splits, T, E]
  int32_t *idx;
  float *w;
  int32_t *counts, *offsets, *perm, *slot_pos, *plan_scratch;
  TcTile *tiles_up, *tiles_down;
  int *tile_counts;
  uint16_t *xp;   // [slots, H]; reused for the routed expert outputs
  uint16_t *hmid; // [slots, I]
  uint16_t *s1;   // [T, Is]
  uint16_t *sh;   // [T, H]
  size_t bytes;
};

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

MoeWorkspace carve(const nk_moe_layer &L, int64_t T, uint8_t *base) {
  MoeWorkspace ws{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    void *p = base ? base + off : nullptr;
    off += align256(bytes);
    return p;
  };
  const int64_t E = L.experts, K = L.top_k, H = L.hidden, I = L.inter, S = T * K;
  ws.scores = (float *)take(sizeof(float) * T * E);
  ws.router_partial = (float *)take(sizeof(float) * T * E * kRouterMaxSplits);
  ws.idx = (int32_t *)take(sizeof(int32_t) * S);
  ws.w = (float *)take(sizeof(float) * S);
  ws.counts = (int32_t *)take(sizeof(int32_t) * E);
  ws.offsets = (int32_t *)take(sizeof(int32_t) * (E + 1));
  ws.perm = (int32_t *)take(sizeof(int32_t) * S);
  ws.slot_pos = (int32_t *)take(sizeof(int32_t) * S);
  ws.plan_scratch = (int32_t *)take(plan_scratch_bytes(S, E));
  const int64_t max_tiles_up = ceil_div(I, 128) * (ceil_div(S, kMoeBN) + E);
  const int64_t max_tiles_down = ceil_div(H, 128) * (ceil_div(S, kMoeBN) + E);
  ws.tiles_up = (TcTile *)take(sizeof(TcTile) * max_tiles_up);
  ws.tiles_down = (TcTile *)take(sizeof(TcTile) * max_tiles_down);
  ws.tile_counts = (int *)take(sizeof(int) * 2);
  ws.xp = (uint16_t *)take(2 * S * H);
  ws.hmid = (uint16_t *)take(2 * S * I);
  if (L.shared_inter > 0) {
    ws.s1 = (uint16_t *)take(2 * T * L.shared_inter);
    ws.sh = (uint16_t *)take(2 * T * H);
  }
  ws.bytes = off;
  return ws;
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
  if (L->weight_kind != NK_W_BF16 && L->weight_kind != NK_W_INT8_ROW)
    return fail(NK_UNSUPPORTED, "weight_kind");
  if (L->route_mode < NK_ROUTE_SIGMOID || L->route_mode > NK_ROUTE_SIGMOID_RENORM)
    return fail(NK_UNSUPPORTED, "route_mode");
  if (!L->router_w3 || !L->up_w || !L->down_w) return fail(NK_INVALID_PARAMS, "missing weights");
  if (L->weight_kind == NK_W_INT8_ROW && (!L->up_scale || !L->down_scale))
    return fail(NK_INVALID_PARAMS, "INT8_ROW weights need scales");
  if (L->shared_inter > 0 && (!L->shared_up_w || !L->shared_down_w))
    return fail(NK_INVALID_PARAMS, "missing shared expert weights");
  if (L->shared_inter > 0 && L->weight_kind == NK_W_INT8_ROW &&
      (!L->shared_up_scale || !L->shared_down_scale))
    return fail(NK_INVALID_PARAMS, "INT8_ROW shared expert needs scales");
  return NK_OK;
}

TcArgs base_args(int *err) {
  TcArgs a{};
  a.w_scale = 1.0f;
  a.err = err;
  return a;
}

// Dense Y[T, n_out] = act(X[T, k] · W[n_out, k]ᵀ ...) through the tcgen05 kernel.
nk_status dense(int wk, const void *w, const float *row_scale, const float *bias,
                const uint16_t *x, int64_t T, int64_t k, int64_t n_out, void *y, bool y_f32,
                bool relu2, int *err, cudaStream_t s) {
  const int bn = T <= 64 ? 64 : 256;
  TcArgs a = base_args(err);
  a.f_tiles = (int)ceil_div(n_out, 128);
  a.t_tiles = (int)ceil_div(T, bn);
  a.n_features = (int)n_out;
  a.n_tokens = (int)T;
  a.k_blocks = (int)ceil_div(k, 64);
  a.y = y;
  a.ldy = n_out;
  a.y_f32 = y_f32;
  a.row_scale = row_scale;
  a.bias = bias;
  a.relu2 = relu2;
  int64_t tiles = (int64_t)a.f_tiles * a.t_tiles;
  int grid = (int)(tiles < num_sms() ? tiles : num_sms());
  return tc_gemm(wk, w, n_out, k, wk == WK_BF16 ? 2 * k : k, x, T, k, k, bn, a, grid, s);
}

}  // namespace

nk_status moe_forward(const nk_moe_layer &L, const uint16_t *x, int64_t T, void *out,
                      int out_dtype, int32_t *indices, float *weights, void *workspace,
                      size_t ws_bytes, cudaStream_t s) {
  MoeWorkspace need = carve(L, T, nullptr);
  if (!workspace || ws_bytes < need.bytes) {
    nk_status st = fail(NK_WORKSPACE_TOO_SMALL, "workspace smaller than nk_moe_workspace_bytes");
    tls_error().expected = need.bytes;
    tls_error().actual = ws_bytes;
    return st;
  }
  MoeWorkspace ws = carve(L, T, reinterpret_cast<uint8_t *>(workspace));
  int *err = device_error_ptr();
  const int64_t E = L.experts, K = L.top_k, H = L.hidden, I = L.inter, S = T * K;
  const int wk = L.weight_kind == NK_W_INT8_ROW ? WK_INT8 : WK_BF16;
  int32_t *idx = indices ? indices : ws.idx;
  float *rw = weights ? weights : ws.w;
  nk_status st;

  StageTimer &tm = timer();
  tm.recorded = false;
  tm.mark(0, s);
  // 1. router scores [T, E] f32: x · (hi + mid + lo)ᵀ.  K is split over CTAs into
  //    f32 partial sums, reduced in split order; the bias is added after the
  //    GEMM as linear.rs:333-339 does.
  {
    const int64_t hp = ceil_div(H, 64) * 64;
    const int bn = T <= 64 ? 64 : 256;
    const int k_blocks = (int)(3 * hp / 64);
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
    st = tc_gemm(WK_BF16, L.router_w3, E, 3 * hp, 3 * hp * 2, x, T, H, H, bn, a, grid, s);
    if (st != NK_OK) return st;
    const int64_t n = T * E;
    router_reduce_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(
        ws.router_partial, splits, n, (int)E, L.router_b, ws.scores);
    st = check_launch("router_reduce_kernel");
    if (st != NK_OK) return st;
  }
  tm.mark(1, s);
  // 2. routing, 3. plan
  st = launch_route(ws.scores, T, (int)E, (int)K, L.route_mode, idx, rw, s);
  if (st != NK_OK) return st;
  st = launch_plan(idx, S, (int)E, ws.counts, ws.offsets, ws.perm, ws.slot_pos, ws.plan_scratch, s);
  if (st != NK_OK) return st;
  build_tiles_kernel<<<1, 1024, 0, s>>>(ws.counts, ws.offsets, (int)E, (int)I, kMoeBN,
                                        ws.tiles_up, ws.tile_counts);
  build_tiles_kernel<<<1, 1024, 0, s>>>(ws.counts, ws.offsets, (int)E, (int)H, kMoeBN,
                                        ws.tiles_down, ws.tile_counts + 1);
  st = check_launch("build_tiles_kernel");
  if (st != NK_OK) return st;
  tm.mark(2, s);
  // 4. gather routed token rows in expert order
  {
    const int warps = 8;
    gather_rows_kernel<<<(unsigned)ceil_div(S, warps), warps * 32, 0, s>>>(
        reinterpret_cast<const uint4 *>(x), ws.perm, S, (int)K, H / 8,
        reinterpret_cast<uint4 *>(ws.xp));
    st = check_launch("gather_rows_kernel");
    if (st != NK_OK) return st;
  }
  tm.mark(3, s);
  // 5. grouped up-projection + relu2: hmid[pos, :] = relu2(xp[pos] · up_eᵀ + b)
  {
    TcArgs a = base_args(err);
    a.tiles = ws.tiles_up;
    a.tile_count = ws.tile_counts;
    a.k_blocks = (int)ceil_div(H, 64);
    a.y = ws.hmid;
    a.ldy = I;
    a.row_scale = wk == WK_INT8 ? L.up_scale : nullptr;
    a.bias = L.up_b;
    a.relu2 = 1;
    st = tc_gemm(wk, L.up_w, E * I, H, wk == WK_BF16 ? 2 * H : H, ws.xp, S, H, H, kMoeBN, a,
                 num_sms(), s);
    if (st != NK_OK) return st;
  }
  tm.mark(4, s);
  // 6. grouped down-projection: y[pos, :] = hmid[pos] · down_eᵀ + b  (into xp's storage)
  uint16_t *yrouted = ws.xp;
  {
    TcArgs a = base_args(err);
    a.tiles = ws.tiles_down;
    a.tile_count = ws.tile_counts + 1;
    a.k_blocks = (int)ceil_div(I, 64);
    a.y = yrouted;
    a.ldy = H;
    a.row_scale = wk == WK_INT8 ? L.down_scale : nullptr;
    a.bias = L.down_b;
    st = tc_gemm(wk, L.down_w, E * H, I, wk == WK_BF16 ? 2 * I : I, ws.hmid, S, I, I, kMoeBN, a,
                 num_sms(), s);
    if (st != NK_OK) return st;
  }
  tm.mark(5, s);
  // 7. shared expert over all tokens
  if (L.shared_inter > 0) {
    const int64_t Is = L.shared_inter;
    st = dense(wk, L.shared_up_w, wk == WK_INT8 ? L.shared_up_scale : nullptr, L.shared_up_b, x,
               T, H, Is, ws.s1, false, true, err, s);
    if (st != NK_OK) return st;
    st = dense(wk, L.shared_down_w, wk == WK_INT8 ? L.shared_down_scale : nullptr,
               L.shared_down_b, ws.s1, T, Is, H, ws.sh, false, false, err, s);
    if (st != NK_OK) return st;
  }
  tm.mark(6, s);
  // 8. combine in rank order
  if (out_dtype == NK_F32)
    combine_kernel<true><<<(unsigned)T, 128, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16 *>(yrouted),
        reinterpret_cast<const __nv_bfloat16 *>(ws.sh), rw, ws.slot_pos, H, (int)K, out);
  else
    combine_kernel<false><<<(unsigned)T, 128, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16 *>(yrouted),
        reinterpret_cast<const __nv_bfloat16 *>(ws.sh), rw, ws.slot_pos, H, (int)K, out);
  st = check_launch("combine_kernel");
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

}  // extern "C"
