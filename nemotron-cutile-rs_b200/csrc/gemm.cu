// gemm.cu — GEMM entry points of nk.h: the reference-layout f32 GEMM
// (f64 accumulation, SIMT) and the projection GEMMs, which dispatch to the
// tcgen05 kernel (gemm_tc.cu) or, for shapes TMA cannot address (a row pitch
// that is not a multiple of 16 bytes), to a plain CUDA kernel.
#include <cmath>
#include <cstdlib>

#include "gemm_tc.h"

namespace nk {

// ---------------------------------------------------------------- f32 GEMM
// C[M,N] = A[M,K]·B[K,N] with f64 accumulation, rounded once to f32 — the
// arithmetic of gemm_into_host (gemm.rs:99-109).  64x64 output tile, 256
// threads, 4x4 outputs per thread, K staged 16 at a time through shared memory.
__global__ void __launch_bounds__(256) gemm_f32_f64acc_kernel(const float *__restrict__ A,
                                                              const float *__restrict__ B,
                                                              float *__restrict__ C, int64_t M,
                                                              int64_t K, int64_t N) {
  __shared__ double As[16][64 + 1];
  __shared__ double Bs[16][64 + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t row0 = (int64_t)blockIdx.y * 64, col0 = (int64_t)blockIdx.x * 64;
  double acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += 16) {
    for (int e = threadIdx.x; e < 16 * 64; e += 256) {
      int kk = e / 64, r = e % 64;  // A: element (row0+r, k0+kk)
      int64_t gr = row0 + r, gk = k0 + kk;
      As[kk][r] = (gr < M && gk < K) ? (double)A[gr * K + gk] : 0.0;
      int64_t gc = col0 + r;  // B: element (k0+kk, col0+r), coalesced along N
      Bs[kk][r] = (gk < K && gc < N) ? (double)B[gk * N + gc] : 0.0;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      double a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fma(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int64_t r = row0 + ty + 16 * i, c = col0 + tx + 16 * j;
      if (r < M && c < N) C[r * N + c] = (float)acc[i][j];
    }
}

// ------------------------------------------------------- projection helpers
// Two-way split of f32 activations into bf16 hi | lo halves, written as
// X2[m, 0:Kp] = hi, X2[m, Kp:2Kp] = lo (zero padded to Kp = ceil(K/64)*64).
// hi + lo keeps the top 16 of the 24 significand bits (relative error below
// 2^-16 per element), well inside the f32-activation bar of 1e-3.
__global__ void split_f32_kernel(const float *__restrict__ x, __nv_bfloat16 *__restrict__ x2,
                                 int64_t M, int64_t K, int64_t Kp) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= M * Kp) return;
  int64_t m = idx / Kp, k = idx - m * Kp;
  float v = k < K ? x[m * K + k] : 0.0f;
  __nv_bfloat16 hi = __float2bfloat16_rn(v);
  __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
  x2[m * 2 * Kp + k] = hi;
  x2[m * 2 * Kp + Kp + k] = lo;
}

nk_status launch_split_f32(const float *x, int64_t m, int64_t k, int64_t kp, uint16_t *x2,
                           cudaStream_t stream) {
  const int64_t total = m * kp;
  split_f32_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, stream>>>(
      x, reinterpret_cast<__nv_bfloat16 *>(x2), m, k, kp);
  return check_launch("split_f32_kernel");
}

// Plain CUDA projection for shapes outside the TMA envelope: one thread per
// output, f32 accumulation, the same epilogue as the tensor-core kernel.
template <int WK>
__global__ void proj_simt_kernel(const void *__restrict__ x, int x_f32,
                                 const void *__restrict__ w, float w_scale, int zp,
                                 const float *__restrict__ row_scale,
                                 const float *__restrict__ bias, void *__restrict__ y, int y_f32,
                                 int relu2, int64_t M, int64_t K, int64_t N) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= M * N) return;
  int64_t m = idx / N, n = idx - m * N;
  float acc = 0.0f;
  for (int64_t k = 0; k < K; ++k) {
    float xv = x_f32 ? reinterpret_cast<const float *>(x)[m * K + k]
                     : __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(x)[m * K + k]);
    float wv;
    if (WK == WK_BF16) {
      wv = __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(w)[n * K + k]);
    } else if (WK == WK_INT8) {
      wv = (float)reinterpret_cast<const int8_t *>(w)[n * K + k];
    } else {
      int64_t flat = k * N + n;  // reference [K,N] layout
      uint8_t b = reinterpret_cast<const uint8_t *>(w)[flat >> 1];
      wv = (float)((int)((flat & 1) ? (b >> 4) : (b & 0xF)) - zp);
    }
    acc = fmaf(xv, wv, acc);
  }
  float o = acc * w_scale;
  if (row_scale) o *= row_scale[n];
  if (bias) o += bias[n];
  if (relu2) o = nk_relu2(o);
  if (y_f32)
    reinterpret_cast<float *>(y)[idx] = o;
  else
    reinterpret_cast<__nv_bfloat16 *>(y)[idx] = __float2bfloat16_rn(o);
}

// y[m, n] = act(Σ_s partial[s][m, n] + bias[n]), partial sums added in split order.
// Launched as a programmatic dependent of the GEMM: its blocks are scheduled
// while the GEMM runs and wait (griddepcontrol.wait) for its completion, so the
// launch latency is hidden.  Loads of four splits are issued together.
__global__ void splitk_reduce_kernel(const float *__restrict__ part, int splits, int64_t mn,
                                     int64_t n, const float *__restrict__ bias, int relu2,
                                     void *__restrict__ y, int y_f32) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= mn) return;
  float acc = part[i];
  int s = 1;
  for (; s + 4 <= splits; s += 4) {
    const float a0 = part[(int64_t)s * mn + i], a1 = part[(int64_t)(s + 1) * mn + i];
    const float a2 = part[(int64_t)(s + 2) * mn + i], a3 = part[(int64_t)(s + 3) * mn + i];
    acc = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc, a0), a1), a2), a3);
  }
  for (; s < splits; ++s) acc = __fadd_rn(acc, part[(int64_t)s * mn + i]);
  if (bias) acc = __fadd_rn(acc, bias[i % n]);
  if (relu2) acc = nk_relu2(acc);
  if (y_f32)
    reinterpret_cast<float *>(y)[i] = acc;
  else
    reinterpret_cast<__nv_bfloat16 *>(y)[i] = __float2bfloat16_rn(acc);
}

// Launches splitk_reduce_kernel as a programmatic dependent of the previous kernel.
static nk_status launch_splitk_reduce(const float *part, int splits, int64_t mn, int64_t n,
                                      const float *bias, bool relu2, void *y, bool y_f32,
                                      cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ceil_div(mn, 256));
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  NK_CUDA_TRY(cudaLaunchKernelEx(&cfg, splitk_reduce_kernel, part, splits, mn, n, bias,
                                 (int)relu2, y, (int)y_f32));
  return check_launch("splitk_reduce_kernel");
}

// Decode-size projections on the weight-streaming kernel (gemv.cu).
int gemv_splits(int wk, int64_t n, int64_t k, int64_t *k_per_split);
void launch_gemv(int wk, const void *x, bool x_f32, int m, const void *w, int64_t n, int64_t k,
                 int64_t kps, int splits, float w_scale, const float *row_scale,
                 const float *bias, int relu2, void *y, int y_f32, float *part,
                 cudaStream_t s);

// K splits for a projection whose token dimension fits one tile (decode
// shapes, HBM-bound).  Cost model in bytes moved: the weight stream stretched
// by wave quantisation (units of work over whole waves of SMs), plus the f32
// partial sums written and read back, plus a fixed cost for the extra reduce
// launch.  Each split keeps >= 4 K blocks.
static int choose_k_splits(int f_tiles, int t_tiles, int k_blocks, int sms, double w_bytes,
                           int64_t m, int64_t n) {
  if (t_tiles != 1) return 1;
  auto cost = [&](int s) {
    const double units = (double)f_tiles * s;
    const double eff = units / (std::ceil(units / sms) * sms);
    double c = w_bytes / eff;
    if (s > 1) c += 8.0 * s * (double)m * (double)n + 20e6;
    return c;
  };
  int best_s = 1;
  double best = cost(1);
  for (int s = 2; s <= 32 && k_blocks / s >= 4; ++s) {
    const double c = cost(s);
    if (c < best * 0.97) {
      best = c;
      best_s = s;
    }
  }
  return best_s;
}

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// How one projection runs: which kernel, its K splits and the scratch it
// needs ([split activations (f32 x)] [split-K partial sums]).
struct ProjPlan {
  enum { SIMT, GEMV, TC } path;
  int gemv_splits = 1;
  int64_t gemv_kps = 0;
  int k_blocks = 0, w_period = 0, bn = 0, splits = 1, pair = 1;
  int64_t kp = 0;
  size_t xsplit_bytes = 0, part_off = 0, part_bytes = 0, scratch_bytes = 0;
};

static ProjPlan plan_projection(int wk, bool aligned, int x_dtype, int64_t m, int64_t k,
                                int64_t n) {
  ProjPlan p;
  bool tc_ok = aligned;
  if (wk == WK_BF16) tc_ok &= (k % 8) == 0;
  if (wk == WK_INT8) tc_ok &= (k % 16) == 0;
  if (wk == WK_INT4KN) tc_ok &= (n % 32) == 0;
  if (x_dtype == NK_BF16) tc_ok &= (k % 8) == 0;
  if (!tc_ok) {
    p.path = ProjPlan::SIMT;
    return p;
  }
  // One or two token rows: stream the weights through registers (gemv.cu);
  // measured faster than the tensor-core kernel there, slower from 4 rows.
  // NK_GEMV=0 keeps such shapes on the tensor-core kernel (a tuning probe).
  static const bool gemv_on = [] {
    const char *e = getenv("NK_GEMV");
    return !(e && e[0] == '0');
  }();
  if (gemv_on && m <= 2 && (wk == WK_BF16 || wk == WK_INT8) && (k % 16) == 0 &&
      (x_dtype == NK_BF16 || (k % 4) == 0)) {
    p.path = ProjPlan::GEMV;
    p.gemv_splits = gemv_splits(wk, n, k, &p.gemv_kps);
    p.part_bytes = p.gemv_splits > 1 ? (size_t)p.gemv_splits * m * n * 4 : 0;
    p.scratch_bytes = p.part_bytes;
    return p;
  }
  p.path = ProjPlan::TC;
  p.k_blocks = (int)ceil_div(k, 64);
  p.kp = ceil_div(k, 64) * 64;
  if (x_dtype == NK_F32) {
    p.w_period = (int)(p.kp / 64);
    p.k_blocks = 2 * p.w_period;
  }
  p.bn = m <= 16 ? 16 : (m <= 64 ? 64 : 256);
  const int f_tiles = (int)ceil_div(n, 128), t_tiles = (int)ceil_div(m, p.bn);
  const double w_bytes = (double)n * (double)k * (wk == WK_BF16 ? 2.0 : wk == WK_INT8 ? 1.0 : 0.5);
  int splits = choose_k_splits(f_tiles, t_tiles, p.k_blocks, num_sms(), w_bytes, m, n);
  if (const char *e = getenv("NK_SPLITK")) {  // tuning override: forced K split count
    int v = atoi(e);
    if (v >= 1 && v <= p.k_blocks) splits = v;
  }
  {  // every split gets at least one K block
    const int per = (p.k_blocks + splits - 1) / splits;
    splits = (p.k_blocks + per - 1) / per;
  }
  p.splits = splits;
  // Prefill shapes (more than one token tile) can run on CTA pairs: 256-feature
  // tiles, each SM loading half of every token tile.  Measured no faster than
  // single CTAs for bf16 weights and slower for int8 on B200, so opt-in
  // (NK_PAIR=1).
  static const bool pair_ok = [] {
    const char *e = getenv("NK_PAIR");
    return e && e[0] == '1';
  }();
  p.pair = (pair_ok && t_tiles >= 2 && p.bn == 256) ? 2 : 1;
  p.xsplit_bytes = x_dtype == NK_F32 ? (size_t)(m * 2 * p.kp * 2) : 0;
  p.part_off = (p.xsplit_bytes + 255) & ~size_t(255);
  p.part_bytes = splits > 1 ? (size_t)splits * m * n * 4 : 0;
  p.scratch_bytes = p.xsplit_bytes + p.part_bytes > 0 ? p.part_off + p.part_bytes : 0;
  return p;
}

static nk_status check_proj_args(int x_dtype, int y_dtype, int64_t m, int64_t k, int64_t n) {
  if (m <= 0 || k <= 0 || n <= 0) return fail(NK_INVALID_SHAPE, "m, k and n must be positive");
  if (x_dtype != NK_BF16 && x_dtype != NK_F32) return fail(NK_UNSUPPORTED, "x_dtype");
  if (y_dtype != NK_BF16 && y_dtype != NK_F32) return fail(NK_UNSUPPORTED, "y_dtype");
  if (m > (1ll << 30) || n > (1ll << 30) || k > (1ll << 30))
    return fail(NK_INVALID_SHAPE, "dimension too large");
  return NK_OK;
}

// Shared driver for nk_gemm_bf16 / nk_gemm_w8row / nk_gemm_w4a (and their
// _ws forms).  workspace: caller-owned scratch of at least the planned bytes,
// or null for the library's per-(device, stream) scratch.
nk_status projection(int wk, const void *x, int x_dtype, const void *w, float w_scale, int zp,
                     const float *row_scale, const float *bias, void *y, int y_dtype,
                     int64_t m, int64_t k, int64_t n, int flags, cudaStream_t stream,
                     void *workspace = nullptr, size_t workspace_bytes = 0) {
  nk_status st = check_proj_args(x_dtype, y_dtype, m, k, n);
  if (st != NK_OK) return st;
  int *err = device_error_ptr();
  const bool relu2 = (flags & NK_EPI_RELU2) != 0;
  const ProjPlan p = plan_projection(wk, aligned16(x) && aligned16(w), x_dtype, m, k, n);

  uint8_t *buf = nullptr;
  if (p.scratch_bytes > 0) {
    if (workspace) {
      if (workspace_bytes < p.scratch_bytes) {
        st = fail(NK_WORKSPACE_TOO_SMALL, "workspace smaller than nk_gemm_workspace_bytes");
        tls_error().expected = p.scratch_bytes;
        tls_error().actual = workspace_bytes;
        return st;
      }
      buf = reinterpret_cast<uint8_t *>(workspace);
    } else {
      void *b = nullptr;
      st = scratch(p.scratch_bytes, &b, stream);
      if (st != NK_OK) return st;
      buf = reinterpret_cast<uint8_t *>(b);
    }
  }

  if (p.path == ProjPlan::SIMT) {
    int64_t total = m * n;
    int threads = 256;
    int64_t blocks = (total + threads - 1) / threads;
    if (wk == WK_BF16)
      proj_simt_kernel<WK_BF16><<<(unsigned)blocks, threads, 0, stream>>>(
          x, x_dtype == NK_F32, w, w_scale, zp, row_scale, bias, y, y_dtype == NK_F32, relu2, m,
          k, n);
    else if (wk == WK_INT8)
      proj_simt_kernel<WK_INT8><<<(unsigned)blocks, threads, 0, stream>>>(
          x, x_dtype == NK_F32, w, w_scale, zp, row_scale, bias, y, y_dtype == NK_F32, relu2, m,
          k, n);
    else
      proj_simt_kernel<WK_INT4KN><<<(unsigned)blocks, threads, 0, stream>>>(
          x, x_dtype == NK_F32, w, w_scale, zp, row_scale, bias, y, y_dtype == NK_F32, relu2, m,
          k, n);
    return check_launch("proj_simt_kernel");
  }

  if (p.path == ProjPlan::GEMV) {
    const int splits = p.gemv_splits;
    float *part = splits > 1 ? reinterpret_cast<float *>(buf) : nullptr;
    launch_gemv(wk, x, x_dtype == NK_F32, (int)m, w, n, k, p.gemv_kps, splits, w_scale,
                row_scale, splits > 1 ? nullptr : bias, splits > 1 ? 0 : (int)relu2, y,
                y_dtype == NK_F32, part, stream);
    st = check_launch("gemv_kernel");
    if (st != NK_OK || splits == 1) return st;
    return launch_splitk_reduce(part, splits, m * n, n, bias, relu2, y, y_dtype == NK_F32,
                                stream);
  }

  const uint16_t *xb = reinterpret_cast<const uint16_t *>(x);
  int64_t x_k = k, ldx = k;
  if (x_dtype == NK_F32) {
    st = launch_split_f32(reinterpret_cast<const float *>(x), m, k, p.kp,
                          reinterpret_cast<uint16_t *>(buf), stream);
    if (st != NK_OK) return st;
    xb = reinterpret_cast<const uint16_t *>(buf);
    x_k = 2 * p.kp;
    ldx = 2 * p.kp;
  }
  const int splits = p.splits, pair = p.pair;
  const int t_tiles = (int)ceil_div(m, p.bn);
  TcArgs a{};
  a.f_tiles = (int)ceil_div(n, 128 * pair);
  a.t_tiles = t_tiles;
  a.n_features = (int)n;
  a.n_tokens = (int)m;
  a.k_blocks = p.k_blocks;
  a.w_k_period = p.w_period;
  a.x_k_period = 0;
  a.w_scale = w_scale;
  a.row_scale = row_scale;
  a.w_zero_point = zp;
  a.err = err;
  a.ldy = n;
  if (splits > 1) {  // partial sums (row scale is linear, applied per split)
    a.k_splits = splits;
    a.split_stride = m * n;
    a.y = buf + p.part_off;
    a.y_f32 = 1;
  } else {
    a.y = y;
    a.y_f32 = y_dtype == NK_F32;
    a.bias = bias;
    a.relu2 = relu2;
  }
  int64_t tiles = (int64_t)a.f_tiles * t_tiles * splits;
  const int slots = num_sms() / pair;  // concurrent tiles
  int grid = (int)(tiles < slots ? tiles : slots) * pair;
  int64_t ldw_bytes = wk == WK_BF16 ? k * 2 : (wk == WK_INT8 ? k : n / 2);
  st = tc_gemm(wk, w, n, k, ldw_bytes, xb, m, x_k, ldx, p.bn, a, grid, stream, pair);
  if (st != NK_OK || splits == 1) return st;
  const int64_t mn = m * n;
  return launch_splitk_reduce(reinterpret_cast<const float *>(buf + p.part_off), splits, mn, n,
                              bias, relu2, y, y_dtype == NK_F32, stream);
}

size_t projection_scratch_bytes(int wk, int x_dtype, int64_t m, int64_t k, int64_t n) {
  return plan_projection(wk, true, x_dtype, m, k, n).scratch_bytes;
}

}  // namespace nk

using namespace nk;

extern "C" {

nk_status nk_gemm_f32(const float *lhs, size_t lhs_len, const float *rhs, size_t rhs_len,
                      float *out, size_t out_len, size_t m, size_t k, size_t n, void *stream) {
  uint64_t ll, rl, ol;
  if (m == 0 || k == 0 || n == 0 || !mul_ok(m, k, &ll) || !mul_ok(k, n, &rl) ||
      !mul_ok(m, n, &ol))
    return fail(NK_INVALID_SHAPE, "invalid GEMM shape");
  if (lhs_len != ll) return fail_length("lhs", ll, lhs_len);
  if (rhs_len != rl) return fail_length("rhs", rl, rhs_len);
  if (out_len != ol) return fail_length("output", ol, out_len);
  dim3 grid((unsigned)ceil_div((int64_t)n, 64), (unsigned)ceil_div((int64_t)m, 64));
  if (grid.y > 65535) return fail(NK_UNSUPPORTED, "m too large for one launch");
  gemm_f32_f64acc_kernel<<<grid, 256, 0, as_stream(stream)>>>(lhs, rhs, out, (int64_t)m,
                                                              (int64_t)k, (int64_t)n);
  return check_launch("gemm_f32_f64acc_kernel");
}

nk_status nk_gemm_bf16(const void *x, int32_t x_dtype, const uint16_t *w, const float *bias,
                       void *y, int32_t y_dtype, int64_t m, int64_t k, int64_t n, int32_t flags,
                       void *stream) {
  return projection(WK_BF16, x, x_dtype, w, 1.0f, 0, nullptr, bias, y, y_dtype, m, k, n, flags,
                    as_stream(stream));
}

nk_status nk_gemm_w8row(const void *x, int32_t x_dtype, const int8_t *wq, const float *scales,
                        const float *bias, void *y, int32_t y_dtype, int64_t m, int64_t k,
                        int64_t n, int32_t flags, void *stream) {
  return projection(WK_INT8, x, x_dtype, wq, 1.0f, 0, scales, bias, y, y_dtype, m, k, n, flags,
                    as_stream(stream));
}

nk_status nk_gemm_workspace_bytes(int32_t weight_kind, int32_t x_dtype, int64_t m, int64_t k,
                                  int64_t n, size_t *bytes) {
  nk_status st = check_proj_args(x_dtype, NK_F32, m, k, n);
  if (st != NK_OK) return st;
  int wk;
  if (weight_kind == NK_W_BF16) wk = WK_BF16;
  else if (weight_kind == NK_W_INT8_ROW) wk = WK_INT8;
  else if (weight_kind == NK_W_INT4_AFFINE) wk = WK_INT4KN;
  else return fail(NK_UNSUPPORTED, "weight_kind");
  if (!bytes) return fail(NK_INVALID_PARAMS, "bytes is null");
  *bytes = projection_scratch_bytes(wk, x_dtype, m, k, n);
  return ok();
}

nk_status nk_gemm_bf16_ws(const void *x, int32_t x_dtype, const uint16_t *w, const float *bias,
                          void *y, int32_t y_dtype, int64_t m, int64_t k, int64_t n,
                          int32_t flags, void *workspace, size_t workspace_bytes, void *stream) {
  nk_status st = projection(WK_BF16, x, x_dtype, w, 1.0f, 0, nullptr, bias, y, y_dtype, m, k, n,
                            flags, as_stream(stream), workspace, workspace_bytes);
  return st == NK_OK ? ok() : st;
}

nk_status nk_gemm_w8row_ws(const void *x, int32_t x_dtype, const int8_t *wq, const float *scales,
                           const float *bias, void *y, int32_t y_dtype, int64_t m, int64_t k,
                           int64_t n, int32_t flags, void *workspace, size_t workspace_bytes,
                           void *stream) {
  nk_status st = projection(WK_INT8, x, x_dtype, wq, 1.0f, 0, scales, bias, y, y_dtype, m, k, n,
                            flags, as_stream(stream), workspace, workspace_bytes);
  return st == NK_OK ? ok() : st;
}

nk_status nk_gemm_w4a_ws(const void *x, int32_t x_dtype, const uint8_t *packed, size_t packed_len,
                         float scale, uint32_t zero_point, const float *bias, void *y,
                         int32_t y_dtype, int64_t m, int64_t k, int64_t n, int32_t flags,
                         void *workspace, size_t workspace_bytes, void *stream) {
  if (m <= 0 || k <= 0 || n <= 0) return fail(NK_INVALID_SHAPE, "m, k and n must be positive");
  nk_status st = nk_validate_int4_params(scale, zero_point);
  if (st != NK_OK) return st;
  uint64_t count = (uint64_t)k * (uint64_t)n;
  uint64_t expect = count / 2 + (count & 1);
  if (packed_len != expect) return fail_length("packed_weights", expect, packed_len);
  st = projection(WK_INT4KN, x, x_dtype, packed, scale, (int)zero_point, nullptr, bias, y,
                  y_dtype, m, k, n, flags, as_stream(stream), workspace, workspace_bytes);
  return st == NK_OK ? ok() : st;
}

nk_status nk_gemm_w4a(const void *x, int32_t x_dtype, const uint8_t *packed, size_t packed_len,
                      float scale, uint32_t zero_point, const float *bias, void *y,
                      int32_t y_dtype, int64_t m, int64_t k, int64_t n, int32_t flags,
                      void *stream) {
  if (m <= 0 || k <= 0 || n <= 0) return fail(NK_INVALID_SHAPE, "m, k and n must be positive");
  nk_status st = nk_validate_int4_params(scale, zero_point);
  if (st != NK_OK) return st;
  uint64_t count = (uint64_t)k * (uint64_t)n;
  uint64_t expect = count / 2 + (count & 1);
  if (packed_len != expect) return fail_length("packed_weights", expect, packed_len);
  return projection(WK_INT4KN, x, x_dtype, packed, scale, (int)zero_point, nullptr, bias, y,
                    y_dtype, m, k, n, flags, as_stream(stream));
}

}  // extern "C"
