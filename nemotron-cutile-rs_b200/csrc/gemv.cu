// gemv.cu — decode-size projections (at most 4 token rows): Y = X·Wᵀ with
// the weights streamed straight from HBM into registers.
//
// With a handful of tokens every weight element feeds at most 4 FMAs, so
// the projection is a pure weight stream (HBM-bound) and the tensor cores buy
// nothing; what matters is keeping enough bytes in flight and touching every
// weight byte once.  A warp owns R weight rows (4 bf16, 8 int8); each lane
// reads 16 consecutive K elements of each row per step (32 bytes of bf16, 16 of int8;
// the next step's are loaded before the current step is used), converts them
// to f32 in registers and multiplies them with the same 16 K elements of
// every token row (read through L1: X is small and shared by all warps).
// The prefetched weights stay packed (bf16 / int8) until used, which keeps
// two 256-thread blocks resident per SM.  Partial sums stay in registers
// (R x MT per lane) and are reduced across the warp once at the end.  Long K is split over
// blockIdx.y so that the grid covers every SM several times; split partials
// are summed in split order by splitk_reduce_kernel (deterministic).
#include "gemm_tc.cuh"
#include "nk_common.cuh"

namespace nk {

// 16 K elements of a weight row, kept packed: 2 x 16 bytes (bf16) or 16 bytes (int8).
struct Packed16 {
  uint4 a, b;
};
__device__ __forceinline__ void fetch16(const __nv_bfloat16 *p, Packed16 &q) {
  q.a = __ldg(reinterpret_cast<const uint4 *>(p));
  q.b = __ldg(reinterpret_cast<const uint4 *>(p) + 1);
}
__device__ __forceinline__ void fetch16(const int8_t *p, Packed16 &q) {
  q.a = __ldg(reinterpret_cast<const uint4 *>(p));
}
__device__ __forceinline__ void unpack16(const Packed16 &q, __nv_bfloat16 *, float (&v)[16]) {
  const uint32_t w[8] = {q.a.x, q.a.y, q.a.z, q.a.w, q.b.x, q.b.y, q.b.z, q.b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ void unpack16(const Packed16 &q, int8_t *, float (&v)[16]) {
  // Exact int8 -> f32 on the FMA pipe: the biased byte u = v + 128 placed in
  // the mantissa of 2^23 gives 2^23 + u, minus (2^23 + 128) leaves v.
  const uint32_t w[4] = {q.a.x ^ 0x80808080u, q.a.y ^ 0x80808080u, q.a.z ^ 0x80808080u,
                         q.a.w ^ 0x80808080u};
#pragma unroll
  for (int i = 0; i < 16; ++i)
    v[i] = __uint_as_float(__byte_perm(w[i >> 2], 0x4B000000u, 0x7540 | (i & 3))) -
           8388736.0f;
}
__device__ __forceinline__ void load16(const __nv_bfloat16 *p, float (&v)[16]) {
  Packed16 q;
  fetch16(p, q);
  unpack16(q, (__nv_bfloat16 *)nullptr, v);
}
__device__ __forceinline__ void load16(const float *p, float (&v)[16]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 a = __ldg(reinterpret_cast<const float4 *>(p) + i);
    v[4 * i] = a.x; v[4 * i + 1] = a.y; v[4 * i + 2] = a.z; v[4 * i + 3] = a.w;
  }
}

// Block = 8 warps, warp w owns rows n0 + w*R .. +R-1; grid = (ceil(N / 8R), splits).
template <typename WT, typename XT, int MT, int R>
__global__ void __launch_bounds__(256, 2) gemv_kernel(const XT *__restrict__ x, int m,
                                                   const WT *__restrict__ w, int64_t n,
                                                   int64_t k, int64_t k_per_split, float w_scale,
                                                   const float *__restrict__ row_scale,
                                                   const float *__restrict__ bias, int relu2,
                                                   void *__restrict__ y, int y_f32,
                                                   float *__restrict__ part) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const int64_t row0 = ((int64_t)blockIdx.x * 8 + (threadIdx.x >> 5)) * R;
  const int split = blockIdx.y;
  const int64_t kb = (int64_t)split * k_per_split;
  const int64_t ke = kb + k_per_split < k ? kb + k_per_split : k;
  float acc[R][MT];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[r][t] = 0.0f;

  const WT *wr[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int64_t row = row0 + r < n ? row0 + r : n - 1;  // tail rows read a valid row
    wr[r] = w + row * k;
  }
  // 16 K elements per lane per step (512 per warp); the next step's weights
  // are fetched before the current step's FMAs.
  int64_t kk = kb + lane * 16;
  Packed16 nxt[R];
  if (kk < ke) {
#pragma unroll
    for (int r = 0; r < R; ++r) fetch16(wr[r] + kk, nxt[r]);
  }
  for (; kk < ke; kk += 512) {
    Packed16 cur[R];
#pragma unroll
    for (int r = 0; r < R; ++r) cur[r] = nxt[r];
    if (kk + 512 < ke) {
#pragma unroll
      for (int r = 0; r < R; ++r) fetch16(wr[r] + kk + 512, nxt[r]);
    }
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      if (t < m) {
        float xv[16];
        load16(x + (int64_t)t * k + kk, xv);
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float wv[16];  // unpacked per token row: a few ALU ops, no registers held
          unpack16(cur[r], (WT *)nullptr, wv);
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[r][t] = fmaf(wv[j], xv[j], acc[r][t]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[r][t] += __shfl_xor_sync(0xffffffffu, acc[r][t], o);
  if (lane != 0) return;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int64_t row = row0 + r;
    if (row >= n) break;
    const float mul = w_scale * (row_scale ? row_scale[row] : 1.0f);
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      if (t >= m) break;
      float o = acc[r][t] * mul;
      if (part) {
        part[((int64_t)split * m + t) * n + row] = o;
      } else {
        if (bias) o = __fadd_rn(o, bias[row]);
        if (relu2) o = nk_relu2(o);
        if (y_f32)
          reinterpret_cast<float *>(y)[(int64_t)t * n + row] = o;
        else
          reinterpret_cast<__nv_bfloat16 *>(y)[(int64_t)t * n + row] = __float2bfloat16_rn(o);
      }
    }
  }
}

template <typename WT, typename XT, int MT>
static void launch_gemv_t(const void *x, int m, const void *w, int64_t n, int64_t k, int64_t kps,
                          int splits, float w_scale, const float *row_scale, const float *bias,
                          int relu2, void *y, int y_f32, float *part, cudaStream_t s) {
  constexpr int R = sizeof(WT) == 1 ? 8 : 4;  // 128 weight bytes per lane per step
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ceil_div(n, 8 * R), (unsigned)splits);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, gemv_kernel<WT, XT, MT, R>, reinterpret_cast<const XT *>(x), m,
                     reinterpret_cast<const WT *>(w), n, k, kps, w_scale, row_scale, bias, relu2,
                     y, y_f32, part);
}

template <typename WT, typename XT>
static void launch_gemv_m(const void *x, int m, const void *w, int64_t n, int64_t k, int64_t kps,
                          int splits, float w_scale, const float *row_scale, const float *bias,
                          int relu2, void *y, int y_f32, float *part, cudaStream_t s) {
  if (m <= 1)
    launch_gemv_t<WT, XT, 1>(x, m, w, n, k, kps, splits, w_scale, row_scale, bias, relu2, y,
                             y_f32, part, s);
  else if (m <= 2)
    launch_gemv_t<WT, XT, 2>(x, m, w, n, k, kps, splits, w_scale, row_scale, bias, relu2, y,
                             y_f32, part, s);
  else
    launch_gemv_t<WT, XT, 4>(x, m, w, n, k, kps, splits, w_scale, row_scale, bias, relu2, y,
                             y_f32, part, s);
}

// Splits of K: enough blocks for ~4 per SM, each split >= 2048 K elements,
// a multiple of 512 (one step of the warp's lanes).
int gemv_splits(int wk, int64_t n, int64_t k, int64_t *k_per_split) {
  const int R = wk == WK_INT8 ? 8 : 4;
  const int64_t blocks_n = ceil_div(n, 8 * R);
  int64_t splits = ceil_div((int64_t)num_sms() * 4, blocks_n);
  const int64_t max_splits = k / 2048 > 1 ? k / 2048 : 1;
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  int64_t kps = ceil_div(ceil_div(k, splits), 512) * 512;
  splits = ceil_div(k, kps);
  *k_per_split = kps;
  return (int)splits;
}

void launch_gemv(int wk, const void *x, bool x_f32, int m, const void *w, int64_t n, int64_t k,
                 int64_t kps, int splits, float w_scale, const float *row_scale,
                 const float *bias, int relu2, void *y, int y_f32, float *part,
                 cudaStream_t s) {
  if (wk == WK_BF16) {
    if (x_f32)
      launch_gemv_m<__nv_bfloat16, float>(x, m, w, n, k, kps, splits, w_scale, row_scale, bias,
                                          relu2, y, y_f32, part, s);
    else
      launch_gemv_m<__nv_bfloat16, __nv_bfloat16>(x, m, w, n, k, kps, splits, w_scale,
                                                  row_scale, bias, relu2, y, y_f32, part, s);
  } else {
    if (x_f32)
      launch_gemv_m<int8_t, float>(x, m, w, n, k, kps, splits, w_scale, row_scale, bias, relu2,
                                   y, y_f32, part, s);
    else
      launch_gemv_m<int8_t, __nv_bfloat16>(x, m, w, n, k, kps, splits, w_scale, row_scale,
                                           bias, relu2, y, y_f32, part, s);
  }
}

}  // namespace nk
