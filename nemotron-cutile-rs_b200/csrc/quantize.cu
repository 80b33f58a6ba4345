// quantize.cu — INT4-affine pack/unpack/quantize/dequantize (the reference's
// format, quantize.rs:53-204), int8 per-row quantization, and the weight
// layout conversions the projection GEMMs read.
#include <math.h>

#include "nk_common.cuh"

namespace nk {

// First index i < n with pred(i) true, via atomicMin on a 64-bit word.
__global__ void first_nonfinite_kernel(const float *__restrict__ v, uint64_t n,
                                       unsigned long long *first) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    if (!isfinite(v[i])) atomicMin(first, (unsigned long long)i);
}

__global__ void first_above15_kernel(const uint8_t *__restrict__ v, uint64_t n,
                                     unsigned long long *first) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    if (v[i] > 0x0F) atomicMin(first, (unsigned long long)i);
}

// quantize.rs:59-81: even index -> low nibble, odd -> high nibble.
__global__ void pack_int4_kernel(const uint8_t *__restrict__ v, uint64_t n,
                                 uint8_t *__restrict__ packed, uint64_t packed_len) {
  for (uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; b < packed_len;
       b += (uint64_t)gridDim.x * blockDim.x) {
    uint8_t lo = v[2 * b];
    uint8_t hi = (2 * b + 1 < n) ? v[2 * b + 1] : 0;
    packed[b] = (uint8_t)(lo | (hi << 4));
  }
}

__global__ void unpack_int4_kernel(const uint8_t *__restrict__ packed, uint64_t n,
                                   uint8_t *__restrict__ out) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    uint8_t b = packed[i >> 1];
    out[i] = (i & 1) ? ((b >> 4) & 0x0F) : (b & 0x0F);
  }
}

// quantize_scalar (quantize.rs:188-200): round(v/scale + zp) half away from
// zero, clamped to [0, 15].  IEEE division and addition, no contraction.
__device__ __forceinline__ uint8_t quant4(float v, float scale, float zp) {
  float s = __fadd_rn(__fdiv_rn(v, scale), zp);
  float q = fminf(fmaxf(roundf(s), 0.0f), 15.0f);
  return (uint8_t)q;
}

__global__ void quantize_int4_kernel(const float *__restrict__ v, uint64_t n, float scale,
                                     float zp, uint8_t *__restrict__ packed,
                                     uint64_t packed_len) {
  for (uint64_t b = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; b < packed_len;
       b += (uint64_t)gridDim.x * blockDim.x) {
    uint8_t lo = quant4(v[2 * b], scale, zp);
    uint8_t hi = (2 * b + 1 < n) ? quant4(v[2 * b + 1], scale, zp) : 0;
    packed[b] = (uint8_t)(lo | (hi << 4));
  }
}

// dequantize_scalar (quantize.rs:202-204): (code - zp) * scale.
__global__ void dequantize_int4_kernel(const uint8_t *__restrict__ packed, uint64_t n,
                                       float scale, float zp, float *__restrict__ out) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    uint8_t b = packed[i >> 1];
    float code = (float)((i & 1) ? ((b >> 4) & 0x0F) : (b & 0x0F));
    out[i] = __fmul_rn(__fsub_rn(code, zp), scale);
  }
}

// One CTA per weight row: absmax reduction, then codes.
__global__ void quantize_int8_row_kernel(const float *__restrict__ w, int64_t k,
                                         int8_t *__restrict__ q, float *__restrict__ scales) {
  const float *row = w + (int64_t)blockIdx.x * k;
  float amax = 0.0f;
  for (int64_t c = threadIdx.x; c < k; c += blockDim.x) amax = fmaxf(amax, fabsf(row[c]));
  __shared__ float red[32];
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float s = __fdiv_rn(red[0], 127.0f);
  if (threadIdx.x == 0) scales[blockIdx.x] = s;
  int8_t *qrow = q + (int64_t)blockIdx.x * k;
  for (int64_t c = threadIdx.x; c < k; c += blockDim.x) {
    float v = 0.0f;
    if (s > 0.0f) v = fminf(fmaxf(roundf(__fdiv_rn(row[c], s)), -127.0f), 127.0f);
    qrow[c] = (int8_t)v;
  }
}

// f32 [E,H] -> bf16 [E, 3*Hp] = hi | mid | lo, zero padded to Hp = ceil(H/64)*64.
__global__ void router_split_kernel(const float *__restrict__ w, int64_t E, int64_t H,
                                    int64_t Hp, __nv_bfloat16 *__restrict__ w3) {
  int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= E * Hp) return;
  int64_t e = idx / Hp, h = idx - e * Hp;
  float v = h < H ? w[e * H + h] : 0.0f;
  __nv_bfloat16 hi = __float2bfloat16_rn(v);
  float r1 = __fsub_rn(v, __bfloat162float(hi));
  __nv_bfloat16 mid = __float2bfloat16_rn(r1);
  float r2 = __fsub_rn(r1, __bfloat162float(mid));
  __nv_bfloat16 lo = __float2bfloat16_rn(r2);
  __nv_bfloat16 *row = w3 + e * 3 * Hp;
  row[h] = hi;
  row[Hp + h] = mid;
  row[2 * Hp + h] = lo;
}

// INT4 codes in the reference's [K,N] nibble layout (flat index k*N + n in
// byte index/2, low nibble for even index) -> feature-major [N, K/2] bytes
// (byte n*K/2 + k/2, low nibble for even k), `batch` matrices back to back.
__global__ void int4_kn_to_nk_kernel(const uint8_t *__restrict__ kn, int64_t batch, int64_t K,
                                     int64_t N, uint8_t *__restrict__ nk) {
  const int64_t per = N * (K / 2);
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= batch * per) return;
  const int64_t b = idx / per, r = idx - b * per;
  const int64_t n = r / (K / 2), kk = (r - n * (K / 2)) * 2;
  const uint8_t *src = kn + b * ((K * N + 1) / 2);
  auto code = [&](int64_t k) -> uint32_t {
    const int64_t f = k * N + n;
    return (src[f >> 1] >> ((f & 1) * 4)) & 0xFu;
  };
  nk[idx] = (uint8_t)(code(kk) | (code(kk + 1) << 4));
}

// f32 [K,N] -> bf16 [N,K] (32x32 tiles through shared memory).
__global__ void pack_kn_kernel(const float *__restrict__ src, int64_t K, int64_t N,
                               __nv_bfloat16 *__restrict__ dst) {
  __shared__ float tile[32][33];
  int64_t k0 = (int64_t)blockIdx.y * 32, n0 = (int64_t)blockIdx.x * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    int64_t k = k0 + r, n = n0 + threadIdx.x;
    tile[r][threadIdx.x] = (k < K && n < N) ? src[k * N + n] : 0.0f;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    int64_t n = n0 + r, k = k0 + threadIdx.x;
    if (n < N && k < K) dst[n * K + k] = __float2bfloat16_rn(tile[threadIdx.x][r]);
  }
}

static unsigned grid_for(uint64_t n) {
  uint64_t b = (n + 255) / 256;
  uint64_t cap = (uint64_t)num_sms() * 16;
  return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

// Runs a "first offending index" scan; *first = UINT64_MAX when none.
template <typename Launch>
static nk_status scan_first(cudaStream_t stream, Launch launch, uint64_t *first) {
  void *buf = nullptr;
  nk_status st = scratch(sizeof(unsigned long long), &buf, stream);
  if (st != NK_OK) return st;
  unsigned long long *d = reinterpret_cast<unsigned long long *>(buf);
  NK_CUDA_TRY(cudaMemsetAsync(d, 0xFF, sizeof(*d), stream));
  launch(d);
  st = check_launch("scan kernel");
  if (st != NK_OK) return st;
  unsigned long long h = 0;
  NK_CUDA_TRY(cudaMemcpyAsync(&h, d, sizeof(h), cudaMemcpyDeviceToHost, stream));
  NK_CUDA_TRY(cudaStreamSynchronize(stream));
  *first = h;
  return NK_OK;
}

}  // namespace nk

using namespace nk;

extern "C" {

nk_status nk_validate_int4_params(float scale, uint32_t zero_point) {
  if (!isfinite(scale) || scale <= 0.0f || zero_point > 0x0F) {
    nk_status s = fail(NK_INVALID_PARAMS, "int4 params need a finite scale > 0 and zero_point <= 15");
    tls_error().value = scale;
    tls_error().byte_value = zero_point;
    return s;
  }
  return ok();
}

nk_status nk_pack_int4(const uint8_t *values, size_t count, uint8_t *packed, size_t packed_len,
                       void *stream) {
  uint64_t expect = count / 2 + (count & 1);
  if (packed_len != expect) return fail_length("packed", expect, packed_len);
  if (count == 0) return ok();
  cudaStream_t s = as_stream(stream);
  uint64_t first = 0;
  nk_status st = scan_first(
      s,
      [&](unsigned long long *d) {
        first_above15_kernel<<<grid_for(count), 256, 0, s>>>(values, count, d);
      },
      &first);
  if (st != NK_OK) return st;
  if (first != ~0ull) {
    uint8_t v = 0;
    NK_CUDA_TRY(cudaMemcpy(&v, values + first, 1, cudaMemcpyDeviceToHost));
    st = fail(NK_INT4_OUT_OF_RANGE, "int4 value out of range");
    tls_error().byte_value = v;
    tls_error().index = first;
    return st;
  }
  pack_int4_kernel<<<grid_for(packed_len), 256, 0, s>>>(values, count, packed, packed_len);
  return check_launch("pack_int4_kernel");
}

nk_status nk_unpack_int4(const uint8_t *packed, size_t packed_len, size_t count, uint8_t *out,
                         size_t out_len, void *stream) {
  uint64_t expect = count / 2 + (count & 1);
  if (packed_len != expect) return fail_length("packed", expect, packed_len);
  if (out_len != count) return fail_length("output", count, out_len);
  if (count == 0) return ok();
  unpack_int4_kernel<<<grid_for(count), 256, 0, as_stream(stream)>>>(packed, count, out);
  return check_launch("unpack_int4_kernel");
}

nk_status nk_quantize_int4(const float *values, size_t count, float scale, uint32_t zero_point,
                           uint8_t *packed, size_t packed_len, void *stream) {
  nk_status st = nk_validate_int4_params(scale, zero_point);
  if (st != NK_OK) return st;
  cudaStream_t s = as_stream(stream);
  if (count > 0) {
    uint64_t first = 0;
    st = scan_first(
        s,
        [&](unsigned long long *d) {
          first_nonfinite_kernel<<<grid_for(count), 256, 0, s>>>(values, count, d);
        },
        &first);
    if (st != NK_OK) return st;
    if (first != ~0ull) {
      float v = 0.0f;
      NK_CUDA_TRY(cudaMemcpy(&v, values + first, sizeof(float), cudaMemcpyDeviceToHost));
      st = fail(NK_NON_FINITE_INPUT, "non-finite input");
      tls_error().index = first;
      tls_error().value = v;
      return st;
    }
  }
  uint64_t expect = count / 2 + (count & 1);
  if (packed_len != expect) return fail_length("packed", expect, packed_len);
  if (count == 0) return ok();
  quantize_int4_kernel<<<grid_for(packed_len), 256, 0, s>>>(values, count, scale,
                                                           (float)zero_point, packed, packed_len);
  return check_launch("quantize_int4_kernel");
}

nk_status nk_dequantize_int4(const uint8_t *packed, size_t packed_len, size_t count, float scale,
                             uint32_t zero_point, float *out, size_t out_len, void *stream) {
  nk_status st = nk_validate_int4_params(scale, zero_point);
  if (st != NK_OK) return st;
  if (out_len != count) return fail_length("output", count, out_len);
  uint64_t expect = count / 2 + (count & 1);
  if (packed_len != expect) return fail_length("packed", expect, packed_len);
  if (count == 0) return ok();
  dequantize_int4_kernel<<<grid_for(count), 256, 0, as_stream(stream)>>>(packed, count, scale,
                                                                         (float)zero_point, out);
  return check_launch("dequantize_int4_kernel");
}

nk_status nk_quantize_int8_row(const float *w, int64_t n, int64_t k, int8_t *wq, float *scales,
                               void *stream) {
  if (n <= 0 || k <= 0) return fail(NK_INVALID_SHAPE, "n and k must be positive");
  if (n > 0x7fffffff) return fail(NK_UNSUPPORTED, "too many rows");
  cudaStream_t s = as_stream(stream);
  uint64_t count = (uint64_t)n * (uint64_t)k, first = 0;
  nk_status st = scan_first(
      s,
      [&](unsigned long long *d) {
        first_nonfinite_kernel<<<grid_for(count), 256, 0, s>>>(w, count, d);
      },
      &first);
  if (st != NK_OK) return st;
  if (first != ~0ull) {
    float v = 0.0f;
    NK_CUDA_TRY(cudaMemcpy(&v, w + first, sizeof(float), cudaMemcpyDeviceToHost));
    st = fail(NK_NON_FINITE_INPUT, "non-finite weight");
    tls_error().index = first;
    tls_error().value = v;
    return st;
  }
  quantize_int8_row_kernel<<<(unsigned)n, 256, 0, s>>>(w, k, wq, scales);
  return check_launch("quantize_int8_row_kernel");
}

nk_status nk_router_split(const float *router_w, int64_t experts, int64_t hidden,
                          uint16_t *router_w3, void *stream) {
  if (experts <= 0 || hidden <= 0) return fail(NK_INVALID_SHAPE, "experts and hidden > 0");
  int64_t hp = ceil_div(hidden, 64) * 64, total = experts * hp;
  router_split_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, as_stream(stream)>>>(
      router_w, experts, hidden, hp, reinterpret_cast<__nv_bfloat16 *>(router_w3));
  return check_launch("router_split_kernel");
}

nk_status nk_int4_kn_to_nk(const uint8_t *packed_kn, int64_t batch, int64_t k, int64_t n,
                           uint8_t *packed_nk, void *stream) {
  if (batch <= 0 || k <= 0 || n <= 0) return fail(NK_INVALID_SHAPE, "batch, k and n must be positive");
  if (k % 2) return fail(NK_UNSUPPORTED, "k must be even");
  const int64_t total = batch * n * (k / 2);
  int4_kn_to_nk_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, as_stream(stream)>>>(
      packed_kn, batch, k, n, packed_nk);
  return check_launch("int4_kn_to_nk_kernel");
}

nk_status nk_linear_pack_kn(const float *w_kn, int64_t k, int64_t n, uint16_t *w_nk,
                            void *stream) {
  if (k <= 0 || n <= 0) return fail(NK_INVALID_SHAPE, "k and n must be positive");
  dim3 grid((unsigned)ceil_div(n, 32), (unsigned)ceil_div(k, 32));
  pack_kn_kernel<<<grid, dim3(32, 8), 0, as_stream(stream)>>>(
      w_kn, k, n, reinterpret_cast<__nv_bfloat16 *>(w_nk));
  return check_launch("pack_kn_kernel");
}

}  // extern "C"
