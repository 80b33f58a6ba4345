// model.cu — the steps either side of every projection in the decoder:
// embedding gather (nemotron-kernels/src/embedding.rs), the block residual
// fused with the next block's RMSNorm (nemotron-nn/src/block.rs:112-154),
// and the greedy pick over the lm_head logits (nemotron-model/src/model.rs:
// 325-337).  All HBM-bound; one pass over the data each.
#include "nk_common.cuh"

namespace nk {

// --------------------------------------------------------------- embedding
// Row t of out = table[ids[t]] (f32 or bf16 table and output; 16-byte chunks
// when both rows allow it).  Out-of-range ids are flagged, not read.
template <typename TIn, typename TOut>
__global__ void embed_kernel(const TIn *__restrict__ table, const int32_t *__restrict__ ids,
                             int64_t n, int64_t vocab, int64_t hidden, TOut *__restrict__ out,
                             unsigned long long *bad) {
  const int64_t t = blockIdx.x;
  if (t >= n) return;
  const int32_t id = ids[t];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0 && bad) atomicMin(bad, (unsigned long long)t);
    return;
  }
  const TIn *src = table + (int64_t)id * hidden;
  TOut *dst = out + t * hidden;
  for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) {
    const float v = (float)src[i];
    dst[i] = (TOut)v;
  }
}

// ------------------------------------------------- residual + next RMSNorm
// h = residual + delta (f32, the block output, block.rs:145-151), written to
// h_out (may alias residual); normed = rms_norm(h) * weight (rms_norm.rs:
// 117-123 as the next block's input norm), written bf16 or f32.  One block of
// 256 threads per row; delta may be NULL (the first block: norm only).
template <bool BF16_OUT>
__global__ void __launch_bounds__(256) add_norm_kernel(
    const float *residual, const float *__restrict__ delta, int64_t W,
    const float *__restrict__ weight, float eps, float *h_out, void *__restrict__ normed) {
  const int64_t row = blockIdx.x;
  const float *r = residual + row * W;
  const float *d = delta ? delta + row * W : nullptr;
  float *h = h_out + row * W;
  double sum = 0.0;
  for (int64_t i = threadIdx.x; i < W; i += blockDim.x) {
    const float v = d ? __fadd_rn(r[i], d[i]) : r[i];
    h[i] = v;
    sum += (double)v * (double)v;
  }
  __shared__ double part[8];
  __shared__ float scale_s;
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    double tot = 0.0;
    for (int i = 0; i < 8; ++i) tot += part[i];
    scale_s = 1.0f / sqrtf((float)(tot / (double)W) + eps);
  }
  __syncthreads();
  const float sc = scale_s;
  for (int64_t i = threadIdx.x; i < W; i += blockDim.x) {
    const float v = __fmul_rn(__fmul_rn(h[i], sc), weight[i]);
    if (BF16_OUT)
      reinterpret_cast<__nv_bfloat16 *>(normed)[row * W + i] = __float2bfloat16_rn(v);
    else
      reinterpret_cast<float *>(normed)[row * W + i] = v;
  }
}

// ------------------------------------------------------------------ argmax
// Total order of f32 as an unsigned key (f32::total_cmp): negative values
// reversed below positive ones, NaN at either end by its sign.
__device__ __forceinline__ uint32_t total_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// One block per row: the index of the maximum under total_cmp, the last one
// among equals (Iterator::max_by keeps the later of equal elements).
template <typename T>
__global__ void __launch_bounds__(256) argmax_kernel(const T *__restrict__ x, int64_t ld,
                                                     int64_t n, int32_t *__restrict__ out) {
  const T *r = x + (int64_t)blockIdx.x * ld;
  uint64_t best = 0;  // (key << 32) | index: larger key, then larger index
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const uint64_t k = ((uint64_t)total_key((float)r[i]) << 32) | (uint64_t)i;
    best = k > best ? k : best;
  }
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t v = __shfl_xor_sync(0xffffffffu, best, o);
    best = v > best ? v : best;
  }
  __shared__ uint64_t part[8];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < 8; ++i) best = part[i] > best ? part[i] : best;
    best = part[0] > best ? part[0] : best;
    out[blockIdx.x] = (int32_t)(best & 0xFFFFFFFFu);
  }
}

}  // namespace nk

using namespace nk;

extern "C" {

nk_status nk_embedding_lookup(const void *table, int32_t table_dtype, size_t table_len,
                              const int32_t *token_ids, int64_t n_tokens, int64_t vocab_size,
                              int64_t hidden_size, void *out, int32_t out_dtype, size_t out_len,
                              int32_t check, void *stream) {
  // embedding.rs:121-191: shape, table length, output length, then the ids.
  if (vocab_size <= 0 || hidden_size <= 0 || n_tokens < 0)
    return fail(NK_INVALID_SHAPE, "embedding needs vocab_size > 0 and hidden_size > 0");
  const uint64_t tl = (uint64_t)vocab_size * hidden_size, ol = (uint64_t)n_tokens * hidden_size;
  if (table_len != tl) return fail_length("table", tl, table_len);
  if (out_len != ol) return fail_length("output", ol, out_len);
  if ((table_dtype != NK_DTYPE_F32 && table_dtype != NK_DTYPE_BF16) ||
      (out_dtype != NK_DTYPE_F32 && out_dtype != NK_DTYPE_BF16))
    return fail(NK_INVALID_PARAMS, "dtypes must be NK_DTYPE_F32 or NK_DTYPE_BF16");
  if (n_tokens == 0) return ok();
  if (n_tokens > 0x7fffffff) return fail(NK_UNSUPPORTED, "n_tokens < 2^31");
  cudaStream_t s = as_stream(stream);
  unsigned long long *bad = nullptr;
  if (check) {
    void *buf = nullptr;
    nk_status st = scratch(sizeof(unsigned long long), &buf, s);
    if (st != NK_OK) return st;
    bad = reinterpret_cast<unsigned long long *>(buf);
    NK_CUDA_TRY(cudaMemsetAsync(bad, 0xFF, sizeof(*bad), s));
  }
  const dim3 grid((unsigned)n_tokens);
  const bool tf = table_dtype == NK_DTYPE_F32, of = out_dtype == NK_DTYPE_F32;
  if (tf && of)
    embed_kernel<float, float><<<grid, 256, 0, s>>>((const float *)table, token_ids, n_tokens,
                                                    vocab_size, hidden_size, (float *)out, bad);
  else if (tf)
    embed_kernel<float, __nv_bfloat16><<<grid, 256, 0, s>>>(
        (const float *)table, token_ids, n_tokens, vocab_size, hidden_size,
        (__nv_bfloat16 *)out, bad);
  else if (of)
    embed_kernel<__nv_bfloat16, float><<<grid, 256, 0, s>>>(
        (const __nv_bfloat16 *)table, token_ids, n_tokens, vocab_size, hidden_size,
        (float *)out, bad);
  else
    embed_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, 256, 0, s>>>(
        (const __nv_bfloat16 *)table, token_ids, n_tokens, vocab_size, hidden_size,
        (__nv_bfloat16 *)out, bad);
  nk_status st = check_launch("embed_kernel");
  if (st != NK_OK || !check) return st;
  unsigned long long h = 0;
  NK_CUDA_TRY(cudaMemcpyAsync(&h, bad, sizeof(h), cudaMemcpyDeviceToHost, s));
  NK_CUDA_TRY(cudaStreamSynchronize(s));
  if (h != ~0ull) {
    int32_t id = 0;
    NK_CUDA_TRY(cudaMemcpy(&id, token_ids + h, sizeof(id), cudaMemcpyDeviceToHost));
    nk_status e = fail(NK_TOKEN_OUT_OF_RANGE, "token id out of range");
    tls_error().index = h;
    tls_error().actual = (uint64_t)(int64_t)id;
    tls_error().expected = (uint64_t)vocab_size;
    return e;
  }
  return ok();
}

nk_status nk_add_rms_norm_rows(const float *residual, const float *delta, int64_t rows,
                               int64_t width, const float *weight, size_t weight_len,
                               float epsilon, float *h_out, void *normed, int32_t normed_dtype,
                               void *stream) {
  if (rows < 0 || width <= 0) return fail(NK_INVALID_SHAPE, "rows >= 0, width > 0");
  if (weight_len != (uint64_t)width) return fail_length("weight", width, weight_len);
  if (epsilon < 0.0f) {
    nk_status e = fail(NK_NEGATIVE_EPSILON, "epsilon must be >= 0");
    tls_error().value = epsilon;
    return e;
  }
  if (normed_dtype != NK_DTYPE_F32 && normed_dtype != NK_DTYPE_BF16)
    return fail(NK_INVALID_PARAMS, "normed_dtype must be NK_DTYPE_F32 or NK_DTYPE_BF16");
  if (rows == 0) return ok();
  if (rows > 0x7fffffff) return fail(NK_UNSUPPORTED, "rows < 2^31");
  cudaStream_t s = as_stream(stream);
  if (normed_dtype == NK_DTYPE_BF16)
    add_norm_kernel<true><<<(unsigned)rows, 256, 0, s>>>(residual, delta, width, weight, epsilon,
                                                         h_out, normed);
  else
    add_norm_kernel<false><<<(unsigned)rows, 256, 0, s>>>(residual, delta, width, weight,
                                                          epsilon, h_out, normed);
  return check_launch("add_norm_kernel");
}

nk_status nk_argmax_rows(const void *x, int32_t x_dtype, int64_t rows, int64_t n, int64_t ld,
                         int32_t *out, void *stream) {
  if (rows < 0 || n <= 0 || ld < n) return fail(NK_INVALID_SHAPE, "rows >= 0, 0 < n <= ld");
  if (n > 0xFFFFFFFFll) return fail(NK_UNSUPPORTED, "n < 2^32");
  if (rows == 0) return ok();
  if (rows > 0x7fffffff) return fail(NK_UNSUPPORTED, "rows < 2^31");
  cudaStream_t s = as_stream(stream);
  if (x_dtype == NK_DTYPE_F32)
    argmax_kernel<float><<<(unsigned)rows, 256, 0, s>>>((const float *)x, ld, n, out);
  else if (x_dtype == NK_DTYPE_BF16)
    argmax_kernel<__nv_bfloat16><<<(unsigned)rows, 256, 0, s>>>((const __nv_bfloat16 *)x, ld,
                                                                n, out);
  else
    return fail(NK_INVALID_PARAMS, "x_dtype must be NK_DTYPE_F32 or NK_DTYPE_BF16");
  return check_launch("argmax_kernel");
}

}  // extern "C"
