// route.cu — MoE top-k routing (moe_routing.rs:118-216) and the expert
// histogram / permutation that turns routes into grouped-GEMM row blocks.
#include <math.h>

#include "nk_common.cuh"
#include "route.h"

namespace nk {

// f32::total_cmp as a signed integer key.
__device__ __forceinline__ int32_t total_key(float f) {
  int32_t b = __float_as_int(f);
  return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}

// exp evaluated in double and rounded once to f32: the correctly rounded
// value in all but vanishingly rare double-rounding cases, which is what the
// reference's libm expf returns for practically every input.
__device__ __forceinline__ float exp_f32(float x) { return (float)exp((double)x); }

// activations.rs:73-81 with IEEE-rounded f32 add and divide.
__device__ __forceinline__ float sigmoid_ref(float x) {
  if (x >= 0.0f) {
    float z = exp_f32(-x);
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, z));
  }
  float z = exp_f32(x);
  return __fdiv_rn(z, __fadd_rn(1.0f, z));
}

constexpr int kRouteWarps = 4;
constexpr int kMaxExperts = 1024;

// One warp per token.  The token's E weights live in shared memory; top-k is
// k rounds of a warp arg-max over (total-order key desc, index asc).
__global__ void __launch_bounds__(kRouteWarps * 32)
    route_kernel(const float *__restrict__ scores, int64_t tokens, int E, int K, int mode,
                 int32_t *__restrict__ indices, float *__restrict__ weights) {
  __shared__ float wsm[kRouteWarps][kMaxExperts];
  __shared__ uint32_t taken[kRouteWarps][kMaxExperts / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kRouteWarps + warp;
  if (t >= tokens) return;
  const float *s = scores + t * E;
  float *w = wsm[warp];
  for (int e = lane; e < E / 32 + 1; e += 32)
    if (e < kMaxExperts / 32) taken[warp][e] = 0;

  if (mode == NK_ROUTE_SOFTMAX) {
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, s[e]);
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int e = lane; e < E; e += 32) w[e] = exp_f32(__fsub_rn(s[e], mx));
    __syncwarp();
    float total = 0.0f;
    if (lane == 0) {  // sequential f32 sum in index order, as Iterator::sum
      total = -0.0f;
      for (int e = 0; e < E; ++e) total = __fadd_rn(total, w[e]);
    }
    total = __shfl_sync(0xffffffffu, total, 0);
    for (int e = lane; e < E; e += 32) w[e] = __fdiv_rn(w[e], total);
  } else {
    for (int e = lane; e < E; e += 32) w[e] = sigmoid_ref(s[e]);
  }
  __syncwarp();

  float sel_w[32];
  int sel_i[32];
  for (int r = 0; r < K; ++r) {
    int32_t best_key = INT32_MIN;
    int best_idx = 0x7fffffff;
    for (int e = lane; e < E; e += 32) {
      if (taken[warp][e >> 5] & (1u << (e & 31))) continue;
      int32_t key = total_key(w[e]);
      if (key > best_key || (key == best_key && e < best_idx)) {
        best_key = key;
        best_idx = e;
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      int32_t ok = __shfl_xor_sync(0xffffffffu, best_key, o);
      int oi = __shfl_xor_sync(0xffffffffu, best_idx, o);
      if (ok > best_key || (ok == best_key && oi < best_idx)) {
        best_key = ok;
        best_idx = oi;
      }
    }
    if (lane == 0) taken[warp][best_idx >> 5] |= 1u << (best_idx & 31);
    __syncwarp();
    sel_i[r] = best_idx;
    sel_w[r] = w[best_idx];
  }
  if (lane == 0) {
    if (mode == NK_ROUTE_SOFTMAX || mode == NK_ROUTE_SIGMOID_RENORM) {
      float sel = -0.0f;
      for (int r = 0; r < K; ++r) sel = __fadd_rn(sel, sel_w[r]);
      for (int r = 0; r < K; ++r) sel_w[r] = __fdiv_rn(sel_w[r], sel);
    }
    for (int r = 0; r < K; ++r) {
      indices[t * K + r] = sel_i[r];
      weights[t * K + r] = sel_w[r];
    }
  }
}

// ------------------------------------------------------------------- plan
constexpr int kPlanChunk = 1024;  // route slots per chunk (one warp walks it in order)

__global__ void plan_count_kernel(const int32_t *__restrict__ idx, int64_t slots, int E,
                                  int32_t *__restrict__ chunk_counts) {
  __shared__ int32_t h[kMaxExperts];
  for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
  __syncthreads();
  int64_t base = (int64_t)blockIdx.x * kPlanChunk;
  for (int i = threadIdx.x; i < kPlanChunk; i += blockDim.x) {
    int64_t s = base + i;
    if (s < slots) {
      int e = idx[s];
      if (e >= 0 && e < E) atomicAdd(&h[e], 1);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) chunk_counts[(int64_t)blockIdx.x * E + e] = h[e];
}

// One block of up to 1024 threads: per-expert prefix over chunks, then an
// exclusive scan over experts.
__global__ void plan_scan_kernel(int32_t *__restrict__ chunk_counts, int nchunks, int E,
                                 int32_t *__restrict__ counts, int32_t *__restrict__ offsets) {
  __shared__ int32_t sc[kMaxExperts];
  const int e = threadIdx.x;
  int32_t total = 0;
  if (e < E) {
    for (int c0 = 0; c0 < nchunks; c0 += 8) {  // 8 loads in flight, then the running sum
      int32_t v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        v[j] = c0 + j < nchunks ? chunk_counts[(int64_t)(c0 + j) * E + e] : 0;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (c0 + j < nchunks) {
          chunk_counts[(int64_t)(c0 + j) * E + e] = total;  // the chunk's base for expert e
          total += v[j];
        }
    }
    counts[e] = total;
  }
  sc[e] = e < E ? total : 0;
  __syncthreads();
  for (int o = 1; o < blockDim.x; o <<= 1) {  // inclusive Hillis-Steele scan
    int32_t v = e >= o ? sc[e - o] : 0;
    __syncthreads();
    sc[e] += v;
    __syncthreads();
  }
  if (e < E) offsets[e] = sc[e] - total;
  if (e == E - 1) offsets[E] = sc[e];
}

__global__ void plan_place_kernel(const int32_t *__restrict__ idx, int64_t slots, int E,
                                  const int32_t *__restrict__ chunk_base,
                                  const int32_t *__restrict__ offsets, int32_t *__restrict__ perm,
                                  int32_t *__restrict__ slot_pos) {
  __shared__ int32_t run[kMaxExperts];
  const int lane = threadIdx.x;  // a single warp walks the chunk in slot order
  for (int e = lane; e < E; e += 32)
    run[e] = offsets[e] + chunk_base[(int64_t)blockIdx.x * E + e];
  __syncwarp();
  int64_t base = (int64_t)blockIdx.x * kPlanChunk;
  for (int g0 = 0; g0 < kPlanChunk; g0 += 32 * 8) {  // 8 loads per lane in flight
    int ev[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t s = base + g0 + j * 32 + lane;
      ev[j] = s < slots ? idx[s] : -1;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t s = base + g0 + j * 32 + lane;
      const bool valid = s < slots && ev[j] >= 0 && ev[j] < E;
      const int e = valid ? ev[j] : -1 - lane;  // unique negative keys for idle lanes
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      const int rank = __popc(peers & ((1u << lane) - 1));
      if (valid) {
        const int pos = run[e] + rank;
        perm[pos] = (int32_t)s;
        slot_pos[s] = pos;
      }
      __syncwarp();
      if (valid && rank == 0) run[e] += __popc(peers);
      __syncwarp();
    }
  }
}

nk_status launch_route(const float *scores, int64_t tokens, int E, int K, int mode,
                       int32_t *indices, float *weights, cudaStream_t stream) {
  if (tokens == 0) return ok();
  unsigned blocks = (unsigned)ceil_div(tokens, kRouteWarps);
  route_kernel<<<blocks, kRouteWarps * 32, 0, stream>>>(scores, tokens, E, K, mode, indices,
                                                        weights);
  return check_launch("route_kernel");
}

size_t plan_scratch_bytes(int64_t slots, int64_t E) {
  return (size_t)(ceil_div(slots, kPlanChunk) + 1) * (size_t)E * sizeof(int32_t);
}

nk_status launch_plan(const int32_t *indices, int64_t slots, int E, int32_t *counts,
                      int32_t *offsets, int32_t *perm, int32_t *slot_pos, int32_t *chunk_scratch,
                      cudaStream_t stream) {
  int nchunks = (int)ceil_div(slots, kPlanChunk);
  if (nchunks == 0) {
    NK_CUDA_TRY(cudaMemsetAsync(counts, 0, sizeof(int32_t) * E, stream));
    NK_CUDA_TRY(cudaMemsetAsync(offsets, 0, sizeof(int32_t) * (E + 1), stream));
    return ok();
  }
  plan_count_kernel<<<nchunks, 256, 0, stream>>>(indices, slots, E, chunk_scratch);
  int threads = 32;
  while (threads < E) threads <<= 1;
  plan_scan_kernel<<<1, threads, 0, stream>>>(chunk_scratch, nchunks, E, counts, offsets);
  plan_place_kernel<<<nchunks, 32, 0, stream>>>(indices, slots, E, chunk_scratch, offsets, perm,
                                                slot_pos);
  return check_launch("plan kernels");
}

}  // namespace nk

using namespace nk;

extern "C" {

nk_status nk_moe_route(const float *scores, size_t scores_len, size_t tokens, size_t experts,
                       size_t top_k, int32_t mode, int32_t *indices, size_t indices_len,
                       float *weights, size_t weights_len, void *stream) {
  if (experts == 0 || top_k == 0 || top_k > experts)
    return fail(NK_INVALID_SHAPE, "routing shape needs 0 < top_k <= experts");
  uint64_t slen, rlen;
  if (!mul_ok(tokens, experts, &slen) || !mul_ok(tokens, top_k, &rlen))
    return fail(NK_INVALID_SHAPE, "routing shape overflows");
  if (scores_len != slen) return fail_length("scores", slen, scores_len);
  if (indices_len != rlen) return fail_length("indices", rlen, indices_len);
  if (weights_len != rlen) return fail_length("weights", rlen, weights_len);
  if (experts > (size_t)kMaxExperts || top_k > 32)
    return fail(NK_UNSUPPORTED, "device router handles experts <= 1024 and top_k <= 32");
  if (mode < NK_ROUTE_SIGMOID || mode > NK_ROUTE_SIGMOID_RENORM)
    return fail(NK_UNSUPPORTED, "unknown routing mode");
  return launch_route(scores, (int64_t)tokens, (int)experts, (int)top_k, mode, indices, weights,
                      as_stream(stream));
}

nk_status nk_moe_plan(const int32_t *indices, int64_t tokens, int64_t top_k, int64_t experts,
                      int32_t *counts, int32_t *offsets, int32_t *perm, int32_t *slot_pos,
                      void *stream) {
  if (experts <= 0 || top_k <= 0 || top_k > experts || tokens < 0)
    return fail(NK_INVALID_SHAPE, "plan shape needs 0 < top_k <= experts");
  if (experts > kMaxExperts) return fail(NK_UNSUPPORTED, "experts > 1024");
  int64_t slots = tokens * top_k;
  void *buf = nullptr;
  cudaStream_t s = as_stream(stream);
  nk_status st = scratch(plan_scratch_bytes(slots, experts), &buf, s);
  if (st != NK_OK) return st;
  return launch_plan(indices, slots, (int)experts, counts, offsets, perm, slot_pos,
                     reinterpret_cast<int32_t *>(buf), s);
}

}  // extern "C"
