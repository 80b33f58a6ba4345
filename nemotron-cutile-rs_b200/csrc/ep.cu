// ep.cu — expert-parallel row exchange over NVLink peer memory.
//
// G ranks; rank g owns experts [g*El, (g+1)*El), El = E/G.  Every rank routes
// its own tokens (nk_moe_dispatch) and all-gathers its per-expert row counts,
// giving every rank the matrix C[s][e] (rows of source rank s routed to
// expert e).  From C alone each rank derives, without any host round trip:
//   * where each of its routed rows lands in the owner's receive buffer, laid
//     out [source rank][local expert][row] (ep_plan_kernel: send_base),
//   * the segments of its own receive buffer (seg_rows) for nk_moe_experts,
//   * where each received row goes back: the source rank's expert-ordered
//     slot position (yoff), which is exactly where nk_moe_combine reads it.
// ep_dispatch_kernel gathers token rows from x and stores them directly into
// the owners' receive buffers (peer pointers, plain 16-byte stores over
// NVLink); ep_return_kernel stores expert outputs directly into the source
// ranks' result buffers.  Buffers are shared with cudaIpc* handles.
#include "nk_common.cuh"

namespace nk {

// One block.  C: [G][E] row counts (all ranks).  Outputs (this rank = me):
//   send_base[e]  first row of my block for expert e in owner(e)'s receive buffer
//   seg_rows[s*El + j]  rows from source s for my local expert j
//   rstart[s*El + j]    first row of that segment in my receive buffer
//   yoff[s*El + j]      its first row in source s's expert-ordered result buffer
//   total[0]            rows I receive
__global__ void ep_plan_kernel(const int32_t *__restrict__ C, int G, int E, int me,
                               int32_t *__restrict__ send_base, int32_t *__restrict__ seg_rows,
                               int32_t *__restrict__ rstart, int32_t *__restrict__ yoff,
                               int32_t *__restrict__ total) {
  const int El = E / G;
  // send_base: for each expert e (owner g), rows of all sources s < me for
  // g's experts, plus my rows for g's experts before e.
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int g = e / El;
    int base = 0;
    for (int s = 0; s < me; ++s)
      for (int j = 0; j < El; ++j) base += C[s * E + g * El + j];
    for (int j = g * El; j < e; ++j) base += C[me * E + j];
    send_base[e] = base;
  }
  // receive-side tables for my experts, in [source][local expert] order
  if (threadIdx.x == 0) {
    int run = 0;
    for (int s = 0; s < G; ++s) {
      int prefix = 0;  // exclusive prefix of C[s][:] up to my first expert
      for (int e = 0; e < me * El; ++e) prefix += C[s * E + e];
      for (int j = 0; j < El; ++j) {
        const int c = C[s * E + me * El + j];
        seg_rows[s * El + j] = c;
        rstart[s * El + j] = run;
        yoff[s * El + j] = prefix;
        run += c;
        prefix += c;
      }
    }
    total[0] = run;
  }
}

// One warp per route slot: row x[t] (t = slot / top_k) goes to expert e's
// owner at receive row send_base[e] + (slot_pos - offsets[e]).
__global__ void ep_dispatch_kernel(const uint4 *__restrict__ x, int64_t slots, int top_k,
                                   int64_t row_vecs, const int32_t *__restrict__ idx,
                                   const int32_t *__restrict__ slot_pos,
                                   const int32_t *__restrict__ offsets,
                                   const int32_t *__restrict__ send_base, int El,
                                   const uint64_t *__restrict__ peer_recv) {
  const int64_t sl = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (sl >= slots) return;
  const int e = idx[sl];
  const int64_t row = (int64_t)send_base[e] + (slot_pos[sl] - offsets[e]);
  uint4 *dst = reinterpret_cast<uint4 *>(peer_recv[e / El]) + row * row_vecs;
  const uint4 *src = x + (sl / top_k) * row_vecs;
  for (int64_t v = threadIdx.x & 31; v < row_vecs; v += 32) dst[v] = src[v];
  __threadfence_system();  // the peer reads these rows after the next collective
}

// One block per received segment (source s, local expert j): rows go back to
// source s's result buffer starting at yoff.
__global__ void ep_return_kernel(const uint4 *__restrict__ y, int64_t row_vecs,
                                 const int32_t *__restrict__ seg_rows,
                                 const int32_t *__restrict__ rstart,
                                 const int32_t *__restrict__ yoff, int El,
                                 const uint64_t *__restrict__ peer_out) {
  const int b = blockIdx.x;
  const int s = b / El;
  const int n = seg_rows[b];
  uint4 *dst = reinterpret_cast<uint4 *>(peer_out[s]) + (int64_t)yoff[b] * row_vecs;
  const uint4 *src = y + (int64_t)rstart[b] * row_vecs;
  const int64_t total = (int64_t)n * row_vecs;
  for (int64_t v = threadIdx.x; v < total; v += blockDim.x) dst[v] = src[v];
  __threadfence_system();
}

}  // namespace nk

using namespace nk;

extern "C" {

nk_status nk_ipc_alloc(size_t bytes, void **ptr, uint8_t *handle64) {
  if (!ptr || !handle64 || bytes == 0) return fail(NK_INVALID_PARAMS, "ptr, handle, bytes > 0");
  NK_CUDA_TRY(cudaMalloc(ptr, bytes));
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return fail_cuda(e, "cudaIpcGetMemHandle");
  }
  memcpy(handle64, &h, sizeof(h));
  return ok();
}

nk_status nk_ipc_open(const uint8_t *handle64, void **ptr) {
  if (!ptr || !handle64) return fail(NK_INVALID_PARAMS, "handle and ptr");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  NK_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return ok();
}

nk_status nk_ipc_close(void *ptr) {
  NK_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return ok();
}

nk_status nk_ipc_free(void *ptr) {
  NK_CUDA_TRY(cudaFree(ptr));
  return ok();
}

nk_status nk_ep_plan(const int32_t *counts_all, int32_t ranks, int32_t experts, int32_t rank,
                     int32_t *send_base, int32_t *seg_rows, int32_t *seg_start,
                     int32_t *return_offset, int32_t *received_rows, void *stream) {
  if (ranks <= 0 || experts <= 0 || experts % ranks || rank < 0 || rank >= ranks)
    return fail(NK_INVALID_SHAPE, "experts must split evenly over ranks; 0 <= rank < ranks");
  ep_plan_kernel<<<1, 256, 0, as_stream(stream)>>>(counts_all, ranks, experts, rank, send_base,
                                                   seg_rows, seg_start, return_offset,
                                                   received_rows);
  return check_launch("ep_plan_kernel");
}

nk_status nk_ep_dispatch(const uint16_t *x, int64_t tokens, int64_t hidden, int32_t top_k,
                         const int32_t *indices, const int32_t *slot_pos, const int32_t *offsets,
                         const int32_t *send_base, int32_t experts_per_rank,
                         const uint64_t *peer_recv, void *stream) {
  if (tokens < 0 || hidden <= 0 || hidden % 8 || top_k <= 0 || experts_per_rank <= 0)
    return fail(NK_INVALID_SHAPE, "tokens >= 0, hidden % 8 == 0, top_k > 0");
  const int64_t slots = tokens * top_k;
  if (slots == 0) return ok();
  const int warps = 8;
  ep_dispatch_kernel<<<(unsigned)ceil_div(slots, warps), warps * 32, 0, as_stream(stream)>>>(
      reinterpret_cast<const uint4 *>(x), slots, top_k, hidden / 8, indices, slot_pos, offsets,
      send_base, experts_per_rank, peer_recv);
  return check_launch("ep_dispatch_kernel");
}

nk_status nk_ep_return(const uint16_t *expert_rows, int64_t hidden, int32_t ranks,
                       int32_t experts_per_rank, const int32_t *seg_rows,
                       const int32_t *seg_start, const int32_t *return_offset,
                       const uint64_t *peer_out, void *stream) {
  if (hidden <= 0 || hidden % 8 || ranks <= 0 || experts_per_rank <= 0)
    return fail(NK_INVALID_SHAPE, "hidden % 8 == 0, ranks > 0, experts_per_rank > 0");
  ep_return_kernel<<<(unsigned)(ranks * experts_per_rank), 256, 0, as_stream(stream)>>>(
      reinterpret_cast<const uint4 *>(expert_rows), hidden / 8, seg_rows, seg_start,
      return_offset, experts_per_rank, peer_out);
  return check_launch("ep_return_kernel");
}

}  // extern "C"
