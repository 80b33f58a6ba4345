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

// One block.  C: [G][E] row counts (all ranks).  The local experts may be
// split into `phases` equal groups received (and computed) one after the
// other; phase h's rows live in their own region of the receive buffer,
// starting at row h * cap, ordered [source rank][local expert of the phase].
// Segment index of (source s, local expert j) with Elh = El / phases:
// (h * G + s) * Elh + (j % Elh), h = j / Elh.  Outputs (this rank = me):
//   send_base[e]  first receive row (absolute) of my block for expert e at owner(e)
//   seg_rows[seg], rstart[seg] (absolute row), yoff[seg] (row of source s's
//   expert-ordered result buffer), total[0] rows received over all phases.
__global__ void ep_plan_kernel(const int32_t *__restrict__ C, int G, int E, int me, int phases,
                               int64_t cap, int32_t *__restrict__ send_base,
                               int32_t *__restrict__ seg_rows, int32_t *__restrict__ rstart,
                               int32_t *__restrict__ yoff, int32_t *__restrict__ total) {
  const int El = E / G, Elh = El / phases;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int g = e / El, j = e % El, h = j / Elh, jj = j % Elh;
    const int first = g * El + h * Elh;  // owner's first expert of the phase
    int64_t base = (int64_t)h * cap;
    for (int s = 0; s < me; ++s)
      for (int q = 0; q < Elh; ++q) base += C[s * E + first + q];
    for (int q = 0; q < jj; ++q) base += C[me * E + first + q];
    send_base[e] = (int32_t)base;
  }
  if (threadIdx.x == 0) {
    int all = 0;
    for (int h = 0; h < phases; ++h) {
      int64_t run = (int64_t)h * cap;
      for (int s = 0; s < G; ++s) {
        int prefix = 0;  // source s's rows for experts before this phase's first of mine
        for (int e = 0; e < me * El + h * Elh; ++e) prefix += C[s * E + e];
        for (int jj = 0; jj < Elh; ++jj) {
          const int c = C[s * E + me * El + h * Elh + jj];
          const int seg = (h * G + s) * Elh + jj;
          seg_rows[seg] = c;
          rstart[seg] = (int32_t)run;
          yoff[seg] = prefix;
          run += c;
          prefix += c;
          all += c;
        }
      }
    }
    total[0] = all;
  }
}

// One warp per route slot: row x[t] (t = slot / top_k) goes to expert e's
// owner at receive row send_base[e] + (slot_pos - offsets[e]).
// With phases > 1 only the slots routed to local experts of `phase` move.
__global__ void ep_dispatch_kernel(const uint4 *__restrict__ x, int64_t slots, int top_k,
                                   int64_t row_vecs, const int32_t *__restrict__ idx,
                                   const int32_t *__restrict__ slot_pos,
                                   const int32_t *__restrict__ offsets,
                                   const int32_t *__restrict__ send_base, int El, int phases,
                                   int phase, const uint64_t *__restrict__ peer_recv) {
  const int64_t sl = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (sl >= slots) return;
  const int e = idx[sl];
  if (phases > 1 && (e % El) / (El / phases) != phase) return;
  const int64_t row = (int64_t)send_base[e] + (slot_pos[sl] - offsets[e]);
  uint4 *dst = reinterpret_cast<uint4 *>(peer_recv[e / El]) + row * row_vecs;
  const uint4 *src = x + (sl / top_k) * row_vecs;
  for (int64_t v = threadIdx.x & 31; v < row_vecs; v += 32) dst[v] = src[v];
  __threadfence_system();  // the peer reads these rows after the next collective
}

// One block per received segment (source s, local expert j): rows go back to
// source s's result buffer starting at yoff.
// Segments seg0 .. seg0 + gridDim.x - 1 (phase-major order, Elh local
// experts per source within a phase).
__global__ void ep_return_kernel(const uint4 *__restrict__ y, int64_t row_vecs,
                                 const int32_t *__restrict__ seg_rows,
                                 const int32_t *__restrict__ rstart,
                                 const int32_t *__restrict__ yoff, int G, int Elh, int seg0,
                                 const uint64_t *__restrict__ peer_out) {
  const int b = seg0 + blockIdx.x;
  const int s = (b % (G * Elh)) / Elh;
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

nk_status nk_ep_plan_phased(const int32_t *counts_all, int32_t ranks, int32_t experts,
                            int32_t rank, int32_t phases, int64_t phase_capacity_rows,
                            int32_t *send_base, int32_t *seg_rows, int32_t *seg_start,
                            int32_t *return_offset, int32_t *received_rows, void *stream) {
  if (ranks <= 0 || experts <= 0 || experts % ranks || rank < 0 || rank >= ranks)
    return fail(NK_INVALID_SHAPE, "experts must split evenly over ranks; 0 <= rank < ranks");
  if (phases <= 0 || (experts / ranks) % phases)
    return fail(NK_INVALID_SHAPE, "local experts must split evenly over the phases");
  if (phases > 1 && (phase_capacity_rows <= 0 || phases * phase_capacity_rows >= (1ll << 31)))
    return fail(NK_INVALID_PARAMS, "0 < phases * phase_capacity_rows < 2^31");
  ep_plan_kernel<<<1, 256, 0, as_stream(stream)>>>(counts_all, ranks, experts, rank, phases,
                                                   phases > 1 ? phase_capacity_rows : 0,
                                                   send_base, seg_rows, seg_start,
                                                   return_offset, received_rows);
  return check_launch("ep_plan_kernel");
}

nk_status nk_ep_plan(const int32_t *counts_all, int32_t ranks, int32_t experts, int32_t rank,
                     int32_t *send_base, int32_t *seg_rows, int32_t *seg_start,
                     int32_t *return_offset, int32_t *received_rows, void *stream) {
  return nk_ep_plan_phased(counts_all, ranks, experts, rank, 1, 0, send_base, seg_rows,
                           seg_start, return_offset, received_rows, stream);
}

nk_status nk_ep_dispatch_phase(const uint16_t *x, int64_t tokens, int64_t hidden, int32_t top_k,
                               const int32_t *indices, const int32_t *slot_pos,
                               const int32_t *offsets, const int32_t *send_base,
                               int32_t experts_per_rank, int32_t phases, int32_t phase,
                               const uint64_t *peer_recv, void *stream) {
  if (tokens < 0 || hidden <= 0 || hidden % 8 || top_k <= 0 || experts_per_rank <= 0)
    return fail(NK_INVALID_SHAPE, "tokens >= 0, hidden % 8 == 0, top_k > 0");
  if (phases <= 0 || experts_per_rank % phases || phase < 0 || phase >= phases)
    return fail(NK_INVALID_SHAPE, "0 <= phase < phases, phases dividing experts_per_rank");
  const int64_t slots = tokens * top_k;
  if (slots == 0) return ok();
  const int warps = 8;
  ep_dispatch_kernel<<<(unsigned)ceil_div(slots, warps), warps * 32, 0, as_stream(stream)>>>(
      reinterpret_cast<const uint4 *>(x), slots, top_k, hidden / 8, indices, slot_pos, offsets,
      send_base, experts_per_rank, phases, phase, peer_recv);
  return check_launch("ep_dispatch_kernel");
}

nk_status nk_ep_dispatch(const uint16_t *x, int64_t tokens, int64_t hidden, int32_t top_k,
                         const int32_t *indices, const int32_t *slot_pos, const int32_t *offsets,
                         const int32_t *send_base, int32_t experts_per_rank,
                         const uint64_t *peer_recv, void *stream) {
  return nk_ep_dispatch_phase(x, tokens, hidden, top_k, indices, slot_pos, offsets, send_base,
                              experts_per_rank, 1, 0, peer_recv, stream);
}

nk_status nk_ep_return_segments(const uint16_t *expert_rows, int64_t hidden, int32_t ranks,
                                int32_t experts_per_phase, int32_t first_segment,
                                int32_t n_segments, const int32_t *seg_rows,
                                const int32_t *seg_start, const int32_t *return_offset,
                                const uint64_t *peer_out, void *stream) {
  if (hidden <= 0 || hidden % 8 || ranks <= 0 || experts_per_phase <= 0 || first_segment < 0 ||
      n_segments < 0)
    return fail(NK_INVALID_SHAPE, "hidden % 8 == 0, ranks > 0, experts_per_phase > 0");
  if (n_segments == 0) return ok();
  ep_return_kernel<<<(unsigned)n_segments, 256, 0, as_stream(stream)>>>(
      reinterpret_cast<const uint4 *>(expert_rows), hidden / 8, seg_rows, seg_start,
      return_offset, ranks, experts_per_phase, first_segment, peer_out);
  return check_launch("ep_return_kernel");
}

nk_status nk_ep_return(const uint16_t *expert_rows, int64_t hidden, int32_t ranks,
                       int32_t experts_per_rank, const int32_t *seg_rows,
                       const int32_t *seg_start, const int32_t *return_offset,
                       const uint64_t *peer_out, void *stream) {
  return nk_ep_return_segments(expert_rows, hidden, ranks, experts_per_rank, 0,
                               ranks * experts_per_rank, seg_rows, seg_start, return_offset,
                               peer_out, stream);
}

}  // extern "C"
