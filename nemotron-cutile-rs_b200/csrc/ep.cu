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
#include "ep.h"
#include "nk_ptx.cuh"

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
                               int32_t *__restrict__ yoff, int32_t *__restrict__ total,
                               int32_t *__restrict__ pull_tab = nullptr,
                               int32_t *__restrict__ arrived = nullptr) {
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
    if (pull_tab && phases == 1) {
      // segment (s, j): rows contiguous in source s's send buffer (expert
      // order, from yoff) and in this receive buffer (from rstart); clipped
      // to the receive capacity (the excess is reported by ep_capacity_kernel)
      for (int g = 0; g < G * El; ++g) {
        int rows = seg_rows[g];
        const int64_t room = cap - (int64_t)rstart[g];
        if ((int64_t)rows > room) rows = room > 0 ? (int)room : 0;
        pull_tab[g * 3 + 0] = yoff[g];
        pull_tab[g * 3 + 1] = rstart[g];
        pull_tab[g * 3 + 2] = rows;
        arrived[g] = 0;
      }
    }
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

// ------------------------------------------------------- native EP context
// Device barrier: thread p (< G) publishes `epoch` into rank p's flag word for
// this rank (a release store to the system scope after every prior store of
// this thread block), then waits until this rank's flag words from all ranks
// reach `epoch` (acquire loads), giving up after NK_WAIT_LIMIT_NS with
// NK_TIMEOUT.  The kernels before it on the stream have completed, so all of
// this rank's earlier peer stores are ordered before the flag.
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ void ep_barrier_body(const uint64_t *__restrict__ peer_flags, uint32_t *my_flags,
                                int G, int me, uint32_t epoch, int *err) {
  const int p = threadIdx.x;
  __threadfence_system();  // this thread's peer stores, before the block's flag stores
  __syncthreads();
  if (p < G) st_release_sys(reinterpret_cast<uint32_t *>(peer_flags[p]) + me, epoch);
  if (p < G) {
    const uint64_t t0 = nk_globaltimer();
    // flags only grow; wrap-safe comparison
    while ((int32_t)(ld_acquire_sys(my_flags + p) - epoch) < 0) {
      if (nk_globaltimer() - t0 > NK_WAIT_LIMIT_NS) {
        atomicCAS(err, 0, NK_TIMEOUT);
        break;
      }
    }
  }
  __syncthreads();
}

__global__ void ep_barrier_kernel(const uint64_t *__restrict__ peer_flags, uint32_t *my_flags,
                                  int G, int me, uint32_t epoch, int *err) {
  ep_barrier_body(peer_flags, my_flags, G, me, epoch, err);
}

// counts [E] -> row `me` of every rank's counts matrix [G][E], then a barrier.
__global__ void ep_counts_kernel(const int32_t *__restrict__ counts, int E,
                                 const uint64_t *__restrict__ peer_counts,
                                 const uint64_t *__restrict__ peer_flags, uint32_t *my_flags,
                                 int G, int me, uint32_t epoch, int *err) {
  for (int i = threadIdx.x; i < G * E; i += blockDim.x) {
    const int p = i / E, e = i - p * E;
    reinterpret_cast<int32_t *>(peer_counts[p])[me * E + e] = counts[e];
  }
  ep_barrier_body(peer_flags, my_flags, G, me, epoch, err);
}

// Receive capacity check after the plan: more rows than the receive buffer
// holds is reported (NK_WORKSPACE_TOO_SMALL in the device error word) and the
// dispatch of this forward is suppressed by zeroing the send plan's rows.
__global__ void ep_capacity_kernel(int32_t *total, int64_t cap, int *err) {
  if (threadIdx.x == 0 && (int64_t)total[0] > cap) atomicCAS(err, 0, NK_WORKSPACE_TOO_SMALL);
}

static uint64_t *table(const nk_ep_ctx *c, int which) { return c->tables + which * c->ranks; }
const uint64_t *ep_out_table(const nk_ep_ctx *c) { return table(c, 1); }
const uint64_t *ep_send_table(const nk_ep_ctx *c) { return table(c, 4); }
uint16_t *ep_send(const nk_ep_ctx *c) {
  return reinterpret_cast<uint16_t *>(reinterpret_cast<uint8_t *>(c->block) + c->off_send);
}

uint16_t *ep_recv(const nk_ep_ctx *c) { return reinterpret_cast<uint16_t *>(c->block); }
uint16_t *ep_out(const nk_ep_ctx *c) {
  return reinterpret_cast<uint16_t *>(reinterpret_cast<uint8_t *>(c->block) + c->off_out);
}
int32_t *ep_counts_all(const nk_ep_ctx *c) {
  return reinterpret_cast<int32_t *>(reinterpret_cast<uint8_t *>(c->block) + c->off_counts);
}
static uint32_t *ep_flags(const nk_ep_ctx *c) {
  return reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(c->block) + c->off_flags);
}

nk_status ep_exchange_counts(nk_ep_ctx *c, const int32_t *counts, cudaStream_t s) {
  ++c->epoch;
  ep_counts_kernel<<<1, 256, 0, s>>>(counts, (int)c->experts, table(c, 2), table(c, 3),
                                    ep_flags(c), c->ranks, c->rank, c->epoch,
                                    device_error_ptr());
  return check_launch("ep_counts_kernel");
}

nk_status ep_barrier(nk_ep_ctx *c, cudaStream_t s) {
  ++c->epoch;
  ep_barrier_kernel<<<1, 64, 0, s>>>(table(c, 3), ep_flags(c), c->ranks, c->rank, c->epoch,
                                    device_error_ptr());
  return check_launch("ep_barrier_kernel");
}

nk_status ep_plan(nk_ep_ctx *c, cudaStream_t s, bool pull) {
  ep_plan_kernel<<<1, 256, 0, s>>>(ep_counts_all(c), c->ranks, (int)c->experts, c->rank, 1,
                                   c->capacity_rows, c->send_base, c->seg_rows, c->seg_start,
                                   c->ret_off, c->total, pull ? c->pull_tab : nullptr,
                                   c->arrived);
  nk_status st = check_launch("ep_plan_kernel");
  if (st != NK_OK) return st;
  ep_capacity_kernel<<<1, 32, 0, s>>>(c->total, c->capacity_rows, device_error_ptr());
  return check_launch("ep_capacity_kernel");
}

__global__ void ep_dispatch_capped_kernel(const uint4 *__restrict__ x, int64_t slots, int top_k,
                                          int64_t row_vecs, const int32_t *__restrict__ idx,
                                          const int32_t *__restrict__ slot_pos,
                                          const int32_t *__restrict__ offsets,
                                          const int32_t *__restrict__ send_base, int El,
                                          int64_t cap, const uint64_t *__restrict__ peer_recv) {
  const int64_t sl = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (sl < slots) {
    const int e = idx[sl];
    const int64_t row = (int64_t)send_base[e] + (slot_pos[sl] - offsets[e]);
    if (row < cap) {  // over capacity: reported by ep_capacity_kernel
      uint4 *dst = reinterpret_cast<uint4 *>(peer_recv[e / El]) + row * row_vecs;
      const uint4 *src = x + (sl / top_k) * row_vecs;
      for (int64_t v = threadIdx.x & 31; v < row_vecs; v += 32) dst[v] = src[v];
    }
  }
  // the owner reads these rows after the next device barrier (a later kernel
  // on this stream); one system fence per block once its rows are issued
  __syncthreads();
  if (threadIdx.x == 0) __threadfence_system();
}

nk_status ep_dispatch(nk_ep_ctx *c, const uint16_t *x, int64_t tokens, const int32_t *idx,
                      const int32_t *slot_pos, const int32_t *offsets, cudaStream_t s) {
  const int64_t slots = tokens * c->top_k;
  if (slots == 0) return NK_OK;
  const int warps = 8;
  ep_dispatch_capped_kernel<<<(unsigned)ceil_div(slots, warps), warps * 32, 0, s>>>(
      reinterpret_cast<const uint4 *>(x), slots, (int)c->top_k, c->hidden / 8, idx, slot_pos,
      offsets, c->send_base, (int)(c->experts / c->ranks), c->capacity_rows, table(c, 0));
  return check_launch("ep_dispatch_capped_kernel");
}

nk_status ep_return(nk_ep_ctx *c, cudaStream_t s) {
  const int El = (int)(c->experts / c->ranks);
  ep_return_kernel<<<(unsigned)(c->ranks * El), 256, 0, s>>>(
      reinterpret_cast<const uint4 *>(ep_recv(c)), c->hidden / 8, c->seg_rows, c->seg_start,
      c->ret_off, c->ranks, El, 0, table(c, 1));
  return check_launch("ep_return_kernel");
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


// ------------------------------------------------------- native EP context
struct nk_ep_blob {
  uint32_t magic, rank, ranks, pad;
  uint64_t block_bytes;
  cudaIpcMemHandle_t handle;
};

size_t nk_ep_handle_bytes(void) { return sizeof(nk_ep_blob); }

nk_status nk_ep_create(int32_t ranks, int32_t rank, int64_t experts, int64_t hidden,
                       int64_t top_k, int64_t max_tokens, int64_t capacity_rows,
                       nk_ep_ctx **out, void *handle_blob) {
  if (!out || !handle_blob) return fail(NK_INVALID_PARAMS, "out and handle_blob");
  if (ranks <= 0 || ranks > 64 || rank < 0 || rank >= ranks)
    return fail(NK_INVALID_SHAPE, "0 <= rank < ranks <= 64");
  if (experts <= 0 || experts % ranks || hidden <= 0 || hidden % 8 || top_k <= 0 ||
      top_k > experts || max_tokens <= 0)
    return fail(NK_INVALID_SHAPE, "experts % ranks == 0, hidden % 8 == 0, 0 < top_k <= experts");
  if (ranks * (experts / ranks) > 1024) return fail(NK_UNSUPPORTED, "experts <= 1024");
  const int64_t worst = (int64_t)ranks * max_tokens * top_k;
  if (capacity_rows <= 0 || capacity_rows > worst) capacity_rows = worst;
  if (capacity_rows >= (1ll << 31) || max_tokens * top_k >= (1ll << 31))
    return fail(NK_UNSUPPORTED, "receive rows must stay below 2^31");
  nk_ep_ctx *c = new nk_ep_ctx();
  c->ranks = ranks;
  c->rank = rank;
  c->experts = experts;
  c->hidden = hidden;
  c->top_k = top_k;
  c->max_tokens = max_tokens;
  c->capacity_rows = capacity_rows;
  cudaGetDevice(&c->device);
  auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
  c->off_out = al((size_t)capacity_rows * hidden * 2);
  c->off_counts = c->off_out + al((size_t)max_tokens * top_k * hidden * 2);
  c->off_flags = c->off_counts + al((size_t)ranks * experts * 4);
  c->off_send = c->off_flags + al((size_t)ranks * 4);
  c->block_bytes = c->off_send + al((size_t)max_tokens * top_k * hidden * 2);
  const int El = (int)(experts / ranks);
  auto cleanup = [&](nk_status st) {
    if (c->block) cudaFree(c->block);
    if (c->tables) cudaFree(c->tables);
    if (c->send_base) cudaFree(c->send_base);
    delete c;
    return st;
  };
  cudaError_t e = cudaMalloc(&c->block, c->block_bytes);
  if (e != cudaSuccess) return cleanup(fail_cuda(e, "cudaMalloc(ep block)"));
  e = cudaMemset(c->block, 0, c->block_bytes);  // flags start at epoch 0
  if (e == cudaSuccess) e = cudaMalloc(&c->tables, sizeof(uint64_t) * 5 * ranks);
  // plan arrays in one allocation
  const size_t nseg = (size_t)ranks * El;
  if (e == cudaSuccess)
    e = cudaMalloc(&c->send_base, sizeof(int32_t) * (experts + 9 * nseg + 1));
  if (e != cudaSuccess) return cleanup(fail_cuda(e, "cudaMalloc(ep plan)"));
  c->seg_rows = c->send_base + experts;
  c->seg_start = c->seg_rows + nseg;
  c->ret_off = c->seg_start + nseg;
  c->seg_expert = c->ret_off + nseg;
  c->total = c->seg_expert + nseg;
  c->pull_tab = c->total + 1;
  c->arrived = c->pull_tab + 3 * nseg;
  {  // segment order [source rank][local expert]
    int32_t *h = new int32_t[nseg];
    for (size_t i = 0; i < nseg; ++i) h[i] = (int32_t)(i % El);
    e = cudaMemcpy(c->seg_expert, h, sizeof(int32_t) * nseg, cudaMemcpyHostToDevice);
    delete[] h;
    if (e != cudaSuccess) return cleanup(fail_cuda(e, "cudaMemcpy(seg_expert)"));
  }
  nk_ep_blob blob{};
  blob.magic = 0x4e4b4550u;  // "NKEP"
  blob.rank = (uint32_t)rank;
  blob.ranks = (uint32_t)ranks;
  blob.block_bytes = c->block_bytes;
  e = cudaIpcGetMemHandle(&blob.handle, c->block);
  if (e != cudaSuccess) return cleanup(fail_cuda(e, "cudaIpcGetMemHandle"));
  memcpy(handle_blob, &blob, sizeof(blob));
  *out = c;
  return ok();
}

nk_status nk_ep_connect(nk_ep_ctx *c, const void *all_blobs) {
  if (!c || !all_blobs) return fail(NK_INVALID_PARAMS, "ctx and blobs");
  if (c->connected) return fail(NK_INVALID_PARAMS, "already connected");
  const nk_ep_blob *b = reinterpret_cast<const nk_ep_blob *>(all_blobs);
  uint64_t h[5 * 64];
  for (int p = 0; p < c->ranks; ++p) {
    if (b[p].magic != 0x4e4b4550u || (int)b[p].rank != p || (int)b[p].ranks != c->ranks ||
        b[p].block_bytes != c->block_bytes)
      return fail(NK_INVALID_PARAMS, "handle blobs must come from nk_ep_create of every rank "
                                     "with the same shapes, in rank order");
    uint8_t *base;
    if (p == c->rank) {
      base = reinterpret_cast<uint8_t *>(c->block);
    } else {
      void *ptr = nullptr;
      NK_CUDA_TRY(cudaIpcOpenMemHandle(&ptr, b[p].handle, cudaIpcMemLazyEnablePeerAccess));
      c->opened[p] = ptr;
      base = reinterpret_cast<uint8_t *>(ptr);
    }
    h[0 * c->ranks + p] = reinterpret_cast<uint64_t>(base);
    h[1 * c->ranks + p] = reinterpret_cast<uint64_t>(base + c->off_out);
    h[2 * c->ranks + p] = reinterpret_cast<uint64_t>(base + c->off_counts);
    h[3 * c->ranks + p] = reinterpret_cast<uint64_t>(base + c->off_flags);
    h[4 * c->ranks + p] = reinterpret_cast<uint64_t>(base + c->off_send);
  }
  NK_CUDA_TRY(cudaMemcpy(c->tables, h, sizeof(uint64_t) * 5 * c->ranks, cudaMemcpyHostToDevice));
  c->connected = true;
  return ok();
}

nk_status nk_ep_destroy(nk_ep_ctx *c) {
  if (!c) return ok();
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  for (int p = 0; p < c->ranks; ++p)
    if (c->opened[p]) cudaIpcCloseMemHandle(c->opened[p]);
  cudaFree(c->block);
  cudaFree(c->tables);
  cudaFree(c->send_base);
  delete c;
  return ok();
}

nk_status nk_ep_barrier(nk_ep_ctx *c, void *stream) {
  if (!c || !c->connected) return fail(NK_INVALID_PARAMS, "connected context required");
  nk_status st = ep_barrier(c, as_stream(stream));
  return st == NK_OK ? ok() : st;
}

nk_status nk_ep_received_rows(const nk_ep_ctx *c, int32_t *rows_device) {
  if (!c || !rows_device) return fail(NK_INVALID_PARAMS, "ctx and output");
  NK_CUDA_TRY(cudaMemcpyAsync(rows_device, c->total, sizeof(int32_t), cudaMemcpyDeviceToDevice));
  return ok();
}

}  // extern "C"
