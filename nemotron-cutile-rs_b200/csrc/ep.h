// ep.h — the native expert-parallel context shared by ep.cu (buffers, peer
// tables, device barriers) and moe.cu (nk_moe_forward_ep).
#pragma once
#include "nk_common.cuh"

struct nk_ep_ctx {
  int ranks = 0, rank = 0, device = -1;
  int64_t experts = 0, hidden = 0, top_k = 0, max_tokens = 0, capacity_rows = 0;
  // this rank's IPC block: [recv rows][result rows][counts_all][flags][send rows]
  void *block = nullptr;
  size_t block_bytes = 0, off_out = 0, off_counts = 0, off_flags = 0, off_send = 0;
  void *opened[64] = {};      // peers' blocks (cudaIpcOpenMemHandle), null for this rank
  // device tables of the peers' buffers (uint64 addresses, rank order)
  uint64_t *tables = nullptr; // [5][ranks]: recv, out, counts, flags, send
  // plan of the current forward (device)
  int32_t *send_base = nullptr, *seg_rows = nullptr, *seg_start = nullptr, *ret_off = nullptr,
          *total = nullptr, *seg_expert = nullptr;
  // in-kernel pull: [segments][3] (first send row, first receive row, rows)
  // and the rows arrived per segment
  int32_t *pull_tab = nullptr, *arrived = nullptr;
  uint32_t epoch = 0;         // barrier generation (host counter, passed to the kernels)
  bool connected = false;
};

namespace nk {
uint16_t *ep_recv(const nk_ep_ctx *c);
uint16_t *ep_out(const nk_ep_ctx *c);
int32_t *ep_counts_all(const nk_ep_ctx *c);
// Writes this rank's per-expert counts into every rank's counts matrix row
// `rank`, then waits until every rank has done the same (device barrier).
nk_status ep_exchange_counts(nk_ep_ctx *c, const int32_t *counts, cudaStream_t s);
// Device barrier across the ranks: every rank's prior stores on its stream
// are visible to all before any rank continues.  Bounded (NK_TIMEOUT).
nk_status ep_barrier(nk_ep_ctx *c, cudaStream_t s);
// pull: also the per-segment pull table and zeroed arrival counts
nk_status ep_plan(nk_ep_ctx *c, cudaStream_t s, bool pull);
nk_status ep_dispatch(nk_ep_ctx *c, const uint16_t *x, int64_t tokens, const int32_t *idx,
                      const int32_t *slot_pos, const int32_t *offsets, cudaStream_t s);
nk_status ep_return(nk_ep_ctx *c, cudaStream_t s);
// Device table of the ranks' result buffers (uint64 addresses, rank order).
const uint64_t *ep_out_table(const nk_ep_ctx *c);
// This rank's send buffer (routed rows in expert order, read by the owners)
// and the device table of every rank's.
uint16_t *ep_send(const nk_ep_ctx *c);
const uint64_t *ep_send_table(const nk_ep_ctx *c);
}  // namespace nk
