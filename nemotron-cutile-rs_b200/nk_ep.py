"""nk_ep.py — expert-parallel MoE layer over torch.distributed.

Experts are partitioned over G ranks in contiguous ranges (rank g owns
experts [g*E/G, (g+1)*E/G)); every rank keeps the router and the shared
expert and routes its own tokens.  One forward:

  1. dispatch  (token rank)  router GEMM -> top-k -> plan -> routed rows in
                             expert order, so the rows bound for each rank are
                             one contiguous block
  2. all-to-all of the per-expert row counts, then of the routed rows
  3. experts   (expert rank) grouped MLP over the received rows, which arrive
                             as G x E/G segments (source rank major)
  4. all-to-all back: each row returns to its token rank in its original slot
  5. shared expert + combine (token rank), in the reference's rank order
     (nemotron-nn/src/moe.rs:195-246)

The reference runs on one device only (nemotron-kernels/src/device.rs:32-54);
this is the distribution the benchmark configuration asks for.  The row
exchange is NCCL all-to-all-v over NVLink (`torch.distributed` on the NCCL
backend); the row counts must reach the host to size it, which costs one
device synchronisation per layer.

The compute comes from a backend object.  `NkBackend` runs libnk's kernels on
the local GPU; the tests supply a CPU backend built on the oracle to check the
orchestration itself on `gloo` ranks.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

import nk


class NkBackend:
    """libnk stages on the local GPU.

    `dispatch_layer` describes the whole layer (router over all E experts);
    `local_layer` the experts this rank holds (experts = E/G, expert weights
    stacked in local order).  Both are nk.MoeWeights."""

    def __init__(self, dispatch_layer: nk.MoeWeights, local_layer: nk.MoeWeights):
        self.d = dispatch_layer
        self.l = local_layer
        self._ds = dispatch_layer.struct()
        self._ls = local_layer.struct()
        self._ws = {}

    def _buf(self, name, nbytes, device):
        b = self._ws.get(name)
        if b is None or b.numel() < nbytes:
            b = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
            self._ws[name] = b
        return b

    def dispatch(self, x):
        t, h = x.shape
        k, e = self.d.top_k, self.d.experts
        dev = x.device
        idx = torch.empty(t * k, dtype=torch.int32, device=dev)
        w = torch.empty(t * k, dtype=torch.float32, device=dev)
        counts = torch.empty(e, dtype=torch.int32, device=dev)
        offsets = torch.empty(e + 1, dtype=torch.int32, device=dev)
        slot_pos = torch.empty(t * k, dtype=torch.int32, device=dev)
        rows = torch.empty(t * k, h, dtype=torch.bfloat16, device=dev)
        need = ctypes.c_size_t()
        nk.call("nk_moe_dispatch_workspace_bytes", ctypes.byref(self._ds), t, ctypes.byref(need))
        ws = self._buf("dispatch", need.value, dev)
        nk.call("nk_moe_dispatch", ctypes.byref(self._ds), nk.ptr(x), t, nk.ptr(idx), nk.ptr(w),
                nk.ptr(counts), nk.ptr(offsets), nk.ptr(slot_pos), nk.ptr(rows), nk.ptr(ws),
                ws.numel(), nk.stream_ptr())
        return idx, w, counts, slot_pos, rows

    def experts(self, rows, seg_expert, seg_rows):
        n, n_seg = rows.shape[0], seg_rows.numel()
        out = torch.empty_like(rows)
        need = ctypes.c_size_t()
        nk.call("nk_moe_experts_workspace_bytes", ctypes.byref(self._ls), n, n_seg,
                ctypes.byref(need))
        ws = self._buf("experts", need.value, rows.device)
        nk.call("nk_moe_experts", ctypes.byref(self._ls), nk.ptr(rows), n, nk.ptr(seg_expert),
                nk.ptr(seg_rows), n_seg, nk.ptr(out), nk.ptr(ws), ws.numel(), nk.stream_ptr())
        return out

    def shared(self, x):
        if self.d.shared_inter <= 0:
            return None
        t, h = x.shape
        s1 = torch.empty(t, self.d.shared_inter, dtype=torch.bfloat16, device=x.device)
        sh = torch.empty(t, h, dtype=torch.bfloat16, device=x.device)
        nk.call("nk_moe_shared", ctypes.byref(self._ds), nk.ptr(x), t, nk.ptr(s1), nk.ptr(sh),
                nk.stream_ptr())
        return sh

    def combine(self, y, sh, w, slot_pos, tokens, out_dtype):
        h, k = self.d.hidden, self.d.top_k
        out = torch.empty(tokens, h, dtype=out_dtype, device=y.device)
        nk.call("nk_moe_combine", nk.ptr(y), nk.ptr(sh), nk.ptr(w), nk.ptr(slot_pos), tokens, h,
                k, nk.ptr(out), nk.F32 if out_dtype == torch.float32 else nk.BF16,
                nk.stream_ptr())
        return out

    def row_dtype(self):
        return torch.bfloat16


class ExpertParallelMoe:
    """MoeLayer::forward_into with experts sharded over the ranks of `group`."""

    def __init__(self, backend, experts: int, hidden: int, top_k: int, group=None):
        self.be = backend
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if experts % self.world:
            raise ValueError(f"{experts} experts do not split over {self.world} ranks")
        self.E, self.H, self.K = experts, hidden, top_k
        self.E_local = experts // self.world
        self.last_exchange = {}

    def forward(self, x, out_dtype=torch.float32):
        G, El, H = self.world, self.E_local, self.H
        t = x.shape[0]
        idx, w, counts, slot_pos, rows = self.be.dispatch(x)
        # 2a. per-expert counts: row g of `send` goes to rank g (its experts)
        send = counts.reshape(G, El).contiguous()
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        send_rows = send.sum(1).tolist()  # host sync: NCCL needs the split sizes
        recv_rows = recv.sum(1).tolist()
        # 2b. routed rows to the ranks that own their experts
        n_recv = int(sum(recv_rows))
        rbuf = torch.empty(n_recv, H, dtype=rows.dtype, device=rows.device)
        dist.all_to_all_single(rbuf, rows, recv_rows, send_rows, group=self.group)
        # 3. local experts over G x El segments (source rank major)
        seg_rows = recv.reshape(-1).contiguous()
        seg_expert = torch.arange(El, dtype=torch.int32, device=seg_rows.device).repeat(G)
        ybuf = self.be.experts(rbuf, seg_expert, seg_rows)
        # 4. results back to the token ranks, into the dispatch order
        y = torch.empty_like(rows)
        dist.all_to_all_single(y, ybuf, send_rows, recv_rows, group=self.group)
        self.last_exchange = {"sent_rows": send_rows, "received_rows": recv_rows}
        # 5. shared expert and the rank-ordered combine
        sh = self.be.shared(x)
        return self.be.combine(y, sh, w, slot_pos, t, out_dtype), idx, w


def local_expert_slice(tensor, rank, world, experts):
    """Rows of an expert-stacked tensor ([E, ...]) owned by `rank`."""
    el = experts // world
    return tensor[rank * el:(rank + 1) * el]
