"""nk_tp.py — tensor-parallel projections over torch.distributed.

The large dense projections on this path (Mamba2 in/out projections,
mamba2.rs:229-263,353-359; attention Q/K/V/O, attention.rs:170-209; the MLP
pair, mlp.rs:201-208) are `LinearProjection::project_into`
(linear.rs:283-342) calls.  Split over G ranks in the usual pair:

* ColumnParallelLinear: rank g holds output features [g*N/G, (g+1)*N/G) of W
  and computes that slice of Y from the full X — no communication; the
  epilogue (bias, relu2) applies per feature, so it stays local.
* RowParallelLinear: rank g holds input features [g*K/G, (g+1)*K/G) of W and
  the matching slice of X; each rank's f32 partial product is summed over
  ranks with one all-reduce, then the bias is added once (linear.rs:333-339
  adds it after the GEMM).

A column-parallel projection followed by a row-parallel one (up then down)
needs exactly one all-reduce.  The GEMMs are libnk's (nk_gemm_bf16 /
nk_gemm_w8row); the all-reduce is NCCL over NVLink.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

import nk


def _shard(n: int, world: int, rank: int):
    if n % world:
        raise ValueError(f"{n} does not split over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


class ColumnParallelLinear:
    """Y[:, shard] = X · W[shard, :]ᵀ (+ b[shard]) (relu2).  W is [N, K] (output major)."""

    def __init__(self, w_full, bias_full=None, relu2=False, group=None, kind="bf16",
                 scales_full=None):
        self.group = group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        a, b = _shard(w_full.shape[0], self.world, self.rank)
        self.w = w_full[a:b].contiguous()
        self.bias = None if bias_full is None else bias_full[a:b].contiguous()
        self.scales = None if scales_full is None else scales_full[a:b].contiguous()
        self.kind, self.relu2 = kind, relu2
        self.cols = (a, b)

    def forward(self, x, out_dtype=torch.bfloat16):
        return nk.gemm(x, self.w, kind=self.kind, scales=self.scales, bias=self.bias,
                       relu2=self.relu2, out_dtype=out_dtype)


class RowParallelLinear:
    """Y = Σ_g X[:, shard_g] · W[:, shard_g]ᵀ (+ b), one all-reduce of f32 partials."""

    def __init__(self, w_full, bias_full=None, group=None, kind="bf16", scales_full=None):
        self.group = group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        a, b = _shard(w_full.shape[1], self.world, self.rank)
        self.w = w_full[:, a:b].contiguous()
        self.bias = bias_full
        self.scales = scales_full  # per output row: the same on every rank (linear)
        self.kind = kind
        self.k_range = (a, b)

    def forward(self, x_shard, out_dtype=torch.bfloat16):
        part = nk.gemm(x_shard, self.w, kind=self.kind, scales=self.scales,
                       out_dtype=torch.float32)
        dist.all_reduce(part, group=self.group)
        if self.bias is not None:
            part += self.bias
        return part if out_dtype == torch.float32 else part.to(out_dtype)
