"""Tensor-parallel projections (nk_tp) on 2 and 4 gloo ranks on CPU, with the
oracle's LinearProjection restatement (linear.rs:283-342) standing in for the
device GEMM: a column-parallel up projection (relu2) followed by a
row-parallel down projection must reproduce the single-process MLP
(mlp.rs:157-211) up to f32 summation order."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

M, H, I = 9, 16, 24


def _worker(rank, world, port, q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (os.path.join(root, "nemotron-cutile-rs_b200"), os.path.join(root, "oracle")):
        sys.path.insert(0, p)
    import nk
    import oracle as orc
    import nk_tp

    def cpu_gemm(x, w, kind="bf16", scales=None, bias=None, relu2=False, out_dtype=None, **_):
        m, k = x.shape
        n = w.shape[0]
        y = orc.linear(w.numpy().T.copy(), None if bias is None else bias.numpy(), k, n,
                       x.numpy(), m).reshape(m, n)
        if relu2:
            y = np.maximum(y, 0) ** 2
        return torch.from_numpy(y.astype(np.float32))

    nk.gemm = cpu_gemm  # the device GEMM is replaced by the oracle on CPU
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    r = np.random.default_rng(1)
    up = torch.from_numpy((r.standard_normal((I, H)) * 0.3).astype(np.float32))
    up_b = torch.from_numpy((r.standard_normal(I) * 0.1).astype(np.float32))
    down = torch.from_numpy((r.standard_normal((H, I)) * 0.3).astype(np.float32))
    down_b = torch.from_numpy((r.standard_normal(H) * 0.1).astype(np.float32))
    x = torch.from_numpy(r.standard_normal((M, H)).astype(np.float32))
    col = nk_tp.ColumnParallelLinear(up, up_b, relu2=True)
    row = nk_tp.RowParallelLinear(down, down_b)
    h = col.forward(x, out_dtype=torch.float32)
    y = row.forward(h, out_dtype=torch.float32)
    ref = orc.mlp(H, I, up.numpy().T.copy(), up_b.numpy(), down.numpy().T.copy(),
                  down_b.numpy(), x.numpy(), M).reshape(M, H)
    q.put((rank, float(np.max(np.abs(y.numpy() - ref)) / np.max(np.abs(ref))), col.cols,
           row.k_range))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_ranks_match_single_process_mlp(world):
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    part = I // world
    for rank, err, cols, k_range in res:
        assert cols == (rank * part, (rank + 1) * part)
        assert k_range == (rank * part, (rank + 1) * part)
        assert err <= 1e-6, (rank, err)
