"""Tensor-parallel projections on 2 B200s: column-parallel in_proj-like and
row-parallel out_proj-like GEMMs (NCCL all-reduce of f32 partials) must match
the single-GPU projection within the f32-accumulate bar (1e-3).  Skipped when
fewer than 2 GPUs are visible."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "nemotron-cutile-rs_b200"))
    import torch.distributed as dist

    import nk
    import nk_tp

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    g = torch.Generator(device=dev).manual_seed(4)
    M, H, N_in, K_out = 512, 1024, 2320, 2048
    x = torch.randn(M, H, device=dev, generator=g).bfloat16()
    w_in = (torch.randn(N_in, H, device=dev, generator=g) * 0.02).bfloat16()
    b_in = torch.randn(N_in, device=dev, generator=g)
    w_out = (torch.randn(H, K_out, device=dev, generator=g) * 0.02).bfloat16()
    b_out = torch.randn(H, device=dev, generator=g)
    z = torch.randn(M, K_out, device=dev, generator=g).bfloat16()
    col = nk_tp.ColumnParallelLinear(w_in, b_in)
    y_col = col.forward(x, out_dtype=torch.float32)
    ref_col = nk.gemm(x, w_in, bias=b_in)[:, col.cols[0]:col.cols[1]]
    row = nk_tp.RowParallelLinear(w_out, b_out)
    a, b = row.k_range
    y_row = row.forward(z[:, a:b].contiguous(), out_dtype=torch.float32)
    ref_row = nk.gemm(z, w_out, bias=b_out)
    e1 = ((y_col - ref_col).abs().max() / ref_col.abs().max()).item()
    e2 = ((y_row - ref_row).abs().max() / ref_row.abs().max()).item()
    nk.device_status()
    q.put((rank, e1, e2))
    dist.barrier()
    dist.destroy_process_group()


def test_tensor_parallel_two_gpus_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, e1, e2 in res:
        assert e1 <= 1e-3 and e2 <= 1e-3, (rank, e1, e2)
