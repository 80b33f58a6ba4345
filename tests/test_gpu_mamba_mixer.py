"""The Mamba2 mixer end to end on the B200 (projections on the tcgen05 GEMM,
glue kernels between), against the oracle composition of
Mamba2Mixer::forward (mamba2.rs:209-378).

Activations enter the projections in bf16 (the GEMM's operand type) and the
normed rows enter out_proj in bf16, so the end-to-end bar is the BF16 one:
max relative error <= 2e-2.  The oracle sees the same bf16-rounded weights and
projection inputs; everything else in it is the f32/f64 host path."""
import os
import socket

import numpy as np
import pytest
import torch

import nk
import nk_mamba
import oracle as orc
from gpu_util import bf16_round, dev, host, rel_err, rng

pytestmark = pytest.mark.gpu
BF16_TOL = 2e-2


def _proj_ref(x, w):
    """orc.linear with the reference's [in, out] layout from a W [out, in]."""
    rows = x.shape[0]
    return orc.linear(np.ascontiguousarray(w.T), None, w.shape[1], w.shape[0],
                      x.reshape(-1), rows).reshape(rows, w.shape[0])


def _mixer(seed, hidden, C, S, K):
    r = rng(seed)
    f = lambda *s, sc=1.0: (r.standard_normal(s) * sc).astype(np.float32)
    w = dict(inp=f(C, hidden, sc=0.2), dt=f(C, hidden, sc=0.1), b=f(C * S, hidden, sc=0.2),
             c=f(C * S, hidden, sc=0.2), g=f(C, hidden, sc=0.2), out=f(hidden, C, sc=0.2))
    w = {k: bf16_round(v) for k, v in w.items()}
    conv, a, d, nw = f(C, K, sc=0.5), -np.abs(f(C, S)), f(C), f(C)
    m = nk_mamba.Mamba2Mixer(
        hidden, C, S, K, 1e-5, *[nk_mamba.Projection(dev(w[k])) for k in
                                  ("inp", "dt", "b", "c", "g", "out")],
        dev(conv), dev(a), dev(d), dev(nw))
    return m, w, conv, a, d, nw


def _oracle_forward(w, conv, a, d, nw, xh, B, T, C, S, K, conv_state=None, ssm_state=None):
    xb = bf16_round(xh)
    x, dt, b, c, g = (_proj_ref(xb, w[k]) for k in ("inp", "dt", "b", "c", "g"))
    normed, new_conv, fin = orc.mamba2_glue(x, dt, b, c, g, conv, a, nw, 1e-5, B, T, C, S, K,
                                            d=d, conv_state=conv_state, ssm_state=ssm_state)
    return _proj_ref(bf16_round(normed), w["out"]), new_conv, fin


@pytest.mark.parametrize("B,T,hidden,C,S,K", [(1, 12, 32, 16, 8, 4), (2, 9, 64, 32, 16, 4)])
def test_mixer_forward_matches_oracle(cuda, B, T, hidden, C, S, K):
    m, w, conv, a, d, nw = _mixer(B * 10 + T, hidden, C, S, K)
    xh = rng(7).standard_normal((B * T, hidden)).astype(np.float32)
    want, _, _ = _oracle_forward(w, conv, a, d, nw, xh, B, T, C, S, K)
    got = m.forward(dev(xh), B, T)
    torch.cuda.synchronize()
    assert rel_err(host(got), want) <= BF16_TOL


def test_mixer_cache_decode_matches_full_sequence(cuda):
    # mamba2.rs:793-815: decoding token by token through the cache gives the
    # full-sequence outputs.
    B, T, hidden, C, S, K = 2, 6, 32, 16, 8, 4
    m, w, conv, a, d, nw = _mixer(3, hidden, C, S, K)
    xh = rng(8).standard_normal((B, T, hidden)).astype(np.float32)
    full = host(m.forward(dev(xh.reshape(B * T, hidden)), B, T)).reshape(B, T, hidden)
    cache = nk_mamba.Mamba2Cache(B, C, K, S)
    steps = [host(m.forward(dev(np.ascontiguousarray(xh[:, t])), B, 1, cache=cache))
             for t in range(T)]
    step = np.stack(steps, axis=1)
    assert rel_err(step, full) <= 1e-4
    # and the cache holds the oracle's conv/SSM state after the whole sequence
    _, want_conv, want_ssm = _oracle_forward(w, conv, a, d, nw, xh.reshape(B * T, hidden), B, T,
                                             C, S, K)
    assert np.array_equal(host(cache.conv_state), want_conv) or \
        rel_err(host(cache.conv_state), want_conv) <= 1e-6
    assert rel_err(host(cache.ssm_state), want_ssm) <= 1e-3


def _block_weights(seed, hidden, H, P, G, S, K, device):
    g = torch.Generator(device="cpu").manual_seed(seed)
    C = H * P
    W = 2 * C + 2 * G * S + H
    w_in = (torch.randn(W, hidden, generator=g) * 0.05).bfloat16()
    w_out = (torch.randn(hidden, C, generator=g) * 0.05).bfloat16()
    conv = torch.randn(C, K, generator=g) * 0.5
    a = -torch.rand(H, generator=g) - 0.1
    d = torch.randn(H, generator=g)
    nw = torch.randn(C, generator=g)
    return [t.to(device) for t in (w_in, w_out, conv, a, d, nw)]


def _block_oracle(ws, x, hidden, H, P, G, S, K):
    """Expands the fused layout into the reference's per-channel tensors and
    runs the oracle composition (one batch)."""
    w_in, w_out, conv, a, d, nw = [t.float().cpu().numpy() for t in ws]
    C = H * P
    T = x.shape[0]
    fused = _proj_ref(bf16_round(x), w_in)
    z, xs = fused[:, :C], fused[:, C:2 * C]
    bg = fused[:, 2 * C:2 * C + G * S].reshape(T, G, S)
    cg = fused[:, 2 * C + G * S:2 * C + 2 * G * S].reshape(T, G, S)
    dth = fused[:, 2 * C + 2 * G * S:]
    head, grp = np.arange(C) // P, np.arange(C) // (C // G)
    normed, _, _ = orc.mamba2_glue(xs, dth[:, head], bg[:, grp, :].reshape(T, C * S),
                                   cg[:, grp, :].reshape(T, C * S), z, conv,
                                   np.repeat(a[head][:, None], S, axis=1), nw, 1e-5, 1, T, C, S,
                                   K, d=d[head])
    return _proj_ref(bf16_round(normed), w_out)


@pytest.mark.parametrize("H,P,G,S", [(4, 16, 2, 128), (3, 16, 3, 32)])
def test_fused_block_matches_oracle(cuda, H, P, G, S):
    hidden, K, T = 48, 4, 21
    ws = _block_weights(5, hidden, H, P, G, S, K, "cuda")
    blk = nk_mamba.Mamba2Block(*ws, heads=H, head_dim=P, groups=G, state=S, kernel_size=K)
    x = rng(9).standard_normal((T, hidden)).astype(np.float32)
    got = blk.forward(dev(x).bfloat16(), 1, T)
    torch.cuda.synchronize()
    want = _block_oracle(ws, x, hidden, H, P, G, S, K)
    assert rel_err(host(got), want) <= BF16_TOL


def _tp_worker(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "nemotron-cutile-rs_b200"))
    import torch.distributed as dist

    import nk_mamba as nm

    torch.cuda.set_device(rank)
    devc = torch.device("cuda", rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=devc)
    hidden, H, P, G, S, K, T = 256, 8, 32, 2, 128, 4, 100
    ws = _block_weights(6, hidden, H, P, G, S, K, devc)
    x = torch.randn(T, hidden, generator=torch.Generator().manual_seed(2)).to(devc).bfloat16()
    tp = nm.Mamba2Block(*ws, heads=H, head_dim=P, groups=G, state=S, kernel_size=K)
    y_tp = tp.forward(x, 1, T)
    single = nm.Mamba2Block(*ws, heads=H, head_dim=P, groups=G, state=S, kernel_size=K,
                            parallel=False)
    y_1 = single.forward(x, 1, T)
    err = ((y_tp - y_1).abs().max() / y_1.abs().max()).item()
    q.put((rank, err))
    dist.barrier()
    dist.destroy_process_group()


def test_fused_block_tensor_parallel_two_gpus(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, err in res:
        # out_proj inputs are bf16 on both sides; the sums differ only in order.
        assert err <= 1e-2, (rank, err)
