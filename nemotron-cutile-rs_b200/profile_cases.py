"""profile_cases.py — small, self-contained runs of single libnk paths for
profilers (ncu) and quick timing: each case allocates only what its kernels
need, launches them `--iters` times after `--warmup` calls, and prints one
line of CUDA-event timings.

    python nemotron-cutile-rs_b200/profile_cases.py mamba_block --tokens 2048
    python nemotron-cutile-rs_b200/profile_cases.py attention --batch 8 --q-seq 1024
    python nemotron-cutile-rs_b200/profile_cases.py attention --batch 64 --q-seq 1 --kv-len 1280
    python nemotron-cutile-rs_b200/profile_cases.py gemm --m 1 --k 4096 --n 21504
"""
from __future__ import annotations

import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def _timed(torch, fn, warmup, iters):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    e.synchronize()
    return s.elapsed_time(e) / max(iters, 1)


def case_mamba_block(args, torch, nk):
    import nk_mamba

    H, P, G, S, K, hid = 128, 64, 8, 128, 4, 4096
    C = H * P
    W = 2 * C + 2 * G * S + H
    g = torch.Generator(device="cuda").manual_seed(1)
    w_in = (torch.randn(W, hid, device="cuda", generator=g) * 0.02).bfloat16()
    w_out = (torch.randn(hid, C, device="cuda", generator=g) * 0.02).bfloat16()
    conv = torch.randn(C, K, device="cuda", generator=g) * 0.5
    a = -torch.rand(H, device="cuda", generator=g) - 0.5
    d = torch.randn(H, device="cuda", generator=g)
    nw = torch.randn(C, device="cuda", generator=g)
    blk = nk_mamba.Mamba2Block(w_in, w_out, conv, a, d, nw, heads=H, head_dim=P, groups=G,
                               state=S, kernel_size=K, parallel=False)
    x = torch.randn(args.tokens, hid, device="cuda", generator=g).bfloat16()
    ms = _timed(torch, lambda: blk.forward(x, 1, args.tokens), args.warmup, args.iters)
    print(f"mamba_block tokens={args.tokens}: {ms:.3f} ms per forward")


def case_attention(args, torch, nk):
    B, Sq, Hq, Hkv, d = args.batch, args.q_seq, 32, 2, 128
    L = args.kv_len or Sq
    cache = nk.KvCache(B, Hkv, d, ((L + 63) // 64) * 64)
    g = torch.Generator(device="cuda").manual_seed(2)
    kv = torch.randn(B * L, Hkv * d, device="cuda", generator=g).bfloat16()
    cache.append(kv, kv, L)
    q = torch.randn(B * Sq, Hq * d, device="cuda", generator=g).bfloat16()
    ws = [None]

    def run():
        o, ws[0] = nk.attention_gqa(q, cache, Sq, Hq, causal=True, workspace=ws[0])

    ms = _timed(torch, run, args.warmup, args.iters)
    print(f"attention batch={B} q_seq={Sq} kv_len={L}: {ms:.3f} ms per call")


def case_gemm(args, torch, nk):
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(args.m, args.k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(args.n, args.k, device="cuda", generator=g) * 0.02).bfloat16()
    ms = _timed(torch, lambda: nk.gemm(x, w, out_dtype=torch.bfloat16), args.warmup, args.iters)
    print(f"gemm m={args.m} k={args.k} n={args.n}: {ms * 1e3:.1f} us per call "
          f"(back to back, weights L2-resident when they fit)")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["mamba_block", "attention", "gemm"])
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--tokens", type=int, default=2048)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--q-seq", type=int, default=1024)
    ap.add_argument("--kv-len", type=int, default=0)
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--n", type=int, default=21504)
    args = ap.parse_args()
    import torch

    import nk

    {"mamba_block": case_mamba_block, "attention": case_attention,
     "gemm": case_gemm}[args.case](args, torch, nk)


if __name__ == "__main__":
    main()
