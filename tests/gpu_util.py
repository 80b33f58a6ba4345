"""Shared helpers of the GPU parity tests (seeded inputs, bf16 rounding)."""
import numpy as np
import torch


def rng(seed):
    return np.random.default_rng(seed)


def bf16_round(a):
    """f32 values rounded to bf16 (round-to-nearest-even), returned as f32."""
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
    return t.to(torch.bfloat16).to(torch.float32).numpy()


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def host(t):
    return t.detach().float().cpu().numpy() if t.dtype in (torch.bfloat16, torch.float16) \
        else t.detach().cpu().numpy()


def rel_err(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(got - ref))) / max(float(np.max(np.abs(ref))), 1e-30)
