"""Attention core on the B200 (attention.rs:132-302) against the CPU oracle.

* nk_attention_f32 is the reference contract on f32 tensors (f64 dot
  products and sums): the f32-accumulate bar, 1e-3 (in practice ~1e-6).
* nk_attention_gqa is the serving path over the bf16 KV cache with the
  tcgen05 GEMM: its operands are bf16, so the oracle gets the same
  bf16-rounded q/k/v and the bar is the BF16 one, 2e-2."""
import numpy as np
import pytest
import torch

import nk
import oracle as orc
from gpu_util import bf16_round, dev, host, rel_err, rng

pytestmark = pytest.mark.gpu


def _t(a):
    a = np.asarray(a, np.float32).reshape(-1)
    return dev(a) if a.size else torch.empty(0, device="cuda")


def test_attention_f32_kats(cuda, kats):
    for c in kats["attention"]:
        B, Sq, Skv, Hq, Hkv, d = c["shape"]
        out = nk.attention_f32(_t(c["q"]), _t(c["k"]), _t(c["v"]), B, Sq, Skv, Hq, Hkv, d,
                               causal=c["causal"], q_offset=c["q_offset"], scale=c["scale"])
        torch.cuda.synchronize()
        assert np.all(np.abs(host(out) - np.float32(c["out"])) <= c["tol"]), c["name"]


def test_attention_f32_error_kats(cuda, kats):
    for c in kats["attention_errors"]:
        B, Sq, Skv, Hq, Hkv, d = c["shape"]
        out = torch.empty(max(c["out_len"], 1), device="cuda")
        with pytest.raises(nk.NkError) as ei:
            nk.attention_f32(torch.ones(c["q_len"], device="cuda"),
                             torch.ones(c["k_len"], device="cuda"),
                             torch.ones(c["v_len"], device="cuda"), B, Sq, Skv, Hq, Hkv, d,
                             scale=c["scale"], out=out[:c["out_len"]])
        e = ei.value
        assert e.variant == c["error"], c["name"]
        if c["error"] == "LengthMismatch":
            assert (e.argument, e.expected, e.actual) == (c["argument"], c["expected"],
                                                          c["actual"])


@pytest.mark.parametrize("B,Sq,Skv,Hq,Hkv,d,causal,off", [
    (1, 3, 5, 2, 1, 8, False, 0), (2, 7, 7, 4, 2, 16, True, 0), (2, 1, 33, 8, 2, 64, True, 32),
    (1, 40, 40, 32, 2, 128, True, 0)])
def test_attention_f32_matches_oracle(cuda, B, Sq, Skv, Hq, Hkv, d, causal, off):
    r = rng(B + Sq + Skv + d)
    q = r.standard_normal((B, Sq, Hq, d)).astype(np.float32)
    k = r.standard_normal((B, Skv, Hkv, d)).astype(np.float32)
    v = r.standard_normal((B, Skv, Hkv, d)).astype(np.float32)
    want = orc.attention(q, k, v, B, Sq, Skv, Hq, Hkv, d, causal=causal, q_offset=off)
    got = nk.attention_f32(dev(q), dev(k), dev(v), B, Sq, Skv, Hq, Hkv, d, causal=causal,
                           q_offset=off)
    torch.cuda.synchronize()
    assert rel_err(host(got), want) <= 1e-5


def test_attention_f32_no_valid_targets(cuda):
    # A NaN score row (attention.rs:224-230): the first failing row is reported.
    B, Sq, Skv, Hq, Hkv, d = 1, 2, 3, 2, 1, 4
    q = np.ones((B, Sq, Hq, d), np.float32)
    q[0, 1, 0, 0] = np.nan  # row (b=0, q=1, h=0) = 2
    k = np.ones((B, Skv, Hkv, d), np.float32)
    v = np.ones((B, Skv, Hkv, d), np.float32)
    with pytest.raises(orc.OracleError) as oe:
        orc.attention(q, k, v, B, Sq, Skv, Hq, Hkv, d)
    with pytest.raises(nk.NkError) as ne:
        nk.attention_f32(dev(q), dev(k), dev(v), B, Sq, Skv, Hq, Hkv, d)
    assert ne.value.variant == oe.value.variant == "NoValidAttentionTargets"
    assert ne.value.index == oe.value.index == 2


def _gqa_case(seed, B, S_prev, S_new, Hq, Hkv, d, max_len):
    r = rng(seed)
    L = S_prev + S_new
    q = bf16_round(r.standard_normal((B, S_new, Hq, d)).astype(np.float32))
    k = bf16_round(r.standard_normal((B, L, Hkv, d)).astype(np.float32))
    v = bf16_round(r.standard_normal((B, L, Hkv, d)).astype(np.float32))
    return q, k, v, L


@pytest.mark.parametrize("B,S_prev,S_new,Hq,Hkv,d,chunk", [
    (2, 0, 37, 8, 2, 128, None),      # causal prefill, G = 4
    (3, 0, 130, 4, 1, 64, None),      # key tiles above the diagonal skipped
    (2, 70, 1, 32, 2, 128, None),     # decode step, q_offset 70
    (4, 5, 3, 16, 2, 128, "3"),       # chunked pairs
    (1, 0, 300, 32, 2, 128, "1"),     # prefill with 16 queries x 16 heads tiles
    (1, 650, 50, 8, 2, 128, None),    # rows of 700 keys (register softmax, 32 per lane)
    (1, 2097, 3, 4, 2, 64, None)])    # rows of 2100 keys (block softmax)
def test_attention_gqa_matches_oracle(cuda, monkeypatch, B, S_prev, S_new, Hq, Hkv, d, chunk):
    if chunk:
        monkeypatch.setenv("NK_ATTN_CHUNK", chunk)
    max_len = ((S_prev + S_new + 63) // 64) * 64 + 64
    q, k, v, L = _gqa_case(B * 7 + S_new, B, S_prev, S_new, Hq, Hkv, d, max_len)
    cache = nk.KvCache(B, Hkv, d, max_len)
    if S_prev:
        cache.append(dev(k[:, :S_prev].reshape(B * S_prev, Hkv * d)).bfloat16(),
                     dev(v[:, :S_prev].reshape(B * S_prev, Hkv * d)).bfloat16(), S_prev)
    cache.append(dev(np.ascontiguousarray(k[:, S_prev:]).reshape(B * S_new, Hkv * d)).bfloat16(),
                 dev(np.ascontiguousarray(v[:, S_prev:]).reshape(B * S_new, Hkv * d)).bfloat16(),
                 S_new)
    out, ws = nk.attention_gqa(dev(q.reshape(B * S_new, Hq * d)).bfloat16(), cache, S_new, Hq,
                               causal=True, out_dtype=nk.F32)
    torch.cuda.synchronize()
    want = orc.attention(q, k, v, B, S_new, L, Hq, Hkv, d, causal=True, q_offset=S_prev)
    assert rel_err(host(out).reshape(-1), want) <= 2e-2
    assert nk.attention_check(ws) == -1


def test_kv_cache_layout(cuda):
    B, S, Hkv, d, Lmax = 2, 5, 2, 64, 64
    r = rng(1)
    kn = r.standard_normal((B * S, Hkv * d)).astype(np.float32)
    vn = r.standard_normal((B * S, Hkv * d)).astype(np.float32)
    cache = nk.KvCache(B, Hkv, d, Lmax)
    cache.length = 3
    cache.append(dev(kn).bfloat16(), dev(vn).bfloat16(), S)
    torch.cuda.synchronize()
    k = host(cache.k)
    vt = host(cache.vt)
    kr = bf16_round(kn).reshape(B, S, Hkv, d)
    vr = bf16_round(vn).reshape(B, S, Hkv, d)
    assert np.array_equal(k[:, :, 3:3 + S].transpose(0, 2, 1, 3), kr)
    assert np.array_equal(vt[:, :, :, 3:3 + S].transpose(0, 3, 1, 2), vr)
    assert not k[:, :, :3].any() and not k[:, :, 3 + S:].any()
    assert cache.length == 3 + S
