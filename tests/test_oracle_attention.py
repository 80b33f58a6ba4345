"""The CPU oracle's attention core pinned against the reference's inline
known-answer tests (nemotron-kernels/src/attention.rs, transcribed into
tests/golden/reference_kats.json with file:line sources)."""
import numpy as np
import pytest

import oracle as orc


def test_attention_kats(kats):
    for c in kats["attention"]:
        B, Sq, Skv, Hq, Hkv, d = c["shape"]
        out = orc.attention(c["q"], c["k"], c["v"], B, Sq, Skv, Hq, Hkv, d, causal=c["causal"],
                            q_offset=c["q_offset"], scale=c["scale"])
        assert np.all(np.abs(out - np.float32(c["out"])) <= c["tol"]), c["name"]


def test_attention_error_kats(kats):
    for c in kats["attention_errors"]:
        B, Sq, Skv, Hq, Hkv, d = c["shape"]
        with pytest.raises(orc.OracleError) as ei:
            orc.attention(np.ones(c["q_len"]), np.ones(c["k_len"]), np.ones(c["v_len"]), B, Sq,
                          Skv, Hq, Hkv, d, scale=c["scale"], out_len=c["out_len"])
        e = ei.value
        assert e.variant == c["error"], c["name"]
        if c["error"] == "LengthMismatch":
            assert (e.argument, e.expected, e.actual) == (c["argument"], c["expected"],
                                                          c["actual"])
        if c["error"] == "InvalidScale":
            assert e.value == c["value"]


def test_attention_matches_float64_softmax():
    # Independent check of the restatement: softmax(QKᵀ·s)V in float64 numpy.
    r = np.random.default_rng(0)
    B, Sq, Skv, Hq, Hkv, d = 2, 5, 7, 4, 2, 8
    q = r.standard_normal((B, Sq, Hq, d)).astype(np.float32)
    k = r.standard_normal((B, Skv, Hkv, d)).astype(np.float32)
    v = r.standard_normal((B, Skv, Hkv, d)).astype(np.float32)
    out = orc.attention(q, k, v, B, Sq, Skv, Hq, Hkv, d, causal=True, q_offset=2)
    out = out.reshape(B, Sq, Hq, d)
    for b in range(B):
        for i in range(Sq):
            for h in range(Hq):
                kh = h // (Hq // Hkv)
                s = k[b, :, kh].astype(np.float64) @ q[b, i, h].astype(np.float64) / np.sqrt(d)
                s[min(2 + i, Skv - 1) + 1:] = -np.inf
                w = np.exp(s - s.max())
                w /= w.sum()
                ref = w @ v[b, :, kh].astype(np.float64)
                assert np.allclose(out[b, i, h], ref, rtol=1e-5, atol=1e-6)
