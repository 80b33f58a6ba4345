"""The CPU oracle pinned against the reference's own known-answer tests
(transcribed into tests/golden/reference_kats.json with file:line sources)."""
import math

import numpy as np
import pytest

import oracle as orc


def _close(got, want, tol):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape
    assert np.all(np.abs(got - want) <= tol), (got, want)


USIZE_MAX = 2**64 - 1


def test_gemm_kats(kats):
    for c in kats["gemm"]:
        out = orc.gemm(c["lhs"], c["rhs"], c["m"], c["k"], c["n"])
        _close(out, c["out"], c["tol"])


def test_gemm_generated_kat(kats):
    c = kats["gemm_generated"][0]
    m, k, n = c["m"], c["k"], c["n"]
    lhs = ((np.arange(m * k) % 11) - 5.0) * 0.25
    rhs = ((np.arange(k * n) % 7) - 3.0) * 0.5
    out = orc.gemm(lhs, rhs, m, k, n)
    ref = (lhs.reshape(m, k).astype(np.float64) @ rhs.reshape(k, n)).reshape(-1)
    _close(out, ref, c["tol"])


def test_gemm_error_kats(kats):
    for c in kats["gemm_errors"]:
        k = USIZE_MAX if c["k"] == "usize::MAX" else c["k"]
        with pytest.raises(orc.OracleError) as ei:
            orc.gemm(np.zeros(max(c["lhs_len"], 1)), np.zeros(max(c["rhs_len"], 1)), c["m"], k,
                     c["n"], out_len=c["out_len"], lhs_len=c["lhs_len"], rhs_len=c["rhs_len"])
        e = ei.value
        assert e.variant == c["error"], c["name"]
        if c["error"] == "LengthMismatch":
            assert (e.argument, e.expected, e.actual) == (c["argument"], c["expected"], c["actual"])


def test_int4_pack_kats(kats):
    for c in kats["int4_pack"]:
        packed = orc.pack_int4(c["values"])
        assert list(packed) == c["packed"], c["name"]
        assert list(orc.unpack_int4(packed, len(c["values"]))) == c["values"]


def test_int4_quantize_kats(kats):
    for c in kats["int4_quantize"]:
        packed = orc.quantize_int4(c["values"], c["scale"], c["zero_point"])
        assert list(packed) == c["packed"], c["name"]
        if "dequant" in c:
            deq = orc.dequantize_int4(packed, len(c["values"]), c["scale"], c["zero_point"])
            _close(deq, c["dequant"], c.get("tol", 1e-6))


def test_int4_dequantize_kats(kats):
    for c in kats["int4_dequantize"]:
        out = orc.dequantize_int4(c["packed"], c["count"], c["scale"], c["zero_point"])
        _close(out, c["out"], c["tol"])


def test_int4_error_kats(kats):
    for c in kats["int4_errors"]:
        with pytest.raises(orc.OracleError) as ei:
            if c["op"] == "pack":
                orc.pack_int4(c["values"], packed_len=c["packed_len"])
            elif c["op"] == "quantize":
                vals = [float("nan") if v == "nan" else v for v in c["values"]]
                orc.quantize_int4(vals, c["scale"], c["zero_point"], packed_len=c["packed_len"])
            else:
                orc.dequantize_int4(c["packed"], c["count"], c["scale"], c["zero_point"],
                                    out_len=c["out_len"])
        e = ei.value
        assert e.variant == c["error"], c["name"]
        if c["error"] == "LengthMismatch":
            assert (e.argument, e.expected, e.actual) == (c["argument"], c["expected"], c["actual"])
        if c["error"] == "Int4OutOfRange":
            assert e.byte_value == c["byte_value"]
        if c["error"] == "NonFiniteInput":
            assert e.index == c["index"] and math.isnan(e.value)


def test_route_kats(kats):
    for c in kats["route"]:
        mode = orc.SOFTMAX if c["mode"] == "softmax" else orc.SIGMOID
        idx, w = orc.route(c["scores"], c["tokens"], c["experts"], c["top_k"], mode)
        assert list(idx) == c["indices"], c["name"]
        _close(w, c["weights"], c["tol"])


def test_route_model_like_formula(kats):
    c = kats["route_generated"][2]
    t, e, k = c["tokens"], c["experts"], c["top_k"]
    scores = np.array([((ex % 17) - 8.0) * 0.375 + tok * 0.125 - 0.05
                       for tok in range(t) for ex in range(e)], np.float32)
    idx, w = orc.route(scores, t, e, k)
    # highest score per token is (16-8)*0.375 = 3.0 at experts 16, 33, 50, ... (ties -> lower index)
    assert list(idx[:k]) == [16, 33, 50, 67, 84, 101]
    assert np.all(np.diff(w[:k]) <= 0)


def test_route_error_kats(kats):
    for c in kats["route_errors"]:
        with pytest.raises(orc.OracleError) as ei:
            orc.route(np.zeros(max(c["scores_len"], 1)), c["tokens"], c["experts"], c["top_k"],
                      scores_len=c["scores_len"], indices_len=c["indices_len"],
                      weights_len=c["weights_len"])
        e = ei.value
        assert e.variant == c["error"], c["name"]
        if c["error"] == "LengthMismatch":
            assert (e.argument, e.expected, e.actual) == (c["argument"], c["expected"], c["actual"])


def test_linear_kats(kats):
    for c in kats["linear"]:
        out = orc.linear(c["weights"], c["bias"], c["input_dim"], c["output_dim"], c["input"],
                         c["rows"])
        _close(out, c["out"], c["tol"])


def test_linear_int4_materialize(kats):
    c = kats["linear_int4"][0]
    packed = orc.quantize_int4(c["dense_source"], c["scale"], c["zero_point"])
    deq = orc.dequantize_int4(packed, len(c["dense_source"]), c["scale"], c["zero_point"])
    _close(deq, c["dequant"], c["tol"])


def test_mlp_kats(kats):
    for c in kats["mlp"]:
        out = orc.mlp(c["hidden"], c["inter"], c["up_w"], c["up_b"], c["down_w"], c["down_b"],
                      c["input"], c["rows"])
        _close(out, c["out"], c["tol"])


def test_moe_kats(kats):
    for c in kats["moe"]:
        e = c["experts"]
        up = np.ones((e, 1, 1), np.float32)
        down = np.array(c["expert_scales"], np.float32).reshape(e, 1, 1)
        sh = c["shared_scale"]
        out, _, _ = orc.moe(1, e, c["top_k"], 1, 1 if sh is not None else 0, c["router_w"],
                            c["router_b"], up, None, down, None,
                            np.ones(1) if sh is not None else None, None,
                            np.array([sh]) if sh is not None else None, None, c["input"], 1)
        _close(out, c["out"], c["tol"])


def test_int8_row_extension_formula():
    w = np.array([[0.5, -1.0, 0.25, 0.0], [0.0, 0.0, 0.0, 0.0], [127.0, 63.5, -0.5, 1.0]],
                 np.float32)
    q, s = orc.quantize_int8_row(w)
    assert s[0] == np.float32(1.0) / np.float32(127.0)
    assert list(q[0]) == [64, -127, 32, 0]  # 63.5 rounds half away from zero
    assert s[1] == 0 and list(q[1]) == [0, 0, 0, 0]
    assert s[2] == 1.0 and list(q[2]) == [127, 64, -1, 1]


def test_renorm_extension_sums_to_one():
    rng = np.random.default_rng(0)
    scores = rng.standard_normal((16, 128)).astype(np.float32)
    idx_raw, w_raw = orc.route(scores, 16, 128, 6, orc.SIGMOID)
    idx, w = orc.route(scores, 16, 128, 6, orc.SIGMOID_RENORM)
    assert np.array_equal(idx, idx_raw)
    assert np.allclose(w.reshape(16, 6).sum(1), 1.0, atol=1e-6)
    assert np.allclose(w.reshape(16, 6), w_raw.reshape(16, 6) / w_raw.reshape(16, 6).sum(1, keepdims=True), rtol=1e-6)


def test_histogram_is_stable_permutation():
    rng = np.random.default_rng(1)
    idx = rng.integers(0, 8, size=50 * 3).astype(np.int32)
    counts, offs, perm = orc.route_histogram(idx, 50, 3, 8)
    assert counts.sum() == 150 and np.array_equal(np.bincount(idx, minlength=8), counts)
    for e in range(8):
        seg = perm[offs[e]: offs[e] + counts[e]]
        assert np.all(idx[seg] == e) and np.all(np.diff(seg) > 0)
