"""INT4-affine quantize/pack/unpack/dequantize on the B200, bit-exact against
the oracle (quantize.rs:59-204) and the reference KATs."""
import math

import numpy as np
import pytest
import torch

import nk
import oracle as orc
from gpu_util import dev, host, rng

pytestmark = pytest.mark.gpu


def _u8(a, cuda):
    return torch.tensor(list(a), dtype=torch.uint8, device=cuda) if len(a) else \
        torch.empty(1, dtype=torch.uint8, device=cuda)


def q4(values, scale, zp, cuda, packed_len=None):
    v = torch.tensor(values, dtype=torch.float32, device=cuda) if len(values) else \
        torch.empty(1, device=cuda)
    n = len(values)
    pl = (n + 1) // 2 if packed_len is None else packed_len
    out = torch.full((max(pl, 1),), 0xFF, dtype=torch.uint8, device=cuda)
    nk.call("nk_quantize_int4", nk.ptr(v), n, scale, zp, nk.ptr(out), pl, nk.stream_ptr())
    return host(out[:pl])


def test_quantize_kats(cuda, kats):
    for c in kats["int4_quantize"]:
        got = q4(c["values"], c["scale"], c["zero_point"], cuda)
        assert list(got) == c["packed"], c["name"]


def test_pack_unpack_kats(cuda, kats):
    for c in kats["int4_pack"]:
        n = len(c["values"])
        vals = _u8(c["values"], cuda)
        packed = torch.empty(max((n + 1) // 2, 1), dtype=torch.uint8, device=cuda)
        nk.call("nk_pack_int4", nk.ptr(vals), n, nk.ptr(packed), (n + 1) // 2, nk.stream_ptr())
        assert list(host(packed[:(n + 1) // 2])) == c["packed"]
        out = torch.empty(max(n, 1), dtype=torch.uint8, device=cuda)
        nk.call("nk_unpack_int4", nk.ptr(packed), (n + 1) // 2, n, nk.ptr(out), n, nk.stream_ptr())
        torch.cuda.synchronize()
        assert list(host(out[:n])) == c["values"]


def test_dequantize_kats(cuda, kats):
    for c in kats["int4_dequantize"]:
        pk = _u8(c["packed"], cuda)
        out = torch.full((c["count"],), -1.0, device=cuda)
        nk.call("nk_dequantize_int4", nk.ptr(pk), len(c["packed"]), c["count"], c["scale"],
                c["zero_point"], nk.ptr(out), c["count"], nk.stream_ptr())
        torch.cuda.synchronize()
        assert np.allclose(host(out), c["out"], atol=c["tol"], rtol=0)


def test_error_kats_on_device(cuda, kats):
    for c in kats["int4_errors"]:
        with pytest.raises(nk.NkError) as ei:
            if c["op"] == "pack":
                vals = _u8(c["values"], cuda)
                out = torch.empty(1, dtype=torch.uint8, device=cuda)
                nk.call("nk_pack_int4", nk.ptr(vals), len(c["values"]), nk.ptr(out),
                        c["packed_len"], nk.stream_ptr())
            elif c["op"] == "quantize":
                vals = [float("nan") if v == "nan" else v for v in c["values"]]
                q4(vals, c["scale"], c["zero_point"], cuda, packed_len=c["packed_len"])
            else:
                pk = _u8(c["packed"], cuda)
                out = torch.empty(max(c["out_len"], 1), device=cuda)
                nk.call("nk_dequantize_int4", nk.ptr(pk), len(c["packed"]), c["count"],
                        c["scale"], c["zero_point"], nk.ptr(out), c["out_len"], nk.stream_ptr())
        e = ei.value
        assert e.variant == c["error"], c["name"]
        if c["error"] == "LengthMismatch":
            assert (e.argument, e.expected, e.actual) == (c["argument"], c["expected"], c["actual"])
        if c["error"] == "Int4OutOfRange":
            assert e.byte_value == c["byte_value"]
        if c["error"] == "NonFiniteInput":
            assert e.index == c["index"] and math.isnan(e.value)


def test_quantize_random_bit_exact_with_ties(cuda):
    r = rng(0)
    n = 1_000_001  # odd: a trailing half byte
    v = (r.standard_normal(n) * 3).astype(np.float32)
    v[::97] = (np.round(v[::97] * 2) / 2).astype(np.float32)  # exact .5 multiples: rounding ties
    for scale, zp in [(0.5, 8), (0.37, 3), (1.0, 0), (0.1, 15)]:
        ref = orc.quantize_int4(v, scale, zp)
        got = q4(v.tolist(), scale, zp, cuda) if n < 1000 else None
        vt = dev(v)
        out = torch.empty(ref.size, dtype=torch.uint8, device=cuda)
        nk.call("nk_quantize_int4", nk.ptr(vt), n, scale, zp, nk.ptr(out), ref.size, nk.stream_ptr())
        assert np.array_equal(host(out), ref), (scale, zp)
        deq = torch.empty(n, device=cuda)
        nk.call("nk_dequantize_int4", nk.ptr(out), ref.size, n, scale, zp, nk.ptr(deq), n,
                nk.stream_ptr())
        assert np.array_equal(host(deq), orc.dequantize_int4(ref, n, scale, zp))
        del got


def test_non_finite_reports_first_index(cuda):
    v = np.zeros(5000, np.float32)
    v[1234] = np.inf
    v[4000] = np.nan
    with pytest.raises(nk.NkError) as ei:
        q4(v.tolist(), 1.0, 8, cuda)
    assert ei.value.variant == "NonFiniteInput" and ei.value.index == 1234
    assert math.isinf(ei.value.value)


def test_pack_out_of_range_reports_first_value(cuda):
    vals = torch.tensor([1, 2, 15, 16, 200], dtype=torch.uint8, device=cuda)
    out = torch.empty(3, dtype=torch.uint8, device=cuda)
    with pytest.raises(nk.NkError) as ei:
        nk.call("nk_pack_int4", nk.ptr(vals), 5, nk.ptr(out), 3, nk.stream_ptr())
    assert ei.value.variant == "Int4OutOfRange" and ei.value.byte_value == 16


def test_int8_row_quantize_bit_exact(cuda):
    r = rng(2)
    w = (r.standard_normal((300, 1000)) * 0.02).astype(np.float32)
    w[5] = 0.0
    w[7, 3] = 0.5
    w[7, 4] = -0.5
    q_ref, s_ref = orc.quantize_int8_row(w)
    q, s = nk.quantize_int8_row(dev(w))
    assert np.array_equal(host(q), q_ref) and np.array_equal(host(s), s_ref)
