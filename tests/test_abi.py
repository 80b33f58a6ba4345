"""The C ABI (include/nk.h) without a GPU: the library loads, exports every
declared symbol, and host-side validation mirrors the reference's error
variants and order (no device work is reached on these paths)."""
import ctypes
import os
import re

import pytest

import nk
from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "nk.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^(?:nk_status|int32_t)\s+(nk_\w+)\s*\(", text, re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = nk.lib()
    syms = declared_symbols()
    assert len(syms) >= 19
    for s in syms:
        assert hasattr(lib, s), s
        assert s in nk._SIGS, f"binding lacks {s}"
    assert lib.nk_version() == 100


def err():
    return nk.last_error()


def test_gemm_f32_shape_then_length_order():
    lib = nk.lib()
    # gemm.rs:491-496 zero dim
    assert lib.nk_gemm_f32(None, 1, None, 1, None, 1, 0, 1, 1, None) == nk.INVALID_SHAPE
    # gemm.rs:500-508 overflow
    assert lib.nk_gemm_f32(None, 1, None, 1, None, 2, 2, 2**64 - 1, 1, None) == nk.INVALID_SHAPE
    # lhs before rhs before output (gemm.rs:114-147)
    assert lib.nk_gemm_f32(None, 1, None, 1, None, 1, 1, 2, 1, None) == nk.LENGTH_MISMATCH
    e = err()
    assert (e.argument, e.expected, e.actual) == (b"lhs", 2, 1)
    assert lib.nk_gemm_f32(None, 2, None, 1, None, 1, 1, 2, 1, None) == nk.LENGTH_MISMATCH
    assert err().argument == b"rhs"
    assert lib.nk_gemm_f32(None, 2, None, 4, None, 1, 1, 2, 2, None) == nk.LENGTH_MISMATCH
    e = err()
    assert (e.argument, e.expected, e.actual) == (b"output", 2, 1)


def test_int4_param_and_length_validation():
    lib = nk.lib()
    assert lib.nk_validate_int4_params(0.5, 8) == nk.OK
    assert lib.nk_validate_int4_params(0.0, 8) == nk.INVALID_PARAMS
    assert lib.nk_validate_int4_params(float("inf"), 8) == nk.INVALID_PARAMS
    assert lib.nk_validate_int4_params(0.5, 16) == nk.INVALID_PARAMS
    # quantize.rs:507-514: params checked first
    assert lib.nk_quantize_int4(None, 1, 0.0, 8, None, 1, None) == nk.INVALID_PARAMS
    # quantize.rs:551-566 output length before packed length
    assert lib.nk_dequantize_int4(None, 1, 2, 1.0, 0, None, 1, None) == nk.LENGTH_MISMATCH
    e = err()
    assert (e.argument, e.expected, e.actual) == (b"output", 2, 1)
    assert lib.nk_pack_int4(None, 3, None, 1, None) == nk.LENGTH_MISMATCH
    assert err().argument == b"packed"
    assert lib.nk_unpack_int4(None, 2, 4, None, 3, None) == nk.LENGTH_MISMATCH
    assert err().argument == b"output"
    # empty input is valid and does no device work (quantize.rs:491-501)
    assert lib.nk_pack_int4(None, 0, None, 0, None) == nk.OK
    assert lib.nk_unpack_int4(None, 0, 0, None, 0, None) == nk.OK
    assert lib.nk_dequantize_int4(None, 0, 0, 0.5, 8, None, 0, None) == nk.OK


def test_w4a_validation_order():
    lib = nk.lib()
    assert lib.nk_gemm_w4a(None, nk.BF16, None, 2, 0.0, 8, None, None, nk.F32, 1, 2, 2, 0,
                           None) == nk.INVALID_PARAMS
    assert lib.nk_gemm_w4a(None, nk.BF16, None, 1, 0.5, 8, None, None, nk.F32, 1, 2, 2, 0,
                           None) == nk.LENGTH_MISMATCH
    e = err()
    assert (e.argument, e.expected, e.actual) == (b"packed_weights", 2, 1)


def test_route_validation_order():
    lib = nk.lib()
    # moe_routing.rs:707-726
    assert lib.nk_moe_route(None, 0, 1, 0, 1, 0, None, 1, None, 1, None) == nk.INVALID_SHAPE
    assert lib.nk_moe_route(None, 2, 1, 2, 3, 0, None, 3, None, 3, None) == nk.INVALID_SHAPE
    # moe_routing.rs:731-790: scores, indices, weights
    assert lib.nk_moe_route(None, 3, 2, 2, 1, 0, None, 2, None, 2, None) == nk.LENGTH_MISMATCH
    e = err()
    assert (e.argument, e.expected, e.actual) == (b"scores", 4, 3)
    assert lib.nk_moe_route(None, 2, 1, 2, 2, 0, None, 1, None, 2, None) == nk.LENGTH_MISMATCH
    assert err().argument == b"indices"
    assert lib.nk_moe_route(None, 2, 1, 2, 2, 0, None, 2, None, 1, None) == nk.LENGTH_MISMATCH
    assert err().argument == b"weights"
    # empty token batch is valid (moe_routing.rs:696-702)
    assert lib.nk_moe_route(None, 0, 0, 4, 2, 0, None, 0, None, 0, None) == nk.OK


def test_moe_layer_validation():
    lib = nk.lib()
    s = nk.NkMoeLayer()
    s.hidden, s.experts, s.top_k, s.inter = 8, 2, 3, 16
    b = ctypes.c_size_t()
    assert lib.nk_moe_workspace_bytes(ctypes.byref(s), 4, ctypes.byref(b)) == nk.INVALID_SHAPE
    s.top_k = 1
    s.router_w3 = s.up_w = s.down_w = 16
    assert lib.nk_moe_workspace_bytes(ctypes.byref(s), 0, ctypes.byref(b)) == nk.INVALID_ROW_COUNT
    assert lib.nk_moe_workspace_bytes(ctypes.byref(s), 4, ctypes.byref(b)) == nk.OK
    assert b.value > 0
    assert lib.nk_moe_forward(ctypes.byref(s), None, 4, None, nk.F32, None, None, None, 0,
                              None) == nk.WORKSPACE_TOO_SMALL


def test_moe_pipeline_validation():
    # nk_moe_pipeline_*: argument checks come before any device call.
    lib = nk.lib()
    s = nk.NkMoeLayer()
    s.hidden, s.experts, s.top_k, s.inter = 8, 2, 1, 16
    s.router_w3 = s.up_w = s.down_w = 16
    p = ctypes.c_void_p()
    assert lib.nk_moe_pipeline_create(None, 4, nk.F32, None, None, None,
                                      ctypes.byref(p)) == nk.INVALID_PARAMS
    assert lib.nk_moe_pipeline_create(ctypes.byref(s), 0, nk.F32, None, None, None,
                                      ctypes.byref(p)) == nk.INVALID_ROW_COUNT
    assert lib.nk_moe_pipeline_create(ctypes.byref(s), 4, 9, None, None, None,
                                      ctypes.byref(p)) == nk.UNSUPPORTED
    assert lib.nk_moe_pipeline_create(ctypes.byref(s), 4, nk.F32, 16, None, None,
                                      ctypes.byref(p)) == nk.INVALID_PARAMS  # some streams, not all
    assert p.value is None
    assert lib.nk_moe_pipeline_submit(None, None, 4, None, None) == nk.INVALID_PARAMS
    assert lib.nk_moe_pipeline_wait(None) == nk.INVALID_PARAMS
    assert lib.nk_moe_pipeline_destroy(None) == nk.OK


def test_mamba_glue_validation_order():
    lib = nk.lib()
    # conv1d.rs:126-158: shape, then input, weights, output lengths
    assert lib.nk_conv1d(None, 0, None, 0, 1, 0, 1, None, 0, None) == nk.INVALID_SHAPE
    assert lib.nk_conv1d(None, 1, None, 2, 2, 1, 2, None, 2, None) == nk.LENGTH_MISMATCH
    assert (err().argument, err().expected, err().actual) == (b"input", 2, 1)
    assert lib.nk_conv1d(None, 2, None, 1, 2, 1, 2, None, 2, None) == nk.LENGTH_MISMATCH
    assert err().argument == b"weights"
    assert lib.nk_conv1d(None, 2, None, 2, 2, 1, 2, None, 1, None) == nk.LENGTH_MISMATCH
    assert err().argument == b"output"
    # ssm.rs:177-245: shape (seq 0 is invalid here), then input .. final_state
    z = [None, 0]
    assert lib.nk_selective_scan(*z * 7, 0.0, 0, 0, 1, 1, None, 0, None, 1, None) \
        == nk.INVALID_SHAPE
    lens = [1, 1, 1, 0, 1]  # b is short
    args = []
    for n in lens:
        args += [None, n]
    args += [None, 0, None, 0]  # d, initial_state absent
    assert lib.nk_selective_scan(*args, 0.0, 0, 1, 1, 1, None, 1, None, 1, None) \
        == nk.LENGTH_MISMATCH
    assert (err().argument, err().expected, err().actual) == (b"b", 1, 0)
    # rms_norm.rs:146-183 then :108-115: empty, weight, gate, output, epsilon
    assert lib.nk_rms_norm(None, 0, None, 0, None, 0, 1e-5, None, 0, None) == nk.EMPTY_INPUT
    assert lib.nk_rms_norm(None, 2, None, 1, None, 0, 1e-5, None, 2, None) == nk.LENGTH_MISMATCH
    assert (err().argument, err().expected, err().actual) == (b"weight", 2, 1)
    g = ctypes.c_void_p(16)  # non-NULL gate: only its length is read
    assert lib.nk_rms_norm(None, 2, None, 2, g, 1, 1e-5, None, 2, None) == nk.LENGTH_MISMATCH
    assert err().argument == b"gate"
    assert lib.nk_rms_norm(None, 2, None, 2, None, 0, -1.0, None, 2, None) \
        == nk.NEGATIVE_EPSILON
    assert err().value == -1.0
