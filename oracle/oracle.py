"""oracle.py — numpy binding of the CPU parity oracle (nk_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm, never by the product.  Builds
oracle/_build/liboracle.so on first use if it is missing (gcc only).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(_HERE, "_build", "liboracle.so")

SIGMOID, SOFTMAX, SIGMOID_RENORM = 0, 1, 2
ERR_NAMES = {0: "Ok", 1: "InvalidShape", 2: "LengthMismatch", 3: "InvalidParams",
             4: "Int4OutOfRange", 5: "NonFiniteInput", 6: "InvalidRowCount"}


class OrcError(ctypes.Structure):
    _fields_ = [("code", ctypes.c_int), ("argument", ctypes.c_char_p),
                ("expected", ctypes.c_uint64), ("actual", ctypes.c_uint64),
                ("index", ctypes.c_uint64), ("value", ctypes.c_float),
                ("byte_value", ctypes.c_uint32)]


class OracleError(Exception):
    def __init__(self, e: OrcError):
        self.code = e.code
        self.variant = ERR_NAMES.get(e.code, str(e.code))
        self.argument = e.argument.decode() if e.argument else ""
        self.expected, self.actual = int(e.expected), int(e.actual)
        self.index, self.value, self.byte_value = int(e.index), float(e.value), int(e.byte_value)
        super().__init__(f"{self.variant} {self.argument} {self.expected} {self.actual}")


_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        _lib = ctypes.CDLL(LIB)
        _lib.orc_sigmoid.restype = ctypes.c_float
        _lib.orc_sigmoid.argtypes = [ctypes.c_float]
        _lib.orc_relu2.restype = ctypes.c_float
        _lib.orc_relu2.argtypes = [ctypes.c_float]
        _lib.orc_quantize_int4.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_float,
                                           ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t,
                                           ctypes.c_void_p]
        _lib.orc_dequantize_int4.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
                                             ctypes.c_float, ctypes.c_uint32, ctypes.c_void_p,
                                             ctypes.c_size_t, ctypes.c_void_p]
        _lib.orc_validate_int4_params.argtypes = [ctypes.c_float, ctypes.c_uint32, ctypes.c_void_p]
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _check(rc, err):
    if rc != 0:
        raise OracleError(err)


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def gemm(lhs, rhs, m, k, n, out_len=None, lhs_len=None, rhs_len=None):
    """gemm_host (gemm.rs:84-112): row-major f32, f64 accumulation."""
    lhs, rhs = _f32(lhs), _f32(rhs)
    out_len = m * n if out_len is None else out_len
    out = np.zeros(max(out_len, 1), np.float32)
    err = OrcError()
    rc = lib().orc_gemm(_p(lhs), ctypes.c_size_t(lhs.size if lhs_len is None else lhs_len),
                        _p(rhs), ctypes.c_size_t(rhs.size if rhs_len is None else rhs_len),
                        ctypes.c_size_t(m), ctypes.c_size_t(k), ctypes.c_size_t(n), _p(out),
                        ctypes.c_size_t(out_len), ctypes.byref(err))
    _check(rc, err)
    return out[:out_len]


def gemm_rows(lhs, rhs, m, k, n, rows, threads=1):
    lhs, rhs = _f32(lhs), _f32(rhs)
    out = np.zeros(rows * n, np.float32)
    lib().orc_gemm_rows(_p(lhs), _p(rhs), ctypes.c_size_t(m), ctypes.c_size_t(k),
                        ctypes.c_size_t(n), ctypes.c_size_t(rows), _p(out), ctypes.c_int(threads))
    return out


def pack_int4(values, packed_len=None):
    v = np.ascontiguousarray(values, dtype=np.uint8)
    packed_len = (v.size + 1) // 2 if packed_len is None else packed_len
    out = np.zeros(max(packed_len, 1), np.uint8)
    err = OrcError()
    rc = lib().orc_pack_int4(_p(v), ctypes.c_size_t(v.size), _p(out), ctypes.c_size_t(packed_len),
                             ctypes.byref(err))
    _check(rc, err)
    return out[:packed_len]


def unpack_int4(packed, count, out_len=None):
    pk = np.ascontiguousarray(packed, dtype=np.uint8)
    out_len = count if out_len is None else out_len
    out = np.zeros(max(out_len, 1), np.uint8)
    err = OrcError()
    rc = lib().orc_unpack_int4(_p(pk), ctypes.c_size_t(pk.size), ctypes.c_size_t(count), _p(out),
                               ctypes.c_size_t(out_len), ctypes.byref(err))
    _check(rc, err)
    return out[:out_len]


def quantize_int4(values, scale, zero_point, packed_len=None):
    v = _f32(values)
    packed_len = (v.size + 1) // 2 if packed_len is None else packed_len
    out = np.zeros(max(packed_len, 1), np.uint8)
    err = OrcError()
    rc = lib().orc_quantize_int4(_p(v), v.size, scale, zero_point, _p(out), packed_len,
                                 ctypes.byref(err))
    _check(rc, err)
    return out[:packed_len]


def dequantize_int4(packed, count, scale, zero_point, out_len=None):
    pk = np.ascontiguousarray(packed, dtype=np.uint8)
    out_len = count if out_len is None else out_len
    out = np.zeros(max(out_len, 1), np.float32)
    err = OrcError()
    rc = lib().orc_dequantize_int4(_p(pk), pk.size, count, scale, zero_point, _p(out), out_len,
                                   ctypes.byref(err))
    _check(rc, err)
    return out[:out_len]


def validate_int4_params(scale, zero_point):
    err = OrcError()
    _check(lib().orc_validate_int4_params(scale, zero_point, ctypes.byref(err)), err)


def quantize_int8_row(w):
    w = _f32(w)
    n, k = w.shape
    q = np.zeros((n, k), np.int8)
    s = np.zeros(n, np.float32)
    err = OrcError()
    rc = lib().orc_quantize_int8_row(_p(w), ctypes.c_size_t(n), ctypes.c_size_t(k), _p(q), _p(s),
                                     ctypes.byref(err))
    _check(rc, err)
    return q, s


def route(scores, tokens, experts, top_k, mode=SIGMOID, scores_len=None, indices_len=None,
          weights_len=None):
    s = _f32(np.asarray(scores).reshape(-1)) if np.asarray(scores).size else np.zeros(1, np.float32)
    scores_len = np.asarray(scores).size if scores_len is None else scores_len
    rl = tokens * top_k
    il = rl if indices_len is None else indices_len
    wl = rl if weights_len is None else weights_len
    idx = np.zeros(max(il, 1), np.int32)
    w = np.zeros(max(wl, 1), np.float32)
    err = OrcError()
    rc = lib().orc_route(_p(s), ctypes.c_size_t(scores_len), ctypes.c_size_t(tokens),
                         ctypes.c_size_t(experts), ctypes.c_size_t(top_k), ctypes.c_int(mode),
                         _p(idx), ctypes.c_size_t(il), _p(w), ctypes.c_size_t(wl),
                         ctypes.byref(err))
    _check(rc, err)
    return idx[:il], w[:wl]


def route_histogram(indices, tokens, top_k, experts):
    idx = np.ascontiguousarray(indices, dtype=np.int32)
    counts = np.zeros(experts, np.int32)
    offs = np.zeros(experts, np.int32)
    perm = np.zeros(max(tokens * top_k, 1), np.int32)
    lib().orc_route_histogram(_p(idx), ctypes.c_size_t(tokens), ctypes.c_size_t(top_k),
                              ctypes.c_size_t(experts), _p(counts), _p(offs), _p(perm))
    return counts, offs, perm[: tokens * top_k]


def linear(w, bias, input_dim, output_dim, x, rows):
    """LinearProjection::project (linear.rs:273-342); w is [input_dim, output_dim]."""
    w, bias, x = _f32(w), _f32(bias), _f32(x)
    out = np.zeros(max(rows * output_dim, 1), np.float32)
    err = OrcError()
    rc = lib().orc_linear(_p(w), _p(bias), ctypes.c_size_t(input_dim), ctypes.c_size_t(output_dim),
                          _p(x), ctypes.c_size_t(x.size), ctypes.c_size_t(rows), _p(out),
                          ctypes.c_size_t(rows * output_dim), ctypes.byref(err))
    _check(rc, err)
    return out[: rows * output_dim]


def mlp(hidden, inter, up_w, up_b, down_w, down_b, x, rows):
    up_w, up_b, down_w, down_b, x = map(_f32, (up_w, up_b, down_w, down_b, x))
    out = np.zeros(rows * hidden, np.float32)
    err = OrcError()
    rc = lib().orc_mlp(ctypes.c_size_t(hidden), ctypes.c_size_t(inter), _p(up_w), _p(up_b),
                       _p(down_w), _p(down_b), _p(x), ctypes.c_size_t(rows), _p(out),
                       ctypes.byref(err))
    _check(rc, err)
    return out


def moe(hidden, experts, top_k, inter, shared_inter, router_w, router_b, up_w, up_b, down_w,
        down_b, sh_up_w, sh_up_b, sh_down_w, sh_down_b, x, rows, mode=SIGMOID):
    """MoeLayer::forward (moe.rs:148-249).  Weights in the reference [in, out] layout;
    expert tensors stacked: up_w [E, H, I], down_w [E, I, H]."""
    args = [_f32(a) for a in (router_w, router_b, up_w, up_b, down_w, down_b, sh_up_w, sh_up_b,
                              sh_down_w, sh_down_b, x)]
    out = np.zeros(rows * hidden, np.float32)
    idx = np.zeros(rows * top_k, np.int32)
    w = np.zeros(rows * top_k, np.float32)
    err = OrcError()
    rc = lib().orc_moe(ctypes.c_size_t(hidden), ctypes.c_size_t(experts), ctypes.c_size_t(top_k),
                       ctypes.c_size_t(inter), ctypes.c_size_t(shared_inter),
                       *[_p(a) for a in args[:10]], ctypes.c_int(mode), _p(args[10]),
                       ctypes.c_size_t(rows), _p(out), _p(idx), _p(w), ctypes.byref(err))
    _check(rc, err)
    return out, idx, w


def sigmoid(x: float) -> float:
    return lib().orc_sigmoid(x)


def relu2(x: float) -> float:
    return lib().orc_relu2(x)
