"""nk.py — Python binding of libnk's C ABI (include/nk.h) over ctypes.

Device memory, streams and process groups come from PyTorch; every compute
call goes through libnk.so (sm_100a kernels).  There is no CPU path: when
libnk.so is missing or no GPU is present, calls raise.

The wrappers mirror the reference's kernel-wrapper API
(nemotron-kernels/src/{gemm,quantize,moe_routing}.rs): same argument order
and the same error variants, raised as NkError with the variant's payload.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("NK_LIB_PATH") or os.path.join(_HERE, "libnk.so")

# status codes (nk.h)
OK, INVALID_SHAPE, LENGTH_MISMATCH, INVALID_PARAMS, INT4_OUT_OF_RANGE = 0, 1, 2, 3, 4
NON_FINITE_INPUT, INVALID_ROW_COUNT, UNSUPPORTED, DEVICE_ERROR, TIMEOUT = 5, 6, 7, 8, 9
WORKSPACE_TOO_SMALL, INVALID_DELTA_T, EMPTY_INPUT, NEGATIVE_EPSILON = 10, 11, 12, 13
HEAD_COUNT_MISMATCH, INVALID_SCALE, NO_VALID_TARGETS, ZERO_PARTITION = 14, 15, 16, 17
TOKEN_OUT_OF_RANGE = 18
STATUS_NAMES = {
    0: "Ok", 1: "InvalidShape", 2: "LengthMismatch", 3: "InvalidParams",
    4: "Int4OutOfRange", 5: "NonFiniteInput", 6: "InvalidRowCount", 7: "Unsupported",
    8: "DeviceError", 9: "Timeout", 10: "WorkspaceTooSmall", 11: "InvalidDeltaT",
    12: "EmptyInput", 13: "NegativeEpsilon", 14: "HeadCountMismatch", 15: "InvalidScale",
    16: "NoValidAttentionTargets", 17: "ZeroPartition", 18: "TokenOutOfRange",
}
F32, BF16 = 0, 1
EPI_RELU2 = 1
ROUTE_SIGMOID, ROUTE_SOFTMAX, ROUTE_SIGMOID_RENORM = 0, 1, 2
W_BF16, W_INT8_ROW, W_INT4_AFFINE = 0, 1, 2

_c = ctypes
_sz = _c.c_size_t
_i64 = _c.c_int64
_i32 = _c.c_int32
_u32 = _c.c_uint32
_p = _c.c_void_p
_f = _c.c_float


class NkErrorInfo(_c.Structure):
    _fields_ = [
        ("code", _c.c_int32),
        ("argument", _c.c_char * 32),
        ("expected", _c.c_uint64),
        ("actual", _c.c_uint64),
        ("index", _c.c_uint64),
        ("value", _c.c_float),
        ("byte_value", _c.c_uint32),
        ("message", _c.c_char * 256),
    ]


class NkMoeLayer(_c.Structure):
    _fields_ = [
        ("hidden", _i64), ("experts", _i64), ("top_k", _i64), ("inter", _i64),
        ("shared_inter", _i64), ("route_mode", _i32), ("weight_kind", _i32),
        ("router_w3", _p), ("router_b", _p),
        ("up_w", _p), ("up_scale", _p), ("up_b", _p),
        ("down_w", _p), ("down_scale", _p), ("down_b", _p),
        ("shared_up_w", _p), ("shared_up_scale", _p), ("shared_up_b", _p),
        ("shared_down_w", _p), ("shared_down_scale", _p), ("shared_down_b", _p),
        ("up_zero_point", _p), ("down_zero_point", _p),
        ("shared_up_zero_point", _p), ("shared_down_zero_point", _p),
        ("router_norms", _p),
    ]


class NkConvArgs(_c.Structure):
    _fields_ = [
        ("batch", _i64), ("seq", _i64), ("channels", _i64), ("kernel_size", _i64),
        ("x", _p), ("ld_x", _i64), ("weights", _p), ("prefix", _p), ("silu", _i32),
        ("y", _p), ("ld_y", _i64), ("state_out", _p), ("f32_accumulate", _i32),
    ]


class NkScanArgs(_c.Structure):
    _fields_ = [
        ("batch", _i64), ("seq", _i64), ("channels", _i64), ("states", _i64),
        ("x", _p), ("ld_x", _i64),
        ("dt", _p), ("ld_dt", _i64), ("dt_group", _i32),
        ("a", _p), ("a_group", _i32), ("a_per_state", _i32),
        ("b", _p), ("c", _p), ("ld_bc", _i64), ("bc_group", _i32),
        ("d", _p), ("d_group", _i32),
        ("initial_state", _p),
        ("delta_bias", _f), ("softplus", _i32),
        ("y", _p), ("ld_y", _i64),
        ("final_state", _p),
        ("check_delta_t", _i32),
    ]


class NkError(Exception):
    """A libnk status other than NK_OK, with the matching Rust variant's payload."""

    def __init__(self, info: NkErrorInfo):
        self.code = int(info.code)
        self.variant = STATUS_NAMES.get(self.code, str(self.code))
        self.argument = info.argument.decode()
        self.expected = int(info.expected)
        self.actual = int(info.actual)
        self.index = int(info.index)
        self.value = float(info.value)
        self.byte_value = int(info.byte_value)
        self.message = info.message.decode(errors="replace")
        super().__init__(f"{self.variant}: {self.message}")


# name -> (restype, argtypes)
_SIGS = {
    "nk_last_error": (_i32, [_p]),
    "nk_version": (_i32, []),
    "nk_device_status": (_i32, [_p]),
    "nk_gemm_f32": (_i32, [_p, _sz, _p, _sz, _p, _sz, _sz, _sz, _sz, _p]),
    "nk_gemm_bf16": (_i32, [_p, _i32, _p, _p, _p, _i32, _i64, _i64, _i64, _i32, _p]),
    "nk_gemm_w8row": (_i32, [_p, _i32, _p, _p, _p, _p, _i32, _i64, _i64, _i64, _i32, _p]),
    "nk_gemm_w8row_f32_static": (_i32, [_p, _p, _p, _p, _p, _i32, _i64, _i64, _i64, _i32, _p]),
    "nk_gemm_w4a": (_i32, [_p, _i32, _p, _sz, _f, _u32, _p, _p, _i32, _i64, _i64, _i64, _i32, _p]),
    "nk_gemm_workspace_bytes": (_i32, [_i32, _i32, _i64, _i64, _i64, _p]),
    "nk_gemm_bf16_ws": (_i32, [_p, _i32, _p, _p, _p, _i32, _i64, _i64, _i64, _i32, _p, _sz, _p]),
    "nk_gemm_w8row_ws": (_i32, [_p, _i32, _p, _p, _p, _p, _i32, _i64, _i64, _i64, _i32, _p, _sz,
                                _p]),
    "nk_gemm_w4a_ws": (_i32, [_p, _i32, _p, _sz, _f, _u32, _p, _p, _i32, _i64, _i64, _i64, _i32,
                              _p, _sz, _p]),
    "nk_scratch_release": (_i32, [_p]),
    "nk_ep_handle_bytes": (_sz, []),
    "nk_ep_create": (_i32, [_i32, _i32, _i64, _i64, _i64, _i64, _i64, _p, _p]),
    "nk_ep_connect": (_i32, [_p, _p]),
    "nk_moe_forward_ep_workspace_bytes": (_i32, [_p, _p, _p, _i64, _p]),
    "nk_moe_forward_ep": (_i32, [_p, _p, _p, _p, _i64, _p, _i32, _p, _p, _p, _sz, _p]),
    "nk_ep_barrier": (_i32, [_p, _p]),
    "nk_ep_received_rows": (_i32, [_p, _p]),
    "nk_ep_destroy": (_i32, [_p]),
    "nk_pack_int4": (_i32, [_p, _sz, _p, _sz, _p]),
    "nk_unpack_int4": (_i32, [_p, _sz, _sz, _p, _sz, _p]),
    "nk_quantize_int4": (_i32, [_p, _sz, _f, _u32, _p, _sz, _p]),
    "nk_int4_kn_to_nk": (_i32, [_p, _i64, _i64, _i64, _p, _p]),
    "nk_router_norms": (_i32, [_p, _i64, _i64, _p, _p]),
    "nk_dequantize_int4": (_i32, [_p, _sz, _sz, _f, _u32, _p, _sz, _p]),
    "nk_validate_int4_params": (_i32, [_f, _u32]),
    "nk_quantize_int8_row": (_i32, [_p, _i64, _i64, _p, _p, _p]),
    "nk_moe_route": (_i32, [_p, _sz, _sz, _sz, _sz, _i32, _p, _sz, _p, _sz, _p]),
    "nk_moe_plan": (_i32, [_p, _i64, _i64, _i64, _p, _p, _p, _p, _p]),
    "nk_router_split": (_i32, [_p, _i64, _i64, _p, _p]),
    "nk_linear_pack_kn": (_i32, [_p, _i64, _i64, _p, _p]),
    "nk_moe_workspace_bytes": (_i32, [_p, _i64, _p]),
    "nk_moe_forward": (_i32, [_p, _p, _i64, _p, _i32, _p, _p, _p, _sz, _p]),
    "nk_selftest_wait_timeout": (_i32, [_p]),
    "nk_moe_pipeline_create": (_i32, [_p, _i64, _i32, _p, _p, _p, _p]),
    "nk_moe_pipeline_submit": (_i32, [_p, _p, _i64, _p, _p]),
    "nk_moe_pipeline_wait": (_i32, [_p]),
    "nk_moe_pipeline_destroy": (_i32, [_p]),
    "nk_moe_dispatch_workspace_bytes": (_i32, [_p, _i64, _p]),
    "nk_moe_dispatch": (_i32, [_p, _p, _i64, _p, _p, _p, _p, _p, _p, _p, _sz, _p]),
    "nk_moe_experts_workspace_bytes": (_i32, [_p, _i64, _i32, _p]),
    "nk_moe_experts": (_i32, [_p, _p, _i64, _p, _p, _i32, _p, _p, _sz, _p]),
    "nk_moe_shared": (_i32, [_p, _p, _i64, _p, _p, _p]),
    "nk_moe_combine": (_i32, [_p, _p, _p, _p, _i64, _i64, _i64, _p, _i32, _p]),
    "nk_ipc_alloc": (_i32, [_sz, _p, _p]),
    "nk_ipc_open": (_i32, [_p, _p]),
    "nk_ipc_close": (_i32, [_p]),
    "nk_ipc_free": (_i32, [_p]),
    "nk_ep_plan": (_i32, [_p, _i32, _i32, _i32, _p, _p, _p, _p, _p, _p]),
    "nk_ep_dispatch": (_i32, [_p, _i64, _i64, _i32, _p, _p, _p, _p, _i32, _p, _p]),
    "nk_ep_return": (_i32, [_p, _i64, _i32, _i32, _p, _p, _p, _p, _p]),
    "nk_ep_plan_phased": (_i32, [_p, _i32, _i32, _i32, _i32, _i64, _p, _p, _p, _p, _p, _p]),
    "nk_ep_dispatch_phase": (_i32, [_p, _i64, _i64, _i32, _p, _p, _p, _p, _i32, _i32, _i32, _p,
                                    _p]),
    "nk_ep_return_segments": (_i32, [_p, _i64, _i32, _i32, _i32, _i32, _p, _p, _p, _p, _p]),
    "nk_conv1d": (_i32, [_p, _sz, _p, _sz, _i64, _i64, _i64, _p, _sz, _p]),
    "nk_conv1d_ex": (_i32, [_p, _p]),
    "nk_selective_scan": (_i32, [_p, _sz, _p, _sz, _p, _sz, _p, _sz, _p, _sz, _p, _sz, _p, _sz,
                                 _f, _i32, _i64, _i64, _i64, _p, _sz, _p, _sz, _p]),
    "nk_selective_scan_ex": (_i32, [_p, _p]),
    "nk_rms_norm": (_i32, [_p, _sz, _p, _sz, _p, _sz, _f, _p, _sz, _p]),
    "nk_rms_norm_rows": (_i32, [_p, _i64, _i64, _i64, _p, _sz, _p, _i64, _f, _p, _i64, _i32,
                                _p]),
    "nk_row_sumsq": (_i32, [_p, _i64, _i64, _i64, _p, _p]),
    "nk_rms_norm_rows_presummed": (_i32, [_p, _i64, _i64, _i64, _p, _sz, _p, _i64, _p, _i64,
                                          _f, _p, _i64, _i32, _p]),
    "nk_attention_f32": (_i32, [_p, _sz, _p, _sz, _p, _sz, _i64, _i64, _i64, _i64, _i64, _i64,
                                _i32, _i64, _i32, _f, _p, _sz, _p]),
    "nk_kv_append": (_i32, [_p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p, _p]),
    "nk_attention_workspace_bytes": (_i32, [_i64, _i64, _i64, _i64, _i64, _i64, _i64, _p]),
    "nk_attention_gqa": (_i32, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i32,
                                _i64, _i32, _f, _p, _i32, _p, _sz, _p]),
    "nk_attention_check": (_i32, [_p, _p, _p]),
    "nk_embedding_lookup": (_i32, [_p, _i32, _sz, _p, _i64, _i64, _i64, _p, _i32, _sz, _i32, _p]),
    "nk_add_rms_norm_rows": (_i32, [_p, _p, _i64, _i64, _p, _sz, _f, _p, _p, _i32, _p]),
    "nk_argmax_rows": (_i32, [_p, _i32, _i64, _i64, _i64, _p, _p]),
    "nk_set_stage_timing": (_i32, [_i32]),
    "nk_moe_stage_times": (_i32, [_p, _i32, _p]),
}
MOE_STAGES = ("router", "route_plan", "gather", "up_proj", "down_proj", "shared_expert",
              "combine")


def set_stage_timing(enable: bool) -> None:
    call("nk_set_stage_timing", 1 if enable else 0)


def moe_stage_times() -> dict:
    """Per-stage milliseconds of this thread's last nk_moe_forward (see nk.h)."""
    arr = (ctypes.c_float * len(MOE_STAGES))()
    n = ctypes.c_int32(0)
    call("nk_moe_stage_times", arr, len(MOE_STAGES), ctypes.byref(n))
    return {MOE_STAGES[i]: float(arr[i]) for i in range(n.value)}

_lib = None


def lib() -> ctypes.CDLL:
    """Loads libnk.so (built in-tree by `make -C nemotron-cutile-rs_b200`)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libnk.so not built: {LIB_PATH} (run make -C {_HERE})")
        h = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


def last_error() -> NkErrorInfo:
    info = NkErrorInfo()
    lib().nk_last_error(ctypes.byref(info))
    return info


def check(status: int) -> None:
    if status != OK:
        raise NkError(last_error())


def call(name: str, *args) -> None:
    """Calls an nk_* entry point and raises NkError on a non-OK status."""
    check(getattr(lib(), name)(*args))


# ----------------------------------------------------------------- torch glue
def ptr(t) -> int | None:
    """Device address of a tensor (None for None)."""
    return None if t is None else t.data_ptr()


def stream_ptr(stream=None) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("libnk entry points take device tensors")


# ------------------------------------------------------------ kernel wrappers
def gemm_f32(lhs, rhs, m: int, k: int, n: int, out=None, stream=None):
    """nemotron_kernels::gemm::gemm / gemm_into (gemm.rs:318-363)."""
    import torch

    _require_cuda(lhs, rhs, out)
    if out is None:
        out = torch.empty(m * n if m * n > 0 else 1, dtype=torch.float32, device=lhs.device)
        out_len = m * n
    else:
        out_len = out.numel()
    call("nk_gemm_f32", ptr(lhs), lhs.numel(), ptr(rhs), rhs.numel(), ptr(out), out_len,
         m, k, n, stream_ptr(stream))
    return out


def gemm_workspace_bytes(kind: str, x_dtype, m: int, k: int, n: int) -> int:
    """nk_gemm_workspace_bytes: scratch the *_ws projections need for this shape."""
    import torch

    wk = {"bf16": W_BF16, "int8": W_INT8_ROW, "int4": W_INT4_AFFINE}[kind]
    b = ctypes.c_size_t(0)
    call("nk_gemm_workspace_bytes", wk, F32 if x_dtype == torch.float32 else BF16, m, k, n,
         ctypes.byref(b))
    return b.value


def gemm(x, w, *, kind: str = "bf16", bias=None, scales=None, scale: float = 1.0,
         zero_point: int = 0, n: int | None = None, out_dtype=None, relu2: bool = False,
         stream=None, workspace=None):
    """Projection Y[M,N] = X[M,K]·Wᵀ (+bias) (relu2) — LinearProjection::project_into.

    kind: "bf16" (w bf16 [N,K]), "int8" (w int8 [N,K], scales f32 [N]),
    "int4" (w uint8 packed reference layout [K,N], scale/zero_point).
    workspace: optional uint8 device tensor of >= gemm_workspace_bytes (the
    *_ws entry points); by default the library's per-stream scratch.
    """
    import torch

    _require_cuda(x, w, bias, scales)
    m, k = x.shape
    x_dtype = F32 if x.dtype == torch.float32 else BF16
    if kind == "int4":
        assert n is not None
    else:
        n = w.shape[0]
    out_dtype = out_dtype or torch.float32
    y = torch.empty((m, n), dtype=out_dtype, device=x.device)
    y_dtype = F32 if out_dtype == torch.float32 else BF16
    flags = EPI_RELU2 if relu2 else 0
    s = stream_ptr(stream)
    if workspace is not None:
        wsp, wsn = ptr(workspace), workspace.numel()
        if kind == "bf16":
            call("nk_gemm_bf16_ws", ptr(x), x_dtype, ptr(w), ptr(bias), ptr(y), y_dtype, m, k, n,
                 flags, wsp, wsn, s)
        elif kind == "int8":
            call("nk_gemm_w8row_ws", ptr(x), x_dtype, ptr(w), ptr(scales), ptr(bias), ptr(y),
                 y_dtype, m, k, n, flags, wsp, wsn, s)
        elif kind == "int4":
            call("nk_gemm_w4a_ws", ptr(x), x_dtype, ptr(w), w.numel(), float(scale),
                 int(zero_point), ptr(bias), ptr(y), y_dtype, m, k, n, flags, wsp, wsn, s)
        else:
            raise ValueError(kind)
        return y
    if kind == "bf16":
        call("nk_gemm_bf16", ptr(x), x_dtype, ptr(w), ptr(bias), ptr(y), y_dtype, m, k, n, flags, s)
    elif kind == "int8":
        call("nk_gemm_w8row", ptr(x), x_dtype, ptr(w), ptr(scales), ptr(bias), ptr(y), y_dtype,
             m, k, n, flags, s)
    elif kind == "int4":
        call("nk_gemm_w4a", ptr(x), x_dtype, ptr(w), w.numel(), float(scale), int(zero_point),
             ptr(bias), ptr(y), y_dtype, m, k, n, flags, s)
    else:
        raise ValueError(kind)
    return y


def moe_route(scores, tokens: int, experts: int, top_k: int, mode: int = ROUTE_SIGMOID,
              stream=None):
    """moe_routing::moe_route / moe_route_softmax (moe_routing.rs:499-532)."""
    import torch

    _require_cuda(scores)
    dev = scores.device
    n = max(tokens * top_k, 1)  # placeholder storage when the batch is empty
    idx = torch.empty(n, dtype=torch.int32, device=dev)
    w = torch.empty(n, dtype=torch.float32, device=dev)
    call("nk_moe_route", ptr(scores), scores.numel(), tokens, experts, top_k, mode, ptr(idx),
         tokens * top_k, ptr(w), tokens * top_k, stream_ptr(stream))
    return idx[: tokens * top_k], w[: tokens * top_k]


def moe_plan(indices, tokens: int, top_k: int, experts: int, stream=None):
    import torch

    dev = indices.device
    slots = tokens * top_k
    counts = torch.empty(experts, dtype=torch.int32, device=dev)
    offsets = torch.empty(experts + 1, dtype=torch.int32, device=dev)
    perm = torch.empty(max(slots, 1), dtype=torch.int32, device=dev)
    pos = torch.empty(max(slots, 1), dtype=torch.int32, device=dev)
    call("nk_moe_plan", ptr(indices), tokens, top_k, experts, ptr(counts), ptr(offsets),
         ptr(perm), ptr(pos), stream_ptr(stream))
    return counts, offsets, perm[:slots], pos[:slots]


def quantize_int8_row(w, stream=None):
    import torch

    n, k = w.shape
    q = torch.empty((n, k), dtype=torch.int8, device=w.device)
    s = torch.empty(n, dtype=torch.float32, device=w.device)
    call("nk_quantize_int8_row", ptr(w), n, k, ptr(q), ptr(s), stream_ptr(stream))
    return q, s


def quantize_int4_experts(w, zero_point: int = 8, stream=None):
    """Expert weights w [E, N, K] (output-major, any float dtype) in the
    reference's INT4-affine format, one per-tensor (scale, zero_point) per
    expert: scale = max|W_e| / 7 as the benchmark configurations state, codes
    from nk_quantize_int4 (quantize.rs:131-144) on W_eᵀ in the reference's
    [K, N] = [input_dim, output_dim] layout.  Returns (codes [E, N, K/2] uint8
    feature-major for NK_W_INT4_AFFINE, scales f32 [E], zero points uint8 [E],
    reference packed bytes [E, ceil(K*N/2)])."""
    import torch

    e, n, k = w.shape
    wf = w.float()
    scales = (wf.abs().amax(dim=(1, 2)) / 7.0).to(torch.float32)
    kn_len = (k * n + 1) // 2
    packed = torch.empty((e, kn_len), dtype=torch.uint8, device=w.device)
    sc = scales.cpu().tolist()
    for i in range(e):
        t = wf[i].t().contiguous()  # [K, N]
        call("nk_quantize_int4", ptr(t), k * n, float(sc[i]), zero_point, ptr(packed[i]), kn_len,
             stream_ptr(stream))
    codes = torch.empty((e, n, k // 2), dtype=torch.uint8, device=w.device)
    call("nk_int4_kn_to_nk", ptr(packed), e, k, n, ptr(codes), stream_ptr(stream))
    zps = torch.full((e,), zero_point, dtype=torch.uint8, device=w.device)
    return codes, scales, zps, packed


def router_split(w, stream=None):
    import torch

    e, h = w.shape
    hp = (h + 63) // 64 * 64
    w3 = torch.empty((e, 3 * hp), dtype=torch.bfloat16, device=w.device)
    call("nk_router_split", ptr(w), e, h, ptr(w3), stream_ptr(stream))
    return w3


@dataclass
class MoeWeights:
    """Device tensors of one MoE layer in libnk's layouts (see nk_moe_layer)."""
    hidden: int
    experts: int
    top_k: int
    inter: int
    shared_inter: int
    route_mode: int
    weight_kind: int
    router_w3: object
    router_b: object = None
    up_w: object = None
    up_scale: object = None
    up_b: object = None
    down_w: object = None
    down_scale: object = None
    down_b: object = None
    shared_up_w: object = None
    shared_up_scale: object = None
    shared_up_b: object = None
    shared_down_w: object = None
    shared_down_scale: object = None
    shared_down_b: object = None
    up_zero_point: object = None          # INT4_AFFINE: uint8 [E]
    down_zero_point: object = None
    shared_up_zero_point: object = None   # uint8 [1]
    shared_down_zero_point: object = None
    router_norms: object = None           # f32 [2E] (nk_router_norms), or computed per call

    def struct(self) -> NkMoeLayer:
        s = NkMoeLayer()
        for f in ("hidden", "experts", "top_k", "inter", "shared_inter", "route_mode",
                  "weight_kind"):
            setattr(s, f, getattr(self, f))
        for f in ("router_w3", "router_b", "up_w", "up_scale", "up_b", "down_w", "down_scale",
                  "down_b", "shared_up_w", "shared_up_scale", "shared_up_b", "shared_down_w",
                  "shared_down_scale", "shared_down_b", "up_zero_point", "down_zero_point",
                  "shared_up_zero_point", "shared_down_zero_point", "router_norms"):
            setattr(s, f, ptr(getattr(self, f)))
        return s


def ensure_router_norms(weights: MoeWeights) -> None:
    """Fills weights.router_norms once (nk_router_norms) so that forwards skip it."""
    import torch

    if weights.router_norms is None and weights.router_w3 is not None:
        weights.router_norms = torch.empty(2 * weights.experts, dtype=torch.float32,
                                           device=weights.router_w3.device)
        call("nk_router_norms", ptr(weights.router_w3), weights.experts, weights.hidden,
             ptr(weights.router_norms), stream_ptr())


class MoeLayer:
    """Device MoE layer: MoeLayer::forward_into (nemotron-nn/src/moe.rs:154-249)."""

    def __init__(self, weights: MoeWeights):
        ensure_router_norms(weights)
        self.weights = weights
        self._struct = weights.struct()
        self._ws = None

    def workspace_bytes(self, tokens: int) -> int:
        b = ctypes.c_size_t(0)
        call("nk_moe_workspace_bytes", ctypes.byref(self._struct), tokens, ctypes.byref(b))
        return b.value

    def forward(self, x, out=None, out_dtype=None, indices=None, weights=None, stream=None,
                workspace=None):
        """workspace: an optional uint8 device buffer shared by several layers
        (grown in place, as a one-element list [tensor]); by default the layer
        keeps its own."""
        import torch

        t = x.shape[0]
        need = self.workspace_bytes(t)
        if workspace is not None:
            if workspace[0] is None or workspace[0].numel() < need:
                workspace[0] = None
                workspace[0] = torch.empty(need, dtype=torch.uint8, device=x.device)
            self._ws = workspace[0]
        elif self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=x.device)
        if out is None:
            out = torch.empty((t, self.weights.hidden), dtype=out_dtype or torch.float32,
                              device=x.device)
        od = F32 if out.dtype == torch.float32 else BF16
        call("nk_moe_forward", ctypes.byref(self._struct), ptr(x), t, ptr(out), od, ptr(indices),
             ptr(weights), ptr(self._ws), self._ws.numel(), stream_ptr(stream))
        return out


class MoePipeline:
    """Host-buffer MoE forwards (nk_moe_pipeline_*): submit(x_host, out_host)
    copies x in, runs the layer and copies out, overlapping the copies of
    adjacent submissions with the forward in between.  x_host / out_host are
    CPU tensors (pinned for the copies to overlap); results are valid after
    wait().  streams: optional (h2d, compute, d2h) torch.cuda.Stream triple."""

    def __init__(self, layer: MoeLayer, max_tokens: int, out_dtype=None, streams=None):
        import torch

        self.layer = layer  # keeps the weights (and the layer struct) alive
        self.streams = streams
        od = BF16 if out_dtype == torch.bfloat16 else F32
        self.out_dtype = torch.bfloat16 if od == BF16 else torch.float32
        self.max_tokens = max_tokens
        h = ctypes.c_void_p()
        sp = [None, None, None] if streams is None else [s.cuda_stream for s in streams]
        call("nk_moe_pipeline_create", ctypes.byref(layer._struct), max_tokens, od, *sp,
             ctypes.byref(h))
        self._h = h

    def submit(self, x_host, out_host, indices_host=None):
        import torch

        for t in (x_host, out_host, indices_host):
            if t is not None and (t.is_cuda or not t.is_contiguous()):
                raise ValueError("host tensors must be contiguous CPU tensors")
        hidden, top_k = self.layer.weights.hidden, self.layer.weights.top_k
        if x_host.dtype != torch.bfloat16 or x_host.dim() != 2 or x_host.shape[1] != hidden:
            raise ValueError(f"x_host must be bf16 [tokens, {hidden}]")
        tokens = x_host.shape[0]
        if out_host.dtype != self.out_dtype or out_host.numel() < tokens * hidden:
            raise ValueError("out_host must hold tokens x hidden values of the pipeline's dtype")
        if indices_host is not None and (indices_host.dtype != torch.int32 or
                                         indices_host.numel() < tokens * top_k):
            raise ValueError("indices_host must hold tokens x top_k int32 values")
        call("nk_moe_pipeline_submit", self._h, x_host.data_ptr(), tokens, out_host.data_ptr(),
             None if indices_host is None else indices_host.data_ptr())

    def wait(self):
        call("nk_moe_pipeline_wait", self._h)

    def close(self):
        if self._h:
            call("nk_moe_pipeline_destroy", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def device_status(stream=None) -> None:
    call("nk_device_status", stream_ptr(stream))


# ------------------------------------------------------------- Mamba2 glue
def _numel(t) -> int:
    return 0 if t is None else t.numel()


def conv1d(inp, weights, seq: int, channels: int, kernel_size: int, out=None, stream=None):
    """depthwise_causal_conv1d (conv1d.rs:78-124, 325-345) on device f32 tensors."""
    import torch

    _require_cuda(inp, weights, out)
    if out is None:
        out = torch.empty(max(seq * channels, 1), dtype=torch.float32, device=inp.device)
        out_len = seq * channels
    else:
        out_len = out.numel()
    call("nk_conv1d", ptr(inp), inp.numel(), ptr(weights), weights.numel(), seq, channels,
         kernel_size, ptr(out), out_len, stream_ptr(stream))
    return out[:out_len]


def conv1d_ex(x, weights, batch: int, seq: int, channels: int, kernel_size: int, *,
              ld_x=None, prefix=None, silu=False, y=None, ld_y=None, state_out=None,
              f32_accumulate=False, stream=None):
    """Batched causal conv with conv-cache history and fused SiLU (mamba2.rs:276-312)."""
    import torch

    _require_cuda(x, weights, prefix, y, state_out)
    if y is None:
        y = torch.empty(batch * seq, channels, dtype=torch.float32, device=x.device)
        ld_y = channels
    a = NkConvArgs(batch, seq, channels, kernel_size, ptr(x), ld_x or channels, ptr(weights),
                   ptr(prefix), 1 if silu else 0, ptr(y), ld_y or channels, ptr(state_out),
                   1 if f32_accumulate else 0)
    call("nk_conv1d_ex", ctypes.byref(a), stream_ptr(stream))
    return y


def selective_scan(inp, delta_t, a, b, c, seq: int, channels: int, states: int, *, d=None,
                   initial_state=None, delta_bias: float = 0.0, softplus: bool = False,
                   out=None, final_state=None, stream=None):
    """selective_scan (ssm.rs:123-175, 614-624).  Returns (values, final_state)."""
    import torch

    _require_cuda(inp, delta_t, a, b, c, d, initial_state, out, final_state)
    dev = inp.device
    ol = seq * channels if out is None else out.numel()
    fl = channels * states if final_state is None else final_state.numel()
    if out is None:
        out = torch.empty(max(ol, 1), dtype=torch.float32, device=dev)
    if final_state is None:
        final_state = torch.empty(max(fl, 1), dtype=torch.float32, device=dev)
    call("nk_selective_scan", ptr(inp), inp.numel(), ptr(delta_t), delta_t.numel(), ptr(a),
         a.numel(), ptr(b), b.numel(), ptr(c), c.numel(), ptr(d), _numel(d),
         ptr(initial_state), _numel(initial_state), delta_bias, 1 if softplus else 0, seq,
         channels, states, ptr(out), ol, ptr(final_state), fl, stream_ptr(stream))
    return out[:ol], final_state[:fl]


def selective_scan_ex(args: NkScanArgs, stream=None) -> None:
    """Strided / shared-parameter scan (nk_selective_scan_ex); args hold device pointers."""
    call("nk_selective_scan_ex", ctypes.byref(args), stream_ptr(stream))


def rms_norm(inp, weight, epsilon: float, gate=None, out=None, stream=None):
    """rms_norm_into_host / gated_rms_norm_into_host (rms_norm.rs:64-106) on device."""
    import torch

    _require_cuda(inp, weight, gate, out)
    n = inp.numel()
    ol = n if out is None else out.numel()
    if out is None:
        out = torch.empty(max(n, 1), dtype=torch.float32, device=inp.device)
    call("nk_rms_norm", ptr(inp), n, ptr(weight), weight.numel(), ptr(gate), _numel(gate),
         epsilon, ptr(out), ol, stream_ptr(stream))
    return out[:ol]


def rms_norm_rows(x, weight, epsilon: float, gate=None, out_dtype: int = F32, out=None,
                  stream=None):
    """Row-wise (gated) RMSNorm (rms_norm.rs:291-360, mamba2.rs:567-586); x is [rows, width]
    (row stride taken from the tensor), gate likewise or None."""
    import torch

    _require_cuda(x, weight, gate, out)
    rows, width = x.shape
    if out is None:
        out = torch.empty(rows, width, device=x.device,
                          dtype=torch.bfloat16 if out_dtype == BF16 else torch.float32)
    call("nk_rms_norm_rows", ptr(x), rows, width, x.stride(0), ptr(weight), weight.numel(),
         ptr(gate), gate.stride(0) if gate is not None else 0, epsilon, ptr(out),
         out.stride(0), out_dtype, stream_ptr(stream))
    return out


def row_sumsq(x, out=None, stream=None):
    """f64 sum of squares of each row of x [rows, width] (nk_row_sumsq)."""
    import torch

    _require_cuda(x, out)
    rows, width = x.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.float64, device=x.device)
    call("nk_row_sumsq", ptr(x), rows, width, x.stride(0), ptr(out), stream_ptr(stream))
    return out


def rms_norm_rows_presummed(x, weight, epsilon: float, sumsq, total_width: int, gate=None,
                            out_dtype: int = F32, out=None, stream=None):
    """Row-wise (gated) RMSNorm of the local columns of rows split over ranks;
    sumsq [rows] f64 holds the full rows' sums of squares."""
    import torch

    _require_cuda(x, weight, gate, sumsq, out)
    rows, width = x.shape
    if out is None:
        out = torch.empty(rows, width, device=x.device,
                          dtype=torch.bfloat16 if out_dtype == BF16 else torch.float32)
    call("nk_rms_norm_rows_presummed", ptr(x), rows, width, x.stride(0), ptr(weight),
         weight.numel(), ptr(gate), gate.stride(0) if gate is not None else 0, ptr(sumsq),
         total_width, epsilon, ptr(out), out.stride(0), out_dtype, stream_ptr(stream))
    return out


# ------------------------------------------------------------ attention core
def attention_f32(q, k, v, batch, q_seq, kv_seq, q_heads, kv_heads, head_dim, *, causal=False,
                  q_offset=0, scale=None, out=None, stream=None):
    """scaled_dot_product_attention (attention.rs:204-302) on f32 [B, S, H, d] device tensors."""
    import torch

    _require_cuda(q, k, v, out)
    n = batch * q_seq * q_heads * head_dim
    ol = n if out is None else out.numel()
    if out is None:
        out = torch.empty(max(n, 1), dtype=torch.float32, device=q.device)
    call("nk_attention_f32", ptr(q), q.numel(), ptr(k), k.numel(), ptr(v), v.numel(), batch,
         q_seq, kv_seq, q_heads, kv_heads, head_dim, 1 if causal else 0, q_offset,
         0 if scale is None else 1, 0.0 if scale is None else scale, ptr(out), ol,
         stream_ptr(stream))
    return out[:ol]


class KvCache:
    """The serving KV cache: K [B, Hkv, max_len, d] and V transposed
    [B, Hkv, d, max_len], bf16, zero-initialised (nk_kv_append)."""

    def __init__(self, batch, kv_heads, head_dim, max_len, device="cuda"):
        import torch

        self.batch, self.kv_heads, self.head_dim, self.max_len = batch, kv_heads, head_dim, max_len
        self.k = torch.zeros(batch, kv_heads, max_len, head_dim, dtype=torch.bfloat16,
                             device=device)
        self.vt = torch.zeros(batch, kv_heads, head_dim, max_len, dtype=torch.bfloat16,
                              device=device)
        self.length = 0

    def append(self, k_new, v_new, seq, stream=None):
        """k_new / v_new bf16 [batch*seq, kv_heads*head_dim] at positions length.. ."""
        _require_cuda(k_new, v_new)
        call("nk_kv_append", ptr(k_new), ptr(v_new), self.batch, seq, self.kv_heads,
             self.head_dim, self.length, self.max_len, ptr(self.k), ptr(self.vt),
             stream_ptr(stream))
        self.length += seq


def attention_gqa(q, cache: KvCache, q_seq, q_heads, *, causal=True, q_offset=None, scale=None,
                  out_dtype=BF16, out=None, workspace=None, stream=None):
    """Grouped-query attention of q bf16 [B*q_seq, q_heads*d] over the cache's
    first `cache.length` positions (nk_attention_gqa).  q_offset defaults to
    cache.length - q_seq (the queries are the last q_seq positions)."""
    import torch

    _require_cuda(q, out, workspace)
    B, Hkv, d, L = cache.batch, cache.kv_heads, cache.head_dim, cache.length
    if q_offset is None:
        q_offset = L - q_seq
    need = ctypes.c_size_t(0)
    call("nk_attention_workspace_bytes", B, q_seq, L, cache.max_len, q_heads, Hkv, d,
         ctypes.byref(need))
    if workspace is None or workspace.numel() < need.value:
        workspace = torch.empty(need.value, dtype=torch.uint8, device=q.device)
    if out is None:
        out = torch.empty(B * q_seq, q_heads * d, device=q.device,
                          dtype=torch.float32 if out_dtype == F32 else torch.bfloat16)
    call("nk_attention_gqa", ptr(q), ptr(cache.k), ptr(cache.vt), B, q_seq, L, cache.max_len,
         q_heads, Hkv, d, 1 if causal else 0, q_offset, 0 if scale is None else 1,
         0.0 if scale is None else scale, ptr(out), out_dtype, ptr(workspace),
         workspace.numel(), stream_ptr(stream))
    return out, workspace


def attention_check(workspace, stream=None) -> int:
    """First output row without a finite score in the last nk_attention_gqa, or -1."""
    r = ctypes.c_int64(0)
    call("nk_attention_check", ptr(workspace), ctypes.byref(r), stream_ptr(stream))
    return r.value


# ------------------------------------------------- decoder steps around projections
def _dtype_code(t):
    import torch

    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.bfloat16:
        return BF16
    raise TypeError(f"unsupported dtype {t.dtype}")


def embedding_lookup(table, token_ids, vocab_size, hidden_size, *, out=None, out_dtype=None,
                     check=True, stream=None):
    """embedding_lookup (embedding.rs:73-91); token_ids int32 on the device."""
    import torch

    _require_cuda(table, token_ids, out)
    n = token_ids.numel()
    if out is None:
        dt = out_dtype or table.dtype
        out = torch.empty(n, hidden_size, dtype=dt, device=table.device)
    call("nk_embedding_lookup", ptr(table), _dtype_code(table), table.numel(), ptr(token_ids), n,
         vocab_size, hidden_size, ptr(out), _dtype_code(out), out.numel(), 1 if check else 0,
         stream_ptr(stream))
    return out


def add_rms_norm_rows(residual, delta, weight, epsilon, *, h_out=None, normed=None,
                      normed_dtype=BF16, stream=None):
    """Block residual (block.rs:145-151) fused with the next RMSNorm; returns (h, normed)."""
    import torch

    _require_cuda(residual, delta, weight, h_out, normed)
    rows, width = residual.shape
    h_out = residual if h_out is None else h_out
    if normed is None:
        normed = torch.empty(rows, width, device=residual.device,
                             dtype=torch.bfloat16 if normed_dtype == BF16 else torch.float32)
    call("nk_add_rms_norm_rows", ptr(residual), ptr(delta), rows, width, ptr(weight),
         weight.numel(), epsilon, ptr(h_out), ptr(normed), _dtype_code(normed),
         stream_ptr(stream))
    return h_out, normed


def argmax_rows(x, *, out=None, stream=None):
    """predict_next_token's pick (model.rs:325-337) per row of x [rows, n]."""
    import torch

    _require_cuda(x, out)
    rows, n = x.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=x.device)
    call("nk_argmax_rows", ptr(x), _dtype_code(x), rows, n, x.stride(0), ptr(out),
         stream_ptr(stream))
    return out
