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


# ------------------------------------------------------------ Mamba2 glue

ERR_NAMES.update({11: "InvalidDeltaT", 12: "EmptyInput", 13: "NegativeEpsilon"})


def silu(x: float) -> float:
    f = lib().orc_silu
    f.restype, f.argtypes = ctypes.c_float, [ctypes.c_float]
    return f(x)


def silu_array(values):
    """silu_in_place_host (activations.rs:95-97) through the C restatement (libm expf)."""
    v = np.array(np.asarray(values, dtype=np.float32).reshape(-1), dtype=np.float32, copy=True)
    if v.size:
        lib().orc_silu_in_place(_p(v), ctypes.c_size_t(v.size))
    return v


def conv1d(inp, weights, seq, channels, kernel_size, input_len=None, weights_len=None,
           out_len=None):
    """depthwise_causal_conv1d_into_host (conv1d.rs:78-124)."""
    x = _f32(np.asarray(inp).reshape(-1)) if np.asarray(inp).size else np.zeros(1, np.float32)
    w = _f32(np.asarray(weights).reshape(-1)) if np.asarray(weights).size else np.zeros(1, np.float32)
    il = np.asarray(inp).size if input_len is None else input_len
    wl = np.asarray(weights).size if weights_len is None else weights_len
    ol = seq * channels if out_len is None else out_len
    out = np.zeros(max(ol, 1), np.float32)
    err = OrcError()
    rc = lib().orc_conv1d(_p(x), ctypes.c_size_t(il), _p(w), ctypes.c_size_t(wl),
                          ctypes.c_size_t(seq), ctypes.c_size_t(channels),
                          ctypes.c_size_t(kernel_size), _p(out), ctypes.c_size_t(ol),
                          ctypes.byref(err))
    _check(rc, err)
    return out[:ol]


def _arr(a):
    if a is None:
        return None, 0
    a = np.asarray(a, dtype=np.float32).reshape(-1)
    return (np.ascontiguousarray(a) if a.size else np.zeros(1, np.float32)), a.size


def selective_scan(inp, delta_t, a, b, c, seq, channels, states, d=None, initial_state=None,
                   delta_bias=0.0, softplus=False, out_len=None, final_state_len=None):
    """selective_scan_into_host (ssm.rs:123-175).  Returns (values, final_state)."""
    args = [_arr(v) for v in (inp, delta_t, a, b, c, d, initial_state)]
    ol = seq * channels if out_len is None else out_len
    fl = channels * states if final_state_len is None else final_state_len
    out = np.zeros(max(ol, 1), np.float32)
    fin = np.zeros(max(fl, 1), np.float32)
    err = OrcError()
    flat = []
    for arr, n in args:
        flat += [_p(arr), ctypes.c_size_t(n)]
    rc = lib().orc_selective_scan(*flat, ctypes.c_float(delta_bias), ctypes.c_int(int(softplus)),
                                  ctypes.c_size_t(seq), ctypes.c_size_t(channels),
                                  ctypes.c_size_t(states), _p(out), ctypes.c_size_t(ol),
                                  _p(fin), ctypes.c_size_t(fl), ctypes.byref(err))
    _check(rc, err)
    return out[:ol], fin[:fl]


def rms_norm(inp, weight, epsilon, gate=None, out_len=None):
    """rms_norm_into_host / gated_rms_norm_into_host (rms_norm.rs:64-144)."""
    (x, n), (w, wn), (g, gn) = _arr(inp), _arr(weight), _arr(gate)
    ol = n if out_len is None else out_len
    out = np.zeros(max(ol, 1), np.float32)
    err = OrcError()
    rc = lib().orc_rms_norm(_p(x), ctypes.c_size_t(n), _p(w), ctypes.c_size_t(wn), _p(g),
                            ctypes.c_size_t(gn), ctypes.c_float(epsilon), _p(out),
                            ctypes.c_size_t(ol), ctypes.byref(err))
    _check(rc, err)
    return out[:ol]


def rms_norm_rows(inp, weight, epsilon, row_width, gate=None):
    """Row-wise contract (rms_norm.rs:224-252): each row of `row_width` normalised alone."""
    x = np.asarray(inp, np.float32).reshape(-1, row_width)
    g = None if gate is None else np.asarray(gate, np.float32).reshape(-1, row_width)
    return np.concatenate([rms_norm(x[r], weight, epsilon, None if g is None else g[r])
                           for r in range(x.shape[0])])


def mamba2_glue(x_proj, delta_t, b, c, gate, conv_weights, ssm_a, norm_weight, epsilon,
                batch, seq, channels, states, kernel_size, d=None, conv_state=None,
                ssm_state=None):
    """The stages of Mamba2Mixer::forward (mamba2.rs:264-375) between the five
    input projections and out_proj, per batch: conv input = K-1 cached (or
    zero) steps + x; depthwise conv; drop the prefix; SiLU; selective scan with
    softplus(dt), delta_bias 0; gated RMSNorm per row of width C.

    Inputs are [batch*seq, width] row-major (x/dt/gate width C, b/c width C*S).
    Returns (normalised [batch*seq, C], new conv_state [batch, K-1, C],
    final ssm_state [batch, C, S])."""
    C, S, K, T = channels, states, kernel_size, seq
    P = K - 1
    xs = np.asarray(x_proj, np.float32).reshape(batch, T, C)
    dts = np.asarray(delta_t, np.float32).reshape(batch, T, C)
    bs = np.asarray(b, np.float32).reshape(batch, T * C * S)
    cs = np.asarray(c, np.float32).reshape(batch, T * C * S)
    gs = np.asarray(gate, np.float32).reshape(batch, T, C)
    out = np.zeros((batch, T, C), np.float32)
    new_conv = np.zeros((batch, P, C), np.float32)
    fin = np.zeros((batch, C, S), np.float32)
    for bi in range(batch):
        prefix = (np.zeros((P, C), np.float32) if conv_state is None
                  else np.asarray(conv_state, np.float32).reshape(batch, P, C)[bi])
        conv_in = np.concatenate([prefix, xs[bi]], axis=0)
        conv = conv1d(conv_in, conv_weights, T + P, C, K).reshape(T + P, C)[P:]
        act = silu_array(conv)
        init = None if ssm_state is None else np.asarray(ssm_state, np.float32).reshape(batch, -1)[bi]
        vals, f = selective_scan(act, dts[bi], ssm_a, bs[bi], cs[bi], T, C, S, d=d,
                                 initial_state=init, delta_bias=0.0, softplus=True)
        out[bi] = rms_norm_rows(vals, norm_weight, epsilon, C, gate=gs[bi]).reshape(T, C)
        new_conv[bi] = conv_in[len(conv_in) - P:] if P else new_conv[bi]
        fin[bi] = f.reshape(C, S)
    return out.reshape(batch * T, C), new_conv, fin


# ------------------------------------------------------------ attention core

ERR_NAMES.update({14: "HeadCountMismatch", 15: "InvalidScale", 16: "NoValidAttentionTargets",
                  17: "ZeroPartition"})


def attention(q, k, v, batch, q_seq, kv_seq, q_heads, kv_heads, head_dim, causal=False,
              q_offset=0, scale=None, out_len=None):
    """scaled_dot_product_attention_into_host (attention.rs:204-302); [B, S, H, d] layouts."""
    (qa, qn), (ka, kn), (va, vn) = _arr(q), _arr(k), _arr(v)
    ol = batch * q_seq * q_heads * head_dim if out_len is None else out_len
    out = np.zeros(max(ol, 1), np.float32)
    err = OrcError()
    rc = lib().orc_attention(_p(qa), ctypes.c_size_t(qn), _p(ka), ctypes.c_size_t(kn), _p(va),
                             ctypes.c_size_t(vn), ctypes.c_size_t(batch), ctypes.c_size_t(q_seq),
                             ctypes.c_size_t(kv_seq), ctypes.c_size_t(q_heads),
                             ctypes.c_size_t(kv_heads), ctypes.c_size_t(head_dim),
                             ctypes.c_int(int(causal)), ctypes.c_size_t(q_offset),
                             ctypes.c_int(0 if scale is None else 1),
                             ctypes.c_float(0.0 if scale is None else scale), _p(out),
                             ctypes.c_size_t(ol), ctypes.byref(err))
    _check(rc, err)
    return out[:ol]


# ------------------------------------------------------------ decoder composition

def _bf16(a):
    """Round-to-nearest-even to bf16, kept in f32 (the serving path's operand type)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(a), a, out).astype(np.float32)


def embedding(table, token_ids, vocab, hidden):
    """embedding_lookup_into_host (embedding.rs:73-91, validation :121-191)."""
    table = np.asarray(table, np.float32).reshape(-1)
    if vocab == 0 or hidden == 0:
        raise ValueError("InvalidShape")
    if table.size != vocab * hidden:
        raise ValueError("LengthMismatch table")
    ids = np.asarray(token_ids, np.int64).reshape(-1)
    for t in ids:
        if t >= vocab or t < 0:
            raise ValueError(f"TokenOutOfRange {t}")
    return table.reshape(vocab, hidden)[ids].copy()


def argmax_total(row):
    """predict_next_token's pick (model.rs:325-337): max under f32::total_cmp,
    the last index among equal maxima (Iterator::max_by)."""
    u = np.asarray(row, np.float32).view(np.uint32).astype(np.uint64)
    key = np.where(u & 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000)
    m = key.max()
    return int(np.nonzero(key == m)[0][-1])


def _linear_rows(x, w_out_in):
    """LinearProjection::project with W given [out, in] (orc.linear takes [in, out])."""
    rows = x.shape[0]
    n_out, n_in = w_out_in.shape
    return linear(np.ascontiguousarray(w_out_in.T), None, n_in, n_out, x.reshape(-1),
                  rows).reshape(rows, n_out)


def mamba2_fused_block(x, w_in, w_out, conv, a_head, d_head, norm_w, heads, head_dim, groups,
                       state, kernel_size, eps, batch, seq, conv_state=None, ssm_state=None):
    """The fused-layout Mamba2 block restated on the reference stages: in_proj
    (rows z | x | B | C | dt), then mamba2_glue on the per-channel expansion
    (dt, A, D per head; B, C per group), then out_proj of the bf16-rounded
    normed rows.  Returns (y, new conv_state, new ssm_state)."""
    C = heads * head_dim
    T = x.shape[0]
    fused = _linear_rows(_bf16(x), w_in)
    z, xs = fused[:, :C], fused[:, C:2 * C]
    bg = fused[:, 2 * C:2 * C + groups * state].reshape(T, groups, state)
    cg = fused[:, 2 * C + groups * state:2 * C + 2 * groups * state].reshape(T, groups, state)
    dth = fused[:, 2 * C + 2 * groups * state:]
    head, grp = np.arange(C) // head_dim, np.arange(C) // (C // groups)
    normed, new_conv, fin = mamba2_glue(
        xs, dth[:, head], bg[:, grp, :].reshape(T, C * state), cg[:, grp, :].reshape(T, C * state),
        z, conv, np.repeat(a_head[head][:, None], state, axis=1), norm_w, eps, batch, seq, C,
        state, kernel_size, d=d_head[head], conv_state=conv_state, ssm_state=ssm_state)
    return _linear_rows(_bf16(normed), w_out), new_conv, fin


def decoder_forward(cfg, w, tokens, batch, seq, state=None):
    """NemotronModel::forward_tokens (model.rs:258-323) over NemotronBlock::forward_into
    (block.rs:84-157) with the serving path's bf16 operand rounding: the
    normed block inputs, attention q/k/v/o and the MoE inputs are rounded to
    bf16 as the device path feeds its GEMMs.  `w` holds host (numpy) weights:
    embed [V,H], lm_head [V,H], norms [L+1][H], layers[i] dicts.  `state`
    (optional, updated) carries per-layer caches: attention (k, v) lists,
    Mamba (conv, ssm).  Returns logits of every row [batch*seq, V]."""
    H, eps = cfg.hidden, cfg.eps
    h = embedding(w["embed"], tokens, cfg.vocab, H)
    if state is None:
        state = [None] * len(cfg.layer_kinds)
    for i, kind in enumerate(cfg.layer_kinds):
        normed = _bf16(rms_norm_rows(h, w["norms"][i], eps, H).reshape(-1, H))
        lw = w["layers"][i]
        if kind == "mamba":
            st = state[i] or (None, None)
            m, cs, ss = mamba2_fused_block(normed, lw["w_in"], lw["w_out"], lw["conv"], lw["a"],
                                           lw["d"], lw["norm"], cfg.mamba_heads,
                                           cfg.mamba_head_dim, cfg.mamba_groups, cfg.mamba_state,
                                           cfg.conv_kernel, eps, batch, seq, st[0], st[1])
            state[i] = (cs, ss)
        elif kind == "moe":
            Is = cfg.shared_inter
            m, _, _ = moe(H, cfg.experts, cfg.top_k, cfg.moe_inter, Is, lw["router"].T.copy(),
                          None, lw["up"].transpose(0, 2, 1).copy(), None,
                          lw["down"].transpose(0, 2, 1).copy(), None,
                          lw["sup"].T.copy() if Is else None, None,
                          lw["sdown"].T.copy() if Is else None, None, normed, normed.shape[0],
                          cfg.route_mode)
            m = m.reshape(-1, H)
        else:
            hq, hkv, d = cfg.q_heads, cfg.kv_heads, cfg.head_dim
            q = _bf16(_linear_rows(normed, lw["wq"])).reshape(batch, seq, hq, d)
            k = _bf16(_linear_rows(normed, lw["wk"])).reshape(batch, seq, hkv, d)
            v = _bf16(_linear_rows(normed, lw["wv"])).reshape(batch, seq, hkv, d)
            prev = state[i]
            if prev is not None:
                k = np.concatenate([prev[0], k], axis=1)
                v = np.concatenate([prev[1], v], axis=1)
            state[i] = (k, v)
            L = k.shape[1]
            o = attention(q, k, v, batch, seq, L, hq, hkv, d, causal=True, q_offset=L - seq)
            m = _linear_rows(_bf16(o.reshape(batch * seq, hq * d)), lw["wo"])
        h = h + m.reshape(h.shape)
    normed = _bf16(rms_norm_rows(h, w["norms"][-1], eps, H).reshape(-1, H))
    return _linear_rows(normed, w["lm_head"]), state
