"""Mamba2 glue on the B200 against the CPU oracle (conv1d.rs, ssm.rs,
rms_norm.rs, mamba2.rs:264-375).

Bars: the conv without SiLU and the RMSNorm are bit-exact (same f64
accumulation, correctly rounded f32 sqrt/reciprocal, separately rounded
multiplies); results through expf/logf (SiLU, softplus, the scan's
transition) are f32 accumulate, max relative error <= 1e-3."""
import numpy as np
import pytest
import torch

import nk
import oracle as orc
from gpu_util import dev, host, rel_err, rng

pytestmark = pytest.mark.gpu
F32_TOL = 1e-3


def _t(a):
    a = np.asarray(a, np.float32).reshape(-1)
    return dev(a) if a.size else torch.empty(0, device="cuda")


# ----------------------------------------------------------------- conv1d
def test_conv1d_kats(cuda, kats):
    for c in kats["conv1d"]:
        out = nk.conv1d(_t(c["input"]), _t(c["weights"]), c["seq"], c["channels"],
                        c["kernel_size"])
        torch.cuda.synchronize()
        assert np.all(np.abs(host(out) - np.asarray(c["out"], np.float32)) <= c["tol"]), c["name"]


def test_conv1d_error_kats(cuda, kats):
    for c in kats["conv1d_errors"]:
        out = torch.empty(max(c["out_len"], 1), device="cuda")
        with pytest.raises(nk.NkError) as ei:
            nk.conv1d(torch.zeros(c["input_len"], device="cuda"),
                      torch.zeros(c["weights_len"], device="cuda"), c["seq"], c["channels"],
                      c["kernel_size"], out=out[:c["out_len"]])
        e = ei.value
        assert e.variant == c["error"], c["name"]
        if c["error"] == "LengthMismatch":
            assert (e.argument, e.expected, e.actual) == (c["argument"], c["expected"],
                                                          c["actual"])


@pytest.mark.parametrize("seq,C,K", [(1, 1, 1), (7, 5, 4), (64, 96, 4), (300, 257, 3),
                                     (33, 64, 32)])
def test_conv1d_bit_exact(cuda, seq, C, K):
    r = rng(seq * 1000 + C + K)
    x = r.standard_normal(seq * C).astype(np.float32)
    w = (r.standard_normal(C * K) * 0.5).astype(np.float32)
    ref = orc.conv1d(x, w, seq, C, K)
    out = host(nk.conv1d(dev(x), dev(w), seq, C, K))
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("f32acc", [False, True])
@pytest.mark.parametrize("B,T,C,K,with_prefix", [(1, 9, 16, 4, False), (3, 17, 40, 4, True),
                                                 (2, 2, 8, 4, True), (2, 1, 8, 4, True),
                                                 (2, 5, 8, 1, False)])
def test_conv1d_ex_history_silu_state(cuda, B, T, C, K, with_prefix, f32acc):
    # mamba2.rs:276-312: history ++ x, drop the history rows, SiLU, new cache.
    r = rng(B * 100 + T * 10 + C)
    P = K - 1
    x = r.standard_normal((B, T, C)).astype(np.float32)
    w = (r.standard_normal((C, K)) * 0.5).astype(np.float32)
    prefix = r.standard_normal((B, P, C)).astype(np.float32) if with_prefix else None
    want_y, want_state = [], []
    for b in range(B):
        hist = prefix[b] if with_prefix else np.zeros((P, C), np.float32)
        ext = np.concatenate([hist, x[b]], axis=0)
        conv = orc.conv1d(ext, w, T + P, C, K).reshape(T + P, C)[P:]
        want_y.append(orc.silu_array(conv).reshape(T, C))
        want_state.append(ext[len(ext) - P:])
    want_y = np.stack(want_y)
    pre_d = dev(prefix) if with_prefix else None
    state = torch.empty(B, max(P, 1), C, device="cuda")
    y = nk.conv1d_ex(dev(x), dev(w), B, T, C, K, prefix=pre_d, silu=True,
                     state_out=state if P else None, f32_accumulate=f32acc)
    torch.cuda.synchronize()
    assert rel_err(host(y).reshape(B, T, C), want_y) <= F32_TOL
    assert np.allclose(host(y).reshape(B, T, C), want_y, rtol=1e-5, atol=1e-5)
    if P:
        assert np.array_equal(host(state)[:, :P], np.stack(want_state))
    if with_prefix and P:
        # In-place cache update: state_out == prefix.
        y2 = nk.conv1d_ex(dev(x), dev(w), B, T, C, K, prefix=pre_d, silu=True,
                          state_out=pre_d, f32_accumulate=f32acc)
        torch.cuda.synchronize()
        assert np.array_equal(host(pre_d), np.stack(want_state))
        assert np.array_equal(host(y2), host(y))


# ------------------------------------------------------------------ scan
def test_scan_kats(cuda, kats):
    for c in kats["scan"]:
        v, f = nk.selective_scan(_t(c["input"]), _t(c["delta_t"]), _t(c["a"]), _t(c["b"]),
                                 _t(c["c"]), c["seq"], c["channels"], c["states"],
                                 d=None if c["d"] is None else _t(c["d"]),
                                 initial_state=None if c["initial_state"] is None
                                 else _t(c["initial_state"]),
                                 delta_bias=c["delta_bias"], softplus=c["softplus"])
        torch.cuda.synchronize()
        assert np.all(np.abs(host(v) - np.float32(c["values"])) <= c["tol"]), c["name"]
        assert np.all(np.abs(host(f) - np.float32(c["final_state"])) <= c["tol"]), c["name"]


def test_scan_error_kats(cuda, kats):
    for c in kats["scan_errors"]:
        with pytest.raises(nk.NkError) as ei:
            nk.selective_scan(_t(c["input"]), _t(c["delta_t"]), _t(c["a"]), _t(c["b"]),
                              _t(c["c"]), c["seq"], c["channels"], c["states"],
                              d=None if c["d"] is None else _t(c["d"]),
                              initial_state=None if c["initial_state"] is None
                              else _t(c["initial_state"]), softplus=c["softplus"])
        e = ei.value
        assert e.variant == c["error"], c["name"]
        if c["error"] == "LengthMismatch":
            assert (e.argument, e.expected, e.actual) == (c["argument"], c["expected"],
                                                          c["actual"])
        if c["error"] == "InvalidDeltaT":
            assert divmod(e.index, c["channels"]) == (c["timestep"], c["channel"])
            assert e.value == c["value"]


def test_scan_invalid_delta_t_first_in_time_order(cuda):
    dt = np.array([1.0, 1.0, 1.0, -2.0, np.inf, 1.0], np.float32)
    with pytest.raises(nk.NkError) as ei:
        nk.selective_scan(dev(np.ones(6, np.float32)), dev(dt), dev(np.zeros(2, np.float32)),
                          dev(np.ones(6, np.float32)), dev(np.ones(6, np.float32)), 3, 2, 1)
    assert ei.value.variant == "InvalidDeltaT" and ei.value.index == 3
    assert ei.value.value == -2.0
    # softplus(NaN) is NaN: rejected too (ssm.rs:280).
    dt = np.array([0.5, np.nan], np.float32)
    with pytest.raises(nk.NkError) as ei:
        nk.selective_scan(dev(np.ones(2, np.float32)), dev(dt), dev(np.zeros(1, np.float32)),
                          dev(np.ones(2, np.float32)), dev(np.ones(2, np.float32)), 2, 1, 1,
                          softplus=True)
    assert ei.value.index == 1


def _scan_case(seed, T, C, S, with_d, with_init):
    r = rng(seed)
    return dict(
        x=r.standard_normal(T * C).astype(np.float32),
        dt=(r.standard_normal(T * C) * 0.5).astype(np.float32),
        a=(-np.abs(r.standard_normal(C * S))).astype(np.float32),
        b=r.standard_normal(T * C * S).astype(np.float32),
        c=r.standard_normal(T * C * S).astype(np.float32),
        d=r.standard_normal(C).astype(np.float32) if with_d else None,
        init=r.standard_normal(C * S).astype(np.float32) if with_init else None)


@pytest.mark.parametrize("T,C,S,with_d,with_init,spl",
                         [(5, 3, 1, True, False, None), (16, 7, 2, False, True, None),
                          (40, 33, 16, True, True, None), (64, 20, 64, True, True, None),
                          (48, 17, 128, True, False, None), (48, 17, 128, True, True, "8"),
                          (45, 17, 128, True, True, None), (3, 17, 128, True, True, None),
                          (32, 9, 100, False, True, None), (24, 5, 256, True, True, None)])
def test_scan_reference_layout(cuda, monkeypatch, T, C, S, with_d, with_init, spl):
    if spl:
        monkeypatch.setenv("NK_SCAN_CFG", spl)
    p = _scan_case(T * 7 + C * 3 + S, T, C, S, with_d, with_init)
    vals, fin = orc.selective_scan(p["x"], p["dt"], p["a"], p["b"], p["c"], T, C, S, d=p["d"],
                                   initial_state=p["init"], softplus=True)
    v, f = nk.selective_scan(dev(p["x"]), dev(p["dt"]), dev(p["a"]), dev(p["b"]), dev(p["c"]),
                             T, C, S, d=None if p["d"] is None else dev(p["d"]),
                             initial_state=None if p["init"] is None else dev(p["init"]),
                             softplus=True)
    torch.cuda.synchronize()
    assert rel_err(host(v), vals) <= F32_TOL
    assert rel_err(host(f), fin) <= F32_TOL


def _expand_grouped(T, C, S, H, G, r, a_h, d_h):
    """Mamba2 layout (one dt/A/D per head of C/H channels, B/C per group of C/G)
    and its per-channel expansion, which is the reference layout."""
    hd, gw = C // H, C // G
    dt_h = (r.standard_normal((T, H)) * 0.5).astype(np.float32)
    b_g = r.standard_normal((T, G, S)).astype(np.float32)
    c_g = r.standard_normal((T, G, S)).astype(np.float32)
    head = np.arange(C) // hd
    grp = np.arange(C) // gw
    ref = dict(dt=dt_h[:, head], a=np.repeat(a_h[head][:, None], S, axis=1), d=d_h[head],
               b=b_g[:, grp, :], c=c_g[:, grp, :])
    return dict(dt=dt_h, a=a_h, d=d_h, b=b_g, c=c_g, hd=hd, gw=gw), ref


@pytest.mark.parametrize("B,T,C,S,H,G,cfg", [(1, 32, 64, 16, 4, 2, None),
                                             (2, 20, 128, 64, 8, 4, None),
                                             (1, 24, 96, 128, 6, 2, None),
                                             (2, 37, 128, 128, 4, 2, None),
                                             (2, 37, 128, 128, 4, 2, "1"),
                                             (2, 37, 128, 128, 4, 2, "2"),
                                             (2, 37, 128, 128, 4, 2, "4"),
                                             (3, 16, 256, 128, 4, 2, "5"),
                                             (1, 19, 96, 128, 6, 2, "2"),
                                             (1, 5, 64, 128, 2, 1, None),
                                             (3, 16, 256, 128, 4, 2, None)])
def test_scan_grouped_fused_layout(cuda, monkeypatch, B, T, C, S, H, G, cfg):
    if cfg:
        monkeypatch.setenv("NK_SCAN_CFG", cfg)
    # The Mamba2 layout read in place from one fused row [x | B | C | dt].
    r = rng(B * 31 + T + C + S)
    x = r.standard_normal((B, T, C)).astype(np.float32)
    init = r.standard_normal((B, C, S)).astype(np.float32)
    a_h = (-np.abs(r.standard_normal(H))).astype(np.float32)
    d_h = r.standard_normal(H).astype(np.float32)
    grouped, refs = [], []
    for _ in range(B):
        g, ref = _expand_grouped(T, C, S, H, G, r, a_h, d_h)
        grouped.append(g)
        refs.append(ref)
    hd, gw = grouped[0]["hd"], grouped[0]["gw"]
    width = C + 2 * G * S + H + 4  # padded row, like a wider in_proj output
    fused = np.zeros((B, T, width), np.float32)
    for b in range(B):
        fused[b, :, :C] = x[b]
        fused[b, :, C:C + G * S] = grouped[b]["b"].reshape(T, G * S)
        fused[b, :, C + G * S:C + 2 * G * S] = grouped[b]["c"].reshape(T, G * S)
        fused[b, :, C + 2 * G * S:C + 2 * G * S + H] = grouped[b]["dt"]
    fd = dev(fused)
    a_d, d_d, init_d = dev(a_h), dev(d_h), dev(init)
    y = torch.empty(B * T, C, device="cuda")
    fin = torch.empty(B, C, S, device="cuda")
    base = fd.data_ptr()
    args = nk.NkScanArgs(
        B, T, C, S, base, width, base + 4 * (C + 2 * G * S), width, hd, a_d.data_ptr(), hd, 0,
        base + 4 * C, base + 4 * (C + G * S), width, gw, d_d.data_ptr(), hd,
        init_d.data_ptr(), 0.0, 1, y.data_ptr(), C, fin.data_ptr(), 1)
    nk.selective_scan_ex(args)
    torch.cuda.synchronize()
    for b in range(B):
        ref = refs[b]
        vals, f = orc.selective_scan(x[b], ref["dt"], ref["a"], ref["b"], ref["c"], T, C, S,
                                     d=ref["d"], initial_state=init[b], softplus=True)
        assert rel_err(host(y).reshape(B, T, C)[b], vals.reshape(T, C)) <= F32_TOL
        assert rel_err(host(fin)[b], f.reshape(C, S)) <= F32_TOL
    # InvalidDeltaT: the first bad (t, ch) in t-major order (ssm.rs:135-145); a
    # head's dt is shared, so it is the head's first channel.
    bad_t, bad_h = T // 2, H - 1
    fused[0, bad_t, C + 2 * G * S + bad_h] = np.nan
    fd.copy_(torch.from_numpy(fused))
    with pytest.raises(nk.NkError) as ei:
        nk.selective_scan_ex(args)
    assert ei.value.variant == "InvalidDeltaT"
    assert ei.value.index == bad_t * C + bad_h * hd


def test_scan_final_state_in_place(cuda):
    T, C, S = 12, 10, 32
    p = _scan_case(5, T, C, S, True, True)
    vals, fin = orc.selective_scan(p["x"], p["dt"], p["a"], p["b"], p["c"], T, C, S, d=p["d"],
                                   initial_state=p["init"], softplus=True)
    state = dev(p["init"])
    v, f = nk.selective_scan(dev(p["x"]), dev(p["dt"]), dev(p["a"]), dev(p["b"]), dev(p["c"]),
                             T, C, S, d=dev(p["d"]), initial_state=state, softplus=True,
                             final_state=state)
    torch.cuda.synchronize()
    assert rel_err(host(state), fin) <= F32_TOL
    assert rel_err(host(v), vals) <= F32_TOL


# ------------------------------------------------------------------ norm
def test_rms_norm_kats(cuda, kats):
    for c in kats["rms_norm"]:
        out = nk.rms_norm(_t(c["input"]), _t(c["weight"]), c["epsilon"],
                          gate=None if c["gate"] is None else _t(c["gate"]))
        torch.cuda.synchronize()
        assert np.all(np.abs(host(out) - np.float32(c["out"])) <= c["tol"]), c["name"]


def test_rms_norm_error_kats(cuda, kats):
    for c in kats["rms_norm_errors"]:
        with pytest.raises(nk.NkError) as ei:
            nk.rms_norm(_t(c["input"]), _t(c["weight"]), c["epsilon"],
                        gate=None if c["gate"] is None else _t(c["gate"]))
        e = ei.value
        assert e.variant == c["error"], c["name"]
        if c["error"] == "LengthMismatch":
            assert (e.argument, e.expected, e.actual) == (c["argument"], c["expected"],
                                                          c["actual"])
        if c["error"] == "NegativeEpsilon":
            assert e.value == c["value"]


@pytest.mark.parametrize("rows,width,gated", [(1, 1, False), (3, 7, True), (17, 2688, False),
                                              (9, 8192, True), (64, 1000, True)])
def test_rms_norm_rows_bit_exact(cuda, rows, width, gated):
    r = rng(rows * 7 + width)
    x = r.standard_normal((rows, width)).astype(np.float32)
    w = r.standard_normal(width).astype(np.float32)
    g = r.standard_normal((rows, width)).astype(np.float32) if gated else None
    ref = orc.rms_norm_rows(x, w, 1e-5, width, gate=g).reshape(rows, width)
    out = nk.rms_norm_rows(dev(x), dev(w), 1e-5, gate=None if g is None else dev(g))
    torch.cuda.synchronize()
    got = host(out)
    # f64 sums in another order can move the f32 mean square by one ulp at most.
    assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1e-30)) <= 2e-7
    bf = nk.rms_norm_rows(dev(x), dev(w), 1e-5, gate=None if g is None else dev(g),
                          out_dtype=nk.BF16)
    torch.cuda.synchronize()
    assert torch.equal(bf, torch.from_numpy(got).cuda().to(torch.bfloat16))


def test_rms_norm_rows_strided_views(cuda):
    r = rng(3)
    full = r.standard_normal((6, 50)).astype(np.float32)
    x, g = full[:, 10:30], full[:, 30:50]
    w = r.standard_normal(20).astype(np.float32)
    ref = orc.rms_norm_rows(np.ascontiguousarray(x), w, 1e-6, 20,
                            gate=np.ascontiguousarray(g)).reshape(6, 20)
    fd = dev(full)
    out = nk.rms_norm_rows(fd[:, 10:30], dev(w), 1e-6, gate=fd[:, 30:50])
    torch.cuda.synchronize()
    assert np.allclose(host(out), ref, rtol=2e-7, atol=0)


# ------------------------------------------------------------- mixer glue
@pytest.mark.parametrize("B,T,C,S,K,cached", [(1, 16, 32, 16, 4, False),
                                              (2, 12, 48, 64, 4, True)])
def test_glue_pipeline_matches_oracle(cuda, B, T, C, S, K, cached):
    """conv(+cache) -> SiLU -> scan(softplus dt, D, SSM cache) -> gated norm,
    the composition of mamba2.rs:276-351, against the oracle's mamba2_glue."""
    r = rng(B + T + C + S)
    f = lambda *s, sc=1.0: (r.standard_normal(s) * sc).astype(np.float32)
    x, dt, bm, cm, g = f(B * T, C), f(B * T, C, sc=0.5), f(B * T, C * S), f(B * T, C * S), \
        f(B * T, C)
    w, a, nw, d = f(C, K, sc=0.5), -np.abs(f(C, S)), f(C), f(C)
    P = K - 1
    conv0 = f(B, P, C) if cached else None
    ssm0 = f(B, C, S, sc=0.1) if cached else None
    want, want_conv, want_ssm = orc.mamba2_glue(x, dt, bm, cm, g, w, a, nw, 1e-5, B, T, C, S, K,
                                                d=d, conv_state=conv0, ssm_state=ssm0)
    conv_state = dev(conv0) if cached else None
    ssm_state = dev(ssm0) if cached else None
    act = nk.conv1d_ex(dev(x), dev(w), B, T, C, K, prefix=conv_state, silu=True,
                       state_out=conv_state)
    y = torch.empty(B * T, C, device="cuda")
    fin = ssm_state if cached else torch.empty(B, C, S, device="cuda")
    dtd, ad, bd, cd, dd = dev(dt), dev(a), dev(bm), dev(cm), dev(d)
    args = nk.NkScanArgs(B, T, C, S, act.data_ptr(), C, dtd.data_ptr(), C, 1, ad.data_ptr(), 1,
                         1, bd.data_ptr(), cd.data_ptr(), C * S, 1, dd.data_ptr(), 1,
                         ssm_state.data_ptr() if cached else None, 0.0, 1, y.data_ptr(), C,
                         fin.data_ptr(), 1)
    nk.selective_scan_ex(args)
    out = nk.rms_norm_rows(y, dev(nw), 1e-5, gate=dev(g))
    torch.cuda.synchronize()
    assert rel_err(host(out), want) <= F32_TOL
    assert rel_err(host(fin), want_ssm) <= F32_TOL
    if cached:
        assert np.array_equal(host(conv_state), want_conv)
