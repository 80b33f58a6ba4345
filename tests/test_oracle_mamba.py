"""The CPU oracle's Mamba2 glue (conv1d, selective scan, RMSNorm) pinned
against the reference's own known-answer tests (conv1d.rs, ssm.rs,
rms_norm.rs inline tests, transcribed into tests/golden/reference_kats.json
with file:line sources), plus the mixer-level properties mamba2.rs tests."""
import numpy as np
import pytest

import oracle as orc


def _close(got, want, tol):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape
    assert np.all(np.abs(got - want) <= tol), (got, want)


def test_conv1d_kats(kats):
    for c in kats["conv1d"]:
        out = orc.conv1d(c["input"], c["weights"], c["seq"], c["channels"], c["kernel_size"])
        _close(out, c["out"], c["tol"])


def test_conv1d_error_kats(kats):
    for c in kats["conv1d_errors"]:
        with pytest.raises(orc.OracleError) as ei:
            orc.conv1d(np.zeros(c["input_len"]), np.zeros(c["weights_len"]), c["seq"],
                       c["channels"], c["kernel_size"], input_len=c["input_len"],
                       weights_len=c["weights_len"], out_len=c["out_len"])
        e = ei.value
        assert e.variant == c["error"], c["name"]
        if c["error"] == "LengthMismatch":
            assert (e.argument, e.expected, e.actual) == (c["argument"], c["expected"],
                                                          c["actual"]), c["name"]


def test_scan_kats(kats):
    for c in kats["scan"]:
        vals, fin = orc.selective_scan(c["input"], c["delta_t"], c["a"], c["b"], c["c"],
                                       c["seq"], c["channels"], c["states"], d=c["d"],
                                       initial_state=c["initial_state"],
                                       delta_bias=c["delta_bias"], softplus=c["softplus"])
        _close(vals, c["values"], c["tol"])
        _close(fin, c["final_state"], c["tol"])


def test_scan_error_kats(kats):
    for c in kats["scan_errors"]:
        with pytest.raises(orc.OracleError) as ei:
            orc.selective_scan(c["input"], c["delta_t"], c["a"], c["b"], c["c"], c["seq"],
                               c["channels"], c["states"], d=c["d"],
                               initial_state=c["initial_state"], softplus=c["softplus"])
        e = ei.value
        assert e.variant == c["error"], c["name"]
        if c["error"] == "LengthMismatch":
            assert (e.argument, e.expected, e.actual) == (c["argument"], c["expected"],
                                                          c["actual"])
        if c["error"] == "InvalidDeltaT":
            assert divmod(e.index, c["channels"]) == (c["timestep"], c["channel"])
            assert e.value == c["value"]


def test_rms_norm_kats(kats):
    for c in kats["rms_norm"]:
        out = orc.rms_norm(c["input"], c["weight"], c["epsilon"], gate=c["gate"])
        _close(out, c["out"], c["tol"])


def test_rms_norm_error_kats(kats):
    for c in kats["rms_norm_errors"]:
        with pytest.raises(orc.OracleError) as ei:
            orc.rms_norm(c["input"], c["weight"], c["epsilon"], gate=c["gate"])
        e = ei.value
        assert e.variant == c["error"], c["name"]
        if c["error"] == "LengthMismatch":
            assert (e.argument, e.expected, e.actual) == (c["argument"], c["expected"],
                                                          c["actual"])
        if c["error"] == "NegativeEpsilon":
            assert e.value == c["value"]


def test_scan_invalid_delta_t_reports_first_in_time_order():
    # ssm.rs:135-145 checks dt step by step, channel-minor: the first bad (t, ch).
    dt = np.array([1.0, 1.0, 1.0, -2.0, np.inf, 1.0], np.float32)  # seq 3, C 2
    with pytest.raises(orc.OracleError) as ei:
        orc.selective_scan(np.ones(6), dt, np.zeros(2), np.ones(6), np.ones(6), 3, 2, 1)
    assert ei.value.variant == "InvalidDeltaT" and ei.value.index == 3


def _mixer_case(seed, batch, seq, C, S, K):
    r = np.random.default_rng(seed)
    f = lambda *s, sc=1.0: (r.standard_normal(s) * sc).astype(np.float32)
    return dict(x=f(batch * seq, C), dt=f(batch * seq, C, sc=0.5), b=f(batch * seq, C * S),
                c=f(batch * seq, C * S), g=f(batch * seq, C), w=f(C, K, sc=0.5),
                a=-np.abs(f(C, S)), nw=f(C), d=f(C))


def test_glue_decode_with_cache_matches_full_sequence():
    # mamba2.rs:793-815: stepping with the conv/SSM caches equals the full pass.
    B, T, C, S, K = 2, 5, 3, 4, 3
    p = _mixer_case(1, B, T, C, S, K)
    full, _, _ = orc.mamba2_glue(p["x"], p["dt"], p["b"], p["c"], p["g"], p["w"], p["a"],
                                 p["nw"], 1e-5, B, T, C, S, K, d=p["d"])
    resh = lambda a, w: a.reshape(B, T, w)
    conv, ssm = None, None
    steps = []
    for t in range(T):
        sl = lambda a, w: resh(a, w)[:, t:t + 1].reshape(B, w)
        y, conv, ssm = orc.mamba2_glue(sl(p["x"], C), sl(p["dt"], C), sl(p["b"], C * S),
                                       sl(p["c"], C * S), sl(p["g"], C), p["w"], p["a"],
                                       p["nw"], 1e-5, B, 1, C, S, K, d=p["d"],
                                       conv_state=conv, ssm_state=ssm)
        steps.append(y.reshape(B, 1, C))
    step = np.concatenate(steps, axis=1).reshape(B * T, C)
    assert np.max(np.abs(step - full)) <= 1e-5 * max(1.0, float(np.max(np.abs(full))))
