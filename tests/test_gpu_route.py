"""Top-k routing and the expert plan on the B200: indices and expert counts
bit-exact against the oracle (moe_routing.rs:118-216), weights within the
reference's own GPU tolerance (5e-6, moe_routing.rs:820)."""
import numpy as np
import pytest
import torch

import nk
import oracle as orc
from gpu_util import dev, host, rng

pytestmark = pytest.mark.gpu
MODES = {"sigmoid": nk.ROUTE_SIGMOID, "softmax": nk.ROUTE_SOFTMAX}


def route(scores, t, e, k, mode):
    s = dev(np.asarray(scores, np.float32).reshape(-1)) if t * e else torch.empty(0, device="cuda")
    idx, w = nk.moe_route(s, t, e, k, mode)
    torch.cuda.synchronize()
    return host(idx), host(w)


def test_route_kats(cuda, kats):
    for c in kats["route"]:
        idx, w = route(c["scores"], c["tokens"], c["experts"], c["top_k"], MODES[c["mode"]])
        assert list(idx) == c["indices"], c["name"]
        assert np.allclose(w, c["weights"], atol=c["tol"], rtol=0), c["name"]


def test_route_generated_kats(cuda, kats):
    for c in kats["route_generated"]:
        t, e, k = c["tokens"], c["experts"], c["top_k"]
        if "score_formula" in c:
            scores = np.array([((ex % 17) - 8.0) * 0.375 + tok * 0.125 - 0.05
                               for tok in range(t) for ex in range(e)], np.float32)
        else:
            scores = np.array(c["scores"], np.float32)
        mode = MODES[c["mode"]]
        ri, rw = orc.route(scores, t, e, k, mode)
        idx, w = route(scores, t, e, k, mode)
        assert np.array_equal(idx, ri), c["name"]
        assert np.allclose(w, rw, atol=c["tol"], rtol=0)


@pytest.mark.parametrize("mode", [orc.SIGMOID, orc.SOFTMAX, orc.SIGMOID_RENORM])
@pytest.mark.parametrize("t,e,k", [(4096, 128, 6), (333, 64, 8), (100, 1000, 32), (50, 3, 3)])
def test_route_random_bit_exact(cuda, mode, t, e, k):
    r = rng(t + e + k + mode)
    scores = (r.standard_normal((t, e)) * 1.5).astype(np.float32)
    # ties: duplicate some scores within a row; extremes saturate sigmoid to 1.0 / 0.0
    scores[::7, 1] = scores[::7, 0]
    scores[::11, : min(e, 5)] = 40.0
    scores[::13, -1] = -200.0
    ri, rw = orc.route(scores, t, e, k, mode)
    idx, w = route(scores, t, e, k, mode)
    assert np.array_equal(idx, ri)
    # weights: the reference's own GPU tolerance (moe_routing.rs:820); almost all
    # are bit-identical (libm expf vs a double exp rounded once differ in rare ulps)
    assert np.max(np.abs(w - rw)) <= 5e-6
    assert np.mean(w == rw) > 0.99


def test_route_nan_and_inf(cuda):
    scores = np.array([[0.0, np.nan, 1.0, -np.inf, np.inf, 2.0]], np.float32)
    for mode in (orc.SIGMOID, orc.SIGMOID_RENORM):
        ri, rw = orc.route(scores, 1, 6, 4, mode)
        idx, w = route(scores, 1, 6, 4, mode)
        assert np.array_equal(idx, ri)
        assert np.array_equal(np.isnan(w), np.isnan(rw))


def test_plan_bit_exact(cuda):
    r = rng(9)
    # several chunks of 1024 routes, a partial chunk, wide expert counts
    for (t, k, e) in [(4096, 6, 128), (1, 2, 4), (3000, 8, 1000), (10, 3, 3),
                      (16384, 4, 256), (20000, 4, 128), (500, 2, 257)]:
        idx = r.integers(0, e, size=t * k).astype(np.int32)
        idx[: t * k // 3] = 0  # a hot expert
        counts_ref, offs_ref, perm_ref = orc.route_histogram(idx, t, k, e)
        counts, offs, perm, pos = nk.moe_plan(dev(idx), t, k, e)
        torch.cuda.synchronize()
        assert np.array_equal(host(counts), counts_ref)
        assert np.array_equal(host(offs)[:e], offs_ref) and host(offs)[e] == t * k
        assert np.array_equal(host(perm), perm_ref)
        inv = np.empty(t * k, np.int64)
        inv[perm_ref] = np.arange(t * k)
        assert np.array_equal(host(pos), inv)
