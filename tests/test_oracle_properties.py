"""Size-independent properties of the CPU oracle (the checker), on seeded
random inputs: INT4 pack/unpack and quantize/dequantize round trips, the
top-k routing invariants, and the expert plan as a stable permutation.
They hold for any size, so they also back the full-size device checks."""
import numpy as np
import pytest

import oracle as orc


@pytest.mark.parametrize("n", [1, 2, 7, 1000, 4097])
def test_int4_pack_unpack_round_trip(n):
    codes = np.random.default_rng(n).integers(0, 16, n).astype(np.uint8)
    packed = orc.pack_int4(codes)
    assert packed.size == (n + 1) // 2
    assert np.array_equal(orc.unpack_int4(packed, n), codes)
    if n % 2:  # the unused high nibble of the last byte stays zero
        assert packed[-1] >> 4 == 0


@pytest.mark.parametrize("zp", [0, 8, 15])
def test_int4_quantize_dequantize_error_bound(zp):
    r = np.random.default_rng(zp)
    scale = np.float32(0.05)
    lo, hi = (0 - zp) * scale, (15 - zp) * scale
    v = r.uniform(lo - 0.2, hi + 0.2, 3001).astype(np.float32)
    deq = orc.dequantize_int4(orc.quantize_int4(v, float(scale), zp), v.size, float(scale), zp)
    inside = (v >= lo) & (v <= hi)
    # inside the representable range: within half a step (plus f32 slack)
    assert np.all(np.abs(deq[inside] - v[inside]) <= scale / 2 + 1e-6)
    # outside: clamped to the nearest end of the range
    assert np.all(deq[v < lo] == np.float32(lo)) and np.all(deq[v > hi] == np.float32(hi))


@pytest.mark.parametrize("mode", [orc.SIGMOID, orc.SOFTMAX, orc.SIGMOID_RENORM])
def test_route_invariants(mode):
    t, e, k = 257, 64, 6
    scores = np.random.default_rng(mode).standard_normal((t, e)).astype(np.float32)
    scores[3, :] = 0.25  # all experts tied: the lowest indices win
    idx, w = orc.route(scores, t, e, k, mode)
    idx, w = idx.reshape(t, k), w.reshape(t, k)
    for row in range(t):
        assert len(set(idx[row])) == k and idx[row].min() >= 0 and idx[row].max() < e
    assert list(idx[3]) == list(range(k))
    if mode == orc.SIGMOID:  # weights are the selected sigmoids, non-increasing
        assert np.all(np.diff(w, axis=1) <= 0)
        sig = 1.0 / (1.0 + np.exp(-scores.astype(np.float64)))
        assert np.allclose(w, np.take_along_axis(sig, idx, 1), rtol=1e-6)
    else:  # renormalised over the selected k
        assert np.allclose(w.sum(axis=1), 1.0, atol=1e-6)
    # every unselected expert ranks below the k-th selected one
    if mode != orc.SOFTMAX:
        sig = 1.0 / (1.0 + np.exp(-scores.astype(np.float64)))
        kth = np.take_along_axis(sig, idx[:, -1:], 1)
        mask = np.ones((t, e), bool)
        np.put_along_axis(mask, idx, False, 1)
        assert np.all(sig[mask].reshape(t, e - k) <= kth + 1e-12)


def test_plan_is_a_stable_permutation():
    t, k, e = 1000, 4, 37
    idx = np.random.default_rng(1).integers(0, e, t * k).astype(np.int32)
    counts, offs, perm = orc.route_histogram(idx, t, k, e)
    assert np.array_equal(counts, np.bincount(idx, minlength=e))
    assert np.array_equal(offs, np.concatenate([[0], np.cumsum(counts)[:-1]]))
    assert np.array_equal(np.sort(perm), np.arange(t * k))
    for x in range(e):  # each expert's block holds its slots in slot order
        block = perm[offs[x]:offs[x] + counts[x]]
        assert np.all(idx[block] == x) and np.all(np.diff(block) > 0)
