"""The projection entry points called concurrently: two host threads, each
with its own CUDA stream, run decode-shape projections (K split over CTAs,
so each call needs f32 partial-sum scratch) at the same time.  With the
library scratch (one block per device and stream) and with caller-owned
workspaces (the *_ws entry points), every result must equal the oracle's
LinearProjection restatement (linear.rs:283-342) within the f32-accumulate
bar (1e-3 for f32 activations and int8 codes) — no call may see another's
partial sums.  Also: scratch growth is refused during stream capture."""
import threading

import numpy as np
import pytest
import torch

import nk
import oracle as orc
from gpu_util import bf16_round, dev, host, rel_err, rng

pytestmark = pytest.mark.gpu


def _case(seed, m, k, n):
    r = rng(seed)
    x = r.standard_normal((m, k)).astype(np.float32)
    w = (r.standard_normal((n, k)) * 0.02).astype(np.float32)
    q, s = nk.quantize_int8_row(dev(w))
    deq = host(q).astype(np.float32) * host(s)[:, None]
    ref = orc.linear(deq.T.copy(), None, k, n, x, m).reshape(m, n)
    return dict(x=dev(x), q=q, s=s, ref=ref, shape=(m, k, n))


@pytest.mark.parametrize("use_ws", [False, True], ids=["stream_scratch", "caller_workspace"])
def test_concurrent_decode_projections_two_streams(cuda, use_ws):
    cases = [_case(1, 16, 4096, 4096), _case(2, 8, 2048, 6144)]
    for c in cases:  # these shapes split K, so they use scratch
        m, k, n = c["shape"]
        assert nk.gemm_workspace_bytes("int8", torch.float32, m, k, n) > 0
    outs = [[], []]
    errors = []

    def worker(i):
        try:
            c = cases[i]
            m, k, n = c["shape"]
            st = torch.cuda.Stream()
            ws = None
            if use_ws:
                ws = torch.empty(nk.gemm_workspace_bytes("int8", torch.float32, m, k, n),
                                 dtype=torch.uint8, device="cuda")
            with torch.cuda.stream(st):
                for _ in range(40):
                    outs[i].append(nk.gemm(c["x"], c["q"], kind="int8", scales=c["s"],
                                           stream=st, workspace=ws))
            st.synchronize()
        except Exception as e:  # noqa: BLE001 (reported below)
            errors.append(e)

    ts = [threading.Thread(target=worker, args=(i,)) for i in range(2)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errors, errors
    nk.device_status()
    for i, c in enumerate(cases):
        for y in outs[i]:
            assert rel_err(host(y), c["ref"]) <= 1e-3


def test_workspace_too_small_is_reported(cuda):
    c = _case(3, 16, 4096, 4096)
    m, k, n = c["shape"]
    need = nk.gemm_workspace_bytes("int8", torch.float32, m, k, n)
    small = torch.empty(need - 256, dtype=torch.uint8, device="cuda")
    with pytest.raises(nk.NkError) as e:
        nk.gemm(c["x"], c["q"], kind="int8", scales=c["s"], workspace=small)
    assert e.value.code == nk.WORKSPACE_TOO_SMALL


def test_scratch_growth_refused_during_capture(cuda):
    st = torch.cuda.Stream()
    nk.call("nk_scratch_release", st.cuda_stream)  # this stream has no block yet
    c = _case(4, 16, 4096, 4096)
    g = torch.cuda.CUDAGraph()
    with pytest.raises(nk.NkError) as e:
        with torch.cuda.graph(g, stream=st):
            nk.gemm(c["x"], c["q"], kind="int8", scales=c["s"], stream=st)
    assert e.value.code == nk.WORKSPACE_TOO_SMALL
    # after a warm-up call on the stream the same capture succeeds
    with torch.cuda.stream(st):
        nk.gemm(c["x"], c["q"], kind="int8", scales=c["s"], stream=st)
    st.synchronize()
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2, stream=st):
        y = nk.gemm(c["x"], c["q"], kind="int8", scales=c["s"], stream=st)
    g2.replay()
    torch.cuda.synchronize()
    assert rel_err(host(y), c["ref"]) <= 1e-3
