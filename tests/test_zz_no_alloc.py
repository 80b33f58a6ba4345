"""The allocation-free int8-row projection (nk_gemm_w8row_f32_static).

Some callers cannot allow a library to call cudaMalloc — a host that owns all
device memory through its own pool, or a latency-critical path where an
allocation would synchronise the device.  This entry point keeps its
activation-split buffer in a fixed device array inside libnk instead.  The
test calls it through the C ABI twice in a row with different inputs and
checks each result against the oracle's LinearProjection restatement
(linear.rs:283-342, f64 sums over the dequantized int8 weights) and against
the regular entry point (nk_gemm_w8row with f32 activations), within the
f32-accumulate tolerance used by the GEMM tests; and that once its kernels
are loaded a call changes the device's free memory by nothing.  It runs last
(file name) and works alone in a fresh process as well."""
import numpy as np
import pytest
import torch

import nk
import oracle as orc

pytestmark = pytest.mark.gpu
FP32_TOL = 1e-3


def static_call(x, q, s, n, out_dtype=torch.float32, bias=None):
    m, k = x.shape
    y = torch.empty((m, n), dtype=out_dtype, device=x.device)
    nk.call("nk_gemm_w8row_f32_static", nk.ptr(x), nk.ptr(q), nk.ptr(s), nk.ptr(bias), nk.ptr(y),
            nk.F32 if out_dtype == torch.float32 else nk.BF16, m, k, n, 0, nk.stream_ptr())
    return y


def test_static_variant_matches_regular_entry_point_twice(cuda):
    g = torch.Generator(device=cuda).manual_seed(0)
    m, k, n = 64, 2048, 2048  # the single quantized linear of the benchmark configurations
    w = torch.randn(n, k, device=cuda, generator=g) * 0.02
    q, s = nk.quantize_int8_row(w)
    bias = torch.randn(n, device=cuda, generator=g)
    deq = (q.float() * s[:, None]).cpu().numpy()  # [n, k]
    for call in range(2):
        x = torch.randn(m, k, device=cuda, generator=g)
        ref = nk.gemm(x, q, kind="int8", scales=s, bias=bias)
        got = static_call(x, q, s, n, bias=bias)
        torch.cuda.synchronize()
        err = ((got - ref).abs().max() / ref.abs().max()).item()
        assert err <= FP32_TOL, (call, err)
        oracle = orc.linear(deq.T.copy(), bias.cpu().numpy(), k, n, x.cpu().numpy(), m)
        o = oracle.reshape(m, n)
        g_h = got.cpu().numpy()
        assert np.max(np.abs(g_h - o)) / np.max(np.abs(o)) <= FP32_TOL, call
    nk.device_status()


def test_static_variant_allocates_nothing(cuda):
    g = torch.Generator(device=cuda).manual_seed(5)
    n, k = 1024, 2048
    q, s = nk.quantize_int8_row(torch.randn(n, k, device=cuda, generator=g) * 0.02)
    xs = {m: torch.randn(m, k, device=cuda, generator=g) for m in (16, 200, 960)}
    ys = {m: torch.empty(m, n, device=cuda) for m in xs}

    def call(m):
        nk.call("nk_gemm_w8row_f32_static", nk.ptr(xs[m]), nk.ptr(q), nk.ptr(s), None,
                nk.ptr(ys[m]), nk.F32, m, k, n, 0, nk.stream_ptr())

    call(16)   # loads the kernels (small and large token tiles) and resolves
    call(200)  # the array's address
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    call(960)  # larger than any earlier call: 960 * 4 * 2048 bytes = 7.5 MiB
    call(960)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    ref = nk.gemm(xs[960], q, kind="int8", scales=s)
    assert ((ys[960] - ref).abs().max() / ref.abs().max()).item() <= FP32_TOL


def test_static_variant_odd_k_padding_is_rewritten(cuda):
    g = torch.Generator(device=cuda).manual_seed(1)
    for (m, k, n) in [(200, 2048, 384), (7, 80, 256)]:  # a large call, then a padded one
        w = torch.randn(n, k, device=cuda, generator=g) * 0.02
        q, s = nk.quantize_int8_row(w)
        x = torch.randn(m, k, device=cuda, generator=g)
        ref = nk.gemm(x, q, kind="int8", scales=s)
        got = static_call(x, q, s, n)
        torch.cuda.synchronize()
        assert ((got - ref).abs().max() / ref.abs().max()).item() <= FP32_TOL


def test_static_variant_rejects_oversize(cuda):
    m, k, n = 4096, 1024, 128  # 4096 * 4 * 1024 bytes = 16 MiB > 8 MiB
    x = torch.zeros(m, k, device=cuda)
    q = torch.zeros(n, k, dtype=torch.int8, device=cuda)
    s = torch.ones(n, device=cuda)
    with pytest.raises(nk.NkError) as ei:
        static_call(x, q, s, n)
    assert ei.value.variant == "WorkspaceTooSmall"
    assert ei.value.expected == m * 4 * k and ei.value.actual == 8 << 20
