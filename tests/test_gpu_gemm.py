"""GEMM parity on the B200 through the C ABI against the CPU oracle
(gemm.rs:91-112 / linear.rs:283-342 restated).  Tolerances (stated per
test): f32 accumulate of exact (bf16-representable) inputs -> 1e-3
max|y-r|/max|r|; bf16 outputs -> 2e-2."""
import numpy as np
import pytest
import torch

import nk
import oracle as orc
from gpu_util import bf16_round, dev, host, rel_err, rng

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-3
BF16_TOL = 2e-2


def test_gemm_f32_kats(cuda, kats):
    for c in kats["gemm"]:
        lhs = dev(np.array(c["lhs"], np.float32))
        rhs = dev(np.array(c["rhs"], np.float32))
        out = torch.full((c["m"] * c["n"],), -1.0, device=cuda)  # _into overwrites
        nk.gemm_f32(lhs, rhs, c["m"], c["k"], c["n"], out=out)
        torch.cuda.synchronize()
        assert np.allclose(host(out), c["out"], atol=c["tol"], rtol=0), c["name"]


def test_gemm_f32_matches_oracle_bitwise_mostly(cuda):
    r = rng(0)
    for (m, k, n) in [(32, 32, 32), (5, 77, 9), (64, 300, 130), (1, 2048, 64)]:
        a = r.standard_normal(m * k).astype(np.float32)
        b = r.standard_normal(k * n).astype(np.float32)
        ref = orc.gemm(a, b, m, k, n)
        got = host(nk.gemm_f32(dev(a), dev(b), m, k, n))
        # f64 accumulation in another order rounds to the same f32 almost always
        assert rel_err(got, ref) <= 1e-6
        assert np.mean(got == ref) > 0.999


def test_gemm_f32_length_errors_on_device_tensors(cuda):
    lhs = torch.zeros(4, device=cuda)
    rhs = torch.zeros(4, device=cuda)
    out = torch.zeros(3, device=cuda)
    with pytest.raises(nk.NkError) as ei:
        nk.gemm_f32(lhs, rhs, 2, 2, 2, out=out)
    assert (ei.value.variant, ei.value.argument, ei.value.expected, ei.value.actual) == \
        ("LengthMismatch", "output", 4, 3)


SHAPES = [(1, 64, 128), (7, 200, 96), (16, 256, 256), (64, 512, 384), (65, 128, 130),
          (130, 320, 384), (300, 512, 200), (513, 192, 256)]


def _oracle_proj(x, w_nk, bias=None, relu2=False):
    """Y = X·Wᵀ (+b) (relu2) with the reference arithmetic (W given [N,K])."""
    m, k = x.shape
    n = w_nk.shape[0]
    y = orc.linear(w_nk.T.copy(), bias, k, n, x, m).reshape(m, n)
    if relu2:
        y = np.maximum(y, 0) ** 2
    return y


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_gemm_bf16_matches_oracle(cuda, m, k, n):
    r = rng(m * 131 + k + n)
    x = bf16_round(r.standard_normal((m, k)))
    w = bf16_round(r.standard_normal((n, k)) * 0.02)
    ref = _oracle_proj(x, w)
    y = nk.gemm(dev(x, torch.bfloat16), dev(w, torch.bfloat16), out_dtype=torch.float32)
    torch.cuda.synchronize()
    nk.device_status()
    assert rel_err(host(y), ref) <= FP32_TOL
    yb = nk.gemm(dev(x, torch.bfloat16), dev(w, torch.bfloat16), out_dtype=torch.bfloat16)
    assert rel_err(host(yb), ref) <= BF16_TOL


@pytest.mark.parametrize("m,k,n", [(3, 128, 256), (200, 256, 130)])
def test_gemm_bias_relu2_epilogue(cuda, m, k, n):
    r = rng(7)
    x = bf16_round(r.standard_normal((m, k)))
    w = bf16_round(r.standard_normal((n, k)) * 0.05)
    b = r.standard_normal(n).astype(np.float32)
    ref = _oracle_proj(x, w, b, relu2=True)
    y = nk.gemm(dev(x, torch.bfloat16), dev(w, torch.bfloat16), bias=dev(b), relu2=True)
    assert rel_err(host(y), ref) <= FP32_TOL


@pytest.mark.parametrize("m,k,n", [(64, 2048, 256), (5, 100, 64), (130, 256, 128)])
def test_gemm_f32_activations_split(cuda, m, k, n):
    r = rng(11)
    x = r.standard_normal((m, k)).astype(np.float32)
    w = bf16_round(r.standard_normal((n, k)) * 0.02)
    ref = _oracle_proj(x, w)
    y = nk.gemm(dev(x), dev(w, torch.bfloat16))
    assert rel_err(host(y), ref) <= FP32_TOL


@pytest.mark.parametrize("m,k,n", [(64, 2048, 256), (1, 512, 128), (257, 256, 384), (9, 48, 40)])
def test_gemm_int8_row(cuda, m, k, n):
    r = rng(3)
    w = (r.standard_normal((n, k)) * 0.02).astype(np.float32)
    q_ref, s_ref = orc.quantize_int8_row(w)
    q, s = nk.quantize_int8_row(dev(w))
    assert np.array_equal(host(q), q_ref) and np.array_equal(host(s), s_ref)
    deq = q_ref.astype(np.float32) * s_ref[:, None]
    for xdt in ("bf16", "f32"):
        x = r.standard_normal((m, k)).astype(np.float32)
        if xdt == "bf16":
            x = bf16_round(x)
        ref = _oracle_proj(x, deq)
        xd = dev(x, torch.bfloat16) if xdt == "bf16" else dev(x)
        y = nk.gemm(xd, q, kind="int8", scales=s)
        assert rel_err(host(y), ref) <= FP32_TOL, xdt


def test_config1_int8_linear_full_size(cuda):
    """Benchmark config 1 at its own size and seed: X f32 [64, 2048] ~ N(0,1),
    W f32 [2048, 2048] ~ N(0, 0.02), int8 per-row absmax quantization (bytes
    and scales bit-exact), Y = X·dequant(W)ᵀ within the f32-accumulate bar."""
    r = rng(0)
    x = r.standard_normal((64, 2048)).astype(np.float32)
    w = (r.standard_normal((2048, 2048)) * 0.02).astype(np.float32)
    q_ref, s_ref = orc.quantize_int8_row(w)
    q, s = nk.quantize_int8_row(dev(w))
    assert np.array_equal(host(q), q_ref) and np.array_equal(host(s), s_ref)
    ref = _oracle_proj(x, q_ref.astype(np.float32) * s_ref[:, None])
    y = nk.gemm(dev(x), q, kind="int8", scales=s)
    assert rel_err(host(y), ref) <= FP32_TOL


@pytest.mark.parametrize("m,k,n", [(64, 2048, 256), (1, 256, 64), (200, 128, 96), (3, 40, 10)])
def test_gemm_int4_reference_layout(cuda, m, k, n):
    """Linear with INT4-affine weights in the reference [K,N] layout, dequantized in-kernel."""
    r = rng(5)
    w_kn = (r.standard_normal((k, n)) * 0.02).astype(np.float32)
    scale = float(np.float32(np.abs(w_kn).max() / 7.0))
    packed_ref = orc.quantize_int4(w_kn.reshape(-1), scale, 8)
    packed = torch.empty(packed_ref.size, dtype=torch.uint8, device=cuda)
    nk.call("nk_quantize_int4", nk.ptr(dev(w_kn.reshape(-1))), k * n, scale, 8, nk.ptr(packed),
            packed.numel(), nk.stream_ptr())
    assert np.array_equal(host(packed), packed_ref)
    deq_kn = orc.dequantize_int4(packed_ref, k * n, scale, 8).reshape(k, n)
    x = bf16_round(r.standard_normal((m, k)))
    ref = orc.linear(deq_kn, None, k, n, x, m).reshape(m, n)
    y = nk.gemm(dev(x, torch.bfloat16), packed, kind="int4", scale=scale, zero_point=8, n=n)
    assert rel_err(host(y), ref) <= FP32_TOL
    xf = r.standard_normal((m, k)).astype(np.float32)
    ref = orc.linear(deq_kn, None, k, n, xf, m).reshape(m, n)
    y = nk.gemm(dev(xf), packed, kind="int4", scale=scale, zero_point=8, n=n)
    assert rel_err(host(y), ref) <= FP32_TOL


def test_gemm_large_against_torch_fp32(cuda):
    """Full-size config-2 shape checked against a torch fp32 matmul of the same bf16 values."""
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device=cuda).manual_seed(0)
    for (m, k, n) in [(2048, 4096, 4096), (128, 4096, 21504), (16, 21504, 4096)]:
        x = torch.randn(m, k, device=cuda, generator=g).to(torch.bfloat16)
        w = (torch.randn(n, k, device=cuda, generator=g) * 0.02).to(torch.bfloat16)
        ref = x.float() @ w.float().t()
        y = nk.gemm(x, w, out_dtype=torch.float32)
        err = ((y - ref).abs().max() / ref.abs().max()).item()
        assert err <= FP32_TOL, (m, k, n, err)
    nk.device_status()


def test_gemm_cta_pair_path_matches_single_cta(cuda):
    """The tcgen05 cta_group::2 path (opt-in, NK_PAIR=1) in a fresh process."""
    import os
    import subprocess
    import sys
    code = (
        "import sys; sys.path.insert(0, 'nemotron-cutile-rs_b200');"
        "import torch, nk;"
        "g = torch.Generator(device='cuda').manual_seed(0);"
        "x = torch.randn(700, 512, device='cuda', generator=g).bfloat16();"
        "w = (torch.randn(520, 512, device='cuda', generator=g) * 0.02).bfloat16();"
        "q, s = nk.quantize_int8_row(w.float());"
        "ref = x.float() @ w.float().t();"
        "y = nk.gemm(x, w);"
        "e1 = ((y - ref).abs().max() / ref.abs().max()).item();"
        "ref8 = x.float() @ (q.float() * s[:, None]).t();"
        "y8 = nk.gemm(x, q, kind='int8', scales=s);"
        "e2 = ((y8 - ref8).abs().max() / ref8.abs().max()).item();"
        "nk.device_status(); print(e1, e2)")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True,
                       env=dict(os.environ, NK_PAIR="1"), timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    e1, e2 = map(float, r.stdout.split())
    assert e1 <= FP32_TOL and e2 <= FP32_TOL


@pytest.mark.parametrize("kind", ["bf16", "int8"])
@pytest.mark.parametrize("m,k,n,xf32", [(1, 4096, 21504, False), (4, 4096, 3000, False), (16, 4096, 3000, False),
                                        (2, 21504, 512, False), (3, 1024, 333, True),
                                        (12, 2048, 64, True), (9, 8, 5, False)])
def test_decode_weight_stream_matches_oracle(cuda, kind, m, k, n, xf32):
    """Projections of <= 16 tokens take the weight-streaming kernel (gemv.cu):
    bf16 or int8-row weights, bf16 or f32 activations, split K, bias + relu2."""
    r = rng(m * 7 + k + n)
    x = r.standard_normal((m, k)).astype(np.float32)
    if not xf32:
        x = bf16_round(x)
    w = (r.standard_normal((n, k)) * 0.02).astype(np.float32)
    b = r.standard_normal(n).astype(np.float32)
    if kind == "bf16":
        wr = bf16_round(w)
        wd, scales = dev(wr, torch.bfloat16), None
    else:
        q, s = nk.quantize_int8_row(dev(w))
        wr = host(q).astype(np.float32) * host(s)[:, None]
        wd, scales = q, s
    ref = _oracle_proj(x, wr, b, relu2=True)
    xd = dev(x) if xf32 else dev(x, torch.bfloat16)
    y = nk.gemm(xd, wd, kind=kind, scales=scales, bias=dev(b), relu2=True)
    torch.cuda.synchronize()
    assert rel_err(host(y), ref) <= 1e-3
