"""bench.py — MoE layer throughput (benchmark config 3) through libnk on B200.

A step is one MoeLayer forward (router GEMM -> top-6 routing -> grouped expert
GEMMs -> shared expert -> combine) over T=4096 tokens per GPU, hidden 2688,
128 experts of width 1856, shared expert 3712, bf16 weights ~ N(0, 0.02),
activations ~ N(0, 1), seeded synthetic data.  Weak scaling: every rank runs
its own 4096 tokens.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl nk|reference]
                    [--weights bf16|int8]

`--impl reference` times the reference's CPU algorithm (the committed C
restatement in oracle/, since the Rust reference cannot be built here) on
all host cores, over a bounded token sample per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "nemotron-cutile-rs_b200"))

METRIC = "grouped/quantized GEMM TFLOP/s (% tensor peak) & MoE tokens/s at 1-8 B200"
T, H, E, K, I, IS = 4096, 2688, 128, 6, 1856, 3712
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        d["source"] = "measured"
        return d
    d = dict(FALLBACK_PEAKS)
    d["source"] = "fallback"
    return d


def layer_flops(tokens):
    routed = 2 * tokens * K * (H * I + I * H)
    shared = 2 * tokens * (H * IS + IS * H)
    router = 2 * tokens * H * E
    return routed, shared, router


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.lines = []
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(gpu_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.th.join(timeout=2)
        sm, smax, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "power_w_max": max(power) if power else None,
                "samples": len(sm), "reasons": sorted(reasons)}


# ---------------------------------------------------------------- weights
def make_weights(torch, nk, dev, kind, seed=1234):
    g = torch.Generator(device=dev).manual_seed(seed)

    def randn(*shape, std=1.0):
        return torch.randn(*shape, device=dev, generator=g, dtype=torch.float32).mul_(std)

    router = randn(E, H, std=0.02)
    w = nk.MoeWeights(hidden=H, experts=E, top_k=K, inter=I, shared_inter=IS,
                      route_mode=nk.ROUTE_SIGMOID_RENORM,
                      weight_kind={"bf16": nk.W_BF16, "int8": nk.W_INT8_ROW,
                                   "int4": nk.W_INT4_AFFINE}[kind],
                      router_w3=nk.router_split(router))
    shapes = {"up": (E, I, H), "down": (E, H, I), "shared_up": (IS, H), "shared_down": (H, IS)}
    for name, shp in shapes.items():
        f = randn(*shp, std=0.02).to(torch.bfloat16)
        if kind == "bf16":
            setattr(w, f"{name}_w", f)
        elif kind == "int4":  # the reference's INT4-affine format, one scale per expert
            codes, sc, zp, _ = nk.quantize_int4_experts(f.reshape(-1, *shp[-2:]))
            setattr(w, f"{name}_w", codes if len(shp) == 3 else codes[0])
            setattr(w, f"{name}_scale", sc)
            setattr(w, f"{name}_zero_point", zp)
            del f
        else:
            q, s = nk.quantize_int8_row(f.float().reshape(-1, shp[-1]))
            setattr(w, f"{name}_w", q.reshape(shp))
            setattr(w, f"{name}_scale", s)
            del f
    host_ref = {"router": router}
    return w, host_ref


# ---------------------------------------------------------------- cpu side
def cpu_sample(weights_np, x_np, tokens, threads, orc, outputs=None):
    """Oracle MoE (the reference's algorithm, gathered rows) over `tokens` rows
    split across `threads` host threads; returns seconds.  outputs: a dict
    that receives "out" [tokens, H] and "idx" [tokens, k]."""
    from concurrent.futures import ThreadPoolExecutor

    chunks = [c for c in _split(tokens, threads) if c[1] > c[0]]
    res = {}

    def run(c):
        a, b = c
        res[a] = orc.moe(H, E, K, I, IS, weights_np["router_kn"], None, weights_np["up_kn"],
                         None, weights_np["down_kn"], None, weights_np["sup_kn"], None,
                         weights_np["sdown_kn"], None, x_np[a:b], b - a, orc.SIGMOID_RENORM)

    t0 = time.perf_counter()
    if len(chunks) == 1:
        run(chunks[0])
    else:
        with ThreadPoolExecutor(len(chunks)) as ex:
            list(ex.map(run, chunks))
    dt = time.perf_counter() - t0
    if outputs is not None:
        import numpy as np

        outputs["out"] = np.concatenate([res[c[0]][0].reshape(-1, H) for c in chunks])
        outputs["idx"] = np.concatenate([res[c[0]][1].reshape(-1, K) for c in chunks])
    return dt


def cpu_as_written(weights_np, x_np, rows, threads, orc):
    """MoeLayer::forward_into as the reference computes it (moe.rs:195-246): every
    expert selected anywhere in the batch runs its MLP over ALL the batch's rows;
    at T = 4096 tokens all 128 experts are selected, so per token that is the
    router, 128 expert MLPs and the shared expert.  Times that work for `rows`
    tokens (the 128 expert MLPs over the rows, split over `threads`); returns
    seconds per token."""
    from concurrent.futures import ThreadPoolExecutor

    xs = x_np[:rows]

    def expert(e):
        orc.mlp(H, I, weights_np["up_kn"][e], None, weights_np["down_kn"][e], None, xs, rows)

    t0 = time.perf_counter()
    orc.linear(weights_np["router_kn"], None, H, E, xs, rows)
    orc.mlp(H, IS, weights_np["sup_kn"], None, weights_np["sdown_kn"], None, xs, rows)
    with ThreadPoolExecutor(max(threads, 1)) as ex:
        list(ex.map(expert, range(E)))
    return (time.perf_counter() - t0) / rows


def cpu_info():
    model = "unknown"
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    model = ln.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu_model": model, "nproc": os.cpu_count()}


def _split(n, parts):
    return [(n * i // parts, n * (i + 1) // parts) for i in range(parts)]


def host_weights_from_numpy(seed=1234):
    """Reference-layout ([in, out]) f32 weights generated on the host."""
    import numpy as np

    r = np.random.default_rng(seed)

    def randn(*shape):
        return (r.standard_normal(shape, dtype=np.float32) * np.float32(0.02))

    return {"router_kn": randn(H, E), "up_kn": randn(E, H, I), "down_kn": randn(E, I, H),
            "sup_kn": randn(H, IS), "sdown_kn": randn(IS, H)}


def host_weights_from_device(torch, w, router):
    """The GPU arm's own weights, converted to the reference layout (bf16 weights only)."""
    def t(x, perm):
        return x.float().permute(*perm).contiguous().cpu().numpy()

    return {"router_kn": router.t().contiguous().cpu().numpy(),
            "up_kn": t(w.up_w, (0, 2, 1)), "down_kn": t(w.down_w, (0, 2, 1)),
            "sup_kn": t(w.shared_up_w, (1, 0)), "sdown_kn": t(w.shared_down_w, (1, 0))}


def calibrate_tokens(fn, budget_s, max_tokens):
    """Token count whose sample takes about budget_s seconds."""
    t2 = fn(2)
    per = max(t2 / 2, 1e-4)
    return max(2, min(max_tokens, int(budget_s / per))), per


class L2Flush:
    """Evicts L2 between timed steps: a 256 MiB write (the recipe's flush)
    followed by a 256 MiB read, so that the lines left in L2 are clean and the
    timed kernel does not pay for writing the flush's dirty lines back."""

    def __init__(self, torch, dev):
        self.w = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        self.r = torch.zeros(64 << 20, dtype=torch.float32, device=dev)
        self.acc = torch.empty((), dtype=torch.float32, device=dev)
        self.torch = torch

    def __call__(self):
        self.w.zero_()
        self.torch.sum(self.r, dim=0, out=self.acc)


def gemm_sweep(torch, nk, dev, reps=5, ms=(1, 16, 128, 2048, 8192), cublas=True):
    """Benchmark config 2: Y = X·Wᵀ over (K,N) in {(4096,4096), (4096,21504),
    (21504,4096)} and the given M, with bf16, int8-per-row and the reference's
    INT4-affine weights (nk_gemm_w4a, [K,N] nibble layout); per shape the mean
    of `reps` CUDA-event timings of a graph replay with an L2 flush before
    each; cuBLAS (torch.matmul, bf16) timed the same way for context."""
    pk = peaks()
    flush = L2Flush(torch, dev)
    g = torch.Generator(device=dev).manual_seed(5)
    res = []

    def timed(fn):
        """Device time of one call: the call is captured once into a CUDA graph
        (after a warm-up call that sizes libnk's scratch) and the graph is
        replayed, so host-side launch overhead is excluded for both libnk and
        cuBLAS."""
        side = torch.cuda.Stream()
        with torch.cuda.stream(side):  # libnk's scratch is per stream: warm up on
            fn()                        # the stream the capture uses
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            fn()
        ts = []
        for _ in range(reps + 1):
            flush()
            a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            graph.replay()
            b_.record()
            b_.synchronize()
            ts.append(a.elapsed_time(b_))
        return sum(ts[1:]) / reps

    def entry(ms_, flops, bytes_):
        return {"us": round(ms_ * 1e3, 2), "tflops": round(flops / ms_ / 1e9, 1),
                "gbs": round(bytes_ / ms_ / 1e6, 1),
                "tensor_frac": round(flops / ms_ / 1e9 / pk["bf16_tflops"], 3),
                "hbm_frac": round(bytes_ / ms_ / 1e6 / pk["hbm_gbs"], 3)}

    for (k, n) in [(4096, 4096), (4096, 21504), (21504, 4096)]:
        w = (torch.randn(n, k, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        q, s = nk.quantize_int8_row(w.float())
        _, s4, _, p4 = nk.quantize_int4_experts(w.reshape(1, n, k))  # reference [K,N] codes
        p4, s4 = p4[0], float(s4[0].item())
        for m in ms:
            x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
            row = {"m": m, "k": k, "n": n}
            flops = 2 * m * n * k
            kinds = [("bf16", 2, lambda: nk.gemm(x, w, out_dtype=torch.bfloat16)),
                     ("int8", 1, lambda: nk.gemm(x, q, kind="int8", scales=s,
                                                 out_dtype=torch.bfloat16)),
                     ("int4", 0.5, lambda: nk.gemm(x, p4, kind="int4", scale=s4, zero_point=8,
                                                   n=n, out_dtype=torch.bfloat16))]
            if cublas:
                kinds.append(("cublas_bf16", 2, lambda: torch.matmul(x, w.t())))
            for kind, wb, fn in kinds:
                bytes_ = wb * n * k + 2 * m * k + 2 * m * n
                row[kind] = entry(timed(fn), flops, bytes_)
            res.append(row)
    return res


def config1_linear(torch, nk, dev, reps=20):
    """Benchmark config 1 at its own size and seed: X f32 [64, 2048] ~ N(0,1),
    W [2048, 2048] ~ N(0, 0.02) quantized int8 per output row, Y = X·dequant(W)ᵀ
    through nk_gemm_w8row with f32 activations (CUDA events, L2 flushed)."""
    pk = peaks()
    flush = L2Flush(torch, dev)
    g = torch.Generator(device=dev).manual_seed(0)
    m, k, n = 64, 2048, 2048
    x = torch.randn(m, k, device=dev, generator=g)
    q, s = nk.quantize_int8_row(torch.randn(n, k, device=dev, generator=g) * 0.02)
    nk.gemm(x, q, kind="int8", scales=s)
    ts = []
    for _ in range(reps + 1):
        flush()
        a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        nk.gemm(x, q, kind="int8", scales=s)
        b_.record()
        b_.synchronize()
        ts.append(a.elapsed_time(b_))
    ms_ = sum(ts[1:]) / reps
    bytes_ = 4 * m * k + n * k + 4 * n + 4 * m * n
    return {"config": "benchmark config 1: int8 per-row weights, f32 X [64, 2048], "
                      "W [2048, 2048], seed 0 (eager call incl. launch)",
            "us": round(ms_ * 1e3, 2), "gbs": round(bytes_ / ms_ / 1e6, 1),
            "hbm_frac": round(bytes_ / ms_ / 1e6 / pk["hbm_gbs"], 3),
            "gflops": round(2 * m * n * k / ms_ / 1e6, 1)}


def tp_projections(torch, dev, world, reps=10):
    """Benchmark config 4's GEMMs at T=8192: Mamba2 in_proj [4096 -> 18560]
    column-parallel and out_proj [8192 -> 4096] row-parallel with one NCCL
    all-reduce of f32 partials, over the `world` ranks (strong scaling)."""
    import torch.distributed as dist

    import nk
    import nk_tp

    T_, HM, NIN, KOUT = 8192, 4096, 18560, 8192
    g = torch.Generator(device=dev).manual_seed(9)
    x = torch.randn(T_, HM, device=dev, generator=g).to(torch.bfloat16)
    w_in = (torch.randn(NIN, HM, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    w_out = (torch.randn(HM, KOUT, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    z = torch.randn(T_, KOUT, device=dev, generator=g).to(torch.bfloat16)
    if world > 1:
        col, row = nk_tp.ColumnParallelLinear(w_in), nk_tp.RowParallelLinear(w_out)
        a, b_ = row.k_range
        zs = z[:, a:b_].contiguous()
        step = lambda: (col.forward(x), row.forward(zs))  # noqa: E731
    else:
        step = lambda: (nk.gemm(x, w_in, out_dtype=torch.bfloat16),  # noqa: E731
                        nk.gemm(z, w_out, out_dtype=torch.bfloat16))
    for _ in range(3):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_.record()
    for _ in range(reps):
        step()
    e_.record()
    e_.synchronize()
    ms = s_.elapsed_time(e_) / reps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    flops = 2 * T_ * HM * NIN + 2 * T_ * KOUT * HM
    res = {"config": "Mamba2 in_proj 4096->18560 (column-parallel) + out_proj 8192->4096 "
                     "(row-parallel, NCCL all-reduce), T=8192 bf16",
           "ms": round(ms, 4), "tflops_total": round(flops / ms / 1e9, 1),
           "tflops_per_gpu": round(flops / ms / 1e9 / world, 1), "n_gpus": world}
    res["block"] = mamba_block(torch, dev, world, w_in, w_out, x, reps)
    return res


def mamba_block(torch, dev, world, w_in, w_out, x, reps):
    """The whole config-4 Mamba2 block: in_proj GEMM -> causal conv + SiLU ->
    selective scan (d_state 128, 128 heads x 64, 8 groups) -> gated RMSNorm ->
    out_proj GEMM (+ the norm's and the output's all-reduces under TP).
    Stage times come from CUDA events on the launching stream."""
    import torch.distributed as dist

    import nk
    import nk_mamba

    H, P, G, S, K = 128, 64, 8, 128, 4
    C = H * P
    g = torch.Generator(device=dev).manual_seed(11)
    conv = torch.randn(C, K, device=dev, generator=g) * 0.5
    a = -torch.rand(H, device=dev, generator=g) - 0.5
    d = torch.randn(H, device=dev, generator=g)
    nw = torch.randn(C, device=dev, generator=g)
    blk = nk_mamba.Mamba2Block(w_in, w_out, conv, a, d, nw, heads=H, head_dim=P, groups=G,
                               state=S, kernel_size=K)
    T_ = x.shape[0]
    for _ in range(3):
        blk.forward(x, 1, T_)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_.record()
    for _ in range(reps):
        blk.forward(x, 1, T_)
    e_.record()
    e_.synchronize()
    ms = s_.elapsed_time(e_) / reps
    # one more pass with events between the stages (same kernels, same stream)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
    C_l, W = blk.C, blk.width
    evs[0].record()
    fused = nk.gemm(x, blk.w_in, out_dtype=torch.float32)
    evs[1].record()
    act = nk.conv1d_ex(fused[:, C_l:2 * C_l], blk.conv_w, 1, T_, C_l, K, ld_x=W, silu=True,
                       f32_accumulate=True)
    y = torch.empty(T_, C_l, device=dev)
    fin = torch.empty(1, C_l, S, device=dev)
    base = fused.data_ptr()
    args = nk.NkScanArgs(1, T_, C_l, S, act.data_ptr(), C_l,
                         base + 4 * (2 * C_l + 2 * blk.G * S), W, P, blk.a.data_ptr(), P, 0,
                         base + 4 * 2 * C_l, base + 4 * (2 * C_l + blk.G * S), W, blk.bc_group,
                         blk.d.data_ptr(), P, None, 0.0, 1, y.data_ptr(), C_l, fin.data_ptr(), 0)
    evs[2].record()
    nk.selective_scan_ex(args)
    evs[3].record()
    normed = nk.rms_norm_rows(y, blk.norm_w, 1e-5, gate=fused[:, :C_l], out_dtype=nk.BF16)
    nk.gemm(normed, blk.w_out, out_dtype=torch.float32)
    evs[4].record()
    evs[4].synchronize()
    stages = {"in_proj": evs[0].elapsed_time(evs[1]), "conv_silu": evs[1].elapsed_time(evs[2]),
              "scan": evs[2].elapsed_time(evs[3]), "norm_out_proj": evs[3].elapsed_time(evs[4])}
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    scan_updates = T_ * C_l * S
    return {"config": "Mamba2 block (in_proj, conv+SiLU, selective scan d_state 128, gated "
                      "RMSNorm, out_proj), T=8192, hidden 4096, 128 heads x 64, 8 groups",
            "ms": round(ms, 4), "tokens_per_s": round(T_ / (ms / 1e3)),
            "stages_ms_rank0": {k: round(v, 4) for k, v in stages.items()},
            "scan_state_updates_per_s": round(scan_updates / (stages["scan"] / 1e3) / 1e9, 1),
            "scan_unit": "G state updates/s (per GPU)", "n_gpus": world}


def decoder_e2e(torch, dev, batch=64, prompt_len=1024, gen=256):
    """Benchmark config 5: the random-initialised 52-layer hybrid decoder
    (23 Mamba2, 23 MoE as config 3, 6 GQA attention; hidden 2688, vocab
    131072) on one GPU: prefill `batch` prompts of `prompt_len` random ids,
    then greedy-decode `gen` tokens per sequence reusing the KV / conv / SSM
    states.  Device time with CUDA events; tokens/s counts generated tokens."""
    import nk
    import nk_model

    cfg = nk_model.DecoderConfig()
    model = nk_model.Decoder(cfg, device=dev)
    g = torch.Generator(device=dev).manual_seed(3)
    prompt = torch.randint(0, cfg.vocab, (batch, prompt_len), device=dev, generator=g,
                           dtype=torch.int32)
    model.generate(prompt[:, :64], 4)  # warm-up: kernels, workspaces, clocks
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    state = model.new_state(batch, prompt_len + gen)
    out = torch.empty(batch, gen, dtype=torch.int32, device=dev)
    ev[0].record()
    logits = model.forward(prompt.reshape(-1).contiguous(), batch, prompt_len, state)
    tok = nk.argmax_rows(logits)
    ev[1].record()
    for step in range(gen):
        out[:, step] = tok
        if step + 1 == gen:
            break
        logits = model.forward(tok, batch, 1, state)
        tok = nk.argmax_rows(logits)
    ev[2].record()
    ev[2].synchronize()
    prefill_ms, decode_ms = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
    total = prefill_ms + decode_ms
    weights_gb = sum(t.numel() * t.element_size() for t in _decoder_tensors(model)) / 1e9
    return {"config": "52-layer hybrid decoder (pattern " + cfg.pattern + "), hidden 2688, "
                      "vocab 131072, MoE 128x1856 top-6 + shared 3712, GQA 32/2 x 128, Mamba2 "
                      "64 heads x 64, 8 groups, d_state 128; batch 64, prompt 1024, greedy 256",
            "tokens_per_s": round(batch * gen / (total / 1e3), 1),
            "prefill_ms": round(prefill_ms, 2), "decode_ms": round(decode_ms, 2),
            "prefill_tokens_per_s": round(batch * prompt_len / (prefill_ms / 1e3)),
            "decode_ms_per_step": round(decode_ms / max(gen - 1, 1), 3),
            "weights_gb": round(weights_gb, 2), "n_gpus": 1,
            "first_tokens": out[0, :8].tolist()}


def _decoder_tensors(model):
    yield model.embed
    yield model.lm_head
    for kind, layer in model.layers:
        for v in layer.raw.values():
            if v is not None:
                yield v


class EpTimer:
    """Wraps nk_ep.NkBackend and times its stages with CUDA events on the
    current stream (dispatch, grouped experts, shared + combine); the rest of
    a step is the NCCL exchange."""

    def __init__(self, be, torch):
        self.be, self.torch = be, torch
        self.ev = []

    def _mark(self, name):
        e = self.torch.cuda.Event(enable_timing=True)
        e.record()
        self.ev.append((name, e))

    def dispatch(self, x, gather=True):
        self.ev = []
        self._mark("start")
        r = self.be.dispatch(x, gather=gather)
        self._mark("dispatch")
        return r

    def experts(self, rows, seg_expert, seg_rows):
        self._mark("exchange_in")
        r = self.be.experts(rows, seg_expert, seg_rows)
        self._mark("experts")
        return r

    def experts_into(self, rows, seg_expert, seg_rows, out):
        self._mark("exchange_in")
        r = self.be.experts_into(rows, seg_expert, seg_rows, out)
        self._mark("experts")
        return r

    def shared(self, x):
        return self.be.shared(x)  # may run on a side stream: not timed separately

    def combine(self, *a):
        self._mark("exchange_out")
        r = self.be.combine(*a)
        self._mark("combine")
        return r

    def step_times(self):
        """Milliseconds per stage name on the compute stream (summed over the
        exchange phases, whose experts are timed one after the other)."""
        self.ev[-1][1].synchronize()
        out = {}
        for i in range(1, len(self.ev)):
            name = self.ev[i][0]
            out[name] = out.get(name, 0.0) + self.ev[i - 1][1].elapsed_time(self.ev[i][1])
        return out


# ---------------------------------------------------------------- profiling cases
# `bench.py --case NAME ...` runs one libnk path alone (only what its kernels
# need on the device) and prints one line of CUDA-event timings: the small,
# self-contained commands the ncu summaries under profiles/ were taken with.
def _case_timed(torch, fn, warmup, iters):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    e.synchronize()
    return s.elapsed_time(e) / max(iters, 1)


def case_mamba_block(args, torch, nk):
    import nk_mamba

    H, P, G, S, K, hid = 128, 64, 8, 128, 4, 4096
    C = H * P
    W = 2 * C + 2 * G * S + H
    g = torch.Generator(device="cuda").manual_seed(1)
    w_in = (torch.randn(W, hid, device="cuda", generator=g) * 0.02).bfloat16()
    w_out = (torch.randn(hid, C, device="cuda", generator=g) * 0.02).bfloat16()
    conv = torch.randn(C, K, device="cuda", generator=g) * 0.5
    a = -torch.rand(H, device="cuda", generator=g) - 0.5
    d = torch.randn(H, device="cuda", generator=g)
    nw = torch.randn(C, device="cuda", generator=g)
    blk = nk_mamba.Mamba2Block(w_in, w_out, conv, a, d, nw, heads=H, head_dim=P, groups=G,
                               state=S, kernel_size=K, parallel=False)
    x = torch.randn(args.tokens, hid, device="cuda", generator=g).bfloat16()
    ms = _case_timed(torch, lambda: blk.forward(x, 1, args.tokens), args.warmup, args.iters)
    print(f"mamba_block tokens={args.tokens}: {ms:.3f} ms per forward")


def case_attention(args, torch, nk):
    B, Sq, Hq, Hkv, d = args.batch, args.q_seq, 32, 2, 128
    L = args.kv_len or Sq
    cache = nk.KvCache(B, Hkv, d, ((L + 63) // 64) * 64)
    g = torch.Generator(device="cuda").manual_seed(2)
    kv = torch.randn(B * L, Hkv * d, device="cuda", generator=g).bfloat16()
    cache.append(kv, kv, L)
    q = torch.randn(B * Sq, Hq * d, device="cuda", generator=g).bfloat16()
    ws = [None]

    def run():
        o, ws[0] = nk.attention_gqa(q, cache, Sq, Hq, causal=True, workspace=ws[0])

    ms = _case_timed(torch, run, args.warmup, args.iters)
    print(f"attention batch={B} q_seq={Sq} kv_len={L}: {ms:.3f} ms per call")


def case_gemm(args, torch, nk):
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(args.m, args.k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(args.n, args.k, device="cuda", generator=g) * 0.02).bfloat16()
    ms = _case_timed(torch, lambda: nk.gemm(x, w, out_dtype=torch.bfloat16), args.warmup, args.iters)
    print(f"gemm m={args.m} k={args.k} n={args.n}: {ms * 1e3:.1f} us per call "
          f"(back to back, weights L2-resident when they fit)")


PROFILE_CASES = {"mamba_block": "case_mamba_block", "attention": "case_attention",
                 "gemm": "case_gemm"}


# ---------------------------------------------------------------- arms
def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as orc

    threads = os.cpu_count() or 1
    wnp = host_weights_from_numpy()
    x = np.random.default_rng(7).standard_normal((T, H), dtype=np.float32)
    x = x.astype(np.float32)
    n_tok, _ = calibrate_tokens(lambda n: cpu_sample(wnp, x, n, min(threads, n), orc), 20.0 /
                                max(args.steps, 1), T)
    for _ in range(args.warmup):
        cpu_sample(wnp, x, min(threads, n_tok), min(threads, n_tok), orc)
    secs = [cpu_sample(wnp, x, n_tok, min(threads, n_tok), orc) for _ in range(args.steps)]
    total = sum(secs)
    value = n_tok * args.steps / total
    # MoeLayer::forward_into as written runs every selected expert over all T
    # rows (moe.rs:195-246): timed on a small row sample, rate per token.
    aw_rows = max(2, min(8, threads))
    aw_per_tok = cpu_as_written(wnp, x, aw_rows, threads, orc)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32/f64-accumulate", "data": "synthetic",
        "config": config_dict(args, "reference"),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": min(threads, n_tok),
                         "kind": "port", **cpu_info(),
                         "sample": f"{n_tok} of {T} tokens per step, the reference's MoE host "
                                   "algorithm (oracle/nk_oracle.c, gathered rows: each token "
                                   f"through its {K} experts) over {min(threads, n_tok)} threads",
                         "as_written": {
                             "value": 1.0 / aw_per_tok, "unit": "tokens/s",
                             "cores": threads,
                             "sample": f"timed: {aw_rows} tokens through the router, all {E} "
                                       "expert MLPs and the shared expert, as moe.rs:195-246 "
                                       f"computes a {T}-token batch (every selected expert over "
                                       "all rows; all 128 are selected at this batch size)"}},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print_json(line)
    return 0


def config_dict(args, impl):
    return {"workload": "MoE layer prefill (benchmark config 3)", "tokens_per_gpu": T,
            "hidden": H, "experts": E, "top_k": K, "expert_inter": I, "shared_inter": IS,
            "routing": "sigmoid top-6 renormalised", "weights": args.weights,
            "parallelism": (f"expert-parallel x{args.gpus}: {E // max(args.gpus, 1)} experts per "
                            "rank, routed rows exchanged by "
                            + {"native": "nk_moe_forward_ep (libnk: NVLink peer stores, device "
                                         "barriers, no host sync)",
                               "peer": "NVLink peer stores (libnk kernels, Python-ordered)",
                               "nccl": "NCCL all-to-all-v"}[args.exchange]
                            if args.gpus > 1 else "single GPU, all experts"),
            "l2": "flushed between timed steps: 256 MiB written, then 256 MiB read (clean lines)",
            "launch": "CUDA graph of the nk_moe_forward call" if args.graph
                      else "eager launches",
            "impl": impl}


def nk_arm(args):
    import numpy as np
    import torch

    import nk

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev)
    nk.lib()

    w, ref = make_weights(torch, nk, dev, args.weights)
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    x = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty(T, H, device=dev, dtype=torch.float32)
    idx = torch.empty(T * K, device=dev, dtype=torch.int32)
    flush = L2Flush(torch, dev)
    x_host = x.cpu().pin_memory()
    out_host = torch.empty(T, H, dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream()
    xin = torch.empty_like(x)
    ep_timer = None
    if world == 1:
        layer = nk.MoeLayer(w)
        fwd = lambda: layer.forward(x, out=out, indices=idx)  # noqa: E731
    else:
        from nk_ep import (ExpertParallelMoe, NkBackend, PeerExpertParallelMoe,
                           local_expert_slice)

        el = E // world
        lw = nk.MoeWeights(hidden=H, experts=el, top_k=1, inter=I, shared_inter=0,
                           route_mode=w.route_mode, weight_kind=w.weight_kind,
                           router_w3=w.router_w3,
                           up_w=local_expert_slice(w.up_w, rank, world, E),
                           down_w=local_expert_slice(w.down_w, rank, world, E),
                           up_scale=None if w.up_scale is None else
                           w.up_scale.reshape(E, I)[rank * el:(rank + 1) * el].reshape(-1),
                           down_scale=None if w.down_scale is None else
                           w.down_scale.reshape(E, H)[rank * el:(rank + 1) * el].reshape(-1))
        if args.exchange == "native":
            from nk_ep import NativeExpertParallelMoe, local_layer

            ep = NativeExpertParallelMoe(w, local_layer(w, rank, world), max_tokens=T)
        else:
            ep_timer = EpTimer(NkBackend(w, lw), torch)
            if args.exchange == "nccl":
                ep = ExpertParallelMoe(ep_timer, E, H, K)
            else:
                ep = PeerExpertParallelMoe(ep_timer, E, H, K, max_tokens=T,
                                           phases=int(os.environ.get("NK_EP_PHASES", "1")))

        def fwd():
            if args.exchange == "native":
                ep.forward(x, out=out, indices=idx)
            else:
                out.copy_(ep.forward(x)[0])

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    native = world > 1 and args.exchange == "native"
    nk.set_stage_timing(world == 1 or native)  # events created during warm-up, before capture
    for _ in range(args.warmup):
        fwd()
    nk.device_status()
    barrier()

    # With --graph the step replays a CUDA graph captured from the C-ABI call
    # (the 13 kernel launches of one forward), stage-timing events included.
    if args.graph and world == 1:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fwd()
        fwd = graph.replay
    sampler = ClockSampler(local)
    time.sleep(0.2)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    stage_sum = {}
    barrier()
    for i in range(args.steps):
        flush()
        starts[i].record(stream)
        fwd()
        ends[i].record(stream)
        if world == 1:
            times = nk.moe_stage_times()
        elif native:  # the same marks; between them the exchange phases
            names = {"router": "router", "route_plan": "route_plan", "gather": "exchange_in",
                     "up_proj": "up_proj", "down_proj": "down_proj_and_return",
                     "shared_expert": "shared_wait", "combine": "combine"}
            times = {names[k2]: v for k2, v in nk.moe_stage_times().items()}
        else:
            times = ep_timer.step_times()
        for kname, v in times.items():
            stage_sum[kname] = stage_sum.get(kname, 0.0) + v
    barrier()

    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]

    # e2e: host (pinned) input -> device -> forward -> host output, every step.
    # One GPU: through the host-buffer executor (nk_moe_pipeline_*), whose
    # copies of adjacent steps overlap the forward in between.  No separate
    # L2 flush there: every step streams the experts' weights (1.3-2.6 GB, > the
    # 126 MB L2) and copies its input in fresh from the host.
    # Several GPUs: copy in, expert-parallel forward, copy out back to back on
    # one stream (the same three-stream schedule around the Python-orchestrated
    # exchange measured slower: 1.6 M against 3.5 M tokens/s at N = 2).
    if world == 1:
        nk.set_stage_timing(False)
        pstreams = [torch.cuda.Stream(dev) for _ in range(3)]
        pipe = nk.MoePipeline(layer, T, streams=pstreams)
        out_hosts = [out_host, torch.empty(T, H, dtype=torch.float32).pin_memory()]
        for i in range(max(args.warmup, 2)):
            pipe.submit(x_host, out_hosts[i % 2])
        pipe.wait()
        barrier()
        e_start = torch.cuda.Event(enable_timing=True)
        e_end = torch.cuda.Event(enable_timing=True)
        e_start.record(pstreams[0])
        pstreams[1].wait_event(e_start)
        pstreams[2].wait_event(e_start)
        for i in range(args.steps):
            pipe.submit(x_host, out_hosts[i % 2])
        e_end.record(pstreams[2])
        pipe.wait()
        barrier()
        e2e_ms = [e_start.elapsed_time(e_end)]
        pipe.close()
    elif native:
        # Native expert parallelism needs no host synchronisation, so the copies
        # of adjacent steps overlap the forward between them: host->device on
        # one stream, the forward on the compute stream, device->host on a
        # third, with two device buffers each for the input and the output.
        nk.set_stage_timing(False)
        h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        xins = [torch.empty_like(x), torch.empty_like(x)]
        outs = [torch.empty_like(out), torch.empty_like(out)]
        out_hosts = [out_host, torch.empty(T, H, dtype=torch.float32).pin_memory()]
        copied = [torch.cuda.Event() for _ in range(2)]
        computed = [torch.cuda.Event() for _ in range(2)]
        drained = [torch.cuda.Event() for _ in range(2)]
        consumed = [torch.cuda.Event() for _ in range(2)]

        def e2e_steps(n):
            for i in range(n):
                b = i % 2
                if i >= 2:
                    h2d.wait_event(consumed[b])  # the forward of step i-2 read xins[b]
                with torch.cuda.stream(h2d):
                    xins[b].copy_(x_host, non_blocking=True)
                    copied[b].record(h2d)
                stream.wait_event(copied[b])
                if i >= 2:
                    stream.wait_event(drained[b])  # outs[b] copied out by step i-2
                ep.forward(xins[b], out=outs[b], indices=idx)
                consumed[b].record(stream)
                computed[b].record(stream)
                d2h.wait_event(computed[b])
                with torch.cuda.stream(d2h):
                    out_hosts[b].copy_(outs[b], non_blocking=True)
                    drained[b].record(d2h)

        e2e_steps(max(args.warmup, 2))
        barrier()
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record(stream)
        h2d.wait_event(e_start)
        e2e_steps(args.steps)
        d2h.synchronize()
        e_end.record(d2h)
        barrier()
        e2e_ms = [e_start.elapsed_time(e_end)]
    else:
        e_starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        e_ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        barrier()
        for i in range(args.steps):
            flush()
            e_starts[i].record(stream)
            xin.copy_(x_host, non_blocking=True)
            out.copy_(ep.forward(xin)[0])
            out_host.copy_(out, non_blocking=True)
            e_ends[i].record(stream)
        barrier()
        e2e_ms = [s.elapsed_time(e) for s, e in zip(e_starts, e_ends)]
    clocks = sampler.stop()
    nk.device_status()

    total_ms = sum(step_ms)
    total_e2e = sum(e2e_ms)
    if world == 1:  # up/down stages; the shared expert runs beside them when overlapped
        grouped_ms = (stage_sum.get("up_proj", 0.0) + stage_sum.get("down_proj", 0.0) +
                      stage_sum.get("shared_expert", 0.0)) / args.steps
    elif native:  # the down stage includes the return exchange and its barrier
        grouped_ms = (stage_sum.get("up_proj", 0.0) +
                      stage_sum.get("down_proj_and_return", 0.0)) / args.steps
    else:
        grouped_ms = stage_sum.get("experts", 0.0) / args.steps
    if world > 1:
        t = torch.tensor([total_ms, total_e2e, grouped_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms, total_e2e, _ = t.tolist()

    tp_result = tp_projections(torch, dev, world) if args.tp else None
    if rank == 0:
        pk = peaks()
        wbytes_per = {"bf16": 2, "int8": 1, "int4": 0.5}[args.weights]
        if world == 1:
            counts = np.bincount(idx.cpu().numpy(), minlength=E)
            active = int((counts > 0).sum())
            rows = T * K
        else:  # this rank's experts and the rows it received in the last step
            active = E // world
            rows = (int(sum(ep.last_exchange["received_rows"])) if args.exchange == "nccl"
                    else ep.received_rows() if native else int(ep.total.item()))
        expert_w_bytes = active * 2 * I * H * wbytes_per
        act_bytes = rows * H * 2 + 2 * rows * I * 2 + rows * H * 2
        grouped_bytes = expert_w_bytes + act_bytes
        grouped_flops = 4 * rows * H * I
        if world == 1:  # the shared expert shares the window: its weights and activations
            grouped_bytes += 2 * IS * H * wbytes_per + T * H * 2 + 2 * T * IS * 2 + T * H * 2
            grouped_flops += 4 * T * H * IS
        routed, shared, router = layer_flops(T)
        tokens_total = T * world * args.steps
        value = tokens_total / (total_ms / 1e3)
        ach_gbs = grouped_bytes / (grouped_ms / 1e3) / 1e9 if grouped_ms > 0 else float("nan")
        traffic = None
        tp = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tp):
            with open(tp) as f:
                traffic = json.load(f).get(f"moe_grouped_{args.weights}") if world == 1 else None
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16" if args.weights == "bf16" else f"bf16 activations, {args.weights} weights",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights)",
            "config": config_dict(args, "nk"),
            "tflops": (routed + shared + router) * world * args.steps / (total_ms / 1e3) / 1e12,
            "tensor_frac_of_measured": ((routed + shared + router) / (total_ms / args.steps / 1e3)
                                        / 1e12) / pk["bf16_tflops"],
            "stages_ms": {k2: v / args.steps for k2, v in stage_sum.items()},
            "roofline": {
                "kernel": ("tc_gemm_kernel: grouped expert up/down projections with the shared "
                           "expert's two GEMMs running beside them (4 launches per step)"
                           if world == 1 else
                           "tc_gemm_kernel: grouped up/down projections of this rank's experts"),
                "bound": "hbm", "achieved": ach_gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": ach_gbs / pk["hbm_gbs"], "traffic": traffic,
                "peak_source": pk["source"],
                "algorithmic_bytes_per_step": grouped_bytes,
                "tensor_tflops": grouped_flops / (grouped_ms / 1e3) / 1e12,
                "tensor_frac": grouped_flops / (grouped_ms / 1e3) / 1e12 / pk["bf16_tflops"],
            },
            "e2e": {"value": tokens_total / (total_e2e / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": T * H * 2, "d2h_bytes_per_step": T * H * 4},
            "clocks": clocks,
            # libnk kernels per forward: one GPU 16 (router GEMM, router norms,
            # candidates, rescore, selection, plan count / scan / place, gather,
            # tile lists, up, down, shared up / down, combine); native expert
            # parallel 21 (no gather; counts exchange, exchange plan, capacity
            # check, dispatch, 2 barriers and return instead); the Python-ordered
            # exchanges 17.  Timed region: K steps, then K e2e steps.
            "gpu_launches": ({1: 16}.get(world, 21 if native else 17)) * args.steps * 2,
        }
        line["e2e"]["how"] = (
            "nk_moe_pipeline_submit per step (host-buffer executor: pinned x in, f32 out back; "
            "copies of adjacent steps overlap the forward; no L2 flush: each step streams "
            "all routed experts' weights, 1.3-2.6 GB > L2)"
            if world == 1 else
            "nk_moe_forward_ep per step with host->device and device->host copies on their own "
            "streams, overlapping the adjacent steps' forwards (pinned x in, f32 out back)"
            if native else "copy in, forward, copy out back to back per step")
        if world == 1 and not args.no_gemm_rows:
            line["config1_linear"] = config1_linear(torch, nk, dev)
            line["config2_gemm_rows"] = gemm_sweep(torch, nk, dev, ms=(1, 16, 128, 8192),
                                                   cublas=False)
        if args.tp:
            line["tp_projections"] = tp_result
        if args.e2e and world == 1:
            line["e2e_decoder"] = decoder_e2e(torch, dev)
        if world == 1 and args.sweep:
            line["gemm_sweep"] = gemm_sweep(torch, nk, dev)
        if world == 1 and not args.no_cpu_baseline and args.weights == "bf16":
            sys.path.insert(0, os.path.join(ROOT, "oracle"))
            import oracle as orc

            wnp = host_weights_from_device(torch, w, ref["router"])
            xs = x[:64].float().cpu().numpy()
            n_tok, _ = calibrate_tokens(lambda n: cpu_sample(wnp, xs, n, 1, orc), 15.0, 64)
            outs = {}
            secs = cpu_sample(wnp, xs, n_tok, 1, orc, outputs=outs)
            # the sample doubles as a parity check of the timed GPU forward
            gi = idx.reshape(T, K)[:n_tok].cpu().numpy()
            go = out[:n_tok].cpu().numpy()
            routes_equal = bool(np.array_equal(gi, outs["idx"]))
            rel = float(np.max(np.abs(go - outs["out"])) / np.max(np.abs(outs["out"])))
            assert routes_equal and rel <= 2e-2, (routes_equal, rel)
            aw_per_tok = cpu_as_written(wnp, xs, 2, 1, orc)
            line["cpu_baseline"] = {
                "value": n_tok / secs, "unit": "tokens/s", "cores": 1, "kind": "port",
                **cpu_info(),
                "sample": f"{n_tok} of {T} tokens: oracle/nk_oracle.c restatement of "
                          "MoeLayer::forward_into (f64-accumulate GEMM loops) on the GPU arm's "
                          "weights, single thread, gathered rows",
                "agrees_with_gpu": {"routes_equal": routes_equal, "max_rel_err": rel},
                "as_written": {"value": 1.0 / aw_per_tok, "unit": "tokens/s", "cores": 1,
                               "sample": "timed: 2 tokens through the router, all 128 expert "
                                         "MLPs and the shared expert (moe.rs:195-246 at a "
                                         "4096-token batch)"}}
        print_json(line)
    if world > 1:
        if native:
            ep.close()
        torch.distributed.destroy_process_group()
    return 0


def main():
    # Libraries (NCCL) may print to stdout; the contract is one JSON line there.
    # Keep the real stdout for that line and send everything else to stderr.
    json_fd = os.dup(1)
    os.dup2(2, 1)
    global print_json
    json_out = os.fdopen(json_fd, "w")

    def print_json(obj):
        json_out.write(json.dumps(obj) + "\n")
        json_out.flush()

    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["nk", "reference"], default="nk")
    ap.add_argument("--weights", choices=["bf16", "int8", "int4"], default="bf16")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemm-rows", action="store_true",
                    help="skip the config-1 and config-2 projection rows of the default line")
    ap.add_argument("--tokens", type=int, default=T,
                    help="tokens per GPU (profiling captures use a smaller case)")
    ap.add_argument("--experts", type=int, default=E)
    ap.add_argument("--exchange", choices=["native", "peer", "nccl"], default="native",
                    help="expert-parallel exchange: the native C-ABI executor (default), the "
                         "Python-ordered peer-store exchange, or NCCL all-to-all-v")
    ap.add_argument("--tp", action="store_true",
                    help="also time config 4's tensor-parallel projections")
    ap.add_argument("--sweep", action="store_true",
                    help="also time the config-2 dense / int8 GEMM sweep (adds ~1 min)")
    ap.add_argument("--e2e", action="store_true",
                    help="also run config 5: the 52-layer decoder, batch 64, prompt 1024, "
                         "256 greedy tokens (1 GPU; adds ~1 min)")
    ap.add_argument("--graph", action="store_true",
                    help="replay the forward as a captured CUDA graph (measured no faster "
                         "than eager launches: the step is device-bound)")
    ap.add_argument("--case", choices=sorted(PROFILE_CASES),
                    help="run one libnk path alone for profiling (see the profiles/ commands)")
    ap.add_argument("--iters", type=int, default=3, help="--case: timed calls")
    ap.add_argument("--batch", type=int, default=8, help="--case attention")
    ap.add_argument("--q-seq", type=int, default=1024, help="--case attention")
    ap.add_argument("--kv-len", type=int, default=0, help="--case attention")
    ap.add_argument("--m", type=int, default=1, help="--case gemm")
    ap.add_argument("--k", type=int, default=4096, help="--case gemm")
    ap.add_argument("--n", type=int, default=21504, help="--case gemm")
    args = ap.parse_args()
    if args.case:
        import torch

        import nk

        globals()[PROFILE_CASES[args.case]](args, torch, nk)
        return 0
    globals()["T"], globals()["E"] = args.tokens, args.experts
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return reference_arm(args)
    return nk_arm(args)


if __name__ == "__main__":
    sys.exit(main())
