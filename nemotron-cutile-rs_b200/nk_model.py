"""nk_model.py — the Nemotron-H-style hybrid decoder on libnk: embedding,
Mamba2 / MoE / GQA-attention blocks with pre-norm residuals, final norm,
lm_head and greedy decoding with KV / conv / SSM state reuse.

Structure (nemotron-model/src/model.rs:258-337, nemotron-nn/src/block.rs:
84-157): h = embedding(tokens); per block h = h + mixer(rms_norm(h)); logits
= lm_head(rms_norm(h)); the next token is the last row's argmax.  Each block's
residual add is fused with the following RMSNorm (nk_add_rms_norm_rows).

Unlike the reference, which recomputes the whole prefix for every generated
token (model.rs:281, generate.rs:48-58) and has no batch dimension, this
decoder prefills a batch of prompts once and then decodes one token per
sequence per step, reusing the attention KV cache and the Mamba conv / SSM
states.  The Mamba mixer uses the fused in_proj layout (z, x, B, C, dt per
head / group: nk_mamba.Mamba2Block); the reference's per-channel B/C layout
would need a B projection of conv_channels*state_size = 4096*128 outputs per
layer at this scale.  Weights are bf16 [out, in]; the residual stream is f32.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

import nk
import nk_mamba


@dataclass
class DecoderConfig:
    """ModelConfig (nemotron-model/src/config.rs:189-236) fields the decoder uses."""
    vocab: int = 131072
    hidden: int = 2688
    pattern: str = "MEMEM*EMEMEM*EMEMEM*EMEMEM*EMEMEM*EMEMEMEM*EMEMEMEME"
    eps: float = 1e-5
    # Mamba2
    mamba_heads: int = 64
    mamba_head_dim: int = 64
    mamba_groups: int = 8
    mamba_state: int = 128
    conv_kernel: int = 4
    # MoE
    experts: int = 128
    top_k: int = 6
    moe_inter: int = 1856
    shared_inter: int = 3712
    route_mode: int = nk.ROUTE_SIGMOID_RENORM
    # attention
    q_heads: int = 32
    kv_heads: int = 2
    head_dim: int = 128
    # init
    std: float = 0.02
    seed: int = 0
    layer_kinds: list = field(default_factory=list)

    def __post_init__(self):
        kinds = {"M": "mamba", "E": "moe", "*": "attention", "-": "mlp"}
        self.layer_kinds = [kinds[c] for c in self.pattern]


class AttentionMixer:
    """AttentionLayer (nemotron-nn/src/attention.rs:43-209) over a KV cache:
    Q/K/V projections (bf16), nk_kv_append, causal GQA attention, O projection."""

    def __init__(self, wq, wk, wv, wo, q_heads, kv_heads, head_dim):
        self.wq, self.wk, self.wv, self.wo = wq, wk, wv, wo
        self.hq, self.hkv, self.d = q_heads, kv_heads, head_dim
        self.ws = None

    def forward(self, x, batch, seq, cache: nk.KvCache, workspace=None):
        """workspace: optional one-element list holding a buffer shared by layers."""
        q = nk.gemm(x, self.wq, out_dtype=torch.bfloat16)
        k = nk.gemm(x, self.wk, out_dtype=torch.bfloat16)
        v = nk.gemm(x, self.wv, out_dtype=torch.bfloat16)
        cache.append(k, v, seq)
        slot = workspace if workspace is not None else [self.ws]
        o, slot[0] = nk.attention_gqa(q, cache, seq, self.hq, causal=True, out_dtype=nk.BF16,
                                      workspace=slot[0])
        if workspace is None:
            self.ws = slot[0]
        return nk.gemm(o, self.wo, out_dtype=torch.float32)


class Decoder:
    """Random-initialised decoder of `cfg` on one GPU (weights ~N(0, std²))."""

    def __init__(self, cfg: DecoderConfig, device="cuda", weights=None):
        self.cfg = cfg
        self.dev = device
        g = torch.Generator(device=device).manual_seed(cfg.seed)

        def randn(*shape, std=cfg.std, dtype=torch.bfloat16):
            return (torch.randn(*shape, device=device, generator=g) * std).to(dtype)

        randn.uniform = lambda *shape: torch.rand(*shape, device=device, generator=g)

        H = cfg.hidden
        w = weights or {}
        self.embed = w.get("embed", randn(cfg.vocab, H, std=1.0))
        self.lm_head = w.get("lm_head", randn(cfg.vocab, H))
        self.norms = w.get("norms", [1.0 + randn(H, std=0.1, dtype=torch.float32)
                                     for _ in range(len(cfg.layer_kinds) + 1)])
        self.moe_ws = [None]   # one workspace shared by the MoE layers
        self.attn_ws = [None]  # and one by the attention layers
        self.layers = []
        for i, kind in enumerate(cfg.layer_kinds):
            lw = w.get(("layer", i))
            if kind == "mamba":
                self.layers.append(self._mamba(lw, randn))
            elif kind == "moe":
                self.layers.append(self._moe(lw, randn))
            elif kind == "attention":
                self.layers.append(self._attention(lw, randn))
            else:
                raise ValueError(f"unsupported layer kind {kind}")

    # ---- layer construction -------------------------------------------------
    def _mamba(self, lw, randn):
        c = self.cfg
        C = c.mamba_heads * c.mamba_head_dim
        W = 2 * C + 2 * c.mamba_groups * c.mamba_state + c.mamba_heads
        lw = lw or dict(
            w_in=randn(W, c.hidden), w_out=randn(c.hidden, C),
            conv=randn(C, c.conv_kernel, std=0.5, dtype=torch.float32),
            a=-(0.5 + randn.uniform(c.mamba_heads)),
            d=randn(c.mamba_heads, std=1.0, dtype=torch.float32),
            norm=1.0 + randn(C, std=0.1, dtype=torch.float32))
        blk = nk_mamba.Mamba2Block(lw["w_in"], lw["w_out"], lw["conv"], lw["a"], lw["d"],
                                   lw["norm"], heads=c.mamba_heads, head_dim=c.mamba_head_dim,
                                   groups=c.mamba_groups, state=c.mamba_state,
                                   kernel_size=c.conv_kernel, epsilon=c.eps, parallel=False)
        blk.raw = lw
        return ("mamba", blk)

    def _moe(self, lw, randn):
        c = self.cfg
        lw = lw or dict(
            router=randn(c.experts, c.hidden, dtype=torch.float32),
            up=randn(c.experts, c.moe_inter, c.hidden), down=randn(c.experts, c.hidden, c.moe_inter),
            sup=randn(c.shared_inter, c.hidden) if c.shared_inter else None,
            sdown=randn(c.hidden, c.shared_inter) if c.shared_inter else None)
        mw = nk.MoeWeights(hidden=c.hidden, experts=c.experts, top_k=c.top_k, inter=c.moe_inter,
                           shared_inter=c.shared_inter, route_mode=c.route_mode,
                           weight_kind=nk.W_BF16, router_w3=nk.router_split(lw["router"]),
                           up_w=lw["up"], down_w=lw["down"], shared_up_w=lw["sup"],
                           shared_down_w=lw["sdown"])
        layer = nk.MoeLayer(mw)
        layer.raw = lw
        return ("moe", layer)

    def _attention(self, lw, randn):
        c = self.cfg
        qd, kvd = c.q_heads * c.head_dim, c.kv_heads * c.head_dim
        lw = lw or dict(wq=randn(qd, c.hidden), wk=randn(kvd, c.hidden),
                        wv=randn(kvd, c.hidden), wo=randn(c.hidden, qd))
        m = AttentionMixer(lw["wq"], lw["wk"], lw["wv"], lw["wo"], c.q_heads, c.kv_heads,
                           c.head_dim)
        m.raw = lw
        return ("attention", m)

    # ---- state ----------------------------------------------------------------
    def new_state(self, batch, max_len):
        """Per-layer caches: KV caches (attention), conv + SSM states (Mamba)."""
        c = self.cfg
        C = c.mamba_heads * c.mamba_head_dim
        st = []
        for kind, _ in self.layers:
            if kind == "attention":
                st.append(nk.KvCache(batch, c.kv_heads, c.head_dim,
                                     ((max_len + 63) // 64) * 64, device=self.dev))
            elif kind == "mamba":
                st.append((torch.zeros(batch, c.conv_kernel - 1, C, device=self.dev),
                           torch.zeros(batch, C, c.mamba_state, device=self.dev)))
            else:
                st.append(None)
        return st

    # ---- forward --------------------------------------------------------------
    def forward(self, tokens, batch, seq, state, logits_rows="last"):
        """tokens int32 [batch*seq] (device), appended to `state`.  Returns the
        logits (f32) of the last position of every sequence ([batch, vocab]),
        or of every row with logits_rows="all"."""
        c = self.cfg
        rows = batch * seq
        h = nk.embedding_lookup(self.embed, tokens, c.vocab, c.hidden, out_dtype=torch.float32,
                                check=False)
        h, normed = nk.add_rms_norm_rows(h, None, self.norms[0], c.eps)
        for i, ((kind, layer), st) in enumerate(zip(self.layers, state)):
            if kind == "mamba":
                m = layer.forward(normed, batch, seq, conv_state=st[0], ssm_state=st[1])
            elif kind == "moe":
                m = layer.forward(normed, out_dtype=torch.float32, workspace=self.moe_ws)
            else:
                m = layer.forward(normed, batch, seq, st, workspace=self.attn_ws)
            h, normed = nk.add_rms_norm_rows(h, m, self.norms[i + 1], c.eps)
        if logits_rows == "last" and seq > 1:
            last = normed.view(batch, seq, c.hidden)[:, -1].contiguous()
        else:
            last = normed
        return nk.gemm(last, self.lm_head, out_dtype=torch.float32)

    def generate(self, prompt, steps, max_len=None):
        """Greedy decoding: prompt int32 [batch, T] on the device; returns the
        generated ids [batch, steps] (int32, device).  No host synchronisation
        between steps."""
        batch, T = prompt.shape
        state = self.new_state(batch, max_len or T + steps)
        logits = self.forward(prompt.reshape(-1).contiguous(), batch, T, state)
        out = torch.empty(batch, steps, dtype=torch.int32, device=prompt.device)
        tok = nk.argmax_rows(logits)
        for s in range(steps):
            out[:, s] = tok
            if s + 1 == steps:
                break
            logits = self.forward(tok, batch, 1, state)
            tok = nk.argmax_rows(logits)
        return out
