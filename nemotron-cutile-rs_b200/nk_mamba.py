"""nk_mamba.py — the Mamba2 mixer on libnk: projections on the tcgen05 GEMM,
glue (conv, SiLU, selective scan, gated RMSNorm) on the glue kernels.

Two layouts, one set of kernels:

* Mamba2Mixer mirrors nemotron-nn/src/mamba2.rs (struct :75-91, forward
  :209-378): six separate projections (input, delta_t, B, C, gate, output),
  per-channel B/C of width conv_channels*state_size, per-channel dt and A,
  optional conv/SSM cache (Mamba2Cache, :36-72).  Same stage order: five
  input projections, then per batch conv(history ++ x) -> drop history ->
  SiLU -> selective scan (softplus dt, delta_bias 0) -> gated RMSNorm per row
  -> output projection; the cache is updated in place.
* Mamba2Block is the fused layout of the config-4 block: one in_proj whose
  output row is [z | x | B (ngroups*S) | C (ngroups*S) | dt (heads)], read in
  place by the glue (dt, A and D per head, B/C per group); z gates the norm
  (no SiLU, as mamba2.rs:345-351 gates with the raw gate projection) and the
  conv runs over x only, as the reference's.  Under tensor parallelism each
  rank holds whole heads and whole groups (column split of in_proj, row split
  of out_proj + one all-reduce; the norm's row mean square is all-reduced
  first, since the reference normalises over all channels of a row).

Weights are bf16 [out, in] (the projection GEMM's weight-stationary layout);
activations are f32 between stages, as in the reference.
"""
from __future__ import annotations

import torch

import nk


class Projection:
    """LinearProjection::project (linear.rs:273-342) on nk.gemm: Y = X·Wᵀ (+ b),
    W bf16 [output_dim, input_dim], f32 result (the bias is added in f32
    after the GEMM, as linear.rs:333-339)."""

    def __init__(self, w, bias=None):
        self.w = w.to(torch.bfloat16).contiguous()
        self.bias = None if bias is None else bias.float().contiguous()
        self.output_dim, self.input_dim = self.w.shape

    def project(self, x, out_dtype=torch.float32):
        xb = x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)
        return nk.gemm(xb.contiguous(), self.w, bias=self.bias, out_dtype=out_dtype)


class Mamba2Cache:
    """Mamba2Cache (mamba2.rs:36-72): conv_state [B, K-1, C], ssm_state [B, C, S]."""

    def __init__(self, batch_size, conv_channels, conv_kernel_size, state_size, device="cuda"):
        p = max(conv_kernel_size - 1, 0)
        self.conv_state = torch.zeros(batch_size, p, conv_channels, device=device)
        self.ssm_state = torch.zeros(batch_size, conv_channels, state_size, device=device)


class Mamba2Mixer:
    """Mamba2Mixer (mamba2.rs:75-378) with the reference's per-channel layout."""

    def __init__(self, hidden_size, conv_channels, state_size, conv_kernel_size, epsilon,
                 input_projection, delta_t_projection, b_projection, c_projection,
                 gate_projection, output_projection, conv_weights, ssm_a, direct_term,
                 rms_norm_weight):
        C, S = conv_channels, state_size
        for name, pr, i, o in (("input_projection", input_projection, hidden_size, C),
                               ("delta_t_projection", delta_t_projection, hidden_size, C),
                               ("b_projection", b_projection, hidden_size, C * S),
                               ("c_projection", c_projection, hidden_size, C * S),
                               ("gate_projection", gate_projection, hidden_size, C),
                               ("output_projection", output_projection, C, hidden_size)):
            if (pr.input_dim, pr.output_dim) != (i, o):  # mamba2.rs:119-154
                raise ValueError(f"{name} shape mismatch: expected ({i} -> {o}), "
                                 f"got ({pr.input_dim} -> {pr.output_dim})")
        self.hidden_size, self.C, self.S, self.K, self.eps = hidden_size, C, S, conv_kernel_size, \
            epsilon
        self.inp, self.dtp, self.bp, self.cp, self.gp, self.outp = (
            input_projection, delta_t_projection, b_projection, c_projection, gate_projection,
            output_projection)
        self.conv_w = conv_weights.float().contiguous()
        self.a = ssm_a.float().contiguous()
        self.d = None if direct_term is None else direct_term.float().contiguous()
        self.norm_w = rms_norm_weight.float().contiguous()

    def forward(self, hidden, batch, seq, cache: Mamba2Cache | None = None):
        C, S, K = self.C, self.S, self.K
        rows = batch * seq
        x = self.inp.project(hidden)
        dt = self.dtp.project(hidden)
        b = self.bp.project(hidden)
        c = self.cp.project(hidden)
        gate = self.gp.project(hidden)
        act = nk.conv1d_ex(x, self.conv_w, batch, seq, C, K, silu=True,
                           prefix=cache.conv_state if cache is not None and K > 1 else None,
                           state_out=cache.conv_state if cache is not None and K > 1 else None)
        y = torch.empty(rows, C, device=hidden.device)
        fin = cache.ssm_state if cache is not None else torch.empty(batch, C, S,
                                                                    device=hidden.device)
        args = nk.NkScanArgs(batch, seq, C, S, act.data_ptr(), C, dt.data_ptr(), C, 1,
                             self.a.data_ptr(), 1, 1, b.data_ptr(), c.data_ptr(), C * S, 1,
                             nk.ptr(self.d), 1,
                             cache.ssm_state.data_ptr() if cache is not None else None,
                             0.0, 1, y.data_ptr(), C, fin.data_ptr(), 1)
        nk.selective_scan_ex(args)
        normed = nk.rms_norm_rows(y, self.norm_w, self.eps, gate=gate, out_dtype=nk.BF16)
        return self.outp.project(normed)


class Mamba2Block:
    """The config-4 Mamba2 block in the fused layout, optionally tensor-parallel.

    in_proj W [2*C + 2*G*S + H, hidden] (rows: z, x, B, C, dt), out_proj W
    [hidden, C].  With `group` of world size N (N divides G and H), rank r
    keeps heads [r*H/N, (r+1)*H/N) (their z, x and dt rows), groups
    [r*G/N, (r+1)*G/N) (their B and C rows) and the matching columns of
    out_proj; the gated norm's row sums of squares are summed over the ranks
    (one all-reduce of T doubles), then the partial outputs with one
    all-reduce of the f32 result."""

    def __init__(self, w_in, w_out, conv_w, a_head, d_head, norm_w, *, heads, head_dim,
                 groups, state, kernel_size=4, epsilon=1e-5, group=None, parallel=True):
        import torch.distributed as dist

        H, P, G, S = heads, head_dim, groups, state
        C = H * P
        world = 1
        if parallel and dist.is_available() and dist.is_initialized():
            world = dist.get_world_size(group)
        rank = dist.get_rank(group) if world > 1 else 0
        if H % world or G % world:
            raise ValueError("heads and groups must split evenly over the ranks")
        Hl, Gl = H // world, G // world
        Cl = Hl * P
        c0 = rank * Cl
        z_rows = torch.arange(c0, c0 + Cl)
        x_rows = C + torch.arange(c0, c0 + Cl)
        b_rows = 2 * C + torch.arange(rank * Gl * S, (rank + 1) * Gl * S)
        cc_rows = 2 * C + G * S + torch.arange(rank * Gl * S, (rank + 1) * Gl * S)
        dt_rows = 2 * C + 2 * G * S + torch.arange(rank * Hl, (rank + 1) * Hl)
        rows = torch.cat([z_rows, x_rows, b_rows, cc_rows, dt_rows]).to(w_in.device)
        self.w_in = w_in.index_select(0, rows).to(torch.bfloat16).contiguous()
        self.w_out = w_out[:, c0:c0 + Cl].to(torch.bfloat16).contiguous()
        self.conv_w = conv_w[c0:c0 + Cl].float().contiguous()
        self.a = a_head[rank * Hl:(rank + 1) * Hl].float().contiguous()
        self.d = d_head[rank * Hl:(rank + 1) * Hl].float().contiguous()
        self.norm_w = norm_w[c0:c0 + Cl].float().contiguous()
        self.H, self.P, self.G, self.S, self.K, self.eps = Hl, P, Gl, S, kernel_size, epsilon
        self.C = Cl
        self.width = 2 * Cl + 2 * Gl * S + Hl
        self.world, self.group = world, group
        # Channels per B/C group on this rank: the global ratio C/G.
        self.bc_group = C // G

    def forward(self, x, batch, seq, conv_state=None, ssm_state=None, conv_f32=True):
        """x bf16 [batch*seq, hidden] -> f32 [batch*seq, hidden] (summed over ranks)."""
        import torch.distributed as dist

        C, S, K, W = self.C, self.S, self.K, self.width
        rows = batch * seq
        fused = nk.gemm(x, self.w_in, out_dtype=torch.float32)  # [rows, W]
        base = fused.data_ptr()
        act = nk.conv1d_ex(fused[:, C:2 * C], self.conv_w, batch, seq, C, K, ld_x=W, silu=True,
                           prefix=conv_state, state_out=conv_state, f32_accumulate=conv_f32)
        y = torch.empty(rows, C, device=x.device)
        fin = ssm_state if ssm_state is not None else torch.empty(batch, C, S, device=x.device)
        args = nk.NkScanArgs(
            batch, seq, C, S, act.data_ptr(), C,
            base + 4 * (2 * C + 2 * self.G * S), W, self.P,  # dt per head
            self.a.data_ptr(), self.P, 0,                     # A per head
            base + 4 * 2 * C, base + 4 * (2 * C + self.G * S), W, self.bc_group,
            self.d.data_ptr(), self.P,
            nk.ptr(ssm_state), 0.0, 1, y.data_ptr(), C, fin.data_ptr(), 0)
        nk.selective_scan_ex(args)
        if self.world > 1:
            # The norm spans all C*world channels of a row (mamba2.rs:345-351):
            # sum the per-rank f64 sums of squares first.
            ss = nk.row_sumsq(y)
            dist.all_reduce(ss, group=self.group)
            normed = nk.rms_norm_rows_presummed(y, self.norm_w, self.eps, ss, C * self.world,
                                                gate=fused[:, :C], out_dtype=nk.BF16)
        else:
            normed = nk.rms_norm_rows(y, self.norm_w, self.eps, gate=fused[:, :C],
                                      out_dtype=nk.BF16)
        out = nk.gemm(normed, self.w_out, out_dtype=torch.float32)
        if self.world > 1:
            dist.all_reduce(out, group=self.group)
        return out
