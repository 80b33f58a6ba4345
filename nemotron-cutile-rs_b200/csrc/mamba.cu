// mamba.cu — the Mamba2 glue between in_proj and out_proj: causal depthwise
// conv (+ conv-cache history, + SiLU), selective scan, (gated) RMSNorm rows.
//
// All three are HBM- or latency-bound elementwise/recurrent kernels; none is
// GEMM-shaped, so none touches the tensor cores:
//   * conv: one thread per (row, channel), channel fastest (coalesced), K taps
//     read from L1/L2, f64 accumulation as conv1d.rs:98-113 does (bit-exact),
//     or an f32 FMA chain on request (FP64 is slow on this part).
//   * scan: sequential in time, parallel over (batch, channel, state), the
//     states in registers; the lane split and the time blocking are described
//     at scan_kernel.
//   * norm: one block per row, f64 sum of squares (rms_norm.rs:117-122),
//     correctly rounded f32 sqrt and reciprocal, then x*scale*w(*gate) with
//     separately rounded multiplies: bit-identical to the host formula up to
//     the f64 summation order.
#include <type_traits>

#include "nk_common.cuh"
#include "nk_ptx.cuh"

namespace nk {

__device__ __forceinline__ float silu_f32(float x) {
  // activations.rs:64-81: x * sigmoid(x), sigmoid in the sign-split form.
  float sig;
  if (x >= 0.0f) {
    sig = 1.0f / (1.0f + expf(-x));
  } else {
    const float z = expf(x);
    sig = z / (1.0f + z);
  }
  return x * sig;
}

__device__ __forceinline__ float softplus_f32(float v) {
  // ssm.rs:257-263
  return v > 20.0f ? v : logf(1.0f + expf(v));
}

// ---------------------------------------------------------------------- conv
template <bool SILU, bool F64>
__global__ void __launch_bounds__(256) conv_kernel(const float *__restrict__ x, int64_t ld_x,
                                                   const float *__restrict__ prefix,
                                                   const float *__restrict__ w, int K,
                                                   int64_t T, int64_t C, float *__restrict__ y,
                                                   int64_t ld_y) {
  // grid.x = row (b*T + t), grid.y * 256 + thread = channel: no 64-bit division.
  const int64_t row = blockIdx.x;
  const int64_t ch = (int64_t)blockIdx.y * blockDim.x + threadIdx.x;
  if (ch >= C) return;
  const int P = K - 1;
  const int64_t b = row / T, t = row - b * T;
  double acc = 0.0;
  float accf = 0.0f;
  for (int tap = 0; tap < K; ++tap) {
    const int64_t src = t - tap;
    float v;
    if (src >= 0) {
      v = x[(row - tap) * ld_x + ch];
    } else if (prefix) {
      v = prefix[(b * P + (P + src)) * C + ch];  // src >= -P since tap <= P
    } else {
      break;  // zero history: the reference stops at timestep < tap
    }
    const float wv = w[ch * K + (K - 1 - tap)];
    if (F64)
      acc += (double)v * (double)wv;
    else
      accf = fmaf(v, wv, accf);
  }
  float out = F64 ? (float)acc : accf;
  if (SILU) out = silu_f32(out);
  y[row * ld_y + ch] = out;
}

// Same result, KC = kernel_size fixed at compile time: a thread computes RT
// consecutive steps of one channel, loading the RT + KC - 1 inputs they need
// up front (all loads in flight at once instead of one dependent load per
// tap), then forms the RT outputs from registers.
template <bool SILU, bool F64, int KC, int RT>
__global__ void __launch_bounds__(256) conv_rows_kernel(const float *__restrict__ x,
                                                        int64_t ld_x,
                                                        const float *__restrict__ prefix,
                                                        const float *__restrict__ w, int64_t T,
                                                        int64_t C, float *__restrict__ y,
                                                        int64_t ld_y) {
  constexpr int P = KC - 1;
  const int64_t ch = (int64_t)blockIdx.y * blockDim.x + threadIdx.x;
  if (ch >= C) return;
  const int64_t b = blockIdx.z;
  const int64_t t0 = (int64_t)blockIdx.x * RT;
  float wv[KC];
#pragma unroll
  for (int j = 0; j < KC; ++j) wv[j] = w[ch * KC + j];
  // v[e] = input at step t0 - P + e; valid[e] false where there is no history.
  float v[RT + P];
  bool valid[RT + P];
#pragma unroll
  for (int e = 0; e < RT + P; ++e) {
    const int64_t t = t0 - P + e;
    valid[e] = true;
    v[e] = 0.0f;
    if (t >= T) {
      valid[e] = false;
    } else if (t >= 0) {
      v[e] = x[(b * T + t) * ld_x + ch];
    } else if (prefix) {
      v[e] = prefix[(b * P + (P + t)) * C + ch];
    } else {
      valid[e] = false;
    }
  }
#pragma unroll
  for (int r = 0; r < RT; ++r) {
    if (t0 + r >= T) break;
    double acc = 0.0;
    float accf = 0.0f;
#pragma unroll
    for (int tap = 0; tap < KC; ++tap) {
      const int e = r + P - tap;  // step t0 + r - tap
      if (valid[e]) {
        if (F64)
          acc += (double)v[e] * (double)wv[KC - 1 - tap];
        else
          accf = fmaf(v[e], wv[KC - 1 - tap], accf);
      }
    }
    float out = F64 ? (float)acc : accf;
    if (SILU) out = silu_f32(out);
    y[(b * T + t0 + r) * ld_y + ch] = out;
  }
}

// state_out[b][r] = (history ++ x)[T + r], r < P.  One thread per (b, ch),
// rows ascending, so an in-place update (state_out == prefix) reads row T+r
// before any thread overwrites it.
__global__ void conv_state_kernel(const float *__restrict__ x, int64_t ld_x,
                                  const float *prefix, int P, int64_t T, int64_t C,
                                  int64_t batch, float *state_out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= batch * C) return;
  const int64_t b = i / C, ch = i % C;
  for (int r = 0; r < P; ++r) {
    const int64_t e = T + r;  // index into history ++ x
    float v;
    if (e >= P)
      v = x[(b * T + (e - P)) * ld_x + ch];
    else
      v = prefix ? prefix[(b * P + e) * C + ch] : 0.0f;
    state_out[(b * P + r) * C + ch] = v;
  }
}

// ---------------------------------------------------------------------- scan
struct ScanDev {
  int64_t T, C, S;
  const float *x; int64_t ld_x;
  const float *dt; int64_t ld_dt; int dt_group;
  const float *a; int a_group;
  const float *b; const float *c; int64_t ld_bc; int bc_group;
  const float *d; int d_group;
  const float *init;
  float delta_bias; int softplus;
  float *y; int64_t ld_y;
  float *fin;
  unsigned long long *bad;  // first invalid (b*T+t)*C+ch, or NULL
};

// Block = 128 threads.  LPC lanes of a warp (a power of two) share one
// channel, lane `sub` owning the SPL consecutive states s0 = sub*SPL.  Time
// advances in blocks of U steps (U divides LPC):
//   * lane sub < U loads x and dt of step t0+sub once and computes softplus
//     and the per-head transition exp(dt*A) there; each step broadcasts them
//     with a shuffle, so the transcendental work is not repeated per lane;
//   * each lane keeps its partial output sum of every step of the block and
//     the LPC lanes then reduce all U sums at once: plain butterflies over
//     the lane bits >= U, then a transposing halving over the lower bits, so
//     lane sub ends holding step t0 + (sub & (U-1)) and U lanes store in
//     parallel (U-1 shuffles per step instead of log2(LPC));
//   * B and C rows of the next step are loaded before the current step.
// Accumulation: with per-state A (the reference layout) every product
// c*h is widened to f64 and summed in f64 as ssm.rs:161-163 does; with
// per-head A (the Mamba2 layout) the sum over states runs in f32 (a lane's
// SPL products pairwise, then the lane tree): FP64 issues at a small
// fraction of the FP32 rate on this part, and f32 keeps the output within
// the f32-accumulate tolerance (1e-3 relative).
template <int SPL, int LPC, int U, bool VEC, bool APS>
__global__ void __launch_bounds__(128) scan_kernel(ScanDev p) {
  using Acc = typename std::conditional<APS, double, float>::type;
  static_assert(LPC >= 1 && LPC <= 32 && U >= 1 && U <= LPC && LPC % U == 0, "lane split");
  const int lane = threadIdx.x & 31;
  const int sub = lane & (LPC - 1);
  const int gbase = lane & ~(LPC - 1);
  const int64_t ch_raw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / LPC;
  const bool live = ch_raw < p.C;
  const int64_t ch = live ? ch_raw : p.C - 1;  // dead lanes mirror the last channel
  const int64_t bi = blockIdx.y;
  const int s0 = sub * SPL;
  const int S = (int)p.S;
  const int64_t T = p.T;

  float h[SPL], av[SPL];
#pragma unroll
  for (int j = 0; j < SPL; ++j) {
    const int s = s0 + j;
    h[j] = (p.init && s < S) ? p.init[(bi * p.C + ch) * p.S + s] : 0.0f;
    av[j] = (APS && s < S) ? p.a[(ch / p.a_group) * p.S + s] : 0.0f;
  }
  const float a_head = APS ? 0.0f : p.a[ch / p.a_group];
  const float dv = p.d ? p.d[ch / p.d_group] : 0.0f;

  const float *xp = p.x + bi * T * p.ld_x + ch;
  const float *dtp = p.dt + bi * T * p.ld_dt + ch / p.dt_group;
  const int64_t bc_off = bi * T * p.ld_bc + (ch / p.bc_group) * p.S + s0;
  const float *bp = p.b + bc_off;
  const float *cp = p.c + bc_off;
  float *yp = p.y + bi * T * p.ld_y + ch;

  auto load_bc = [&](int64_t t, float *bv, float *cv) {
    const float *bq = bp + t * p.ld_bc;
    const float *cq = cp + t * p.ld_bc;
    if (VEC) {
#pragma unroll
      for (int j = 0; j < SPL; j += 4) {
        const float4 u = __ldg(reinterpret_cast<const float4 *>(bq + j));
        const float4 v = __ldg(reinterpret_cast<const float4 *>(cq + j));
        bv[j] = u.x; bv[j + 1] = u.y; bv[j + 2] = u.z; bv[j + 3] = u.w;
        cv[j] = v.x; cv[j + 1] = v.y; cv[j + 2] = v.z; cv[j + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < SPL; ++j) {
        const bool in = s0 + j < S;
        bv[j] = in ? __ldg(bq + j) : 0.0f;
        cv[j] = in ? __ldg(cq + j) : 0.0f;
      }
    }
  };

  float bn[SPL], cn[SPL];
  load_bc(0, bn, cn);
  // Lane sub < U owns step t0+sub of a block: raw x / dt, prefetched a block ahead.
  float xr_next = 0.0f, dr_next = 0.0f;
  if (sub < U && sub < T) {
    xr_next = xp[(int64_t)sub * p.ld_x];
    dr_next = dtp[(int64_t)sub * p.ld_dt];
  }

  for (int64_t t0 = 0; t0 < T; t0 += U) {
    const int nsteps = (int)(T - t0 < U ? T - t0 : U);  // uniform across the warp
    // Per-step scalars of this block (valid in lanes sub < nsteps).
    const float my_x = xr_next;
    const float my_raw = dr_next + p.delta_bias;
    {
      const int64_t tn = t0 + U + sub;
      if (sub < U && tn < T) {
        xr_next = xp[tn * p.ld_x];
        dr_next = dtp[tn * p.ld_dt];
      }
    }
    const float my_dt = p.softplus ? softplus_f32(my_raw) : my_raw;
    if (p.bad && live && sub < nsteps && (!isfinite(my_dt) || my_dt < 0.0f))
      atomicMin(p.bad, (unsigned long long)((bi * T + t0 + sub) * p.C + ch));
    const float my_tr = APS ? 0.0f : expf(my_dt * a_head);

    Acc part[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      part[u] = Acc(0);
      if (u < nsteps) {
        const float xv = __shfl_sync(0xffffffffu, my_x, gbase + u);
        const float dtv = __shfl_sync(0xffffffffu, my_dt, gbase + u);
        const float trh = APS ? 0.0f : __shfl_sync(0xffffffffu, my_tr, gbase + u);
        float bv[SPL], cv[SPL];
#pragma unroll
        for (int j = 0; j < SPL; ++j) { bv[j] = bn[j]; cv[j] = cn[j]; }
        if (t0 + u + 1 < T) load_bc(t0 + u + 1, bn, cn);
        float q[SPL];
        Acc acc = Acc(0);
#pragma unroll
        for (int j = 0; j < SPL; ++j) {
          if (VEC || s0 + j < S) {
            const float tr = APS ? expf(dtv * av[j]) : trh;
            const float mix = dtv * bv[j] * xv;
            h[j] = tr * h[j] + mix;
            q[j] = cv[j] * h[j];
            if (APS) acc += (double)q[j];
          } else {
            q[j] = 0.0f;
          }
        }
        if (!APS) {
#pragma unroll
          for (int w = 1; w < SPL; w <<= 1)
#pragma unroll
            for (int j = 0; j + w < SPL; j += 2 * w) q[j] += q[j + w];
          acc = q[0];
        }
        if (p.d && sub == 0) acc += (Acc)(dv * xv);
        part[u] = acc;
      }
    }
    // Butterflies over lane bits >= U: every lane gets the full sums over them.
#pragma unroll
    for (int o = LPC / 2; o >= U; o >>= 1)
#pragma unroll
      for (int u = 0; u < U; ++u) part[u] += __shfl_xor_sync(0xffffffffu, part[u], o);
    // Transposing halving over lane bits < U.
#pragma unroll
    for (int o = U / 2; o >= 1; o >>= 1) {
      const bool up = (sub & o) != 0;
#pragma unroll
      for (int i = 0; i < o; ++i) {
        const Acc send = up ? part[i] : part[i + o];
        const Acc keep = up ? part[i + o] : part[i];
        part[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
      }
    }
    const int mine = sub & (U - 1);
    if (live && sub < U && mine < nsteps) yp[(t0 + mine) * p.ld_y] = (float)part[0];
  }
  if (p.fin && live) {
#pragma unroll
    for (int j = 0; j < SPL; ++j)
      if (s0 + j < S) p.fin[(bi * p.C + ch) * p.S + s0 + j] = h[j];
  }
}

// --------------------------------------------------- staged scan (Mamba2 layout)
// The Mamba2 layout shares dt and A across a head and B/C across a group; when
// a block's channels lie in one head and one group, the whole block needs per
// step one B row, one C row (S = 128 floats each), its x values and one dt.
// Those are staged into shared memory U = 8 steps at a time with cp.async (3
// stages in flight), so the recurrence reads them at shared-memory latency:
//   * threads 0..U-1 compute softplus(dt) and exp(dt*A) of the chunk's steps
//     once for the block (InvalidDeltaT is checked there);
//   * a thread owns NCH channels (16 apart) and, as lane sub of 8, the states
//     32*m + 4*sub + i (m, i < 4): each float4 shared-memory read of the 8
//     lanes covers 128 contiguous bytes (no bank conflicts) and feeds NCH
//     channels;
//   * dt*B is formed once per state and step (the head's dt), then
//     mix = (dt*B)*x, h = exp(dt*A)*h + mix, and the state sum runs in f32;
//     the transposing lane reduction of scan_kernel then stores 8 steps at once.
namespace staged {
constexpr int S = 128, U = 8, STAGES = 3;
template <int CH>
struct __align__(16) Stage {
  float b[U][S];
  float c[U][S];
  float x[U][CH];
  float dt[U];
  float pad[U];  // keeps sizeof a multiple of 16
};
}  // namespace staged

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void *smem, const void *gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int NCH, int THREADS, int LPC>
__global__ void __launch_bounds__(THREADS, 256 / THREADS) scan_staged_kernel(ScanDev p) {
  using namespace staged;
  static_assert(LPC == 8 || LPC == 16, "8 or 16 lanes per channel");
  constexpr int SPL = S / LPC;           // states per lane
  constexpr int M4 = SPL / 4;            // float4 groups per lane
  constexpr int STRIDE = 4 * LPC;        // states between a lane's groups
  constexpr int GROUPS = THREADS / LPC;  // channel slots per block
  constexpr int CH = GROUPS * NCH;       // channels per block
  static_assert(U * (CH / 4) <= THREADS && U <= THREADS, "copy split");
  __shared__ Stage<CH> st[STAGES];
  __shared__ float2 s_dttr[U];
  const int tid = threadIdx.x;
  const int sub = tid & (LPC - 1);
  const int cl = tid / LPC;  // channel slot; owns channels cl + GROUPS*n
  const int64_t ch0 = (int64_t)blockIdx.x * CH;
  const int64_t bi = blockIdx.y;
  const int64_t T = p.T;
  const int64_t row0 = bi * T;

  const float a_head = p.a[ch0 / p.a_group];
  float dv[NCH];
#pragma unroll
  for (int n = 0; n < NCH; ++n) dv[n] = p.d ? p.d[(ch0 + cl + GROUPS * n) / p.d_group] : 0.0f;
  const float *bsrc = p.b + row0 * p.ld_bc + (ch0 / p.bc_group) * S;
  const float *csrc = p.c + row0 * p.ld_bc + (ch0 / p.bc_group) * S;
  const float *xsrc = p.x + row0 * p.ld_x + ch0;
  const float *dsrc = p.dt + row0 * p.ld_dt + ch0 / p.dt_group;

  auto issue = [&](int64_t k) {
    const int64_t t0 = k * U;
    Stage<CH> &g = st[k % STAGES];
    const int n = (int)(T - t0 < U ? T - t0 : U);
    // B and C: n rows x 32 pieces of 16 bytes each (index bits: row | which | piece).
#pragma unroll
    for (int i = tid; i < U * 2 * (S / 4); i += THREADS) {
      const int r = i / (2 * (S / 4)), which = (i / (S / 4)) & 1, q = i % (S / 4);
      if (r < n) {
        const float *src = (which ? csrc : bsrc) + (t0 + r) * p.ld_bc + q * 4;
        cp_async16(which ? &g.c[r][q * 4] : &g.b[r][q * 4], src);
      }
    }
    if (tid < U * (CH / 4)) {
      const int r = tid / (CH / 4), q = tid % (CH / 4);
      if (r < n) cp_async16(&g.x[r][q * 4], xsrc + (t0 + r) * p.ld_x + q * 4);
    }
    if (tid >= THREADS - U && tid - (THREADS - U) < n) {
      const int r = tid - (THREADS - U);
      cp_async4(&g.dt[r], dsrc + (t0 + r) * p.ld_dt);
    }
  };

  float h[NCH][SPL];
#pragma unroll
  for (int n = 0; n < NCH; ++n)
#pragma unroll
    for (int m = 0; m < M4; ++m) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (p.init)
        v = *reinterpret_cast<const float4 *>(
            p.init + (bi * p.C + ch0 + cl + GROUPS * n) * S + STRIDE * m + 4 * sub);
      h[n][4 * m] = v.x; h[n][4 * m + 1] = v.y; h[n][4 * m + 2] = v.z; h[n][4 * m + 3] = v.w;
    }

  const int64_t chunks = (T + U - 1) / U;
  issue(0);
  cp_async_commit();
  if (chunks > 1) issue(1);
  cp_async_commit();
  for (int64_t k = 0; k < chunks; ++k) {
    if (k + 2 < chunks) issue(k + 2);
    cp_async_commit();
    cp_async_wait<STAGES - 1>();
    __syncthreads();
    const Stage<CH> &g = st[k % STAGES];
    const int64_t t0 = k * U;
    const int nsteps = (int)(T - t0 < U ? T - t0 : U);
    if (tid < nsteps) {
      const float raw = g.dt[tid] + p.delta_bias;
      const float dtv = p.softplus ? softplus_f32(raw) : raw;
      if (p.bad && (!isfinite(dtv) || dtv < 0.0f)) {
        // Every channel of the block shares this dt: the first in t-major
        // order is the block's first channel.
        atomicMin(p.bad, (unsigned long long)((row0 + t0 + tid) * p.C + ch0));
      }
      s_dttr[tid] = make_float2(dtv, expf(dtv * a_head));
    }
    __syncthreads();

    float part[NCH][U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
#pragma unroll
      for (int n = 0; n < NCH; ++n) part[n][u] = 0.0f;
      if (u < nsteps) {
        const float2 dttr = s_dttr[u];
        const float dtv = dttr.x, tr = dttr.y;
        float xv[NCH];
#pragma unroll
        for (int n = 0; n < NCH; ++n) xv[n] = g.x[u][cl + GROUPS * n];
        float q[NCH][4];
#pragma unroll
        for (int n = 0; n < NCH; ++n) q[n][0] = q[n][1] = q[n][2] = q[n][3] = 0.0f;
#pragma unroll
        for (int m = 0; m < M4; ++m) {
          const float4 bv = *reinterpret_cast<const float4 *>(&g.b[u][STRIDE * m + 4 * sub]);
          const float4 cv = *reinterpret_cast<const float4 *>(&g.c[u][STRIDE * m + 4 * sub]);
          const float db[4] = {dtv * bv.x, dtv * bv.y, dtv * bv.z, dtv * bv.w};
          const float cc[4] = {cv.x, cv.y, cv.z, cv.w};
#pragma unroll
          for (int n = 0; n < NCH; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              float &hs = h[n][4 * m + i];
              hs = tr * hs + db[i] * xv[n];
              q[n][i] += cc[i] * hs;
            }
        }
#pragma unroll
        for (int n = 0; n < NCH; ++n) {
          float acc = (q[n][0] + q[n][1]) + (q[n][2] + q[n][3]);
          if (p.d && sub == 0) acc += dv[n] * xv[n];
          part[n][u] = acc;
        }
      }
    }
    // Butterflies over lane bits >= U, then the transposing halving.
#pragma unroll
    for (int o = LPC / 2; o >= U; o >>= 1)
#pragma unroll
      for (int n = 0; n < NCH; ++n)
#pragma unroll
        for (int u = 0; u < U; ++u) part[n][u] += __shfl_xor_sync(0xffffffffu, part[n][u], o);
#pragma unroll
    for (int o = U / 2; o >= 1; o >>= 1) {
      const bool up = (sub & o) != 0;
#pragma unroll
      for (int n = 0; n < NCH; ++n)
#pragma unroll
        for (int i = 0; i < o; ++i) {
          const float send = up ? part[n][i] : part[n][i + o];
          const float keep = up ? part[n][i + o] : part[n][i];
          part[n][i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    if (sub < U && sub < nsteps) {
#pragma unroll
      for (int n = 0; n < NCH; ++n)
        p.y[(row0 + t0 + sub) * p.ld_y + ch0 + cl + GROUPS * n] = part[n][0];
    }
    __syncthreads();  // stage k % STAGES is refilled by the next iteration's issue
  }
  cp_async_wait<0>();
  if (p.fin) {
#pragma unroll
    for (int n = 0; n < NCH; ++n)
#pragma unroll
      for (int m = 0; m < M4; ++m)
        *reinterpret_cast<float4 *>(p.fin + (bi * p.C + ch0 + cl + GROUPS * n) * S + STRIDE * m +
                                    4 * sub) =
            make_float4(h[n][4 * m], h[n][4 * m + 1], h[n][4 * m + 2], h[n][4 * m + 3]);
  }
}

// ---------------------------------------------------------------------- norm
// Block-wide f64 sum over 256 threads (result valid in every thread).
__device__ __forceinline__ double block_sum_256(double v) {
  __shared__ double part[8];
  __shared__ double total;
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < 8; ++i) t += part[i];
    total = t;
  }
  __syncthreads();
  return total;
}

// presum == NULL: the row's own f64 sum of squares over W; else presum[row]
// is the sum over the full row of total_w elements (the row split over
// tensor-parallel ranks, summed by an all-reduce).
template <bool GATE, bool BF16>
__global__ void __launch_bounds__(256) rms_rows_kernel(const float *__restrict__ x, int64_t ld_x,
                                                       const float *__restrict__ w,
                                                       const float *__restrict__ g,
                                                       int64_t ld_g, int64_t W, float eps,
                                                       const double *__restrict__ presum,
                                                       int64_t total_w, void *__restrict__ out,
                                                       int64_t ld_out) {
  const int64_t row = blockIdx.x;
  const float *xr = x + row * ld_x;
  double tot;
  if (presum) {
    tot = presum[row];
  } else {
    double sum = 0.0;
    for (int64_t i = threadIdx.x; i < W; i += blockDim.x) sum += (double)xr[i] * (double)xr[i];
    tot = block_sum_256(sum);
  }
  // rms_norm.rs:117-123: mean square in f64, cast to f32, + eps, sqrt, reciprocal.
  const float denom = sqrtf((float)(tot / (double)total_w) + eps);
  const float scale = 1.0f / denom;
  for (int64_t i = threadIdx.x; i < W; i += blockDim.x) {
    float v = __fmul_rn(__fmul_rn(xr[i], scale), w[i]);
    if (GATE) v = __fmul_rn(v, g[row * ld_g + i]);
    if (BF16)
      reinterpret_cast<__nv_bfloat16 *>(out)[row * ld_out + i] = __float2bfloat16_rn(v);
    else
      reinterpret_cast<float *>(out)[row * ld_out + i] = v;
  }
}

__global__ void __launch_bounds__(256) row_sumsq_kernel(const float *__restrict__ x, int64_t ld_x,
                                                        int64_t W, double *__restrict__ out) {
  const float *xr = x + (int64_t)blockIdx.x * ld_x;
  double sum = 0.0;
  for (int64_t i = threadIdx.x; i < W; i += blockDim.x) sum += (double)xr[i] * (double)xr[i];
  sum = block_sum_256(sum);
  if (threadIdx.x == 0) out[blockIdx.x] = sum;
}

// ---------------------------------------------------------------- launchers
static nk_status launch_conv(const nk_conv_args &a, cudaStream_t s) {
  const int64_t rows = a.batch * a.seq;
  constexpr int RT = 8;
  if (rows > 0 && a.kernel_size == 4 && a.batch <= 65535 && ceil_div(a.channels, 256) <= 65535) {
    const dim3 grid((unsigned)ceil_div(a.seq, RT), (unsigned)ceil_div(a.channels, 256),
                    (unsigned)a.batch);
    auto kern = a.silu ? (a.f32_accumulate ? conv_rows_kernel<true, false, 4, RT>
                                           : conv_rows_kernel<true, true, 4, RT>)
                       : (a.f32_accumulate ? conv_rows_kernel<false, false, 4, RT>
                                           : conv_rows_kernel<false, true, 4, RT>);
    kern<<<grid, 256, 0, s>>>(a.x, a.ld_x, a.prefix, a.weights, a.seq, a.channels, a.y, a.ld_y);
    nk_status st = check_launch("conv_rows_kernel");
    if (st != NK_OK) return st;
  } else if (rows > 0) {
    if (rows > 0x7fffffff || ceil_div(a.channels, 256) > 65535)
      return fail(NK_UNSUPPORTED, "conv1d: rows < 2^31 and channels < 2^24");
    const dim3 grid((unsigned)rows, (unsigned)ceil_div(a.channels, 256));
    auto kern = a.silu ? (a.f32_accumulate ? conv_kernel<true, false> : conv_kernel<true, true>)
                       : (a.f32_accumulate ? conv_kernel<false, false> : conv_kernel<false, true>);
    kern<<<grid, 256, 0, s>>>(a.x, a.ld_x, a.prefix, a.weights, (int)a.kernel_size, a.seq,
                              a.channels, a.y, a.ld_y);
    nk_status st = check_launch("conv_kernel");
    if (st != NK_OK) return st;
  }
  if (a.state_out && a.kernel_size > 1 && a.batch * a.channels > 0) {
    conv_state_kernel<<<(unsigned)ceil_div(a.batch * a.channels, 256), 256, 0, s>>>(
        a.x, a.ld_x, a.prefix, (int)a.kernel_size - 1, a.seq, a.channels, a.batch, a.state_out);
    return check_launch("conv_state_kernel");
  }
  return ok();
}

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <int SPL, int LPC, int U>
static void scan_dispatch(const ScanDev &p, bool vec, bool aps, dim3 grid, cudaStream_t s) {
  if (vec) {
    if (aps) scan_kernel<SPL, LPC, U, true, true><<<grid, 128, 0, s>>>(p);
    else scan_kernel<SPL, LPC, U, true, false><<<grid, 128, 0, s>>>(p);
  } else {
    if (aps) scan_kernel<SPL, LPC, U, false, true><<<grid, 128, 0, s>>>(p);
    else scan_kernel<SPL, LPC, U, false, false><<<grid, 128, 0, s>>>(p);
  }
}

static nk_status launch_scan(const nk_scan_args &a, cudaStream_t s) {
  if (a.batch <= 0 || a.seq <= 0 || a.channels <= 0 || a.states <= 0)
    return fail(NK_INVALID_SHAPE, "selective scan needs batch, seq, channels, states > 0");
  if (a.states > 512) return fail(NK_UNSUPPORTED, "selective scan supports states <= 512");
  if (!a.x || !a.dt || !a.a || !a.b || !a.c || !a.y)
    return fail(NK_INVALID_PARAMS, "x, dt, a, b, c, y are required");
  if (a.dt_group <= 0 || a.a_group <= 0 || a.bc_group <= 0 || (a.d && a.d_group <= 0))
    return fail(NK_INVALID_PARAMS, "group sizes must be >= 1");
  // Lane split by state count (SPL states per lane, LPC lanes per channel):
  // 16 states per lane up to S = 128 (8 lanes), then 16 or 32 lanes.
  // Probes (tuning and tests): NK_SCAN_CFG=8 selects 8 states x 16 lanes at
  // S <= 128, =1 the generic kernel where the staged one applies, =2 the
  // staged kernel with one channel per thread, =3 with 128-thread blocks,
  // =4 / =5 with 16 lanes per channel (128 / 64 threads).
  int spl = 16, lpc;
  if (a.states <= 16) lpc = 1;
  else if (a.states <= 32) lpc = 2;
  else if (a.states <= 64) lpc = 4;
  else if (a.states <= 128) lpc = 8;
  else if (a.states <= 256) lpc = 16;
  else lpc = 32;
  const char *env = getenv("NK_SCAN_CFG");
  if (env && atoi(env) == 8 && a.states > 64 && a.states <= 128) {
    spl = 8;
    lpc = 16;
  }
  const bool vec = (a.states % spl == 0) && (a.ld_bc % 4 == 0) && aligned16(a.b) &&
                   aligned16(a.c);

  ScanDev p;
  p.T = a.seq; p.C = a.channels; p.S = a.states;
  p.x = a.x; p.ld_x = a.ld_x;
  p.dt = a.dt; p.ld_dt = a.ld_dt; p.dt_group = a.dt_group;
  p.a = a.a; p.a_group = a.a_group;
  p.b = a.b; p.c = a.c; p.ld_bc = a.ld_bc; p.bc_group = a.bc_group;
  p.d = a.d; p.d_group = a.d ? a.d_group : 1;
  p.init = a.initial_state;
  p.delta_bias = a.delta_bias; p.softplus = a.softplus;
  p.y = a.y; p.ld_y = a.ld_y;
  p.fin = a.final_state;
  p.bad = nullptr;
  if (a.check_delta_t) {
    void *buf = nullptr;
    nk_status st = scratch(sizeof(unsigned long long), &buf, s);
    if (st != NK_OK) return st;
    p.bad = reinterpret_cast<unsigned long long *>(buf);
    NK_CUDA_TRY(cudaMemsetAsync(p.bad, 0xFF, sizeof(unsigned long long), s));
  }
  const dim3 grid((unsigned)ceil_div(a.channels * lpc, 128), (unsigned)a.batch);
  const bool aps = a.a_per_state != 0;
  // Staged kernel: NCH channels per thread, LPC lanes per channel slot, all
  // of a block's channels in one dt/A head and one B/C group.  Default: 2
  // channels per thread, 8 lanes, 64-thread blocks (16 channels per block).
  int nch = 2, threads = 64, slpc = 8;
  if (env && atoi(env) == 2) nch = 1;
  if (env && atoi(env) == 3) threads = 128;
  if (env && atoi(env) == 4) { slpc = 16; threads = 128; }
  if (env && atoi(env) == 5) slpc = 16;
  auto staged_fits = [&](int nc, int th, int lp) {
    const int64_t ch = (int64_t)(th / lp) * nc;
    return !aps && a.states == staged::S && a.channels % ch == 0 && a.dt_group % ch == 0 &&
           a.a_group % ch == 0 && a.bc_group % ch == 0 && a.ld_bc % 4 == 0 &&
           a.ld_x % 4 == 0 && aligned16(a.b) && aligned16(a.c) && aligned16(a.x) &&
           (!a.initial_state || aligned16(a.initial_state)) &&
           (!a.final_state || aligned16(a.final_state)) && !(env && atoi(env) == 1);
  };
  if (!staged_fits(nch, threads, slpc)) {
    nch = 1;
    threads = 64;
    slpc = 8;
  }
  if (staged_fits(nch, threads, slpc)) {
    const dim3 g((unsigned)(a.channels / ((threads / slpc) * nch)), (unsigned)a.batch);
    if (slpc == 16 && threads == 128)
      scan_staged_kernel<2, 128, 16><<<g, 128, 0, s>>>(p);
    else if (slpc == 16)
      scan_staged_kernel<2, 64, 16><<<g, 64, 0, s>>>(p);
    else if (nch == 2 && threads == 128)
      scan_staged_kernel<2, 128, 8><<<g, 128, 0, s>>>(p);
    else if (nch == 2)
      scan_staged_kernel<2, 64, 8><<<g, 64, 0, s>>>(p);
    else
      scan_staged_kernel<1, 64, 8><<<g, 64, 0, s>>>(p);
  }
  else if (spl == 8) scan_dispatch<8, 16, 8>(p, vec, aps, grid, s);
  else if (lpc == 1) scan_dispatch<16, 1, 1>(p, vec, aps, grid, s);
  else if (lpc == 2) scan_dispatch<16, 2, 2>(p, vec, aps, grid, s);
  else if (lpc == 4) scan_dispatch<16, 4, 4>(p, vec, aps, grid, s);
  else if (lpc == 8) scan_dispatch<16, 8, 8>(p, vec, aps, grid, s);
  else if (lpc == 16) scan_dispatch<16, 16, 8>(p, vec, aps, grid, s);
  else scan_dispatch<16, 32, 8>(p, vec, aps, grid, s);
  nk_status st = check_launch("scan_kernel");
  if (st != NK_OK || !a.check_delta_t) return st;

  unsigned long long h = 0;
  NK_CUDA_TRY(cudaMemcpyAsync(&h, p.bad, sizeof(h), cudaMemcpyDeviceToHost, s));
  NK_CUDA_TRY(cudaStreamSynchronize(s));
  if (h != ~0ull) {
    // Recompute the offending dt on the host from the device value.
    const int64_t ch = (int64_t)(h % (unsigned long long)a.channels);
    const int64_t row = (int64_t)(h / (unsigned long long)a.channels);
    float raw = 0.0f;
    NK_CUDA_TRY(cudaMemcpy(&raw, a.dt + row * a.ld_dt + ch / a.dt_group, sizeof(float),
                           cudaMemcpyDeviceToHost));
    raw += a.delta_bias;
    const float dtv = a.softplus ? (raw > 20.0f ? raw : logf(1.0f + expf(raw))) : raw;
    nk_status e = fail(NK_INVALID_DELTA_T, "delta_t must be finite and >= 0");
    tls_error().index = h;
    tls_error().value = dtv;
    return e;
  }
  return ok();
}

static nk_status launch_rms_rows(const float *x, int64_t rows, int64_t width, int64_t ld_x,
                                 const float *w, const float *g, int64_t ld_g, float eps,
                                 const double *presum, int64_t total_w, void *out,
                                 int64_t ld_out, int out_dtype, cudaStream_t s) {
  if (rows == 0) return ok();
  if (rows > 0x7fffffff) return fail(NK_UNSUPPORTED, "rms norm rows < 2^31");
  const bool bf = out_dtype == NK_DTYPE_BF16;
  const dim3 grid((unsigned)rows);
  auto kern = g ? (bf ? rms_rows_kernel<true, true> : rms_rows_kernel<true, false>)
                : (bf ? rms_rows_kernel<false, true> : rms_rows_kernel<false, false>);
  kern<<<grid, 256, 0, s>>>(x, ld_x, w, g, ld_g, width, eps, presum, total_w, out, ld_out);
  return check_launch("rms_rows_kernel");
}

static nk_status fail_eps(float eps) {
  nk_status e = fail(NK_NEGATIVE_EPSILON, "epsilon must be >= 0");
  tls_error().value = eps;
  return e;
}

}  // namespace nk

using namespace nk;

extern "C" {

nk_status nk_conv1d(const float *input, size_t input_len, const float *weights,
                    size_t weights_len, int64_t seq, int64_t channels, int64_t kernel_size,
                    float *out, size_t out_len, void *stream) {
  // conv1d.rs:126-158 validation order.
  if (seq < 0 || channels <= 0 || kernel_size <= 0)
    return fail(NK_INVALID_SHAPE, "conv1d needs channel_count > 0 and kernel_size > 0");
  const uint64_t n = (uint64_t)seq * (uint64_t)channels;
  if (input_len != n) return fail_length("input", n, input_len);
  if (weights_len != (uint64_t)channels * (uint64_t)kernel_size)
    return fail_length("weights", (uint64_t)channels * kernel_size, weights_len);
  if (out_len != n) return fail_length("output", n, out_len);
  nk_conv_args a{};
  a.batch = 1; a.seq = seq; a.channels = channels; a.kernel_size = kernel_size;
  a.x = input; a.ld_x = channels; a.weights = weights; a.prefix = nullptr; a.silu = 0;
  a.y = out; a.ld_y = channels; a.state_out = nullptr;
  return launch_conv(a, as_stream(stream));
}

nk_status nk_conv1d_ex(const nk_conv_args *args, void *stream) {
  if (!args) return fail(NK_INVALID_PARAMS, "args");
  const nk_conv_args &a = *args;
  if (a.batch < 0 || a.seq < 0 || a.channels <= 0 || a.kernel_size <= 0)
    return fail(NK_INVALID_SHAPE, "conv1d needs channels > 0, kernel_size > 0, batch/seq >= 0");
  if (a.ld_x < a.channels || a.ld_y < a.channels)
    return fail(NK_INVALID_PARAMS, "row strides must be >= channels");
  if (a.batch * a.seq > 0 && (!a.x || !a.y || !a.weights))
    return fail(NK_INVALID_PARAMS, "x, weights, y are required");
  return launch_conv(a, as_stream(stream));
}

nk_status nk_selective_scan(const float *input, size_t input_len, const float *delta_t,
                            size_t delta_t_len, const float *a, size_t a_len, const float *b,
                            size_t b_len, const float *c, size_t c_len, const float *d,
                            size_t d_len, const float *initial_state, size_t initial_state_len,
                            float delta_bias, int32_t apply_softplus, int64_t seq,
                            int64_t channels, int64_t states, float *out, size_t out_len,
                            float *final_state, size_t final_state_len, void *stream) {
  // ssm.rs:177-245 validation order.
  if (seq <= 0 || channels <= 0 || states <= 0)
    return fail(NK_INVALID_SHAPE, "selective scan needs sequence_len, channel_count, state_size > 0");
  const uint64_t n = (uint64_t)seq * channels, sm = (uint64_t)channels * states,
                 bl = (uint64_t)seq * channels * states;
  if (input_len != n) return fail_length("input", n, input_len);
  if (delta_t_len != n) return fail_length("delta_t", n, delta_t_len);
  if (a_len != sm) return fail_length("a", sm, a_len);
  if (b_len != bl) return fail_length("b", bl, b_len);
  if (c_len != bl) return fail_length("c", bl, c_len);
  if (d && d_len != (uint64_t)channels) return fail_length("d", channels, d_len);
  if (initial_state && initial_state_len != sm)
    return fail_length("initial_state", sm, initial_state_len);
  if (out_len != n) return fail_length("output", n, out_len);
  if (final_state_len != sm) return fail_length("final_state", sm, final_state_len);
  nk_scan_args s{};
  s.batch = 1; s.seq = seq; s.channels = channels; s.states = states;
  s.x = input; s.ld_x = channels;
  s.dt = delta_t; s.ld_dt = channels; s.dt_group = 1;
  s.a = a; s.a_group = 1; s.a_per_state = 1;
  s.b = b; s.c = c; s.ld_bc = channels * states; s.bc_group = 1;
  s.d = d; s.d_group = 1;
  s.initial_state = initial_state;
  s.delta_bias = delta_bias; s.softplus = apply_softplus;
  s.y = out; s.ld_y = channels;
  s.final_state = final_state;
  s.check_delta_t = 1;
  return launch_scan(s, as_stream(stream));
}

nk_status nk_selective_scan_ex(const nk_scan_args *args, void *stream) {
  if (!args) return fail(NK_INVALID_PARAMS, "args");
  return launch_scan(*args, as_stream(stream));
}

nk_status nk_rms_norm(const float *input, size_t len, const float *weight, size_t weight_len,
                      const float *gate, size_t gate_len, float epsilon, float *out,
                      size_t out_len, void *stream) {
  // rms_norm.rs:146-183 then rms_host :108-115.
  if (len == 0) return fail(NK_EMPTY_INPUT, "rms norm input is empty");
  if (weight_len != len) return fail_length("weight", len, weight_len);
  if (gate && gate_len != len) return fail_length("gate", len, gate_len);
  if (out_len != len) return fail_length("output", len, out_len);
  if (epsilon < 0.0f) return fail_eps(epsilon);
  return launch_rms_rows(input, 1, (int64_t)len, (int64_t)len, weight, gate, (int64_t)len,
                         epsilon, nullptr, (int64_t)len, out, (int64_t)len, NK_DTYPE_F32,
                         as_stream(stream));
}

nk_status nk_rms_norm_rows(const float *x, int64_t rows, int64_t width, int64_t ld_x,
                           const float *weight, size_t weight_len, const float *gate,
                           int64_t ld_gate, float epsilon, void *out, int64_t ld_out,
                           int32_t out_dtype, void *stream) {
  // rms_norm.rs:186-218 (validate_tensor_lengths) order.
  if (rows < 0 || width < 0) return fail(NK_INVALID_SHAPE, "rows, width >= 0");
  if (rows * width == 0) return fail(NK_EMPTY_INPUT, "rms norm input is empty");
  if (epsilon < 0.0f) return fail_eps(epsilon);
  if (weight_len != (uint64_t)width) return fail_length("weight", width, weight_len);
  if (ld_x < width || ld_out < width || (gate && ld_gate < width))
    return fail(NK_INVALID_PARAMS, "row strides must be >= width");
  if (out_dtype != NK_DTYPE_F32 && out_dtype != NK_DTYPE_BF16)
    return fail(NK_INVALID_PARAMS, "out_dtype must be NK_DTYPE_F32 or NK_DTYPE_BF16");
  return launch_rms_rows(x, rows, width, ld_x, weight, gate, ld_gate, epsilon, nullptr, width,
                         out, ld_out, out_dtype, as_stream(stream));
}

nk_status nk_row_sumsq(const float *x, int64_t rows, int64_t width, int64_t ld_x, double *sumsq,
                       void *stream) {
  if (rows < 0 || width <= 0 || ld_x < width) return fail(NK_INVALID_SHAPE, "rows >= 0, 0 < width <= ld_x");
  if (rows == 0) return ok();
  if (rows > 0x7fffffff) return fail(NK_UNSUPPORTED, "rows < 2^31");
  row_sumsq_kernel<<<(unsigned)rows, 256, 0, as_stream(stream)>>>(x, ld_x, width, sumsq);
  return check_launch("row_sumsq_kernel");
}

nk_status nk_rms_norm_rows_presummed(const float *x, int64_t rows, int64_t width, int64_t ld_x,
                                     const float *weight, size_t weight_len, const float *gate,
                                     int64_t ld_gate, const double *sumsq, int64_t total_width,
                                     float epsilon, void *out, int64_t ld_out,
                                     int32_t out_dtype, void *stream) {
  if (rows < 0 || width <= 0 || total_width < width)
    return fail(NK_INVALID_SHAPE, "rows >= 0, 0 < width <= total_width");
  if (epsilon < 0.0f) return fail_eps(epsilon);
  if (weight_len != (uint64_t)width) return fail_length("weight", width, weight_len);
  if (!sumsq) return fail(NK_INVALID_PARAMS, "sumsq is required");
  if (ld_x < width || ld_out < width || (gate && ld_gate < width))
    return fail(NK_INVALID_PARAMS, "row strides must be >= width");
  if (out_dtype != NK_DTYPE_F32 && out_dtype != NK_DTYPE_BF16)
    return fail(NK_INVALID_PARAMS, "out_dtype must be NK_DTYPE_F32 or NK_DTYPE_BF16");
  return launch_rms_rows(x, rows, width, ld_x, weight, gate, ld_gate, epsilon, sumsq,
                         total_width, out, ld_out, out_dtype, as_stream(stream));
}

}  // extern "C"
