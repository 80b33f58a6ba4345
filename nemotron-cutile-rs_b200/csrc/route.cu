// route.cu — MoE top-k routing (moe_routing.rs:118-216) and the expert
// histogram / permutation that turns routes into grouped-GEMM row blocks.
#include <math.h>

#include "nk_common.cuh"
#include "route.h"

namespace nk {

// f32::total_cmp as a signed integer key.
__device__ __forceinline__ int32_t total_key(float f) {
  int32_t b = __float_as_int(f);
  return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}

// exp evaluated in double and rounded once to f32: the correctly rounded
// value in all but vanishingly rare double-rounding cases, which is what the
// reference's libm expf returns for practically every input.
__device__ __forceinline__ float exp_f32(float x) { return (float)exp((double)x); }

// activations.rs:73-81 with IEEE-rounded f32 add and divide.
__device__ __forceinline__ float sigmoid_ref(float x) {
  if (x >= 0.0f) {
    float z = exp_f32(-x);
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, z));
  }
  float z = exp_f32(x);
  return __fdiv_rn(z, __fadd_rn(1.0f, z));
}

constexpr int kRouteWarps = 4;
constexpr int kMaxExperts = 1024;

// One warp per token.  The token's E weights live in shared memory; top-k is
// k rounds of a warp arg-max over (total-order key desc, index asc).
__global__ void __launch_bounds__(kRouteWarps * 32)
    route_kernel(const float *__restrict__ scores, int64_t tokens, int E, int K, int mode,
                 int32_t *__restrict__ indices, float *__restrict__ weights) {
  __shared__ float wsm[kRouteWarps][kMaxExperts];
  __shared__ uint32_t taken[kRouteWarps][kMaxExperts / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kRouteWarps + warp;
  if (t >= tokens) return;
  const float *s = scores + t * E;
  float *w = wsm[warp];
  for (int e = lane; e < E / 32 + 1; e += 32)
    if (e < kMaxExperts / 32) taken[warp][e] = 0;

  if (mode == NK_ROUTE_SOFTMAX) {
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, s[e]);
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int e = lane; e < E; e += 32) w[e] = exp_f32(__fsub_rn(s[e], mx));
    __syncwarp();
    float total = 0.0f;
    if (lane == 0) {  // sequential f32 sum in index order, as Iterator::sum
      total = -0.0f;
      for (int e = 0; e < E; ++e) total = __fadd_rn(total, w[e]);
    }
    total = __shfl_sync(0xffffffffu, total, 0);
    for (int e = lane; e < E; e += 32) w[e] = __fdiv_rn(w[e], total);
  } else {
    for (int e = lane; e < E; e += 32) w[e] = sigmoid_ref(s[e]);
  }
  __syncwarp();

  float sel_w[32];
  int sel_i[32];
  for (int r = 0; r < K; ++r) {
    int32_t best_key = INT32_MIN;
    int best_idx = 0x7fffffff;
    for (int e = lane; e < E; e += 32) {
      if (taken[warp][e >> 5] & (1u << (e & 31))) continue;
      int32_t key = total_key(w[e]);
      if (key > best_key || (key == best_key && e < best_idx)) {
        best_key = key;
        best_idx = e;
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      int32_t ok = __shfl_xor_sync(0xffffffffu, best_key, o);
      int oi = __shfl_xor_sync(0xffffffffu, best_idx, o);
      if (ok > best_key || (ok == best_key && oi < best_idx)) {
        best_key = ok;
        best_idx = oi;
      }
    }
    if (lane == 0) taken[warp][best_idx >> 5] |= 1u << (best_idx & 31);
    __syncwarp();
    sel_i[r] = best_idx;
    sel_w[r] = w[best_idx];
  }
  if (lane == 0) {
    if (mode == NK_ROUTE_SOFTMAX || mode == NK_ROUTE_SIGMOID_RENORM) {
      float sel = -0.0f;
      for (int r = 0; r < K; ++r) sel = __fadd_rn(sel, sel_w[r]);
      for (int r = 0; r < K; ++r) sel_w[r] = __fdiv_rn(sel_w[r], sel);
    }
    for (int r = 0; r < K; ++r) {
      indices[t * K + r] = sel_i[r];
      weights[t * K + r] = sel_w[r];
    }
  }
}

// --------------------------------------------------------- exact routing
// The MoE layer's router scores come from a tensor-core GEMM (f32 accumulate
// over exact bf16 products), while the reference routes on
// s_e = (f32)(Σ_k f64(x_k)·f64(W_ek)) summed in k order (gemm.rs:99-109) plus
// the bias in f32 (linear.rs:333-339).  The three kernels below make the
// selected experts, their order and their weights identical to the
// reference's:
//
//  A route_cand_kernel (warp per token).  Every approximate score s~ lies
//    within d_e = c·|x|_2·|W_e|_2 + 2^-21·(|s~_e| + |b_e|) of s_e: c =
//    (products per accumulator + split partials + 2)·2^-22 bounds the tensor
//    core's f32 accumulation (each step errs by at most 2^-23 of the magnitude
//    it adds, counted twice), through Σ|x_k·W_ek| <= |x|_2·|W_e|_2; the last
//    term covers the f32 roundings of both sums and of the bias addition.
//    sigmoid is monotone, so σ(s~_e - d_e) <= σ(s_e) <= σ(s~_e + d_e).  The
//    k-th largest lower bound L is at most the reference's k-th weight: every
//    expert the reference selects has σ(s~_e + d_e) >= L, and an expert below
//    L can never be selected.  The candidates (typically k or k+1 of E) are
//    appended to per-expert pair lists.
//  B route_rescore_kernel (block per expert).  The expert's weight row is
//    staged in shared memory as f64 (hi + mid + lo is the f32 weight exactly);
//    each warp sums x·W for four tokens at a time in f64, from exact products,
//    in its own order.  Two summation orders of the same H terms differ by at
//    most 2·(H-1)·2^-53·Σ|terms| <= 2·H·2^-53·|x|_2·|W_e|_2 = r, so the
//    reference's f64 sum lies in [T - r, T + r]; when both ends round to the
//    same f32, that is the reference's score.  Otherwise (the sum sits next to
//    an f32 rounding midpoint, about one pair in 10^4) one lane runs the
//    reference's own sequential loop.
//  C route_select_kernel (warp per token).  Top-k among the candidates by
//    (weight desc by total order, expert index asc) on the exact scores,
//    renormalised as the mode asks.
//
// Softmax routing depends on every score; tokens whose scores or norm are not
// finite cannot be bounded; tokens with more than kCandCap candidates are
// improbable: those tokens are rescored over all E experts by kernel C.
constexpr int kCandCap = 16;
constexpr int kRouterMaxSplits = 16;  // the router GEMM's split-K limit
constexpr int kCandWarps = 4;
constexpr int kSelWarps = 8;  // tokens per block of kernel C = tokens per plan chunk
constexpr int kRescoreWarps = 8;
constexpr int kRescoreBatch = 4;  // tokens per warp pass in kernel B

// Per-expert |W_e|_2 and |lo_e|_2 (rounded up), from the exact f32 weights;
// a block per expert.
__global__ void __launch_bounds__(256) router_wnorm_kernel(const __nv_bfloat16 *__restrict__ w3,
                                                           int64_t hp, int H,
                                                           float *__restrict__ wnorm,
                                                           float *__restrict__ lonorm) {
  __shared__ double part[2][8];
  const int e = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const __nv_bfloat16 *row = w3 + (int64_t)e * 3 * hp;
  double acc = 0.0, acl = 0.0;
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    const float lo = __bfloat162float(row[2 * hp + h]);
    const double v = (double)__fadd_rn(
        __fadd_rn(__bfloat162float(row[h]), __bfloat162float(row[hp + h])), lo);
    acc = fma(v, v, acc);
    acl = fma((double)lo, (double)lo, acl);
  }
  for (int o = 16; o > 0; o >>= 1) {
    acc += __shfl_xor_sync(0xffffffffu, acc, o);
    acl += __shfl_xor_sync(0xffffffffu, acl, o);
  }
  if (lane == 0) {
    part[0][warp] = acc;
    part[1][warp] = acl;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0, l = 0.0;
    for (int i = 0; i < 8; ++i) {
      t += part[0][i];
      l += part[1][i];
    }
    // rounded up, then widened by a relative 2^-40 for the summation order
    wnorm[e] = __double2float_ru(sqrt(t) * (1.0 + 0x1p-40));
    lonorm[e] = __double2float_ru(sqrt(l) * (1.0 + 0x1p-40));
  }
}

__device__ __forceinline__ float exact_weight(const __nv_bfloat16 *hi, int64_t hp, int h) {
  return __fadd_rn(__fadd_rn(__bfloat162float(hi[h]), __bfloat162float(hi[hp + h])),
                   __bfloat162float(hi[2 * hp + h]));
}

// The reference's loop for one (token, expert): x row and the exact f32 weights.
__device__ __noinline__ double sequential_score(const __nv_bfloat16 *__restrict__ x,
                                                const __nv_bfloat16 *__restrict__ w3, int64_t hp,
                                                int H, int e) {
  const __nv_bfloat16 *row = w3 + (int64_t)e * 3 * hp;
  double acc = 0.0;
  for (int h = 0; h < H; ++h)
    acc = __dadd_rn(acc, __dmul_rn((double)__bfloat162float(x[h]), (double)exact_weight(row, hp, h)));
  return acc;
}

// One (token, expert) score with the whole warp (kernel C's fallback path):
// a warp-order f64 sum checked against the midpoint bound, else lane 0's
// sequential loop.  Returns the same value on every lane.
__device__ float exact_score_warp(const __nv_bfloat16 *__restrict__ x,
                                  const __nv_bfloat16 *__restrict__ w3, int64_t hp, int H, int e,
                                  const float *__restrict__ bias, int lane) {
  const __nv_bfloat16 *row = w3 + (int64_t)e * 3 * hp;
  double t = 0.0, mag = 0.0;
  for (int h = lane; h < H; h += 32) {
    const double p = (double)__bfloat162float(x[h]) * (double)exact_weight(row, hp, h);
    t += p;
    mag += fabs(p);
  }
  for (int o = 16; o > 0; o >>= 1) {
    t += __shfl_xor_sync(0xffffffffu, t, o);
    mag += __shfl_xor_sync(0xffffffffu, mag, o);
  }
  const double r = 2.0 * (double)H * 0x1p-53 * mag * (1.0 + 0x1p-20) + 0x1p-1074;
  float s = (float)(t - r);
  if (!(s == (float)(t + r))) {  // near an f32 midpoint, or not finite
    double seq = 0.0;
    if (lane == 0) seq = sequential_score(x, w3, hp, H, e);
    s = (float)__shfl_sync(0xffffffffu, seq, 0);
  }
  if (bias) s = __fadd_rn(s, bias[e]);
  return s;
}

// Warp arg-max over (key desc, position asc) of the entries not yet taken.
__device__ __forceinline__ void warp_best(const int32_t *key, const uint32_t *taken, int n,
                                          int lane, int32_t &best_key, int &best_i) {
  best_key = INT32_MIN;
  best_i = 0x7fffffff;
  for (int i = lane; i < n; i += 32) {
    if (taken[i >> 5] & (1u << (i & 31))) continue;
    if (key[i] > best_key || (key[i] == best_key && i < best_i)) {
      best_key = key[i];
      best_i = i;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const int32_t ok = __shfl_xor_sync(0xffffffffu, best_key, o);
    const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
    if (ok > best_key || (ok == best_key && oi < best_i)) {
      best_key = ok;
      best_i = oi;
    }
  }
}

struct ExactRouteWs {
  float *wnorm;      // [E] |W_e|_2
  float *lonorm;     // [E] |lo_e|_2, the part of W_e the router GEMM skips
  float *xnorm;      // [T]
  int32_t *n_cand;   // [T]; -1: rescore all E in kernel C
  int32_t *cand;     // [T, kCandCap] expert ids in ascending order
  float *exact;      // [T, kCandCap] exact scores of cand
  int32_t *e_count;  // [E] pairs per expert
  int32_t *pairs;    // [E, T] flat candidate slots t*kCandCap + i
};

// Kernel A.  The approximate scores are the router GEMM's split-K partial sums
// added in split order, plus the bias (linear.rs:333-339).  The GEMM reads
// W's hi + mid parts, so the bound adds |x|_2·|lo_e|_2 for the part it skips.
// Candidates: hi_e >= L where L is the k-th largest lower bound (in the score
// domain, as sigmoid is monotone), plus the experts whose sigmoid may round to
// the same f32 as sigmoid(L) although hi_e < L: those within `win` of L are
// compared in the weight domain.  win makes sigma(L) - sigma(hi) exceed two
// f32 ulps beyond it: for L <= 0, d ln sigma/ds = 1 - sigma >= 1/2, so 2^-10
// suffices while sigma(L) is a normal f32 (L >= -80; below that the token
// rescores all experts); for L > 0 the slope is smallest at L, so win =
// 2^-19 / sigma'(L) (twice the need, covering the fast exp used for it).
// Scores and bounds stay in registers: EPL experts per lane.
template <int EPL>
__global__ void __launch_bounds__(kCandWarps * 32)
    route_cand_kernel(const float *__restrict__ partial, int splits, int64_t split_stride,
                      const __nv_bfloat16 *__restrict__ x, int64_t tokens, int H,
                      const float *__restrict__ bias, float c, int E, int K, int mode,
                      ExactRouteWs ws) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kCandWarps + warp;
  if (t >= tokens) return;
  const __nv_bfloat16 *xr = x + t * (int64_t)H;

  // |x|_2 rounded up: bf16 squares are exact in f32; the f32 sum of H
  // positive terms (and the 5 shuffle additions) is below the true sum by at
  // most (H + 64)·2^-23 relative.
  float xs = 0.0f;
  for (int v = lane; v < (H >> 3); v += 32) {  // H % 8 == 0 (MoE layer contract)
    const uint4 q = reinterpret_cast<const uint4 *>(xr)[v];
    const uint32_t a[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float lo = __uint_as_float(a[i] << 16), hi = __uint_as_float(a[i] & 0xFFFF0000u);
      xs = fmaf(lo, lo, xs);
      xs = fmaf(hi, hi, xs);
    }
  }
  for (int o = 16; o > 0; o >>= 1) xs += __shfl_xor_sync(0xffffffffu, xs, o);
  const float xn = __fsqrt_ru(__fmul_ru(xs, 1.0f + (float)(H + 64) * 0x1p-23f));
  if (lane == 0) ws.xnorm[t] = xn;

  float lower[EPL], upper[EPL];
  bool all = mode == NK_ROUTE_SOFTMAX || !isfinite(xn);
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = j * 32 + lane;
    lower[j] = -INFINITY;
    upper[j] = -INFINITY;
    if (e < E) {
      const float *p = partial + t * E + e;
      float part[kRouterMaxSplits];  // every split's load in flight before the ordered sum
#pragma unroll
      for (int k = 0; k < kRouterMaxSplits; ++k)
        part[k] = k < splits ? p[(int64_t)k * split_stride] : 0.0f;
      float s = part[0];
#pragma unroll
      for (int k = 1; k < kRouterMaxSplits; ++k)
        if (k < splits) s = __fadd_rn(s, part[k]);
      const float b = bias ? bias[e] : 0.0f;
      if (bias) s = __fadd_rn(s, b);
      all |= !isfinite(s);
      const float d = __fadd_ru(__fadd_ru(__fmul_ru(__fmul_ru(c, xn), ws.wnorm[e]),
                                          __fmul_ru(xn, ws.lonorm[e])),
                                __fmul_ru(0x1p-21f, __fadd_ru(fabsf(s), fabsf(b))));
      lower[j] = __fsub_rd(s, d);
      upper[j] = __fadd_ru(s, d);
    }
  }
  all = __any_sync(0xffffffffu, all);
  if (all) {
    if (lane == 0) ws.n_cand[t] = -1;
    return;
  }
  uint32_t taken = 0;  // bit j: expert j*32 + lane
  float L = 0.0f;
  for (int r = 0; r < K; ++r) {  // k-th largest lower bound
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      const int e = j * 32 + lane;
      if (e < E && !(taken >> j & 1u) && (lower[j] > bv || (lower[j] == bv && e < bi))) {
        bv = lower[j];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    L = bv;
  }
  if (L < -80.0f) {
    if (lane == 0) ws.n_cand[t] = -1;
    return;
  }
  float win = 0x1p-10f;
  if (L > 0.0f) {
    const float sg = 1.0f / (1.0f + __expf(-L));
    const float slope = sg * (1.0f - sg);
    const float w2 = slope > 0.0f ? 0x1p-19f / slope : INFINITY;
    if (w2 > win) win = w2;
  }
  // weight-domain comparison only for experts inside the window below L
  bool need = false;
#pragma unroll
  for (int j = 0; j < EPL; ++j)
    need |= j * 32 + lane < E && upper[j] < L && upper[j] >= L - win;
  const bool any_window = __any_sync(0xffffffffu, need);
  const int32_t keyL = any_window ? total_key(sigmoid_ref(L)) : 0;
  uint32_t member = 0;
  int n = 0;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = j * 32 + lane;
    bool v = e < E && upper[j] >= L;
    if (!v && any_window && e < E && upper[j] >= L - win)
      v = total_key(sigmoid_ref(upper[j])) >= keyL;
    const unsigned m = __ballot_sync(0xffffffffu, v);
    if (v) member |= 1u << j;
    n += __popc(m);
  }
  if (n > kCandCap) {
    if (lane == 0) ws.n_cand[t] = -1;
    return;
  }
  int base = 0;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const bool v = member >> j & 1u;
    const unsigned m = __ballot_sync(0xffffffffu, v);
    if (v) {
      const int e = j * 32 + lane;
      const int i = base + __popc(m & ((1u << lane) - 1));
      ws.cand[t * kCandCap + i] = e;
      const int slot = atomicAdd(&ws.e_count[e], 1);
      ws.pairs[(int64_t)e * tokens + slot] = (int32_t)(t * kCandCap + i);
    }
    base += __popc(m);
  }
  if (lane == 0) ws.n_cand[t] = n;
}

// bf16 bits (in the upper half of u) as the f64 value x·2^-896: the f32 bit
// pattern shifted into the f64 fields without rebiasing the exponent (exact
// for every finite value, subnormals included).
__device__ __forceinline__ double bf16hi_scaled(uint32_t u) {
  return __hiloint2double((int)((u & 0x80000000u) | ((u >> 3) & 0x0FFFE000u)), 0);
}

// Second test for a sum that the first bound left next to an f32 midpoint.
// Sequential summation errs by at most u·Σ_i |seq_i| (u = 2^-53, seq_i the
// running sums), and |seq_i| exceeds the exact prefix sum P_i by at most
// i·u·A (A = Σ|p|), so one pass that forms every prefix sum in order — a
// lane-local scan of eight products, a warp scan of the lane totals, and the
// running carry — bounds the reference's result far more tightly than the
// worst case: |seq - T| <= u·Σ|P^_i|·(1+2^-30) + (iters+32)·u·A, where T is
// the computed total (every computed prefix sum is at most iters + 16
// roundings away from the exact one).  Products are scaled by 2^-896 (x is widened without
// rebiasing), so the bounds are in the same scale.  Returns true and the f32
// score when the rounding is decided.
__device__ __forceinline__ bool prefix_bound_score(const uint4 *__restrict__ xr,
                                                   const double *__restrict__ wrow, int H,
                                                   int vecs, int iters, int lane, float &out) {
  double carry = 0.0, absP = 0.0, A = 0.0;
  for (int i = 0; i < iters; ++i) {
    const int v = i * 32 + lane;
    double q[8];
    double run = 0.0;
    if (v < vecs) {
      const uint4 xv = xr[v];
      const uint32_t a[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const double p0 = bf16hi_scaled(a[k] << 16) * wrow[(i * 8 + 2 * k) * 32 + lane];
        const double p1 = bf16hi_scaled(a[k]) * wrow[(i * 8 + 2 * k + 1) * 32 + lane];
        A += fabs(p0) + fabs(p1);
        run += p0;
        q[2 * k] = run;
        run += p1;
        q[2 * k + 1] = run;
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) q[k] = 0.0;
    }
    double incl = run;  // inclusive warp scan of the lane totals
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const double base = carry + (incl - run);
    if (v < vecs) {
#pragma unroll
      for (int k = 0; k < 8; ++k) absP += fabs(base + q[k]);
    }
    carry += __shfl_sync(0xffffffffu, incl, 31);
  }
  // elements past the last full vector (H % 8), in order by lane 0
  if (lane == 0)
    for (int h = vecs * 8; h < H; ++h) {
      const uint32_t u = (uint32_t)__bfloat16_as_ushort(
                             reinterpret_cast<const __nv_bfloat16 *>(xr)[h]) << 16;
      const double p = bf16hi_scaled(u) * wrow[iters * 256 + (h - vecs * 8)];
      A += fabs(p);
      carry += p;
      absP += fabs(carry);
    }
  for (int o = 16; o > 0; o >>= 1) {
    absP += __shfl_xor_sync(0xffffffffu, absP, o);
    A += __shfl_xor_sync(0xffffffffu, A, o);
  }
  carry = __shfl_sync(0xffffffffu, carry, 0);
  const double t = carry * 0x1p+896;
  const double r =
      (0x1p-53 * absP * (1.0 + 0x1p-30) + (double)(iters + 32) * 0x1p-53 * A) * 0x1p+896 + 0x1p-1000;
  const float lo = (float)(t - r);
  out = lo;
  return lo == (float)(t + r);
}

// Kernel B.  Shared memory: the expert's weights as f64, vector-interleaved so
// that lane l of a warp reads consecutive words: W[(v*8 + j)] for vector
// v = i*32 + l sits at ws_row[(i*8 + j)*32 + l]; the H % 8 tail after them.
__global__ void __launch_bounds__(kRescoreWarps * 32)
    route_rescore_kernel(const __nv_bfloat16 *__restrict__ x, int64_t tokens, int H,
                         const __nv_bfloat16 *__restrict__ w3, int64_t hp,
                         const float *__restrict__ bias, ExactRouteWs ws) {
  extern __shared__ double wrow[];
  const int e = blockIdx.x;
  const int cnt = ws.e_count[e];
  const int nwarps = gridDim.y * kRescoreWarps;
  const int gw = blockIdx.y * kRescoreWarps + (threadIdx.x >> 5);
  const int nbatch = (cnt + kRescoreBatch - 1) / kRescoreBatch;
  if ((int)blockIdx.y * kRescoreWarps >= nbatch) return;  // no work for this block
  const int lane = threadIdx.x & 31;
  const int vecs = H >> 3, iters = (vecs + 31) >> 5;
  const __nv_bfloat16 *row = w3 + (int64_t)e * 3 * hp;
  for (int v = threadIdx.x; v < vecs; v += blockDim.x) {  // hp % 8 == 0: 16-byte rows
    const uint4 hv = reinterpret_cast<const uint4 *>(row)[v];
    const uint4 mv = reinterpret_cast<const uint4 *>(row + hp)[v];
    const uint4 lv = reinterpret_cast<const uint4 *>(row + 2 * hp)[v];
    const uint32_t ha[4] = {hv.x, hv.y, hv.z, hv.w}, ma[4] = {mv.x, mv.y, mv.z, mv.w};
    const uint32_t la[4] = {lv.x, lv.y, lv.z, lv.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int sh = (j & 1) ? 0 : 16;
      const float w = __fadd_rn(__fadd_rn(__uint_as_float((ha[j >> 1] << sh) & 0xFFFF0000u),
                                          __uint_as_float((ma[j >> 1] << sh) & 0xFFFF0000u)),
                                __uint_as_float((la[j >> 1] << sh) & 0xFFFF0000u));
      wrow[((v >> 5) * 8 + j) * 32 + (v & 31)] = (double)w;
    }
  }
  for (int h = vecs * 8 + threadIdx.x; h < H; h += blockDim.x)
    wrow[iters * 256 + (h - vecs * 8)] = (double)exact_weight(row, hp, h);
  __syncthreads();
  const double wn = (double)ws.wnorm[e];
  const float b = bias ? bias[e] : 0.0f;

  for (int batch = gw; batch < nbatch; batch += nwarps) {
    int slot[kRescoreBatch];
    const uint4 *xr[kRescoreBatch];
    double acc[kRescoreBatch];
#pragma unroll
    for (int j = 0; j < kRescoreBatch; ++j) {
      const int p = batch * kRescoreBatch + j;
      slot[j] = p < cnt ? ws.pairs[(int64_t)e * tokens + p] : -1;
      const int64_t t = slot[j] >= 0 ? slot[j] / kCandCap : 0;
      xr[j] = reinterpret_cast<const uint4 *>(x + t * (int64_t)H);
      acc[j] = 0.0;
    }
    // two iterations of x vectors in flight ahead of the arithmetic
    uint4 q0[kRescoreBatch], q1[kRescoreBatch];
#pragma unroll
    for (int j = 0; j < kRescoreBatch; ++j) {
      q0[j] = lane < vecs ? xr[j][lane] : make_uint4(0, 0, 0, 0);
      q1[j] = lane + 32 < vecs ? xr[j][lane + 32] : make_uint4(0, 0, 0, 0);
    }
#pragma unroll 3
    for (int i = 0; i < iters; ++i) {
      const int v = i * 32 + lane;
      uint4 q2[kRescoreBatch];
#pragma unroll
      for (int j = 0; j < kRescoreBatch; ++j)
        q2[j] = v + 64 < vecs ? xr[j][v + 64] : make_uint4(0, 0, 0, 0);
      if (v < vecs) {
        double w[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) w[k] = wrow[(i * 8 + k) * 32 + lane];
#pragma unroll
        for (int j = 0; j < kRescoreBatch; ++j) {
          const uint32_t a[4] = {q0[j].x, q0[j].y, q0[j].z, q0[j].w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            acc[j] = fma(bf16hi_scaled(a[k] << 16), w[2 * k], acc[j]);
            acc[j] = fma(bf16hi_scaled(a[k]), w[2 * k + 1], acc[j]);
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kRescoreBatch; ++j) {
        q0[j] = q1[j];
        q1[j] = q2[j];
      }
    }
    for (int h = vecs * 8 + lane; h < H; h += 32) {
      const double w = wrow[iters * 256 + (h - vecs * 8)];
#pragma unroll
      for (int j = 0; j < kRescoreBatch; ++j) {
        const uint32_t u =
            (uint32_t)__bfloat16_as_ushort(reinterpret_cast<const __nv_bfloat16 *>(xr[j])[h]) << 16;
        acc[j] = fma(bf16hi_scaled(u), w, acc[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < kRescoreBatch; ++j)
      for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
#pragma unroll
    for (int j = 0; j < kRescoreBatch; ++j) {
      if (slot[j] < 0) continue;
      const double tsum = acc[j] * 0x1p+896;
      const double xn = (double)ws.xnorm[slot[j] / kCandCap];
      const double r = 2.0 * (double)H * 0x1p-53 * xn * wn * (1.0 + 0x1p-20) + 0x1p-1000;
      float s = (float)(tsum - r);
      if (!(s == (float)(tsum + r)) && !prefix_bound_score(xr[j], wrow, H, vecs, iters, lane, s)) {
        // still undecided (rare): lane 0 runs the reference's sequential sum
        const __nv_bfloat16 *xb = reinterpret_cast<const __nv_bfloat16 *>(xr[j]);
        double seq = 0.0;
        if (lane == 0)
          for (int h = 0; h < H; ++h) {
            const int v = h >> 3;
            const double w = v < vecs ? wrow[((v >> 5) * 8 + (h & 7)) * 32 + (v & 31)]
                                      : wrow[iters * 256 + (h - vecs * 8)];
            seq = __dadd_rn(seq, __dmul_rn((double)__bfloat162float(xb[h]), w));
          }
        s = (float)__shfl_sync(0xffffffffu, seq, 0);
      }
      if (bias) s = __fadd_rn(s, b);
      if (lane == 0) ws.exact[slot[j]] = s;
    }
  }
}

// One token of kernel C: top-k over its candidates' exact scores.  sel
// (shared memory, 32 ints) receives the k selected experts in rank order.
__device__ void route_select_token(const __nv_bfloat16 *__restrict__ x, int64_t t, int H,
                                   const __nv_bfloat16 *__restrict__ w3, int64_t hp,
                                   const float *__restrict__ bias, int E, int K, int mode,
                                   const ExactRouteWs &ws, int32_t *__restrict__ indices,
                                   float *__restrict__ weights, int32_t *smem, int32_t *sel,
                                   int lane) {
  const int Ep = (E + 31) & ~31, words = Ep / 32;
  int32_t *key = smem;
  float *val = reinterpret_cast<float *>(key + Ep);
  int32_t *cand = key + 2 * Ep;
  uint32_t *tk = reinterpret_cast<uint32_t *>(key + 3 * Ep);
  for (int i = lane; i < words; i += 32) tk[i] = 0;
  int n = ws.n_cand[t];
  if (n >= 0) {
    for (int i = lane; i < n; i += 32) {
      cand[i] = ws.cand[t * kCandCap + i];
      val[i] = ws.exact[t * kCandCap + i];
    }
  } else {  // every expert, a warp per score
    n = E;
    const __nv_bfloat16 *xr = x + t * (int64_t)H;
    for (int e = 0; e < E; ++e) {
      const float v = exact_score_warp(xr, w3, hp, H, e, bias, lane);
      if (lane == 0) {
        cand[e] = e;
        val[e] = v;
      }
    }
  }
  __syncwarp();
  if (mode == NK_ROUTE_SOFTMAX) {  // n == E, cand[i] == i (moe_routing.rs:188-216)
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, val[e]);
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    __syncwarp();
    for (int e = lane; e < E; e += 32) val[e] = exp_f32(__fsub_rn(val[e], mx));
    __syncwarp();
    float total = 0.0f;
    if (lane == 0) {  // sequential f32 sum in index order, as Iterator::sum
      total = -0.0f;
      for (int e = 0; e < E; ++e) total = __fadd_rn(total, val[e]);
    }
    total = __shfl_sync(0xffffffffu, total, 0);
    for (int e = lane; e < E; e += 32) val[e] = __fdiv_rn(val[e], total);
  } else {
    for (int i = lane; i < n; i += 32) val[i] = sigmoid_ref(val[i]);
  }
  __syncwarp();
  for (int i = lane; i < n; i += 32) key[i] = total_key(val[i]);
  __syncwarp();
  // candidates are in expert order, so the position breaks ties like the index
  float sel_w[32];
  int sel_i[32];
  for (int r = 0; r < K; ++r) {
    int32_t bk;
    int bi;
    warp_best(key, tk, n, lane, bk, bi);
    if (lane == 0) tk[bi >> 5] |= 1u << (bi & 31);
    __syncwarp();
    sel_i[r] = cand[bi];
    sel_w[r] = val[bi];
  }
  if (lane == 0) {
    if (mode == NK_ROUTE_SOFTMAX || mode == NK_ROUTE_SIGMOID_RENORM) {
      float total = -0.0f;
      for (int r = 0; r < K; ++r) total = __fadd_rn(total, sel_w[r]);
      for (int r = 0; r < K; ++r) sel_w[r] = __fdiv_rn(sel_w[r], total);
    }
    for (int r = 0; r < K; ++r) {
      indices[t * K + r] = sel_i[r];
      weights[t * K + r] = sel_w[r];
      sel[r] = sel_i[r];
    }
  }
}

// Kernel C.  A block of kSelWarps tokens is one chunk of the expert plan:
// besides the routes it writes the chunk's per-expert histogram
// (chunk_counts[block][e]) and each slot's rank among the chunk's slots of
// the same expert in slot order (slot_rank), so the expert-ordered position
// of a slot is offsets[e] + (slots of expert e in earlier chunks) + rank: the
// stable (token, rank) order of the reference's per-expert loops.
// Shared memory: per warp keys, values, candidates [Ep], taken [Ep/32]; then
// the block's histogram [E] and its selections [kSelWarps][K].
__global__ void __launch_bounds__(kSelWarps * 32)
    route_select_kernel(const __nv_bfloat16 *__restrict__ x, int64_t tokens, int H,
                        const __nv_bfloat16 *__restrict__ w3, int64_t hp,
                        const float *__restrict__ bias, int E, int K, int mode, ExactRouteWs ws,
                        int32_t *__restrict__ indices, float *__restrict__ weights,
                        int32_t *__restrict__ chunk_counts, int32_t *__restrict__ slot_rank) {
  extern __shared__ int32_t sel_sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kSelWarps + warp;
  const int Ep = (E + 31) & ~31, words = Ep / 32;
  int32_t *hist = sel_sm + kSelWarps * (3 * Ep + words);
  int32_t *bsel = hist + Ep;  // [kSelWarps][32]
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  for (int i = threadIdx.x; i < kSelWarps * 32; i += blockDim.x) bsel[i] = -1;
  __syncthreads();
  if (t < tokens) route_select_token(x, t, H, w3, hp, bias, E, K, mode, ws, indices, weights,
                                     sel_sm + (int64_t)warp * (3 * Ep + words), bsel + warp * 32,
                                     lane);
  __syncthreads();
  // histogram and ranks of the block's slots
  if (t < tokens && lane < K) {
    const int e = bsel[warp * 32 + lane];
    atomicAdd(&hist[e], 1);
    int rank = 0;
    for (int w2 = 0; w2 < warp; ++w2)
      for (int r = 0; r < K; ++r) rank += bsel[w2 * 32 + r] == e;
    slot_rank[t * K + lane] = rank;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    chunk_counts[(int64_t)blockIdx.x * E + e] = hist[e];
}

// Chunk histograms [nchunks][E] -> each chunk's base per expert (in place)
// and counts[E]: a block per expert; each thread sums a run of consecutive
// chunks, a block scan of the run totals, then the runs are written back.
__global__ void __launch_bounds__(256) chunk_scan_kernel(int32_t *__restrict__ chunk_counts,
                                                         int nchunks, int E,
                                                         int32_t *__restrict__ counts) {
  __shared__ int32_t wsum[8];
  const int e = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (nchunks + 255) / 256;
  const int c0 = tid * per, c1 = c0 + per < nchunks ? c0 + per : nchunks;
  int32_t run = 0;
  for (int c = c0; c < c1; ++c) run += chunk_counts[(int64_t)c * E + e];
  int32_t incl = run;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  int32_t before = 0;
  for (int w = 0; w < warp; ++w) before += wsum[w];
  int32_t base = before + incl - run;
  for (int c = c0; c < c1; ++c) {
    const int64_t i = (int64_t)c * E + e;
    const int32_t v = chunk_counts[i];
    chunk_counts[i] = base;
    base += v;
  }
  if (tid == 255) counts[e] = before + incl;
}

// counts[E] -> offsets[E+1] (exclusive scan), one warp.
__global__ void offsets_scan_kernel(const int32_t *__restrict__ counts, int E,
                                    int32_t *__restrict__ offsets) {
  const int lane = threadIdx.x;
  int32_t carry = 0;
  for (int e0 = 0; e0 < E; e0 += 32) {
    const int e = e0 + lane;
    const int32_t v = e < E ? counts[e] : 0;
    int32_t incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (e < E) offsets[e] = carry + incl - v;
    carry += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) offsets[E] = carry;
}

// Expert-ordered position of every route slot (offsets[e] + the chunk's base
// for e + the slot's rank in its chunk); optionally the token row copied there.
__global__ void scatter_rows_kernel(const uint4 *__restrict__ x, const int32_t *__restrict__ idx,
                                    const int32_t *__restrict__ slot_rank,
                                    const int32_t *__restrict__ chunk_base,
                                    const int32_t *__restrict__ offsets, int64_t slots, int K,
                                    int E, int64_t row_vecs, int32_t *__restrict__ slot_pos,
                                    uint4 *__restrict__ xp) {
  const int64_t s = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (s >= slots) return;
  const int64_t t = s / K, c = t / kSelWarps;
  const int e = idx[s];
  const int64_t pos = offsets[e] + chunk_base[c * E + e] + slot_rank[s];
  if ((threadIdx.x & 31) == 0) slot_pos[s] = (int32_t)pos;
  if (!xp) return;
  const uint4 *src = x + t * row_vecs;
  uint4 *dst = xp + pos * row_vecs;
  for (int64_t v = threadIdx.x & 31; v < row_vecs; v += 32) dst[v] = src[v];
}

size_t route_exact_scratch_bytes(int64_t tokens, int64_t E, int K) {
  auto a = [](size_t v) { return (v + 255) & ~size_t(255); };
  const int64_t chunks = ceil_div(tokens, kSelWarps);
  return 2 * a(4 * E) + a(4 * tokens) + a(4 * tokens) + 2 * a(4 * tokens * kCandCap) + a(4 * E) +
         a(4 * E * tokens) + a(4 * tokens * K) + a(4 * chunks * E);
}

nk_status launch_route_exact(const float *partial, int splits, const uint16_t *x,
                             int64_t tokens, int H, const uint16_t *w3, const float *bias,
                             const float *norms, float c, int E, int K, int mode, void *scratch,
                             int32_t *indices, float *weights, int32_t *counts, int32_t *offsets,
                             int32_t *slot_pos, uint16_t *xp, cudaStream_t stream) {
  if (tokens == 0) {
    NK_CUDA_TRY(cudaMemsetAsync(counts, 0, sizeof(int32_t) * E, stream));
    NK_CUDA_TRY(cudaMemsetAsync(offsets, 0, sizeof(int32_t) * (E + 1), stream));
    return ok();
  }
  auto a = [](size_t v) { return (v + 255) & ~size_t(255); };
  uint8_t *p = reinterpret_cast<uint8_t *>(scratch);
  ExactRouteWs ws;
  ws.wnorm = (float *)p; p += a(4 * E);
  ws.lonorm = (float *)p; p += a(4 * E);
  ws.xnorm = (float *)p; p += a(4 * tokens);
  ws.n_cand = (int32_t *)p; p += a(4 * tokens);
  ws.cand = (int32_t *)p; p += a(4 * tokens * kCandCap);
  ws.exact = (float *)p; p += a(4 * tokens * kCandCap);
  ws.e_count = (int32_t *)p; p += a(4 * E);
  ws.pairs = (int32_t *)p; p += a(4 * E * tokens);
  int32_t *slot_rank = (int32_t *)p; p += a(4 * tokens * K);
  int32_t *chunk_counts = (int32_t *)p;
  const int64_t hp = ceil_div(H, 64) * 64;
  const __nv_bfloat16 *w = reinterpret_cast<const __nv_bfloat16 *>(w3);
  const __nv_bfloat16 *xb = reinterpret_cast<const __nv_bfloat16 *>(x);
  NK_CUDA_TRY(cudaMemsetAsync(ws.e_count, 0, sizeof(int32_t) * E, stream));
  nk_status st;
  if (norms) {  // precomputed by nk_router_norms: |W_e|_2 then |lo_e|_2
    ws.wnorm = const_cast<float *>(norms);
    ws.lonorm = const_cast<float *>(norms) + E;
  } else {
    router_wnorm_kernel<<<(unsigned)E, 256, 0, stream>>>(w, hp, H, ws.wnorm, ws.lonorm);
    st = check_launch("router_wnorm_kernel");
    if (st != NK_OK) return st;
  }
  const int ep = (E + 31) & ~31;
  const unsigned cand_blocks = (unsigned)ceil_div(tokens, kCandWarps);
  const unsigned sel_blocks = (unsigned)ceil_div(tokens, kSelWarps);
  const size_t smem_c = sizeof(int32_t) * (kSelWarps * (3 * ep + ep / 32) + ep + kSelWarps * 32);
  const size_t smem_b = sizeof(double) * ((size_t)(((H >> 3) + 31) >> 5) * 256 + 8);
  if (smem_b > 200 * 1024) return fail(NK_UNSUPPORTED, "exact routing needs hidden <= 25000");
  if (smem_b > 48 * 1024)
    NK_CUDA_TRY(cudaFuncSetAttribute(route_rescore_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_b));
  if (smem_c > 48 * 1024)
    NK_CUDA_TRY(cudaFuncSetAttribute(route_select_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_c));
  {
    const int epl = (E + 31) / 32;
    auto launch = [&](auto kern) {
      kern<<<cand_blocks, kCandWarps * 32, 0, stream>>>(partial, splits, tokens * E, xb, tokens,
                                                        H, bias, c, E, K, mode, ws);
    };
    if (epl <= 1) launch(route_cand_kernel<1>);
    else if (epl <= 2) launch(route_cand_kernel<2>);
    else if (epl <= 4) launch(route_cand_kernel<4>);
    else if (epl <= 8) launch(route_cand_kernel<8>);
    else if (epl <= 16) launch(route_cand_kernel<16>);
    else launch(route_cand_kernel<32>);
  }
  st = check_launch("route_cand_kernel");
  if (st != NK_OK) return st;
  if (mode != NK_ROUTE_SOFTMAX) {
    // blocks per expert: enough warps for the expected pairs (about T·k/E per expert)
    int64_t per = ceil_div(tokens * (K + 1), (int64_t)E);
    int gy = (int)ceil_div(ceil_div(per, kRescoreBatch), kRescoreWarps);
    if (gy < 1) gy = 1;
    if (gy > 64) gy = 64;
    route_rescore_kernel<<<dim3((unsigned)E, (unsigned)gy), kRescoreWarps * 32, smem_b, stream>>>(
        xb, tokens, H, w, hp, bias, ws);
    st = check_launch("route_rescore_kernel");
    if (st != NK_OK) return st;
  }
  route_select_kernel<<<sel_blocks, kSelWarps * 32, smem_c, stream>>>(
      xb, tokens, H, w, hp, bias, E, K, mode, ws, indices, weights, chunk_counts, slot_rank);
  st = check_launch("route_select_kernel");
  if (st != NK_OK) return st;
  // chunk histograms -> per-chunk bases (in place), counts, offsets
  chunk_scan_kernel<<<(unsigned)E, 256, 0, stream>>>(chunk_counts, (int)sel_blocks, E, counts);
  offsets_scan_kernel<<<1, 32, 0, stream>>>(counts, E, offsets);
  st = check_launch("chunk_scan_kernel");
  if (st != NK_OK) return st;
  const int64_t slots = tokens * K;
  const int warps = 8;
  scatter_rows_kernel<<<(unsigned)ceil_div(slots, warps), warps * 32, 0, stream>>>(
      reinterpret_cast<const uint4 *>(x), indices, slot_rank, chunk_counts, offsets, slots, K, E,
      H / 8, slot_pos, reinterpret_cast<uint4 *>(xp));
  return check_launch("scatter_rows_kernel");
}

nk_status launch_router_norms(const uint16_t *w3, int64_t E, int64_t H, float *norms,
                              cudaStream_t stream) {
  const int64_t hp = ceil_div(H, 64) * 64;
  router_wnorm_kernel<<<(unsigned)E, 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16 *>(w3), hp, (int)H, norms, norms + E);
  return check_launch("router_wnorm_kernel");
}

// ------------------------------------------------------------------- plan
constexpr int kPlanChunk = 1024;  // route slots per chunk (one warp walks it in order)

__global__ void plan_count_kernel(const int32_t *__restrict__ idx, int64_t slots, int E,
                                  int32_t *__restrict__ chunk_counts) {
  __shared__ int32_t h[kMaxExperts];
  for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
  __syncthreads();
  int64_t base = (int64_t)blockIdx.x * kPlanChunk;
  for (int i = threadIdx.x; i < kPlanChunk; i += blockDim.x) {
    int64_t s = base + i;
    if (s < slots) {
      int e = idx[s];
      if (e >= 0 && e < E) atomicAdd(&h[e], 1);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) chunk_counts[(int64_t)blockIdx.x * E + e] = h[e];
}

// One block of up to 1024 threads: per-expert prefix over chunks, then an
// exclusive scan over experts.
__global__ void plan_scan_kernel(int32_t *__restrict__ chunk_counts, int nchunks, int E,
                                 int32_t *__restrict__ counts, int32_t *__restrict__ offsets) {
  __shared__ int32_t sc[kMaxExperts];
  const int e = threadIdx.x;
  int32_t total = 0;
  if (e < E) {
    for (int c0 = 0; c0 < nchunks; c0 += 8) {  // 8 loads in flight, then the running sum
      int32_t v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        v[j] = c0 + j < nchunks ? chunk_counts[(int64_t)(c0 + j) * E + e] : 0;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (c0 + j < nchunks) {
          chunk_counts[(int64_t)(c0 + j) * E + e] = total;  // the chunk's base for expert e
          total += v[j];
        }
    }
    counts[e] = total;
  }
  sc[e] = e < E ? total : 0;
  __syncthreads();
  for (int o = 1; o < blockDim.x; o <<= 1) {  // inclusive Hillis-Steele scan
    int32_t v = e >= o ? sc[e - o] : 0;
    __syncthreads();
    sc[e] += v;
    __syncthreads();
  }
  if (e < E) offsets[e] = sc[e] - total;
  if (e == E - 1) offsets[E] = sc[e];
}

__global__ void plan_place_kernel(const int32_t *__restrict__ idx, int64_t slots, int E,
                                  const int32_t *__restrict__ chunk_base,
                                  const int32_t *__restrict__ offsets, int32_t *__restrict__ perm,
                                  int32_t *__restrict__ slot_pos) {
  __shared__ int32_t run[kMaxExperts];
  const int lane = threadIdx.x;  // a single warp walks the chunk in slot order
  for (int e = lane; e < E; e += 32)
    run[e] = offsets[e] + chunk_base[(int64_t)blockIdx.x * E + e];
  __syncwarp();
  int64_t base = (int64_t)blockIdx.x * kPlanChunk;
  for (int g0 = 0; g0 < kPlanChunk; g0 += 32 * 8) {  // 8 loads per lane in flight
    int ev[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t s = base + g0 + j * 32 + lane;
      ev[j] = s < slots ? idx[s] : -1;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t s = base + g0 + j * 32 + lane;
      const bool valid = s < slots && ev[j] >= 0 && ev[j] < E;
      const int e = valid ? ev[j] : -1 - lane;  // unique negative keys for idle lanes
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      const int rank = __popc(peers & ((1u << lane) - 1));
      if (valid) {
        const int pos = run[e] + rank;
        perm[pos] = (int32_t)s;
        slot_pos[s] = pos;
      }
      __syncwarp();
      if (valid && rank == 0) run[e] += __popc(peers);
      __syncwarp();
    }
  }
}

nk_status launch_route(const float *scores, int64_t tokens, int E, int K, int mode,
                       int32_t *indices, float *weights, cudaStream_t stream) {
  if (tokens == 0) return ok();
  unsigned blocks = (unsigned)ceil_div(tokens, kRouteWarps);
  route_kernel<<<blocks, kRouteWarps * 32, 0, stream>>>(scores, tokens, E, K, mode, indices,
                                                        weights);
  return check_launch("route_kernel");
}

size_t plan_scratch_bytes(int64_t slots, int64_t E) {
  return (size_t)(ceil_div(slots, kPlanChunk) + 1) * (size_t)E * sizeof(int32_t);
}

nk_status launch_plan(const int32_t *indices, int64_t slots, int E, int32_t *counts,
                      int32_t *offsets, int32_t *perm, int32_t *slot_pos, int32_t *chunk_scratch,
                      cudaStream_t stream) {
  int nchunks = (int)ceil_div(slots, kPlanChunk);
  if (nchunks == 0) {
    NK_CUDA_TRY(cudaMemsetAsync(counts, 0, sizeof(int32_t) * E, stream));
    NK_CUDA_TRY(cudaMemsetAsync(offsets, 0, sizeof(int32_t) * (E + 1), stream));
    return ok();
  }
  plan_count_kernel<<<nchunks, 256, 0, stream>>>(indices, slots, E, chunk_scratch);
  int threads = 32;
  while (threads < E) threads <<= 1;
  plan_scan_kernel<<<1, threads, 0, stream>>>(chunk_scratch, nchunks, E, counts, offsets);
  plan_place_kernel<<<nchunks, 32, 0, stream>>>(indices, slots, E, chunk_scratch, offsets, perm,
                                                slot_pos);
  return check_launch("plan kernels");
}

}  // namespace nk

using namespace nk;

extern "C" {

nk_status nk_moe_route(const float *scores, size_t scores_len, size_t tokens, size_t experts,
                       size_t top_k, int32_t mode, int32_t *indices, size_t indices_len,
                       float *weights, size_t weights_len, void *stream) {
  if (experts == 0 || top_k == 0 || top_k > experts)
    return fail(NK_INVALID_SHAPE, "routing shape needs 0 < top_k <= experts");
  uint64_t slen, rlen;
  if (!mul_ok(tokens, experts, &slen) || !mul_ok(tokens, top_k, &rlen))
    return fail(NK_INVALID_SHAPE, "routing shape overflows");
  if (scores_len != slen) return fail_length("scores", slen, scores_len);
  if (indices_len != rlen) return fail_length("indices", rlen, indices_len);
  if (weights_len != rlen) return fail_length("weights", rlen, weights_len);
  if (experts > (size_t)kMaxExperts || top_k > 32)
    return fail(NK_UNSUPPORTED, "device router handles experts <= 1024 and top_k <= 32");
  if (mode < NK_ROUTE_SIGMOID || mode > NK_ROUTE_SIGMOID_RENORM)
    return fail(NK_UNSUPPORTED, "unknown routing mode");
  return launch_route(scores, (int64_t)tokens, (int)experts, (int)top_k, mode, indices, weights,
                      as_stream(stream));
}

nk_status nk_moe_plan(const int32_t *indices, int64_t tokens, int64_t top_k, int64_t experts,
                      int32_t *counts, int32_t *offsets, int32_t *perm, int32_t *slot_pos,
                      void *stream) {
  if (experts <= 0 || top_k <= 0 || top_k > experts || tokens < 0)
    return fail(NK_INVALID_SHAPE, "plan shape needs 0 < top_k <= experts");
  if (experts > kMaxExperts) return fail(NK_UNSUPPORTED, "experts > 1024");
  int64_t slots = tokens * top_k;
  void *buf = nullptr;
  cudaStream_t s = as_stream(stream);
  nk_status st = scratch(plan_scratch_bytes(slots, experts), &buf, s);
  if (st != NK_OK) return st;
  return launch_plan(indices, slots, (int)experts, counts, offsets, perm, slot_pos,
                     reinterpret_cast<int32_t *>(buf), s);
}

}  // extern "C"
