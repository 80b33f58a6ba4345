// attention.cu — the attention core between the Q/K/V and O projections
// (nemotron-kernels/src/attention.rs), with a KV cache.
//
// Two paths:
//   * nk_attention_f32 — the reference contract (attention.rs:204-302) on f32
//     [B, S, H, d] tensors: f64 dot products, f32 scale, softmax with an f64
//     partition, f64 output sums.  A warp per (batch, query, head) row.
//   * nk_attention_gqa — the bf16 serving path over a KV cache.  Scores and
//     the value sum are grouped GEMMs on the tcgen05 projection kernel:
//       S = Q·Kᵀ   one tile list over every (batch, KV head) pair: the K cache
//                  rows are the weight side (128 keys per tile), the query rows
//                  of the pair's query heads the token side;
//       P = softmax(scale·S) with the causal mask, normalised, bf16;
//       O = P·V    the V cache is stored transposed ([d, L] per pair), so its
//                  d rows are the weight side and P the token side.
//     Queries are first regrouped [B, Hkv, S, G, d] (G = Hq/Hkv) so that each
//     pair's rows are contiguous, and the output regrouped back.  Key tiles
//     entirely above the causal diagonal are left out of the score tile list.
//     Pairs are processed in chunks so that the score buffer stays bounded.
#include "gemm_tc.h"
#include "nk_common.cuh"

namespace nk {

// ------------------------------------------------------------- f32 contract
// Warp per row (b, qi, h); scores of the row in `scores` (global scratch).
__global__ void attn_f32_kernel(const float *__restrict__ q, const float *__restrict__ k,
                                const float *__restrict__ v, int B, int Sq, int Skv, int Hq,
                                int Hkv, int d, int causal, int64_t q_offset, float scale,
                                float *__restrict__ scores, float *__restrict__ out,
                                unsigned long long *bad_target,
                                unsigned long long *bad_partition) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)B * Sq * Hq;
  if (row >= rows) return;
  const int h = (int)(row % Hq);
  const int64_t bq = row / Hq;  // b * Sq + qi
  const int qi = (int)(bq % Sq), b = (int)(bq / Sq);
  const int kh = h / (Hq / Hkv);
  int64_t max_key = Skv - 1;
  if (causal) {
    const int64_t lim = q_offset + qi;
    max_key = lim < Skv - 1 ? lim : Skv - 1;
  }
  float *sc = scores + row * (int64_t)Skv;
  const float *qr = q + row * (int64_t)d;
  // attention.rs:148-185: f64 dot, cast to f32, times the f32 scale.
  float mx = -INFINITY;
  for (int64_t j = 0; j < Skv; ++j) {
    float s = -INFINITY;
    if (!causal || j <= max_key) {
      const float *kr = k + (((int64_t)b * Skv + j) * Hkv + kh) * d;
      double acc = 0.0;
      for (int dd = lane; dd < d; dd += 32) acc += (double)qr[dd] * (double)kr[dd];
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      s = (float)acc * scale;
    }
    if (lane == 0) sc[j] = s;
    if (isfinite(s)) mx = fmaxf(mx, s);
  }
  if (!isfinite(mx)) {
    if (lane == 0) atomicMin(bad_target, (unsigned long long)row);
    return;
  }
  __syncwarp();
  // attention.rs:232-251: f32 exp, f64 partition (lanes then a fixed tree).
  double part = 0.0;
  for (int64_t j = lane; j < Skv; j += 32) {
    const float s = sc[j];
    if (isfinite(s)) part += (double)expf(s - mx);
  }
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if (part == 0.0) {
    if (lane == 0) atomicMin(bad_partition, (unsigned long long)row);
    return;
  }
  const float inv = (float)(1.0 / part);
  // attention.rs:262-291: f64 sum of f32 (weight * inv) times v.
  for (int dd = lane; dd < d; dd += 32) {
    double acc = 0.0;
    for (int64_t j = 0; j < Skv; ++j) {
      const float s = sc[j];
      if (!isfinite(s)) continue;
      const float w = expf(s - mx);
      if (w == 0.0f) continue;
      acc += (double)(w * inv) * (double)v[(((int64_t)b * Skv + j) * Hkv + kh) * d + dd];
    }
    out[row * (int64_t)d + dd] = (float)acc;
  }
}

// --------------------------------------------------------------- KV cache
// k_new / v_new: [B * S, Hkv * d] bf16 (projection outputs).  K cache
// [B, Hkv, Lmax, d]; V cache transposed [B, Hkv, d, Lmax].  Steps pos0..pos0+S-1.
__global__ void kv_append_kernel(const __nv_bfloat16 *__restrict__ k_new,
                                 const __nv_bfloat16 *__restrict__ v_new, int B, int S, int Hkv,
                                 int d, int64_t pos0, int64_t Lmax,
                                 __nv_bfloat16 *__restrict__ k_cache,
                                 __nv_bfloat16 *__restrict__ vt_cache) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)B * S * Hkv * d;
  if (i >= total) return;
  const int dd = (int)(i % d);
  const int64_t r = i / d;
  const int h = (int)(r % Hkv);
  const int64_t bs = r / Hkv;
  const int s = (int)(bs % S), b = (int)(bs / S);
  const int64_t pos = pos0 + s;
  const int64_t pair = (int64_t)b * Hkv + h;
  k_cache[(pair * Lmax + pos) * d + dd] = k_new[i];
  vt_cache[(pair * d + dd) * Lmax + pos] = v_new[i];
}

// --------------------------------------------------------------- GQA path
// q [B, S, Hq, d] -> qp [B, Hkv, S, G, d] (pairs p0 .. p0+np-1 only).  A
// thread moves 16 bytes; 256 / dv rows per block (dv = d/8 chunks per row);
// the row index is decomposed once per row in 32-bit arithmetic.
__global__ void __launch_bounds__(256) q_regroup_kernel(const uint4 *__restrict__ q, int S,
                                                        int Hq, int Hkv, int dv, int p0,
                                                        int rows, uint4 *__restrict__ qp) {
  const int rpb = 256 / dv;
  const int r = blockIdx.x * rpb + (int)threadIdx.x / dv;  // ((lp * S) + s) * G + g
  const int c = (int)threadIdx.x % dv;
  if (r >= rows || (int)threadIdx.x >= rpb * dv) return;
  const int G = Hq / Hkv;
  const int g = r % G, sr = r / G, s = sr % S, p = p0 + sr / S;
  const int b = p / Hkv, kh = p % Hkv;
  qp[(int64_t)r * dv + c] = q[(((int64_t)b * S + s) * Hq + kh * G + g) * dv + c];
}

// op [pairs, S, G, d] f32 (local) -> out [B, S, Hq, d] (f32 or bf16).  A
// thread moves 4 values; 256 / (d/4) rows per block.
__global__ void __launch_bounds__(256) o_scatter_kernel(const float4 *__restrict__ op, int S,
                                                        int Hq, int Hkv, int d4, int p0,
                                                        int rows, void *__restrict__ out,
                                                        int out_f32) {
  const int rpb = 256 / d4;
  const int r = blockIdx.x * rpb + (int)threadIdx.x / d4;
  const int c = (int)threadIdx.x % d4;
  if (r >= rows || (int)threadIdx.x >= rpb * d4) return;
  const int G = Hq / Hkv;
  const int g = r % G, sr = r / G, s = sr % S, p = p0 + sr / S;
  const int b = p / Hkv, kh = p % Hkv;
  const float4 v = op[(int64_t)r * d4 + c];
  const int64_t o = (((int64_t)b * S + s) * Hq + kh * G + g) * d4 + c;  // in float4 units
  if (out_f32) {
    reinterpret_cast<float4 *>(out)[o] = v;
  } else {
    __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t *>(&lo);
    pk.y = *reinterpret_cast<uint32_t *>(&hi);
    reinterpret_cast<uint2 *>(out)[o] = pk;
  }
}

// Score tiles: block = one pair (p0 + blockIdx.x); thread = token tile.  Key
// tile f is kept when its first key can be attended by the tile's last query.
__global__ void score_tiles_kernel(int np, int S, int G, int L, int64_t Lmax, int bn, int causal,
                                   int64_t q_offset, int64_t p0, TcTile *__restrict__ tiles,
                                   int *__restrict__ count) {
  __shared__ int sc[1024];
  const int rows = S * G;
  const int tt_n = (rows + bn - 1) / bn;
  const int ft_n = (L + 127) / 128;
  const int lp = blockIdx.x;  // local pair
  int n_mine = 0, fmax = 0;
  const int tt = threadIdx.x;
  if (tt < tt_n) {
    fmax = ft_n - 1;
    if (causal) {
      int last_row = (tt + 1) * bn - 1;
      if (last_row > rows - 1) last_row = rows - 1;
      const int64_t last_key = q_offset + last_row / G;
      const int64_t f = last_key / 128;
      fmax = (int)(f < ft_n - 1 ? f : ft_n - 1);
    }
    n_mine = fmax + 1;
  }
  sc[threadIdx.x] = n_mine;
  __syncthreads();
  for (int o = 1; o < (int)blockDim.x; o <<= 1) {
    const int v = threadIdx.x >= (unsigned)o ? sc[threadIdx.x - o] : 0;
    __syncthreads();
    sc[threadIdx.x] += v;
    __syncthreads();
  }
  const int per_pair = sc[blockDim.x - 1];
  if (blockIdx.x == 0 && threadIdx.x == 0) *count = per_pair * np;
  if (tt >= tt_n) return;
  const int base = lp * per_pair + sc[threadIdx.x] - n_mine;
  const int64_t p = p0 + lp;
  for (int f = 0; f <= fmax; ++f) {
    TcTile t;
    t.w_row = (int)(p * Lmax + (int64_t)f * 128);
    t.x_row = (lp * S * G) + tt * bn;
    const int fv = L - f * 128, tv = rows - tt * bn;
    t.valid = ((fv > 128 ? 128 : fv) << 16) | (tv > bn ? bn : tv);
    t.out_col0 = f * 128;
    tiles[base + f] = t;
  }
}

// Value tiles: one per (pair, token tile); the pair's d rows of the
// transposed V cache are the weight side.
__global__ void value_tiles_kernel(int np, int S, int G, int d, int bn, int64_t p0,
                                   TcTile *__restrict__ tiles, int *__restrict__ count) {
  const int rows = S * G;
  const int tt_n = (rows + bn - 1) / bn;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i == 0) *count = np * tt_n;
  if (i >= (int64_t)np * tt_n) return;
  const int lp = (int)(i / tt_n), tt = (int)(i % tt_n);
  TcTile t;
  t.w_row = (int)((p0 + lp) * d);
  t.x_row = lp * rows + tt * bn;
  const int tv = rows - tt * bn;
  t.valid = (d << 16) | (tv > bn ? bn : tv);
  t.out_col0 = 0;
  tiles[i] = t;
}

// Row softmax of one score row (local row r = (lp * S + s) * G + g): keys
// 0..lim get exp(scale*S - max) / sum, keys lim+1 .. kpad-1 get 0.  f32 exp
// as attention.rs:232-251; the partition is summed in f32 within a lane
// (at most VPT terms, each <= 1) and in f64 across lanes.
__device__ __forceinline__ void flag_row(unsigned long long *bad, int64_t r, int S, int G,
                                         int64_t p0, int Hq, int Hkv) {
  const int g = (int)(r % G), s = (int)((r / G) % S);
  const int64_t p = p0 + r / ((int64_t)S * G);
  const int64_t b = p / Hkv, kh = p % Hkv;
  atomicMin(bad, (unsigned long long)(((b * S + s) * Hq) + kh * G + g));
}

// Warp per row, the row in registers (VPT values per lane, kpad <= 32 * VPT).
template <int VPT>
__global__ void __launch_bounds__(256) attn_softmax_warp_kernel(
    const float *__restrict__ S_, int64_t lds, int S, int G, int L, int kpad, int causal,
    int64_t q_offset, float scale, int64_t p0, int Hq, int Hkv, __nv_bfloat16 *__restrict__ P,
    int64_t ldp, int64_t rows, unsigned long long *bad_target) {
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int s = (int)((r / G) % S);
  int64_t lim = L - 1;
  if (causal) {
    const int64_t l = q_offset + s;
    lim = l < L - 1 ? l : L - 1;
  }
  const float *sr = S_ + r * lds;
  float v[VPT];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int j = lane + 32 * i;
    v[i] = -INFINITY;
    if (j <= lim) {
      const float t = sr[j] * scale;
      if (isfinite(t)) v[i] = t;
    }
    mx = fmaxf(mx, v[i]);
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  __nv_bfloat16 *pr = P + r * ldp;
  if (!isfinite(mx)) {
    if (lane == 0) flag_row(bad_target, r, S, G, p0, Hq, Hkv);
#pragma unroll
    for (int i = 0; i < VPT; ++i)
      if (lane + 32 * i < kpad) pr[lane + 32 * i] = __float2bfloat16_rn(0.0f);
    return;
  }
  float part_f = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    v[i] = v[i] == -INFINITY ? 0.0f : expf(v[i] - mx);
    part_f += v[i];
  }
  double part = (double)part_f;
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  const float inv = (float)(1.0 / part);
#pragma unroll
  for (int i = 0; i < VPT; ++i)
    if (lane + 32 * i < kpad) pr[lane + 32 * i] = __float2bfloat16_rn(v[i] * inv);
}

// Rows longer than the register kernels take: a block of 128 threads per row.
__global__ void __launch_bounds__(128) attn_softmax_kernel(
    const float *__restrict__ S_, int64_t lds, int S, int G, int L, int kpad, int causal,
    int64_t q_offset, float scale, int64_t p0, int Hq, int Hkv, __nv_bfloat16 *__restrict__ P,
    int64_t ldp, unsigned long long *bad_target) {
  const int64_t r = blockIdx.x;
  const int s = (int)((r / G) % S);
  int64_t lim = L - 1;
  if (causal) {
    const int64_t l = q_offset + s;
    lim = l < L - 1 ? l : L - 1;
  }
  const float *sr = S_ + r * lds;
  __nv_bfloat16 *pr = P + r * ldp;
  __shared__ float red_f[4];
  __shared__ double red_d[4];
  float mx = -INFINITY;
  for (int64_t j = threadIdx.x; j <= lim; j += blockDim.x) {
    const float v = sr[j] * scale;
    if (isfinite(v)) mx = fmaxf(mx, v);
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red_f[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red_f[0], red_f[1]), fmaxf(red_f[2], red_f[3]));
  if (!isfinite(mx)) {
    if (threadIdx.x == 0) flag_row(bad_target, r, S, G, p0, Hq, Hkv);
    for (int64_t j = threadIdx.x; j < kpad; j += blockDim.x) pr[j] = __float2bfloat16_rn(0.0f);
    return;
  }
  float part_f = 0.0f;
  for (int64_t j = threadIdx.x; j <= lim; j += blockDim.x) {
    const float v = sr[j] * scale;
    if (isfinite(v)) part_f += expf(v - mx);
  }
  double part = (double)part_f;
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red_d[threadIdx.x >> 5] = part;
  __syncthreads();
  part = (red_d[0] + red_d[1]) + (red_d[2] + red_d[3]);
  const float inv = (float)(1.0 / part);
  for (int64_t j = threadIdx.x; j < kpad; j += blockDim.x) {
    float w = 0.0f;
    if (j <= lim) {
      const float v = sr[j] * scale;
      if (isfinite(v)) w = expf(v - mx) * inv;
    }
    pr[j] = __float2bfloat16_rn(w);
  }
}

struct GqaShape {
  int64_t B, S, L, Lmax, Hq, Hkv, d;
};

// Workspace layout for a chunk of `np` pairs.
struct GqaWs {
  unsigned long long *flag;  // first row with no finite score (offset 0 of the workspace)
  uint16_t *qp, *p;
  float *s;
  float *op;
  TcTile *score_tiles, *value_tiles;
  int *counts;
  size_t bytes;
};

static int64_t kpad_of(int64_t L) { return ceil_div(L, 64) * 64; }
static int64_t lds_of(int64_t L) { return ceil_div(L, 128) * 128; }

static GqaWs carve_gqa(const GqaShape &g, int64_t np, int bn, uint8_t *base) {
  GqaWs w{};
  const int64_t G = g.Hq / g.Hkv, rows = np * g.S * G;
  const int64_t tt = ceil_div(g.S * G, bn), ft = ceil_div(g.L, 128);
  size_t off = 0;
  auto take = [&](size_t n) {
    size_t o = off;
    off = (off + n + 255) & ~size_t(255);
    return base ? base + o : nullptr;
  };
  w.flag = reinterpret_cast<unsigned long long *>(take(sizeof(unsigned long long)));
  w.qp = reinterpret_cast<uint16_t *>(take((size_t)rows * g.d * 2));
  w.s = reinterpret_cast<float *>(take((size_t)rows * lds_of(g.L) * 4));
  w.p = reinterpret_cast<uint16_t *>(take((size_t)rows * kpad_of(g.L) * 2));
  w.op = reinterpret_cast<float *>(take((size_t)rows * g.d * 4));
  w.score_tiles = reinterpret_cast<TcTile *>(take((size_t)np * tt * ft * sizeof(TcTile)));
  w.value_tiles = reinterpret_cast<TcTile *>(take((size_t)np * tt * sizeof(TcTile)));
  w.counts = reinterpret_cast<int *>(take(2 * sizeof(int)));
  w.bytes = off;
  return w;
}

// Pairs per chunk: the score buffer of a chunk stays under ~1 GiB.
static int64_t chunk_pairs(const GqaShape &g) {
  const int64_t G = g.Hq / g.Hkv;
  const int64_t per = g.S * G * lds_of(g.L) * 4;
  int64_t np = (int64_t)(1ll << 30) / (per > 0 ? per : 1);
  if (const char *e = getenv("NK_ATTN_CHUNK")) {  // test probe: pairs per chunk
    const int64_t v = atoll(e);
    if (v >= 1) np = v;
  }
  if (np < 1) np = 1;
  const int64_t pairs = g.B * g.Hkv;
  return np < pairs ? np : pairs;
}

static int bn_of(const GqaShape &g) { return g.S * (g.Hq / g.Hkv) <= 64 ? 64 : 256; }

}  // namespace nk

using namespace nk;

extern "C" {

nk_status nk_attention_f32(const float *query, size_t query_len, const float *key,
                           size_t key_len, const float *value, size_t value_len, int64_t batch,
                           int64_t q_seq, int64_t kv_seq, int64_t q_heads, int64_t kv_heads,
                           int64_t head_dim, int32_t causal, int64_t q_offset,
                           int32_t has_scale, float scale, float *out, size_t out_len,
                           void *stream) {
  // attention.rs:304-357, then the output length (:212-218), then the scale (:82-93).
  if (batch <= 0 || q_seq <= 0 || kv_seq <= 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0)
    return fail(NK_INVALID_SHAPE, "attention shape dimensions must be positive");
  if (q_heads % kv_heads) {
    nk_status e = fail(NK_HEAD_COUNT_MISMATCH, "query heads must be a multiple of KV heads");
    tls_error().expected = (uint64_t)q_heads;
    tls_error().actual = (uint64_t)kv_heads;
    return e;
  }
  const uint64_t ql = (uint64_t)batch * q_seq * q_heads * head_dim;
  const uint64_t kl = (uint64_t)batch * kv_seq * kv_heads * head_dim;
  if (query_len != ql) return fail_length("query", ql, query_len);
  if (key_len != kl) return fail_length("key", kl, key_len);
  if (value_len != kl) return fail_length("value", kl, value_len);
  if (out_len != ql) return fail_length("output", ql, out_len);
  const float sc = has_scale ? scale : 1.0f / sqrtf((float)head_dim);
  if (!isfinite(sc) || sc <= 0.0f) {
    nk_status e = fail(NK_INVALID_SCALE, "softmax scale must be finite and > 0");
    tls_error().value = sc;
    return e;
  }
  if (q_offset < 0) return fail(NK_INVALID_PARAMS, "q_offset >= 0");
  cudaStream_t s = as_stream(stream);
  const int64_t rows = batch * q_seq * q_heads;
  void *buf = nullptr;
  const size_t score_bytes = (size_t)rows * kv_seq * 4;
  nk_status st = scratch(256 + score_bytes, &buf, s);
  if (st != NK_OK) return st;
  unsigned long long *bad = reinterpret_cast<unsigned long long *>(buf);
  NK_CUDA_TRY(cudaMemsetAsync(bad, 0xFF, 2 * sizeof(unsigned long long), s));
  float *scores = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(buf) + 256);
  attn_f32_kernel<<<(unsigned)ceil_div(rows, 4), 128, 0, s>>>(
      query, key, value, (int)batch, (int)q_seq, (int)kv_seq, (int)q_heads, (int)kv_heads,
      (int)head_dim, causal, q_offset, sc, scores, out, bad, bad + 1);
  st = check_launch("attn_f32_kernel");
  if (st != NK_OK) return st;
  unsigned long long h[2];
  NK_CUDA_TRY(cudaMemcpyAsync(h, bad, sizeof(h), cudaMemcpyDeviceToHost, s));
  NK_CUDA_TRY(cudaStreamSynchronize(s));
  // The first failing row in (batch, query, head) order, as the host loop finds it.
  const unsigned long long first = h[0] < h[1] ? h[0] : h[1];
  if (first != ~0ull) {
    nk_status e = first == h[0]
                      ? fail(NK_NO_VALID_TARGETS, "no finite attention score in a row")
                      : fail(NK_ZERO_PARTITION, "softmax partition is zero");
    tls_error().index = first;
    return e;
  }
  return ok();
}

nk_status nk_kv_append(const uint16_t *k_new, const uint16_t *v_new, int64_t batch, int64_t seq,
                       int64_t kv_heads, int64_t head_dim, int64_t pos0, int64_t max_len,
                       uint16_t *k_cache, uint16_t *vt_cache, void *stream) {
  if (batch <= 0 || seq <= 0 || kv_heads <= 0 || head_dim <= 0)
    return fail(NK_INVALID_SHAPE, "batch, seq, kv_heads, head_dim > 0");
  if (pos0 < 0 || pos0 + seq > max_len)
    return fail(NK_INVALID_PARAMS, "cache positions pos0 .. pos0+seq-1 must lie in [0, max_len)");
  const int64_t total = batch * seq * kv_heads * head_dim;
  kv_append_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, as_stream(stream)>>>(
      reinterpret_cast<const __nv_bfloat16 *>(k_new),
      reinterpret_cast<const __nv_bfloat16 *>(v_new), (int)batch, (int)seq, (int)kv_heads,
      (int)head_dim, pos0, max_len, reinterpret_cast<__nv_bfloat16 *>(k_cache),
      reinterpret_cast<__nv_bfloat16 *>(vt_cache));
  return check_launch("kv_append_kernel");
}

static nk_status gqa_validate(const GqaShape &g) {
  if (g.B <= 0 || g.S <= 0 || g.L <= 0 || g.Hq <= 0 || g.Hkv <= 0 || g.d <= 0)
    return fail(NK_INVALID_SHAPE, "attention shape dimensions must be positive");
  if (g.Hq % g.Hkv) return fail(NK_HEAD_COUNT_MISMATCH, "query heads must be a multiple of KV heads");
  if (g.L > g.Lmax) return fail(NK_INVALID_PARAMS, "kv_len <= max_len");
  if (g.d != 64 && g.d != 128) return fail(NK_UNSUPPORTED, "head_dim must be 64 or 128");
  if (g.Lmax % 64) return fail(NK_UNSUPPORTED, "max_len must be a multiple of 64");
  if (ceil_div(g.S * (g.Hq / g.Hkv), bn_of(g)) > 1024)
    return fail(NK_UNSUPPORTED, "q_seq * (q_heads / kv_heads) must be <= 262144");
  if (g.B * g.Hkv * g.Lmax >= (1ll << 31) || g.B * g.S * g.Hq >= (1ll << 31))
    return fail(NK_UNSUPPORTED, "cache or query rows must be < 2^31");
  return NK_OK;
}

nk_status nk_attention_workspace_bytes(int64_t batch, int64_t q_seq, int64_t kv_len,
                                       int64_t max_len, int64_t q_heads, int64_t kv_heads,
                                       int64_t head_dim, size_t *bytes) {
  if (!bytes) return fail(NK_INVALID_PARAMS, "bytes");
  GqaShape g{batch, q_seq, kv_len, max_len, q_heads, kv_heads, head_dim};
  nk_status st = gqa_validate(g);
  if (st != NK_OK) return st;
  *bytes = carve_gqa(g, chunk_pairs(g), bn_of(g), nullptr).bytes;
  return ok();
}

nk_status nk_attention_gqa(const uint16_t *q, const uint16_t *k_cache, const uint16_t *vt_cache,
                           int64_t batch, int64_t q_seq, int64_t kv_len, int64_t max_len,
                           int64_t q_heads, int64_t kv_heads, int64_t head_dim, int32_t causal,
                           int64_t q_offset, int32_t has_scale, float scale, void *out,
                           int32_t out_dtype, void *workspace, size_t workspace_bytes,
                           void *stream) {
  GqaShape g{batch, q_seq, kv_len, max_len, q_heads, kv_heads, head_dim};
  nk_status st = gqa_validate(g);
  if (st != NK_OK) return st;
  const float sc = has_scale ? scale : 1.0f / sqrtf((float)head_dim);
  if (!isfinite(sc) || sc <= 0.0f) {
    nk_status e = fail(NK_INVALID_SCALE, "softmax scale must be finite and > 0");
    tls_error().value = sc;
    return e;
  }
  if (q_offset < 0) return fail(NK_INVALID_PARAMS, "q_offset >= 0");
  if (out_dtype != NK_DTYPE_F32 && out_dtype != NK_DTYPE_BF16)
    return fail(NK_INVALID_PARAMS, "out_dtype must be NK_DTYPE_F32 or NK_DTYPE_BF16");
  if (!q || !k_cache || !vt_cache || !out || !workspace)
    return fail(NK_INVALID_PARAMS, "q, caches, out and workspace are required");
  if (((uintptr_t)q | (uintptr_t)k_cache | (uintptr_t)vt_cache | (uintptr_t)workspace) & 15)
    return fail(NK_INVALID_PARAMS, "q, caches and workspace must be 16-byte aligned");
  const int bn = bn_of(g);
  const int64_t np_max = chunk_pairs(g);
  GqaWs w = carve_gqa(g, np_max, bn, reinterpret_cast<uint8_t *>(workspace));
  if (workspace_bytes < w.bytes) {
    nk_status e = fail(NK_WORKSPACE_TOO_SMALL, "attention workspace too small");
    tls_error().expected = w.bytes;
    tls_error().actual = workspace_bytes;
    return e;
  }
  cudaStream_t s = as_stream(stream);
  int *err = device_error_ptr();
  unsigned long long *bad = w.flag;
  NK_CUDA_TRY(cudaMemsetAsync(bad, 0xFF, sizeof(unsigned long long), s));

  const int64_t G = g.Hq / g.Hkv, pairs = g.B * g.Hkv;
  const int64_t lds = lds_of(g.L), kpad = kpad_of(g.L);
  const int tt_n = (int)ceil_div(g.S * G, bn);
  for (int64_t p0 = 0; p0 < pairs; p0 += np_max) {
    const int64_t np = pairs - p0 < np_max ? pairs - p0 : np_max;
    const int64_t rows = np * g.S * G;
    const int dv = (int)(g.d / 8);  // uint4 per head row
    q_regroup_kernel<<<(unsigned)ceil_div(rows, 256 / dv), 256, 0, s>>>(
        reinterpret_cast<const uint4 *>(q), (int)g.S, (int)g.Hq, (int)g.Hkv, dv, (int)p0,
        (int)rows, reinterpret_cast<uint4 *>(w.qp));
    score_tiles_kernel<<<(unsigned)np, 1024, 0, s>>>((int)np, (int)g.S, (int)G, (int)g.L, g.Lmax,
                                                     bn, causal, q_offset, p0, w.score_tiles,
                                                     w.counts);
    value_tiles_kernel<<<(unsigned)ceil_div(np * tt_n, 256), 256, 0, s>>>(
        (int)np, (int)g.S, (int)G, (int)g.d, bn, p0, w.value_tiles, w.counts + 1);
    st = check_launch("attention tile lists");
    if (st != NK_OK) return st;
    {  // S = Qp · Kᵀ (f32)
      TcArgs a{};
      a.w_scale = 1.0f;
      a.err = err;
      a.tiles = w.score_tiles;
      a.tile_count = w.counts;
      a.k_blocks = (int)ceil_div(g.d, 64);
      a.y = w.s;
      a.ldy = lds;
      a.y_f32 = 1;
      st = tc_gemm(WK_BF16, k_cache, pairs * g.Lmax, g.d, g.d * 2, w.qp, rows, g.d, g.d, bn, a,
                   num_sms(), s);
      if (st != NK_OK) return st;
    }
    {
      __nv_bfloat16 *pb = reinterpret_cast<__nv_bfloat16 *>(w.p);
      const unsigned wg = (unsigned)ceil_div(rows, 8);
#define NK_SOFTMAX_WARP(V)                                                                  \
  attn_softmax_warp_kernel<V><<<wg, 256, 0, s>>>(w.s, lds, (int)g.S, (int)G, (int)g.L,      \
                                                (int)kpad, causal, q_offset, sc, p0,        \
                                                (int)g.Hq, (int)g.Hkv, pb, kpad, rows, bad)
      if (kpad <= 128) NK_SOFTMAX_WARP(4);
      else if (kpad <= 512) NK_SOFTMAX_WARP(16);
      else if (kpad <= 1024) NK_SOFTMAX_WARP(32);
      else if (kpad <= 2048) NK_SOFTMAX_WARP(64);
      else
        attn_softmax_kernel<<<(unsigned)rows, 128, 0, s>>>(
            w.s, lds, (int)g.S, (int)G, (int)g.L, (int)kpad, causal, q_offset, sc, p0,
            (int)g.Hq, (int)g.Hkv, pb, kpad, bad);
#undef NK_SOFTMAX_WARP
    }
    st = check_launch("attn_softmax_kernel");
    if (st != NK_OK) return st;
    {  // O = P · V (the transposed V cache is the weight side)
      TcArgs a{};
      a.w_scale = 1.0f;
      a.err = err;
      a.tiles = w.value_tiles;
      a.tile_count = w.counts + 1;
      a.k_blocks = (int)(kpad / 64);
      a.y = w.op;
      a.ldy = g.d;
      a.y_f32 = 1;
      st = tc_gemm(WK_BF16, vt_cache, pairs * g.d, g.Lmax, g.Lmax * 2, w.p, rows, kpad, kpad,
                   bn, a, num_sms(), s);
      if (st != NK_OK) return st;
    }
    o_scatter_kernel<<<(unsigned)ceil_div(rows, 256 / (g.d / 4)), 256, 0, s>>>(
        reinterpret_cast<const float4 *>(w.op), (int)g.S, (int)g.Hq, (int)g.Hkv, (int)(g.d / 4),
        (int)p0, (int)rows, out, out_dtype == NK_DTYPE_F32);
    st = check_launch("o_scatter_kernel");
    if (st != NK_OK) return st;
  }
  return ok();
}

nk_status nk_attention_check(const void *workspace, int64_t *first_bad_row, void *stream) {
  // The workspace's first word: the first output row (b*S + s)*Hq + h of the
  // last nk_attention_gqa that used it whose scores had no finite value
  // (NoValidAttentionTargets), or -1.  Synchronises `stream`.
  if (!first_bad_row || !workspace) return fail(NK_INVALID_PARAMS, "workspace, first_bad_row");
  unsigned long long h = 0;
  NK_CUDA_TRY(cudaMemcpyAsync(&h, workspace, sizeof(h), cudaMemcpyDeviceToHost,
                              as_stream(stream)));
  NK_CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
  *first_bad_row = h == ~0ull ? -1 : (int64_t)h;
  return ok();
}

}  // extern "C"
