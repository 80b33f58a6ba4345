/*
 * nk_oracle.c — CPU restatement of the nemotron-cutile-rs host path.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker; never linked into libnk.so).
 * Compile with -ffp-contract=off so that every f32 multiply and add rounds
 * separately, as the Rust reference's do.  Citations are file:line within the
 * nemotron-cutile-rs project.
 */
#include "nk_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>

static int set_err(orc_error *err, int code) {
  if (err) err->code = code;
  return code;
}

static int len_err(orc_error *err, const char *arg, uint64_t expected, uint64_t actual) {
  if (err) {
    err->code = ORC_LENGTH_MISMATCH;
    err->argument = arg;
    err->expected = expected;
    err->actual = actual;
  }
  return ORC_LENGTH_MISMATCH;
}

/* activations.rs:68-71 — `x.max(0.0)` returns 0 for NaN, as fmaxf does. */
float orc_relu2(float x) {
  float r = fmaxf(x, 0.0f);
  return r * r;
}

/* activations.rs:73-81 — branch-stable sigmoid with f32 exp (libm expf). */
float orc_sigmoid(float x) {
  if (x >= 0.0f) {
    float z = expf(-x);
    return 1.0f / (1.0f + z);
  } else {
    float z = expf(x);
    return z / (1.0f + z);
  }
}

/* checked_shape_lengths (gemm.rs:192-208): zero dim or usize overflow -> InvalidShape. */
static int gemm_lengths(size_t m, size_t k, size_t n, size_t *ll, size_t *rl, size_t *ol) {
  if (m == 0 || k == 0 || n == 0) return ORC_INVALID_SHAPE;
  if (__builtin_mul_overflow(m, k, ll)) return ORC_INVALID_SHAPE;
  if (__builtin_mul_overflow(k, n, rl)) return ORC_INVALID_SHAPE;
  if (__builtin_mul_overflow(m, n, ol)) return ORC_INVALID_SHAPE;
  return ORC_OK;
}

/* gemm.rs:91-112 with validate_shape gemm.rs:114-147 (shape, lhs, rhs, output). */
int orc_gemm(const float *lhs, size_t lhs_len, const float *rhs, size_t rhs_len, size_t m,
             size_t k, size_t n, float *out, size_t out_len, orc_error *err) {
  size_t ll, rl, ol;
  if (gemm_lengths(m, k, n, &ll, &rl, &ol) != ORC_OK) return set_err(err, ORC_INVALID_SHAPE);
  if (lhs_len != ll) return len_err(err, "lhs", ll, lhs_len);
  if (rhs_len != rl) return len_err(err, "rhs", rl, rhs_len);
  if (out_len != ol) return len_err(err, "output", ol, out_len);
  for (size_t row = 0; row < m; ++row) {
    for (size_t col = 0; col < n; ++col) {
      double acc = 0.0;
      for (size_t depth = 0; depth < k; ++depth)
        acc += (double)lhs[row * k + depth] * (double)rhs[depth * n + col];
      out[row * n + col] = (float)acc;
    }
  }
  return set_err(err, ORC_OK);
}

typedef struct {
  const float *lhs, *rhs;
  float *out;
  size_t k, n, r0, r1;
} gemm_rows_job;

static void *gemm_rows_worker(void *p) {
  gemm_rows_job *j = (gemm_rows_job *)p;
  for (size_t row = j->r0; row < j->r1; ++row)
    for (size_t col = 0; col < j->n; ++col) {
      double acc = 0.0;
      for (size_t depth = 0; depth < j->k; ++depth)
        acc += (double)j->lhs[row * j->k + depth] * (double)j->rhs[depth * j->n + col];
      j->out[row * j->n + col] = (float)acc;
    }
  return NULL;
}

/* The gemm.rs:99-109 loop over rows [0, row_limit), split into contiguous row
 * ranges over `threads` POSIX threads (threads <= 1: the plain scalar loop). */
void orc_gemm_rows(const float *lhs, const float *rhs, size_t m, size_t k, size_t n,
                   size_t row_limit, float *out, int threads) {
  size_t rows = row_limit < m ? row_limit : m;
  if (threads < 1) threads = 1;
  if ((size_t)threads > rows) threads = (int)(rows ? rows : 1);
  gemm_rows_job jobs[256];
  pthread_t tids[256];
  if (threads > 256) threads = 256;
  for (int t = 0; t < threads; ++t) {
    jobs[t] = (gemm_rows_job){lhs, rhs, out, k, n, rows * t / threads, rows * (t + 1) / threads};
  }
  for (int t = 1; t < threads; ++t) pthread_create(&tids[t], NULL, gemm_rows_worker, &jobs[t]);
  gemm_rows_worker(&jobs[0]);
  for (int t = 1; t < threads; ++t) pthread_join(tids[t], NULL);
}

/* ---------------------------------------------------------------- quantize */

static size_t packed_len_of(size_t count) { return count / 2 + (count & 1); } /* quantize.rs:49-51 */

/* quantize.rs:59-81: length check, zero-fill, then per element (range check first). */
int orc_pack_int4(const uint8_t *values, size_t count, uint8_t *packed, size_t packed_len,
                  orc_error *err) {
  size_t expect = packed_len_of(count);
  if (packed_len != expect) return len_err(err, "packed", expect, packed_len);
  memset(packed, 0, packed_len);
  for (size_t i = 0; i < count; ++i) {
    uint8_t v = values[i];
    if (v > 0x0F) {
      if (err) err->byte_value = v;
      return set_err(err, ORC_INT4_OUT_OF_RANGE);
    }
    packed[i / 2] |= (i % 2 == 0) ? v : (uint8_t)(v << 4);
  }
  return set_err(err, ORC_OK);
}

/* quantize.rs:89-120 */
int orc_unpack_int4(const uint8_t *packed, size_t packed_len, size_t count, uint8_t *out,
                    size_t out_len, orc_error *err) {
  size_t expect = packed_len_of(count);
  if (packed_len != expect) return len_err(err, "packed", expect, packed_len);
  if (out_len != count) return len_err(err, "output", count, out_len);
  for (size_t i = 0; i < count; ++i) {
    uint8_t b = packed[i / 2];
    out[i] = (i % 2 == 0) ? (b & 0x0F) : ((b >> 4) & 0x0F);
  }
  return set_err(err, ORC_OK);
}

/* quantize.rs:180-186 */
int orc_validate_int4_params(float scale, uint32_t zero_point, orc_error *err) {
  if (!isfinite(scale) || scale <= 0.0f || zero_point > 0x0F)
    return set_err(err, ORC_INVALID_PARAMS);
  return set_err(err, ORC_OK);
}

/* quantize.rs:131-144 + quantize_scalar :188-200.  Validation order: params,
 * then every value (NonFiniteInput), then the packed length (inside pack). */
int orc_quantize_int4(const float *values, size_t count, float scale, uint32_t zero_point,
                      uint8_t *packed, size_t packed_len, orc_error *err) {
  if (orc_validate_int4_params(scale, zero_point, err) != ORC_OK) return ORC_INVALID_PARAMS;
  uint8_t *codes = (uint8_t *)malloc(count ? count : 1);
  for (size_t i = 0; i < count; ++i) {
    float v = values[i];
    if (!isfinite(v)) {
      free(codes);
      if (err) {
        err->index = i;
        err->value = v;
      }
      return set_err(err, ORC_NON_FINITE_INPUT);
    }
    float scaled = v / scale + (float)zero_point;
    float q = roundf(scaled); /* Rust f32::round: half away from zero */
    if (q < 0.0f) q = 0.0f;
    if (q > 15.0f) q = 15.0f;
    codes[i] = (uint8_t)q;
  }
  int rc = orc_pack_int4(codes, count, packed, packed_len, err);
  free(codes);
  return rc;
}

/* quantize.rs:156-178 + dequantize_scalar :202-204.  Order: params, output
 * length, then unpack (packed length). */
int orc_dequantize_int4(const uint8_t *packed, size_t packed_len, size_t count, float scale,
                        uint32_t zero_point, float *out, size_t out_len, orc_error *err) {
  if (orc_validate_int4_params(scale, zero_point, err) != ORC_OK) return ORC_INVALID_PARAMS;
  if (out_len != count) return len_err(err, "output", count, out_len);
  size_t expect = packed_len_of(count);
  if (packed_len != expect) return len_err(err, "packed", expect, packed_len);
  for (size_t i = 0; i < count; ++i) {
    uint8_t b = packed[i / 2];
    uint8_t code = (i % 2 == 0) ? (b & 0x0F) : ((b >> 4) & 0x0F);
    out[i] = ((float)code - (float)zero_point) * scale;
  }
  return set_err(err, ORC_OK);
}

/* EXTENSION (not in the reference): s[n] = max_k |W[n,k]| / 127,
 * q = clamp(round_half_away(W/s), -127, 127); an all-zero row gives s = 0, q = 0.
 * Non-finite weights are rejected like quantize_scalar (quantize.rs:193-195). */
int orc_quantize_int8_row(const float *w, size_t n, size_t k, int8_t *q, float *scales,
                          orc_error *err) {
  if (n == 0 || k == 0) return set_err(err, ORC_INVALID_SHAPE);
  for (size_t i = 0; i < n * k; ++i)
    if (!isfinite(w[i])) {
      if (err) {
        err->index = i;
        err->value = w[i];
      }
      return set_err(err, ORC_NON_FINITE_INPUT);
    }
  for (size_t r = 0; r < n; ++r) {
    float amax = 0.0f;
    for (size_t c = 0; c < k; ++c) amax = fmaxf(amax, fabsf(w[r * k + c]));
    float s = amax / 127.0f;
    scales[r] = s;
    for (size_t c = 0; c < k; ++c) {
      float v = 0.0f;
      if (s > 0.0f) {
        v = roundf(w[r * k + c] / s);
        if (v < -127.0f) v = -127.0f;
        if (v > 127.0f) v = 127.0f;
      }
      q[r * k + c] = (int8_t)v;
    }
  }
  return set_err(err, ORC_OK);
}

/* ----------------------------------------------------------------- routing */

/* f32::total_cmp key (IEEE totalOrder as a signed integer). */
static int32_t total_key(float f) {
  int32_t b;
  memcpy(&b, &f, 4);
  return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}

typedef struct {
  int32_t key;
  int32_t index;
  float weight;
} ranked;

/* sort_by: right.total_cmp(left) then left_index.cmp(right_index)
 * (moe_routing.rs:177-181, :202-206): weight descending, index ascending. */
static int ranked_cmp(const void *a, const void *b) {
  const ranked *l = (const ranked *)a, *r = (const ranked *)b;
  if (l->key != r->key) return l->key > r->key ? -1 : 1;
  return l->index < r->index ? -1 : (l->index > r->index);
}

/* moe_routing.rs:272-284 */
static int validate_route_shape(size_t experts, size_t top_k) {
  return (experts == 0 || top_k == 0 || top_k > experts) ? ORC_INVALID_SHAPE : ORC_OK;
}

int orc_route(const float *scores, size_t scores_len, size_t tokens, size_t experts,
              size_t top_k, int mode, int32_t *indices, size_t indices_len, float *weights,
              size_t weights_len, orc_error *err) {
  /* validate_route (moe_routing.rs:218-238) then validate_route_outputs (:240-270). */
  if (validate_route_shape(experts, top_k) != ORC_OK) return set_err(err, ORC_INVALID_SHAPE);
  size_t slen = tokens * experts, rlen = tokens * top_k;
  if (scores_len != slen) return len_err(err, "scores", slen, scores_len);
  if (indices_len != rlen) return len_err(err, "indices", rlen, indices_len);
  if (weights_len != rlen) return len_err(err, "weights", rlen, weights_len);
  ranked *buf = (ranked *)malloc(sizeof(ranked) * experts);
  for (size_t t = 0; t < tokens; ++t) {
    const float *s = scores + t * experts;
    if (mode == ORC_ROUTE_SOFTMAX) {
      /* select_top_k_softmax (moe_routing.rs:188-216) */
      float mx = -INFINITY;
      for (size_t e = 0; e < experts; ++e) mx = fmaxf(mx, s[e]);
      float total = -0.0f;
      for (size_t e = 0; e < experts; ++e) {
        buf[e].index = (int32_t)e;
        buf[e].weight = expf(s[e] - mx);
      }
      for (size_t e = 0; e < experts; ++e) total += buf[e].weight;
      for (size_t e = 0; e < experts; ++e) {
        buf[e].weight /= total;
        buf[e].key = total_key(buf[e].weight);
      }
      qsort(buf, experts, sizeof(ranked), ranked_cmp);
      float sel = -0.0f;
      for (size_t r = 0; r < top_k; ++r) sel += buf[r].weight;
      for (size_t r = 0; r < top_k; ++r) {
        indices[t * top_k + r] = buf[r].index;
        weights[t * top_k + r] = buf[r].weight / sel;
      }
    } else {
      /* select_top_k (moe_routing.rs:168-186) */
      for (size_t e = 0; e < experts; ++e) {
        buf[e].index = (int32_t)e;
        buf[e].weight = orc_sigmoid(s[e]);
        buf[e].key = total_key(buf[e].weight);
      }
      qsort(buf, experts, sizeof(ranked), ranked_cmp);
      for (size_t r = 0; r < top_k; ++r) {
        indices[t * top_k + r] = buf[r].index;
        weights[t * top_k + r] = buf[r].weight;
      }
      if (mode == ORC_ROUTE_SIGMOID_RENORM) {
        /* EXTENSION: the softmax router's selected-weight renormalisation
         * (moe_routing.rs:207-215) applied to sigmoid weights. */
        float sel = -0.0f;
        for (size_t r = 0; r < top_k; ++r) sel += weights[t * top_k + r];
        for (size_t r = 0; r < top_k; ++r) weights[t * top_k + r] /= sel;
      }
    }
  }
  free(buf);
  return set_err(err, ORC_OK);
}

void orc_route_histogram(const int32_t *indices, size_t tokens, size_t top_k, size_t experts,
                         int32_t *counts, int32_t *offsets, int32_t *perm) {
  memset(counts, 0, sizeof(int32_t) * experts);
  for (size_t i = 0; i < tokens * top_k; ++i) counts[indices[i]]++;
  int32_t run = 0;
  for (size_t e = 0; e < experts; ++e) {
    offsets[e] = run;
    run += counts[e];
  }
  if (!perm) return;
  int32_t *fill = (int32_t *)calloc(experts ? experts : 1, sizeof(int32_t));
  for (size_t i = 0; i < tokens * top_k; ++i) {
    int32_t e = indices[i];
    perm[offsets[e] + fill[e]++] = (int32_t)i;
  }
  free(fill);
}

/* ------------------------------------------------------------------ layers */

/* linear.rs:283-342: row count, input length, output length, GEMM, then bias
 * added in f32 row by row. */
int orc_linear(const float *w, const float *bias, size_t input_dim, size_t output_dim,
               const float *x, size_t x_len, size_t rows, float *out, size_t out_len,
               orc_error *err) {
  if (input_dim == 0 || output_dim == 0) return set_err(err, ORC_INVALID_SHAPE);
  if (rows == 0) return set_err(err, ORC_INVALID_ROW_COUNT);
  if (x_len != rows * input_dim) return len_err(err, "input", rows * input_dim, x_len);
  if (out_len != rows * output_dim) return len_err(err, "output", rows * output_dim, out_len);
  int rc = orc_gemm(x, x_len, w, input_dim * output_dim, rows, input_dim, output_dim, out,
                    out_len, err);
  if (rc != ORC_OK) return rc;
  if (bias)
    for (size_t r = 0; r < rows; ++r)
      for (size_t c = 0; c < output_dim; ++c) out[r * output_dim + c] += bias[c];
  return set_err(err, ORC_OK);
}

/* mlp.rs:157-211: up.project -> relu2 in place -> down.project_into. */
int orc_mlp(size_t hidden, size_t inter, const float *up_w, const float *up_b,
            const float *down_w, const float *down_b, const float *x, size_t rows,
            float *out, orc_error *err) {
  if (hidden == 0 || inter == 0) return set_err(err, ORC_INVALID_SHAPE);
  if (rows == 0) return set_err(err, ORC_INVALID_ROW_COUNT);
  float *act = (float *)malloc(sizeof(float) * rows * inter);
  int rc = orc_linear(up_w, up_b, hidden, inter, x, rows * hidden, rows, act, rows * inter, err);
  if (rc == ORC_OK) {
    for (size_t i = 0; i < rows * inter; ++i) act[i] = orc_relu2(act[i]);
    rc = orc_linear(down_w, down_b, inter, hidden, act, rows * inter, rows, out, rows * hidden,
                    err);
  }
  free(act);
  return rc;
}

/* moe.rs:154-249 */
int orc_moe(size_t hidden, size_t experts, size_t top_k, size_t inter, size_t shared_inter,
            const float *router_w, const float *router_b, const float *up_w, const float *up_b,
            const float *down_w, const float *down_b, const float *sh_up_w,
            const float *sh_up_b, const float *sh_down_w, const float *sh_down_b,
            int route_mode, const float *x, size_t rows, float *out, int32_t *out_indices,
            float *out_weights, orc_error *err) {
  if (hidden == 0 || experts == 0 || top_k == 0 || top_k > experts)
    return set_err(err, ORC_INVALID_SHAPE);
  if (rows == 0) return set_err(err, ORC_INVALID_ROW_COUNT);
  int rc;
  float *scores = (float *)malloc(sizeof(float) * rows * experts);
  rc = orc_linear(router_w, router_b, hidden, experts, x, rows * hidden, rows, scores,
                  rows * experts, err);
  if (rc != ORC_OK) {
    free(scores);
    return rc;
  }
  int32_t *idx = (int32_t *)malloc(sizeof(int32_t) * rows * top_k);
  float *wts = (float *)malloc(sizeof(float) * rows * top_k);
  rc = orc_route(scores, rows * experts, rows, experts, top_k, route_mode, idx, rows * top_k,
                 wts, rows * top_k, err);
  free(scores);
  if (rc != ORC_OK) {
    free(idx);
    free(wts);
    return rc;
  }
  /* Expert outputs for the routed rows: y_slot[(t*top_k + r)*hidden + c]. */
  int32_t *counts = (int32_t *)malloc(sizeof(int32_t) * experts);
  int32_t *offs = (int32_t *)malloc(sizeof(int32_t) * experts);
  int32_t *perm = (int32_t *)malloc(sizeof(int32_t) * rows * top_k);
  orc_route_histogram(idx, rows, top_k, experts, counts, offs, perm);
  float *yslot = (float *)malloc(sizeof(float) * rows * top_k * hidden);
  for (size_t e = 0; e < experts && rc == ORC_OK; ++e) {
    size_t cnt = (size_t)counts[e];
    if (!cnt) continue;
    float *xe = (float *)malloc(sizeof(float) * cnt * hidden);
    float *ye = (float *)malloc(sizeof(float) * cnt * hidden);
    for (size_t j = 0; j < cnt; ++j) {
      size_t slot = (size_t)perm[offs[e] + j];
      memcpy(xe + j * hidden, x + (slot / top_k) * hidden, sizeof(float) * hidden);
    }
    rc = orc_mlp(hidden, inter, up_w + e * hidden * inter, up_b ? up_b + e * inter : NULL,
                 down_w + e * inter * hidden, down_b ? down_b + e * hidden : NULL, xe, cnt, ye,
                 err);
    for (size_t j = 0; j < cnt && rc == ORC_OK; ++j) {
      size_t slot = (size_t)perm[offs[e] + j];
      memcpy(yslot + slot * hidden, ye + j * hidden, sizeof(float) * hidden);
    }
    free(xe);
    free(ye);
  }
  float *shared = NULL;
  if (rc == ORC_OK && sh_up_w) {
    shared = (float *)malloc(sizeof(float) * rows * hidden);
    rc = orc_mlp(hidden, shared_inter, sh_up_w, sh_up_b, sh_down_w, sh_down_b, x, rows, shared,
                 err);
  }
  if (rc == ORC_OK) {
    /* output.fill(0); out += shared; out += w_r * expert_r in rank order (moe.rs:195-246) */
    for (size_t t = 0; t < rows; ++t) {
      float *o = out + t * hidden;
      for (size_t c = 0; c < hidden; ++c) o[c] = 0.0f;
      if (shared)
        for (size_t c = 0; c < hidden; ++c) o[c] += shared[t * hidden + c];
      for (size_t r = 0; r < top_k; ++r) {
        float w = wts[t * top_k + r];
        const float *y = yslot + (t * top_k + r) * hidden;
        for (size_t c = 0; c < hidden; ++c) o[c] += w * y[c];
      }
    }
    if (out_indices) memcpy(out_indices, idx, sizeof(int32_t) * rows * top_k);
    if (out_weights) memcpy(out_weights, wts, sizeof(float) * rows * top_k);
  }
  free(shared);
  free(yslot);
  free(counts);
  free(offs);
  free(perm);
  free(idx);
  free(wts);
  return rc == ORC_OK ? set_err(err, ORC_OK) : rc;
}

uint16_t orc_f32_to_bf16(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

float orc_bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* ------------------------------------------------------------ Mamba2 glue */

/* activations.rs:64-66 */
float orc_silu(float x) { return x * orc_sigmoid(x); }

/* conv1d.rs:78-124, validation order conv1d.rs:126-158. */
int orc_conv1d(const float *input, size_t input_len, const float *weights, size_t weights_len,
               size_t seq, size_t channels, size_t kernel_size, float *out, size_t out_len,
               orc_error *err) {
  if (channels == 0 || kernel_size == 0) return set_err(err, ORC_INVALID_SHAPE);
  if (input_len != seq * channels) return len_err(err, "input", seq * channels, input_len);
  if (weights_len != channels * kernel_size)
    return len_err(err, "weights", channels * kernel_size, weights_len);
  if (out_len != seq * channels) return len_err(err, "output", seq * channels, out_len);
  for (size_t t = 0; t < seq; ++t)
    for (size_t ch = 0; ch < channels; ++ch) {
      double acc = 0.0;
      for (size_t tap = 0; tap < kernel_size && tap <= t; ++tap)
        acc += (double)input[(t - tap) * channels + ch] *
               (double)weights[ch * kernel_size + (kernel_size - 1 - tap)];
      out[t * channels + ch] = (float)acc;
    }
  return set_err(err, ORC_OK);
}

/* ssm.rs:257-263: threshold 20, otherwise ln(1 + e^v) in f32. */
static float orc_softplus(float v) { return v > 20.0f ? v : logf(1.0f + expf(v)); }

/* ssm.rs:123-175 */
int orc_selective_scan(const float *input, size_t input_len, const float *delta_t,
                       size_t delta_t_len, const float *a, size_t a_len, const float *b,
                       size_t b_len, const float *c, size_t c_len, const float *d, size_t d_len,
                       const float *initial_state, size_t initial_state_len, float delta_bias,
                       int apply_softplus, size_t seq, size_t channels, size_t states,
                       float *out, size_t out_len, float *final_state, size_t final_state_len,
                       orc_error *err) {
  if (seq == 0 || channels == 0 || states == 0) return set_err(err, ORC_INVALID_SHAPE);
  const size_t n = seq * channels, sm = channels * states, bl = seq * channels * states;
  if (input_len != n) return len_err(err, "input", n, input_len);
  if (delta_t_len != n) return len_err(err, "delta_t", n, delta_t_len);
  if (a_len != sm) return len_err(err, "a", sm, a_len);
  if (b_len != bl) return len_err(err, "b", bl, b_len);
  if (c_len != bl) return len_err(err, "c", bl, c_len);
  if (d && d_len != channels) return len_err(err, "d", channels, d_len);
  if (initial_state && initial_state_len != sm)
    return len_err(err, "initial_state", sm, initial_state_len);
  if (out_len != n) return len_err(err, "output", n, out_len);
  if (final_state_len != sm) return len_err(err, "final_state", sm, final_state_len);

  if (initial_state)
    memcpy(final_state, initial_state, sizeof(float) * sm);
  else
    memset(final_state, 0, sizeof(float) * sm);

  for (size_t t = 0; t < seq; ++t)
    for (size_t ch = 0; ch < channels; ++ch) {
      const size_t i = t * channels + ch;
      const float x = input[i];
      const float raw = delta_t[i] + delta_bias;
      const float dt = apply_softplus ? orc_softplus(raw) : raw;
      if (!isfinite(dt) || dt < 0.0f) {
        if (err) {
          err->code = ORC_INVALID_DELTA_T;
          err->index = i;
          err->value = dt;
        }
        return ORC_INVALID_DELTA_T;
      }
      double acc = 0.0;
      for (size_t s = 0; s < states; ++s) {
        const size_t m = ch * states + s, o = i * states + s;
        const float transition = expf(dt * a[m]);
        const float mix = dt * b[o] * x;
        const float next = transition * final_state[m] + mix;
        final_state[m] = next;
        acc += (double)(c[o] * next);
      }
      if (d) acc += (double)(d[ch] * x);
      out[i] = (float)acc;
    }
  return set_err(err, ORC_OK);
}

/* rms_norm.rs:64-144: lengths (validate_lengths :146-183), then rms_host
 * :108-124 (empty, negative epsilon, f64 mean square cast to f32, + eps,
 * sqrt), reciprocal, x * scale * weight (* gate). */
int orc_rms_norm(const float *input, size_t len, const float *weight, size_t weight_len,
                 const float *gate, size_t gate_len, float epsilon, float *out, size_t out_len,
                 orc_error *err) {
  if (len == 0) return set_err(err, ORC_EMPTY_INPUT);
  if (weight_len != len) return len_err(err, "weight", len, weight_len);
  if (gate && gate_len != len) return len_err(err, "gate", len, gate_len);
  if (out_len != len) return len_err(err, "output", len, out_len);
  if (epsilon < 0.0f) {
    if (err) {
      err->code = ORC_NEGATIVE_EPSILON;
      err->value = epsilon;
    }
    return ORC_NEGATIVE_EPSILON;
  }
  double sum = 0.0;
  for (size_t i = 0; i < len; ++i) sum += (double)input[i] * (double)input[i];
  const float denom = sqrtf((float)(sum / (double)len) + epsilon);
  const float scale = 1.0f / denom;
  for (size_t i = 0; i < len; ++i) {
    float v = input[i] * scale * weight[i];
    if (gate) v *= gate[i];
    out[i] = v;
  }
  return set_err(err, ORC_OK);
}

/* activations.rs:95-97 (silu_in_place_host). */
void orc_silu_in_place(float *values, size_t n) {
  for (size_t i = 0; i < n; ++i) values[i] = orc_silu(values[i]);
}

/* ----------------------------------------------------------- attention core */

static size_t attn_off(size_t b, size_t s, size_t h, size_t d, size_t seq, size_t heads,
                       size_t hd) {
  return ((b * seq + s) * heads + h) * hd + d; /* attention.rs:450-460 */
}

/* attention.rs:204-302 */
int orc_attention(const float *q, size_t q_len, const float *k, size_t k_len, const float *v,
                  size_t v_len, size_t batch, size_t q_seq, size_t kv_seq, size_t q_heads,
                  size_t kv_heads, size_t head_dim, int causal, size_t q_offset, int has_scale,
                  float scale, float *out, size_t out_len, orc_error *err) {
  if (!batch || !q_seq || !kv_seq || !q_heads || !kv_heads || !head_dim)
    return set_err(err, ORC_INVALID_SHAPE);
  if (q_heads % kv_heads) return set_err(err, ORC_HEAD_COUNT_MISMATCH);
  const size_t ql = batch * q_seq * q_heads * head_dim, kl = batch * kv_seq * kv_heads * head_dim;
  if (q_len != ql) return len_err(err, "query", ql, q_len);
  if (k_len != kl) return len_err(err, "key", kl, k_len);
  if (v_len != kl) return len_err(err, "value", kl, v_len);
  if (out_len != ql) return len_err(err, "output", ql, out_len);
  const float sc = has_scale ? scale : 1.0f / sqrtf((float)head_dim); /* :82-93 */
  if (!isfinite(sc) || sc <= 0.0f) {
    if (err) {
      err->code = ORC_INVALID_SCALE;
      err->value = sc;
    }
    return ORC_INVALID_SCALE;
  }
  const size_t group = q_heads / kv_heads;
  float *scores = (float *)malloc(sizeof(float) * kv_seq);
  float *weights = (float *)malloc(sizeof(float) * kv_seq);
  int rc = ORC_OK;
  for (size_t b = 0; b < batch && rc == ORC_OK; ++b)
    for (size_t qi = 0; qi < q_seq && rc == ORC_OK; ++qi) {
      size_t max_key = kv_seq - 1;
      if (causal) {
        const size_t lim = q_offset + qi;
        max_key = lim < kv_seq - 1 ? lim : kv_seq - 1;
      }
      for (size_t h = 0; h < q_heads && rc == ORC_OK; ++h) {
        const size_t kh = h / group;
        for (size_t j = 0; j < kv_seq; ++j) {
          scores[j] = -INFINITY;
          if (causal && j > max_key) continue;
          double s = 0.0;
          for (size_t d = 0; d < head_dim; ++d)
            s += (double)q[attn_off(b, qi, h, d, q_seq, q_heads, head_dim)] *
                 (double)k[attn_off(b, j, kh, d, kv_seq, kv_heads, head_dim)];
          scores[j] = (float)s * sc;
        }
        float mx = -INFINITY;
        for (size_t j = 0; j < kv_seq; ++j)
          if (isfinite(scores[j])) mx = fmaxf(mx, scores[j]);
        if (!isfinite(mx)) {
          if (err) {
            err->code = ORC_NO_VALID_TARGETS;
            err->index = (b * q_seq + qi) * q_heads + h;
          }
          rc = ORC_NO_VALID_TARGETS;
          break;
        }
        double part = 0.0;
        for (size_t j = 0; j < kv_seq; ++j) {
          if (isfinite(scores[j])) {
            weights[j] = expf(scores[j] - mx);
            part += (double)weights[j];
          } else {
            weights[j] = 0.0f;
          }
        }
        if (part == 0.0) {
          if (err) {
            err->code = ORC_ZERO_PARTITION;
            err->index = (b * q_seq + qi) * q_heads + h;
          }
          rc = ORC_ZERO_PARTITION;
          break;
        }
        const float inv = (float)(1.0 / part);
        for (size_t d = 0; d < head_dim; ++d) {
          double acc = 0.0;
          for (size_t j = 0; j < kv_seq; ++j) {
            if (weights[j] == 0.0f) continue;
            acc += (double)(weights[j] * inv) *
                   (double)v[attn_off(b, j, kh, d, kv_seq, kv_heads, head_dim)];
          }
          out[attn_off(b, qi, h, d, q_seq, q_heads, head_dim)] = (float)acc;
        }
      }
    }
  free(scores);
  free(weights);
  return rc == ORC_OK ? set_err(err, ORC_OK) : rc;
}
