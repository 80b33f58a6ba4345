/*
 * nk_oracle.h — CPU restatement of the nemotron-cutile-rs host path for the
 * GEMM / quantized-linear / MoE hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker: the pytest
 * suite, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm
 * are its only callers.  The product (libnk.so) never links, loads or calls it.
 *
 * Every function restates one reference function (cited file:line within the
 * nemotron-cutile-rs project) with the same loop order, the same accumulation
 * widths (f64 for GEMM, f32 elsewhere) and the same validation order, and
 * returns the same error variant as an integer code plus detail fields.
 *
 * Two functions are EXTENSIONS that the reference does not contain (its
 * quantizer is INT4-affine per tensor only, and its sigmoid router does not
 * renormalise):
 *   orc_quantize_int8_row     (int8 symmetric per-output-row absmax)
 *   orc_route (mode SIGMOID_RENORM)
 * Their parity is pinned only by the restated formula and hand-built KATs.
 */
#ifndef NK_ORACLE_H
#define NK_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Error codes share their numbering with include/nk.h (NK_*). */
enum {
  ORC_OK = 0,
  ORC_INVALID_SHAPE = 1,
  ORC_LENGTH_MISMATCH = 2,
  ORC_INVALID_PARAMS = 3,
  ORC_INT4_OUT_OF_RANGE = 4,
  ORC_NON_FINITE_INPUT = 5,
  ORC_INVALID_ROW_COUNT = 6,
  ORC_INVALID_DELTA_T = 11,  /* ssm.rs SsmError::InvalidDeltaT; index = t*C + ch */
  ORC_EMPTY_INPUT = 12,      /* rms_norm.rs RmsNormError::EmptyInput */
  ORC_NEGATIVE_EPSILON = 13, /* rms_norm.rs RmsNormError::NegativeEpsilon; value = eps */
  ORC_HEAD_COUNT_MISMATCH = 14, /* attention.rs HeadCountMismatch / InvalidHeadGrouping */
  ORC_INVALID_SCALE = 15,       /* attention.rs InvalidScale; value = scale */
  ORC_NO_VALID_TARGETS = 16,    /* attention.rs NoValidAttentionTargets; index = (b*Sq+q)*Hq+h */
  ORC_ZERO_PARTITION = 17,      /* attention.rs ZeroPartition; index as above */
};

typedef struct orc_error {
  int code;
  const char *argument; /* LengthMismatch argument name */
  uint64_t expected;
  uint64_t actual;
  uint64_t index;       /* NonFiniteInput index */
  float value;          /* NonFiniteInput value */
  uint32_t byte_value;  /* Int4OutOfRange value */
} orc_error;

/* Routing modes. */
enum { ORC_ROUTE_SIGMOID = 0, ORC_ROUTE_SOFTMAX = 1, ORC_ROUTE_SIGMOID_RENORM = 2 };

/* activations.rs:68-81 */
float orc_relu2(float x);
float orc_sigmoid(float x);

/* gemm.rs:91-112 (+ validate_shape :114-147, checked_shape_lengths :192-208). */
int orc_gemm(const float *lhs, size_t lhs_len, const float *rhs, size_t rhs_len,
             size_t m, size_t k, size_t n, float *out, size_t out_len, orc_error *err);

/* quantize.rs:59-81 */
int orc_pack_int4(const uint8_t *values, size_t count, uint8_t *packed, size_t packed_len,
                  orc_error *err);
/* quantize.rs:89-120 */
int orc_unpack_int4(const uint8_t *packed, size_t packed_len, size_t count, uint8_t *out,
                    size_t out_len, orc_error *err);
/* quantize.rs:131-144 */
int orc_quantize_int4(const float *values, size_t count, float scale, uint32_t zero_point,
                      uint8_t *packed, size_t packed_len, orc_error *err);
/* quantize.rs:156-178 */
int orc_dequantize_int4(const uint8_t *packed, size_t packed_len, size_t count, float scale,
                        uint32_t zero_point, float *out, size_t out_len, orc_error *err);
/* quantize.rs:180-186 */
int orc_validate_int4_params(float scale, uint32_t zero_point, orc_error *err);

/* EXTENSION: int8 per-output-row symmetric absmax quantization of W[N,K]. */
int orc_quantize_int8_row(const float *w, size_t n, size_t k, int8_t *q, float *scales,
                          orc_error *err);

/* moe_routing.rs:118-141 (+ :98-112 softmax, select_top_k :168-186,
 * select_top_k_softmax :188-216, validate_route :218-238).  Indices are
 * written as int32. */
int orc_route(const float *scores, size_t scores_len, size_t tokens, size_t experts,
              size_t top_k, int mode, int32_t *indices, size_t indices_len, float *weights,
              size_t weights_len, orc_error *err);

/* Derived routing bookkeeping (not in the reference, which runs experts over all rows):
 * counts[e] = #{(t,r): idx[t,r] = e}; offsets = exclusive scan of counts;
 * perm lists route slots t*top_k+r grouped by expert, ascending slot order
 * inside each expert (stable). */
void orc_route_histogram(const int32_t *indices, size_t tokens, size_t top_k, size_t experts,
                         int32_t *counts, int32_t *offsets, int32_t *perm);

/* linear.rs:283-342: Y = X·W (+ b); W row-major [input_dim, output_dim]. */
int orc_linear(const float *w, const float *bias, size_t input_dim, size_t output_dim,
               const float *x, size_t x_len, size_t rows, float *out, size_t out_len,
               orc_error *err);

/* mlp.rs:157-211: down(relu2(up(x))). */
int orc_mlp(size_t hidden, size_t inter, const float *up_w, const float *up_b,
            const float *down_w, const float *down_b, const float *x, size_t rows,
            float *out, orc_error *err);

/* moe.rs:154-249.  Expert e's weights live at up_w + e*hidden*inter and
 * down_w + e*inter*hidden (each in the reference [input_dim, output_dim]
 * layout); biases may be NULL.  shared_* may be NULL (no shared expert).
 * route_mode selects the router (SIGMOID is the reference; RENORM the
 * extension).  The reference evaluates each selected expert over all rows;
 * row t of an MLP depends only on row t of its input, so this restatement
 * evaluates only the rows routed to the expert and produces the same values. */
int orc_moe(size_t hidden, size_t experts, size_t top_k, size_t inter, size_t shared_inter,
            const float *router_w, const float *router_b, const float *up_w, const float *up_b,
            const float *down_w, const float *down_b, const float *sh_up_w,
            const float *sh_up_b, const float *sh_down_w, const float *sh_down_b,
            int route_mode, const float *x, size_t rows, float *out, int32_t *out_indices,
            float *out_weights, orc_error *err);

/* Timing helper for the CPU baseline: the reference GEMM loop over the first
 * `row_limit` rows only (the loop cost is linear in rows).  Optional
 * row-range parallelism over POSIX threads when threads > 1 (a parallelised
 * restatement, not the reference). */
void orc_gemm_rows(const float *lhs, const float *rhs, size_t m, size_t k, size_t n,
                   size_t row_limit, float *out, int threads);

/* ---- Mamba2 glue (the stages between in_proj and out_proj) ---- */

/* activations.rs:64-66: x * sigmoid(x). */
float orc_silu(float x);
/* activations.rs:95-97 */
void orc_silu_in_place(float *values, size_t n);

/* conv1d.rs:78-124 (+ validate_shape :126-158): depthwise causal conv,
 * input [seq, C], weights [C, K] applied reversed (tap j reads t-j with
 * weights[ch*K + K-1-j]), f64 accumulation, zero history before t = 0. */
int orc_conv1d(const float *input, size_t input_len, const float *weights, size_t weights_len,
               size_t seq, size_t channels, size_t kernel_size, float *out, size_t out_len,
               orc_error *err);

/* ssm.rs:123-175 (+ validate_params :177-211, validate_shape :239-245,
 * softplus :257-263, validated_delta_t :265-288).  d and initial_state may be
 * NULL.  On InvalidDeltaT, err->index = t*C + ch and err->value = dt. */
int orc_selective_scan(const float *input, size_t input_len, const float *delta_t,
                       size_t delta_t_len, const float *a, size_t a_len, const float *b,
                       size_t b_len, const float *c, size_t c_len, const float *d, size_t d_len,
                       const float *initial_state, size_t initial_state_len, float delta_bias,
                       int apply_softplus, size_t seq, size_t channels, size_t states,
                       float *out, size_t out_len, float *final_state, size_t final_state_len,
                       orc_error *err);

/* rms_norm.rs:64-144: rms_norm_into_host (gate NULL) / gated_rms_norm_into_host.
 * One vector; the row-wise contract applies this per row. */
int orc_rms_norm(const float *input, size_t len, const float *weight, size_t weight_len,
                 const float *gate, size_t gate_len, float epsilon, float *out, size_t out_len,
                 orc_error *err);

/* ---- attention core (nemotron-kernels/src/attention.rs) ---- */

/* scaled_dot_product_attention_into_host (attention.rs:204-302) with
 * attention_scores_host (:132-190), validate_shape (:304-357) and
 * AttentionOptions::resolve_scale (:82-93).  q [B, Sq, Hq, d], k/v
 * [B, Skv, Hkv, d], out [B, Sq, Hq, d].  scale <= 0 with has_scale = 0 means
 * the default 1/sqrt(d). */
int orc_attention(const float *q, size_t q_len, const float *k, size_t k_len, const float *v,
                  size_t v_len, size_t batch, size_t q_seq, size_t kv_seq, size_t q_heads,
                  size_t kv_heads, size_t head_dim, int causal, size_t q_offset, int has_scale,
                  float scale, float *out, size_t out_len, orc_error *err);

/* bf16 helpers shared by the tests: round-to-nearest-even f32 -> bf16. */
uint16_t orc_f32_to_bf16(float x);
float orc_bf16_to_f32(uint16_t b);

#ifdef __cplusplus
}
#endif
#endif
