/*
 * nk.h — C ABI of libnk, the B200 (sm_100a) implementation of the
 * nemotron-cutile-rs matrix-multiplication hot path.
 *
 * Each entry point replaces one function of the reference's Rust kernel
 * wrappers (paths are within the nemotron-cutile-rs project).  The Rust side
 * keeps its public API and swaps the body for an `extern "C"` call.
 *
 * Conventions
 *   - Every function returns an nk_status.  NK_OK is 0.  On error, the
 *     calling thread's nk_error_info (nk_last_error) holds the detail that
 *     the matching Rust error variant carries.
 *   - Validation order is the reference's: shape first, then argument
 *     lengths in the reference's order.  Lengths are element counts
 *     (the Rust slice / GpuTensor::numel values).
 *   - Pointers named x, w, y, out, scores, ... are DEVICE pointers unless the
 *     name ends in _host.  Calls are asynchronous on `stream` (a
 *     cudaStream_t; NULL = the legacy default stream) unless stated.
 *   - Conditions only the device can detect (a non-finite value during
 *     quantization, an int4 code above 15, a kernel wait that timed out)
 *     are reported by the functions that document a synchronisation, or
 *     by nk_device_status().
 *   - No entry point falls back to a CPU implementation.
 */
#ifndef NK_H
#define NK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ---------------------------------------------------------------- status */
typedef int nk_status;
enum {
  NK_OK = 0,
  NK_INVALID_SHAPE = 1,      /* GemmError::InvalidShape, QuantizeError/MoeRoutingError InvalidShape */
  NK_LENGTH_MISMATCH = 2,    /* *::LengthMismatch{argument, expected, actual} */
  NK_INVALID_PARAMS = 3,     /* QuantizeError::InvalidParams */
  NK_INT4_OUT_OF_RANGE = 4,  /* QuantizeError::Int4OutOfRange(u8) */
  NK_NON_FINITE_INPUT = 5,   /* QuantizeError::NonFiniteInput{index, value} */
  NK_INVALID_ROW_COUNT = 6,  /* LinearError/MlpError/MoeError::InvalidRowCount */
  NK_UNSUPPORTED = 7,        /* a layout/dtype combination libnk does not implement */
  NK_DEVICE_ERROR = 8,       /* *::DeviceError(String) */
  NK_TIMEOUT = 9,            /* a bounded device-side wait gave up */
  NK_WORKSPACE_TOO_SMALL = 10,
  NK_INVALID_DELTA_T = 11,   /* SsmError::InvalidDeltaT (index = (b*seq + t)*C + ch, value = dt) */
  NK_EMPTY_INPUT = 12,       /* RmsNormError::EmptyInput */
  NK_NEGATIVE_EPSILON = 13,  /* RmsNormError::NegativeEpsilon (value = epsilon) */
  NK_HEAD_COUNT_MISMATCH = 14, /* AttentionError::HeadCountMismatch (expected = Hq, actual = Hkv) */
  NK_INVALID_SCALE = 15,     /* AttentionError::InvalidScale (value = scale) */
  NK_NO_VALID_TARGETS = 16,  /* AttentionError::NoValidAttentionTargets (index = (b*Sq + q)*Hq + h) */
  NK_ZERO_PARTITION = 17,    /* AttentionError::ZeroPartition (index as above) */
  NK_TOKEN_OUT_OF_RANGE = 18 /* EmbeddingError::TokenOutOfRange (actual = token id, expected = vocab, index = position) */
};

typedef struct nk_error_info {
  int32_t code;
  char argument[32];   /* LengthMismatch argument name ("lhs", "rhs", "output", ...) */
  uint64_t expected;
  uint64_t actual;
  uint64_t index;      /* NonFiniteInput index */
  float value;         /* NonFiniteInput value */
  uint32_t byte_value; /* Int4OutOfRange value */
  char message[256];   /* human-readable; DeviceError carries the CUDA error string */
} nk_error_info;

/* Copies the calling thread's last error into *out; returns its code. */
nk_status nk_last_error(nk_error_info *out);
/* Library version (major*10000 + minor*100 + patch). */
int32_t nk_version(void);
/* Synchronises `stream` and reports a device-side failure recorded by any
 * libnk kernel on the current device since the last call (NK_TIMEOUT when a
 * bounded wait gave up), then clears it. */
nk_status nk_device_status(void *stream);

/* Failure-detection self test: launches one kernel whose bounded device-side
 * wait (the kind every libnk kernel uses on its barriers) runs out after
 * about 2 s because nothing completes it; the kernel records NK_TIMEOUT and
 * returns, so the next nk_device_status(stream) reports NK_TIMEOUT (and
 * clears it) and the context stays usable.  No fault, trap or hang. */
nk_status nk_selftest_wait_timeout(void *stream);

/* dtypes of activations / outputs */
enum { NK_F32 = 0, NK_BF16 = 1 };
/* epilogue flags */
enum { NK_EPI_RELU2 = 1 };

/* ------------------------------------------------------------------ GEMM */

/* Replaces nemotron_kernels::gemm::{gemm, gemm_into} (gemm.rs:318-363) and
 * the host loop gemm_into_host (gemm.rs:91-112).
 * C[M,N] = A[M,K] · B[K,N], f32 row-major, the reference layout, accumulated
 * in f64 and rounded once to f32 like the host loop.  Validation follows
 * validate_shape (gemm.rs:114-147): zero dim or overflow -> NK_INVALID_SHAPE,
 * then lhs, rhs, output lengths -> NK_LENGTH_MISMATCH. Writes `out` in place. */
nk_status nk_gemm_f32(const float *lhs, size_t lhs_len, const float *rhs, size_t rhs_len,
                      float *out, size_t out_len, size_t m, size_t k, size_t n, void *stream);

/* The projection GEMM behind LinearProjection::project_into
 * (nemotron-nn/src/linear.rs:283-342), which Mamba2 in/out projections
 * (mamba2.rs:229-263,353-359), attention Q/K/V/O (attention.rs:170-209) and the
 * MLP/MoE experts (mlp.rs:201-208) call:
 *   Y[M,N] = epilogue( X[M,K] · Wᵀ ),  W stored [N,K] (K contiguous).
 * x_dtype: NK_BF16 or NK_F32 (f32 activations are split into two bf16
 * halves, hi + lo, which keep the top 16 of the 24 significand bits, so the
 * product carries ~16 mantissa bits of x).  y_dtype: NK_BF16 or NK_F32.
 * bias: f32 [N] or NULL, added after the GEMM as linear.rs:333-339 does.
 * flags: NK_EPI_RELU2 applies relu2 (activations.rs:68-71) after the bias,
 * fusing mlp.rs:205.  Accumulation is f32 in tensor memory.
 *
 * Scratch: decode shapes split K over CTAs (f32 partial sums) and f32
 * activations need their bf16 split; these calls keep that scratch in a
 * library block per (device, stream), grown on first need (cudaMalloc) and
 * reused.  Calls on different streams never share it; calls on one stream
 * are ordered by the stream.  Growth is refused with NK_WORKSPACE_TOO_SMALL
 * while the stream is being captured into a CUDA graph: run each shape once
 * before capturing.  nk_scratch_release frees a stream's block.  The *_ws
 * forms below take caller-owned scratch instead and allocate nothing. */
nk_status nk_gemm_bf16(const void *x, int32_t x_dtype, const uint16_t *w, const float *bias,
                       void *y, int32_t y_dtype, int64_t m, int64_t k, int64_t n, int32_t flags,
                       void *stream);

/* Same contract with int8 weights quantized per output row (symmetric absmax,
 * nk_quantize_int8_row): W ≈ diag(scales) · wq, wq [N,K] int8, scales f32 [N].
 * Dequantization happens inside the GEMM (codes are exact in bf16; the row
 * scale is applied in the epilogue).  Not in the reference: it is the format
 * the benchmark configurations name. */
nk_status nk_gemm_w8row(const void *x, int32_t x_dtype, const int8_t *wq, const float *scales,
                        const float *bias, void *y, int32_t y_dtype, int64_t m, int64_t k,
                        int64_t n, int32_t flags, void *stream);

/* Same contract with the reference's INT4-affine per-tensor weights
 * (quantize.rs:131-204) in the reference's own linear layout: element (k, n)
 * of the [K,N] = [input_dim, output_dim] matrix (linear.rs:324) has flat
 * index k*N+n and lives in byte index/2, low nibble for even index
 * (quantize.rs:59-81).  W = (code - zero_point) * scale, dequantized inside
 * the GEMM.  Replaces the materialise-then-GEMM route of
 * Int4LinearWeights::materialize_dense (linear.rs:126-131), which the
 * reference's project() refuses (linear.rs:316-321).  packed_len must be
 * ceil(K*N/2). */
nk_status nk_gemm_w4a(const void *x, int32_t x_dtype, const uint8_t *packed, size_t packed_len,
                      float scale, uint32_t zero_point, const float *bias, void *y,
                      int32_t y_dtype, int64_t m, int64_t k, int64_t n, int32_t flags,
                      void *stream);

/* Scratch bytes a projection of this shape needs (0 when none):
 * weight_kind NK_W_BF16 / NK_W_INT8_ROW / NK_W_INT4_AFFINE, x_dtype as above.
 * The same shapes and kinds always need the same bytes on one device. */
nk_status nk_gemm_workspace_bytes(int32_t weight_kind, int32_t x_dtype, int64_t m, int64_t k,
                                  int64_t n, size_t *bytes);

/* nk_gemm_bf16 / nk_gemm_w8row / nk_gemm_w4a with caller-owned scratch
 * (device memory of at least nk_gemm_workspace_bytes; may be NULL when that
 * is 0): re-entrant across host threads and streams as long as concurrent
 * calls get distinct workspaces.  NK_WORKSPACE_TOO_SMALL when it is short. */
nk_status nk_gemm_bf16_ws(const void *x, int32_t x_dtype, const uint16_t *w, const float *bias,
                          void *y, int32_t y_dtype, int64_t m, int64_t k, int64_t n,
                          int32_t flags, void *workspace, size_t workspace_bytes, void *stream);
nk_status nk_gemm_w8row_ws(const void *x, int32_t x_dtype, const int8_t *wq, const float *scales,
                           const float *bias, void *y, int32_t y_dtype, int64_t m, int64_t k,
                           int64_t n, int32_t flags, void *workspace, size_t workspace_bytes,
                           void *stream);
nk_status nk_gemm_w4a_ws(const void *x, int32_t x_dtype, const uint8_t *packed, size_t packed_len,
                         float scale, uint32_t zero_point, const float *bias, void *y,
                         int32_t y_dtype, int64_t m, int64_t k, int64_t n, int32_t flags,
                         void *workspace, size_t workspace_bytes, void *stream);

/* Frees the library scratch block of `stream` on the current device (after
 * the stream's queued work).  The next call on that stream allocates again. */
nk_status nk_scratch_release(void *stream);

/* Allocation-free variant of nk_gemm_w8row for f32 activations.  It has no
 * counterpart in the reference.  For callers that cannot let a library call
 * cudaMalloc (a host whose device memory belongs to its own pool, or a
 * latency-critical path where an allocation would synchronise the device):
 * the bf16 hi | lo split of x lives in a fixed 8 MiB device array inside
 * libnk, held by every GPU that loads the library until exit, instead of the
 * library's growable scratch.  m * 4 * ceil(k/64)*64 bytes must fit in 8 MiB
 * (NK_WORKSPACE_TOO_SMALL otherwise); k % 16 == 0.  All calls on a device
 * share the array, so calls that overlap on the GPU race; each call rewrites
 * all of it that it reads.  The first call on a device resolves the array's
 * device address and should come before any stream capture.  Same output
 * contract as nk_gemm_w8row(x_dtype = NK_F32). */
nk_status nk_gemm_w8row_f32_static(const float *x, const int8_t *wq, const float *scales,
                                   const float *bias, void *y, int32_t y_dtype, int64_t m,
                                   int64_t k, int64_t n, int32_t flags, void *stream);

/* -------------------------------------------------------------- quantize */

/* quantize.rs:59-81 pack_int4_into_host.  Synchronises `stream` (the range
 * check is a device reduction): NK_INT4_OUT_OF_RANGE reports the first value
 * above 15, as the host loop does.  packed_len must be ceil(count/2). */
nk_status nk_pack_int4(const uint8_t *values, size_t count, uint8_t *packed, size_t packed_len,
                       void *stream);
/* quantize.rs:89-120 unpack_int4_into_host. */
nk_status nk_unpack_int4(const uint8_t *packed, size_t packed_len, size_t count, uint8_t *out,
                         size_t out_len, void *stream);
/* quantize.rs:131-144 quantize_int4_into_host: code = clamp(round_half_away(v/scale + zp), 0, 15).
 * Synchronises `stream`: the first non-finite input is reported as
 * NK_NON_FINITE_INPUT{index, value} and nothing is written, as the host
 * loop returns before packing. */
nk_status nk_quantize_int4(const float *values, size_t count, float scale, uint32_t zero_point,
                           uint8_t *packed, size_t packed_len, void *stream);
/* quantize.rs:156-178 dequantize_int4_into_host (and the async dequantize_int4,
 * quantize.rs:333-349): out = (code - zp) * scale, f32. */
nk_status nk_dequantize_int4(const uint8_t *packed, size_t packed_len, size_t count, float scale,
                             uint32_t zero_point, float *out, size_t out_len, void *stream);
/* quantize.rs:180-186 validate_int4_params (host only, no device work). */
nk_status nk_validate_int4_params(float scale, uint32_t zero_point);
/* Int8 per-output-row symmetric absmax quantization of W [N,K] f32:
 * scales[n] = max|W[n,:]| / 127, wq = clamp(round_half_away(W/scale), -127, 127),
 * an all-zero row gives scale 0 and codes 0.  Synchronises `stream`; a
 * non-finite weight is reported as NK_NON_FINITE_INPUT.  Not in the
 * reference (the benchmark configurations name this format). */
nk_status nk_quantize_int8_row(const float *w, int64_t n, int64_t k, int8_t *wq, float *scales,
                               void *stream);

/* ---------------------------------------------------------------- routing */

enum {
  NK_ROUTE_SIGMOID = 0,        /* select_top_k, moe_routing.rs:168-186 (the reference router) */
  NK_ROUTE_SOFTMAX = 1,        /* select_top_k_softmax, moe_routing.rs:188-216 */
  NK_ROUTE_SIGMOID_RENORM = 2  /* sigmoid top-k, selected weights renormalised to sum 1
                                  (the benchmark configuration; not in the reference) */
};

/* Replaces moe_route / moe_route_softmax (moe_routing.rs:499-532) and the
 * host loops moe_route_into_host / moe_route_softmax_into_host
 * (moe_routing.rs:118-166).  scores f32 [tokens, experts] row-major;
 * indices int32 [tokens, top_k] (the reference's usize), weights f32.
 * Ranking uses f32 total order, weight descending then expert index
 * ascending, on sigmoid values computed as the reference computes them
 * (the exponential is evaluated in double and rounded once to f32).
 * Validation: experts == 0, top_k == 0 or top_k > experts -> NK_INVALID_SHAPE,
 * then scores, indices, weights lengths.  tokens == 0 is valid and a no-op.
 * The device kernel handles experts <= 1024 and top_k <= 32 (NK_UNSUPPORTED
 * beyond). */
nk_status nk_moe_route(const float *scores, size_t scores_len, size_t tokens, size_t experts,
                       size_t top_k, int32_t mode, int32_t *indices, size_t indices_len,
                       float *weights, size_t weights_len, void *stream);

/* Expert histogram and permutation derived from routing indices (the
 * reference has none: it runs every selected expert over all rows,
 * moe.rs:226-233).  counts[e] = #{(t,r): indices[t*top_k+r] == e};
 * offsets = exclusive prefix sum of counts (experts+1 entries, the last is
 * tokens*top_k); perm[offsets[e] + j] = the j-th route slot t*top_k+r (in
 * ascending slot order) that selected e; slot_pos[t*top_k+r] = its position
 * in perm.  Deterministic.  Requires experts <= 1024. */
nk_status nk_moe_plan(const int32_t *indices, int64_t tokens, int64_t top_k, int64_t experts,
                      int32_t *counts, int32_t *offsets, int32_t *perm, int32_t *slot_pos,
                      void *stream);

/* -------------------------------------------------------------- MoE layer */

enum { NK_W_BF16 = 0, NK_W_INT8_ROW = 1, NK_W_INT4_AFFINE = 2 };

/* Weights of one MoE layer, all device pointers, in the layouts the B200
 * kernels read (each GEMM weight is [out_features, in_features], K contiguous;
 * nk_linear_pack_kn converts the reference's [in, out] layout).
 * Expert tensors are stacked over experts. */
typedef struct nk_moe_layer {
  int64_t hidden;        /* H */
  int64_t experts;       /* E */
  int64_t top_k;         /* k */
  int64_t inter;         /* I, routed expert width */
  int64_t shared_inter;  /* Is, 0 = no shared expert */
  int32_t route_mode;    /* NK_ROUTE_* */
  int32_t weight_kind;   /* NK_W_BF16, NK_W_INT8_ROW or NK_W_INT4_AFFINE (experts and
                            shared expert) */
  const uint16_t *router_w3; /* [E, 3*Hp] bf16, Hp = ceil(H/64)*64: the f32 router weight
                                [E,H] split exactly into three zero-padded bf16 parts
                                (nk_router_split); scores carry f32 accuracy */
  const float *router_b;     /* [E] or NULL */
  const void *up_w;          /* [E, I, H]; INT4_AFFINE: codes [E, I, H/2] (nk_int4_kn_to_nk) */
  const float *up_scale;     /* [E, I] (INT8_ROW); [E] per-expert scale (INT4_AFFINE) */
  const float *up_b;         /* [E, I] or NULL */
  const void *down_w;        /* [E, H, I]; INT4_AFFINE: codes [E, H, I/2] */
  const float *down_scale;   /* [E, H] (INT8_ROW); [E] (INT4_AFFINE) */
  const float *down_b;       /* [E, H] or NULL */
  const void *shared_up_w;   /* [Is, H] */
  const float *shared_up_scale;
  const float *shared_up_b;
  const void *shared_down_w; /* [H, Is] */
  const float *shared_down_scale;
  const float *shared_down_b;
  /* INT4_AFFINE zero points (quantize.rs:180-186 params, one per expert):
   * W = (code - zero_point) * scale, dequantized inside the GEMMs. */
  const uint8_t *up_zero_point;          /* [E] */
  const uint8_t *down_zero_point;        /* [E] */
  const uint8_t *shared_up_zero_point;   /* [1] */
  const uint8_t *shared_down_zero_point; /* [1] */
  /* [2E]: |W_e|_2 and |lo_e|_2 of the router weight (nk_router_norms), which
   * bound the tensor-core router's error; NULL: computed on every call. */
  const float *router_norms;
} nk_moe_layer;

/* The router weight's per-expert norms for nk_moe_layer.router_norms: once
 * per layer, after nk_router_split (norms: [2E] f32). */
nk_status nk_router_norms(const uint16_t *router_w3, int64_t experts, int64_t hidden,
                          float *norms, void *stream);

/* Splits a router weight f32 [E,H] into the [E, 3*Hp] bf16 triple used by
 * nk_moe_forward (hi | mid | lo, each zero padded to Hp = ceil(H/64)*64;
 * hi + mid + lo == the f32 value for every normal f32). */
nk_status nk_router_split(const float *router_w, int64_t experts, int64_t hidden,
                          uint16_t *router_w3, void *stream);

/* Converts a reference-layout linear weight f32 [K,N] (input_dim x output_dim,
 * linear.rs:324) into the [N,K] bf16 layout the GEMMs read. */
nk_status nk_linear_pack_kn(const float *w_kn, int64_t k, int64_t n, uint16_t *w_nk,
                            void *stream);

/* Repacks INT4 codes from the reference's [K,N] nibble layout (quantize.rs:
 * flat index k*N + n in byte index/2, low nibble for even index; each of the
 * `batch` matrices ceil(K*N/2) bytes, back to back) into the feature-major
 * layout NK_W_INT4_AFFINE expert weights use: [N, K/2] bytes, byte n*K/2 + k/2,
 * low nibble for even k (batch * N * K/2 bytes).  k even. */
nk_status nk_int4_kn_to_nk(const uint8_t *packed_kn, int64_t batch, int64_t k, int64_t n,
                           uint8_t *packed_nk, void *stream);

/* Device workspace (bytes) nk_moe_forward needs for `tokens` rows. */
nk_status nk_moe_workspace_bytes(const nk_moe_layer *layer, int64_t tokens, size_t *bytes);

/* Replaces MoeLayer::forward_into (nemotron-nn/src/moe.rs:154-249):
 * router projection -> top-k routing -> per-expert MLP relu2(x·upᵀ)·downᵀ on
 * the tokens routed to it (grouped GEMMs) -> out[t] = shared(x)[t] +
 * Σ_r w[t,r]·expert_{idx[t,r]}(x)[t], summed in rank order in f32 like
 * moe.rs:207-246.  x bf16 [tokens, H]; out [tokens, H] in out_dtype.
 * indices/weights (int32/f32 [tokens, top_k]) receive the routing when not
 * NULL.  workspace: device memory of nk_moe_workspace_bytes. */
nk_status nk_moe_forward(const nk_moe_layer *layer, const uint16_t *x, int64_t tokens,
                         void *out, int32_t out_dtype, int32_t *indices, float *weights,
                         void *workspace, size_t workspace_bytes, void *stream);

/* ------------------------------------------------ host-buffer MoE executor
 * MoeLayer::forward_into (moe.rs:154-249) for callers whose activations live
 * in HOST memory (the reference's *_into_host convention): each submission
 * copies x_host (bf16 [tokens, H]) to the device, runs nk_moe_forward and
 * copies out (out_dtype [tokens, H]) and, when indices_host is not NULL, the
 * routing indices (int32 [tokens, top_k]) back.  Two device slots and three
 * streams (host->device, compute, device->host) let the copies of adjacent
 * submissions overlap the forward in between; forwards run in submission
 * order.  Host buffers must stay valid, and out_host / indices_host unread,
 * until nk_moe_pipeline_wait returns; page-locked host memory (cudaHostAlloc
 * / cudaHostRegister) is needed for the copies to overlap.  Streams: all
 * three given (cudaStream_t) or all NULL (the executor creates its own).
 * `layer`'s device weights must outlive the executor. */
typedef struct nk_moe_pipeline nk_moe_pipeline;
nk_status nk_moe_pipeline_create(const nk_moe_layer *layer, int64_t max_tokens,
                                 int32_t out_dtype, void *h2d_stream, void *compute_stream,
                                 void *d2h_stream, nk_moe_pipeline **out);
nk_status nk_moe_pipeline_submit(nk_moe_pipeline *p, const uint16_t *x_host, int64_t tokens,
                                 void *out_host, int32_t *indices_host);
/* Blocks until every submission has completed; then reports a device-side
 * error like nk_device_status. */
nk_status nk_moe_pipeline_wait(nk_moe_pipeline *p);
nk_status nk_moe_pipeline_destroy(nk_moe_pipeline *p);

/* ------------------------------------------ MoE stages (expert parallelism)
 * nk_moe_forward in three separable stages, so that the routed rows can be
 * exchanged between ranks that own disjoint, contiguous ranges of experts
 * (rank g owns experts [g*E/G, (g+1)*E/G)).  The reference has no
 * distribution (one device, nemotron-kernels/src/device.rs:32-54); these
 * split MoeLayer::forward_into (moe.rs:154-249) at its natural seams. */

/* Stage 1 on the rank that owns the tokens: router GEMM, top-k routing
 * (moe_routing.rs:168-216), expert plan and the gather of routed rows.
 * indices/weights [tokens, top_k]; counts [E]; offsets [E+1] (exclusive
 * prefix of counts); slot_pos [tokens*top_k]; routed_rows [tokens*top_k, H]
 * bf16, ordered by expert, so the rows for each expert range are contiguous
 * (routed_rows NULL: no gather, for nk_ep_dispatch).
 * workspace: nk_moe_dispatch_workspace_bytes. */
nk_status nk_moe_dispatch_workspace_bytes(const nk_moe_layer *layer, int64_t tokens,
                                          size_t *bytes);
nk_status nk_moe_dispatch(const nk_moe_layer *layer, const uint16_t *x, int64_t tokens,
                          int32_t *indices, float *weights, int32_t *counts, int32_t *offsets,
                          int32_t *slot_pos, uint16_t *routed_rows, void *workspace,
                          size_t workspace_bytes, void *stream);

/* Stage 2 on the rank that owns the experts: the per-expert MLP
 * relu2(row·upᵀ + b)·downᵀ + b (mlp.rs:157-211) over rows [n_rows, H] bf16
 * laid out as n_segments back-to-back segments; segment s has seg_rows[s]
 * rows for the layer's expert seg_expert[s] (device int32 arrays; seg_expert
 * NULL = segment s is expert s).  `layer` describes the LOCAL experts only
 * (experts = experts held here; router and shared expert unused).  out
 * [n_rows, H] bf16 may alias rows.  n_segments <= 1024. */
nk_status nk_moe_experts_workspace_bytes(const nk_moe_layer *layer, int64_t n_rows,
                                         int32_t n_segments, size_t *bytes);
nk_status nk_moe_experts(const nk_moe_layer *layer, const uint16_t *rows, int64_t n_rows,
                         const int32_t *seg_expert, const int32_t *seg_rows, int32_t n_segments,
                         uint16_t *out, void *workspace, size_t workspace_bytes, void *stream);

/* The shared expert on the token rank: out [tokens, H] bf16 =
 * relu2(x·shared_upᵀ + b)·shared_downᵀ + b; scratch [tokens, Is] bf16. */
nk_status nk_moe_shared(const nk_moe_layer *layer, const uint16_t *x, int64_t tokens,
                        uint16_t *scratch, uint16_t *out, void *stream);

/* Stage 3 on the token rank: out[t] = shared[t] + Σ_r weights[t,r] ·
 * expert_rows[slot_pos[t*top_k + r]], in rank order in f32 (moe.rs:195-246);
 * shared may be NULL.  expert_rows are in the order routed_rows had. */
nk_status nk_moe_combine(const uint16_t *expert_rows, const uint16_t *shared, const float *weights,
                         const int32_t *slot_pos, int64_t tokens, int64_t hidden, int64_t top_k,
                         void *out, int32_t out_dtype, void *stream);

/* ------------------------------------- expert-parallel exchange over NVLink
 * Rows move between ranks by direct stores into peer memory shared with CUDA
 * IPC handles; no host synchronisation.  Rank g owns experts
 * [g*El, (g+1)*El), El = experts/ranks.  counts_all is the [ranks, experts]
 * matrix of every rank's nk_moe_dispatch counts (an all-gather). */

/* Device buffer for peer access: cudaMalloc + its 64-byte IPC handle. */
nk_status nk_ipc_alloc(size_t bytes, void **ptr, uint8_t *handle64);
/* Maps a peer's buffer from its handle (peer access enabled lazily). */
nk_status nk_ipc_open(const uint8_t *handle64, void **ptr);
nk_status nk_ipc_close(void *ptr);
nk_status nk_ipc_free(void *ptr);

/* Exchange plan for rank `rank` (device int32 outputs):
 *   send_base[experts]: first receive row of this rank's block for each expert
 *     in the owner's receive buffer (layout [source rank][local expert][row]);
 *   seg_rows/seg_start[ranks*El]: the segments of this rank's receive buffer
 *     (for nk_moe_experts with seg_expert = j repeated per source);
 *   return_offset[ranks*El]: where each segment goes back, as a row of the
 *     source rank's expert-ordered result buffer;
 *   received_rows[1]. */
nk_status nk_ep_plan(const int32_t *counts_all, int32_t ranks, int32_t experts, int32_t rank,
                     int32_t *send_base, int32_t *seg_rows, int32_t *seg_start,
                     int32_t *return_offset, int32_t *received_rows, void *stream);
/* The same plan with the local experts split into `phases` equal groups that
 * are received and computed one after the other (the exchange of one phase
 * overlaps the experts of another).  Phase h's rows start at receive row
 * h * phase_capacity_rows, ordered [source rank][local expert of the phase];
 * segment index (h * ranks + s) * (El / phases) + (j % (El / phases)) for
 * source s and local expert j.  seg_start and send_base are absolute rows.
 * phases = 1 is nk_ep_plan. */
nk_status nk_ep_plan_phased(const int32_t *counts_all, int32_t ranks, int32_t experts,
                            int32_t rank, int32_t phases, int64_t phase_capacity_rows,
                            int32_t *send_base, int32_t *seg_rows, int32_t *seg_start,
                            int32_t *return_offset, int32_t *received_rows, void *stream);

/* Gathers x[token] for every route slot and stores it into the owning rank's
 * receive buffer (peer_recv: device array of `ranks` peer base pointers,
 * this rank's own buffer included).  indices/slot_pos/offsets from
 * nk_moe_dispatch; send_base from nk_ep_plan. */
nk_status nk_ep_dispatch(const uint16_t *x, int64_t tokens, int64_t hidden, int32_t top_k,
                         const int32_t *indices, const int32_t *slot_pos, const int32_t *offsets,
                         const int32_t *send_base, int32_t experts_per_rank,
                         const uint64_t *peer_recv, void *stream);

/* Stores each received segment's expert outputs into its source rank's
 * result buffer (peer_out: device array of `ranks` peer base pointers) at
 * return_offset, i.e. at the slot order nk_moe_combine reads. */
nk_status nk_ep_return(const uint16_t *expert_rows, int64_t hidden, int32_t ranks,
                       int32_t experts_per_rank, const int32_t *seg_rows,
                       const int32_t *seg_start, const int32_t *return_offset,
                       const uint64_t *peer_out, void *stream);
/* Phase `phase` of nk_ep_dispatch under nk_ep_plan_phased: only the slots
 * routed to that phase's local experts move. */
nk_status nk_ep_dispatch_phase(const uint16_t *x, int64_t tokens, int64_t hidden, int32_t top_k,
                               const int32_t *indices, const int32_t *slot_pos,
                               const int32_t *offsets, const int32_t *send_base,
                               int32_t experts_per_rank, int32_t phases, int32_t phase,
                               const uint64_t *peer_recv, void *stream);
/* nk_ep_return for segments first_segment .. first_segment+n_segments-1 of a
 * phased plan (experts_per_phase = El / phases). */
nk_status nk_ep_return_segments(const uint16_t *expert_rows, int64_t hidden, int32_t ranks,
                                int32_t experts_per_phase, int32_t first_segment,
                                int32_t n_segments, const int32_t *seg_rows,
                                const int32_t *seg_start, const int32_t *return_offset,
                                const uint64_t *peer_out, void *stream);

/* ------------------------------------------- native expert parallelism
 * MoeLayer::forward_into (moe.rs:154-249) over G ranks, one process per GPU,
 * the experts split evenly (rank g holds experts [g*E/G, (g+1)*E/G)); the
 * layout the benchmark configurations ask for, not in the reference (which
 * runs on one device, device.rs:32-54).  Every call below is issued by every
 * rank, in the same order, on one stream per rank.
 *
 *   1. nk_ep_create on every rank: allocates this rank's exchange memory
 *      (receive rows, result rows, the counts matrix, barrier flags) and
 *      writes a handle blob of nk_ep_handle_bytes() bytes.
 *   2. The caller gathers the blobs of all ranks, in rank order, with its own
 *      collective (NCCL / MPI all-gather, a key-value store) and hands them to
 *      nk_ep_connect, which maps the peers' memory (CUDA IPC).
 *   3. nk_moe_forward_ep per layer call: routing on this rank -> per-expert
 *      counts written into every rank's counts matrix -> device barrier ->
 *      exchange plan -> routed rows stored straight into their expert owners'
 *      receive buffers over NVLink -> barrier -> this rank's grouped experts
 *      -> results stored straight back -> barrier -> shared expert (on a side
 *      stream meanwhile) + combine in rank order.  No host synchronisation,
 *      no library collective; the barriers are flag words in peer memory,
 *      each wait bounded (NK_TIMEOUT in nk_device_status when a peer does not
 *      arrive within 2 s).  Plain peer loads and stores only (no multicast).
 *      The down projection's epilogue stores the results straight into the
 *      source ranks' buffers (no separate return kernel).  With the
 *      environment variable NK_EP_PULL=1 and bf16 experts, the routed rows
 *      are instead pulled by the owners' up projection from the sources' send
 *      buffers (no dispatch kernel, no barrier before the experts).
 *   4. nk_ep_destroy after every rank has finished its last forward (for
 *      example after nk_ep_barrier and a stream synchronisation).
 *
 * capacity_rows: receive rows per rank (0: the worst case ranks * max_tokens
 * * top_k); a forward that routes more rows to one rank reports
 * NK_WORKSPACE_TOO_SMALL through nk_device_status and drops the excess. */
typedef struct nk_ep_ctx nk_ep_ctx;
size_t nk_ep_handle_bytes(void);
nk_status nk_ep_create(int32_t ranks, int32_t rank, int64_t experts, int64_t hidden,
                       int64_t top_k, int64_t max_tokens, int64_t capacity_rows,
                       nk_ep_ctx **out, void *handle_blob);
nk_status nk_ep_connect(nk_ep_ctx *ctx, const void *all_blobs);
/* layer: the whole layer (router over all E experts, shared expert); local:
 * this rank's E/G experts stacked in local order (same kind and widths; int8
 * / INT4 scales and zero points sliced to the local experts). */
nk_status nk_moe_forward_ep_workspace_bytes(const nk_ep_ctx *ctx, const nk_moe_layer *layer,
                                            const nk_moe_layer *local, int64_t tokens,
                                            size_t *bytes);
nk_status nk_moe_forward_ep(nk_ep_ctx *ctx, const nk_moe_layer *layer, const nk_moe_layer *local,
                            const uint16_t *x, int64_t tokens, void *out, int32_t out_dtype,
                            int32_t *indices, float *weights, void *workspace,
                            size_t workspace_bytes, void *stream);
/* A device barrier across the ranks on `stream` (bounded like the others). */
nk_status nk_ep_barrier(nk_ep_ctx *ctx, void *stream);
/* Rows this rank received in the last forward (device int32, copied on the
 * legacy stream). */
nk_status nk_ep_received_rows(const nk_ep_ctx *ctx, int32_t *rows_device);
nk_status nk_ep_destroy(nk_ep_ctx *ctx);

/* ---------------------------------------------------------------- tracing */

/* Stage timing of nk_moe_forward (not in the reference, whose only timing is
 * wall-clock around whole calls, nemotron-validate/src/benchmark.rs:465-500).
 * While enabled on the calling thread, nk_moe_forward records CUDA events on
 * its stream between stages; nk_moe_stage_times waits for the last call's
 * final event and returns the milliseconds of each stage:
 *   0 router GEMM, 1 routing + plan + tile lists, 2 token gather,
 *   3 grouped up-projection, 4 grouped down-projection, 5 shared expert,
 *   6 combine.
 * A forward captured into a CUDA graph while timing is enabled records its
 * events as graph nodes; after each replay nk_moe_stage_times reads them. */
nk_status nk_set_stage_timing(int32_t enable);
nk_status nk_moe_stage_times(float *ms, int32_t capacity, int32_t *count);

#if defined(__GNUC__)
/* ===================================================== Mamba2 glue ====
 * The stages of Mamba2Mixer::forward (nemotron-nn/src/mamba2.rs:264-375)
 * between the input projections and out_proj: causal depthwise conv (with
 * the conv cache as history), SiLU, selective scan, gated RMSNorm.  All f32,
 * as in the reference.  Pointers are device pointers. */

/* Replaces depthwise_causal_conv1d_into_host / depthwise_causal_conv1d
 * (nemotron-kernels/src/conv1d.rs:78-124, 325-345).  input [seq, channels],
 * weights [channels, kernel_size] (tap j reads step t-j with weight
 * kernel_size-1-j), f64 accumulation.  Errors: InvalidShape (channels or
 * kernel_size 0), LengthMismatch input / weights / output; seq 0 is valid. */
nk_status nk_conv1d(const float *input, size_t input_len, const float *weights,
                    size_t weights_len, int64_t seq, int64_t channels, int64_t kernel_size,
                    float *out, size_t out_len, void *stream);

/* Batched conv as Mamba2Mixer::forward runs it (mamba2.rs:276-312): per batch,
 * history = the K-1 cached steps (prefix, [batch, K-1, channels]) or zeros;
 * y = conv(history ++ x) without the history rows, optionally SiLU'd
 * (activations.rs:95-97); state_out (NULL or [batch, K-1, channels], may be
 * the prefix itself) receives the last K-1 steps of history ++ x. */
typedef struct nk_conv_args {
  int64_t batch, seq, channels, kernel_size;
  const float *x; int64_t ld_x;   /* x[(b*seq + t)*ld_x + ch] */
  const float *weights;           /* [channels, kernel_size] */
  const float *prefix;            /* NULL: zero history */
  int32_t silu;
  float *y; int64_t ld_y;         /* y[(b*seq + t)*ld_y + ch] */
  float *state_out;               /* NULL: not written */
  int32_t f32_accumulate;         /* 0: f64 as the reference (bit-exact); 1: f32 FMA chain */
} nk_conv_args;
nk_status nk_conv1d_ex(const nk_conv_args *args, void *stream);

/* Replaces selective_scan_into_host / selective_scan (nemotron-kernels/src/
 * ssm.rs:123-175, 614-624): reference layouts input/delta_t [seq, C],
 * a [C, S], b/c [seq, C, S], d [C] or NULL, initial_state [C, S] or NULL;
 * writes out [seq, C] and final_state [C, S].  Validation order and errors
 * as ssm.rs:177-288 (InvalidShape, LengthMismatch, InvalidDeltaT for the
 * first (t, ch) in t-major order whose dt is non-finite or negative).  The
 * dt check reads back one word, so this call synchronises `stream`. */
nk_status nk_selective_scan(const float *input, size_t input_len, const float *delta_t,
                            size_t delta_t_len, const float *a, size_t a_len, const float *b,
                            size_t b_len, const float *c, size_t c_len, const float *d,
                            size_t d_len, const float *initial_state, size_t initial_state_len,
                            float delta_bias, int32_t apply_softplus, int64_t seq,
                            int64_t channels, int64_t states, float *out, size_t out_len,
                            float *final_state, size_t final_state_len, void *stream);

/* Strided / shared-parameter form of the same recurrence.  Channel ch of a
 * group shares a parameter row: with every *_group = 1, a_per_state = 1 and
 * ld_bc = C*S this is exactly the reference layout; the Mamba2 layout (one
 * dt, A and D per head, B/C per group, all read in place from the fused
 * in_proj output) sets dt_group = a_group = d_group = head_dim,
 * a_per_state = 0, bc_group = C / ngroups. */
typedef struct nk_scan_args {
  int64_t batch, seq, channels, states;
  const float *x; int64_t ld_x;                       /* x[(b*seq + t)*ld_x + ch] */
  const float *dt; int64_t ld_dt; int32_t dt_group;   /* dt[(b*seq + t)*ld_dt + ch/dt_group] */
  const float *a; int32_t a_group; int32_t a_per_state;
      /* a[(ch/a_group)*states + s] if a_per_state, else a[ch/a_group] */
  const float *b; const float *c; int64_t ld_bc; int32_t bc_group;
      /* b[(b*seq + t)*ld_bc + (ch/bc_group)*states + s] */
  const float *d; int32_t d_group;                    /* NULL or d[ch/d_group] */
  const float *initial_state;                         /* NULL or [batch, C, S] */
  float delta_bias; int32_t softplus;
  float *y; int64_t ld_y;                             /* y[(b*seq + t)*ld_y + ch] */
  float *final_state;                                 /* NULL or [batch, C, S]; may alias initial_state */
  int32_t check_delta_t;  /* 1: synchronise and report InvalidDeltaT; 0: no readback (graph capture) */
} nk_scan_args;
nk_status nk_selective_scan_ex(const nk_scan_args *args, void *stream);

/* Replaces rms_norm_into_host (gate NULL) / gated_rms_norm_into_host
 * (nemotron-kernels/src/rms_norm.rs:64-106): one vector of `len`.
 * Errors: EmptyInput, LengthMismatch weight / gate / output, NegativeEpsilon. */
nk_status nk_rms_norm(const float *input, size_t len, const float *weight, size_t weight_len,
                      const float *gate, size_t gate_len, float epsilon, float *out,
                      size_t out_len, void *stream);

/* Row-wise contract of rms_norm / gated_rms_norm (rms_norm.rs:291-360) and
 * gated_rms_norm_rows (mamba2.rs:567-586): each of `rows` rows of `width`
 * normalised alone.  out_dtype NK_DTYPE_F32 or NK_DTYPE_BF16 (round to
 * nearest even, to feed out_proj directly).  gate may be NULL. */
enum { NK_DTYPE_F32 = 0, NK_DTYPE_BF16 = 1 };
nk_status nk_rms_norm_rows(const float *x, int64_t rows, int64_t width, int64_t ld_x,
                           const float *weight, size_t weight_len, const float *gate,
                           int64_t ld_gate, float epsilon, void *out, int64_t ld_out,
                           int32_t out_dtype, void *stream);

/* The same norm with each row split over tensor-parallel ranks (a rank holds
 * `width` of the row's `total_width` columns): nk_row_sumsq writes each local
 * row's f64 sum of squares, the caller sums them over the ranks (one
 * all-reduce of `rows` doubles), and nk_rms_norm_rows_presummed normalises
 * the local columns with the full-row mean square sumsq[row] / total_width. */
nk_status nk_row_sumsq(const float *x, int64_t rows, int64_t width, int64_t ld_x, double *sumsq,
                       void *stream);
nk_status nk_rms_norm_rows_presummed(const float *x, int64_t rows, int64_t width, int64_t ld_x,
                                     const float *weight, size_t weight_len, const float *gate,
                                     int64_t ld_gate, const double *sumsq, int64_t total_width,
                                     float epsilon, void *out, int64_t ld_out,
                                     int32_t out_dtype, void *stream);

/* ===================================================== attention core ====
 * nemotron-kernels/src/attention.rs; layouts [batch, seq, heads, head_dim]. */

/* Replaces scaled_dot_product_attention_into_host / scaled_dot_product_attention
 * (attention.rs:204-302, 849-884) on f32 device tensors: f64 dot products,
 * f32 scale (default 1/sqrt(head_dim) when has_scale = 0), f32 exp with an
 * f64 partition, f64 output sums.  causal masks keys beyond
 * min(q_offset + q, kv_seq - 1).  Validation order and errors as
 * attention.rs:304-357 then the output length then the scale; the row
 * errors (NoValidAttentionTargets, ZeroPartition) report the first row in
 * (batch, query, head) order.  Synchronises `stream`. */
nk_status nk_attention_f32(const float *query, size_t query_len, const float *key,
                           size_t key_len, const float *value, size_t value_len, int64_t batch,
                           int64_t q_seq, int64_t kv_seq, int64_t q_heads, int64_t kv_heads,
                           int64_t head_dim, int32_t causal, int64_t q_offset,
                           int32_t has_scale, float scale, float *out, size_t out_len,
                           void *stream);

/* KV cache (the serving path's replacement for KvCache::append, cache.rs:74-110):
 * k_cache bf16 [batch, kv_heads, max_len, head_dim], vt_cache bf16
 * [batch, kv_heads, head_dim, max_len] (V stored transposed).  Writes steps
 * pos0 .. pos0+seq-1 from the K/V projection outputs k_new / v_new
 * [batch*seq, kv_heads*head_dim] bf16.  Allocate the caches zeroed: the
 * value GEMM reads up to 63 positions past kv_len (multiplied by 0). */
nk_status nk_kv_append(const uint16_t *k_new, const uint16_t *v_new, int64_t batch, int64_t seq,
                       int64_t kv_heads, int64_t head_dim, int64_t pos0, int64_t max_len,
                       uint16_t *k_cache, uint16_t *vt_cache, void *stream);

/* Grouped-query attention of q bf16 [batch*q_seq, q_heads*head_dim] over the
 * first kv_len cache positions: scores and value sums on the tcgen05 GEMM
 * (bf16 operands, f32 accumulation), softmax as the reference (f32 exp, f64
 * partition).  out [batch*q_seq, q_heads*head_dim], f32 or bf16 (out_dtype).
 * head_dim 64 or 128, max_len a multiple of 64.  A row without a finite
 * score is flagged in the workspace (nk_attention_check), not raised, so
 * the call does not synchronise. */
nk_status nk_attention_workspace_bytes(int64_t batch, int64_t q_seq, int64_t kv_len,
                                       int64_t max_len, int64_t q_heads, int64_t kv_heads,
                                       int64_t head_dim, size_t *bytes);
nk_status nk_attention_gqa(const uint16_t *q, const uint16_t *k_cache, const uint16_t *vt_cache,
                           int64_t batch, int64_t q_seq, int64_t kv_len, int64_t max_len,
                           int64_t q_heads, int64_t kv_heads, int64_t head_dim, int32_t causal,
                           int64_t q_offset, int32_t has_scale, float scale, void *out,
                           int32_t out_dtype, void *workspace, size_t workspace_bytes,
                           void *stream);
nk_status nk_attention_check(const void *workspace, int64_t *first_bad_row, void *stream);

/* ============================================ decoder steps around projections ====
 * Embedding gather, block residual + RMSNorm, greedy pick. */

/* Replaces embedding_lookup_into_host / embedding_lookup (nemotron-kernels/src/
 * embedding.rs:73-91, 121-191): out[t] = table[token_ids[t]].  table
 * [vocab_size, hidden_size] and out f32 or bf16 (NK_DTYPE_*).  Validation
 * order: InvalidShape, LengthMismatch table / output, then TokenOutOfRange
 * for the first bad id when check = 1 (which synchronises `stream`; with
 * check = 0 bad ids leave their rows unwritten). */
nk_status nk_embedding_lookup(const void *table, int32_t table_dtype, size_t table_len,
                              const int32_t *token_ids, int64_t n_tokens, int64_t vocab_size,
                              int64_t hidden_size, void *out, int32_t out_dtype, size_t out_len,
                              int32_t check, void *stream);

/* The residual of NemotronBlock::forward_into (nemotron-nn/src/block.rs:145-151)
 * fused with the next RMSNorm (rms_norm.rs:117-123, the next block's input
 * norm or the final norm, model.rs:296-301): per row of width,
 * h_out = residual + delta (f32; delta NULL: h_out = residual; h_out may be
 * residual) and normed = h_out * (1/sqrt(mean(h_out²) + epsilon)) * weight,
 * f32 or bf16 (normed_dtype). */
nk_status nk_add_rms_norm_rows(const float *residual, const float *delta, int64_t rows,
                               int64_t width, const float *weight, size_t weight_len,
                               float epsilon, float *h_out, void *normed, int32_t normed_dtype,
                               void *stream);

/* Greedy pick of predict_next_token (nemotron-model/src/model.rs:325-337) per
 * row of x [rows, n] (row pitch ld, f32 or bf16): the index of the maximum
 * under f32::total_cmp, the last one among equal maxima (Iterator::max_by). */
nk_status nk_argmax_rows(const void *x, int32_t x_dtype, int64_t rows, int64_t n, int64_t ld,
                         int32_t *out, void *stream);

#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* NK_H */
