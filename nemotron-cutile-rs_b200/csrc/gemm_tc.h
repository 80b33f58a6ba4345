// gemm_tc.h — host interface of the tcgen05 projection GEMM.
#pragma once
#include "gemm_tc.cuh"

namespace nk {

// Launches tc_gemm_kernel.  Weight operand (A): wk = WK_BF16 / WK_INT8 with
// w_rows feature rows of w_k elements, row pitch ldw_bytes; or WK_INT4KN with
// the reference [K,N] nibble layout (w_rows = N features, w_k = K rows,
// ldw_bytes = N/2).  Activations (B): bf16 [x_rows, x_k], pitch ldx_elems.
// bn: 256, 64 or 16 token rows per tile.  grid: CTAs (persistent over tiles).
// pair = 2: clusters of two CTAs share 256-feature tiles (tcgen05 cta_group::2);
// needs bn = 256, an even grid, and tiles of 256 features (f_tiles / tile lists
// built with 256-row feature tiles).
// fa = 2: single CTAs with two accumulators: 256-feature tiles (lists built
// with 256-row feature tiles), bn = 256.
nk_status tc_gemm(int wk, const void *w, int64_t w_rows, int64_t w_k, int64_t ldw_bytes,
                  const uint16_t *x, int64_t x_rows, int64_t x_k, int64_t ldx_elems, int bn,
                  TcArgs args, int grid, cudaStream_t stream, int pair = 1, int fa = 1);

// f32 activations [m, k] -> bf16 hi | lo halves [m, 2*kp] (kp = ceil(k/64)*64,
// zero padded; every element written), the operand of the f32-activation
// projections: hi + lo carries the top 16 significand bits of each value.
nk_status launch_split_f32(const float *x, int64_t m, int64_t k, int64_t kp, uint16_t *x2,
                           cudaStream_t stream);

}  // namespace nk
