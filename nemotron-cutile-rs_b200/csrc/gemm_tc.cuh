// gemm_tc.cuh — the sm_100a projection GEMM shared by every libnk entry point.
//
//   D[f, t] = Σ_k W[f, k] · X[t, k]          (tcgen05.mma, f32 accumulators in TMEM)
//   Y[t, out_col0 + f] = epilogue(D[f, t])   (stored transposed: Y is [tokens, features])
//
// The weight operand is always the MMA "A" side (128 feature rows per tile)
// and the activations the "B" side (up to BN token rows per tile), so one
// kernel serves decode (a handful of tokens: N of the MMA shrinks to 16) and
// prefill, dense and grouped (MoE) alike.  Weights come as bf16 [N,K], int8
// [N,K] (per-row scale) or the reference's INT4-affine [K,N] nibble layout;
// the quantized kinds are dequantized inside the kernel by "transform"
// warps that turn the raw TMA tile into the bf16 128-byte-swizzled tile the
// tensor core reads.
//
// Warp roles (one CTA per SM, persistent over a tile list):
//   warp 0      TMA producer (one lane)
//   warp 1      TMEM allocator + MMA issuer (one lane)
//   warps 2-5   epilogue: TMEM -> registers -> scale/bias/relu2/token weight -> global
//   warps 6-13  transform (quantized weights only)
// Every mbarrier wait is bounded (mbar_wait); on a timeout the kernel records
// NK_TIMEOUT, drains its own TMA loads and MMAs, frees TMEM and returns.
#pragma once

#include <cuda.h>

#include "nk_common.cuh"
#include "nk_ptx.cuh"

namespace nk {

// WK_INT8: int8 [N,K] per-row scaled; WK_INT4KN: the reference's INT4 [K,N]
// nibble layout; WK_INT4NK: INT4 codes feature-major [N, K/2 bytes] (element
// (n, k) in byte n*K/2 + k/2, low nibble for even k), per-group scale/zero.
enum WeightKind { WK_BF16 = 0, WK_INT8 = 1, WK_INT4KN = 2, WK_INT4NK = 3 };



struct TcTile {  // one output tile: 128 (256 for CTA pairs) features x up to BN tokens
  int w_row;       // first weight row (feature) in the weight tensor map
  int x_row;       // first activation row in the activation tensor map
  int valid;       // (f_valid << 16) | t_valid
  int out_col0;    // output column of feature 0 of the tile
  int y_row = 0;   // y_rank >= 0: output row of token 0 in rank y_rank's buffer
  int y_rank = -1; // -1: output row x_row + j of args.y
  int src = -1;    // >= 0: segment whose rows this launch pulls in (args.pull_tab)
};

struct TcArgs {
  // tile list: dense grid (tiles == nullptr) or an explicit list
  int f_tiles, t_tiles;     // dense: features N in 128-row tiles, tokens M in BN-row tiles
  int n_features, n_tokens; // dense extents
  const TcTile *tiles;      // grouped: list written by a device kernel
  const int *tile_count;    // grouped: number of valid entries in `tiles`
  int k_blocks;             // 64-wide K blocks of the contraction
  int w_k_period;           // >0: weight K block = kb % w_k_period
  int x_k_period;           // >0: activation K block = kb % x_k_period
  int k_splits;             // dense only: >1 splits K over tiles; split s writes its
  long long split_stride;   //   partial sums at y + s * split_stride (elements)
  // epilogue
  void *y;
  long long ldy;
  int y_f32;
  float w_scale;            // per-tensor weight scale (INT4); 1 otherwise
  const float *row_scale;   // [features] per weight row (INT8 row scale) or null
  const float *bias;        // [features] or null
  const float *tok_scale;   // [activation rows] per token (routing weight) or null
  const uint64_t *y_peers;  // tiles with y_rank >= 0: output buffers by rank (peer memory)
  int relu2;
  int w_zero_point;         // INT4 zero point
  // per-group (expert) INT4 parameters: group g = weight row / group_rows
  const float *group_scale; // [groups] or null
  const uint8_t *group_zp;  // [groups] or null (w_zero_point then)
  int group_rows;
  // In-kernel pull of routed rows (expert parallel, FA == 2 kernels): copy
  // warps in every CTA copy each receive segment's rows from its source
  // rank's send buffer (peer memory) into the receive buffer, segments in the
  // order pull_rot, pull_rot + 1, ... (mod pull_segs), and add the rows they
  // copied to pull_arrived[segment].  The producer starts a tile with
  // src >= 0 (its segment) only once that segment's rows have all arrived.
  const uint64_t *pull_src; // [ranks] send buffers (bf16 rows); segment g's
  int pull_seg_per_rank;    //   source rank is g / pull_seg_per_rank
  const int32_t *pull_tab;  // [segments][3]: first send row, first receive row, rows
  int *pull_arrived;        // [segments] rows arrived; zero before the launch
  void *pull_dst;           // receive buffer (bf16 rows)
  int pull_segs, pull_rot;
  long long pull_row_vecs;  // 16-byte words per row
  int *err;
};

// Activation tensor maps with token boxes of 16, 32, 64, 96, ..., 256 rows
// (boxes above the tile's BN unused): each stage loads the token rows with
// ONE TMA copy of the smallest box that covers the rows the MMA reads, so a
// decode tile of a few tokens, or an expert's 192 routed rows, does not move
// a full BN-row tile.  In CTA pairs each CTA loads its half of the MMA's rows
// with the smallest box (up to BN/2 rows) covering them.
constexpr int kTokenBoxes = 9;
__host__ __device__ constexpr int token_box_rows(int i) { return i < 2 ? 16 << i : 32 * i; }
struct TokenMaps {
  CUtensorMap m[kTokenBoxes];
};

// Raw (quantized) weight tile as TMA delivers it.  Feature-major kinds load
// 128 bytes of every weight row at once (whole 128-byte lines): kGroup K
// blocks per raw tile, int8 [128 rows x 2 K blocks of 64 B], INT4 [128 rows x
// 4 K blocks of 32 B]; the reference INT4 [K,N] layout [64 K rows x 64 B
// (128 features)] one K block per tile.
template <int WK>
struct WeightTile {
  static constexpr int kGroup = WK == WK_INT8 ? 2 : (WK == WK_INT4NK ? 4 : 1);
  static constexpr int kRowBytes = WK == WK_INT8 ? 64 : (WK == WK_INT4NK ? 32 : 64);
  static constexpr int kRawBytes =
      WK == WK_BF16 ? 0 : (WK == WK_INT4KN ? 64 * 64 : 128 * 128);
};

// PAIR = 1: one CTA computes 128·FA features x BN tokens.
// PAIR = 2: a cluster of two CTAs computes 256 features x BN tokens with
// tcgen05.mma.cta_group::2; each CTA holds 128 weight rows and BN/2 token rows.
// FA = 2 (single CTAs, bf16 weights): each stage carries two 128-row weight
// tiles against one token tile, accumulated in two TMEM accumulators (2·BN
// columns: the whole tile set, so there is one accumulator set instead of two
// double-buffered ones); the token bytes per weight byte halve.
template <int WK, int BN, int PAIR = 1, int FA = 1>
struct TcConfig {
  static_assert(FA == 1 || (FA == 2 && PAIR == 1 && WK == WK_BF16),
                "two accumulators only for single CTAs with bf16 weights");
  static constexpr bool kQuant = WK != WK_BF16;
#ifndef NK_DECODE_KB
#define NK_DECODE_KB 2
#endif
  // K blocks (64 wide) per stage: decode tiles (few token rows, tiny MMAs)
  // carry two, halving the per-stage hand-offs between the warp roles.
  static constexpr int kKB = (PAIR == 1 && FA == 1 && BN <= 64 && WK != WK_INT4KN) ? NK_DECODE_KB : 1;
  static constexpr int kATileBytes = 128 * 128;     // 128 weight rows x 64 bf16
  static constexpr int kABytes = kATileBytes * FA * kKB;
  static constexpr int kBRows = BN / PAIR;          // token rows loaded per CTA
  static constexpr int kBTileBytes = kBRows * 128;  // kBRows x 64 bf16
  static constexpr int kBBytes = kBTileBytes * kKB;
  static constexpr int kStageBytes = kABytes + kBBytes;
#ifndef NK_STAGES_MAX
#define NK_STAGES_MAX 16
#endif
  // Quantized kinds: a main ring of 3-4 stages (bf16 weight tile + token
  // tile) and a separate, deeper ring of raw tiles that the producer fills
  // ahead of it, so conversion never waits on a load.
  static constexpr int kRawTileBytes = WeightTile<WK>::kRawBytes;
  static constexpr int kStages0 =
      kQuant ? (224 * 1024 - (BN <= 64 ? 6 : 4) * kRawTileBytes) / kStageBytes
             : (224 * 1024) / kStageBytes;
  static constexpr int kStages = kStages0 > NK_STAGES_MAX ? NK_STAGES_MAX : kStages0;
  static constexpr int kRawSlots0 =
      kQuant ? (224 * 1024 - kStages * kStageBytes) / kRawTileBytes : 0;
  static constexpr int kRawSlots = kRawSlots0 > 16 ? 16 : kRawSlots0;
#ifndef NK_TRANSFORM_THREADS
#define NK_TRANSFORM_THREADS 256
#endif
  static constexpr int kTransformThreads = kQuant ? NK_TRANSFORM_THREADS : 0;
  static constexpr int kEpiThreads = 128 * FA;      // 4 warps per accumulator
  // FA == 2: two copy warps for the in-kernel pull (idle without one)
  static constexpr int kCopyWarps = FA == 2 ? 2 : 0;
  static constexpr int kThreads = 64 + kEpiThreads + kTransformThreads + 32 * kCopyWarps;
  static constexpr int kAccSlots = 2 / FA;          // accumulator sets in TMEM
  static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  // FA == 2: two 8 KB buffers of 16 tokens x 256 features (and their two
  // barriers), so outputs bound for a peer's memory leave as 512-byte rows
  static constexpr int kEpiStageBytes = FA == 2 ? 2 * 8192 + 64 : 0;
  static constexpr int kSmemBytes =
      1024 + kStages * kStageBytes + kRawSlots * kRawTileBytes + 768 + kEpiStageBytes;
  static_assert(kSmemBytes <= 232448, "dynamic shared memory above the sm_100a limit");
  static constexpr int kFeatRows = 128 * PAIR * FA; // features per output tile
};

}  // namespace nk
