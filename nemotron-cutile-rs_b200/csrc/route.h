// route.h — routing / plan launchers shared with the MoE layer.
#pragma once
#include "nk_common.cuh"

namespace nk {
nk_status launch_route(const float *scores, int64_t tokens, int E, int K, int mode,
                       int32_t *indices, float *weights, cudaStream_t stream);
// Routing on tensor-core router scores with the reference's exact selection
// and weights (the experts near each token's top-k boundary rescored in f64),
// then the expert plan: counts, offsets and each slot's expert-ordered
// position (slot_pos); with xp, every routed token row copied to its position.
// partial: the router GEMM's f32 split-K partial sums [splits][tokens, E];
// c: their accumulation bound; norms: [2E] from nk_router_norms or null;
// scratch: device memory of route_exact_scratch_bytes(tokens, E, K).
size_t route_exact_scratch_bytes(int64_t tokens, int64_t E, int K);
nk_status launch_route_exact(const float *partial, int splits, const uint16_t *x,
                             int64_t tokens, int H, const uint16_t *w3, const float *bias,
                             const float *norms, float c, int E, int K, int mode, void *scratch,
                             int32_t *indices, float *weights, int32_t *counts, int32_t *offsets,
                             int32_t *slot_pos, uint16_t *xp, cudaStream_t stream);
nk_status launch_router_norms(const uint16_t *w3, int64_t E, int64_t H, float *norms,
                              cudaStream_t stream);
size_t plan_scratch_bytes(int64_t slots, int64_t E);
nk_status launch_plan(const int32_t *indices, int64_t slots, int E, int32_t *counts,
                      int32_t *offsets, int32_t *perm, int32_t *slot_pos, int32_t *chunk_scratch,
                      cudaStream_t stream);
}  // namespace nk
