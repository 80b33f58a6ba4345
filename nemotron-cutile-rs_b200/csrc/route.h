// route.h — routing / plan launchers shared with the MoE layer.
#pragma once
#include "nk_common.cuh"

namespace nk {
nk_status launch_route(const float *scores, int64_t tokens, int E, int K, int mode,
                       int32_t *indices, float *weights, cudaStream_t stream);
size_t plan_scratch_bytes(int64_t slots, int64_t E);
nk_status launch_plan(const int32_t *indices, int64_t slots, int E, int32_t *counts,
                      int32_t *offsets, int32_t *perm, int32_t *slot_pos, int32_t *chunk_scratch,
                      cudaStream_t stream);
}  // namespace nk
