#pragma once
#include "common.cuh"

namespace m3 {

// Depth level sampler over `rows` logit rows of width V (see sampler.cu).  slot32 (optional) maps a row to the slot
// whose seed/counter it uses; embed/next_row (optional) receive embed[code] as the next prefix row.
int launch_topk_sample(const void* logits, bool bf, int64_t ld, int rows, int V, const int32_t* seed,
                       const int32_t* ctr, const int* slot32, int level, float inv_temp, int k, int greedy,
                       int64_t* codes, int64_t code_stride, const bf16* embed, int D, bf16* next_row,
                       int64_t next_stride, cudaStream_t s);

}  // namespace m3
