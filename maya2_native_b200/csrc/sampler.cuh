#pragma once
#include "common.cuh"

namespace m3 {

// Depth level sampler over `rows` logit rows of width V (see sampler.cu).  slot32 (optional) maps a row to the slot
// whose seed/counter it uses; embed/next_row (optional) receive embed[code] as the next prefix row.
// The next depth level's first LayerNorm, done by the sampler CTA of each row once the row's new prefix entry is
// written (one warp per prefix row): for the T rows start .. start+T-1 of row b's prefix (prefix + b * sb), x gets a
// copy (x + (b * T + i) * D) and y = bf16(LayerNorm(row) * w + bias) with fp32 statistics.  Unused when x is null.
struct PrefixLn {
  const bf16* prefix;
  int64_t sb;
  int start, T;
  bf16* x;
  bf16* y;
  const bf16* w;
  const bf16* bias;
  float eps;
};

int launch_topk_sample(const void* logits, bool bf, int64_t ld, int rows, int V, const int32_t* seed,
                       const int32_t* ctr, const int* slot32, int level, float inv_temp, int k, int greedy,
                       int64_t* codes, int64_t code_stride, const bf16* embed, int D, bf16* next_row,
                       int64_t next_stride, cudaStream_t s, const PrefixLn& ln = PrefixLn{});

}  // namespace m3
