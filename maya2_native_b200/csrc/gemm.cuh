#pragma once
#include "common.cuh"

namespace m3 {

// Y[M,N] = X[M,K] . W[N,K]^T (row-major, leading dimensions in elements), fp32 accumulation.
struct GemmDesc {
  const bf16* X;
  int64_t ldx;
  const bf16* W;
  int64_t ldw;
  void* Y;
  int64_t ldy;
  int M, N, K;
  bool y_f32;  // Y stored as fp32 instead of bf16
};

int gemm(const GemmDesc& g, cudaStream_t s);
// GEMV kernel only (M <= 8, K <= 3072); never calls a library that may allocate.
int gemv_only(const GemmDesc& g, cudaStream_t s);
// Persistent warp-specialised tcgen05 GEMM; epi 0 = bf16 out, 1 = fp32 out, 2 = bf16(GELU(bf16(z))).
int umma_gemm_persistent(const GemmDesc& g, int bn, int epi, cudaStream_t s);
// Cluster split-K tcgen05 GEMM for M <= 256 rows (bf16 out): the S K-slices of a column tile are summed through
// distributed shared memory.
int umma_gemm_small(const GemmDesc& g, cudaStream_t s);
// The implementations behind gemm(), selectable for tests and measurement.
enum GemmImpl { kGemmAuto = 0, kGemmGemv = 1, kGemmCublas = 2, kGemmUmma = 3, kGemmUmmaGelu = 4, kGemmUmmaSmall = 5 };
int gemm_impl(const GemmDesc& g, int impl, cudaStream_t s);

}  // namespace m3
