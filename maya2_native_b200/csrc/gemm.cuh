#pragma once
#include "common.cuh"

namespace m3 {

constexpr size_t kBlasWorkspace = 32u << 20;  // cuBLAS workspace per device, and per handle that brings its own

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
  // cuBLAS workspace for this call (nullptr: the device's shared one).  GEMMs that may run concurrently with others
  // on a second stream bring their own, so that no two running library kernels share scratch.
  void* ws = nullptr;
  size_t ws_bytes = 0;
  // Activation applied in the GEMV kernel's epilogue (gemv_path only): kActGelu, Y = bf16(gelu(bf16(X W^T)));
  // kActSwiGLU, W holds N = 2F rows (gate rows, then up rows) and Y is [M, F], Y = bf16(swiglu(gate, up)) of the
  // bf16 gate and up outputs.  Outside the GEMV path the caller applies it with the element-wise kernels.
  int act = 0;
};

constexpr int kActNone = 0, kActGelu = 1, kActSwiGLU = 2;

int gemm(const GemmDesc& g, cudaStream_t s);
// Whether gemm() runs this shape on the GEMV kernel (M <= 8, 16-byte aligned rows), where `act` can be fused.
bool gemv_path(const GemmDesc& g);
// GEMV kernel only (M <= 8, K <= 3072); never calls a library that may allocate.
int gemv_only(const GemmDesc& g, cudaStream_t s);
}  // namespace m3
