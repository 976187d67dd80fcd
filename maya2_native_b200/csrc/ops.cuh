#pragma once
// Element-wise / normalisation kernels shared by the depth and Mimi stages (defined in depth.cu).
#include "common.cuh"

namespace m3 {

// x' = bf16(x + a) [then bf16(x' + c[slot])] stored to xout; y = bf16(LayerNorm(x') * w + b) with fp32 statistics.
// Row r of the input lives at src + (r / T) * sb + (r % T) * st.
__global__ void add_ln_kernel(const bf16* __restrict__ src, int T, int64_t sb, int64_t st,
                              const bf16* __restrict__ a, const bf16* __restrict__ c, int64_t c_slot_stride,
                              const int* __restrict__ slot32, bf16* __restrict__ xout, bf16* __restrict__ y,
                              const bf16* __restrict__ w, const bf16* __restrict__ bias, float eps, int D);

// add_ln_kernel over `rows` rows, one CTA per row (counts its launch).
int launch_add_ln(int rows, const bf16* src, int T, int64_t sb, int64_t st, const bf16* a, const bf16* c,
                   int64_t c_slot_stride, const int* slot32, bf16* xout, bf16* y, const bf16* w, const bf16* bias,
                   float eps, int D, cudaStream_t s);

// In place: f = bf16(gelu_erf(f)) over n8 groups of 8 elements.
__global__ void gelu_kernel(bf16* __restrict__ f, int64_t n8);

// ELU (alpha 1) of nn.ELU; elu8 applies it to 8 packed bf16 values and rounds each result to bf16.
__device__ __forceinline__ float elu(float x) { return x > 0.f ? x : expm1f(x); }

__device__ __forceinline__ uint4 elu8(const uint4& u) {
  float f[8];
  unpack8(u, f);
#pragma unroll
  for (int e = 0; e < 8; ++e) f[e] = elu(f[e]);
  return pack8(f);
}

inline int norm_block(int D) { return D / 8 < 32 ? 32 : (D / 8 > 1024 ? 1024 : (D / 8 + 31) / 32 * 32); }

}  // namespace m3
