// Shared device helpers for the Maya3 decode-tick kernels (sm_100a).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

#include "../../include/maya3_b200.h"

namespace m3 {

using bf16 = __nv_bfloat16;

// ------------------------------------------------------------------------------------------------ errors
// Host-side last-error string (thread-local) returned by m3_last_error().
void set_error(const char* fmt, ...);
const char* last_error();

#define M3_CUDA(call)                                                                        \
  do {                                                                                       \
    cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess) {                                                                 \
      ::m3::set_error("%s:%d %s: %s", __FILE__, __LINE__, #call, cudaGetErrorString(e_));    \
      return M3_ERR_CUDA;                                                                    \
    }                                                                                        \
  } while (0)

#define M3_TRY(call)                  \
  do {                                \
    int s_ = (call);                  \
    if (s_ != M3_OK) return s_;       \
  } while (0)

#define M3_REQUIRE(cond, code, ...)   \
  do {                                \
    if (!(cond)) {                    \
      ::m3::set_error(__VA_ARGS__);   \
      return (code);                  \
    }                                 \
  } while (0)

// Every launch of one of this library's kernels is followed by M3_LAUNCHED(): it counts the launch (the count a
// CUDA graph capture sees is the number of this library's kernels in the graph) and checks the launch error.
void count_launch();
#define M3_LAUNCHED()                  \
  do {                                 \
    ::m3::count_launch();              \
    M3_CUDA(cudaGetLastError());       \
  } while (0)

// Device status word: kernels record the first problem they see (bad index, timed-out wait) and carry on safely;
// the host reads it after the tick's synchronization point.
__device__ __forceinline__ void report(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// ------------------------------------------------------------------------------------------------ numerics
__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
__device__ __forceinline__ float to_f(bf16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ bf16 to_bf(float x) { return __float2bfloat16_rn(x); }
// Round an fp32 value to the nearest bf16 and return it as fp32 (the reference stores every such intermediate).
__device__ __forceinline__ float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Activations of the feed-forward layers on one value, fp32 in and out (the callers round):
// GELU, erf form (F.gelu): 0.5 x (1 + erf(x / sqrt 2)); SwiGLU of a bf16 gate / up pair (serve/fast_backbone.py:201-202,
// F.silu(g) * u in bf16): bf16(silu(g)) * u.  The element-wise kernels and the GEMV epilogues share these, so that
// a fused and an unfused layer give the same bits.
__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.f + erff(x * 0.70710678118654752f)); }
__device__ __forceinline__ float silu_mul1(float g, float u) { return rbf(g / (1.f + expf(-g))) * u; }

__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  f[0] = bf_lo(u.x); f[1] = bf_hi(u.x); f[2] = bf_lo(u.y); f[3] = bf_hi(u.y);
  f[4] = bf_lo(u.z); f[5] = bf_hi(u.z); f[6] = bf_lo(u.w); f[7] = bf_hi(u.w);
}
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint4 pack8(const float* f) {
  return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x a multiple of 32 (<= 1024); `red` needs 32 floats of shared memory.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  return warp_sum(t);
}
__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : -INFINITY;
  return warp_max(t);
}

// ------------------------------------------------------------------------------------------------ async copies
// 1-D bulk copies (the TMA engine's untiled form) into shared memory, completed on an mbarrier.  Every wait is
// bounded: after kSpinLimit polls the waiter records M3_DEV_TIMEOUT and gives up instead of hanging the GPU.
constexpr uint32_t kSpinLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, uint32_t limit = kSpinLimit) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  report(status, M3_DEV_TIMEOUT);
  return false;
}
// Global -> shared bulk copy of `bytes` (multiple of 16; both addresses 16-byte aligned), signalling `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__host__ __device__ inline int cdiv(int a, int b) { return (a + b - 1) / b; }

}  // namespace m3
