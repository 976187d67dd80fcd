// Linear layers: Y[M,N] = X[M,K] . W[N,K]^T with bf16 operands and fp32 accumulation.
//
// Small M (a handful of seats) is weight-bandwidth bound: a GEMV kernel streams each weight row once with 16-byte
// loads, several in flight per lane, over enough CTAs to cover every SM.  Larger M goes to cuBLAS (a plain library GEMM): three
// tcgen05 designs of this library's own were built and measured slower than it on the tick's shapes (a persistent
// warp-specialised kernel, a cluster split-K kernel for M <= 256, and a swap-AB kernel with 128 weight rows per MMA
// tile and fused norm / RoPE / SwiGLU epilogues), so the choice is a fixed function of M alone.
#include <cublas_v2.h>

#include <mutex>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"

namespace m3 {

// ------------------------------------------------------------------------------------------------ GEMV
// One warp produces COLS consecutive output columns for all MT rows; lanes split K in 8-element (16 B) chunks, lane l
// taking chunks l, l + 32, ...  A CTA is kGemvWarps warps, so even a 1024-wide layer runs 256 CTAs over the 148 SMs,
// and each lane keeps UNROLL chunks of every column's weight row in flight (8 for rows of 2048+ elements, else 4,
// which is all of a 1024-element row): the weight stream is bound by HBM,
// not by the few CTAs a wider column block would give.  The activation rows (at most 8 x K, read by every warp) come
// through the read-only data cache.  Per output the chunks are accumulated in order and reduced across the warp by
// the same shuffle tree at any MT or COLS.
constexpr int kGemvWarps = 4;

template <int MT, int COLS, int UNROLL, bool OUT_F32, int ACT>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(const bf16* __restrict__ X, int64_t ldx,
                                                               const bf16* __restrict__ W, int64_t ldw,
                                                               void* __restrict__ Y, int64_t ldy, int M, int N,
                                                               int K) {
  static_assert(ACT != kActSwiGLU || COLS == 2, "a SwiGLU warp computes one gate and one up column");
  static_assert(ACT == kActNone || !OUT_F32, "activations write bf16");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // the warp's columns: n0 + c (c < COLS), or with SwiGLU gate row n0 and up row F + n0 of W (F = N / 2)
  const int wid = blockIdx.x * kGemvWarps + warp;
  const int n0 = ACT == kActSwiGLU ? wid : wid * COLS;
  const int cs = ACT == kActSwiGLU ? N / 2 : 1;
  if (n0 >= (ACT == kActSwiGLU ? N / 2 : N)) return;
  const int kv = K / 8;
  float acc[MT][COLS];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int c = 0; c < COLS; ++c) acc[m][c] = 0.f;
  for (int base = lane; base < kv; base += 32 * UNROLL) {
    uint4 wv[UNROLL][COLS];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int k = base + 32 * u;
#pragma unroll
      for (int c = 0; c < COLS; ++c)
        wv[u][c] = (k < kv && n0 + c * cs < N)
                       ? __ldg(reinterpret_cast<const uint4*>(W + (int64_t)(n0 + c * cs) * ldw) + k)
                       : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int k = base + 32 * u;
      if (k >= kv) break;
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        float xf[8];
        unpack8(m < M ? __ldg(reinterpret_cast<const uint4*>(X + (int64_t)m * ldx) + k) : make_uint4(0, 0, 0, 0),
                xf);
#pragma unroll
        for (int c = 0; c < COLS; ++c) {
          float wf[8];
          unpack8(wv[u][c], wf);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[m][c] = fmaf(xf[e], wf[e], acc[m][c]);
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int c = 0; c < COLS; ++c) acc[m][c] = warp_sum(acc[m][c]);
  if (lane == 0) {
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m >= M) break;
      if constexpr (ACT == kActSwiGLU) {  // the gate and up outputs rounded to bf16 as stored, then combined
        reinterpret_cast<bf16*>(Y)[m * ldy + n0] = to_bf(silu_mul1(rbf(acc[m][0]), rbf(acc[m][1])));
      } else {
#pragma unroll
        for (int c = 0; c < COLS; ++c) {
          if (n0 + c >= N) break;
          if (OUT_F32)
            reinterpret_cast<float*>(Y)[m * ldy + n0 + c] = acc[m][c];
          else if (ACT == kActGelu)
            reinterpret_cast<bf16*>(Y)[m * ldy + n0 + c] = to_bf(gelu_erf(rbf(acc[m][c])));
          else
            reinterpret_cast<bf16*>(Y)[m * ldy + n0 + c] = to_bf(acc[m][c]);
        }
      }
    }
  }
}

// Two columns per warp at 8 rows, where the activation reads would otherwise outweigh the weight stream in the cache
// (and always with SwiGLU: a gate and an up column).
template <int MT, int UNROLL, int ACT, bool OUT_F32>
static void launch_gemv_a(const GemmDesc& g, cudaStream_t s) {
  constexpr int COLS = ACT == kActSwiGLU || MT >= 8 ? 2 : 1;
  const int warps = ACT == kActSwiGLU ? g.N / 2 : cdiv(g.N, COLS);
  gemv_kernel<MT, COLS, UNROLL, OUT_F32, ACT>
      <<<cdiv(warps, kGemvWarps), kGemvWarps * 32, 0, s>>>(g.X, g.ldx, g.W, g.ldw, g.Y, g.ldy, g.M, g.N, g.K);
}

template <int MT, int UNROLL>
static void launch_gemv_u(const GemmDesc& g, cudaStream_t s) {
  if (g.act == kActGelu)
    launch_gemv_a<MT, UNROLL, kActGelu, false>(g, s);
  else if (g.act == kActSwiGLU)
    launch_gemv_a<MT, UNROLL, kActSwiGLU, false>(g, s);
  else if (g.y_f32)
    launch_gemv_a<MT, UNROLL, kActNone, true>(g, s);
  else
    launch_gemv_a<MT, UNROLL, kActNone, false>(g, s);
}

template <int MT>
static int launch_gemv(const GemmDesc& g, cudaStream_t s) {
  if (g.K >= 2048)
    launch_gemv_u<MT, 8>(g, s);
  else
    launch_gemv_u<MT, 4>(g, s);
  M3_LAUNCHED();
  return M3_OK;
}

// ------------------------------------------------------------------------------------------------ cuBLAS
namespace {
struct Blas {
  cublasHandle_t h = nullptr;
  void* ws = nullptr;
  size_t ws_bytes = 0;
};
std::mutex g_blas_mu;
std::vector<Blas> g_blas;  // one per device

int blas_for_current_device(Blas** out) {
  int dev = 0;
  M3_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_blas_mu);
  if ((int)g_blas.size() <= dev) g_blas.resize(dev + 1);
  Blas& b = g_blas[dev];
  if (!b.h) {
    if (cublasCreate(&b.h) != CUBLAS_STATUS_SUCCESS) {
      set_error("cublasCreate failed");
      return M3_ERR_CUDA;
    }
    // A fixed workspace lets cuBLAS calls be captured into CUDA graphs (no allocation at launch).
    b.ws_bytes = kBlasWorkspace;
    M3_CUDA(cudaMalloc(&b.ws, b.ws_bytes));
    cublasSetMathMode(b.h, CUBLAS_DEFAULT_MATH);
  }
  *out = &b;
  return M3_OK;
}
}  // namespace

static int launch_cublas(const GemmDesc& g, cudaStream_t s) {
  Blas* b = nullptr;
  M3_TRY(blas_for_current_device(&b));
  if (cublasSetStream(b->h, s) != CUBLAS_STATUS_SUCCESS ||
      cublasSetWorkspace(b->h, g.ws ? g.ws : b->ws, g.ws ? g.ws_bytes : b->ws_bytes) != CUBLAS_STATUS_SUCCESS) {
    set_error("cublasSetStream/Workspace failed");
    return M3_ERR_CUDA;
  }
  const float alpha = 1.f, beta = 0.f;
  // Row-major Y[M,N] = X W^T  <=>  column-major Y^T[N,M] = W^T(op T of col-major [K,N]) . X^T (col-major [K,M]).
  cublasStatus_t st = cublasGemmEx(b->h, CUBLAS_OP_T, CUBLAS_OP_N, g.N, g.M, g.K, &alpha, g.W, CUDA_R_16BF,
                                   (int)g.ldw, g.X, CUDA_R_16BF, (int)g.ldx, &beta, g.Y,
                                   g.y_f32 ? CUDA_R_32F : CUDA_R_16BF, (int)g.ldy, CUBLAS_COMPUTE_32F,
                                   CUBLAS_GEMM_DEFAULT);
  if (st != CUBLAS_STATUS_SUCCESS) {
    set_error("cublasGemmEx failed (status %d) M=%d N=%d K=%d", (int)st, g.M, g.N, g.K);
    return M3_ERR_CUDA;
  }
  return M3_OK;
}

bool gemv_path(const GemmDesc& g) {
  const bool vec_ok = g.K % 8 == 0 && g.ldx % 8 == 0 && g.ldw % 8 == 0 &&
                      (reinterpret_cast<uintptr_t>(g.X) & 15) == 0 && (reinterpret_cast<uintptr_t>(g.W) & 15) == 0;
  return vec_ok && g.M <= 8 && (size_t)8 * g.K * 2 <= 200 * 1024;
}

int gemm(const GemmDesc& g, cudaStream_t s) {
  M3_REQUIRE(g.M >= 0 && g.N > 0 && g.K > 0, M3_ERR_ARG, "gemm: bad shape M=%d N=%d K=%d", g.M, g.N, g.K);
  M3_REQUIRE(g.act == kActNone || (!g.y_f32 && gemv_path(g) && (g.act != kActSwiGLU || g.N % 2 == 0)),
             M3_ERR_UNSUPPORTED, "gemm: activation %d needs the GEMV path (M=%d N=%d K=%d)", g.act, g.M, g.N, g.K);
  if (g.M == 0) return M3_OK;
  if (gemv_path(g)) {
    if (g.M <= 1) return launch_gemv<1>(g, s);
    if (g.M <= 2) return launch_gemv<2>(g, s);
    if (g.M <= 4) return launch_gemv<4>(g, s);
    return launch_gemv<8>(g, s);
  }
  return launch_cublas(g, s);
}

}  // namespace m3

extern "C" int m3_gemm_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy,
                            int32_t m, int32_t n, int32_t k, int32_t y_f32, m3_stream stream) {
  m3::GemmDesc g{reinterpret_cast<const m3::bf16*>(x), ldx, reinterpret_cast<const m3::bf16*>(w), ldw, y, ldy,
                 m, n, k, y_f32 != 0};
  return m3::gemm(g, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int m3_gemm_bf16_act(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy,
                                int32_t m, int32_t n, int32_t k, int32_t act, m3_stream stream) {
  M3_REQUIRE(act == m3::kActGelu || act == m3::kActSwiGLU, M3_ERR_ARG, "m3_gemm_bf16_act: activation %d", act);
  m3::GemmDesc g{reinterpret_cast<const m3::bf16*>(x), ldx, reinterpret_cast<const m3::bf16*>(w), ldw, y, ldy,
                 m, n, k, false};
  g.act = act;
  return m3::gemm(g, reinterpret_cast<cudaStream_t>(stream));
}

namespace m3 {
// The GEMV kernel alone (M <= 8), never a library call: for paths that must not allocate (cuBLAS creates its handle
// and workspace lazily).  Returns M3_ERR_UNSUPPORTED when the shape or alignment does not fit the GEMV kernel.
int gemv_only(const GemmDesc& g, cudaStream_t s) {
  const bool ok = g.act == kActNone && g.M >= 0 && g.M <= 8 && g.N > 0 && g.K > 0 && g.K % 8 == 0 && g.ldx % 8 == 0 && g.ldw % 8 == 0 &&
                  (reinterpret_cast<uintptr_t>(g.X) & 15) == 0 && (reinterpret_cast<uintptr_t>(g.W) & 15) == 0 &&
                  (size_t)8 * g.K * 2 <= 48 * 1024;
  M3_REQUIRE(ok, M3_ERR_UNSUPPORTED, "gemv_only: M=%d N=%d K=%d outside the GEMV kernel's range", g.M, g.N, g.K);
  if (g.M == 0) return M3_OK;
  if (g.M <= 1) return launch_gemv<1>(g, s);
  if (g.M <= 2) return launch_gemv<2>(g, s);
  if (g.M <= 4) return launch_gemv<4>(g, s);
  return launch_gemv<8>(g, s);
}
}  // namespace m3

