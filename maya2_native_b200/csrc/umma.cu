// Tensor-core linear layers for sm_100a: Y[M,N] = X[M,K] . W[N,K]^T on the 5th-generation tensor cores.
//
// Two kernels: the persistent warp-specialised GEMM (128 x BN output tiles, TMA operand ring, one thread issuing
// tcgen05.mma into two TMEM accumulators, four epilogue warps) and, for decode-sized batches (M <= 256), a cluster
// split-K form whose K-slices meet in distributed shared memory.  Both operands are K-major bf16 (2-D tiled TMA
// copies, 128-byte swizzle, 64 K-elements per stage); MMAs are kind::f16 with fp32 accumulation.  Every wait is
// bounded (kSpinLimit polls) and reports M3_DEV_TIMEOUT instead of hanging.
#include <cuda.h>

#include <algorithm>

#include <mutex>

#include "common.cuh"
#include "gemm.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace m3 {

constexpr int kBM = 128;
constexpr int kBK = 64;               // bf16 elements per stage along K = one 128-byte swizzle row
constexpr int kUmmaK = 16;

// ------------------------------------------------------------------------------------------------ persistent kernel
// Persistent, warp-specialised form: one CTA per SM walks the output tiles (M fastest, so the CTAs running at the
// same time share B tiles in L2).  Warp 0 (one lane) streams A and B tiles by TMA into a STAGES-deep ring; warp 1
// (one lane) issues the tcgen05 MMAs into one of two TMEM accumulators and commits the stage's "empty" barrier after
// each K step and the accumulator's "full" barrier after the last; warps 2-5 (each reads the 32 TMEM lanes its warp
// index allows) drain the other accumulator meanwhile -- so the epilogue of tile i overlaps the main loop of tile
// i+1 -- and re-arm it.  EPI: 0 bf16 rows, 1 fp32 rows, 2 bf16(GELU_erf(bf16(z))) (the depth / Mimi feed-forward
// activation, rounded where the reference rounds).  Every wait is bounded.
constexpr int kPThreads = 192;

// Epilogue of one warp's 32 rows x 32 columns: the values go through a padded shared-memory block so that the
// global stores are whole 64-byte (bf16) or 128-byte (fp32) row segments, 4 or 8 lanes per row.
constexpr int kStgStride = 36;  // words per staged row (32 + 4 pad): conflict-free row writes and segment reads

template <int EPI>
__device__ __forceinline__ void epi_store(void* Y, int64_t ldy, int row0, int M, int col, int N, const uint32_t (&r)[32],
                                          uint32_t* stg, int lane) {
  if (EPI == 1) {  // fp32: row = lane, 32 words
#pragma unroll
    for (int j = 0; j < 32; j += 4)
      *reinterpret_cast<uint4*>(stg + lane * kStgStride + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 8; ++q) {  // 32 rows x 8 chunks of 16 B
      const int i = lane + 32 * q, rr = i >> 3, c = i & 7;
      const int row = row0 + rr;
      if (row < M && col + c * 4 + 4 <= N)
        *reinterpret_cast<uint4*>(reinterpret_cast<float*>(Y) + (int64_t)row * ldy + col + c * 4) =
            *reinterpret_cast<const uint4*>(stg + rr * kStgStride + c * 4);
    }
  } else {  // bf16 (optionally GELU): row = lane, 16 words
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      float f[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        f[e] = __uint_as_float(r[j + e]);
        if (EPI == 2) {
          const float v = rbf(f[e]);
          f[e] = 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
        }
      }
      *reinterpret_cast<uint4*>(stg + lane * kStgStride + j / 2) = pack8(f);
    }
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // 32 rows x 4 chunks of 16 B
      const int i = lane + 32 * q, rr = i >> 2, c = i & 3;
      const int row = row0 + rr;
      if (row < M && col + c * 8 + 8 <= N)
        *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(Y) + (int64_t)row * ldy + col + c * 8) =
            *reinterpret_cast<const uint4*>(stg + rr * kStgStride + c * 4);
    }
  }
  __syncwarp();
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(kPThreads, 1) umma_persistent_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                       const __grid_constant__ CUtensorMap tmB,
                                                                       void* __restrict__ Y, int64_t ldy, int M,
                                                                       int N, int K, int* status) {
  constexpr int kABytes = kBM * kBK * 2, kBBytes = BN * kBK * 2, kStage = kABytes + kBBytes;
  constexpr int kCols = 2 * BN;  // two accumulators
  static_assert(kCols == 64 || kCols == 128 || kCols == 256 || kCols == 512, "TMEM allocation is a power of 2");
  extern __shared__ __align__(1024) unsigned char umma_smem[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(umma_smem) + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + STAGES * kStage);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  uint32_t* stage_out = tmem_slot + 4;  // [4 epilogue warps][32 rows][kStgStride] words
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = cdiv(M, kBM), tiles = mt * cdiv(N, BN), kts = cdiv(K, kBK);
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);  // one arrival per epilogue warp
    }
    fence_mbar_init();
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      bool ok = true;
      int it = 0;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        const int m0 = (tile % mt) * kBM, n0 = (tile / mt) * BN;
        for (int kt = 0; kt < kts; ++kt, ++it) {
          const int s = it % STAGES;
          if (it >= STAGES && !mbar_wait(&empty[s], ((it / STAGES) - 1) & 1, status)) {
            ok = false;
            break;
          }
          unsigned char* st = base + s * kStage;
          mbar_expect_tx(&full[s], kStage);
          tma_load_2d(st, &tmA, kt * kBK, m0, &full[s]);
          tma_load_2d(st + kABytes, &tmB, kt * kBK, n0, &full[s]);
        }
      }
      // let every copy in flight land before the CTA can exit (bounded; only matters after a timeout)
      for (int i = max(0, it - STAGES); i < it; ++i) mbar_wait(&full[i % STAGES], (i / STAGES) & 1, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      constexpr uint32_t idesc = umma_idesc(BN);
      bool ok = true;
      int it = 0, lt = 0;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++lt) {
        const int acc = lt & 1;
        if (lt >= 2 && !mbar_wait(&tempty[acc], ((lt >> 1) - 1) & 1, status)) break;
        tmem_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        for (int kt = 0; kt < kts; ++kt, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&full[s], (it / STAGES) & 1, status)) {
            ok = false;
            break;
          }
          tmem_fence_after();
          const unsigned char* st = base + s * kStage;
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk)
            umma_f16(d, sw128_desc(st + kk * kUmmaK * 2), sw128_desc(st + kABytes + kk * kUmmaK * 2), idesc,
                     (kt | kk) != 0);
          umma_commit(&empty[s]);
        }
        umma_commit(&tfull[acc]);
      }
    }
  } else {  // epilogue warps
    const int lane_base = (warp & 3) * 32;
    uint32_t* stg = stage_out + (warp - 2) * 32 * kStgStride;
    int lt = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++lt) {
      const int acc = lt & 1;
      const bool got = mbar_wait(&tfull[acc], (lt >> 1) & 1, status);
      if (!__all_sync(0xffffffffu, got)) break;
      tmem_fence_after();
      const int m0 = (tile % mt) * kBM, n0 = (tile / mt) * BN;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)lane_base << 16) + (uint32_t)(acc * BN + c0), r);
        if (n0 + c0 < N) epi_store<EPI>(Y, ldy, m0 + lane_base, M, n0 + c0, N, r, stg, lane);
      }
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }
  tmem_fence_before();
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
}

// ------------------------------------------------------------------------------------------------ small-M split-K
// Y = X W^T for M <= 256 rows (a decode step's batch), where a 128-row tile per CTA leaves most SMs idle and walks
// all of K.  A cluster of S CTAs owns one BN-column tile: CTA s streams k-tiles [s*KT/S, (s+1)*KT/S) of W and of
// all 256 rows of X (one 256-row TMA box: rows past M read as zeros) and accumulates both 128-row halves in TMEM
// (columns [0, BN) and [BN, 2 BN)).  The S partial tiles then meet in shared memory: once the whole cluster is past
// its main loop, each CTA stores the rows of its fp32 partial that CTA o owns (rows [o*256/S, (o+1)*256/S)) into
// slot `rank` of CTA o's idle stage buffers through distributed shared memory (remote stores do not stall the
// sender); after a second cluster barrier each CTA sums its S slots in rank order (a fixed order: reruns are
// bit-identical), rounds once to bf16 and stores its rows.  Every CTA reaches both barriers on every path (a timed-out
// wait only skips work), so the cluster never waits on a missing member.
constexpr int kSmallRows = 256;
constexpr int kSmallThreads = 128;

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kSmallThreads, 1) umma_small_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                      const __grid_constant__ CUtensorMap tmB,
                                                                      bf16* __restrict__ Y, int64_t ldy, int M,
                                                                      int N, int KT, int* status) {
  constexpr int kABytes = kSmallRows * kBK * 2, kBBytes = BN * kBK * 2, kStage = kABytes + kBBytes;
  constexpr int kPRow = BN + 4;  // fp32 words per partial row (16 bytes of padding: conflict-free row writes)
  // S slots of ceil(256 / S) rows each: at most 260 rows for S <= 8
  static_assert(260 * kPRow * 4 <= STAGES * kStage, "the partial slots must fit in the stage buffers");
  extern __shared__ __align__(1024) unsigned char umma_smem[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(umma_smem) + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + STAGES * kStage);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  float* part = reinterpret_cast<float*>(base);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = gridDim.x, rank = (int)cluster_rank(), n0 = blockIdx.y * BN;
  const int kt0 = rank * KT / S, kt1 = (rank + 1) * KT / S, nk = kt1 - kt0;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 32) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;
  int issued = 0;
  if (warp == 0 && lane == 0) {  // TMA producer
    for (int kt = 0; kt < nk && ok; ++kt) {
      const int s = kt % STAGES;
      if (kt >= STAGES) ok = mbar_wait(&empty[s], ((kt / STAGES) - 1) & 1, status);
      if (!ok) break;
      unsigned char* st = base + s * kStage;
      mbar_expect_tx(&full[s], kStage);
      tma_load_2d(st, &tmA, (kt0 + kt) * kBK, 0, &full[s]);
      tma_load_2d(st + kABytes, &tmB, (kt0 + kt) * kBK, n0, &full[s]);
      ++issued;
    }
  } else if (warp == 1 && lane == 0) {  // MMA issuer: both 128-row halves per k-step
    constexpr uint32_t idesc = umma_idesc(BN);
    for (int kt = 0; kt < nk && ok; ++kt) {
      const int s = kt % STAGES;
      ok = mbar_wait(&full[s], (kt / STAGES) & 1, status);
      if (!ok) break;
      tmem_fence_after();
      const unsigned char* st = base + s * kStage;
#pragma unroll
      for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
        const uint64_t bd = sw128_desc(st + kABytes + kk * kUmmaK * 2);
        umma_f16(tmem, sw128_desc(st + kk * kUmmaK * 2), bd, idesc, (kt | kk) != 0);
        umma_f16(tmem + BN, sw128_desc(st + kABytes / 2 + kk * kUmmaK * 2), bd, idesc, (kt | kk) != 0);
      }
      umma_commit(&empty[s]);
    }
    umma_commit(done);
  }
  __syncwarp();
  ok = mbar_wait(done, 0, status) && ok;
  if (warp == 0 && lane == 0 && !ok)  // a load may still be landing in the stage buffers: let it finish first
    for (int kt = 0; kt < issued; ++kt) mbar_wait(&full[kt % STAGES], (kt / STAGES) & 1, nullptr);
  ok = __syncthreads_and(ok);
  tmem_fence_after();
  // Every CTA of the cluster is past its main loop (stage buffers idle): push this CTA's partial rows to the CTA
  // that owns them (rows [o*256/S, (o+1)*256/S) belong to rank o), into slot `rank` of the owner's buffers.
  cluster_sync_all();
  const int rows_max = (kSmallRows + S - 1) / S;
  if (ok) {
    const uint32_t pbase = smem_u32(part);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = h * 128 + warp * 32 + lane;
      int o = r * S / kSmallRows;
      while (o + 1 < S && (o + 1) * kSmallRows / S <= r) ++o;
      while (o > 0 && o * kSmallRows / S > r) --o;
      const uint32_t local = pbase + (uint32_t)(((rank * rows_max + (r - o * kSmallRows / S)) * kPRow) * 4);
      uint32_t dst;
      asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(dst) : "r"(local), "r"((uint32_t)o));
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(h * BN + c0), v);
        if (nk == 0)
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0u;
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst + (uint32_t)((c0 + j) * 4)),
                       "r"(v[j]), "r"(v[j + 1]), "r"(v[j + 2]), "r"(v[j + 3])
                       : "memory");
      }
    }
  }
  tmem_fence_before();
  cluster_sync_all();
  // rows [r0, r1) of the tile: the sum of the S partials in rank order, rounded once
  const int r0 = rank * kSmallRows / S, r1 = min((rank + 1) * kSmallRows / S, M);
  constexpr int kQ = BN / 4;  // float4 columns per row
  if (ok) {
    for (int u = threadIdx.x; u < (r1 - r0) * kQ; u += kSmallThreads) {
      const int lr = u / kQ, q = u % kQ;
      const float* src = part + lr * kPRow + q * 4;
      float4 acc = *reinterpret_cast<const float4*>(src);
      for (int p = 1; p < S; ++p) {
        const float4 v = *reinterpret_cast<const float4*>(src + p * rows_max * kPRow);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      const int col = n0 + q * 4;
      if (col < N)
        *reinterpret_cast<uint2*>(Y + (int64_t)(r0 + lr) * ldy + col) =
            make_uint2(pack2(acc.x, acc.y), pack2(acc.z, acc.w));
    }
  }
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN) : "memory");
}

// ------------------------------------------------------------------------------------------------ host
namespace {
EncodeTiled g_encode = nullptr;
std::once_flag g_encode_once;
}  // namespace

int tensor_map_encoder(EncodeTiled* out) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeTiled>(fn);
  });
  M3_REQUIRE(g_encode, M3_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  *out = g_encode;
  return M3_OK;
}

namespace {
// 2-D map over a row-major bf16 matrix [rows, cols] with leading dimension ld (elements); box = 64 cols x box_rows.
int make_map(CUtensorMap* map, const void* ptr, int rows, int cols, int64_t ld, int box_rows) {
  EncodeTiled enc;
  M3_TRY(tensor_map_encoder(&enc));
  M3_REQUIRE((reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && ld % 8 == 0, M3_ERR_ARG,
             "tensor-core GEMM operand must be 16-byte aligned with a leading dimension multiple of 8");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  M3_REQUIRE(r == CUDA_SUCCESS, M3_ERR_ARG, "cuTensorMapEncodeTiled failed (%d) rows=%d cols=%d ld=%lld", (int)r,
             rows, cols, (long long)ld);
  return M3_OK;
}

int* g_umma_status = nullptr;  // device status word for the tensor-core GEMM (one per process, device 0 ordinal)

}  // namespace

int umma_status_ptr(int** out);

namespace {
int g_sm_count = 0;

template <int BN, int STAGES, int EPI>
int launch_persistent(const CUtensorMap& a, const CUtensorMap& b, void* y, int64_t ldy, int M, int N, int K,
                      cudaStream_t s, int* st) {
  constexpr size_t smem = 1024 + (size_t)STAGES * (kBM * kBK * 2 + BN * kBK * 2) + 256 + 4 * 32 * kStgStride * 4;
  static bool attr = false;
  if (!attr) {
    M3_CUDA(cudaFuncSetAttribute(umma_persistent_kernel<BN, STAGES, EPI>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr = true;
  }
  if (!g_sm_count) {
    int dev = 0;
    M3_CUDA(cudaGetDevice(&dev));
    M3_CUDA(cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev));
  }
  const int tiles = cdiv(M, kBM) * cdiv(N, BN);
  umma_persistent_kernel<BN, STAGES, EPI><<<std::min(tiles, g_sm_count), kPThreads, smem, s>>>(a, b, y, ldy, M, N,
                                                                                             K, st);
  M3_LAUNCHED();
  return M3_OK;
}
}  // namespace

// Y = X W^T (epi 0 bf16, 1 fp32, 2 bf16 GELU) with the persistent tcgen05 kernel; bn = 64, 128 or 256.
int umma_gemm_persistent(const GemmDesc& g, int bn, int epi, cudaStream_t s) {
  M3_REQUIRE(g.M > 0 && g.N > 0 && g.K > 0 && g.N % 8 == 0 && g.ldy % 8 == 0, M3_ERR_ARG,
             "umma_gemm_persistent: M=%d N=%d K=%d ldy=%lld", g.M, g.N, g.K, (long long)g.ldy);
  int* st;
  M3_TRY(umma_status_ptr(&st));
  CUtensorMap a, b;
  M3_TRY(make_map(&a, g.X, g.M, g.K, g.ldx, kBM));
  M3_TRY(make_map(&b, g.W, g.N, g.K, g.ldw, bn));
#define M3_PERS(BN_, ST_)                                                                                       \
  if (epi == 0) return launch_persistent<BN_, ST_, 0>(a, b, g.Y, g.ldy, g.M, g.N, g.K, s, st);                \
  if (epi == 1) return launch_persistent<BN_, ST_, 1>(a, b, g.Y, g.ldy, g.M, g.N, g.K, s, st);                \
  return launch_persistent<BN_, ST_, 2>(a, b, g.Y, g.ldy, g.M, g.N, g.K, s, st);
  switch (bn) {
    case 64: { M3_PERS(64, 8) }
    case 128: { M3_PERS(128, 6) }
    case 256: { M3_PERS(256, 4) }
    default: break;
  }
#undef M3_PERS
  set_error("umma_gemm_persistent: BN %d unsupported", bn);
  return M3_ERR_UNSUPPORTED;
}

namespace {
template <int BN, int STAGES>
int launch_small(const CUtensorMap& a, const CUtensorMap& b, bf16* y, int64_t ldy, int M, int N, int K, int S,
                 cudaStream_t s, int* st) {
  constexpr size_t smem = 1024 + (size_t)STAGES * (kSmallRows * kBK * 2 + BN * kBK * 2) + 256;
  static bool attr = false;
  if (!attr) {
    M3_CUDA(cudaFuncSetAttribute(umma_small_kernel<BN, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem));
    attr = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)S, (unsigned)cdiv(N, BN), 1);
  cfg.blockDim = dim3(kSmallThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = (unsigned)S;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  M3_CUDA(cudaLaunchKernelEx(&cfg, umma_small_kernel<BN, STAGES>, a, b, y, ldy, M, N, cdiv(K, kBK), st));
  M3_LAUNCHED();
  return M3_OK;
}
}  // namespace

// Y = X W^T (bf16 out) for M <= 256 with the cluster split-K kernel: BN = 128 when 128-column tiles with up to 8
// K-splits still give ~96+ CTAs, else 64; S = K-splits per tile (cluster size) so that tiles x S fills the SMs.
int umma_gemm_small(const GemmDesc& g, cudaStream_t s) {
  M3_REQUIRE(g.M > 0 && g.M <= kSmallRows && g.N > 0 && g.K > 0 && !g.y_f32 && g.N % 8 == 0 && g.ldy % 4 == 0 &&
                 (reinterpret_cast<uintptr_t>(g.Y) & 7) == 0,
             M3_ERR_ARG, "umma_gemm_small: M=%d N=%d K=%d ldy=%lld (M <= 256, bf16 out, N %% 8 == 0)", g.M, g.N, g.K,
             (long long)g.ldy);
  int* st;
  M3_TRY(umma_status_ptr(&st));
  const int KT = cdiv(g.K, kBK);
  const int bn = (g.N % 128 == 0 && (g.N / 128) * std::min(8, KT) >= 96) ? 128 : 64;
  const int tiles = cdiv(g.N, bn);
  const int S = std::max(1, std::min({8, KT, 148 / tiles}));
  CUtensorMap a, b;
  M3_TRY(make_map(&a, g.X, g.M, g.K, g.ldx, kSmallRows));
  M3_TRY(make_map(&b, g.W, g.N, g.K, g.ldw, bn));
  bf16* y = reinterpret_cast<bf16*>(g.Y);
  if (bn == 128) return launch_small<128, 3>(a, b, y, g.ldy, g.M, g.N, g.K, S, s, st);
  return launch_small<64, 4>(a, b, y, g.ldy, g.M, g.N, g.K, S, s, st);
}

int umma_status_ptr(int** out) {
  if (!g_umma_status) {
    M3_CUDA(cudaMalloc(&g_umma_status, 256));
    M3_CUDA(cudaMemset(g_umma_status, 0, 256));
  }
  *out = g_umma_status;
  return M3_OK;
}


}  // namespace m3
