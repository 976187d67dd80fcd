// Fused SEANet decoder stages on the tensor cores (replace, for the long low-channel stages, the chain
// ELU -> GEMM -> fp32 partials -> overlap fold -> im2col -> GEMM -> bias/ELU -> GEMM -> bias/residual of
// serve/fast_codec.py:104-132 with two kernels per stage whose intermediates never leave the SM).
//
// Both kernels are persistent (a CTA per SM walks a strided list of 64-row tiles), keep their weight slice resident
// in shared memory (rows padded by 16 bytes so ldmatrix reads are conflict-free), and double-buffer the activation
// tiles, which arrive by TMA (3-D tensor maps [stream][step][channel], 64-channel boxes, 128-byte swizzle; causal
// taps are row-shifted boxes, and rows before the first or after the last step of a stream read as zeros).  The
// arithmetic is mma.sync m16n8k16 (bf16 operands, fp32 accumulation) with the reference's bf16 rounding points in the
// epilogues.  All waits are bounded; a CTA that gives up drains its copies and reports M3_DEV_TIMEOUT.
#include <algorithm>

#include "mma.cuh"
#include "ops.cuh"
#include "seanet.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace m3 {

namespace {
constexpr int kUM = 128;                                // transposed conv: output rows per tile (tcgen05 M)
constexpr int kStgRow = 80;                             // transposed conv epilogue staging: bytes per row (64 + pad)
constexpr int kBM = 128;                                // residual block: output rows per tile (8 warps x 16)
constexpr int kResThreads = 256;
constexpr int kResRows = kBM + 2;                       // residual-block tile rows incl. 2 causal history rows
constexpr uint32_t kResBox = (kResRows * 128 + 1023) / 1024 * 1024;  // 130-row box, padded to the swizzle atom
int g_sms = 0;
int g_res_per_sm[2] = {1, 1};  // resident residual-block CTAs per SM (cout 64, 128), from the occupancy calculator
uint16_t* g_elu_lut = nullptr;  // bf16 ELU of the negative bf16 patterns (one per process; device of the first init)

__device__ __forceinline__ unsigned char* align1024(unsigned char* p) {
  return reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~(uintptr_t)1023);
}

// output columns per transposed-conv CTA: the whole row when it fits one MMA (N <= 256), else 128
int convt_bn(int N) { return N <= 256 ? N : 128; }
int convt_stages(int bn) { return bn > 128 ? 2 : 3; }
}  // namespace

// ------------------------------------------------------------------------------------------------ transposed conv
// Output rows t = t0 .. t0+127 of one stream (t = 0..L) against BN output columns: A = the 2-tap rows
// [e[t-1], e[t]] (two row-shifted TMA boxes per 64-channel chunk; rows -1 and L read as zeros), B = Wc rows, on
// tcgen05 (one thread issues the MMAs, fp32 accumulators in TMEM, a STAGES-deep TMA ring).  Epilogue (warp w owns
// TMEM lanes 32w..32w+31 = rows): bf16(z + bias); row 0 adds the previous frame's tail after rounding, as the
// streaming reference does; row L becomes the next tail bf16(bf16(z + b) - b).
template <int BN, int STAGES>
__global__ void __launch_bounds__(128) convt_umma_kernel(
    const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap, const bf16* __restrict__ bias,
    const bf16* __restrict__ tail_in, int64_t in_row, bf16* __restrict__ state, int64_t state_row, int64_t tail_off,
    const int* __restrict__ slot32, bf16* __restrict__ u, int L, int r, int cin, int cout, int* status) {
  constexpr int kA = kUM * 64 * 2, kB = BN * 64 * 2, kStage = kA + kB;
  constexpr int kCols = BN <= 32 ? 32 : (BN <= 64 ? 64 : (BN <= 128 ? 128 : 256));
  const int n0 = blockIdx.x * BN, t0 = blockIdx.y * kUM, b = blockIdx.z;
  const int N = r * cout, KT = 2 * cin / 64, CB = cin / 64;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + STAGES * kStage);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kCols)
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
  if (warp == 0 && lane == 0) {  // TMA producer
    for (int kt = 0; kt < KT && ok; ++kt) {
      const int s = kt % STAGES;
      if (kt >= STAGES) ok = mbar_wait(&empty[s], ((kt / STAGES) - 1) & 1, status);
      if (!ok) break;
      unsigned char* st = base + s * kStage;
      mbar_expect_tx(&full[s], kStage);
      tma_load_3d(st, &amap, (kt % CB) * 64, t0 - 1 + kt / CB, b, &full[s]);
      tma_load_2d(st + kA, &bmap, kt * 64, n0, &full[s]);
    }
  } else if (warp == 1 && lane == 0) {  // MMA issuer
    constexpr uint32_t idesc = umma_idesc(BN);
    for (int kt = 0; kt < KT && ok; ++kt) {
      const int s = kt % STAGES;
      ok = mbar_wait(&full[s], (kt / STAGES) & 1, status);
      if (!ok) break;
      tmem_fence_after();
      const unsigned char* st = base + s * kStage;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_f16(tmem, sw128_desc(st + kk * 32), sw128_desc(st + kA + kk * 32), idesc, (kt | kk) != 0);
      umma_commit(&empty[s]);
    }
    umma_commit(done);
  }
  __syncwarp();
  ok = mbar_wait(done, 0, status) && ok;
  tmem_fence_after();
  const int t = t0 + warp * 32 + lane;
  bf16* st = state + (int64_t)slot32[b] * state_row + tail_off;
  // The stage buffers are idle once every MMA has completed: each warp stages its 32 rows x 32 columns there
  // (lane = row, 64 bytes + 16 of padding so the 16-byte writes are conflict-free) and stores them back as
  // 64-byte row segments, eight rows per instruction.
  unsigned char* stg = base + warp * (32 * kStgRow);
  if (ok) {
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      uint32_t acc[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + c0, acc);
      const int n = n0 + c0, co0 = n % cout;  // a 32-column chunk never crosses a cout block (cout % 32 == 0)
      if (t <= L) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          float bv[8], v[8];
          unpack8(*reinterpret_cast<const uint4*>(bias + co0 + j), bv);
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = rbf(__uint_as_float(acc[j + e]) + bv[e]);
          if (t == L) {
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = v[e] - bv[e];
            *reinterpret_cast<uint4*>(st + n + j) = pack8(v);
            continue;
          }
          if (t == 0) {
            float tv[8];
            unpack8(*reinterpret_cast<const uint4*>(tail_in + (int64_t)b * in_row + n + j), tv);
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = v[e] + tv[e];
          }
          *reinterpret_cast<uint4*>(stg + lane * kStgRow + j * 2) = pack8(v);
        }
      }
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int rr = i * 8 + (lane >> 2), tt = t0 + warp * 32 + rr;
        if (tt < L)
          *reinterpret_cast<uint4*>(u + ((int64_t)b * L + tt) * N + n + (lane & 3) * 8) =
              *reinterpret_cast<const uint4*>(stg + rr * kStgRow + (lane & 3) * 16);
      }
      __syncwarp();
    }
  }
  tmem_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
}

// Persistent form of the same transposed conv for the long stages: a CTA keeps one BN-column slice of the repacked
// weights resident in shared memory (KT k-tiles, loaded once) and walks a strided list of 128-row tiles of every
// stream: a TMA producer warp streams the 2-tap A tiles through a STAGES-deep ring, one thread issues the MMAs into
// two TMEM accumulators (a tile's epilogue overlaps the next tile's MMAs), and eight epilogue warps (two per TMEM
// lane quarter, each taking half of the columns) apply bias / tail / rounding into a double-buffered per-warp
// staging block from which one lane issues a TMA bulk store of the 32 x 32 tile (rows past the stream's end are not
// written).  The bias of the CTA's columns is staged once in shared memory.  Each CTA allocates 2 x 128 TMEM
// columns: releasing a larger allocation at exit measured several microseconds slower.
constexpr int kCpEpiWarps = 8;
constexpr int kCpCtl = 2048;  // barriers, TMEM address, the bias row and the tail rows ahead of the staging blocks
constexpr int kCpTailStage = 1024;  // offset of the epilogue warps' tail rows in the control block
constexpr int kCpThreads = 64 + 32 * kCpEpiWarps;
constexpr int kCpStages = 4;

template <int BN, int KT>
__global__ void __launch_bounds__(kCpThreads, 1) convt_pers_kernel(
    const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
    const __grid_constant__ CUtensorMap smap, const bf16* __restrict__ bias,
    const bf16* __restrict__ tail_in, int64_t in_row, bf16* __restrict__ state, int64_t state_row, int64_t tail_off,
    const int* __restrict__ slot32, bf16* __restrict__ u, int L, int r, int cin, int cout, int R, int* status) {
  constexpr int kA = kUM * 64 * 2, kBt = BN * 64 * 2, CB = KT / 2;
  constexpr int kCols = 2 * BN;
  static_assert(kCols == 256 || kCols == 512, "two accumulators of 128 or 256 columns");
  static_assert(256 + BN * 4 <= kCpTailStage && kCpTailStage + kCpEpiWarps * BN <= kCpCtl,
                "bias row and tail rows fit the control block");
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = align1024(smem_raw);
  unsigned char* bres = base;                       // [KT][BN rows x 128 B] resident weights
  unsigned char* astg = bres + KT * kBt;            // [kCpStages][128 rows x 128 B]
  unsigned char* ctl = astg + kCpStages * kA;     // 256 bytes of barriers and the TMEM address
  uint64_t* bfull = reinterpret_cast<uint64_t*>(ctl);
  uint64_t* full = bfull + 1;
  uint64_t* empty = full + kCpStages;
  uint64_t* tfull = empty + kCpStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  float* bias_s = reinterpret_cast<float*>(ctl + 256);  // [BN] bias of this CTA's columns
  unsigned char* stg_all = ctl + kCpCtl;                // [kCpEpiWarps][2 buffers][32 rows x 64 B, 64-byte swizzle]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int N = r * cout, NC = N / BN, nc = blockIdx.x % NC, cpc = gridDim.x / NC, li = blockIdx.x / NC;
  const int n0 = nc * BN, TT = (L + 1 + kUM - 1) / kUM, tiles = R * TT;
  if (li >= cpc) return;  // grid rounding (the host launches NC x cpc CTAs)
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (threadIdx.x == 0) {
    mbar_init(bfull, 1);
    for (int s = 0; s < kCpStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kCpEpiWarps);
    }
    fence_mbar_init();
  }
  for (int c = threadIdx.x; c < BN; c += blockDim.x) bias_s[c] = to_f(bias[(n0 + c) % cout]);
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp == 0) {
    if (lane == 0) {  // TMA producer: the weight slice once, then the A tiles
      mbar_expect_tx(bfull, KT * kBt);
      for (int kt = 0; kt < KT; ++kt) tma_load_2d(bres + kt * kBt, &bmap, kt * 64, n0, bfull);
      bool ok = true;
      int it = 0;
      for (int j = li; j < tiles && ok; j += cpc) {
        const int b = j / TT, t0 = (j % TT) * kUM;
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = it % kCpStages;
          if (it >= kCpStages && !mbar_wait(&empty[s], ((it / kCpStages) - 1) & 1, status)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], kA);
          tma_load_3d(astg + s * kA, &amap, (kt % CB) * 64, t0 - 1 + kt / CB, b, &full[s]);
        }
      }
      // every copy in flight lands before the CTA can exit (bounded; only matters after a timeout)
      mbar_wait(bfull, 0, nullptr);
      for (int i = max(0, it - kCpStages); i < it; ++i) mbar_wait(&full[i % kCpStages], (i / kCpStages) & 1, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      constexpr uint32_t idesc = umma_idesc(BN);
      bool ok = mbar_wait(bfull, 0, status);
      int it = 0, lt = 0;
      for (int j = li; j < tiles && ok; j += cpc, ++lt) {
        const int acc = lt & 1;
        if (lt >= 2 && !mbar_wait(&tempty[acc], ((lt >> 1) - 1) & 1, status)) break;
        tmem_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * BN);
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = it % kCpStages;
          if (!mbar_wait(&full[s], (it / kCpStages) & 1, status)) {
            ok = false;
            break;
          }
          tmem_fence_after();
          const unsigned char* a = astg + s * kA;
          const unsigned char* bt = bres + kt * kBt;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(d, sw128_desc(a + kk * 32), sw128_desc(bt + kk * 32), idesc, (kt | kk) != 0);
          umma_commit(&empty[s]);
        }
        umma_commit(&tfull[acc]);
      }
    }
  } else {  // epilogue warps: warp w reads TMEM lanes 32 (w % 4) .. +31 = tile rows, columns of half (w - 2) / 4
    const int lane_base = (warp & 3) * 32, cbeg = ((warp - 2) / 4) * (BN / 2);
    unsigned char* stg = stg_all + (warp - 2) * 4096;
    // this warp's 64 columns of the previous frame's tail (row 0's addend), staged in the control block
    bf16* tail_s = reinterpret_cast<bf16*>(ctl + kCpTailStage + (warp - 2) * (BN / 2) * 2);
    int lt = 0, nst = 0;
    for (int j = li; j < tiles; j += cpc, ++lt) {
      const int acc = lt & 1;
      const int b = j / TT, t0 = (j % TT) * kUM, t = t0 + lane_base + lane;
      // global reads the epilogue needs are issued before the wait for the accumulator, which hides their latency:
      // the stream's slot (row L's state write) and, in the warp holding row 0, the previous frame's tail
      const int slot = slot32[b];
      const bool row0 = t0 == 0 && lane_base == 0;
      uint32_t tail2 = 0u;
      if (row0) tail2 = *reinterpret_cast<const uint32_t*>(tail_in + (int64_t)b * in_row + n0 + cbeg + 2 * lane);
      const bool got = mbar_wait(&tfull[acc], (lt >> 1) & 1, status);
      if (!__all_sync(0xffffffffu, got)) break;
      tmem_fence_after();
      if (row0) reinterpret_cast<uint32_t*>(tail_s)[lane] = tail2;
      __syncwarp();
      bf16* st = state + (int64_t)slot * state_row + tail_off;
      // one 32-column chunk: bias, the row-0 tail / row-L state special cases, the swizzled staging block, one TMA
      // store of its 32 rows (the store of the chunk before last must have read its buffer)
      auto chunk = [&](const uint32_t (&v32)[32], int c0) {
        const int n = n0 + c0;
        unsigned char* sb = stg + (nst & 1) * 2048;
        if (nst >= 2 && lane == 0) bulk_wait_read<1>();
        __syncwarp();
        if (t <= L) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(v32[q * 8 + e]) + bias_s[c0 + q * 8 + e];
            if (t == L) {  // the next frame's overlap tail: bf16(bf16(z + b) - b)
#pragma unroll
              for (int e = 0; e < 8; ++e) v[e] = rbf(v[e]) - bias_s[c0 + q * 8 + e];
              *reinterpret_cast<uint4*>(st + n + q * 8) = pack8(v);
              continue;
            }
            if (t == 0) {  // bf16(bf16(z + b) + previous tail)
              float tv[8];
              unpack8(*reinterpret_cast<const uint4*>(tail_s + (c0 - cbeg) + q * 8), tv);
#pragma unroll
              for (int e = 0; e < 8; ++e) v[e] = rbf(v[e]) + tv[e];
            }
            *reinterpret_cast<uint4*>(sb + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4)) = pack8(v);  // one rounding
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(&smap, sb, n, t0 + lane_base, b);
          bulk_commit();
        }
        ++nst;
      };
#pragma unroll 1
      for (int c0 = cbeg; c0 < cbeg + BN / 2; c0 += 64) {  // two TMEM loads in flight per step
        uint32_t va[32], vb[32];
        const uint32_t ta = tmem + ((uint32_t)lane_base << 16) + (uint32_t)(acc * BN + c0);
        tmem_ld32_async(ta, va);
        tmem_ld32_async(ta + 32, vb);
        tmem_wait_ld();
        chunk(va, c0);
        chunk(vb, c0 + 32);
      }
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (lane == 0) bulk_wait_all();  // the stores have read their staging blocks and landed before the CTA exits
    __syncwarp();
  }
  tmem_fence_before();
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
}

constexpr size_t convt_pers_smem(int bn, int kt) {
  return 1024 + (size_t)kt * bn * 128 + (size_t)kCpStages * kUM * 128 + kCpCtl + (size_t)kCpEpiWarps * 4096;
}

// ------------------------------------------------------------------------------------------------ residual block
// ELU of a bf16 value by table: every ELU input in the block is an exact bf16 number, so the rounded result
// bf16(ELU(x)) is a function of the 16 input bits.  x >= 0 maps to itself.  For negative x the table covers the
// magnitudes 2^-9 <= |x| < 8, filled once from expm1f exactly as the elementwise kernels compute it; below 2^-9,
// expm1(x) = x (1 + x/2 + ...) differs from x by less than 2^-10 of |x|, under half a bf16 unit in the last place
// (at least 2^-9 of |x|), so bf16(ELU(x)) = x; at |x| >= 8 it rounds to -1 (e^x < 2^-11); NaN stays NaN.
constexpr uint32_t kEluLo = 0x3B00u;  // bf16 magnitude pattern of 2^-9
constexpr uint32_t kEluHi = 0x4100u;  // of 8
constexpr int kEluLut = (int)(kEluHi - kEluLo);

__device__ __forceinline__ uint32_t elu_bits(uint32_t h, const uint16_t* lut) {
  const uint32_t j = h - (0x8000u | kEluLo);  // unsigned: below the table's first pattern wraps out of range
  if (j < (uint32_t)kEluLut) return lut[j];
  return h - (0x8000u | kEluHi) <= 0xFF80u - (0x8000u | kEluHi) ? 0xBF80u : h;  // -inf <= x <= -8: -1
}
__device__ __forceinline__ uint32_t elu2(uint32_t v, const uint16_t* lut) {
  return elu_bits(v & 0xFFFFu, lut) | (elu_bits(v >> 16, lut) << 16);
}

__global__ void elu_lut_kernel(uint16_t* __restrict__ lut) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= kEluLut) return;
  const float x = __uint_as_float((((uint32_t)i + kEluLo) | 0x8000u) << 16);
  const __nv_bfloat16 y = __float2bfloat16_rn(elu(x));
  lut[i] = *reinterpret_cast<const uint16_t*>(&y);
}

// e = ELU(u + b2 + W2 . ELU(b1 + W1 . [ELU(u)[t-2], ELU(u)[t-1], ELU(u)[t]])) for 128 rows per tile, one warp per
// 16 rows (8 warps): the first GEMM's accumulators become the second GEMM's A fragments in registers.  Values
// between the steps stay as packed bf16 pairs, each rounding point is one paired conversion.  The tile is ELU'd in
// place in shared memory after each thread has kept the raw u values its epilogue adds (the residual); with NBUF = 2
// the next tile's load goes out when a tile starts, with NBUF = 1 (the wide stage, two CTAs per SM) once the first
// GEMM has read the tile.
template <int COUT, int HID>
struct ResCfg {
  static constexpr int NBUF = COUT >= 128 ? 1 : 2;
  static constexpr int MINB = COUT >= 128 ? 2 : 3;  // CTAs per SM the register budget is sized for
};

template <int COUT, int HID>
__global__ void __launch_bounds__(kResThreads, (ResCfg<COUT, HID>::MINB)) res_fused_kernel(
    const __grid_constant__ CUtensorMap umap, const bf16* __restrict__ w1, const bf16* __restrict__ b1,
    const bf16* __restrict__ w2, const bf16* __restrict__ b2, const bf16* __restrict__ hist_in, int64_t in_row,
    bf16* __restrict__ state, int64_t state_row, int64_t hist_off, const int* __restrict__ slot32,
    bf16* __restrict__ e, int Lo, int R, const uint16_t* __restrict__ elu_lut, int* status) {
  constexpr int CB = COUT / 64, K1 = 3 * COUT, NT1 = HID / 8, NT2 = COUT / 8, NBUF = ResCfg<COUT, HID>::NBUF;
  static_assert(COUT % 64 == 0 && HID % 16 == 0, "channel counts");
  const int tps = (Lo + kBM - 1) / kBM;
  const int total = R * tps;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* raw = align1024(smem_raw);                  // [NBUF][CB][kResBox] u as loaded, then ELU(u)
  bf16* W1 = reinterpret_cast<bf16*>(raw + NBUF * CB * kResBox);  // [HID][K1 + 8]
  bf16* W2 = W1 + HID * (K1 + 8);                            // [COUT][HID + 8]
  uint16_t* lut = reinterpret_cast<uint16_t*>(W2 + COUT * (HID + 8));  // [kEluLut]
  uint32_t* b2s = reinterpret_cast<uint32_t*>(lut + kEluLut);  // [COUT / 2] b2 as bf16 pairs
  uint64_t* bar = reinterpret_cast<uint64_t*>(b2s + COUT / 2);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, tq = lane & 3, jm = lane >> 3;
  if (tid == 0) {
    for (int i = 0; i < NBUF; ++i) mbar_init(&bar[i], 1);
    fence_mbar_init();
  }
  for (int i = tid; i < HID * (K1 / 8); i += kResThreads) {
    const int rr = i / (K1 / 8), c8 = i % (K1 / 8);
    *reinterpret_cast<uint4*>(W1 + rr * (K1 + 8) + c8 * 8) =
        *reinterpret_cast<const uint4*>(w1 + (int64_t)rr * K1 + c8 * 8);
  }
  for (int i = tid; i < COUT * (HID / 8); i += kResThreads) {
    const int rr = i / (HID / 8), c8 = i % (HID / 8);
    *reinterpret_cast<uint4*>(W2 + rr * (HID + 8) + c8 * 8) =
        *reinterpret_cast<const uint4*>(w2 + (int64_t)rr * HID + c8 * 8);
  }
  for (int i = tid; i < kEluLut / 8; i += kResThreads)
    reinterpret_cast<uint4*>(lut)[i] = reinterpret_cast<const uint4*>(elu_lut)[i];
  for (int i = tid; i < COUT; i += kResThreads) reinterpret_cast<bf16*>(b2s)[i] = b2[i];
  // this thread's bias columns of epilogue 1 (columns kk*16 + 2tq (+1), +8)
  float bias1[HID / 16][4];
#pragma unroll
  for (int kk = 0; kk < HID / 16; ++kk) {
    const int c0 = kk * 16 + 2 * tq;
    bias1[kk][0] = to_f(b1[c0]);
    bias1[kk][1] = to_f(b1[c0 + 1]);
    bias1[kk][2] = to_f(b1[c0 + 8]);
    bias1[kk][3] = to_f(b1[c0 + 9]);
  }
  __syncthreads();
  auto issue = [&](int tile, int buf) {
    const int b = tile / tps, t0 = (tile % tps) * kBM;
    mbar_expect_tx(&bar[buf], CB * kResRows * 128);
    for (int cb = 0; cb < CB; ++cb)
      tma_load_3d(raw + (buf * CB + cb) * kResBox, &umap, cb * 64, t0 - 2, b, &bar[buf]);
  };
  if (tid == 0 && blockIdx.x < total) issue(blockIdx.x, 0);
  const int m0 = warp * 16;
  int it = 0;
  for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++it) {
    const int buf = NBUF == 2 ? (it & 1) : 0;
    const uint32_t parity = (uint32_t)(it / NBUF) & 1u;
    const bool more = tile + gridDim.x < total;
    if (NBUF == 2 && tid == 0 && more) issue(tile + gridDim.x, buf ^ 1);
    const bool ok = mbar_wait(&bar[buf], parity, status);
    if (__syncthreads_or(!ok)) {
      if (tid == 0) {
        mbar_wait(&bar[buf], parity, nullptr);
        if (NBUF == 2 && more) mbar_wait(&bar[buf ^ 1], ((it + 1) >> 1) & 1, nullptr);
      }
      __syncthreads();
      return;
    }
    const int b = tile / tps, t0 = (tile % tps) * kBM;
    unsigned char* rb = raw + buf * CB * kResBox;
    // the residual: this thread's epilogue elements of u (rows m0 + g (+8), columns ni*8 + 2tq (+1))
    uint32_t ures[NT2][2];
#pragma unroll
    for (int ni = 0; ni < NT2; ++ni)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int co = ni * 8 + 2 * tq;
        ures[ni][hf] = *reinterpret_cast<const uint32_t*>(rb + (co / 64) * kResBox +
                                                          sw128(m0 + g + 8 * hf + 2, (co % 64) / 8) + (co % 8) * 2);
      }
    __syncthreads();
    // ELU of the tile in place (an elementwise pass over the swizzled boxes)
    for (int i = tid; i < CB * kResRows * 8; i += kResThreads) {
      const int cb = i / (kResRows * 8), off = (i % (kResRows * 8)) * 16;
      uint4* p = reinterpret_cast<uint4*>(rb + cb * kResBox + off);
      uint4 v = *p;
      v.x = elu2(v.x, lut);
      v.y = elu2(v.y, lut);
      v.z = elu2(v.z, lut);
      v.w = elu2(v.w, lut);
      *p = v;
    }
    __syncthreads();
    if (t0 == 0) {  // rows t = -2, -1: the previous frame's ELU'd history
      for (int i = tid; i < 2 * (COUT / 8); i += kResThreads) {
        const int rr = i / (COUT / 8), c8 = i % (COUT / 8);
        *reinterpret_cast<uint4*>(rb + (c8 / 8) * kResBox + sw128(rr, c8 % 8)) =
            *reinterpret_cast<const uint4*>(hist_in + (int64_t)b * in_row + rr * COUT + c8 * 8);
      }
      __syncthreads();
    }
    // the new history: ELU(u) rows Lo-2 and Lo-1 of this frame
    for (int hr = 0; hr < 2; ++hr) {
      const int t = Lo - 2 + hr;
      if (t < t0 || t >= t0 + kBM) continue;
      bf16* dst = state + (int64_t)slot32[b] * state_row + hist_off + hr * COUT;
      for (int c8 = tid; c8 < COUT / 8; c8 += kResThreads)
        *reinterpret_cast<uint4*>(dst + c8 * 8) =
            *reinterpret_cast<const uint4*>(rb + (c8 / 8) * kResBox + sw128(t - t0 + 2, c8 % 8));
    }
    // GEMM 1: 16 rows x HID over K1 = 3 taps x COUT
    float acc1[NT1][4];
#pragma unroll
    for (int n = 0; n < NT1; ++n) acc1[n][0] = acc1[n][1] = acc1[n][2] = acc1[n][3] = 0.f;
#pragma unroll
    for (int j = 0; j < 3; ++j)
#pragma unroll
      for (int cb = 0; cb < CB; ++cb) {
        const uint32_t eb = smem_u32(rb + cb * kResBox);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4(eb + sw128(m0 + j + (jm & 1) * 8 + (lane & 7), 2 * kk + (jm >> 1)), a0, a1, a2, a3);
#pragma unroll
          for (int nj = 0; nj < NT1 / 2; ++nj) {
            const int n = nj * 16 + ((jm >> 1) << 3) + (lane & 7);
            uint32_t q0, q1, q2, q3;
            ldsm_x4(smem_u32(W1 + n * (K1 + 8) + j * COUT + cb * 64 + kk * 16 + (jm & 1) * 8), q0, q1, q2, q3);
            mma_bf16(acc1[2 * nj], a0, a1, a2, a3, q0, q1);
            mma_bf16(acc1[2 * nj + 1], a0, a1, a2, a3, q2, q3);
          }
        }
      }
    if (NBUF == 1) {  // every warp has read the tile: the buffer takes the next one while this one finishes
      __syncthreads();
      if (tid == 0 && more) issue(tile + gridDim.x, 0);
    }
    // bf16(ELU(bf16(z + b1))) -> the A fragments of GEMM 2 (k = HID)
    uint32_t a2f[HID / 16][4];
#pragma unroll
    for (int kk = 0; kk < HID / 16; ++kk) {
      const float* lo = acc1[2 * kk];
      const float* hi = acc1[2 * kk + 1];
      a2f[kk][0] = elu2(pack_bf2(lo[0] + bias1[kk][0], lo[1] + bias1[kk][1]), lut);
      a2f[kk][1] = elu2(pack_bf2(lo[2] + bias1[kk][0], lo[3] + bias1[kk][1]), lut);
      a2f[kk][2] = elu2(pack_bf2(hi[0] + bias1[kk][2], hi[1] + bias1[kk][3]), lut);
      a2f[kk][3] = elu2(pack_bf2(hi[2] + bias1[kk][2], hi[3] + bias1[kk][3]), lut);
    }
    // GEMM 2: 16 rows x COUT over K = HID, 64 output columns at a time
#pragma unroll
    for (int c = 0; c < NT2 / 8; ++c) {
      float acc2[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) acc2[n][0] = acc2[n][1] = acc2[n][2] = acc2[n][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < HID / 16; ++kk)
#pragma unroll
        for (int nj = 0; nj < 4; ++nj) {
          const int n = c * 64 + nj * 16 + ((jm >> 1) << 3) + (lane & 7);
          uint32_t q0, q1, q2, q3;
          ldsm_x4(smem_u32(W2 + n * (HID + 8) + kk * 16 + (jm & 1) * 8), q0, q1, q2, q3);
          mma_bf16(acc2[2 * nj], a2f[kk][0], a2f[kk][1], a2f[kk][2], a2f[kk][3], q0, q1);
          mma_bf16(acc2[2 * nj + 1], a2f[kk][0], a2f[kk][1], a2f[kk][2], a2f[kk][3], q2, q3);
        }
      // y = bf16(u + bf16(z + b2)); e = bf16(ELU(y))
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int ni = c * 8 + n, co = ni * 8 + 2 * tq;
        const uint32_t bb = b2s[co / 2];
        const float bl = bf_lo_f(bb), bh = bf_hi_f(bb);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int t = t0 + m0 + g + 8 * hf;
          if (t >= Lo) continue;
          const uint32_t uu = ures[ni][hf];
          const uint32_t z = pack_bf2(acc2[n][2 * hf] + bl, acc2[n][2 * hf + 1] + bh);
          uint32_t y;  // bf16 + bf16 rounded once: the same as the fp32 sum rounded to bf16
          asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(y) : "r"(uu), "r"(z));
          *reinterpret_cast<uint32_t*>(e + ((int64_t)b * Lo + t) * COUT + co) = elu2(y, lut);
        }
      }
    }
    if (NBUF == 2) __syncthreads();
  }
}

// ------------------------------------------------------------------------------------------------ final conv
// PCM[t] = bf16(bias + sum_{j<KT, c<64} W[j][c] e[t - (KT-1) + j][c]) on the tensor cores: the tile of 128 + KT-1 rows
// (rows before the stream's start are the stored history) arrives by TMA, the KT taps are row-shifted ldmatrix reads
// of it, and the single output column is the first of an 8-column mma (the weights are the B operand, zero in the
// other columns).  Warp w computes rows 32w .. 32w+31.
__host__ __device__ constexpr uint32_t fin_box(int kt) { return ((128 + kt - 1) * 128 + 1023) / 1024 * 1024; }

template <int KT>
__global__ void __launch_bounds__(128) final_mma_kernel(const __grid_constant__ CUtensorMap xmap,
                                                        const bf16* __restrict__ w, const bf16* __restrict__ bias,
                                                        const bf16* __restrict__ state, int64_t state_row,
                                                        int64_t hist_off, const int* __restrict__ slot32,
                                                        float* __restrict__ pcm, int L, int* status) {
  constexpr int P = KT - 1, KS = KT * 4;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* xs = align1024(smem_raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(xs + fin_box(KT));
  const int b = blockIdx.x, t0 = blockIdx.y * 128;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, tq = lane & 3, jm = lane >> 3;
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    mbar_expect_tx(bar, (128 + P) * 128);
    tma_load_3d(xs, &xmap, 0, t0 - P, b, bar);
  }
  // B fragments (k = tap * 64 + channel, n = output column): column 0 holds the weights
  uint32_t wb[KS][2];
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(w + ks * 16);
    wb[ks][0] = g == 0 ? wp[tq] : 0u;
    wb[ks][1] = g == 0 ? wp[4 + tq] : 0u;
  }
  const float bv = to_f(bias[0]);
  const bool ok = mbar_wait(bar, 0, status);
  if (__syncthreads_or(!ok)) {
    if (tid == 0) mbar_wait(bar, 0, nullptr);
    __syncthreads();
    return;
  }
  if (t0 == 0) {  // rows t = -P .. -1: the stream's history
    const bf16* hist = state + (int64_t)slot32[b] * state_row + hist_off;
    for (int i = tid; i < P * 8; i += 128)
      *reinterpret_cast<uint4*>(xs + sw128(i / 8, i % 8)) = *reinterpret_cast<const uint4*>(hist + i * 8);
    __syncthreads();
  }
  const uint32_t xb = smem_u32(xs);
#pragma unroll
  for (int mi = 0; mi < 2; ++mi) {
    const int m0 = warp * 32 + mi * 16;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const int j = ks >> 2, kk = ks & 3;
      uint32_t a0, a1, a2, a3;
      ldsm_x4(xb + sw128(m0 + j + (jm & 1) * 8 + (lane & 7), 2 * kk + (jm >> 1)), a0, a1, a2, a3);
      mma_bf16(acc, a0, a1, a2, a3, wb[ks][0], wb[ks][1]);
    }
    if (tq == 0) {
      const int ta = t0 + m0 + g, tb = ta + 8;
      if (ta < L) pcm[(int64_t)b * L + ta] = rbf(acc[0] + bv);
      if (tb < L) pcm[(int64_t)b * L + tb] = rbf(acc[2] + bv);
    }
  }
}

// ------------------------------------------------------------------------------------------------ state snapshot
__global__ void state_snapshot_kernel(const bf16* __restrict__ state, int64_t state_row,
                                      const int* __restrict__ slot32, StateCopy c, bf16* __restrict__ snap,
                                      int64_t snap_row) {
  const int b = blockIdx.x;
  const bf16* src = state + (int64_t)slot32[b] * state_row;
  bf16* dst = snap + (int64_t)b * snap_row;
  for (int q = 0; q < c.n; ++q)
    for (int i = threadIdx.x; i < c.len[q] / 8; i += blockDim.x)
      reinterpret_cast<uint4*>(dst + c.dst_off[q])[i] = reinterpret_cast<const uint4*>(src + c.off[q])[i];
}

__global__ void convt_repack_kernel(const bf16* __restrict__ wt, int r, int cout, int cin, bf16* __restrict__ wc) {
  const int n = blockIdx.x;  // jj * cout + o
  const int jj = n / cout, o = n % cout;
  for (int k = threadIdx.x; k < 2 * cin; k += blockDim.x)
    wc[(int64_t)n * 2 * cin + k] =
        k < cin ? wt[((int64_t)(jj + r) * cout + o) * cin + k] : wt[((int64_t)jj * cout + o) * cin + (k - cin)];
}

// ------------------------------------------------------------------------------------------------ host
int launch_convt_repack(const bf16* wt, int r, int cout, int cin, bf16* wc, cudaStream_t s) {
  convt_repack_kernel<<<r * cout, 256, 0, s>>>(wt, r, cout, cin, wc);
  M3_LAUNCHED();
  return M3_OK;
}

int convt_fused_bn(int N) { return convt_bn(N); }
bool convt_persistent_ok(int cin, int cout, int r) {
  const int KT = 2 * cin / 64;
  return convt_fused_ok(cin, cout, r) && (r * cout) % 128 == 0 && (KT == 4 || KT == 8) &&
         convt_pers_smem(128, KT) <= 227 * 1024;
}

bool convt_fused_ok(int cin, int cout, int r) {
  const int N = r * cout, BN = convt_bn(N);
  return cin % 64 == 0 && cout % 32 == 0 && N % BN == 0 && BN % 16 == 0;
}
bool final_fused_ok(int channels, int taps) { return channels == 64 && (taps == 3 || taps == 7); }

int launch_final_fused(const FinalFused& p, int R, cudaStream_t s, int* status) {
  const dim3 grid(R, (p.L + 127) / 128);
  if (p.taps == 3)
    final_mma_kernel<3><<<grid, 128, fin_box(3) + 1024 + 16, s>>>(p.xmap, p.w, p.bias, p.state, p.state_row,
                                                                   p.hist_off, p.slot32, p.pcm, p.L, status);
  else
    final_mma_kernel<7><<<grid, 128, fin_box(7) + 1024 + 16, s>>>(p.xmap, p.w, p.bias, p.state, p.state_row,
                                                                   p.hist_off, p.slot32, p.pcm, p.L, status);
  M3_LAUNCHED();
  return M3_OK;
}

bool res_fused_ok(int cout, int hid) { return (cout == 64 && hid == 32) || (cout == 128 && hid == 64); }

size_t convt_fused_smem(int cin, int cout, int r) {
  (void)cin;
  const int BN = convt_bn(r * cout);
  return 1024 + (size_t)convt_stages(BN) * (kUM * 128 + BN * 128) + 8 * (2 * 3 + 1) + 16;
}
size_t res_fused_smem(int cout, int hid) {
  const int nbuf = cout >= 128 ? 1 : 2;  // ResCfg::NBUF
  return 1024 + nbuf * (size_t)(cout / 64) * kResBox + (size_t)hid * (3 * cout + 8) * 2 +
         (size_t)cout * (hid + 8) * 2 + (size_t)kEluLut * 2 + (size_t)cout * 2 + 16;
}

int seanet_fused_init() {
  int dev = 0;
  M3_CUDA(cudaGetDevice(&dev));
  M3_CUDA(cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev));
  const int big = 227 * 1024;
  M3_CUDA(cudaFuncSetAttribute(convt_umma_kernel<128, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
  M3_CUDA(cudaFuncSetAttribute(convt_pers_kernel<128, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
  M3_CUDA(cudaFuncSetAttribute(convt_pers_kernel<128, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
  M3_CUDA(cudaFuncSetAttribute(convt_umma_kernel<256, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
  M3_CUDA(cudaFuncSetAttribute(res_fused_kernel<64, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
  M3_CUDA(cudaFuncSetAttribute(res_fused_kernel<128, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, big));
  M3_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&g_res_per_sm[0], res_fused_kernel<64, 32>, kResThreads,
                                                        res_fused_smem(64, 32)));
  M3_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&g_res_per_sm[1], res_fused_kernel<128, 64>, kResThreads,
                                                        res_fused_smem(128, 64)));
  if (!g_elu_lut) {
    M3_CUDA(cudaMalloc(&g_elu_lut, kEluLut * sizeof(uint16_t)));
    elu_lut_kernel<<<(kEluLut + 255) / 256, 256>>>(g_elu_lut);
    M3_CUDA(cudaGetLastError());
    M3_CUDA(cudaDeviceSynchronize());
  }
  return M3_OK;
}

int launch_convt_fused(const ConvTFused& p, int R, cudaStream_t s, int* status, int sms) {
  const int N = p.r * p.cout, BN = convt_bn(N), KT = 2 * p.cin / 64;
  const int nsm = sms > 0 && sms < g_sms ? sms : g_sms;
  if (convt_persistent_ok(p.cin, p.cout, p.r)) {  // the persistent, weight-resident form (128-column slices)
    const int NC = N / 128, tiles = R * ((p.L + 1 + kUM - 1) / kUM);
    const int cpc = std::max(1, std::min(tiles, nsm / NC));
    const dim3 grid(NC * cpc);
    if (KT == 4)
      convt_pers_kernel<128, 4><<<grid, kCpThreads, convt_pers_smem(128, 4), s>>>(
          p.amap, p.bmap, p.smap, p.bias, p.tail_in, p.in_row, p.state, p.state_row, p.tail_off, p.slot32, p.u, p.L,
          p.r, p.cin, p.cout, R, status);
    else
      convt_pers_kernel<128, 8><<<grid, kCpThreads, convt_pers_smem(128, 8), s>>>(
          p.amap, p.bmap, p.smap, p.bias, p.tail_in, p.in_row, p.state, p.state_row, p.tail_off, p.slot32, p.u, p.L,
          p.r, p.cin, p.cout, R, status);
    M3_LAUNCHED();
    return M3_OK;
  }
  const dim3 grid(N / BN, (p.L + 1 + kUM - 1) / kUM, R);
  const size_t smem = convt_fused_smem(p.cin, p.cout, p.r);
  if (BN == 256)
    convt_umma_kernel<256, 2><<<grid, 128, smem, s>>>(p.amap, p.bmap, p.bias, p.tail_in, p.in_row, p.state,
                                                      p.state_row, p.tail_off, p.slot32, p.u, p.L, p.r, p.cin, p.cout,
                                                      status);
  else if (BN == 128)
    convt_umma_kernel<128, 3><<<grid, 128, smem, s>>>(p.amap, p.bmap, p.bias, p.tail_in, p.in_row, p.state,
                                                      p.state_row, p.tail_off, p.slot32, p.u, p.L, p.r, p.cin, p.cout,
                                                      status);
  else
    M3_REQUIRE(false, M3_ERR_UNSUPPORTED, "transposed conv of %d columns has no fused form", N);
  M3_LAUNCHED();
  return M3_OK;
}

int launch_res_fused(const ResFused& p, int R, cudaStream_t s, int* status, int sms) {
  const int nsm = sms > 0 && sms < g_sms ? sms : g_sms;
  const int tiles = R * ((p.Lo + kBM - 1) / kBM);
  const size_t smem = res_fused_smem(p.cout, p.hid);
  const int per_sm = std::max(1, p.cout == 64 ? g_res_per_sm[0] : g_res_per_sm[1]);
  const dim3 grid(std::max(1, std::min(tiles, nsm * per_sm)));
  if (p.cout == 64)
    res_fused_kernel<64, 32><<<grid, kResThreads, smem, s>>>(p.umap, p.w1, p.b1, p.w2, p.b2, p.hist_in, p.in_row, p.state,
                                                     p.state_row, p.hist_off, p.slot32, p.e, p.Lo, R, g_elu_lut, status);
  else
    res_fused_kernel<128, 64><<<grid, kResThreads, smem, s>>>(p.umap, p.w1, p.b1, p.w2, p.b2, p.hist_in, p.in_row, p.state,
                                                      p.state_row, p.hist_off, p.slot32, p.e, p.Lo, R, g_elu_lut, status);
  M3_LAUNCHED();
  return M3_OK;
}

int launch_state_snapshot(const bf16* state, int64_t state_row, const int* slot32, int R, const StateCopy& c,
                          bf16* snap, int64_t snap_row, cudaStream_t s) {
  if (R <= 0 || c.n == 0) return M3_OK;
  state_snapshot_kernel<<<R, 128, 0, s>>>(state, state_row, slot32, c, snap, snap_row);
  M3_LAUNCHED();
  return M3_OK;
}

}  // namespace m3
