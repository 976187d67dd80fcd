// Qwen3 backbone decode over the static per-seat KV cache (replaces serve/fast_backbone.py StaticBackbone).
//
// Per layer: [add+]RMSNorm -> QKV linear -> q/k head RMSNorm + RoPE + K/V cache write -> split-KV decode attention
// -> combine -> o linear -> add+RMSNorm -> gate|up linear -> SiLU*up -> down linear.  The rounding points follow
// the reference's fused path (fuse_rope=True): every stored intermediate is bf16, arithmetic is fp32.
#include <algorithm>
#include <vector>

#include "common.cuh"
#include "mma.cuh"
#include "tma.cuh"
#include "gemm.cuh"

namespace m3 {

constexpr int kHeadDim = 128;

// ------------------------------------------------------------------------------------------------ row setup
// slot and position of every row, validated once per step (pos = lengths[slot] + offset, read before the step's
// length update as serve/fast_backbone.py:178-179), and the work list of the attention.  A decode row is one entry.
// The rows of an inline prompt (consecutive rows of one slot at offsets 0..P-1, as the step lays them out) go in
// groups of `rg` consecutive positions, one entry per group: a group's CTA reads the keys up to its last position once
// for all of its rows instead of once per row.  Entries are written as visit[i] = {first row, slot, last position,
// rows}; the rows of a group after its first get {row, slot, 0, 0} (nothing to do).  The attention visits entries
// longest first (last position descending, then row), so the CTAs with the most keys start first and the short ones
// fill the last wave.  With `sort` the grid is one CTA of a power of two >= rows threads (<= 1024): entries that
// already come longest first keep the identity order after one block vote, others are sorted in shared memory
// (bitonic); without `sort` the order is the identity.
constexpr int kSortRows = 1024;

// rows of the entry starting at row r (0: r is inside a group) and its last position
__device__ __forceinline__ int entry_rows(const int64_t* __restrict__ slots, const int64_t* __restrict__ offsets,
                                          int rows, int r, int rg) {
  if (!offsets) return 1;
  const int64_t o = offsets[r];
  const bool prompt = o > 0 || (r + 1 < rows && offsets[r + 1] == 1 && slots[r + 1] == slots[r]);
  if (!prompt) return 1;
  if (o % rg != 0) return 0;
  int n = 1;
  while (n < rg && r + n < rows && slots[r + n] == slots[r] && offsets[r + n] == o + n) ++n;
  return n;
}

__global__ void prep_rows_kernel(const int64_t* __restrict__ slots, const int64_t* __restrict__ offsets,
                                 const int64_t* __restrict__ lengths, int rows, int max_slots, int capacity, int rg,
                                 int* __restrict__ slot32, int* __restrict__ pos32, int4* __restrict__ visit,
                                 int sort, int* status) {
  __shared__ uint64_t key[kSortRows];
  __shared__ int slot_of[kSortRows];
  __shared__ int rows_of[kSortRows];
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  int64_t p = 0;
  int sl = 0, nr = 0, last = 0;
  if (r < rows) {
    int64_t s = slots[r];
    if (s < 0 || s > max_slots) {
      report(status, M3_DEV_BAD_SLOT);
      s = max_slots;
    }
    p = lengths[s] + (offsets ? offsets[r] : 0);
    if (p < 0 || p >= capacity) {
      report(status, M3_DEV_BAD_POS);
      p = p < 0 ? 0 : capacity - 1;
    }
    sl = (int)s;
    slot32[r] = sl;
    pos32[r] = (int)p;
    nr = entry_rows(slots, offsets, rows, r, rg);
    last = nr > 0 ? (int)min(p + nr - 1, (int64_t)capacity - 1) : 0;
  }
  if (!sort) {
    if (r < rows) visit[r] = make_int4(r, sl, last, nr);
    return;
  }
  // one CTA, n = blockDim.x: keys (last position << 32 | 0x7FFFFFFF - row) sorted descending; group members and
  // padding keys are 0, so they come last
  const int t = threadIdx.x, n = blockDim.x;
  key[t] = t < rows && nr > 0 ? ((uint64_t)(uint32_t)last << 32) | (uint32_t)(0x7FFFFFFF - t) : 0ull;
  slot_of[t] = sl;
  rows_of[t] = nr;
  __syncthreads();
  if (__syncthreads_and(t + 1 >= rows || key[t] > key[t + 1] || (key[t] == 0 && key[t + 1] == 0))) {
    if (t < rows) visit[t] = make_int4(t, sl, last, nr);   // already in order
    return;
  }
  for (int k = 2; k <= n; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      const int o = t ^ j;
      if (o > t) {
        const uint64_t a = key[t], b = key[o];
        if (((t & k) == 0) == (a < b)) {  // descending within blocks whose bit k is clear, ascending elsewhere
          key[t] = b;
          key[o] = a;
        }
      }
      __syncthreads();
    }
  if (t < rows) {
    if (key[t] == 0) {
      visit[t] = make_int4(0, 0, 0, 0);                   // a group member or padding: no work
    } else {
      const int o = 0x7FFFFFFF - (int)(uint32_t)key[t];
      visit[t] = make_int4(o, slot_of[o], (int)(key[t] >> 32), rows_of[o]);
    }
  }
}

int launch_prep_rows(const int64_t* slots, const int64_t* offsets, const int64_t* lengths, int rows, int max_slots,
                     int capacity, int rg, int* slot32, int* pos32, int4* visit, int* status, cudaStream_t s) {
  if (rows <= kSortRows) {
    int n = 32;
    while (n < rows) n <<= 1;
    prep_rows_kernel<<<1, n, 0, s>>>(slots, offsets, lengths, rows, max_slots, capacity, rg, slot32, pos32, visit, 1,
                                     status);
  } else {
    prep_rows_kernel<<<cdiv(rows, 128), 128, 0, s>>>(slots, offsets, lengths, rows, max_slots, capacity, rg, slot32,
                                                     pos32, visit, 0, status);
  }
  M3_LAUNCHED();
  return M3_OK;
}

// lengths.index_add_(0, slots, real) (serve/fast_backbone.py:233); prefill rows of one slot all add.
__global__ void lengths_add_kernel(const int* __restrict__ slot32, const int64_t* __restrict__ real, int rows,
                                   int64_t* __restrict__ lengths) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const int64_t v = real ? real[r] : 1;
  if (v) atomicAdd(reinterpret_cast<unsigned long long*>(lengths + slot32[r]), (unsigned long long)v);
}

// ------------------------------------------------------------------------------------------------ norms
// h' = bf16(h + a) (stored to hout) when a != nullptr, else h' = h;  y = bf16(w * bf16(h' / rms(h'))).
// serve/fast_backbone.py:96-104 (_add_rms) and HF Qwen3RMSNorm.  One CTA per row, 8 elements per thread-step.
__global__ void add_rms_kernel(const bf16* __restrict__ hin, const bf16* __restrict__ a, bf16* __restrict__ hout,
                               bf16* __restrict__ y, const bf16* __restrict__ w, float eps, int n) {
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int nv = n / 8;
  const uint4* hp = reinterpret_cast<const uint4*>(hin + (int64_t)row * n);
  const uint4* ap = a ? reinterpret_cast<const uint4*>(a + (int64_t)row * n) : nullptr;
  constexpr int kMaxPer = 4;  // up to 4 * 8 * blockDim elements per row held in registers
  float v[kMaxPer][8];
  float ss = 0.f;
#pragma unroll
  for (int it = 0; it < kMaxPer; ++it) {
    const int c = threadIdx.x + it * blockDim.x;
    if (c < nv) {
      unpack8(hp[c], v[it]);
      if (ap) {
        float av[8];
        unpack8(ap[c], av);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[it][e] = rbf(v[it][e] + av[e]);
      }
      if (hout) reinterpret_cast<uint4*>(hout + (int64_t)row * n)[c] = ap ? pack8(v[it]) : hp[c];
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(v[it][e], v[it][e], ss);
    }
  }
  ss = block_sum(ss, red);
  const float inv = 1.f / sqrtf(ss / (float)n + eps);
  const uint4* wp = reinterpret_cast<const uint4*>(w);
#pragma unroll
  for (int it = 0; it < kMaxPer; ++it) {
    const int c = threadIdx.x + it * blockDim.x;
    if (c < nv) {
      float wv[8], o[8];
      unpack8(wp[c], wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = rbf(v[it][e] * inv) * wv[e];
      reinterpret_cast<uint4*>(y + (int64_t)row * n)[c] = pack8(o);
    }
  }
}

int launch_add_rms(int rows, const bf16* hin, const bf16* a, bf16* hout, bf16* y, const bf16* w, float eps, int n,
                   cudaStream_t s) {
  add_rms_kernel<<<rows, std::min(1024, std::max(32, (n / 8 + 31) / 32 * 32)), 0, s>>>(hin, a, hout, y, w, eps, n);
  M3_LAUNCHED();
  return M3_OK;
}

// ------------------------------------------------------------------------------------------------ q/k norm + RoPE
// One warp per (row, head): heads [0, H) are query heads written to q; heads [H, H + KV) are key heads written to
// the K cache at (slot, kv head, pos) together with the matching value head (serve/fast_backbone.py:62-92).
// Lane l owns dims (2l, 2l+1) of the first half and (64+2l, 64+2l+1) of the second half (rotate-half pairs).
__global__ void qk_rope_cache_kernel(const bf16* __restrict__ qkv, bf16* __restrict__ q, bf16* __restrict__ kc,
                                     bf16* __restrict__ vc, int64_t slot_stride, int64_t head_stride,
                                     const int* __restrict__ slot32, const int* __restrict__ pos32,
                                     const bf16* __restrict__ cos, const bf16* __restrict__ sin,
                                     const bf16* __restrict__ wq, const bf16* __restrict__ wk, float eps, int H,
                                     int KV) {
  const int row = blockIdx.x;
  const int head = blockIdx.y * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (head >= H + KV) return;
  const int pos = pos32[row];
  const int D = kHeadDim, half = D / 2;
  const int64_t width = (int64_t)(H + 2 * KV) * D;
  const bf16* src = qkv + row * width + (int64_t)head * D;
  const int d1 = 2 * lane, d2 = half + 2 * lane;
  const float2 x1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + d1));
  const float2 x2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + d2));
  float ss = x1.x * x1.x + x1.y * x1.y + x2.x * x2.x + x2.y * x2.y;
  ss = warp_sum(ss);
  const float inv = 1.f / sqrtf(ss / (float)D + eps);
  const bf16* w = head < H ? wq : wk;
  const float2 w1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(w + d1));
  const float2 w2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(w + d2));
  const float y1a = rbf(rbf(x1.x * inv) * w1.x), y1b = rbf(rbf(x1.y * inv) * w1.y);
  const float y2a = rbf(rbf(x2.x * inv) * w2.x), y2b = rbf(rbf(x2.y * inv) * w2.y);
  const bf16* cr = cos + (int64_t)pos * D;
  const bf16* sr = sin + (int64_t)pos * D;
  const float2 c1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(cr + d1));
  const float2 c2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(cr + d2));
  const float2 s1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(sr + d1));
  const float2 s2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(sr + d2));
  const float o1a = y1a * c1.x - y2a * s1.x, o1b = y1b * c1.y - y2b * s1.y;
  const float o2a = y2a * c2.x + y1a * s2.x, o2b = y2b * c2.y + y1b * s2.y;
  bf16* dst;
  if (head < H) {
    dst = q + ((int64_t)row * H + head) * D;
  } else {
    const int kh = head - H;
    const int64_t off = (int64_t)slot32[row] * slot_stride + (int64_t)kh * head_stride + (int64_t)pos * D;
    dst = kc + off;
    const bf16* vsrc = qkv + row * width + (int64_t)(H + KV + kh) * D;
    *reinterpret_cast<uint32_t*>(vc + off + d1) = *reinterpret_cast<const uint32_t*>(vsrc + d1);
    *reinterpret_cast<uint32_t*>(vc + off + d2) = *reinterpret_cast<const uint32_t*>(vsrc + d2);
  }
  *reinterpret_cast<uint32_t*>(dst + d1) = pack2(o1a, o1b);
  *reinterpret_cast<uint32_t*>(dst + d2) = pack2(o2a, o2b);
}

// ------------------------------------------------------------------------------------------------ SwiGLU
// act = bf16(bf16(silu(g)) * u)  (F.silu(g_) * u_ in bf16, serve/fast_backbone.py:201-202).
__global__ void silu_mul_kernel(const bf16* __restrict__ gu, bf16* __restrict__ act, int rows, int F) {
  const int fv = F / 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)rows * fv) return;
  const int64_t r = i / fv, c = i % fv;
  float g[8], u[8], o[8];
  unpack8(reinterpret_cast<const uint4*>(gu + r * 2 * F)[c], g);
  unpack8(reinterpret_cast<const uint4*>(gu + r * 2 * F + F)[c], u);
#pragma unroll
  for (int e = 0; e < 8; ++e) o[e] = rbf(silu_mul1(g[e], u[e]));
  reinterpret_cast<uint4*>(act + r * F)[c] = pack8(o);
}

// ------------------------------------------------------------------------------------------------ attention
// Split-KV decode attention over the static cache (replaces _decode_attn, serve/fast_backbone.py:32-58).
//
// Grid (split, kv head, row).  A CTA owns keys [split*chunk, min((split+1)*chunk, pos+1)) of one (row, kv head)
// and serves all G query heads of that kv head, so every K/V byte is read from HBM once.  Online softmax in the
// exp2 domain with a running max that is only raised when a new score exceeds it by more than 2^8 (the result is
// exact: the same reference max is used for every term of a split).  Splits are merged in the same launch: a row
// whose keys fit one split writes its bf16 output directly; otherwise each CTA publishes (O, m, l) in fp32, and the
// last CTA of the (row, kv head) to take an atomic ticket merges them and re-arms the ticket.
constexpr int kAttnThreads = 128;
constexpr float kLazyRescale = 8.f;

// Final step of a split CTA, thread tid owning head dim tid of the G query heads: (Og, Mg, Lg) is the CTA's
// unnormalised output, running max (exp2 domain) and softmax denominator.  A row whose keys fit one split (n == 1)
// writes bf16(O / L) directly.  Otherwise the CTA publishes its fp32 partial, takes a ticket on its (row, kv head),
// and the last of the n CTAs merges all of them, out = sum_s O_s 2^(m_s - M) / sum_s L_s 2^(m_s - M) with
// M = max_s m_s, and re-arms the ticket for the next launch on the stream.
template <int G>
__device__ __forceinline__ void split_epilogue(const float (&Og)[G], const float (&Mg)[G], const float (&Lg)[G],
                                               int tid, int row, int kvh, int KV, int split, int nsplit, int n,
                                               float* __restrict__ part_o, float2* __restrict__ part_ml,
                                               int* __restrict__ tickets, bf16* __restrict__ out, int H, int* last) {
  bf16* orow = out + ((int64_t)row * H + kvh * G) * kHeadDim;
  if (n == 1) {
#pragma unroll
    for (int g = 0; g < G; ++g) orow[g * kHeadDim + tid] = to_bf(Lg[g] > 0.f ? Og[g] / Lg[g] : 0.f);
    return;
  }
  const int64_t rk = (int64_t)row * KV + kvh;
  const int64_t pidx = rk * nsplit + split;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    part_o[(pidx * G + g) * kHeadDim + tid] = Og[g];
    if (tid == 0) part_ml[pidx * G + g] = make_float2(Mg[g], Lg[g]);
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();  // release: the whole CTA's partial (ordered before this thread by the barrier)
    const int prev = atomicAdd(&tickets[rk], 1);
    __threadfence();  // acquire: the other CTAs' partials, for the merge below
    *last = prev == n - 1;
  }
  __syncthreads();
  if (!*last) return;
  const int64_t pbase = rk * nsplit;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float M = -INFINITY;
    for (int s = 0; s < n; ++s) M = fmaxf(M, __ldcg(&part_ml[(pbase + s) * G + g]).x);
    float O = 0.f, L = 0.f;
    if (M != -INFINITY)
      for (int s = 0; s < n; ++s) {
        const float2 ml = __ldcg(&part_ml[(pbase + s) * G + g]);
        const float sc = ml.x == -INFINITY ? 0.f : exp2f(ml.x - M);
        O = fmaf(__ldcg(&part_o[((pbase + s) * G + g) * kHeadDim + tid]), sc, O);
        L = fmaf(ml.y, sc, L);
      }
    orow[g * kHeadDim + tid] = to_bf(L > 0.f ? O / L : 0.f);
  }
  if (tid == 0) tickets[rk] = 0;
}

// The dot products run on the tensor cores (mma.sync m16n8k16, bf16 operands, fp32 accumulation; the operands are
// exact bf16 values, so only the summation order differs from fp32 FMAs: the reference's kernel is scalar fp32).
// K and V arrive by TMA through per-layer tensor maps over the cache [slot * kv_heads + head][position][128]: a
// 16-token block is four 2 KB boxes (K and V, dims 0-63 and 64-127), 128-byte swizzled so that ldmatrix reads them
// without bank conflicts.  Each of the 4 warps owns every 4th block of the CTA's chunk and its own kMmaStages-deep
// ring (no CTA-wide barrier in the loop).  A CTA serves one work entry: the G query heads of a decode row, or those
// of `rows` consecutive positions of an inline prompt (rows x G <= 16 query vectors, the 16 rows of the mma tile),
// whose keys it then reads once for all of them.  Query vector v = j G + h (row j of the entry, head kv_head G + h)
// sits in mma row v.  Per block:
//   S   = Q K^T       A = Q (the entry's query vectors, rest zero), B = K rows via ldmatrix           (16 mma)
//   P   = 2^(S*scale - m) per query vector with its lazily raised running max m, masked past its own position
//   O^T += V^T P^T    A = V^T via ldmatrix.trans, B = P^T straight from the S accumulators (query vectors 0-7, and
//                     8-15 in a second tile when the entry has more), P split into bf16 hi + lo parts so that the
//                     weights keep ~16 mantissa bits (the reference keeps them in fp32)
// V rows past the entry's last key are zeroed in shared memory before use (0 * stale data must stay 0).
constexpr int kBlkTok = 16;
constexpr int kMmaStages = 2;
constexpr int kBoxBytes = kBlkTok * 128;   // 16 positions x 64 dims x bf16
constexpr int kBlkBytes = 4 * kBoxBytes;   // K lo, K hi, V lo, V hi
constexpr int kQueryVectors = 16;          // the mma tile's rows: query vectors per CTA
constexpr uint32_t kSelftestPolls = 1000;  // m3_backbone_attention_selftest: polls before a wait gives up

struct MmaAttnSmem {
  unsigned char stage[4][kMmaStages][kBlkBytes];  // [warp][stage], every box 1024-byte aligned
  uint64_t bar[4][kMmaStages];
  int last;
};
constexpr int kMmaAttnSmemBytes = (int)sizeof(MmaAttnSmem) + 1024;  // + alignment slack
static_assert(kMmaStages * kBlkBytes >= (kQueryVectors * kHeadDim + 2 * kQueryVectors) * 4,
              "a warp's partial (O and m, l of 16 query vectors) fits in its stage buffers");

// One work entry (GROUP: a prompt group of nrows rows; else a decode row, whose arithmetic then has no trace of the
// group path).
template <int G, bool GROUP>
__device__ __forceinline__ void attn_entry(MmaAttnSmem& sm, const CUtensorMap* kmap, const CUtensorMap* vmap,
                                           const bf16* __restrict__ q, const int4 vis, float* __restrict__ part_o,
                                           float2* __restrict__ part_ml, int* __restrict__ tickets,
                                           bf16* __restrict__ out, int nsplit, int chunk, int H, float qscale,
                                           int* status, int extra_tx) {
  const int nrows = GROUP ? vis.w : 1;
  const int split = blockIdx.x, kvh = blockIdx.y, row = vis.x;
  const int KV = gridDim.y;
  const int pos = vis.z;
  if (GROUP && split > 0) return;      // a prompt group reads all of its keys in one CTA
  const int t0 = GROUP ? 0 : split * chunk;
  if (t0 > pos) return;
  const int ntok = GROUP ? pos + 1 : min(chunk, pos + 1 - t0);
  const int nblk = cdiv(ntok, kBlkTok);
  const int QV = nrows * G;
  const int first = pos - (nrows - 1);  // position of the entry's first row
  const bool hi = GROUP && QV > 8;      // query vectors 8-15 present (uniform over the CTA)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int zc = vis.y * KV + kvh;
  const int nmine = warp < nblk ? (nblk - 1 - warp) / 4 + 1 : 0;  // blocks warp, warp + 4, ...
  const uint32_t polls = extra_tx ? kSelftestPolls : kSpinLimit;  // the self-test's waits give up sooner

  if (tid == 0) {
    for (int w = 0; w < 4; ++w)
      for (int st = 0; st < kMmaStages; ++st) mbar_init(&sm.bar[w][st], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int i) {  // lane 0: this warp's i-th block into stage i % kMmaStages
    unsigned char* st = sm.stage[warp][i % kMmaStages];
    uint64_t* bar = &sm.bar[warp][i % kMmaStages];
    const int y = t0 + (warp + 4 * i) * kBlkTok;
    mbar_expect_tx(bar, kBlkBytes + extra_tx);
    tma_load_3d(st, kmap, 0, y, zc, bar);
    tma_load_3d(st + kBoxBytes, kmap, 64, y, zc, bar);
    tma_load_3d(st + 2 * kBoxBytes, vmap, 0, y, zc, bar);
    tma_load_3d(st + 3 * kBoxBytes, vmap, 64, y, zc, bar);
  };
  if (lane == 0)
    for (int i = 0; i < min(kMmaStages, nmine); ++i) issue(i);

  // A fragments of Q: this lane holds mma rows g (a0, a2) and g + 8 (a1, a3), dims 16ks + 2t (+8); rows >= QV zero
  uint32_t qa[8][4];
  {
    const int v0 = min(g, QV - 1), v1 = min(g + 8, QV - 1);
    const uint32_t* qp0 =
        reinterpret_cast<const uint32_t*>(q + ((int64_t)(row + v0 / G) * H + kvh * G + v0 % G) * kHeadDim);
    const uint32_t* qp1 =
        reinterpret_cast<const uint32_t*>(q + ((int64_t)(row + v1 / G) * H + kvh * G + v1 % G) * kHeadDim);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      qa[ks][0] = g < QV ? qp0[8 * ks + t] : 0u;
      qa[ks][1] = GROUP && g + 8 < QV ? qp1[8 * ks + t] : 0u;
      qa[ks][2] = g < QV ? qp0[8 * ks + 4 + t] : 0u;
      qa[ks][3] = GROUP && g + 8 < QV ? qp1[8 * ks + 4 + t] : 0u;
    }
  }
  // O^T tiles: o[mt] = rows (dims) 16mt + g, 16mt + 8 + g; columns query vectors 2t, 2t + 1 (o2: 8 + 2t, 8 + 2t + 1)
  float o[8][4], o2[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[mt][e] = o2[mt][e] = 0.f;
  // running max and denominator of query vectors g and g + 8, identical in the 4 lanes of quad g
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const int lim0 = first + g / G, lim1 = first + (g + 8) / G;  // the last key each of the two may see
  bool timed_out = false;
  int i = 0;
  for (; i < nmine; ++i) {
    const int stg = i % kMmaStages;
    const bool got = mbar_wait(&sm.bar[warp][stg], (i / kMmaStages) & 1, status, polls);
    if (!__all_sync(0xffffffffu, got)) {
      timed_out = true;
      break;
    }
    unsigned char* st = sm.stage[warp][stg];
    const int b = warp + 4 * i;
    const int nv = min(kBlkTok, ntok - b * kBlkTok);
    if (nv < kBlkTok) {  // zero V rows nv..15 of both boxes
      uint4* v4 = reinterpret_cast<uint4*>(st + 2 * kBoxBytes);
      for (int e = lane; e < 2 * kBlkTok * 8; e += 32)
        if (((e >> 3) & (kBlkTok - 1)) >= nv) v4[e] = make_uint4(0u, 0u, 0u, 0u);
      __syncwarp();
    }
    const uint32_t kb = smem_u32(st), vb = kb + 2 * kBoxBytes;
    const int j = lane >> 3;                           // ldmatrix: this lane addresses row (lane & 7) of matrix j
    const int lr = ((j >> 1) << 3) + (lane & 7), lc = j & 1;
    // S = Q K^T over 16 positions: s[nt] = rows g (c0, c1) and g + 8 (c2, c3) at positions nt*8 + 2t, +1
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t k0, k1, k2, k3;
      ldsm_x4(kb + (ks >> 2) * kBoxBytes + sw128(lr, ((ks & 3) << 1) + lc), k0, k1, k2, k3);
      if constexpr (GROUP) {
        mma_bf16(s[0], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], k0, k1);
        mma_bf16(s[1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], k2, k3);
      } else {
        mma_bf16(s[0], qa[ks][0], 0u, qa[ks][2], 0u, k0, k1);
        mma_bf16(s[1], qa[ks][0], 0u, qa[ks][2], 0u, k2, k3);
      }
    }
    float p[2][4];
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kr = b * kBlkTok + nt * 8 + 2 * t + e;  // key index in the CTA's range
        const bool in = kr < ntok;
        const bool ok0 = g < QV && in && (!GROUP || t0 + kr <= lim0);
        p[nt][e] = ok0 ? s[nt][e] * qscale : -INFINITY;
        mx0 = fmaxf(mx0, p[nt][e]);
        if constexpr (GROUP) {
          const bool ok1 = g + 8 < QV && in && t0 + kr <= lim1;
          p[nt][2 + e] = ok1 ? s[nt][2 + e] * qscale : -INFINITY;
          mx1 = fmaxf(mx1, p[nt][2 + e]);
        }
      }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    float r0 = 1.f, r1 = 1.f;
    if (mx0 > m_run[0] + kLazyRescale) {
      r0 = exp2f(m_run[0] - mx0);
      m_run[0] = mx0;
      l_run[0] *= r0;
    }
    if constexpr (GROUP) {
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      if (mx1 > m_run[1] + kLazyRescale) {
        r1 = exp2f(m_run[1] - mx1);
        m_run[1] = mx1;
        l_run[1] *= r1;
      }
    }
    if (__any_sync(0xffffffffu, r0 != 1.f)) {  // O^T column v lives in the lanes with t = v / 2
      const float ra = __shfl_sync(0xffffffffu, r0, 8 * t), rb = __shfl_sync(0xffffffffu, r0, 8 * t + 4);
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= ra;
        o[mt][1] *= rb;
        o[mt][2] *= ra;
        o[mt][3] *= rb;
      }
    }
    if (hi && __any_sync(0xffffffffu, r1 != 1.f)) {
      const float ra = __shfl_sync(0xffffffffu, r1, 8 * t), rb = __shfl_sync(0xffffffffu, r1, 8 * t + 4);
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        o2[mt][0] *= ra;
        o2[mt][1] *= rb;
        o2[mt][2] *= ra;
        o2[mt][3] *= rb;
      }
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        p[nt][e] = p[nt][e] == -INFINITY ? 0.f : exp2f(p[nt][e] - m_run[0]);
        l_run[0] += p[nt][e];
        if constexpr (GROUP) {
          p[nt][2 + e] = p[nt][2 + e] == -INFINITY ? 0.f : exp2f(p[nt][2 + e] - m_run[1]);
          l_run[1] += p[nt][2 + e];
        }
      }
    const uint32_t h0 = pack_bf2(p[0][0], p[0][1]), h1 = pack_bf2(p[1][0], p[1][1]);
    const uint32_t l0 = pack_bf2(p[0][0] - bf_lo_f(h0), p[0][1] - bf_hi_f(h0));
    const uint32_t l1 = pack_bf2(p[1][0] - bf_lo_f(h1), p[1][1] - bf_hi_f(h1));
    uint32_t h2 = 0u, h3 = 0u, l2 = 0u, l3 = 0u;
    if constexpr (GROUP) {
      h2 = pack_bf2(p[0][2], p[0][3]);
      h3 = pack_bf2(p[1][2], p[1][3]);
      l2 = pack_bf2(p[0][2] - bf_lo_f(h2), p[0][3] - bf_hi_f(h2));
      l3 = pack_bf2(p[1][2] - bf_lo_f(h3), p[1][3] - bf_hi_f(h3));
    }
    // O^T += V^T P^T: per 16 dims, A = V^T (ldmatrix.trans of the V rows), B = P^T of quad g (rows g, then g + 8)
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4_t(vb + (mt >> 2) * kBoxBytes + sw128(lr, ((mt & 3) << 1) + lc), a0, a1, a2, a3);
      mma_bf16(o[mt], a0, a1, a2, a3, h0, h1);
      mma_bf16(o[mt], a0, a1, a2, a3, l0, l1);
      if (hi) {
        mma_bf16(o2[mt], a0, a1, a2, a3, h2, h3);
        mma_bf16(o2[mt], a0, a1, a2, a3, l2, l3);
      }
    }
    __syncwarp();
    if (lane == 0 && i + kMmaStages < nmine) issue(i + kMmaStages);
  }
  if (timed_out) {  // drain this warp's copies still in flight (bounded) before its buffers are reused
    if (lane == 0)
      for (int k = i; k < min(nmine, i + kMmaStages); ++k)
        mbar_wait(&sm.bar[warp][k % kMmaStages], (k / kMmaStages) & 1, nullptr, polls);
    __syncwarp();
#pragma unroll
    for (int mt = 0; mt < 8; ++mt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[mt][e] = o2[mt][e] = 0.f;
    m_run[0] = m_run[1] = -INFINITY;
    l_run[0] = l_run[1] = 0.f;
  }
#pragma unroll
  for (int h = 0; h < (GROUP ? 2 : 1); ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 1);
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 2);
  }
  // the warp's partial, in its own (now idle) stage buffers: wo[16][128], wml[16][2]
  float* wo = reinterpret_cast<float*>(sm.stage[warp][0]);
  float* wml = wo + kQueryVectors * kHeadDim;
#pragma unroll
  for (int mt = 0; mt < 8; ++mt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int v = 2 * t + (e & 1), dim = 16 * mt + g + ((e >> 1) << 3);
      if (v < QV) wo[v * kHeadDim + dim] = o[mt][e];
      if (hi && 8 + v < QV) wo[(8 + v) * kHeadDim + dim] = o2[mt][e];
    }
  if (t == 0) {
    if (g < QV) {
      wml[g * 2] = m_run[0];
      wml[g * 2 + 1] = l_run[0];
    }
    if (GROUP && g + 8 < QV) {
      wml[(g + 8) * 2] = m_run[1];
      wml[(g + 8) * 2 + 1] = l_run[1];
    }
  }
  __syncthreads();
  auto merged = [&](int v, float& O, float& M, float& L) {  // the 4 warps' partials of query vector v, dim tid
    M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w)
      M = fmaxf(M, reinterpret_cast<const float*>(sm.stage[w][0])[kQueryVectors * kHeadDim + v * 2]);
    O = 0.f;
    L = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float* ww = reinterpret_cast<const float*>(sm.stage[w][0]);
      const float mw = ww[kQueryVectors * kHeadDim + v * 2];
      const float sc = mw == -INFINITY ? 0.f : exp2f(mw - M);
      O = fmaf(ww[v * kHeadDim + tid], sc, O);
      L = fmaf(ww[kQueryVectors * kHeadDim + v * 2 + 1], sc, L);
    }
  };
  if constexpr (!GROUP) {
    float Og[G], Mg[G], Lg[G];
#pragma unroll
    for (int gg = 0; gg < G; ++gg) merged(gg, Og[gg], Mg[gg], Lg[gg]);
    split_epilogue<G>(Og, Mg, Lg, tid, row, kvh, KV, split, nsplit, min(nsplit, pos / chunk + 1), part_o, part_ml,
                      tickets, out, H, &sm.last);
  } else {  // one split: every query vector's output directly
    for (int v = 0; v < QV; ++v) {
      float O, M, L;
      merged(v, O, M, L);
      out[((int64_t)(row + v / G) * H + kvh * G + v % G) * kHeadDim + tid] = to_bf(L > 0.f ? O / L : 0.f);
    }
  }
}

template <int G>
__global__ void __launch_bounds__(kAttnThreads) attn_mma_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, const bf16* __restrict__ q,
    const int4* __restrict__ visit,
    float* __restrict__ part_o, float2* __restrict__ part_ml, int* __restrict__ tickets, bf16* __restrict__ out,
    int nsplit, int chunk, int H, float qscale, int* status, int extra_tx) {
  static_assert(G <= 8 && kQueryVectors % G == 0, "the query heads of one kv head fill at most 8 of the 16 mma rows");
  extern __shared__ unsigned char smem_raw[];
  MmaAttnSmem& sm =
      *reinterpret_cast<MmaAttnSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int4 vis = visit[blockIdx.z];  // {first row, slot, last position, rows}
  if (vis.w == 0) return;              // inside a prompt group: the group's first row carries the work
  if (vis.w > 1)
    attn_entry<G, true>(sm, &kmap, &vmap, q, vis, part_o, part_ml, tickets, out, nsplit, chunk, H, qscale, status,
                        extra_tx);
  else
    attn_entry<G, false>(sm, &kmap, &vmap, q, vis, part_o, part_ml, tickets, out, nsplit, chunk, H, qscale, status,
                         extra_tx);
}

}  // namespace m3

// ================================================================================================ handle
using namespace m3;

struct m3_backbone {
  m3_backbone_config c{};
  std::vector<const bf16*> in_norm, wqkv, q_norm, k_norm, wo, post_norm, wgu, wdown;
  std::vector<bf16*> kc, vc;
  bf16** caches = nullptr;  // device [layers * 2]: layer i's K cache at 2i, V cache at 2i + 1 (prefix copies)
  const bf16* final_norm = nullptr;
  const bf16* cos = nullptr;
  const bf16* sin = nullptr;
  int64_t* lengths = nullptr;
  int max_split = 16;
  // scratch
  void* ws = nullptr;
  int* slot32 = nullptr;
  int* pos32 = nullptr;
  int4* visit = nullptr;   // [max_rows] the attention's rows in visiting order (longest first): {row, slot, pos, 0}
  int rows_written = 0;     // rows of slot32/pos32/visit some step has written (bounds the measurement hook)
  int* status = nullptr;
  bf16 *h = nullptr, *y = nullptr, *qkv = nullptr, *q = nullptr, *o = nullptr, *a = nullptr, *gu = nullptr,
       *act = nullptr;
  float* part_o = nullptr;
  float2* part_ml = nullptr;
  int* tickets = nullptr;  // [max_rows][kv_heads] split arrival counters, zero between launches
  std::vector<CUtensorMap> kmap, vmap;  // per layer, over [(max_slots + 1) * kv_heads][capacity][head_dim]
};

namespace {

template <class T>
T* carve(char*& p, size_t count) {
  T* r = reinterpret_cast<T*>(p);
  p += (count * sizeof(T) + 255) / 256 * 256;
  return r;
}

// A slot's first `length` positions of every layer's K and V to (save) or from (load) a packed prefix store
// [layers, 2 (K, V), kv_heads, length, head_dim] bf16: the reference's per-voice prefix KV (maya3/engine.py:276-280,
// a list of per-layer (k, v) [1, kv_heads, length, head_dim]) as one buffer, installed by one launch instead of a copy
// per layer and tensor (serve/fast_backbone.py:316-322).  A CTA moves 16 rows (one token of one KV head each) with 16
// threads per row and 16-byte vectors; grid.y walks (layer, K/V).  Load also sets lengths[slot] = length.
__global__ void prefix_copy_kernel(bf16* const* __restrict__ caches, bf16* __restrict__ store, int64_t slot,
                                   int length, int kv_heads, int capacity, int head_dim, int save,
                                   int64_t* __restrict__ lengths) {
  const int lk = blockIdx.y;
  const int64_t rows = (int64_t)kv_heads * length;
  const int64_t r = (int64_t)blockIdx.x * 16 + (threadIdx.x >> 4);
  if (!save && blockIdx.x == 0 && lk == 0 && threadIdx.x == 0) lengths[slot] = length;
  if (r >= rows) return;
  const int64_t h = r / length, t = r % length;
  uint4* c = reinterpret_cast<uint4*>(caches[lk] + ((slot * kv_heads + h) * capacity + t) * head_dim);
  uint4* st = reinterpret_cast<uint4*>(store + ((int64_t)lk * rows + r) * head_dim);
  for (int i = threadIdx.x & 15; i < head_dim / 8; i += 16) {
    if (save)
      st[i] = c[i];
    else
      c[i] = st[i];
  }
}

// Keys per split: the longest chunk (fewest partial results to merge) that still gives enough CTAs to fill the GPU a
// couple of times over, at most max_split splits, a power of two between 64 and 2048 (a multiple of the 32-token
// stage).  At a full decode batch one split per row measured fastest: the engine orders rows longest first, so the
// long rows' CTAs start first and the short ones fill the last wave.
int choose_chunk(int rows, int ctx, int kv, int max_split) {
  int chunk = 2048;
  while (chunk > 64 && (int64_t)rows * kv * cdiv(ctx, chunk) < 2 * 148 * 3) chunk /= 2;
  while (cdiv(ctx, chunk) > max_split) chunk *= 2;
  return chunk;
}


}  // namespace

extern "C" int m3_backbone_create(const m3_backbone_config* cfg, const m3_backbone_weights* w, m3_backbone** out) {
  M3_REQUIRE(cfg && w && out, M3_ERR_ARG, "m3_backbone_create: null argument");
  const m3_backbone_config& c = *cfg;
  M3_REQUIRE(c.head_dim == kHeadDim, M3_ERR_UNSUPPORTED, "head_dim %d unsupported (128 only)", c.head_dim);
  M3_REQUIRE(c.kv_heads > 0 && c.heads % c.kv_heads == 0, M3_ERR_ARG, "heads %% kv_heads != 0");
  const int G = c.heads / c.kv_heads;
  M3_REQUIRE(G == 1 || G == 2 || G == 4, M3_ERR_UNSUPPORTED, "GQA group %d unsupported", G);
  M3_REQUIRE(c.hidden % 8 == 0 && c.ffn % 8 == 0 && c.hidden <= 4 * 8 * 1024, M3_ERR_UNSUPPORTED,
             "hidden/ffn must be multiples of 8");
  M3_REQUIRE(c.heads + c.kv_heads <= 32, M3_ERR_UNSUPPORTED, "too many heads for the rope kernel");
  M3_REQUIRE(c.layers > 0 && c.max_slots > 0 && c.capacity > 0 && c.max_rows > 0, M3_ERR_ARG, "bad sizes");
  auto* bb = new m3_backbone();
  bb->c = c;
  for (int i = 0; i < c.layers; ++i) {
    bb->in_norm.push_back((const bf16*)w->in_norm[i]);
    bb->wqkv.push_back((const bf16*)w->wqkv[i]);
    bb->q_norm.push_back((const bf16*)w->q_norm[i]);
    bb->k_norm.push_back((const bf16*)w->k_norm[i]);
    bb->wo.push_back((const bf16*)w->wo[i]);
    bb->post_norm.push_back((const bf16*)w->post_norm[i]);
    bb->wgu.push_back((const bf16*)w->wgu[i]);
    bb->wdown.push_back((const bf16*)w->wdown[i]);
    bb->kc.push_back((bf16*)w->k_cache[i]);
    bb->vc.push_back((bf16*)w->v_cache[i]);
  }
  {
    EncodeTiled enc;
    if (tensor_map_encoder(&enc) != M3_OK) {
      delete bb;
      return M3_ERR_CUDA;
    }
    bb->kmap.resize(c.layers);
    bb->vmap.resize(c.layers);
    const cuuint64_t dims[3] = {(cuuint64_t)c.head_dim, (cuuint64_t)c.capacity,
                                (cuuint64_t)(c.max_slots + 1) * c.kv_heads};
    const cuuint64_t strides[2] = {(cuuint64_t)c.head_dim * 2, (cuuint64_t)c.capacity * c.head_dim * 2};
    const cuuint32_t box[3] = {64, (cuuint32_t)kBlkTok, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    for (int i = 0; i < c.layers; ++i)
      for (int kvv = 0; kvv < 2; ++kvv) {
        void* base = kvv ? w->v_cache[i] : w->k_cache[i];
        CUtensorMap* m = kvv ? &bb->vmap[i] : &bb->kmap[i];
        const CUresult r = (reinterpret_cast<uintptr_t>(base) & 15) ? CUDA_ERROR_INVALID_VALUE
                           : enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
          delete bb;
          set_error("m3_backbone_create: tensor map of layer %d %s cache failed (%d); caches must be 16-byte aligned",
                    i, kvv ? "V" : "K", (int)r);
          return M3_ERR_ARG;
        }
      }
  }
  bb->final_norm = (const bf16*)w->final_norm;
  bb->cos = (const bf16*)w->cos;
  bb->sin = (const bf16*)w->sin;
  bb->lengths = w->lengths;
  bb->max_split = std::max(16, cdiv(c.capacity, 512));
  const int R = c.max_rows, Hd = c.hidden, qkvw = (c.heads + 2 * c.kv_heads) * c.head_dim;
  const size_t parts = (size_t)R * c.kv_heads * bb->max_split * G;
  size_t bytes = 0;
  auto add = [&](size_t n) { bytes += (n + 255) / 256 * 256; };
  add(R * 4); add(R * 4); add(R * 16); add(256);
  add((size_t)R * Hd * 2); add((size_t)R * Hd * 2); add((size_t)R * qkvw * 2);
  add((size_t)R * c.heads * c.head_dim * 2); add((size_t)R * c.heads * c.head_dim * 2); add((size_t)R * Hd * 2);
  add((size_t)R * 2 * c.ffn * 2); add((size_t)R * c.ffn * 2);
  add(parts * kHeadDim * 4); add(parts * 8); add((size_t)R * c.kv_heads * 4); add((size_t)c.layers * 2 * 8);
  cudaError_t e = cudaMalloc(&bb->ws, bytes);
  if (e != cudaSuccess) {
    delete bb;
    set_error("m3_backbone_create: cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
    return M3_ERR_CUDA;
  }
  char* p = (char*)bb->ws;
  bb->slot32 = carve<int>(p, R);
  bb->pos32 = carve<int>(p, R);
  bb->visit = carve<int4>(p, R);
  bb->status = carve<int>(p, 64);
  bb->h = carve<bf16>(p, (size_t)R * Hd);
  bb->y = carve<bf16>(p, (size_t)R * Hd);
  bb->qkv = carve<bf16>(p, (size_t)R * qkvw);
  bb->q = carve<bf16>(p, (size_t)R * c.heads * c.head_dim);
  bb->o = carve<bf16>(p, (size_t)R * c.heads * c.head_dim);
  bb->a = carve<bf16>(p, (size_t)R * Hd);
  bb->gu = carve<bf16>(p, (size_t)R * 2 * c.ffn);
  bb->act = carve<bf16>(p, (size_t)R * c.ffn);
  bb->part_o = carve<float>(p, parts * kHeadDim);
  bb->part_ml = carve<float2>(p, parts);
  bb->tickets = carve<int>(p, (size_t)R * c.kv_heads);
  bb->caches = carve<bf16*>(p, (size_t)c.layers * 2);
  std::vector<bf16*> cp;
  for (int i = 0; i < c.layers; ++i) {
    cp.push_back(bb->kc[i]);
    cp.push_back(bb->vc[i]);
  }
  if (cudaMemset(bb->status, 0, 256) != cudaSuccess ||
      cudaMemset(bb->tickets, 0, (size_t)R * c.kv_heads * 4) != cudaSuccess ||
      cudaMemcpy(bb->caches, cp.data(), cp.size() * sizeof(bf16*), cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaFree(bb->ws);
    delete bb;
    set_error("m3_backbone_create: memset failed");
    return M3_ERR_CUDA;
  }
  cudaFuncSetAttribute(attn_mma_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMmaAttnSmemBytes);
  cudaFuncSetAttribute(attn_mma_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMmaAttnSmemBytes);
  cudaFuncSetAttribute(attn_mma_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMmaAttnSmemBytes);
  *out = bb;
  return M3_OK;
}

extern "C" int m3_backbone_destroy(m3_backbone* bb) {
  if (!bb) return M3_OK;
  if (bb->ws) cudaFree(bb->ws);
  delete bb;
  return M3_OK;
}

extern "C" int m3_backbone_status(m3_backbone* bb, int32_t* status, int32_t clear) {
  M3_REQUIRE(bb && status, M3_ERR_ARG, "m3_backbone_status: null argument");
  M3_CUDA(cudaMemcpy(status, bb->status, sizeof(int32_t), cudaMemcpyDeviceToHost));
  if (clear) M3_CUDA(cudaMemset(bb->status, 0, sizeof(int32_t)));
  return M3_OK;
}

// extra_tx: bytes each K/V stage barrier expects beyond its copies; 0 except in m3_backbone_attention_selftest.
static int attention(m3_backbone* bb, int layer, int rows, int ctx, cudaStream_t s, int extra_tx = 0) {
  const m3_backbone_config& c = bb->c;
  const int G = c.heads / c.kv_heads;
  const int chunk = choose_chunk(rows, ctx, c.kv_heads, bb->max_split);
  const int nsplit = cdiv(ctx, chunk);
  const float qscale = (1.f / sqrtf((float)c.head_dim)) * 1.4426950408889634f;
  dim3 grid(nsplit, c.kv_heads, rows);
#define M3_ATTN(GG)                                                                                          \
  attn_mma_kernel<GG><<<grid, kAttnThreads, kMmaAttnSmemBytes, s>>>(                                         \
      bb->kmap[layer], bb->vmap[layer], bb->q, bb->visit, bb->part_o, bb->part_ml,    \
      bb->tickets,                                                                                             \
      bb->o, nsplit, chunk, c.heads, qscale, bb->status, extra_tx);
  if (G == 1) {
    M3_ATTN(1)
  } else if (G == 2) {
    M3_ATTN(2)
  } else {
    M3_ATTN(4)
  }
#undef M3_ATTN
  M3_LAUNCHED();
  return M3_OK;
}

extern "C" int m3_backbone_step(m3_backbone* bb, const int64_t* slots, const int64_t* offsets, const int64_t* real,
                                const void* x, void* out, int32_t rows, int32_t ctx, m3_stream stream) {
  M3_REQUIRE(bb && slots && x && out, M3_ERR_ARG, "m3_backbone_step: null argument");
  const m3_backbone_config& c = bb->c;
  M3_REQUIRE(rows >= 0 && rows <= c.max_rows, M3_ERR_RANGE, "rows %d outside [0, %d]", rows, c.max_rows);
  M3_REQUIRE(ctx > 0 && ctx <= c.capacity, M3_ERR_RANGE, "ctx %d outside (0, %d]", ctx, c.capacity);
  if (rows == 0) return M3_OK;
  bb->rows_written = std::max(bb->rows_written, (int)rows);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int Hd = c.hidden, qkvw = (c.heads + 2 * c.kv_heads) * c.head_dim;
  M3_TRY(launch_prep_rows(slots, offsets, bb->lengths, rows, c.max_slots, c.capacity,
                          kQueryVectors / (c.heads / c.kv_heads), bb->slot32, bb->pos32, bb->visit, bb->status, s));
  const bf16* xin = reinterpret_cast<const bf16*>(x);
  for (int i = 0; i < c.layers; ++i) {
    // h = x, y = RMSNorm(x) on the first layer (HF Qwen3RMSNorm module, one launch); h += a, y = RMSNorm(h) after
    if (i == 0)
      M3_TRY(launch_add_rms(rows, xin, nullptr, bb->h, bb->y, bb->in_norm[0], c.eps, Hd, s));
    else
      M3_TRY(launch_add_rms(rows, bb->h, bb->a, bb->h, bb->y, bb->in_norm[i], c.eps, Hd, s));
    M3_TRY(gemm({bb->y, Hd, bb->wqkv[i], Hd, bb->qkv, qkvw, rows, qkvw, Hd, false}, s));
    qk_rope_cache_kernel<<<dim3(rows, cdiv(c.heads + c.kv_heads, 4)), 128, 0, s>>>(
        bb->qkv, bb->q, bb->kc[i], bb->vc[i], (int64_t)c.kv_heads * c.capacity * c.head_dim,
        (int64_t)c.capacity * c.head_dim, bb->slot32, bb->pos32, bb->cos, bb->sin, bb->q_norm[i], bb->k_norm[i],
        c.eps, c.heads, c.kv_heads);
    M3_LAUNCHED();
    M3_TRY(attention(bb, i, rows, ctx, s));
    M3_TRY(gemm({bb->o, c.heads * c.head_dim, bb->wo[i], c.heads * c.head_dim, bb->a, Hd, rows, Hd,
                 c.heads * c.head_dim, false},
                s));
    M3_TRY(launch_add_rms(rows, bb->h, bb->a, bb->h, bb->y, bb->post_norm[i], c.eps, Hd, s));
    GemmDesc gu{bb->y, Hd, bb->wgu[i], Hd, bb->act, c.ffn, rows, 2 * c.ffn, Hd, false};
    gu.act = kActSwiGLU;
    if (gemv_path(gu)) {  // a few rows: SwiGLU in the GEMV epilogue
      M3_TRY(gemm(gu, s));
    } else {
      M3_TRY(gemm({bb->y, Hd, bb->wgu[i], Hd, bb->gu, 2 * c.ffn, rows, 2 * c.ffn, Hd, false}, s));
      const int64_t nv = (int64_t)rows * (c.ffn / 8);
      silu_mul_kernel<<<(unsigned)((nv + 255) / 256), 256, 0, s>>>(bb->gu, bb->act, rows, c.ffn);
      M3_LAUNCHED();
    }
    M3_TRY(gemm({bb->act, c.ffn, bb->wdown[i], c.ffn, bb->a, Hd, rows, Hd, c.ffn, false}, s));
  }
  M3_TRY(launch_add_rms(rows, bb->h, bb->a, bb->h, reinterpret_cast<bf16*>(out), bb->final_norm, c.eps, Hd, s));
  lengths_add_kernel<<<cdiv(rows, 128), 128, 0, s>>>(bb->slot32, real, rows, bb->lengths);
  M3_LAUNCHED();
  return M3_OK;
}

extern "C" int m3_backbone_attention(m3_backbone* bb, int32_t layer, int32_t rows, int32_t ctx, m3_stream stream) {
  M3_REQUIRE(bb, M3_ERR_ARG, "m3_backbone_attention: null handle");
  M3_REQUIRE(layer >= 0 && layer < bb->c.layers && rows > 0 && rows <= bb->c.max_rows && ctx > 0 &&
                 ctx <= bb->c.capacity,
             M3_ERR_RANGE, "m3_backbone_attention: layer %d rows %d ctx %d out of range", layer, rows, ctx);
  M3_REQUIRE(rows <= bb->rows_written, M3_ERR_RANGE,
             "m3_backbone_attention: rows %d beyond the %d rows a backbone step has set up", rows, bb->rows_written);
  return attention(bb, layer, rows, ctx, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int m3_backbone_attention_selftest(m3_backbone* bb, int32_t layer, int32_t rows, int32_t ctx,
                                              m3_stream stream) {
  M3_REQUIRE(bb, M3_ERR_ARG, "m3_backbone_attention_selftest: null handle");
  M3_REQUIRE(layer >= 0 && layer < bb->c.layers && rows > 0 && rows <= bb->rows_written && rows <= 8 && ctx > 0 &&
                 ctx <= bb->c.capacity,
             M3_ERR_RANGE, "m3_backbone_attention_selftest: layer %d rows %d ctx %d out of range", layer, rows, ctx);
  return attention(bb, layer, rows, ctx, reinterpret_cast<cudaStream_t>(stream), 16);
}

static int prefix_copy(m3_backbone* bb, int32_t slot, void* store, int32_t length, int save, m3_stream stream) {
  M3_REQUIRE(bb && store, M3_ERR_ARG, "prefix copy: null argument");
  const m3_backbone_config& c = bb->c;
  M3_REQUIRE(slot >= 0 && slot < c.max_slots, M3_ERR_RANGE, "prefix copy: slot %d outside [0, %d)", slot,
             c.max_slots);
  M3_REQUIRE(length > 0 && length <= c.capacity, M3_ERR_RANGE, "prefix copy: length %d outside (0, %d]", length,
             c.capacity);
  M3_REQUIRE((reinterpret_cast<uintptr_t>(store) & 15) == 0 && c.head_dim % 8 == 0, M3_ERR_ARG,
             "prefix copy: the store must be 16-byte aligned");
  const dim3 grid(cdiv(c.kv_heads * length, 16), c.layers * 2);
  prefix_copy_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      bb->caches, reinterpret_cast<bf16*>(store), slot, length, c.kv_heads, c.capacity, c.head_dim, save,
      bb->lengths);
  M3_LAUNCHED();
  return M3_OK;
}

extern "C" int m3_backbone_save_prefix(m3_backbone* bb, int32_t slot, void* store, int32_t length, m3_stream stream) {
  return prefix_copy(bb, slot, store, length, 1, stream);
}

extern "C" int m3_backbone_load_prefix(m3_backbone* bb, int32_t slot, const void* store, int32_t length,
                                       m3_stream stream) {
  return prefix_copy(bb, slot, const_cast<void*>(store), length, 0, stream);
}
