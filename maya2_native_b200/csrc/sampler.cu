// Sampling kernels: the depth level sampler (replaces _topk_sample, serve/fast_depth_kernels.py:305-336) and the
// cb0 sampler with controlled stop (replaces Engine._cb0 + row_exponential, maya3/engine.py:652-694,
// serve/fast_depth_kernels.py:339-355).  One CTA per row; the top-k threshold is found by a bitwise search over
// order-preserving integer keys (exact k-th largest, no sort); noise is counter-based Philox, bit-identical to the
// reference's tl.rand stream for the same (seed, counter, level, code).
#include <mutex>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"
#include "sampler.cuh"

namespace m3 {

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy as 1, 2, 3", SC'11) on the counter
// (offset, 0, 0, 0) with key (seed_lo, seed_hi); the first word as a uniform float in [0, 1) the way Triton's
// uint_to_uniform_float folds it: int32 x -> (x < 0 ? -x - 1 : x) * 4.6566127342e-10.
__device__ __forceinline__ float philox_uniform(int32_t seed, uint32_t offset) {
  uint32_t c0 = offset, c1 = 0, c2 = 0, c3 = 0;
  uint32_t k0 = (uint32_t)seed, k1 = seed < 0 ? 0xffffffffu : 0u;  // int32 seed widened to 64 bits
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hb = __umulhi(0xCD9E8D57u, c2), lb = 0xCD9E8D57u * c2;
    const uint32_t ha = __umulhi(0xD2511F53u, c0), la = 0xD2511F53u * c0;
    const uint32_t n0 = hb ^ c1 ^ k0, n2 = ha ^ c3 ^ k1;
    c0 = n0;
    c1 = lb;
    c2 = n2;
    c3 = la;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  int32_t x = (int32_t)c0;
  x = x < 0 ? -x - 1 : x;
  return __fmul_rn((float)x, 4.6566127342e-10f);
}

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

constexpr int kSampThreads = 256;
constexpr int kMaxPer = 16;  // up to 4096 entries per row

// The k-th largest key (1 <= k <= n), exactly: a radix select over four 8-bit digits, most significant first.  Each
// pass histograms the digit of the keys that match the digits chosen so far (one private histogram per warp), then one
// warp scans the 256 bins from the top to find the bin holding the rank-th largest and the rank inside it.
__device__ uint32_t kth_largest_key(const uint32_t (&key)[kMaxPer], int per, int k) {
  constexpr int kWarps = kSampThreads / 32;
  __shared__ int hist[kWarps][256];
  __shared__ int s_digit, s_rank;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint32_t prefix = 0, mask = 0;
  int rank = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < kWarps * 256; i += kSampThreads) (&hist[0][0])[i] = 0;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i)
      if (i < per && (key[i] & mask) == prefix) atomicAdd(&hist[warp][(key[i] >> shift) & 255u], 1);
    __syncthreads();
    for (int b = tid; b < 256; b += kSampThreads) {
      int sum = 0;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) sum += hist[w][b];
      hist[0][b] = sum;
    }
    __syncthreads();
    if (warp == 0) {  // lane l holds digits 255 - 8l .. 248 - 8l
      int c[8], tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = hist[0][255 - 8 * lane - j];
        tot += c[j];
      }
      int incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      int run = incl - tot;
      if (run < rank && rank <= incl) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (run + c[j] >= rank) {
            s_digit = 255 - 8 * lane - j;
            s_rank = rank - run;
            break;
          }
          run += c[j];
        }
      }
    }
    __syncthreads();
    prefix |= (uint32_t)s_digit << shift;
    mask |= 0xFFu << shift;
    rank = s_rank;
  }
  return prefix;
}

// Block argmax with the smallest index among equal maxima (torch / Triton argmax).
__device__ int block_argmax(float v, int idx, float* redv, int* redi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) v = ov, idx = oi;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) redv[threadIdx.x >> 5] = v, redi[threadIdx.x >> 5] = idx;
  __syncthreads();
  v = redv[0];
  idx = redi[0];
#pragma unroll
  for (int w = 1; w < kSampThreads / 32; ++w)
    if (redv[w] > v || (redv[w] == v && redi[w] < idx)) v = redv[w], idx = redi[w];
  return idx;
}

// ------------------------------------------------------------------------------------------------ depth sampler
// x = logits * (1/temp); kth = k-th largest (0 when k is outside [1, V], as the reference's masked sum yields);
// keep x >= kth; greedy -> argmax, else argmax(x - log(-log u)), u = tl.rand(seed, (ctr*32 + level)*V + c).
// Optionally writes the next prefix row embed[code] (serve/fast_depth.py:195-196).
template <typename TL>
__global__ void __launch_bounds__(kSampThreads) topk_sample_kernel(
    const TL* __restrict__ logits, int64_t ld, int V, const int32_t* __restrict__ seed,
    const int32_t* __restrict__ ctr, const int* __restrict__ slot32, int level, float inv_temp, int k, int greedy,
    int64_t* __restrict__ codes, int64_t code_stride, const bf16* __restrict__ embed, int D,
    bf16* __restrict__ next_row, int64_t next_stride, PrefixLn ln) {
  __shared__ float redv[32];
  __shared__ int redi[32];
  __shared__ int s_code;
  const int row = blockIdx.x, tid = threadIdx.x;
  const int per = cdiv(V, kSampThreads);
  const int sl = slot32 ? slot32[row] : row;
  float x[kMaxPer];
  uint32_t key[kMaxPer];
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int c = tid + i * kSampThreads;
    x[i] = -INFINITY;
    key[i] = 0;
    if (i < per && c < V) {
      x[i] = to_f(logits[row * ld + c]) * inv_temp;
      key[i] = order_key(x[i]);
    }
  }
  float kth = 0.f;
  if (k >= 1 && k <= V) kth = key_value(kth_largest_key(key, per, k));
  float best = -INFINITY;
  int bidx = 0x7fffffff;
  const int32_t sd = greedy ? 0 : seed[sl];
  const uint32_t base = greedy ? 0u : ((uint32_t)ctr[sl] * 32u + (uint32_t)level) * (uint32_t)V;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int c = tid + i * kSampThreads;
    if (i < per && c < V) {
      float sc = x[i] >= kth ? x[i] : -INFINITY;
      if (!greedy && sc != -INFINITY) {  // masked entries cannot win: their noise is never drawn
        const float u = fmaxf(philox_uniform(sd, base + (uint32_t)c), 1e-12f);
        sc = sc - logf(-logf(u));
      }
      if (sc > best || bidx == 0x7fffffff) best = sc, bidx = c;
    }
  }
  const int code = block_argmax(best, bidx, redv, redi);
  if (tid == 0) {
    codes[row * code_stride] = code;
    s_code = code;
  }
  if (next_row) {
    __syncthreads();
    const uint4* src = reinterpret_cast<const uint4*>(embed + (int64_t)s_code * D);
    uint4* dst = reinterpret_cast<uint4*>(next_row + row * next_stride);
    for (int i = tid; i < D / 8; i += kSampThreads) dst[i] = src[i];
  }
  if (ln.x) {  // the next level's first LayerNorm over this row's prefix (the new entry included)
    __syncthreads();
    const int warp = tid >> 5, lane = tid & 31, nv = D / 8;
    for (int i = warp; i < ln.T; i += kSampThreads / 32) {
      const uint4* src = reinterpret_cast<const uint4*>(ln.prefix + (int64_t)row * ln.sb + (int64_t)(ln.start + i) * D);
      uint4* xo = reinterpret_cast<uint4*>(ln.x + ((int64_t)row * ln.T + i) * D);
      uint4* yo = reinterpret_cast<uint4*>(ln.y + ((int64_t)row * ln.T + i) * D);
      float v[8], sum = 0.f, sq = 0.f;
      for (int c = lane; c < nv; c += 32) {
        unpack8(src[c], v);
#pragma unroll
        for (int e = 0; e < 8; ++e) sum += v[e];
      }
      const float mean = warp_sum(sum) / (float)D;
      for (int c = lane; c < nv; c += 32) {
        unpack8(src[c], v);
#pragma unroll
        for (int e = 0; e < 8; ++e) sq = fmaf(v[e] - mean, v[e] - mean, sq);
      }
      const float den = sqrtf(warp_sum(sq) / (float)D + ln.eps);
      for (int c = lane; c < nv; c += 32) {
        const uint4 raw = src[c];
        float wv[8], bv[8], o[8];
        unpack8(raw, v);
        unpack8(reinterpret_cast<const uint4*>(ln.w)[c], wv);
        unpack8(reinterpret_cast<const uint4*>(ln.bias)[c], bv);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = (v[e] - mean) / den * wv[e] + bv[e];
        xo[c] = raw;
        yo[c] = pack8(o);
      }
    }
  }
}

int launch_topk_sample(const void* logits, bool bf, int64_t ld, int rows, int V, const int32_t* seed,
                       const int32_t* ctr, const int* slot32, int level, float inv_temp, int k, int greedy,
                       int64_t* codes, int64_t code_stride, const bf16* embed, int D, bf16* next_row,
                       int64_t next_stride, cudaStream_t s, const PrefixLn& ln) {
  M3_REQUIRE(V > 0 && V <= kSampThreads * kMaxPer, M3_ERR_UNSUPPORTED, "sampler width %d unsupported", V);
  M3_REQUIRE(!ln.x || (D % 8 == 0 && ln.y && ln.w && ln.bias && ln.prefix), M3_ERR_ARG, "prefix LayerNorm arguments");
  if (rows == 0) return M3_OK;
  if (bf)
    topk_sample_kernel<bf16><<<rows, kSampThreads, 0, s>>>((const bf16*)logits, ld, V, seed, ctr, slot32, level,
                                                            inv_temp, k, greedy, codes, code_stride, embed, D,
                                                            next_row, next_stride, ln);
  else
    topk_sample_kernel<float><<<rows, kSampThreads, 0, s>>>((const float*)logits, ld, V, seed, ctr, slot32, level,
                                                             inv_temp, k, greedy, codes, code_stride, embed, D,
                                                             next_row, next_stride, ln);
  M3_LAUNCHED();
  return M3_OK;
}

// ------------------------------------------------------------------------------------------------ cb0 sampler
constexpr int kAeos = 2048;
constexpr int kSortN = 4096;

struct Cb0Dev {
  int64_t* frames;
  const int64_t* min_frames;
  float* hazard;
  const float* aeos_bias;
  const float* temp;
  const int64_t* top_k;
  const float* top_p;
  const float* rep;
  const int32_t* seed;
  int32_t* ctr;
  int64_t* hist;
  int rep_win;
  int max_slots;
};

// Descending bitonic sort of (value, index) pairs in shared memory (kSortN entries, padding = -inf).
__device__ void bitonic_sort_desc(float* v, short* ix) {
  for (int size = 2; size <= kSortN; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int i = threadIdx.x; i < kSortN / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = ((lo & size) == 0);
        const float a = v[lo], b = v[hi];
        const bool swap = desc ? (a < b) : (a > b);
        if (swap) {
          v[lo] = b;
          v[hi] = a;
          const short t = ix[lo];
          ix[lo] = ix[hi];
          ix[hi] = t;
        }
      }
    }
  }
  __syncthreads();
}

template <typename TL>
__global__ void __launch_bounds__(kSampThreads) cb0_sample_kernel(const TL* __restrict__ logits, int64_t ld, int V,
                                                                  const int64_t* __restrict__ idx, Cb0Dev st,
                                                                  int apply_rep, int apply_top_p,
                                                                  int64_t* __restrict__ code_out,
                                                                  int64_t* __restrict__ cb0_out, int* status) {
  __shared__ float redf[32];
  __shared__ float redv[32];
  __shared__ int redi[32];
  __shared__ unsigned char pen[kSortN];
  __shared__ float sv[kSortN];
  __shared__ short si[kSortN];
  const int row = blockIdx.x, tid = threadIdx.x;
  const int per = cdiv(V, kSampThreads);
  int64_t slot = idx[row];
  if (slot < 0 || slot > st.max_slots) {
    report(status, M3_DEV_BAD_SLOT);
    slot = st.max_slots;
  }
  // logits / temp (+ AEOS bias) (- presence penalty)   maya3/engine.py:657-665
  const float temp = st.temp[slot];
  if (apply_rep && st.rep_win > 0) {
    for (int i = tid; i < V; i += kSampThreads) pen[i] = 0;
    __syncthreads();
    if (tid < st.rep_win) {
      const int64_t h = st.hist[slot * st.rep_win + tid];
      if (h >= 0 && h < V) pen[h] = 1;
    }
    __syncthreads();
    if (tid == 0 && kAeos < V) pen[kAeos] = 0;
    __syncthreads();
  }
  const float rep = st.rep[slot];
  float x[kMaxPer];
  uint32_t key[kMaxPer];
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int c = tid + i * kSampThreads;
    x[i] = -INFINITY;
    key[i] = 0;
    if (i < per && c < V) {
      float v = to_f(logits[row * ld + c]) / temp;
      if (c == kAeos) v += st.aeos_bias[slot];
      if (apply_rep && st.rep_win > 0) v = v - rep * (pen[c] ? 1.f : 0.f);
      x[i] = v;
      key[i] = order_key(v);
    }
  }
  // top-k: keep x >= k-th largest, k clamped to [1, V]   maya3/engine.py:666-668
  int64_t k = st.top_k[slot];
  k = k < 1 ? 1 : (k > V ? V : k);
  const float kth = key_value(kth_largest_key(key, per, (int)k));
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i)
    if (x[i] < kth) x[i] = -INFINITY;
  // softmax
  auto softmax = [&](float* p) {
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) mx = fmaxf(mx, x[i]);
    mx = block_max(mx, redf);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      p[i] = (i < per && tid + i * kSampThreads < V) ? expf(x[i] - mx) : 0.f;
      sum += p[i];
    }
    sum = block_sum(sum, redf);
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) p[i] = p[i] / sum;
  };
  float p[kMaxPer];
  if (apply_top_p) {  // maya3/engine.py:669-672: drop entries whose preceding sorted mass exceeds top_p
    softmax(p);
    for (int i = tid; i < kSortN; i += kSampThreads) {
      sv[i] = -INFINITY;
      si[i] = (short)i;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      const int c = tid + i * kSampThreads;
      if (i < per && c < V) sv[c] = p[i];
    }
    bitonic_sort_desc(sv, si);
    // inclusive prefix sum of the sorted probabilities: each thread owns 16 consecutive entries
    constexpr int kRun = kSortN / kSampThreads;
    float run[kRun], tot = 0.f;
#pragma unroll
    for (int j = 0; j < kRun; ++j) {
      const float v = fmaxf(sv[tid * kRun + j], 0.f);
      tot += v;
      run[j] = tot;
    }
    // exclusive scan of thread totals
    float incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float t = __shfl_up_sync(0xffffffffu, incl, o);
      if ((tid & 31) >= o) incl += t;
    }
    __syncthreads();
    if ((tid & 31) == 31) redf[tid >> 5] = incl;
    __syncthreads();
    float wpre = 0.f;
    for (int w = 0; w < (tid >> 5); ++w) wpre += redf[w];
    const float pre = wpre + incl - tot;
    const float topp = st.top_p[slot];
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kRun; ++j) {
      const int pos = tid * kRun + j;
      const float spv = fmaxf(sv[pos], 0.f);
      const bool drop = (pre + run[j]) - spv > topp;
      pen[pos] = 0;
      sv[pos] = drop ? 1.f : 0.f;  // reuse as the drop flag of sorted position pos
    }
    __syncthreads();
    for (int pos = tid; pos < kSortN; pos += kSampThreads) {
      const int c = si[pos];
      if (c < V && sv[pos] != 0.f) pen[c] = 1;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
      const int c = tid + i * kSampThreads;
      if (i < per && c < V && pen[c]) x[i] = -INFINITY;
    }
  }
  softmax(p);
  // controlled stop   maya3/engine.py:673-683
  float pa = 0.f, best = -INFINITY;
  int bidx = 0x7fffffff;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int c = tid + i * kSampThreads;
    if (i < per && c < V) {
      if (c == kAeos) pa = p[i];
      if (p[i] > best || bidx == 0x7fffffff) best = p[i], bidx = c;
    }
  }
  const int arg = block_argmax(best, bidx, redv, redi);
  pa = block_sum(pa, redf);  // only one thread holds the AEOS entry
  // renormalise without AEOS, sample by the exponential race   maya3/engine.py:684-688
  float qs = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int c = tid + i * kSampThreads;
    if (c == kAeos) p[i] = 0.f;
    if (i < per && c < V) qs += p[i];
  }
  qs = fmaxf(block_sum(qs, redf), 1e-12f);
  const int32_t sd = st.seed[slot];
  const int32_t cr = st.ctr[slot];
  const uint32_t base = (uint32_t)cr * 32u * 4096u;
  best = -INFINITY;
  bidx = 0x7fffffff;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int c = tid + i * kSampThreads;
    if (i < per && c < V) {
      float r = 0.f;  // p = 0: the ratio is 0 whatever the exponential draw (finite, u >= 1e-12)
      if (p[i] != 0.f) {
        const float u = fmaxf(philox_uniform(sd, base + (uint32_t)c), 1e-12f);
        r = (p[i] / qs) / -logf(u);
      }
      if (r > best || bidx == 0x7fffffff) best = r, bidx = c;
    }
  }
  int cb0 = block_argmax(best, bidx, redv, redi);
  if (cb0 > kAeos - 1) cb0 = kAeos - 1;
  if (tid == 0) {
    const int64_t frames = st.frames[slot];
    const bool can = frames >= st.min_frames[slot];
    float hz = st.hazard[slot];
    if (can) hz = 1.f - (1.f - hz) * (1.f - pa);
    int64_t code = 0;
    if (can && hz >= 0.6f) code = 4;
    if (can && pa >= 0.35f) code = 3;
    if (can && arg == kAeos) code = 2;
    code_out[row] = code;
    cb0_out[row] = cb0;
    st.ctr[slot] = cr + 1;
    if (st.rep_win > 0) {
      int64_t* h = st.hist + slot * st.rep_win;
      for (int w = 0; w + 1 < st.rep_win; ++w) h[w] = h[w + 1];
      h[st.rep_win - 1] = cb0;
    }
    st.hazard[slot] = hz;
    st.frames[slot] = frames + 1;
  }
}

}  // namespace m3

using namespace m3;

struct m3_cb0 {
  m3_cb0_config c{};
  Cb0Dev st{};
  const bf16* head = nullptr;
  void* ws = nullptr;
  bf16* logits = nullptr;
  // n_cls rounded up to 8: the head GEMM runs on a copy of the head padded with zero rows to ldl classes, so the
  // library GEMM gets a multiple-of-8 output width (an odd width falls to its align-1 split-K kernels, 3x slower)
  int ldl = 0;
  int* status = nullptr;
};

extern "C" int m3_cb0_create(const m3_cb0_config* cfg, const m3_cb0_state* s, m3_cb0** out) {
  M3_REQUIRE(cfg && s && out, M3_ERR_ARG, "m3_cb0_create: null argument");
  M3_REQUIRE(cfg->n_cls > 0 && cfg->n_cls <= kSampThreads * kMaxPer, M3_ERR_UNSUPPORTED, "n_cls %d", cfg->n_cls);
  M3_REQUIRE(cfg->rep_win >= 0 && cfg->rep_win <= kSampThreads, M3_ERR_UNSUPPORTED, "rep_win %d", cfg->rep_win);
  M3_REQUIRE(cfg->hidden % 8 == 0, M3_ERR_UNSUPPORTED, "hidden %% 8");
  auto* h = new m3_cb0();
  h->c = *cfg;
  h->st = Cb0Dev{s->frames, s->min_frames, s->hazard, s->aeos_bias, s->temp, s->top_k, s->top_p, s->rep, s->seed,
                 s->ctr, s->hist, cfg->rep_win, cfg->max_slots};
  h->ldl = (cfg->n_cls + 7) / 8 * 8;
  const size_t lb = ((size_t)cfg->max_rows * h->ldl * 2 + 255) / 256 * 256;
  const size_t hb = (size_t)h->ldl * cfg->hidden * 2, real = (size_t)cfg->n_cls * cfg->hidden * 2;
  cudaError_t e = cudaMalloc(&h->ws, lb + 256 + hb);
  if (e == cudaSuccess) {
    h->logits = (bf16*)h->ws;
    h->status = (int*)((char*)h->ws + lb);
    bf16* head = (bf16*)((char*)h->ws + lb + 256);
    h->head = head;
    e = cudaMemset(h->status, 0, 256);
    if (e == cudaSuccess) e = cudaMemcpy(head, s->head, real, cudaMemcpyDeviceToDevice);
    if (e == cudaSuccess) e = cudaMemset((char*)head + real, 0, hb - real);
    if (e != cudaSuccess) cudaFree(h->ws);
  }
  if (e != cudaSuccess) {
    delete h;
    set_error("m3_cb0_create: %s", cudaGetErrorString(e));
    return M3_ERR_CUDA;
  }
  *out = h;
  return M3_OK;
}

extern "C" int m3_cb0_destroy(m3_cb0* s) {
  if (!s) return M3_OK;
  cudaFree(s->ws);
  delete s;
  return M3_OK;
}

extern "C" int m3_cb0_copy_logits(m3_cb0* s, void* dst, int32_t rows, m3_stream stream) {
  M3_REQUIRE(s && dst, M3_ERR_ARG, "m3_cb0_copy_logits: null argument");
  M3_REQUIRE(rows >= 0 && rows <= s->c.max_rows, M3_ERR_RANGE, "rows %d > max_rows %d", rows, s->c.max_rows);
  if (rows == 0) return M3_OK;
  M3_CUDA(cudaMemcpy2DAsync(dst, (size_t)s->c.n_cls * 2, s->logits, (size_t)s->ldl * 2, (size_t)s->c.n_cls * 2, rows,
                            cudaMemcpyDeviceToDevice, reinterpret_cast<cudaStream_t>(stream)));
  return M3_OK;
}

extern "C" int m3_cb0_status(m3_cb0* s, int32_t* status, int32_t clear) {
  M3_REQUIRE(s && status, M3_ERR_ARG, "m3_cb0_status: null argument");
  M3_CUDA(cudaMemcpy(status, s->status, sizeof(int32_t), cudaMemcpyDeviceToHost));
  if (clear) M3_CUDA(cudaMemset(s->status, 0, sizeof(int32_t)));
  return M3_OK;
}

static int cb0_launch(m3_cb0* s, const void* logits, int64_t ld, bool bf, const int64_t* idx, int64_t* code,
                      int64_t* cb0, int rows, int apply_rep, int apply_top_p, cudaStream_t st) {
  if (rows == 0) return M3_OK;
  if (bf)
    cb0_sample_kernel<bf16><<<rows, kSampThreads, 0, st>>>((const bf16*)logits, ld, s->c.n_cls, idx,
                                                            s->st, apply_rep, apply_top_p, code, cb0, s->status);
  else
    cb0_sample_kernel<float><<<rows, kSampThreads, 0, st>>>((const float*)logits, ld, s->c.n_cls, idx,
                                                             s->st, apply_rep, apply_top_p, code, cb0, s->status);
  M3_LAUNCHED();
  return M3_OK;
}

extern "C" int m3_cb0_step(m3_cb0* s, const void* h, const int64_t* idx, int64_t* code, int64_t* cb0, int32_t rows,
                           int32_t apply_rep, int32_t apply_top_p, m3_stream stream) {
  M3_REQUIRE(s && h && idx && code && cb0, M3_ERR_ARG, "m3_cb0_step: null argument");
  M3_REQUIRE(rows >= 0 && rows <= s->c.max_rows, M3_ERR_RANGE, "rows %d > max_rows %d", rows, s->c.max_rows);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // cb0_head in the model dtype (bf16 output), read back as fp32 (tts/model/backbone.py:97, engine.py:657)
  // over the padded head: logits columns n_cls.. are zeros that the sampler never reads
  M3_TRY(gemm({(const bf16*)h, s->c.hidden, s->head, s->c.hidden, s->logits, s->ldl, rows, s->ldl,
               s->c.hidden, false},
              st));
  return cb0_launch(s, s->logits, s->ldl, true, idx, code, cb0, rows, apply_rep, apply_top_p, st);
}

extern "C" int m3_cb0_sample_logits(m3_cb0* s, const float* logits, const int64_t* idx, int64_t* code, int64_t* cb0,
                                    int32_t rows, int32_t apply_rep, int32_t apply_top_p, m3_stream stream) {
  M3_REQUIRE(s && logits && idx && code && cb0, M3_ERR_ARG, "m3_cb0_sample_logits: null argument");
  return cb0_launch(s, logits, s->c.n_cls, false, idx, code, cb0, rows, apply_rep, apply_top_p,
                    reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int m3_topk_sample(const void* logits, int32_t logits_bf16, int32_t rows, int32_t n, const int32_t* seed,
                              const int32_t* ctr, int32_t level, float inv_temp, int32_t top_k, int32_t greedy,
                              int64_t* codes, m3_stream stream) {
  M3_REQUIRE(logits && codes && (greedy || (seed && ctr)), M3_ERR_ARG, "m3_topk_sample: null argument");
  return launch_topk_sample(logits, logits_bf16 != 0, n, rows, n, seed, ctr, nullptr, level, inv_temp, top_k, greedy,
                            codes, 1, nullptr, 0, nullptr, 0, reinterpret_cast<cudaStream_t>(stream));
}

// ================================================================================================ allocation-free cb0 step
// Some callers cannot allocate device memory when they sample: a host that hands this library a fixed device
// budget up front and forbids any later cudaMalloc (every byte of a B200 already mapped to KV caches and weights),
// or a caller on a latency-critical serving thread where cudaMalloc/cudaFree would synchronise the device and stall
// every seat's frame.  For them m3_cb0_step_noalloc runs the same cb0 head + sampler as m3_cb0_step without a handle:
// its only scratch (the bf16 logits and a status word) lives in this file-scope device array, which every GPU that
// loads the library holds until the process exits.
constexpr int kNoAllocRows = 8;      // rows per call (the head GEMM runs on the GEMV kernel, which serves M <= 8)
constexpr int kNoAllocCls = 4096;    // classes per row
constexpr size_t kNoAllocLogitsBytes = (size_t)kNoAllocRows * kNoAllocCls * sizeof(bf16);   // 64 KiB
constexpr size_t kNoAllocScratchBytes = kNoAllocLogitsBytes + 256;                             // + status word
static __device__ __align__(256) unsigned char g_cb0_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_noalloc_mu;
std::vector<void*> g_noalloc_ptr;  // device address of the scratch array, per device ordinal

// Host code cannot use the array's name as a device address: look the address up once per device, with that
// device current.
int noalloc_scratch(void** out) {
  int dev = 0;
  M3_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if ((int)g_noalloc_ptr.size() <= dev) g_noalloc_ptr.resize(dev + 1, nullptr);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_cb0_noalloc_scratch);
    if (e != cudaSuccess) {
      set_error("m3_cb0_step_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev, cudaGetErrorString(e));
      return M3_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return M3_OK;
}
}  // namespace

extern "C" int m3_cb0_step_noalloc(const m3_cb0_config* cfg, const m3_cb0_state* st, const void* h,
                                   const int64_t* idx, int64_t* code, int64_t* cb0, int32_t rows, int32_t apply_rep,
                                   int32_t apply_top_p, m3_stream stream) {
  M3_REQUIRE(cfg && st && st->head && h && idx && code && cb0, M3_ERR_ARG, "m3_cb0_step_noalloc: null argument");
  M3_REQUIRE(rows >= 0 && rows <= kNoAllocRows, M3_ERR_ARG,
             "m3_cb0_step_noalloc: %d rows exceed the allocation-free limit of %d rows per call", rows, kNoAllocRows);
  M3_REQUIRE(cfg->n_cls > 0 && cfg->n_cls <= kNoAllocCls, M3_ERR_ARG,
             "m3_cb0_step_noalloc: %d classes exceed the allocation-free limit of %d", cfg->n_cls, kNoAllocCls);
  M3_REQUIRE(cfg->hidden > 0 && cfg->hidden % 8 == 0 && cfg->hidden <= 3072, M3_ERR_ARG,
             "m3_cb0_step_noalloc: hidden %d must be a multiple of 8 and at most 3072", cfg->hidden);
  M3_REQUIRE(cfg->rep_win >= 0 && cfg->rep_win <= kSampThreads, M3_ERR_ARG,
             "m3_cb0_step_noalloc: rep_win %d exceeds %d", cfg->rep_win, kSampThreads);
  M3_REQUIRE(((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(st->head)) & 15) == 0, M3_ERR_ARG,
             "m3_cb0_step_noalloc: h and the head must start on 16-byte boundaries");
  void* scratch = nullptr;
  M3_TRY(noalloc_scratch(&scratch));
  if (rows == 0) return M3_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  bf16* logits = reinterpret_cast<bf16*>(scratch);
  // the status word is sticky across calls (zero at load, first problem wins) until m3_cb0_noalloc_status clears it
  int* status = reinterpret_cast<int*>(reinterpret_cast<char*>(scratch) + kNoAllocLogitsBytes);
  M3_TRY(gemv_only({(const bf16*)h, cfg->hidden, (const bf16*)st->head, cfg->hidden, logits, cfg->n_cls, rows,
                    cfg->n_cls, cfg->hidden, false},
                   s));
  const Cb0Dev dev{st->frames, st->min_frames, st->hazard, st->aeos_bias, st->temp, st->top_k, st->top_p, st->rep,
                   st->seed, st->ctr, st->hist, cfg->rep_win, cfg->max_slots};
  cb0_sample_kernel<bf16><<<rows, kSampThreads, 0, s>>>(logits, cfg->n_cls, cfg->n_cls, idx, dev, apply_rep,
                                                         apply_top_p, code, cb0, status);
  M3_LAUNCHED();
  return M3_OK;
}

extern "C" int m3_cb0_noalloc_status(int32_t* status, int32_t clear) {
  M3_REQUIRE(status, M3_ERR_ARG, "m3_cb0_noalloc_status: null argument");
  void* scratch = nullptr;
  M3_TRY(noalloc_scratch(&scratch));
  int* word = reinterpret_cast<int*>(reinterpret_cast<char*>(scratch) + kNoAllocLogitsBytes);
  M3_CUDA(cudaMemcpy(status, word, sizeof(int32_t), cudaMemcpyDeviceToHost));
  if (clear) M3_CUDA(cudaMemset(word, 0, sizeof(int32_t)));
  return M3_OK;
}
