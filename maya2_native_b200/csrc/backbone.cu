// Qwen3 backbone decode over the static per-seat KV cache (replaces serve/fast_backbone.py StaticBackbone).
//
// Per layer: [add+]RMSNorm -> QKV linear -> q/k head RMSNorm + RoPE + K/V cache write -> split-KV decode attention
// -> combine -> o linear -> add+RMSNorm -> gate|up linear -> SiLU*up -> down linear.  The rounding points follow
// the reference's fused path (fuse_rope=True): every stored intermediate is bf16, arithmetic is fp32.
#include <algorithm>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"

namespace m3 {

constexpr int kHeadDim = 128;

// ------------------------------------------------------------------------------------------------ row setup
// slot and position of every row, validated once per step (pos = lengths[slot] + offset, read before the step's
// length update as serve/fast_backbone.py:178-179).
__global__ void prep_rows_kernel(const int64_t* __restrict__ slots, const int64_t* __restrict__ offsets,
                                 const int64_t* __restrict__ lengths, int rows, int max_slots, int capacity,
                                 int* __restrict__ slot32, int* __restrict__ pos32, int* status) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  int64_t s = slots[r];
  if (s < 0 || s > max_slots) {
    report(status, M3_DEV_BAD_SLOT);
    s = max_slots;
  }
  int64_t p = lengths[s] + (offsets ? offsets[r] : 0);
  if (p < 0 || p >= capacity) {
    report(status, M3_DEV_BAD_POS);
    p = p < 0 ? 0 : capacity - 1;
  }
  slot32[r] = (int)s;
  pos32[r] = (int)p;
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
        reinterpret_cast<uint4*>(hout + (int64_t)row * n)[c] = pack8(v[it]);
      }
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
  const int head = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
  for (int e = 0; e < 8; ++e) o[e] = rbf(rbf(g[e] / (1.f + expf(-g[e]))) * u[e]);
  reinterpret_cast<uint4*>(act + r * F)[c] = pack8(o);
}

// ------------------------------------------------------------------------------------------------ attention
// Split-KV decode attention over the static cache (replaces _decode_attn, serve/fast_backbone.py:32-58).
//
// Grid (split, kv head, row).  A CTA owns keys [split*chunk, min((split+1)*chunk, pos+1)) of one (row, kv head)
// and serves all G query heads of that kv head, so every K/V byte is read from HBM once.  K and V rows of one
// (slot, head) are contiguous (256 B per token), so each 32-token stage is two 8 KB bulk copies into shared memory,
// kStages deep.  Compute: 4 lanes per token (lane owns 16-byte chunks p, p+4, p+8, p+12 of the head dim), fp32
// dot products, online softmax in the exp2 domain with a warp-uniform running max that is only raised when a new
// score exceeds it by more than 2^8 (the result is exact: the same reference max is used for every term).
constexpr int kStageTok = 32;
constexpr int kStages = 4;
constexpr int kAttnThreads = 128;
constexpr int kTokBytes = kHeadDim * 2;
constexpr float kLazyRescale = 8.f;

template <int G>
struct AttnSmem {
  bf16 k[kStages][kStageTok * kHeadDim];
  bf16 v[kStages][kStageTok * kHeadDim];
  uint64_t bar[kStages];
};

template <int G>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ kc, const bf16* __restrict__ vc, int64_t slot_stride,
    int64_t head_stride, const int* __restrict__ slot32, const int* __restrict__ pos32, float* __restrict__ part_o,
    float2* __restrict__ part_ml, int nsplit, int chunk, int H, float qscale, int* status) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  AttnSmem<G>& sm = *reinterpret_cast<AttnSmem<G>*>(smem_raw);
  const int split = blockIdx.x, kvh = blockIdx.y, row = blockIdx.z;
  const int KV = gridDim.y;
  const int pos = pos32[row];
  const int t0 = split * chunk;
  if (t0 > pos) return;
  const int ntok = min(chunk, pos + 1 - t0);
  const int nst = cdiv(ntok, kStageTok);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tl = warp * 8 + (lane >> 2), p = lane & 3;
  const int64_t base = (int64_t)slot32[row] * slot_stride + (int64_t)kvh * head_stride + (int64_t)t0 * kHeadDim;
  const bf16* kg = kc + base;
  const bf16* vg = vc + base;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&sm.bar[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int st) {
    const int n = min(kStageTok, ntok - st * kStageTok);
    const uint32_t bytes = (uint32_t)n * kTokBytes;
    uint64_t* bar = &sm.bar[st % kStages];
    mbar_expect_tx(bar, 2 * bytes);
    bulk_g2s(sm.k[st % kStages], kg + (int64_t)st * kStageTok * kHeadDim, bytes, bar);
    bulk_g2s(sm.v[st % kStages], vg + (int64_t)st * kStageTok * kHeadDim, bytes, bar);
  };
  int issued = min(kStages, nst);  // meaningful in thread 0 only
  if (tid == 0)
    for (int st = 0; st < issued; ++st) issue(st);

  // this thread's slice of the G query heads, pre-scaled into the exp2 domain
  float qr[G][4][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const uint4* qp = reinterpret_cast<const uint4*>(q + ((int64_t)row * H + kvh * G + g) * kHeadDim);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      unpack8(qp[p + 4 * j], qr[g][j]);
#pragma unroll
      for (int e = 0; e < 8; ++e) qr[g][j][e] *= qscale;
    }
  }
  float m[G], l[G], acc[G][4][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[g][j][e] = 0.f;
  }

  bool timed_out = false;
  for (int st = 0; st < nst; ++st) {
    const int buf = st % kStages;
    const bool got = mbar_wait(&sm.bar[buf], (st / kStages) & 1, status);
    if (got) {
      const bool valid = st * kStageTok + tl < ntok;
      const uint4* krow = reinterpret_cast<const uint4*>(sm.k[buf] + tl * kHeadDim);
      float s[G];
#pragma unroll
      for (int g = 0; g < G; ++g) s[g] = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float kf[8];
        unpack8(krow[p + 4 * j], kf);
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int e = 0; e < 8; ++e) s[g] = fmaf(qr[g][j][e], kf[e], s[g]);
      }
      float pg[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        s[g] += __shfl_xor_sync(0xffffffffu, s[g], 1);
        s[g] += __shfl_xor_sync(0xffffffffu, s[g], 2);
        s[g] = valid ? s[g] : -INFINITY;
        float mx = fmaxf(s[g], __shfl_xor_sync(0xffffffffu, s[g], 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        if (mx > m[g] + kLazyRescale) {  // warp-uniform
          const float r = exp2f(m[g] - mx);
          m[g] = mx;
          l[g] *= r;
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[g][j][e] *= r;
        }
        pg[g] = valid ? exp2f(s[g] - m[g]) : 0.f;
        l[g] += pg[g];
      }
      if (valid) {
        const uint4* vrow = reinterpret_cast<const uint4*>(sm.v[buf] + tl * kHeadDim);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float vf[8];
          unpack8(vrow[p + 4 * j], vf);
#pragma unroll
          for (int g = 0; g < G; ++g)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[g][j][e] = fmaf(pg[g], vf[e], acc[g][j][e]);
        }
      }
    }
    if (__syncthreads_or(!got)) {
      timed_out = true;
      break;
    }
    if (tid == 0 && st + kStages < nst) issue(issued++);
  }
  if (timed_out) {
    // drain the copies still in flight (bounded) before the CTA's shared memory is released
    if (tid == 0)
      for (int st = max(0, issued - kStages); st < issued; ++st)
        mbar_wait(&sm.bar[st % kStages], (st / kStages) & 1, nullptr);
    __syncthreads();
    return;
  }

  // reduce over the 8 token groups of the warp (lanes with equal p share dims; m is warp-uniform)
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      l[g] += __shfl_xor_sync(0xffffffffu, l[g], o);
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][j][e] += __shfl_xor_sync(0xffffffffu, acc[g][j][e], o);
    }
  }
  // cross-warp merge through shared memory (the stage buffers are free now)
  float* wacc = reinterpret_cast<float*>(sm.k[0]);            // [4 warps][G][128]
  float* wml = wacc + 4 * G * kHeadDim;                        // [4 warps][G][2]
  if (lane < 4) {
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) wacc[(warp * G + g) * kHeadDim + (p + 4 * j) * 8 + e] = acc[g][j][e];
    if (lane == 0)
#pragma unroll
      for (int g = 0; g < G; ++g) {
        wml[(warp * G + g) * 2] = m[g];
        wml[(warp * G + g) * 2 + 1] = l[g];
      }
  }
  __syncthreads();
  const int64_t pidx = ((int64_t)row * KV + kvh) * nsplit + split;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, wml[(w * G + g) * 2]);
    float O = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = wml[(w * G + g) * 2];
      const float sc = mw == -INFINITY ? 0.f : exp2f(mw - M);
      O = fmaf(wacc[(w * G + g) * kHeadDim + tid], sc, O);
      L = fmaf(wml[(w * G + g) * 2 + 1], sc, L);
    }
    part_o[(pidx * G + g) * kHeadDim + tid] = O;
    if (tid == 0) part_ml[pidx * G + g] = make_float2(M, L);
  }
}

// Merge the splits of one (row, kv head): out = sum_s O_s 2^(m_s - M) / sum_s L_s 2^(m_s - M), rounded to bf16.
template <int G>
__global__ void __launch_bounds__(kHeadDim) attn_combine_kernel(const float* __restrict__ part_o,
                                                                const float2* __restrict__ part_ml,
                                                                const int* __restrict__ pos32, bf16* __restrict__ out,
                                                                int nsplit, int chunk, int H) {
  const int kvh = blockIdx.x, row = blockIdx.y, KV = gridDim.x, d = threadIdx.x;
  const int n = min(nsplit, pos32[row] / chunk + 1);
  const int64_t pbase = ((int64_t)row * KV + kvh) * nsplit;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float M = -INFINITY;
    for (int s = 0; s < n; ++s) M = fmaxf(M, part_ml[(pbase + s) * G + g].x);
    float O = 0.f, L = 0.f;
    for (int s = 0; s < n; ++s) {
      const float2 ml = part_ml[(pbase + s) * G + g];
      const float sc = exp2f(ml.x - M);
      O = fmaf(part_o[((pbase + s) * G + g) * kHeadDim + d], sc, O);
      L = fmaf(ml.y, sc, L);
    }
    out[((int64_t)row * H + kvh * G + g) * kHeadDim + d] = to_bf(O / L);
  }
}

}  // namespace m3

// ================================================================================================ handle
using namespace m3;

struct m3_backbone {
  m3_backbone_config c{};
  std::vector<const bf16*> in_norm, wqkv, q_norm, k_norm, wo, post_norm, wgu, wdown;
  std::vector<bf16*> kc, vc;
  const bf16* final_norm = nullptr;
  const bf16* cos = nullptr;
  const bf16* sin = nullptr;
  int64_t* lengths = nullptr;
  int max_split = 16;
  // scratch
  void* ws = nullptr;
  int* slot32 = nullptr;
  int* pos32 = nullptr;
  int* status = nullptr;
  bf16 *h = nullptr, *y = nullptr, *qkv = nullptr, *q = nullptr, *o = nullptr, *a = nullptr, *gu = nullptr,
       *act = nullptr;
  float* part_o = nullptr;
  float2* part_ml = nullptr;
};

namespace {

template <class T>
T* carve(char*& p, size_t count) {
  T* r = reinterpret_cast<T*>(p);
  p += (count * sizeof(T) + 255) / 256 * 256;
  return r;
}

// Keys per split: enough CTAs to fill the GPU a couple of times over, at most max_split splits, a power of two
// between 64 and 512 (a multiple of the 32-token stage).
int choose_chunk(int rows, int ctx, int kv, int max_split) {
  int chunk = 512;
  while (chunk > 64 && (int64_t)rows * kv * cdiv(ctx, chunk) < 2 * 148 * 3) chunk /= 2;
  while (cdiv(ctx, chunk) > max_split) chunk *= 2;
  return chunk;
}

int attn_smem_bytes(int G) {
  switch (G) {
    case 1: return sizeof(AttnSmem<1>);
    case 2: return sizeof(AttnSmem<2>);
    default: return sizeof(AttnSmem<4>);
  }
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
  bb->final_norm = (const bf16*)w->final_norm;
  bb->cos = (const bf16*)w->cos;
  bb->sin = (const bf16*)w->sin;
  bb->lengths = w->lengths;
  bb->max_split = std::max(16, cdiv(c.capacity, 512));
  const int R = c.max_rows, Hd = c.hidden, qkvw = (c.heads + 2 * c.kv_heads) * c.head_dim;
  const size_t parts = (size_t)R * c.kv_heads * bb->max_split * G;
  size_t bytes = 0;
  auto add = [&](size_t n) { bytes += (n + 255) / 256 * 256; };
  add(R * 4); add(R * 4); add(256);
  add((size_t)R * Hd * 2); add((size_t)R * Hd * 2); add((size_t)R * qkvw * 2);
  add((size_t)R * c.heads * c.head_dim * 2); add((size_t)R * c.heads * c.head_dim * 2); add((size_t)R * Hd * 2);
  add((size_t)R * 2 * c.ffn * 2); add((size_t)R * c.ffn * 2);
  add(parts * kHeadDim * 4); add(parts * 8);
  cudaError_t e = cudaMalloc(&bb->ws, bytes);
  if (e != cudaSuccess) {
    delete bb;
    set_error("m3_backbone_create: cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
    return M3_ERR_CUDA;
  }
  char* p = (char*)bb->ws;
  bb->slot32 = carve<int>(p, R);
  bb->pos32 = carve<int>(p, R);
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
  if (cudaMemset(bb->status, 0, 256) != cudaSuccess) {
    cudaFree(bb->ws);
    delete bb;
    set_error("m3_backbone_create: memset failed");
    return M3_ERR_CUDA;
  }
  const int smem = attn_smem_bytes(G);
  cudaFuncSetAttribute(attn_split_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(AttnSmem<1>));
  cudaFuncSetAttribute(attn_split_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(AttnSmem<2>));
  cudaFuncSetAttribute(attn_split_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, sizeof(AttnSmem<4>));
  (void)smem;
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

static int attention(m3_backbone* bb, int layer, int rows, int ctx, cudaStream_t s) {
  const m3_backbone_config& c = bb->c;
  const int G = c.heads / c.kv_heads;
  const int chunk = choose_chunk(rows, ctx, c.kv_heads, bb->max_split);
  const int nsplit = cdiv(ctx, chunk);
  const int64_t head_stride = (int64_t)c.capacity * c.head_dim;
  const int64_t slot_stride = (int64_t)c.kv_heads * head_stride;
  const float qscale = (1.f / sqrtf((float)c.head_dim)) * 1.4426950408889634f;
  dim3 grid(nsplit, c.kv_heads, rows);
#define M3_ATTN(GG)                                                                                          \
  attn_split_kernel<GG><<<grid, kAttnThreads, sizeof(AttnSmem<GG>), s>>>(                                    \
      bb->q, bb->kc[layer], bb->vc[layer], slot_stride, head_stride, bb->slot32, bb->pos32, bb->part_o,     \
      bb->part_ml, nsplit, chunk, c.heads, qscale, bb->status);                                             \
  M3_LAUNCHED();                                                                                             \
  attn_combine_kernel<GG><<<dim3(c.kv_heads, rows), kHeadDim, 0, s>>>(bb->part_o, bb->part_ml, bb->pos32,   \
                                                                      bb->o, nsplit, chunk, c.heads);
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
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int Hd = c.hidden, qkvw = (c.heads + 2 * c.kv_heads) * c.head_dim;
  const int norm_threads = std::min(1024, std::max(32, (Hd / 8 + 31) / 32 * 32));
  prep_rows_kernel<<<cdiv(rows, 128), 128, 0, s>>>(slots, offsets, bb->lengths, rows, c.max_slots, c.capacity,
                                                   bb->slot32, bb->pos32, bb->status);
  M3_LAUNCHED();
  const bf16* xin = reinterpret_cast<const bf16*>(x);
  for (int i = 0; i < c.layers; ++i) {
    if (i == 0) {
      // h = x; y = RMSNorm(x) (HF Qwen3RMSNorm module on the first layer)
      M3_CUDA(cudaMemcpyAsync(bb->h, xin, (size_t)rows * Hd * 2, cudaMemcpyDeviceToDevice, s));
      add_rms_kernel<<<rows, norm_threads, 0, s>>>(bb->h, nullptr, nullptr, bb->y, bb->in_norm[0], c.eps, Hd);
    } else {
      add_rms_kernel<<<rows, norm_threads, 0, s>>>(bb->h, bb->a, bb->h, bb->y, bb->in_norm[i], c.eps, Hd);
    }
    M3_LAUNCHED();
    M3_TRY(gemm({bb->y, Hd, bb->wqkv[i], Hd, bb->qkv, qkvw, rows, qkvw, Hd, false}, s));
    qk_rope_cache_kernel<<<rows, 32 * (c.heads + c.kv_heads), 0, s>>>(
        bb->qkv, bb->q, bb->kc[i], bb->vc[i], (int64_t)c.kv_heads * c.capacity * c.head_dim,
        (int64_t)c.capacity * c.head_dim, bb->slot32, bb->pos32, bb->cos, bb->sin, bb->q_norm[i], bb->k_norm[i],
        c.eps, c.heads, c.kv_heads);
    M3_LAUNCHED();
    M3_TRY(attention(bb, i, rows, ctx, s));
    M3_TRY(gemm({bb->o, c.heads * c.head_dim, bb->wo[i], c.heads * c.head_dim, bb->a, Hd, rows, Hd,
                 c.heads * c.head_dim, false},
                s));
    add_rms_kernel<<<rows, norm_threads, 0, s>>>(bb->h, bb->a, bb->h, bb->y, bb->post_norm[i], c.eps, Hd);
    M3_LAUNCHED();
    M3_TRY(gemm({bb->y, Hd, bb->wgu[i], Hd, bb->gu, 2 * c.ffn, rows, 2 * c.ffn, Hd, false}, s));
    const int64_t nv = (int64_t)rows * (c.ffn / 8);
    silu_mul_kernel<<<(unsigned)((nv + 255) / 256), 256, 0, s>>>(bb->gu, bb->act, rows, c.ffn);
    M3_LAUNCHED();
    M3_TRY(gemm({bb->act, c.ffn, bb->wdown[i], c.ffn, bb->a, Hd, rows, Hd, c.ffn, false}, s));
  }
  add_rms_kernel<<<rows, norm_threads, 0, s>>>(bb->h, bb->a, bb->h, reinterpret_cast<bf16*>(out), bb->final_norm,
                                               c.eps, Hd);
  M3_LAUNCHED();
  lengths_add_kernel<<<cdiv(rows, 128), 128, 0, s>>>(bb->slot32, real, rows, bb->lengths);
  M3_LAUNCHED();
  return M3_OK;
}

extern "C" int m3_backbone_attention(m3_backbone* bb, int32_t layer, int32_t rows, int32_t ctx, m3_stream stream) {
  M3_REQUIRE(bb, M3_ERR_ARG, "m3_backbone_attention: null handle");
  M3_REQUIRE(layer >= 0 && layer < bb->c.layers && rows > 0 && rows <= bb->c.max_rows && ctx > 0 &&
                 ctx <= bb->c.capacity,
             M3_ERR_RANGE, "m3_backbone_attention: layer %d rows %d ctx %d out of range", layer, rows, ctx);
  return attention(bb, layer, rows, ctx, reinterpret_cast<cudaStream_t>(stream));
}
