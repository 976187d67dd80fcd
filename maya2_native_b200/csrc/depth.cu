// Depth transformer: the per-frame RVQ level loop (replaces serve/fast_depth.py FastDepth with its fused kernels
// serve/fast_depth_kernels.py) plus the backbone feedback embed (tts/model/audio_io.py:27-35).
//
// For each level l (1..n_q-1) the level's weight group runs its 4 pre-norm layers over the prefix [proj(h)+lvl0,
// emb(cb0), ..., emb(cb_{l-1})] (or, inside a shared group, incrementally over the one new position against the
// group's stored K/V), the last layer only for the final position; then LayerNorm, the level head and the top-k
// sampler, whose kernel also writes the next prefix row.  All rows of the seat batch go through each linear layer
// together, so the weights are read once per level for every seat.
#include <algorithm>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"
#include "mma.cuh"
#include "ops.cuh"
#include "sampler.cuh"

namespace m3 {

// ------------------------------------------------------------------------------------------------ row setup
__global__ void depth_prep_kernel(const int64_t* __restrict__ slots, const int64_t* __restrict__ cb0, int rows,
                                  int max_slots, int n_codes, int* __restrict__ slot32, int* __restrict__ cb032,
                                  int64_t* __restrict__ codes, int n_q, int* status) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  int64_t s = slots[r];
  if (s < 0 || s > max_slots) {
    report(status, M3_DEV_BAD_SLOT);
    s = max_slots;
  }
  int64_t c = cb0[r];
  if (c < 0 || c >= n_codes) {
    report(status, M3_DEV_BAD_CODE);
    c = c < 0 ? 0 : n_codes - 1;
  }
  slot32[r] = (int)s;
  cb032[r] = (int)c;
  codes[(int64_t)r * n_q] = cb0[r];
}

// prefix[:, 0] = bf16(in_proj(h) + level0); prefix[:, 1] = embed[0][cb0]   (serve/fast_depth.py:149-151)
__global__ void prefix_init_kernel(const bf16* __restrict__ proj, const bf16* __restrict__ level0,
                                   const bf16* __restrict__ embed0, const int* __restrict__ cb032,
                                   bf16* __restrict__ prefix, int NL, int D) {
  const int r = blockIdx.x;
  bf16* p = prefix + (int64_t)r * NL * D;
  const uint4* e = reinterpret_cast<const uint4*>(embed0 + (int64_t)cb032[r] * D);
  for (int i = threadIdx.x; i < D / 8; i += blockDim.x) {
    float a[8], b[8];
    unpack8(reinterpret_cast<const uint4*>(proj + (int64_t)r * D)[i], a);
    unpack8(reinterpret_cast<const uint4*>(level0)[i], b);
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = a[k] + b[k];
    reinterpret_cast<uint4*>(p)[i] = pack8(a);
    reinterpret_cast<uint4*>(p + D)[i] = e[i];
  }
}

// ------------------------------------------------------------------------------------------------ LayerNorm
// Row r of the input lives at src + (r / T) * sb + (r % T) * st (elements); optional residual add(s):
// x' = bf16(x + a) then x' = bf16(x' + c[slot]) (serve/fast_depth_kernels.py:280-283), stored to xout (contiguous);
// y = bf16((x' - mean) / sqrt(var + eps) * w + b) with fp32 statistics (:284-289).
__global__ void add_ln_kernel(const bf16* __restrict__ src, int T, int64_t sb, int64_t st,
                              const bf16* __restrict__ a, const bf16* __restrict__ c, int64_t c_slot_stride,
                              const int* __restrict__ slot32, bf16* __restrict__ xout, bf16* __restrict__ y,
                              const bf16* __restrict__ w, const bf16* __restrict__ bias, float eps, int D) {
  __shared__ float red[32];
  const int r = blockIdx.x;
  const int nv = D / 8;
  const bf16* xr = src + (int64_t)(r / T) * sb + (int64_t)(r % T) * st;
  constexpr int kMaxPer = 4;
  float v[kMaxPer][8];
  float sum = 0.f;
#pragma unroll
  for (int it = 0; it < kMaxPer; ++it) {
    const int i = threadIdx.x + it * blockDim.x;
    if (i < nv) {
      unpack8(reinterpret_cast<const uint4*>(xr)[i], v[it]);
      if (a) {
        float av[8];
        unpack8(reinterpret_cast<const uint4*>(a + (int64_t)r * D)[i], av);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[it][e] = rbf(v[it][e] + av[e]);
      }
      if (c) {
        float cv[8];
        unpack8(reinterpret_cast<const uint4*>(c + (int64_t)slot32[r / T] * c_slot_stride)[i], cv);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[it][e] = rbf(v[it][e] + cv[e]);
      }
      if (xout) reinterpret_cast<uint4*>(xout + (int64_t)r * D)[i] = pack8(v[it]);
#pragma unroll
      for (int e = 0; e < 8; ++e) sum += v[it][e];
    }
  }
  const float mean = block_sum(sum, red) / (float)D;
  float sq = 0.f;
#pragma unroll
  for (int it = 0; it < kMaxPer; ++it) {
    const int i = threadIdx.x + it * blockDim.x;
    if (i < nv)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = v[it][e] - mean;
        sq = fmaf(d, d, sq);
      }
  }
  const float var = block_sum(sq, red) / (float)D;
  const float den = sqrtf(var + eps);
#pragma unroll
  for (int it = 0; it < kMaxPer; ++it) {
    const int i = threadIdx.x + it * blockDim.x;
    if (i < nv) {
      float wv[8], bv[8], o[8];
      unpack8(reinterpret_cast<const uint4*>(w)[i], wv);
      unpack8(reinterpret_cast<const uint4*>(bias)[i], bv);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = (v[it][e] - mean) / den * wv[e] + bv[e];
      reinterpret_cast<uint4*>(y + (int64_t)r * D)[i] = pack8(o);
    }
  }
}

int launch_add_ln(int rows, const bf16* src, int T, int64_t sb, int64_t st, const bf16* a, const bf16* c,
                  int64_t c_slot_stride, const int* slot32, bf16* xout, bf16* y, const bf16* w, const bf16* bias,
                  float eps, int D, cudaStream_t s) {
  if (rows <= 0) return M3_OK;
  add_ln_kernel<<<rows, norm_block(D), 0, s>>>(src, T, sb, st, a, c, c_slot_stride, slot32, xout, y, w, bias, eps, D);
  M3_LAUNCHED();
  return M3_OK;
}

// ------------------------------------------------------------------------------------------------ attention
// Tiny attention over at most kMaxKeys positions: query i of seat b sits at absolute position q0 + i and sees keys
// 0..q0+i (causal; the last-position and incremental forms are q0 = n-1 with one query).  One warp per
// (seat, head, query), each lane holding PER consecutive dims; keys go in batches of 8 whose K and V loads are all
// in flight together (the kernel is load-latency bound); fp32 scores with an online softmax over the batches, output
// rounded once (F.scaled_dot_product_attention).
constexpr int kMaxKeys = 64;

struct KeySrc {
  const bf16* k;  // key of (b, j, head h) at k + b*sb + j*sj + h*hd
  const bf16* v;
  int64_t sb, sj;
};

template <int PER>
__device__ __forceinline__ void load_per(const bf16* p, float* f) {
  if constexpr (PER == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    f[0] = bf_lo(u.x); f[1] = bf_hi(u.x); f[2] = bf_lo(u.y); f[3] = bf_hi(u.y);
  } else if constexpr (PER == 2) {
    const uint32_t u = *reinterpret_cast<const uint32_t*>(p);
    f[0] = bf_lo(u); f[1] = bf_hi(u);
  } else {
    f[0] = to_f(*p);
  }
}

template <int PER>
__global__ void depth_attn_kernel(const bf16* __restrict__ qkv, int T, int q0, int Tq, KeySrc ks, int H,
                                  float scale, bf16* __restrict__ out) {
  constexpr int HD = 32 * PER;
  constexpr int KB = 8;  // keys per batch: their loads are all issued before the first dot product
  const int b = blockIdx.x, h = blockIdx.y;
  const int i = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (i >= Tq) return;
  const int D = H * HD;
  const int qp = q0 + i;
  const int nk = min(qp + 1, kMaxKeys);
  const bf16* q = qkv + ((int64_t)b * T + (T - Tq) + i) * 3 * D + (int64_t)h * HD + lane * PER;
  float qv[PER], o[PER];
  load_per<PER>(q, qv);
#pragma unroll
  for (int e = 0; e < PER; ++e) o[e] = 0.f;
  float m = -INFINITY, l = 0.f;
  const bf16* kb = ks.k + (int64_t)b * ks.sb + (int64_t)h * HD + lane * PER;
  const bf16* vb = ks.v + (int64_t)b * ks.sb + (int64_t)h * HD + lane * PER;
  for (int j0 = 0; j0 < nk; j0 += KB) {
    float kf[KB][PER], vf[KB][PER], d[KB];
#pragma unroll
    for (int jj = 0; jj < KB; ++jj) {
      const int j = min(j0 + jj, nk - 1);  // past the last key: reload it, masked below
      load_per<PER>(kb + (int64_t)j * ks.sj, kf[jj]);
      load_per<PER>(vb + (int64_t)j * ks.sj, vf[jj]);
    }
#pragma unroll
    for (int jj = 0; jj < KB; ++jj) {
      d[jj] = 0.f;
#pragma unroll
      for (int e = 0; e < PER; ++e) d[jj] = fmaf(qv[e], kf[jj][e], d[jj]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int jj = 0; jj < KB; ++jj) d[jj] += __shfl_xor_sync(0xffffffffu, d[jj], off);
    float mb = m;
#pragma unroll
    for (int jj = 0; jj < KB; ++jj) {
      d[jj] = j0 + jj < nk ? d[jj] * scale : -INFINITY;
      mb = fmaxf(mb, d[jj]);
    }
    const float c = expf(m - mb);  // m = -inf on the first batch: c = 0
    l *= c;
#pragma unroll
    for (int e = 0; e < PER; ++e) o[e] *= c;
#pragma unroll
    for (int jj = 0; jj < KB; ++jj) {
      const float p = j0 + jj < nk ? expf(d[jj] - mb) : 0.f;
      l += p;
#pragma unroll
      for (int e = 0; e < PER; ++e) o[e] = fmaf(p, vf[jj][e], o[e]);
    }
    m = mb;
  }
  bf16* dst = out + ((int64_t)b * Tq + i) * D + (int64_t)h * HD + lane * PER;
#pragma unroll
  for (int e = 0; e < PER; ++e) dst[e] = to_bf(o[e] / l);
}

// The same attention on the tensor cores for head dim 128 and at most 16 queries and 16 keys: one warp per
// (seat, head).  K and V rows are staged in shared memory (row stride padded to 272 B, so ldmatrix reads are
// conflict-free; rows past the last key are zero), Q fragments come straight from global memory; S = Q K^T is 8
// mma (queries as rows), an exact softmax per query over its visible keys, O = P V with P split into bf16 hi + lo
// (fp32-accurate weights) is 32 mma, O / sum rounded once.
constexpr int kDaRow = 128 + 8;  // staged row stride in elements

__global__ void __launch_bounds__(32) depth_attn_mma_kernel(const bf16* __restrict__ qkv, int T, int q0, int Tq,
                                                            KeySrc ks, int H, float scale, bf16* __restrict__ out) {
  __shared__ __align__(16) bf16 Ks[16 * kDaRow];
  __shared__ __align__(16) bf16 Vs[16 * kDaRow];
  const int b = blockIdx.x, h = blockIdx.y, lane = threadIdx.x, g = lane >> 2, t = lane & 3;
  const int D = H * 128;
  const int nk = q0 + Tq;  // keys 0 .. q0 + Tq - 1 (the last query sees them all)
  const bf16* kb = ks.k + (int64_t)b * ks.sb + (int64_t)h * 128;
  const bf16* vb = ks.v + (int64_t)b * ks.sb + (int64_t)h * 128;
  for (int i = lane; i < 16 * 16; i += 32) {  // 16 rows x 16 chunks of 16 B
    const int j = i >> 4, c = i & 15;
    uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = kv;
    if (j < nk) {
      kv = reinterpret_cast<const uint4*>(kb + (int64_t)j * ks.sj)[c];
      vv = reinterpret_cast<const uint4*>(vb + (int64_t)j * ks.sj)[c];
    }
    *reinterpret_cast<uint4*>(Ks + j * kDaRow + c * 8) = kv;
    *reinterpret_cast<uint4*>(Vs + j * kDaRow + c * 8) = vv;
  }
  // Q fragments: rows g and g + 8 are queries (zero past Tq)
  const bool va = g < Tq, vbq = g + 8 < Tq;
  const uint32_t* qa = reinterpret_cast<const uint32_t*>(qkv + ((int64_t)b * T + (T - Tq) + (va ? g : 0)) * 3 * D +
                                                         (int64_t)h * 128);
  const uint32_t* qb = reinterpret_cast<const uint32_t*>(qkv + ((int64_t)b * T + (T - Tq) + (vbq ? g + 8 : 0)) * 3 *
                                                         D + (int64_t)h * 128);
  __syncwarp();
  const int jm = lane >> 3;
  float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint32_t a0 = va ? qa[8 * kk + t] : 0u, a2 = va ? qa[8 * kk + 4 + t] : 0u;
    const uint32_t a1 = vbq ? qb[8 * kk + t] : 0u, a3 = vbq ? qb[8 * kk + 4 + t] : 0u;
    uint32_t k0, k1, k2, k3;  // B = K^T: matrices (keys 0-7 | 8-15) x (dims 16kk.. | 16kk+8..)
    ldsm_x4(smem_u32(Ks + (((jm >> 1) << 3) + (lane & 7)) * kDaRow + 16 * kk + (jm & 1) * 8), k0, k1, k2, k3);
    mma_bf16(sc[0], a0, a1, a2, a3, k0, k1);
    mma_bf16(sc[1], a0, a1, a2, a3, k2, k3);
  }
  // exact softmax per query row over its visible keys (key j visible to query i iff j <= q0 + i)
  float p[2][4], mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int j = nt * 8 + 2 * t + e;
      p[nt][e] = (va && j <= q0 + g) ? sc[nt][e] * scale : -INFINITY;
      p[nt][2 + e] = (vbq && j <= q0 + g + 8) ? sc[nt][2 + e] * scale : -INFINITY;
      mxa = fmaxf(mxa, p[nt][e]);
      mxb = fmaxf(mxb, p[nt][2 + e]);
    }
  mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
  mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
  mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
  mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
  float la = 0.f, lb = 0.f;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      p[nt][e] = p[nt][e] == -INFINITY ? 0.f : expf(p[nt][e] - mxa);
      p[nt][2 + e] = p[nt][2 + e] == -INFINITY ? 0.f : expf(p[nt][2 + e] - mxb);
      la += p[nt][e];
      lb += p[nt][2 + e];
    }
  la += __shfl_xor_sync(0xffffffffu, la, 1);
  la += __shfl_xor_sync(0xffffffffu, la, 2);
  lb += __shfl_xor_sync(0xffffffffu, lb, 1);
  lb += __shfl_xor_sync(0xffffffffu, lb, 2);
  // A = P (queries x keys): a0 = (g, keys 2t..) n-tile 0 c0c1; a1 = (g+8, ..) c2c3; a2/a3 the same of n-tile 1
  uint32_t ph[4], pl[4];
  const float pv[4][2] = {{p[0][0], p[0][1]}, {p[0][2], p[0][3]}, {p[1][0], p[1][1]}, {p[1][2], p[1][3]}};
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    ph[r] = pack_bf2(pv[r][0], pv[r][1]);
    pl[r] = pack_bf2(pv[r][0] - bf_lo_f(ph[r]), pv[r][1] - bf_hi_f(ph[r]));
  }
  const float ia = la > 0.f ? 1.f / la : 0.f, ib = lb > 0.f ? 1.f / lb : 0.f;
  bf16* oa = out + ((int64_t)b * Tq + g) * D + (int64_t)h * 128;
  bf16* ob = out + ((int64_t)b * Tq + g + 8) * D + (int64_t)h * 128;
#pragma unroll
  for (int dt = 0; dt < 8; ++dt) {  // 16 dims per ldmatrix.trans x4: B = V (keys x dims)
    uint32_t v0, v1, v2, v3;  // matrices (keys 0-7 | 8-15) x (dims 16dt.. | 16dt+8..)
    ldsm_x4_t(smem_u32(Vs + ((jm & 1) * 8 + (lane & 7)) * kDaRow + 16 * dt + (jm >> 1) * 8), v0, v1, v2, v3);
    float o0[4] = {0.f, 0.f, 0.f, 0.f}, o1[4] = {0.f, 0.f, 0.f, 0.f};
    mma_bf16(o0, ph[0], ph[1], ph[2], ph[3], v0, v1);
    mma_bf16(o0, pl[0], pl[1], pl[2], pl[3], v0, v1);
    mma_bf16(o1, ph[0], ph[1], ph[2], ph[3], v2, v3);
    mma_bf16(o1, pl[0], pl[1], pl[2], pl[3], v2, v3);
    const int d0 = 16 * dt + 2 * t, d1 = d0 + 8;
    if (va) {
      *reinterpret_cast<uint32_t*>(oa + d0) = pack_bf2(o0[0] * ia, o0[1] * ia);
      *reinterpret_cast<uint32_t*>(oa + d1) = pack_bf2(o1[0] * ia, o1[1] * ia);
    }
    if (vbq) {
      *reinterpret_cast<uint32_t*>(ob + d0) = pack_bf2(o0[2] * ib, o0[3] * ib);
      *reinterpret_cast<uint32_t*>(ob + d1) = pack_bf2(o1[2] * ib, o1[3] * ib);
    }
  }
}

// kvbuf[b, p0 + t] = (k, v) of qkv rows t of b  (serve/fast_depth.py:170,176)
__global__ void kv_store_kernel(const bf16* __restrict__ qkv, int T, bf16* __restrict__ kv, int NL, int p0, int D) {
  const int b = blockIdx.x, t = blockIdx.y;
  const uint4* src = reinterpret_cast<const uint4*>(qkv + ((int64_t)b * T + t) * 3 * D + D);
  uint4* dst = reinterpret_cast<uint4*>(kv + ((int64_t)b * NL + p0 + t) * 2 * D);
  for (int i = threadIdx.x; i < 2 * D / 8; i += blockDim.x) dst[i] = src[i];
}


// act = bf16(gelu_erf(f))   (F.gelu on the depth dtype)
__global__ void gelu_kernel(bf16* __restrict__ f, int64_t n8) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  float v[8];
  unpack8(reinterpret_cast<const uint4*>(f)[i], v);
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = gelu_erf(v[e]);
  reinterpret_cast<uint4*>(f)[i] = pack8(v);
}

__global__ void ctr_advance_kernel(const int* __restrict__ slot32, int rows, int32_t* __restrict__ ctr) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < rows) atomicAdd(reinterpret_cast<int*>(ctr + slot32[r]), 1);
}

// feedback = RMSNorm(bf16(bf16(sum_k table[code_k + k n_codes]) / sqrt(n_q))), fp32 epsilon (nn.RMSNorm eps=None)
// (tts/model/audio_io.py:33-35 as inlined at serve/fast_depth.py:200-202).
__global__ void feedback_kernel(const int64_t* __restrict__ codes, int NL, int n_codes,
                                const bf16* __restrict__ table, const bf16* __restrict__ w, int D, float inv_scale_div,
                                bf16* __restrict__ out, int* status) {
  __shared__ float red[32];
  __shared__ int cs[64];
  const int r = blockIdx.x;
  for (int k = threadIdx.x; k < NL; k += blockDim.x) {
    int64_t c = codes[(int64_t)r * NL + k];
    if (c < 0 || c >= n_codes) {
      report(status, M3_DEV_BAD_CODE);
      c = c < 0 ? 0 : n_codes - 1;
    }
    cs[k] = (int)c + k * n_codes;
  }
  __syncthreads();
  constexpr int kMaxPer = 4;
  float v[kMaxPer][8];
  float ss = 0.f;
  const int nv = D / 8;
#pragma unroll
  for (int it = 0; it < kMaxPer; ++it) {
    const int i = threadIdx.x + it * blockDim.x;
    if (i < nv) {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[it][e] = 0.f;
      for (int k = 0; k < NL; ++k) {
        float t[8];
        unpack8(reinterpret_cast<const uint4*>(table + (int64_t)cs[k] * D)[i], t);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[it][e] += t[e];
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v[it][e] = rbf(rbf(v[it][e]) / inv_scale_div);
        ss = fmaf(v[it][e], v[it][e], ss);
      }
    }
  }
  ss = block_sum(ss, red);
  const float inv = 1.f / sqrtf(ss / (float)D + 1.1920928955078125e-07f);
#pragma unroll
  for (int it = 0; it < kMaxPer; ++it) {
    const int i = threadIdx.x + it * blockDim.x;
    if (i < nv) {
      float wv[8], o[8];
      unpack8(reinterpret_cast<const uint4*>(w)[i], wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[it][e] * inv * wv[e];
      reinterpret_cast<uint4*>(out + (int64_t)r * D)[i] = pack8(o);
    }
  }
}

}  // namespace m3

// ================================================================================================ handle
using namespace m3;

struct m3_depth {
  m3_depth_config c{};
  const bf16 *in_proj = nullptr, *embed = nullptr, *level0 = nullptr, *norm_w = nullptr, *norm_b = nullptr;
  std::vector<const bf16*> n1_w, n1_b, n2_w, n2_b, qkv, o, f1, f2, heads, cross_kv, cross_o;
  const bf16 *audio_table = nullptr, *audio_norm = nullptr;
  bf16* cross_const = nullptr;
  int32_t *row_seed = nullptr, *row_ctr = nullptr;
  void* ws = nullptr;
  int *slot32 = nullptr, *cb032 = nullptr, *status = nullptr;
  bf16 *prefix = nullptr, *x = nullptr, *x2 = nullptr, *y = nullptr, *qkvb = nullptr, *a = nullptr, *ob = nullptr,
       *ff = nullptr, *logits = nullptr, *proj = nullptr, *kvbuf = nullptr, *spk = nullptr;
  bf16* dbg_logits = nullptr;  // m3_depth_debug_logits: every level's head output kept for inspection
  // the handle's own cuBLAS workspace: two depth handles may run their level loops on two streams at once
  unsigned char* blas_ws = nullptr;
};

// Every GEMM of the level loop runs on the handle's own cuBLAS workspace.
static int dgemm(const m3_depth* d, GemmDesc g, cudaStream_t s) {
  g.ws = d->blas_ws;
  g.ws_bytes = kBlasWorkspace;
  return gemm(g, s);
}

namespace {
template <class T>
T* carve(char*& p, size_t count) {
  T* r = reinterpret_cast<T*>(p);
  p += (count * sizeof(T) + 255) / 256 * 256;
  return r;
}
int norm_threads(int D) { return std::min(1024, std::max(32, (D / 8 + 31) / 32 * 32)); }
}  // namespace

extern "C" int m3_depth_create(const m3_depth_config* cfg, const m3_depth_weights* w, m3_depth** out) {
  M3_REQUIRE(cfg && w && out, M3_ERR_ARG, "m3_depth_create: null argument");
  const m3_depth_config& c = *cfg;
  M3_REQUIRE(c.n_q >= 2 && c.n_q <= 64 && c.n_q <= kMaxKeys, M3_ERR_UNSUPPORTED, "n_q %d", c.n_q);
  M3_REQUIRE(c.d % c.heads == 0 && (c.d / c.heads == 32 || c.d / c.heads == 64 || c.d / c.heads == 128),
             M3_ERR_UNSUPPORTED, "depth head dim must be 32, 64 or 128");
  M3_REQUIRE(c.d % 8 == 0 && c.ffn % 8 == 0 && c.d_backbone % 8 == 0 && c.d <= 8192, M3_ERR_UNSUPPORTED, "sizes");
  auto* d = new m3_depth();
  d->c = c;
  d->in_proj = (const bf16*)w->in_proj;
  d->embed = (const bf16*)w->embed;
  d->level0 = (const bf16*)w->level0;
  d->norm_w = (const bf16*)w->norm_w;
  d->norm_b = (const bf16*)w->norm_b;
  const int GL = c.n_groups * c.layers;
  for (int i = 0; i < GL; ++i) {
    d->n1_w.push_back((const bf16*)w->n1_w[i]);
    d->n1_b.push_back((const bf16*)w->n1_b[i]);
    d->n2_w.push_back((const bf16*)w->n2_w[i]);
    d->n2_b.push_back((const bf16*)w->n2_b[i]);
    d->qkv.push_back((const bf16*)w->qkv[i]);
    d->o.push_back((const bf16*)w->o[i]);
    d->f1.push_back((const bf16*)w->f1[i]);
    d->f2.push_back((const bf16*)w->f2[i]);
  }
  for (int i = 0; i < c.n_q - 1; ++i) d->heads.push_back((const bf16*)w->heads[i]);
  for (int i = 0; i < c.layers; ++i) {
    d->cross_kv.push_back((const bf16*)w->cross_kv[i]);
    d->cross_o.push_back((const bf16*)w->cross_o[i]);
  }
  d->audio_table = (const bf16*)w->audio_table;
  d->audio_norm = (const bf16*)w->audio_norm;
  d->cross_const = (bf16*)w->cross_const;
  d->row_seed = w->row_seed;
  d->row_ctr = w->row_ctr;
  const size_t R = c.max_rows, NL = c.n_q, D = c.d;
  size_t bytes = 0;
  auto add = [&](size_t n) { bytes += (n + 255) / 256 * 256; };
  add(R * 4); add(R * 4); add(256);
  add(R * NL * D * 2);          // prefix
  add(R * NL * D * 2);          // x
  add(R * NL * D * 2);          // x2
  add(R * NL * D * 2);          // y
  add(R * NL * 3 * D * 2);      // qkv
  add(R * NL * D * 2);          // a
  add(R * NL * D * 2);          // o
  add(R * NL * c.ffn * 2);      // ff
  add(R * c.n_codes * 2);       // logits
  add(R * D * 2);               // proj
  add((size_t)c.layers * R * NL * 2 * D * 2);  // kvbuf
  add(4 * D * 2);               // speaker scratch
  add(kBlasWorkspace);          // the handle's own cuBLAS workspace
  cudaError_t e = cudaMalloc(&d->ws, bytes);
  if (e != cudaSuccess) {
    delete d;
    set_error("m3_depth_create: cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
    return M3_ERR_CUDA;
  }
  char* p = (char*)d->ws;
  d->slot32 = carve<int>(p, R);
  d->cb032 = carve<int>(p, R);
  d->status = carve<int>(p, 64);
  d->prefix = carve<bf16>(p, R * NL * D);
  d->x = carve<bf16>(p, R * NL * D);
  d->x2 = carve<bf16>(p, R * NL * D);
  d->y = carve<bf16>(p, R * NL * D);
  d->qkvb = carve<bf16>(p, R * NL * 3 * D);
  d->a = carve<bf16>(p, R * NL * D);
  d->ob = carve<bf16>(p, R * NL * D);
  d->ff = carve<bf16>(p, R * NL * c.ffn);
  d->logits = carve<bf16>(p, R * c.n_codes);
  d->proj = carve<bf16>(p, R * D);
  d->kvbuf = carve<bf16>(p, (size_t)c.layers * R * NL * 2 * D);
  d->spk = carve<bf16>(p, 4 * D);
  d->blas_ws = carve<unsigned char>(p, kBlasWorkspace);
  cudaMemset(d->status, 0, 256);
  *out = d;
  return M3_OK;
}

extern "C" int m3_depth_destroy(m3_depth* d) {
  if (!d) return M3_OK;
  cudaFree(d->ws);
  delete d;
  return M3_OK;
}

extern "C" int m3_depth_status(m3_depth* d, int32_t* status, int32_t clear) {
  M3_REQUIRE(d && status, M3_ERR_ARG, "m3_depth_status: null argument");
  M3_CUDA(cudaMemcpy(status, d->status, sizeof(int32_t), cudaMemcpyDeviceToHost));
  if (clear) M3_CUDA(cudaMemset(d->status, 0, sizeof(int32_t)));
  return M3_OK;
}

extern "C" int m3_depth_debug_logits(m3_depth* d, void* buf, int64_t bytes) {
  M3_REQUIRE(d, M3_ERR_ARG, "m3_depth_debug_logits: null handle");
  const int64_t need = (int64_t)(d->c.n_q - 1) * d->c.max_rows * d->c.n_codes * 2;
  M3_REQUIRE(!buf || bytes >= need, M3_ERR_ARG, "m3_depth_debug_logits: %lld bytes, need %lld", (long long)bytes,
             (long long)need);
  M3_REQUIRE(((uintptr_t)buf & 15) == 0, M3_ERR_ARG, "m3_depth_debug_logits: buffer must be 16-byte aligned");
  d->dbg_logits = (bf16*)buf;
  return M3_OK;
}

extern "C" int m3_depth_set_speaker(m3_depth* d, int32_t slot, const void* mem, float keep, m3_stream stream) {
  M3_REQUIRE(d && mem, M3_ERR_ARG, "m3_depth_set_speaker: null argument");
  M3_REQUIRE(slot >= 0 && slot <= d->c.max_slots, M3_ERR_RANGE, "slot %d outside [0, %d]", slot, d->c.max_slots);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int D = d->c.d;
  for (int li = 0; li < d->c.layers; ++li) {
    bf16* dst = d->cross_const + ((int64_t)slot * d->c.layers + li) * D;
    if (keep == 0.f) {  // o(v * 0) = 0: the layers are bias-free
      M3_CUDA(cudaMemsetAsync(dst, 0, (size_t)D * 2, s));
      continue;
    }
    // kv = kv(mem) (bf16), v = second half; cross = o(v)   (serve/fast_depth.py:80-82)
    M3_TRY(dgemm(d, {(const bf16*)mem, D, d->cross_kv[li], D, d->spk, 2 * D, 1, 2 * D, D, false}, s));
    M3_TRY(dgemm(d, {d->spk + D, D, d->cross_o[li], D, dst, D, 1, D, D, false}, s));
  }
  return M3_OK;
}

extern "C" int m3_depth_step(m3_depth* d, const int64_t* slots, const void* h, const int64_t* cb0, int64_t* codes,
                             void* feedback, int32_t rows, m3_stream stream) {
  M3_REQUIRE(d && slots && h && cb0 && codes && feedback, M3_ERR_ARG, "m3_depth_step: null argument");
  const m3_depth_config& c = d->c;
  M3_REQUIRE(rows >= 0 && rows <= c.max_rows, M3_ERR_RANGE, "rows %d > max_rows %d", rows, c.max_rows);
  if (rows == 0) return M3_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int R = rows, NL = c.n_q, D = c.d, H = c.heads, HD = D / H, L = c.layers;
  const int nt = norm_threads(D);
  const float scale = 1.f / sqrtf((float)HD);
  depth_prep_kernel<<<cdiv(R, 128), 128, 0, s>>>(slots, cb0, R, c.max_slots, c.n_codes, d->slot32, d->cb032, codes,
                                                 NL, d->status);
  M3_LAUNCHED();
  M3_TRY(dgemm(d, {(const bf16*)h, c.d_backbone, d->in_proj, c.d_backbone, d->proj, D, R, D, c.d_backbone, false}, s));
  prefix_init_kernel<<<R, 128, 0, s>>>(d->proj, d->level0, d->embed, d->cb032, d->prefix, NL, D);
  M3_LAUNCHED();
  const int64_t kv_layer = (int64_t)R * NL * 2 * D;
  int previous = -1;
  for (int level = 1; level < NL; ++level) {
    const int group = c.group_of_level[level];
    const int n = level + 1;
    const bool incremental = group == previous;
    const bool reused_later = level + 1 < NL && c.group_of_level[level + 1] == group;
    const int T = incremental ? 1 : n;
    const int start = incremental ? level : 0;
    const int gl = group * L;
    // y = n1(x); x (the residual stream) becomes a contiguous copy of the prefix slice (from level 2 on, the previous
    // level's sampler did this right after writing the new prefix entry)
    if (level == 1)
      M3_TRY(launch_add_ln(R * T, d->prefix + (int64_t)start * D, T, (int64_t)NL * D, D, nullptr, nullptr, 0, nullptr,
                           d->x, d->y, d->n1_w[gl], d->n1_b[gl], c.ln_eps, D, s));
    int Tr = T;  // rows per seat in the residual stream
    for (int li = 0; li < L; ++li) {
      M3_TRY(dgemm(d, {d->y, D, d->qkv[gl + li], D, d->qkvb, 3 * D, R * Tr, 3 * D, D, false}, s));
      bf16* kvl = d->kvbuf + li * kv_layer;
      int Tq = Tr, q0 = start;
      KeySrc ks;
      if (incremental) {
        kv_store_kernel<<<dim3(R, 1), 128, 0, s>>>(d->qkvb, 1, kvl, NL, level, D);
        M3_LAUNCHED();
        ks = {kvl, kvl + D, (int64_t)NL * 2 * D, 2 * D};
        q0 = level;
      } else {
        if (reused_later) {
          kv_store_kernel<<<dim3(R, n), 128, 0, s>>>(d->qkvb, n, kvl, NL, 0, D);
          M3_LAUNCHED();
        }
        ks = {d->qkvb + D, d->qkvb + 2 * D, (int64_t)n * 3 * D, 3 * D};
        if (li == L - 1) {
          Tq = 1;
          q0 = n - 1;
        }
      }
      const dim3 ag(R, H);
      if (HD == 128 && Tq <= 16 && q0 + Tq <= 16)
        depth_attn_mma_kernel<<<ag, 32, 0, s>>>(d->qkvb, Tr, q0, Tq, ks, H, scale, d->a);
      else if (HD == 128)
        depth_attn_kernel<4><<<ag, 32 * Tq, 0, s>>>(d->qkvb, Tr, q0, Tq, ks, H, scale, d->a);
      else if (HD == 64)
        depth_attn_kernel<2><<<ag, 32 * Tq, 0, s>>>(d->qkvb, Tr, q0, Tq, ks, H, scale, d->a);
      else
        depth_attn_kernel<1><<<ag, 32 * Tq, 0, s>>>(d->qkvb, Tr, q0, Tq, ks, H, scale, d->a);
      M3_LAUNCHED();
      M3_TRY(dgemm(d, {d->a, D, d->o[gl + li], D, d->ob, D, R * Tq, D, D, false}, s));
      if (Tq != Tr) {
        // the last layer keeps only each seat's final position (x = x[:, -1:], serve/fast_depth.py:181): the
        // residual add reads row Tr-1 of each seat's block and writes the compact stream
        M3_TRY(launch_add_ln(R, d->x + (int64_t)(Tr - 1) * D, 1, (int64_t)Tr * D, 0, d->ob, nullptr, 0, nullptr, d->x2,
                             d->y, d->n2_w[gl + li], d->n2_b[gl + li], c.ln_eps, D, s));
        std::swap(d->x, d->x2);
        Tr = Tq;
      } else {
        // x, y2 = add_ln(x, o(a), n2)
        M3_TRY(launch_add_ln(R * Tr, d->x, 1, D, 0, d->ob, nullptr, 0, nullptr, d->x, d->y, d->n2_w[gl + li],
                             d->n2_b[gl + li], c.ln_eps, D, s));
      }
      GemmDesc f1{d->y, D, d->f1[gl + li], D, d->ff, c.ffn, R * Tr, c.ffn, D, false};
      f1.act = kActGelu;
      if (!gemv_path(f1)) f1.act = kActNone;  // a few rows: GELU in the GEMV epilogue; else its own pass
      M3_TRY(dgemm(d, f1, s));
      if (f1.act == kActNone) {
        const int64_t n8 = (int64_t)R * Tr * c.ffn / 8;
        gelu_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, s>>>(d->ff, n8);
        M3_LAUNCHED();
      }
      M3_TRY(dgemm(d, {d->ff, c.ffn, d->f2[gl + li], c.ffn, d->ob, D, R * Tr, D, c.ffn, false}, s));
      // x, y = add_ln(x, f, next n1 (or the final norm), cross[slot][li])
      const bf16* nw = li + 1 < L ? d->n1_w[gl + li + 1] : d->norm_w;
      const bf16* nb = li + 1 < L ? d->n1_b[gl + li + 1] : d->norm_b;
      M3_TRY(launch_add_ln(R * Tr, d->x, Tr, (int64_t)Tr * D, D, d->ob, d->cross_const + (int64_t)li * D, (int64_t)L * D,
                    d->slot32, d->x, d->y, nw, nb, c.ln_eps, D, s));
    }
    // level head on the final position, then sample and write the next prefix row
    bf16* lg = d->dbg_logits ? d->dbg_logits + (int64_t)(level - 1) * c.max_rows * c.n_codes : d->logits;
    M3_TRY(dgemm(d, {d->y + (int64_t)(Tr - 1) * D, (int64_t)Tr * D, d->heads[level - 1], D, lg, c.n_codes, R,
                 c.n_codes, D, false},
                s));
    const bool more = n < NL;
    PrefixLn ln{};
    if (more) {  // the next level's first LayerNorm (same slice rule as at the top of the loop)
      const int g2 = c.group_of_level[level + 1];
      const bool inc2 = g2 == group;
      ln = PrefixLn{d->prefix, (int64_t)NL * D, inc2 ? level + 1 : 0, inc2 ? 1 : level + 2, d->x, d->y,
                    d->n1_w[g2 * L], d->n1_b[g2 * L], c.ln_eps};
    }
    M3_TRY(launch_topk_sample(lg, true, c.n_codes, R, c.n_codes, d->row_seed, d->row_ctr, d->slot32, level,
                              c.inv_temp, c.top_k, c.greedy, codes + level, NL,
                              more ? d->embed + (int64_t)level * c.n_codes * D : nullptr, D,
                              more ? d->prefix + (int64_t)n * D : nullptr, (int64_t)NL * D, s, ln));
    previous = group;
  }
  ctr_advance_kernel<<<cdiv(R, 128), 128, 0, s>>>(d->slot32, R, d->row_ctr);
  M3_LAUNCHED();
  feedback_kernel<<<R, norm_threads(c.d_backbone), 0, s>>>(codes, NL, c.n_codes, d->audio_table, d->audio_norm,
                                                           c.d_backbone, sqrtf((float)NL), (bf16*)feedback,
                                                           d->status);
  M3_LAUNCHED();
  return M3_OK;
}

extern "C" int m3_gelu_bf16(void* f, int64_t n8, m3_stream stream) {
  M3_REQUIRE(f && n8 >= 0, M3_ERR_ARG, "m3_gelu_bf16: bad argument");
  if (n8 == 0) return M3_OK;
  m3::gelu_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<m3::bf16*>(f), n8);
  M3_LAUNCHED();
  return M3_OK;
}
