// One-frame streaming Mimi decoder with per-slot state (replaces serve/fast_codec.py StaticMimi).
//
// Layout: activations are channels-last [row, time, channel] so every convolution is a GEMM over (row, time) rows:
// a causal conv of k taps reads its k shifted input rows (the first k-1 come from the slot's history), a
// transposed conv of stride r is X . W^T producing 2r output columns per input step, folded back with the previous
// step's overlap (and the slot's stored tail for the first r outputs).  Rounding follows the reference (HF
// MimiModel modules in the model dtype): each conv output is bias-added and rounded once, the stored convT tail is
// bf16(y - bias), the resnet sum and the transformer residuals round after each add.
#include <algorithm>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"
#include "mma.cuh"
#include "ops.cuh"
#include "seanet.cuh"
#include "tma.cuh"

namespace m3 {

constexpr int64_t kNever = -(1ll << 40);  // key_pos of an empty ring entry (serve/fast_codec.py:25)

struct StageDims {  // one upsampling stage of the SEANet decoder
  int cin, cout, r, L;  // L = input steps per frame
  int64_t tail_off, hist_off;  // offsets (elements) in the slot's state row: convT tail [r, cout], k3 history
};

// ------------------------------------------------------------------------------------------------ RVQ + upsample
// A_sem[b] = sum of semantic codebook rows, A_ac[b] = sum of acoustic rows (bf16 after each add,
// serve/fast_codec.py:134-140).
__global__ void rvq_gather_kernel(const int64_t* __restrict__ codes, int n_q, int n_sem, int cb_size, int cbd,
                                  const bf16* __restrict__ books, bf16* __restrict__ a_sem, bf16* __restrict__ a_ac,
                                  int* status) {
  const int b = blockIdx.x;
  for (int d = threadIdx.x; d < cbd; d += blockDim.x) {
    float sem = 0.f, ac = 0.f;
    for (int k = 0; k < n_q; ++k) {
      int64_t c = codes[(int64_t)b * n_q + k];
      if (c < 0 || c >= cb_size) {
        report(status, M3_DEV_BAD_CODE);
        c = c < 0 ? 0 : cb_size - 1;
      }
      const float e = to_f(books[((int64_t)k * cb_size + c) * cbd + d]);
      if (k < n_sem)
        sem = k == 0 ? e : rbf(sem + e);
      else
        ac = k == n_sem ? e : rbf(ac + e);
    }
    a_sem[(int64_t)b * cbd + d] = to_bf(sem);
    a_ac[(int64_t)b * cbd + d] = to_bf(ac);
  }
}

// x = bf16(P_sem + P_ac) (one 12.5 Hz token), then the depthwise ConvTranspose1d(k = 2s, stride s, no bias) with
// its overlap tail: out[t] = bf16(y[t] + tail[t]) for t < s, new tail = y[s..2s)   (serve/fast_codec.py:112-126).
__global__ void upsample_kernel(const bf16* __restrict__ p_sem, const bf16* __restrict__ p_ac,
                                const bf16* __restrict__ w, int s, const int* __restrict__ slot32,
                                bf16* __restrict__ state, int64_t state_row, bf16* __restrict__ out, int H) {
  const int b = blockIdx.x;
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (c >= H) return;
  bf16* tail = state + (int64_t)slot32[b] * state_row;  // [s, H]
  const float x = rbf(to_f(p_sem[(int64_t)b * H + c]) + to_f(p_ac[(int64_t)b * H + c]));
  float y[16];
  for (int j = 0; j < 2 * s; ++j) y[j] = rbf(x * to_f(w[(int64_t)c * 2 * s + j]));
  for (int t = 0; t < s; ++t) {
    const float prev = to_f(tail[(int64_t)t * H + c]);
    out[((int64_t)b * s + t) * H + c] = to_bf(y[t] + prev);
    tail[(int64_t)t * H + c] = to_bf(y[s + t]);
  }
}

// ------------------------------------------------------------------------------------------------ transformer
// Absolute positions of this frame's tokens and their ring entries (serve/fast_codec.py:153-157).
__global__ void tpos_kernel(const int* __restrict__ slot32, int rows, int T, int ring, const int64_t* __restrict__ tokens,
                            int64_t* __restrict__ key_pos, int64_t* __restrict__ pos_out) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= rows) return;
  const int s = slot32[b];
  const int64_t start = tokens[s];
  for (int t = 0; t < T; ++t) {
    const int64_t p = start + t;
    key_pos[(int64_t)s * ring + (p % ring)] = p;
    pos_out[(int64_t)b * T + t] = p;
  }
}

// q, k <- apply_rotary_pos_emb in the model dtype (each product and the sum rounded); k and v written to the slot's
// ring at pos % ring (keys post-RoPE, serve/fast_codec.py:171-175).  One warp per (row, token, head).
__global__ void mimi_rope_kernel(const bf16* __restrict__ qkv, const int64_t* __restrict__ pos,
                                 const float* __restrict__ inv_freq, const int* __restrict__ slot32, int T, int heads,
                                 int hd, int ring, bf16* __restrict__ q_out, bf16* __restrict__ kring,
                                 bf16* __restrict__ vring, int64_t slot_stride) {
  const int bt = blockIdx.x;  // row * T + t
  const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (h >= heads) return;
  const int b = bt / T;
  const int H = heads * hd, half = hd / 2;
  const int64_t p = pos[bt];
  const bf16* row = qkv + (int64_t)bt * 3 * H;
  const int64_t roff = (int64_t)slot32[b] * slot_stride + ((int64_t)h * ring + (p % ring)) * hd;
  for (int i = lane; i < half; i += 32) {
    const float f = (float)p * inv_freq[i];
    const float cs = rbf(cosf(f)), sn = rbf(sinf(f));  // emb = [f, f]: both halves share cos/sin
    const int d1 = h * hd + i, d2 = d1 + half;
    const float q1 = to_f(row[d1]), q2 = to_f(row[d2]);
    const float k1 = to_f(row[H + d1]), k2 = to_f(row[H + d2]);
    // rotate_half(x) = [-x2, x1]
    q_out[(int64_t)bt * H + d1] = to_bf(rbf(q1 * cs) + rbf(-q2 * sn));
    q_out[(int64_t)bt * H + d2] = to_bf(rbf(q2 * cs) + rbf(q1 * sn));
    kring[roff + i] = to_bf(rbf(k1 * cs) + rbf(-k2 * sn));
    kring[roff + i + half] = to_bf(rbf(k2 * cs) + rbf(k1 * sn));
    vring[roff + i] = row[2 * H + d1];
    vring[roff + i + half] = row[2 * H + d2];
  }
}

// Sliding-window attention of the frame's T queries over the slot's ring: key r is visible to the query at
// position p iff p - window < key_pos[r] <= p (serve/fast_codec.py:158-160,178).
constexpr float kLazyRescale2 = 8.f;  // raise the running max only when a score exceeds it by 2^8

// On the tensor cores for head dims 32 and 64 (the decode attention's design, without splits):
// one CTA of 4 warps per (row, head); the ring is cut into 16-entry blocks, warp w takes blocks w, w+4, ... through
// its own 2-deep TMA ring (tensor maps over kv[layer][k|v] as [slot * heads + head][entry][head_dim]); S = Q K^T with
// the T queries as mma rows, the key_pos window as the mask, online softmax in exp2, O^T += V^T P^T with P split into
// bf16 hi + lo.  Every wait is bounded.
constexpr int kRingBlk = 16;

template <int HD>
__device__ __forceinline__ uint32_t ring_off(int r, int c) {
  if constexpr (HD == 64) return sw128(r, c);  // 128-byte rows, 128-byte swizzle
  else return (uint32_t)(r * HD * 2 + c * 16);  // 64-byte rows, no swizzle
}

template <int HD>
struct RingMmaSmem {
  unsigned char stage[4][2][2 * kRingBlk * HD * 2];  // [warp][stage][K box | V box]
  uint64_t bar[4][2];
};

template <int HD, int T>
__global__ void __launch_bounds__(128) ring_mma_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, const bf16* __restrict__ q,
    const int64_t* __restrict__ key_pos, const int64_t* __restrict__ pos, const int* __restrict__ slot32, int heads,
    int ring, int window, float qscale, bf16* __restrict__ out, int* status) {
  constexpr int BOX = kRingBlk * HD * 2, KS = HD / 16;
  static_assert(T <= 8, "the queries fill at most 8 of the 16 mma rows");
  extern __shared__ unsigned char smem_raw[];
  RingMmaSmem<HD>& sm =
      *reinterpret_cast<RingMmaSmem<HD>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int b = blockIdx.x, h = blockIdx.y, H = heads * HD;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int s = slot32[b];
  const int zc = s * heads + h;
  const int nblk = ring / kRingBlk;
  const int nmine = warp < nblk ? (nblk - 1 - warp) / 4 + 1 : 0;
  if (tid == 0) {
    for (int w = 0; w < 4; ++w)
      for (int st = 0; st < 2; ++st) mbar_init(&sm.bar[w][st], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int i) {
    unsigned char* st = sm.stage[warp][i & 1];
    uint64_t* bar = &sm.bar[warp][i & 1];
    const int y = (warp + 4 * i) * kRingBlk;
    mbar_expect_tx(bar, 2 * BOX);
    tma_load_3d(st, &kmap, 0, y, zc, bar);
    tma_load_3d(st + BOX, &vmap, 0, y, zc, bar);
  };
  if (lane == 0)
    for (int i = 0; i < min(2, nmine); ++i) issue(i);
  uint32_t qa[KS][2];
  {
    const uint32_t* qp = reinterpret_cast<const uint32_t*>(q + ((int64_t)b * T + min(g, T - 1)) * H + h * HD);
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      qa[ks][0] = g < T ? qp[8 * ks + t] : 0u;
      qa[ks][1] = g < T ? qp[8 * ks + 4 + t] : 0u;
    }
  }
  const int64_t pg = pos[(int64_t)b * T + min(g, T - 1)];
  const int64_t* kps = key_pos + (int64_t)s * ring;
  float o[KS][4];
#pragma unroll
  for (int mt = 0; mt < KS; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  bool timed_out = false;
  int i = 0;
  for (; i < nmine; ++i) {
    const bool got = mbar_wait(&sm.bar[warp][i & 1], (i >> 1) & 1, status);
    if (!__all_sync(0xffffffffu, got)) {
      timed_out = true;
      break;
    }
    const uint32_t kb = smem_u32(sm.stage[warp][i & 1]), vb = kb + BOX;
    const int e0 = (warp + 4 * i) * kRingBlk;
    const int j = lane >> 3, lr = ((j >> 1) << 3) + (lane & 7), lc = j & 1;
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      uint32_t k0, k1, k2, k3;
      ldsm_x4(kb + ring_off<HD>(lr, 2 * ks + lc), k0, k1, k2, k3);
      mma_bf16(sc[0], qa[ks][0], 0u, qa[ks][1], 0u, k0, k1);
      mma_bf16(sc[1], qa[ks][0], 0u, qa[ks][1], 0u, k2, k3);
    }
    float p[2][2];
    float mx = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int64_t kp = kps[e0 + nt * 8 + 2 * t + e];
        const bool vis = g < T && kp <= pg && kp > pg - window;
        p[nt][e] = vis ? sc[nt][e] * qscale : -INFINITY;
        mx = fmaxf(mx, p[nt][e]);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    float r = 1.f;
    if (mx > m_run + kLazyRescale2) {
      r = exp2f(m_run - mx);
      m_run = mx;
      l_run *= r;
    }
    if (__any_sync(0xffffffffu, r != 1.f)) {
      const float r0 = __shfl_sync(0xffffffffu, r, 8 * t), r1 = __shfl_sync(0xffffffffu, r, 8 * t + 4);
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) {
        o[mt][0] *= r0;
        o[mt][1] *= r1;
        o[mt][2] *= r0;
        o[mt][3] *= r1;
      }
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        p[nt][e] = p[nt][e] == -INFINITY ? 0.f : exp2f(p[nt][e] - m_run);
        l_run += p[nt][e];
      }
    const uint32_t h0 = pack_bf2(p[0][0], p[0][1]), h1 = pack_bf2(p[1][0], p[1][1]);
    const uint32_t l0 = pack_bf2(p[0][0] - bf_lo_f(h0), p[0][1] - bf_hi_f(h0));
    const uint32_t l1 = pack_bf2(p[1][0] - bf_lo_f(h1), p[1][1] - bf_hi_f(h1));
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4_t(vb + ring_off<HD>(lr, 2 * mt + lc), a0, a1, a2, a3);
      mma_bf16(o[mt], a0, a1, a2, a3, h0, h1);
      mma_bf16(o[mt], a0, a1, a2, a3, l0, l1);
    }
    __syncwarp();
    if (lane == 0 && i + 2 < nmine) issue(i + 2);
  }
  if (timed_out) {  // drain this warp's copies in flight (bounded), publish an empty partial
    if (lane == 0)
      for (int k = i; k < min(nmine, i + 2); ++k) mbar_wait(&sm.bar[warp][k & 1], (k >> 1) & 1, nullptr);
    __syncwarp();
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    m_run = -INFINITY;
    l_run = 0.f;
  }
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  float* wo = reinterpret_cast<float*>(sm.stage[warp][0]);  // [T][HD], then (m, l) per query
  float* wml = wo + T * HD;
#pragma unroll
  for (int mt = 0; mt < KS; ++mt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int qh = 2 * t + (e & 1);
      if (qh < T) wo[qh * HD + 16 * mt + g + ((e >> 1) << 3)] = o[mt][e];
    }
  if (t == 0 && g < T) {
    wml[2 * g] = m_run;
    wml[2 * g + 1] = l_run;
  }
  __syncthreads();
  for (int idx = tid; idx < T * HD; idx += 128) {
    const int qh = idx / HD, d = idx % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, reinterpret_cast<const float*>(sm.stage[w][0])[T * HD + 2 * qh]);
    float O = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float* ww = reinterpret_cast<const float*>(sm.stage[w][0]);
      const float mw = ww[T * HD + 2 * qh];
      const float c = mw == -INFINITY ? 0.f : exp2f(mw - M);
      O = fmaf(ww[qh * HD + d], c, O);
      L = fmaf(ww[T * HD + 2 * qh + 1], c, L);
    }
    out[((int64_t)b * T + qh) * H + h * HD + d] = to_bf(L > 0.f ? O / L : 0.f);
  }
}

// h' = bf16(h + bf16(scale * a)) (MimiLayerScale + residual), stored; y = LayerNorm(h') if w != nullptr.
__global__ void scale_add_ln_kernel(bf16* __restrict__ h, const bf16* __restrict__ a, const bf16* __restrict__ ls,
                                    bf16* __restrict__ y, const bf16* __restrict__ w, const bf16* __restrict__ bias,
                                    float eps, int D) {
  __shared__ float red[32];
  const int r = blockIdx.x;
  constexpr int kMaxPer = 4;
  float v[kMaxPer][8];
  float sum = 0.f;
  const int nv = D / 8;
#pragma unroll
  for (int it = 0; it < kMaxPer; ++it) {
    const int i = threadIdx.x + it * blockDim.x;
    if (i < nv) {
      float hv[8], av[8], sv[8];
      unpack8(reinterpret_cast<const uint4*>(h + (int64_t)r * D)[i], hv);
      unpack8(reinterpret_cast<const uint4*>(a + (int64_t)r * D)[i], av);
      unpack8(reinterpret_cast<const uint4*>(ls)[i], sv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v[it][e] = rbf(hv[e] + rbf(sv[e] * av[e]));
        sum += v[it][e];
      }
      reinterpret_cast<uint4*>(h + (int64_t)r * D)[i] = pack8(v[it]);
    }
  }
  if (!w) return;
  const float mean = block_sum(sum, red) / (float)D;
  float sq = 0.f;
#pragma unroll
  for (int it = 0; it < kMaxPer; ++it) {
    const int i = threadIdx.x + it * blockDim.x;
    if (i < nv)
#pragma unroll
      for (int e = 0; e < 8; ++e) sq = fmaf(v[it][e] - mean, v[it][e] - mean, sq);
  }
  const float den = sqrtf(block_sum(sq, red) / (float)D + eps);
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

__global__ void tokens_advance_kernel(const int* __restrict__ slot32, int rows, int T, int dummy,
                                      int64_t* __restrict__ tokens) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < rows && slot32[b] != dummy) tokens[slot32[b]] += T;
  if (b == 0) tokens[dummy] = 0;  // serve/fast_codec.py:182-183
}

// ------------------------------------------------------------------------------------------------ SEANet

// im2col of a causal stride-1 conv with k taps over joined = [history (k-1 stored rows); act(x)], act = ELU
// (rounded) when elu_in: A[b*L + t, j*C + c] = joined[t + j][c].  One thread per (row, step, 8 channels); the
// history itself is refreshed afterwards by conv_hist_kernel (so no thread reads a row another thread rewrote).
__global__ void im2col_kernel(const bf16* __restrict__ x, int L, int C, int k, int elu_in,
                              const int* __restrict__ slot32, const bf16* __restrict__ state, int64_t state_row,
                              int64_t hist_off, bf16* __restrict__ A) {
  const int b = blockIdx.x;
  const int C8 = C / 8, P = k - 1;
  const int idx = blockIdx.y * blockDim.x + threadIdx.x;
  if (idx >= L * C8) return;
  const int t = idx / C8, c8 = idx % C8;
  const uint4* hist = reinterpret_cast<const uint4*>(state + (int64_t)slot32[b] * state_row + hist_off);
  const uint4* xs = reinterpret_cast<const uint4*>(x + (int64_t)b * L * C);
  uint4* dst = reinterpret_cast<uint4*>(A + ((int64_t)b * L + t) * k * C);
  for (int j = 0; j < k; ++j) {
    const int i = t + j;
    uint4 v;
    if (i < P) {
      v = hist[i * C8 + c8];
    } else {
      v = xs[(int64_t)(i - P) * C8 + c8];
      if (elu_in) v = elu8(v);
    }
    dst[j * C8 + c8] = v;
  }
}

// The conv's history becomes the last k-1 rows of joined (serve/fast_codec.py:106-110).  One thread per
// (row, 8 channels) reads the old rows it needs before writing.
__global__ void conv_hist_kernel(const bf16* __restrict__ x, int L, int C, int k, int elu_in,
                                 const int* __restrict__ slot32, bf16* __restrict__ state, int64_t state_row,
                                 int64_t hist_off) {
  const int b = blockIdx.x;
  const int C8 = C / 8, P = k - 1;
  const int c8 = blockIdx.y * blockDim.x + threadIdx.x;
  if (c8 >= C8 || P == 0) return;
  uint4* hist = reinterpret_cast<uint4*>(state + (int64_t)slot32[b] * state_row + hist_off);
  const uint4* xs = reinterpret_cast<const uint4*>(x + (int64_t)b * L * C);
  uint4 old[8];
  for (int j = 0; j < P; ++j) old[j] = hist[j * C8 + c8];
  for (int j = 0; j < P; ++j) {
    const int i = L + j;
    uint4 v;
    if (i < P) {
      v = old[i];
    } else {
      v = xs[(int64_t)(i - P) * C8 + c8];
      if (elu_in) v = elu8(v);
    }
    hist[j * C8 + c8] = v;
  }
}

// y = bf16(z + bias); mode 1: y = bf16(elu(y)); mode 2: y = bf16(res + y); mode 3: y = bf16(elu(bf16(res + y))).
// Eight elements per thread (y may alias res).
__global__ void bias_epilogue_kernel(const float* __restrict__ z, const bf16* __restrict__ bias, int64_t M, int N,
                                     int mode, const bf16* __restrict__ res, bf16* __restrict__ y) {
  const int64_t i8 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i8 >= M * N / 8) return;
  const int n0 = (int)((i8 * 8) % N);
  const float4 z0 = reinterpret_cast<const float4*>(z)[2 * i8], z1 = reinterpret_cast<const float4*>(z)[2 * i8 + 1];
  float v[8] = {z0.x, z0.y, z0.z, z0.w, z1.x, z1.y, z1.z, z1.w}, bv[8], rv[8];
  unpack8(*reinterpret_cast<const uint4*>(bias + n0), bv);
  if (mode >= 2) unpack8(reinterpret_cast<const uint4*>(res)[i8], rv);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    v[e] = rbf(v[e] + bv[e]);
    if (mode == 1) v[e] = elu(v[e]);
    if (mode >= 2) v[e] = rv[e] + v[e];
    if (mode == 3) v[e] = elu(rbf(v[e]));
  }
  reinterpret_cast<uint4*>(y)[i8] = pack8(v);
}

// y = bf16(elu(x)), eight elements per thread.
__global__ void elu_kernel(const bf16* __restrict__ x, bf16* __restrict__ y, int64_t n8) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n8) reinterpret_cast<uint4*>(y)[i] = elu8(reinterpret_cast<const uint4*>(x)[i]);
}

// Transposed conv fold: Z[b*L + t, j*Co + o] (fp32, j < 2r) are the per-step contributions.  Output step
// s = t*r + jj gets Z[t, jj] + Z[t-1, jj + r]; the conv output is bf16(sum + bias) and the first r outputs add the
// slot's stored tail (serve/fast_codec.py:112-126).  One thread per (row, output step, 8 channels).
__global__ void convt_fold_kernel(const float* __restrict__ Z, const bf16* __restrict__ bias, int L, int r, int Co,
                                  const int* __restrict__ slot32, const bf16* __restrict__ state, int64_t state_row,
                                  int64_t tail_off, bf16* __restrict__ y) {
  const int b = blockIdx.x;
  const int C8 = Co / 8;
  const int idx = blockIdx.y * blockDim.x + threadIdx.x;
  if (idx >= L * r * C8) return;
  const int st = idx / C8, o8 = idx % C8;
  const int t = st / r, jj = st % r;
  const int64_t zr = (int64_t)2 * r * Co;
  const float* zb = Z + (int64_t)b * L * zr;
  const float4* a = reinterpret_cast<const float4*>(zb + (int64_t)t * zr + (int64_t)jj * Co + o8 * 8);
  float4 a0 = a[0], a1 = a[1];
  float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
  if (t > 0) {
    const float4* p = reinterpret_cast<const float4*>(zb + (int64_t)(t - 1) * zr + (int64_t)(jj + r) * Co + o8 * 8);
    const float4 p0 = p[0], p1 = p[1];
    v[0] += p0.x; v[1] += p0.y; v[2] += p0.z; v[3] += p0.w;
    v[4] += p1.x; v[5] += p1.y; v[6] += p1.z; v[7] += p1.w;
  }
  float bv[8];
  unpack8(*reinterpret_cast<const uint4*>(bias + o8 * 8), bv);
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = rbf(v[e] + bv[e]);
  if (t == 0) {
    float tv[8];
    unpack8(*reinterpret_cast<const uint4*>(state + (int64_t)slot32[b] * state_row + tail_off +
                                            (int64_t)jj * Co + o8 * 8), tv);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = v[e] + tv[e];
  }
  reinterpret_cast<uint4*>(y + ((int64_t)b * L * r + st) * Co)[o8] = pack8(v);
}

// New overlap tail = bf16(bf16(Z[L-1, r + jj] + bias) - bias), after the fold has read the old one.
__global__ void convt_tail_kernel(const float* __restrict__ Z, const bf16* __restrict__ bias, int L, int r, int Co,
                                  const int* __restrict__ slot32, bf16* __restrict__ state, int64_t state_row,
                                  int64_t tail_off) {
  const int b = blockIdx.x;
  const int C8 = Co / 8;
  const int idx = blockIdx.y * blockDim.x + threadIdx.x;
  if (idx >= r * C8) return;
  const int jj = idx / C8, o8 = idx % C8;
  const int64_t zr = (int64_t)2 * r * Co;
  const float4* a =
      reinterpret_cast<const float4*>(Z + ((int64_t)b * L + L - 1) * zr + (int64_t)(jj + r) * Co + o8 * 8);
  const float4 a0 = a[0], a1 = a[1];
  const float z[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
  float bv[8], v[8];
  unpack8(*reinterpret_cast<const uint4*>(bias + o8 * 8), bv);
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = rbf(z[e] + bv[e]) - bv[e];
  reinterpret_cast<uint4*>(state + (int64_t)slot32[b] * state_row + tail_off + (int64_t)jj * Co)[o8] = pack8(v);
}

// Final ELU + conv (C -> 1 channel, k taps) -> fp32 PCM.  CTA per (row, 128 output steps): the ELU'd input rows the
// tile needs (history rows for the first tile) are staged in shared memory with a padded row stride.
constexpr int kFinalTile = 128;

__global__ void final_conv_kernel(const bf16* __restrict__ x, int L, int C, int k, const bf16* __restrict__ w,
                                  const bf16* __restrict__ bias, const int* __restrict__ slot32,
                                  const bf16* __restrict__ state, int64_t state_row, int64_t hist_off,
                                  float* __restrict__ pcm, int elu_x) {
  extern __shared__ float fsm[];
  const int b = blockIdx.x, t0 = blockIdx.y * kFinalTile;
  const int P = k - 1, S = C + 1;  // padded stride: conflict-free column reads
  float* xs = fsm;                 // [(kFinalTile + P) rows, S]
  float* ws = fsm + (kFinalTile + P) * S;
  const bf16* hist = state + (int64_t)slot32[b] * state_row + hist_off;
  const int rows = min(kFinalTile, L - t0) + P;
  const int C8 = C / 8;
  const uint4* hist8 = reinterpret_cast<const uint4*>(hist);
  const uint4* x8 = reinterpret_cast<const uint4*>(x + (int64_t)b * L * C);
#pragma unroll 4
  for (int i = threadIdx.x; i < rows * C8; i += blockDim.x) {  // 16-byte loads, several in flight per thread
    const int rr = i / C8, c8 = i % C8;
    const int ji = t0 + rr;  // index into joined = [hist; elu(x)]
    float f[8];
    unpack8(ji < P ? hist8[ji * C8 + c8] : x8[(int64_t)(ji - P) * C8 + c8], f);
    float* d = xs + rr * S + c8 * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) d[e] = (ji < P || !elu_x) ? f[e] : rbf(elu(f[e]));
  }
  for (int i = threadIdx.x; i < k * C; i += blockDim.x) ws[i] = to_f(w[i]);
  __syncthreads();
  const int t = threadIdx.x;
  if (t0 + t >= L) return;
  float acc = 0.f;
  for (int j = 0; j < k; ++j)
    for (int c = 0; c < C; ++c) acc = fmaf(ws[j * C + c], xs[(t + j) * S + c], acc);
  pcm[(int64_t)b * L + t0 + t] = rbf(acc + to_f(bias[0]));
}

}  // namespace m3

// ================================================================================================ handle
using namespace m3;

struct m3_mimi {
  m3_mimi_config c{};
  const bf16 *books = nullptr, *proj_sem = nullptr, *proj_ac = nullptr, *upw = nullptr;
  std::vector<const bf16*> ln1_w, ln1_b, wqkv, wo, ln2_w, ln2_b, fc1, fc2, ls1, ls2;
  const float* inv_freq = nullptr;
  const bf16 *conv0_w = nullptr, *conv0_b = nullptr, *final_w = nullptr, *final_b = nullptr;
  std::vector<const bf16*> convt_w, convt_b, res1_w, res1_b, res2_w, res2_b;
  bf16* state = nullptr;
  bf16* kv = nullptr;
  int64_t *key_pos = nullptr, *tokens = nullptr;
  int64_t state_row = 0, up_off = 0, conv0_off = 0, final_off = 0;
  std::vector<StageDims> stages;
  void* ws = nullptr;
  // the decode's own cuBLAS workspace: a tick may run this decode on a second stream beside other library GEMMs
  unsigned char* blas_ws = nullptr;
  int *slot32 = nullptr, *status = nullptr;
  std::vector<CUtensorMap> kmap, vmap;  // per layer, over kv[layer][k|v] as [slot * heads + head][entry][head_dim]
  // fused SEANet stages (a suffix of the stages: first_fused .. n_ratios-1)
  int first_fused = 1 << 30;
  std::vector<ConvTFused> ct;
  std::vector<ResFused> rs;
  StateCopy snap_regions{};
  FinalFused fin{};
  bool fin_fused = false;
  int sm_budget = 0;  // SMs the persistent SEANet kernels spread over (0: all)
  int64_t snap_row = 0;
  void* fws = nullptr;  // repacked transposed-conv weights + the state snapshot
  bf16* snap = nullptr;
  int64_t* pos = nullptr;
  bf16 *a_sem = nullptr, *a_ac = nullptr, *p_sem = nullptr, *p_ac = nullptr, *h = nullptr, *y = nullptr,
       *qkv = nullptr, *q = nullptr, *att = nullptr, *ob = nullptr, *ff = nullptr, *act0 = nullptr, *act1 = nullptr,
       *col = nullptr, *tmp = nullptr;
  float* z = nullptr;
};

// Every GEMM of the decode runs on the handle's own cuBLAS workspace.
static int mgemm(const m3_mimi* m, GemmDesc g, cudaStream_t s) {
  g.ws = m->blas_ws;
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

// State row layout (elements, channels-last): upsample tail [s, H]; conv0 history [k-1, H]; per stage: convT tail
// [r, cout], resnet k3 history [res_kernel-1, cout]; final conv history [last_kernel-1, num_filters].
int64_t plan(const m3_mimi_config& c, std::vector<StageDims>* st, int64_t* up, int64_t* c0, int64_t* fin) {
  int64_t off = 0;
  *up = off;
  off += (int64_t)c.upsample_stride * c.hidden;
  *c0 = off;
  off += (int64_t)(c.kernel - 1) * c.hidden;
  int ch = (1 << c.n_ratios) * c.num_filters;
  int L = c.upsample_stride;
  for (int i = 0; i < c.n_ratios; ++i) {
    StageDims s{ch, ch / 2, c.ratios[i], L, 0, 0};
    s.tail_off = off;
    off += (int64_t)s.r * s.cout;
    s.hist_off = off;
    off += (int64_t)(c.res_kernel - 1) * s.cout;
    if (st) st->push_back(s);
    L *= s.r;
    ch /= 2;
  }
  *fin = off;
  off += (int64_t)(c.last_kernel - 1) * c.num_filters;
  return off;
}
}  // namespace

extern "C" int64_t m3_mimi_state_elems(const m3_mimi_config* cfg) {
  if (!cfg || cfg->n_ratios < 1 || cfg->n_ratios > 8) return -1;
  int64_t a, b, c;
  return plan(*cfg, nullptr, &a, &b, &c);
}

// Pick the SEANet stages that run fused (the longest suffix of stages whose shapes the fused kernels support) and
// build what they need: repacked transposed-conv weights, the state snapshot layout, and tensor maps over the two
// activation buffers (stage input e in act0 -> transposed-conv output u in act1 -> residual-block output in act0).
static int setup_fused_seanet(m3_mimi* m) {
  const m3_mimi_config& c = m->c;
  const int n = (int)m->stages.size();
  auto a16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  auto fusable = [&](int i) {
    const StageDims& sd = m->stages[i];
    const int hid = sd.cout / c.compress;
    return c.res_kernel == 3 && sd.L >= 16 && convt_fused_ok(sd.cin, sd.cout, sd.r) && res_fused_ok(sd.cout, hid) &&
           sd.tail_off % 8 == 0 && sd.hist_off % 8 == 0 && (sd.r * sd.cout) % 8 == 0 && a16(m->convt_b[i]) &&
           a16(m->res1_w[i]) && a16(m->res2_w[i]);   // the kernels read these with 16-byte loads
  };
  int first = n;
  while (first > 0 && fusable(first - 1)) --first;
  if (first == n || m->state_row % 8 != 0 || n - first > 8) return M3_OK;
  EncodeTiled enc;
  M3_TRY(tensor_map_encoder(&enc));
  size_t wbytes = 0;
  StateCopy sc{};
  int64_t srow = 0;
  for (int i = first; i < n; ++i) {
    const StageDims& sd = m->stages[i];
    wbytes += (size_t)sd.r * sd.cout * 2 * sd.cin * 2;
    sc.off[sc.n] = sd.tail_off;
    sc.len[sc.n] = sd.r * sd.cout;
    sc.dst_off[sc.n++] = srow;
    srow += sd.r * sd.cout;
    sc.off[sc.n] = sd.hist_off;
    sc.len[sc.n] = 2 * sd.cout;
    sc.dst_off[sc.n++] = srow;
    srow += 2 * sd.cout;
  }
  wbytes = (wbytes + 255) / 256 * 256;
  const size_t snap_bytes = (size_t)c.max_rows * srow * 2;
  M3_CUDA(cudaMalloc(&m->fws, wbytes + snap_bytes));
  bf16* wc = (bf16*)m->fws;
  bf16* snap = (bf16*)((char*)m->fws + wbytes);
  M3_TRY(seanet_fused_init());
  auto map3 = [&](CUtensorMap* map, bf16* base, int ch, int steps, int box_rows) -> int {
    const cuuint64_t dims[3] = {(cuuint64_t)ch, (cuuint64_t)steps, (cuuint64_t)c.max_rows};
    const cuuint64_t strides[2] = {(cuuint64_t)ch * 2, (cuuint64_t)steps * ch * 2};
    const cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    M3_REQUIRE(r == CUDA_SUCCESS, M3_ERR_CUDA, "SEANet tensor map failed (%d)", (int)r);
    return M3_OK;
  };
  int si = 0;
  for (int i = first; i < n; ++i, si += 2) {
    const StageDims& sd = m->stages[i];
    ConvTFused ct{};
    M3_TRY(map3(&ct.amap, m->act0, sd.cin, sd.L, 128));
    ct.wc = wc;
    M3_TRY(launch_convt_repack(m->convt_w[i], sd.r, sd.cout, sd.cin, wc, 0));
    {
      const int N = sd.r * sd.cout, K = 2 * sd.cin;
      const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
      const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
      const bool pers = convt_persistent_ok(sd.cin, sd.cout, sd.r);
      const cuuint32_t box[2] = {64, (cuuint32_t)(pers ? 128 : convt_fused_bn(N))};
      const cuuint32_t estr[2] = {1, 1};
      const CUresult r = enc(&ct.bmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, wc, dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      M3_REQUIRE(r == CUDA_SUCCESS, M3_ERR_CUDA, "SEANet weight tensor map failed (%d)", (int)r);
      if (pers) {  // the persistent form stores u by TMA: [R][L][N], 32 x 32 boxes, 64-byte swizzle
        const cuuint64_t ud[3] = {(cuuint64_t)N, (cuuint64_t)sd.L, (cuuint64_t)c.max_rows};
        const cuuint64_t us[2] = {(cuuint64_t)N * 2, (cuuint64_t)sd.L * N * 2};
        const cuuint32_t ub[3] = {32, 32, 1};
        const cuuint32_t ue[3] = {1, 1, 1};
        const CUresult r2 = enc(&ct.smap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, m->act1, ud, us, ub, ue,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                                CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        M3_REQUIRE(r2 == CUDA_SUCCESS, M3_ERR_CUDA, "SEANet output tensor map failed (%d)", (int)r2);
      }
    }
    wc += (size_t)sd.r * sd.cout * 2 * sd.cin;
    ct.bias = m->convt_b[i];
    ct.tail_in = snap + sc.dst_off[si];
    ct.in_row = srow;
    ct.state = m->state;
    ct.state_row = m->state_row;
    ct.tail_off = sd.tail_off;
    ct.slot32 = m->slot32;
    ct.u = m->act1;
    ct.L = sd.L;
    ct.r = sd.r;
    ct.cin = sd.cin;
    ct.cout = sd.cout;
    ResFused rs{};
    M3_TRY(map3(&rs.umap, m->act1, sd.cout, sd.L * sd.r, 130));
    rs.w1 = m->res1_w[i];
    rs.b1 = m->res1_b[i];
    rs.w2 = m->res2_w[i];
    rs.b2 = m->res2_b[i];
    rs.hist_in = snap + sc.dst_off[si + 1];
    rs.in_row = srow;
    rs.state = m->state;
    rs.state_row = m->state_row;
    rs.hist_off = sd.hist_off;
    rs.slot32 = m->slot32;
    rs.e = m->act0;
    rs.Lo = sd.L * sd.r;
    rs.cout = sd.cout;
    rs.hid = sd.cout / c.compress;
    m->ct.push_back(ct);
    m->rs.push_back(rs);
  }
  if (first < n && final_fused_ok(c.num_filters, c.last_kernel) && m->final_off % 8 == 0) {
    const StageDims& ls = m->stages.back();
    M3_TRY(map3(&m->fin.xmap, m->act0, c.num_filters, ls.L * ls.r, 128 + c.last_kernel - 1));
    m->fin.taps = c.last_kernel;
    m->fin.w = m->final_w;
    m->fin.bias = m->final_b;
    m->fin.state = m->state;
    m->fin.state_row = m->state_row;
    m->fin.hist_off = m->final_off;
    m->fin.slot32 = m->slot32;
    m->fin.L = ls.L * ls.r;
    m->fin_fused = true;
  }
  M3_CUDA(cudaDeviceSynchronize());  // the weight repack finished before the first decode
  m->first_fused = first;
  m->snap_regions = sc;
  m->snap_row = srow;
  m->snap = snap;
  return M3_OK;
}

extern "C" int m3_mimi_create(const m3_mimi_config* cfg, const m3_mimi_weights* w, m3_mimi** out) {
  M3_REQUIRE(cfg && w && out, M3_ERR_ARG, "m3_mimi_create: null argument");
  const m3_mimi_config& c = *cfg;
  M3_REQUIRE(c.n_ratios >= 1 && c.n_ratios <= 8, M3_ERR_ARG, "n_ratios %d", c.n_ratios);
  const int hd = c.hidden / c.heads;
  M3_REQUIRE(c.hidden % c.heads == 0 && hd % 8 == 0 && hd <= 128 && c.heads <= 32, M3_ERR_UNSUPPORTED, "head dim");
  M3_REQUIRE(c.ring >= c.window + c.upsample_stride, M3_ERR_ARG, "ring %d", c.ring);
  M3_REQUIRE((hd == 32 || hd == 64) && c.ring % kRingBlk == 0 &&
                 (c.upsample_stride == 1 || c.upsample_stride == 2 || c.upsample_stride == 4),
             M3_ERR_UNSUPPORTED,
             "ring attention: head dim %d (32 or 64), ring %d (a multiple of %d), %d tokens per frame (1, 2 or 4)", hd,
             c.ring, kRingBlk, c.upsample_stride);
  M3_REQUIRE(c.upsample_stride <= 4 && c.upsample_stride <= 8 && c.kernel - 1 <= 8 && c.res_kernel - 1 <= 8 &&
                 c.last_kernel - 1 <= 8,
             M3_ERR_UNSUPPORTED, "kernel sizes");
  M3_REQUIRE(c.hidden % 8 == 0 && c.ffn % 8 == 0, M3_ERR_UNSUPPORTED, "sizes must be multiples of 8");
  auto* m = new m3_mimi();
  m->c = c;
  m->books = (const bf16*)w->codebooks;
  m->proj_sem = (const bf16*)w->proj_sem;
  m->proj_ac = (const bf16*)w->proj_ac;
  m->upw = (const bf16*)w->upsample;
  for (int i = 0; i < c.layers; ++i) {
    m->ln1_w.push_back((const bf16*)w->ln1_w[i]);
    m->ln1_b.push_back((const bf16*)w->ln1_b[i]);
    m->wqkv.push_back((const bf16*)w->wqkv[i]);
    m->wo.push_back((const bf16*)w->wo[i]);
    m->ln2_w.push_back((const bf16*)w->ln2_w[i]);
    m->ln2_b.push_back((const bf16*)w->ln2_b[i]);
    m->fc1.push_back((const bf16*)w->fc1[i]);
    m->fc2.push_back((const bf16*)w->fc2[i]);
    m->ls1.push_back((const bf16*)w->ls1[i]);
    m->ls2.push_back((const bf16*)w->ls2[i]);
  }
  m->inv_freq = w->inv_freq;
  m->conv0_w = (const bf16*)w->conv0_w;
  m->conv0_b = (const bf16*)w->conv0_b;
  m->final_w = (const bf16*)w->final_w;
  m->final_b = (const bf16*)w->final_b;
  for (int i = 0; i < c.n_ratios; ++i) {
    m->convt_w.push_back((const bf16*)w->convt_w[i]);
    m->convt_b.push_back((const bf16*)w->convt_b[i]);
    m->res1_w.push_back((const bf16*)w->res1_w[i]);
    m->res1_b.push_back((const bf16*)w->res1_b[i]);
    m->res2_w.push_back((const bf16*)w->res2_w[i]);
    m->res2_b.push_back((const bf16*)w->res2_b[i]);
  }
  m->state = (bf16*)w->conv_state;
  m->kv = (bf16*)w->kv;
  m->key_pos = w->key_pos;
  m->tokens = w->tokens;
  m->state_row = plan(c, &m->stages, &m->up_off, &m->conv0_off, &m->final_off);
  // scratch sized for max_rows
  const size_t R = c.max_rows, T = c.upsample_stride, H = c.hidden;
  size_t act = R * T * H, col = R * T * c.kernel * H, zf = R * T * H * 2;
  for (const StageDims& s : m->stages) {
    act = std::max(act, R * s.L * s.r * (size_t)s.cout);
    col = std::max(col, R * s.L * s.r * (size_t)c.res_kernel * s.cout);
    zf = std::max(zf, R * s.L * (size_t)2 * s.r * s.cout);
    zf = std::max(zf, R * s.L * s.r * (size_t)s.cout);
  }
  zf = std::max(zf, R * T * (size_t)(1 << c.n_ratios) * c.num_filters);
  act = std::max(act, R * T * (size_t)(1 << c.n_ratios) * c.num_filters);  // conv0 output
  size_t bytes = 0;
  auto add = [&](size_t n) { bytes += (n + 255) / 256 * 256; };
  add(R * 4); add(256); add(R * T * 8);
  add(R * c.codebook_dim * 2); add(R * c.codebook_dim * 2); add(R * H * 2); add(R * H * 2);
  add(R * T * H * 2); add(R * T * H * 2); add(R * T * 3 * H * 2); add(R * T * H * 2); add(R * T * H * 2);
  add(R * T * H * 2); add(R * T * c.ffn * 2);
  add(act * 2); add(act * 2); add(col * 2); add(act * 2); add(zf * 4);
  add(kBlasWorkspace);
  cudaError_t e = cudaMalloc(&m->ws, bytes);
  if (e != cudaSuccess) {
    delete m;
    set_error("m3_mimi_create: cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
    return M3_ERR_CUDA;
  }
  char* p = (char*)m->ws;
  m->slot32 = carve<int>(p, R);
  m->status = carve<int>(p, 64);
  m->pos = carve<int64_t>(p, R * T);
  m->a_sem = carve<bf16>(p, R * c.codebook_dim);
  m->a_ac = carve<bf16>(p, R * c.codebook_dim);
  m->p_sem = carve<bf16>(p, R * H);
  m->p_ac = carve<bf16>(p, R * H);
  m->h = carve<bf16>(p, R * T * H);
  m->y = carve<bf16>(p, R * T * H);
  m->qkv = carve<bf16>(p, R * T * 3 * H);
  m->q = carve<bf16>(p, R * T * H);
  m->att = carve<bf16>(p, R * T * H);
  m->ob = carve<bf16>(p, R * T * H);
  m->ff = carve<bf16>(p, R * T * c.ffn);
  m->act0 = carve<bf16>(p, act);
  m->act1 = carve<bf16>(p, act);
  m->col = carve<bf16>(p, col);
  m->tmp = carve<bf16>(p, act);
  m->z = carve<float>(p, zf);
  m->blas_ws = carve<unsigned char>(p, kBlasWorkspace);
  cudaMemset(m->status, 0, 256);
  {
    EncodeTiled enc;
    if (tensor_map_encoder(&enc) != M3_OK) {
      cudaFree(m->ws);
      delete m;
      return M3_ERR_CUDA;
    }
    const int64_t rows_all = c.max_slots + 1;
    const int64_t kv_half = rows_all * c.heads * c.ring * hd;
    const cuuint64_t dims[3] = {(cuuint64_t)hd, (cuuint64_t)c.ring, (cuuint64_t)(rows_all * c.heads)};
    const cuuint64_t strides[2] = {(cuuint64_t)hd * 2, (cuuint64_t)c.ring * hd * 2};
    const cuuint32_t box[3] = {(cuuint32_t)hd, (cuuint32_t)kRingBlk, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    m->kmap.resize(c.layers);
    m->vmap.resize(c.layers);
    for (int li = 0; li < c.layers; ++li)
      for (int kvv = 0; kvv < 2; ++kvv) {
        bf16* base = m->kv + (int64_t)(2 * li + kvv) * kv_half;
        const CUresult r = (reinterpret_cast<uintptr_t>(base) & 15)
                               ? CUDA_ERROR_INVALID_VALUE
                               : enc(kvv ? &m->vmap[li] : &m->kmap[li], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims,
                                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                     hd == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS) {
          cudaFree(m->ws);
          delete m;
          set_error("m3_mimi_create: ring tensor map of layer %d failed (%d); kv must be 16-byte aligned", li, (int)r);
          return M3_ERR_ARG;
        }
      }
    const int rs = (int)(sizeof(RingMmaSmem<64>) + 1024);
    cudaFuncSetAttribute(ring_mma_kernel<64, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, rs);
    cudaFuncSetAttribute(ring_mma_kernel<64, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, rs);
    cudaFuncSetAttribute(ring_mma_kernel<64, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, rs);
  }
  if (const int rc = setup_fused_seanet(m); rc != M3_OK) {
    m3_mimi_destroy(m);
    return rc;
  }
  *out = m;
  return M3_OK;
}

extern "C" int m3_mimi_destroy(m3_mimi* m) {
  if (!m) return M3_OK;
  cudaFree(m->ws);
  if (m->fws) cudaFree(m->fws);
  delete m;
  return M3_OK;
}

extern "C" int m3_mimi_convt(m3_mimi* m, int32_t stage, int32_t rows, int64_t* bytes, m3_stream stream) {
  M3_REQUIRE(m, M3_ERR_ARG, "m3_mimi_convt: null handle");
  const int n = (int)m->stages.size();
  M3_REQUIRE(stage >= m->first_fused && stage < n && rows > 0 && rows <= m->c.max_rows, M3_ERR_RANGE,
             "m3_mimi_convt: stage %d is not a fused stage or rows %d out of range", stage, rows);
  const StageDims& sd = m->stages[stage];
  ConvTFused ct = m->ct[stage - m->first_fused];
  // the tails go to the snapshot scratch (re-taken at the start of every decode), not to the streams' state
  ct.state = m->snap + m->snap_regions.dst_off[2 * (stage - m->first_fused)];
  ct.state_row = 0;
  ct.tail_off = 0;
  if (bytes) *bytes = ((int64_t)rows * sd.L * sd.cin + (int64_t)rows * sd.L * sd.r * sd.cout) * 2;
  return launch_convt_fused(ct, rows, reinterpret_cast<cudaStream_t>(stream), m->status, m->sm_budget);
}

extern "C" int m3_mimi_set_sm_budget(m3_mimi* m, int32_t sms) {
  M3_REQUIRE(m && sms >= 0, M3_ERR_ARG, "m3_mimi_set_sm_budget: null handle or negative budget");
  m->sm_budget = sms;
  return M3_OK;
}

extern "C" int m3_mimi_status(m3_mimi* m, int32_t* status, int32_t clear) {
  M3_REQUIRE(m && status, M3_ERR_ARG, "m3_mimi_status: null argument");
  M3_CUDA(cudaMemcpy(status, m->status, sizeof(int32_t), cudaMemcpyDeviceToHost));
  if (clear) M3_CUDA(cudaMemset(m->status, 0, sizeof(int32_t)));
  return M3_OK;
}

__global__ void mimi_reset_kernel(bf16* state, int64_t state_row, int64_t* key_pos, int ring, int64_t* tokens,
                                  int slot) {
  for (int64_t i = threadIdx.x; i < state_row; i += blockDim.x) state[(int64_t)slot * state_row + i] = to_bf(0.f);
  for (int i = threadIdx.x; i < ring; i += blockDim.x) key_pos[(int64_t)slot * ring + i] = kNever;
  if (threadIdx.x == 0) tokens[slot] = 0;
}

extern "C" int m3_mimi_reset(m3_mimi* m, int32_t slot, int32_t zero_kv, m3_stream stream) {
  M3_REQUIRE(m, M3_ERR_ARG, "m3_mimi_reset: null handle");
  M3_REQUIRE(slot >= 0 && slot <= m->c.max_slots, M3_ERR_RANGE, "slot %d outside [0, %d]", slot, m->c.max_slots);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  mimi_reset_kernel<<<1, 256, 0, s>>>(m->state, m->state_row, m->key_pos, m->c.ring, m->tokens, slot);
  M3_LAUNCHED();
  if (zero_kv) {  // [layers, 2, rows, heads, ring, hd]: one strided block per (layer, k/v)
    const int hd = m->c.hidden / m->c.heads;
    const size_t blk = (size_t)m->c.heads * m->c.ring * hd;
    const size_t rows = m->c.max_slots + 1;
    for (int l = 0; l < 2 * m->c.layers; ++l)
      M3_CUDA(cudaMemsetAsync(m->kv + ((size_t)l * rows + slot) * blk, 0, blk * 2, s));
  }
  return M3_OK;
}

__global__ void mimi_prep_kernel(const int64_t* __restrict__ slots, int rows, int max_slots, int* __restrict__ slot32,
                                 int* status) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  int64_t s = slots[r];
  if (s < 0 || s > max_slots) {
    report(status, M3_DEV_BAD_SLOT);
    s = max_slots;
  }
  slot32[r] = (int)s;
}

extern "C" int m3_mimi_decode(m3_mimi* m, const int64_t* slots, const int64_t* codes, float* pcm, int32_t rows,
                              m3_stream stream) {
  M3_REQUIRE(m && slots && codes && pcm, M3_ERR_ARG, "m3_mimi_decode: null argument");
  const m3_mimi_config& c = m->c;
  M3_REQUIRE(rows >= 0 && rows <= c.max_rows, M3_ERR_RANGE, "rows %d > max_rows %d", rows, c.max_rows);
  if (rows == 0) return M3_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int R = rows, H = c.hidden, T = c.upsample_stride, hd = H / c.heads;
  const int nb = norm_block(H);
  mimi_prep_kernel<<<cdiv(R, 128), 128, 0, s>>>(slots, R, c.max_slots, m->slot32, m->status);
  M3_LAUNCHED();
  // RVQ decode -> two output projections (1x1 convs, bf16 outputs)
  rvq_gather_kernel<<<R, 128, 0, s>>>(codes, c.n_q, c.n_semantic, c.codebook_size, c.codebook_dim, m->books,
                                      m->a_sem, m->a_ac, m->status);
  M3_LAUNCHED();
  M3_TRY(mgemm(m, {m->a_sem, c.codebook_dim, m->proj_sem, c.codebook_dim, m->p_sem, H, R, H, c.codebook_dim, false},
               s));
  M3_TRY(mgemm(m, {m->a_ac, c.codebook_dim, m->proj_ac, c.codebook_dim, m->p_ac, H, R, H, c.codebook_dim, false},
               s));
  upsample_kernel<<<dim3(R, cdiv(H, 128)), 128, 0, s>>>(m->p_sem, m->p_ac, m->upw, T, m->slot32,
                                                         m->state + m->up_off, m->state_row, m->h, H);
  M3_LAUNCHED();
  // decoder transformer over the frame's T tokens
  tpos_kernel<<<cdiv(R, 128), 128, 0, s>>>(m->slot32, R, T, c.ring, m->tokens, m->key_pos, m->pos);
  M3_LAUNCHED();
  const int64_t rows_all = c.max_slots + 1;
  const int64_t slot_stride = (int64_t)c.heads * c.ring * hd;  // one slot's block inside kv[layer][k|v]
  const int64_t kv_half = rows_all * slot_stride;
  M3_TRY(launch_add_ln(R * T, m->h, 1, H, 0, nullptr, nullptr, 0, nullptr, nullptr, m->y, m->ln1_w[0], m->ln1_b[0],
                c.norm_eps, H, s));
  for (int li = 0; li < c.layers; ++li) {
    M3_TRY(mgemm(m, {m->y, H, m->wqkv[li], H, m->qkv, 3 * H, R * T, 3 * H, H, false}, s));
    bf16* kr = m->kv + (int64_t)li * 2 * kv_half;
    mimi_rope_kernel<<<R * T, 32 * c.heads, 0, s>>>(m->qkv, m->pos, m->inv_freq, m->slot32, T, c.heads, hd, c.ring,
                                                   m->q, kr, kr + kv_half, slot_stride);
    M3_LAUNCHED();
    {
      const dim3 grid(R, c.heads);
      const float qs = 1.4426950408889634f / sqrtf((float)hd);
#define M3_RING_MMA(HDD, TT)                                                                                      \
  ring_mma_kernel<HDD, TT><<<grid, 128, sizeof(RingMmaSmem<HDD>) + 1024, s>>>(                                    \
      m->kmap[li], m->vmap[li], m->q, m->key_pos, m->pos, m->slot32, c.heads, c.ring, c.window, qs, m->att,        \
      m->status)
      if (hd == 64) {
        if (T == 1) M3_RING_MMA(64, 1); else if (T == 2) M3_RING_MMA(64, 2); else M3_RING_MMA(64, 4);
      } else {
        if (T == 1) M3_RING_MMA(32, 1); else if (T == 2) M3_RING_MMA(32, 2); else M3_RING_MMA(32, 4);
      }
#undef M3_RING_MMA
    }
    M3_LAUNCHED();
    M3_TRY(mgemm(m, {m->att, H, m->wo[li], H, m->ob, H, R * T, H, H, false}, s));
    scale_add_ln_kernel<<<R * T, nb, 0, s>>>(m->h, m->ob, m->ls1[li], m->y, m->ln2_w[li], m->ln2_b[li], c.norm_eps,
                                             H);
    M3_LAUNCHED();
    GemmDesc fc1{m->y, H, m->fc1[li], H, m->ff, c.ffn, R * T, c.ffn, H, false};
    fc1.act = kActGelu;
    if (!gemv_path(fc1)) fc1.act = kActNone;  // a few streams: GELU in the GEMV epilogue; else its own pass
    M3_TRY(mgemm(m, fc1, s));
    if (fc1.act == kActNone) {
      const int64_t n8 = (int64_t)R * T * c.ffn / 8;
      gelu_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, s>>>(m->ff, n8);
      M3_LAUNCHED();
    }
    M3_TRY(mgemm(m, {m->ff, c.ffn, m->fc2[li], c.ffn, m->ob, H, R * T, H, c.ffn, false}, s));
    const bool last = li + 1 == c.layers;
    scale_add_ln_kernel<<<R * T, nb, 0, s>>>(m->h, m->ob, m->ls2[li], m->y, last ? nullptr : m->ln1_w[li + 1],
                                             last ? nullptr : m->ln1_b[li + 1], c.norm_eps, H);
    M3_LAUNCHED();
  }
  tokens_advance_kernel<<<cdiv(R, 128), 128, 0, s>>>(m->slot32, R, T, c.max_slots, m->tokens);
  M3_LAUNCHED();
  // SEANet: conv0 (k taps, hidden -> C0)
  const int C0 = (1 << c.n_ratios) * c.num_filters;
  im2col_kernel<<<dim3(R, cdiv(T * H / 8, 256)), 256, 0, s>>>(m->h, T, H, c.kernel, 0, m->slot32, m->state,
                                                                m->state_row, m->conv0_off, m->col);
  M3_LAUNCHED();
  conv_hist_kernel<<<dim3(R, cdiv(H / 8, 128)), 128, 0, s>>>(m->h, T, H, c.kernel, 0, m->slot32, m->state,
                                                              m->state_row, m->conv0_off);
  M3_LAUNCHED();
  M3_TRY(mgemm(m, {m->col, (int64_t)c.kernel * H, m->conv0_w, (int64_t)c.kernel * H, m->z, C0, R * T, C0, c.kernel * H,
               true},
              s));
  int64_t n = (int64_t)R * T * C0 / 8;
  const int nst = c.n_ratios, first_fused = std::min(m->first_fused, nst);
  bias_epilogue_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(m->z, m->conv0_b, (int64_t)R * T, C0,
                                                                   first_fused == 0 ? 1 : 0, nullptr, m->act0);
  M3_LAUNCHED();
  if (first_fused < nst)  // the fused stages read their previous state from a snapshot and rewrite it in place
    M3_TRY(launch_state_snapshot(m->state, m->state_row, m->slot32, R, m->snap_regions, m->snap, m->snap_row, s));
  bf16* x = m->act0;
  bf16* other = m->act1;
  for (int i = 0; i < nst; ++i) {
    const StageDims& sd = m->stages[i];
    if (i >= first_fused) {  // e (act0) -> transposed conv -> u (act1) -> residual block -> next e (act0)
      M3_TRY(launch_convt_fused(m->ct[i - first_fused], R, s, m->status, m->sm_budget));
      M3_TRY(launch_res_fused(m->rs[i - first_fused], R, s, m->status, m->sm_budget));
      x = m->act0;
      continue;
    }
    const int64_t Min = (int64_t)R * sd.L, Mout = Min * sd.r;
    // ELU -> ConvTranspose1d as X . Wt^T (fp32 contributions) -> fold with the overlap tail
    elu_kernel<<<(unsigned)((Min * sd.cin / 8 + 255) / 256), 256, 0, s>>>(x, m->tmp, Min * sd.cin / 8);
    M3_LAUNCHED();
    M3_TRY(mgemm(m, {m->tmp, sd.cin, m->convt_w[i], sd.cin, m->z, 2 * sd.r * sd.cout, (int)Min, 2 * sd.r * sd.cout,
                     sd.cin, true},
                 s));
    convt_fold_kernel<<<dim3(R, cdiv(sd.L * sd.r * sd.cout / 8, 256)), 256, 0, s>>>(
        m->z, m->convt_b[i], sd.L, sd.r, sd.cout, m->slot32, m->state, m->state_row, sd.tail_off, other);
    M3_LAUNCHED();
    convt_tail_kernel<<<dim3(R, cdiv(sd.r * sd.cout / 8, 128)), 128, 0, s>>>(m->z, m->convt_b[i], sd.L, sd.r, sd.cout,
                                                                             m->slot32, m->state, m->state_row,
                                                                             sd.tail_off);
    M3_LAUNCHED();
    std::swap(x, other);  // x = stage output y (residual)
    // resnet: ELU -> conv k3 (history) -> ELU -> conv k1 -> + y
    const int hid = sd.cout / c.compress;
    const int Lo = sd.L * sd.r;
    im2col_kernel<<<dim3(R, cdiv(Lo * sd.cout / 8, 256)), 256, 0, s>>>(x, Lo, sd.cout, c.res_kernel, 1, m->slot32,
                                                                       m->state, m->state_row, sd.hist_off, m->col);
    M3_LAUNCHED();
    conv_hist_kernel<<<dim3(R, cdiv(sd.cout / 8, 128)), 128, 0, s>>>(x, Lo, sd.cout, c.res_kernel, 1, m->slot32,
                                                                      m->state, m->state_row, sd.hist_off);
    M3_LAUNCHED();
    M3_TRY(mgemm(m, {m->col, (int64_t)c.res_kernel * sd.cout, m->res1_w[i], (int64_t)c.res_kernel * sd.cout, m->z, hid,
                 (int)Mout, hid, c.res_kernel * sd.cout, true},
                s));
    n = Mout * hid / 8;
    bias_epilogue_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(m->z, m->res1_b[i], Mout, hid, 1, nullptr,
                                                                     m->tmp);
    M3_LAUNCHED();
    M3_TRY(mgemm(m, {m->tmp, hid, m->res2_w[i], hid, m->z, sd.cout, (int)Mout, sd.cout, hid, true}, s));
    n = Mout * sd.cout / 8;
    if (i + 1 == first_fused && first_fused < nst) {  // the next stage is fused: hand it e = ELU(y) in act0 (in place when x is act0)
      bias_epilogue_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(m->z, m->res2_b[i], Mout, sd.cout, 3, x,
                                                                       m->act0);
      M3_LAUNCHED();
      x = m->act0;
      other = m->act1;
      continue;
    }
    bias_epilogue_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(m->z, m->res2_b[i], Mout, sd.cout, 2, x, other);
    M3_LAUNCHED();
    std::swap(x, other);
  }
  const StageDims& last = m->stages.back();
  const int Lf = last.L * last.r;
  const size_t fsmem = ((size_t)(kFinalTile + c.last_kernel - 1) * (c.num_filters + 1) +
                        (size_t)c.last_kernel * c.num_filters) * sizeof(float);
  const int elu_x = first_fused < nst ? 0 : 1;  // the fused stages hand over ELU(y)
  if (m->fin_fused) {
    FinalFused fp = m->fin;
    fp.pcm = pcm;
    M3_TRY(launch_final_fused(fp, R, s, m->status));
  } else {
    final_conv_kernel<<<dim3(R, cdiv(Lf, kFinalTile)), kFinalTile, fsmem, s>>>(
        x, Lf, c.num_filters, c.last_kernel, m->final_w, m->final_b, m->slot32, m->state, m->state_row,
        m->final_off, pcm, elu_x);
    M3_LAUNCHED();
  }
  conv_hist_kernel<<<dim3(R, cdiv(c.num_filters / 8, 128)), 128, 0, s>>>(x, Lf, c.num_filters, c.last_kernel, elu_x,
                                                                          m->slot32, m->state, m->state_row,
                                                                          m->final_off);
  M3_LAUNCHED();
  return M3_OK;
}
