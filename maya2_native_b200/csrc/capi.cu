// Library-wide C ABI pieces: error reporting, version, and the engine's per-tick readout packing.
#include <atomic>
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

namespace m3 {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

const char* last_error() { return g_err; }

static std::atomic<long long> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

// One row per seat: [stop code, cb0, pcm16 packed four samples per int64] (maya3/engine.py:557-561):
// pcm16 = round(clamp(pcm, -1, 1) * 32767) with round-half-to-even, as torch.round.
__global__ void pack_readout_kernel(const int64_t* __restrict__ code, const int64_t* __restrict__ cb0,
                                    const float* __restrict__ pcm, int64_t* __restrict__ packed, int spf) {
  const int row = blockIdx.x;
  const int words = spf / 4;
  int64_t* out = packed + (int64_t)row * (2 + words);
  if (threadIdx.x == 0) {
    out[0] = code[row];
    out[1] = cb0[row];
  }
  const float4* src = reinterpret_cast<const float4*>(pcm + (int64_t)row * spf);
  for (int w = threadIdx.x; w < words; w += blockDim.x) {
    const float4 v = src[w];
    const float f[4] = {v.x, v.y, v.z, v.w};
    uint64_t word = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float c = fminf(fmaxf(f[e], -1.f), 1.f) * 32767.f;
      const int16_t q = (int16_t)__float2int_rn(c);
      word |= (uint64_t)(uint16_t)q << (16 * e);
    }
    out[2 + w] = (int64_t)word;
  }
}

// One thread waits, with at most `polls` polls, on an mbarrier that nothing arrives on: the bounded-wait path every
// kernel of this library takes when a copy or a peer never completes (it records M3_DEV_TIMEOUT and gives up).
__global__ void selftest_timeout_kernel(int polls, int* status) {
  __shared__ uint64_t bar;
  mbar_init(&bar, 1);
  fence_mbar_init();
  for (int i = 0; i < polls; ++i)
    if (mbar_try_wait(&bar, 0)) return;
  report(status, M3_DEV_TIMEOUT);
  mbar_arrive(&bar);  // complete the phase so the barrier is left in a finished state
}

// One request's slot, every field in one launch (m3_slot_reset).
__global__ void slot_reset_kernel(const m3_slot_state st, const m3_slot_init in) {
  const int s = in.slot;
  if (threadIdx.x == 0) {
    st.frames[s] = 0;
    st.min_frames[s] = in.min_frames;
    st.hazard[s] = 0.f;
    st.aeos_bias[s] = 0.f;
    st.seed[s] = in.seed;
    st.ctr[s] = 0;
    st.temp[s] = in.temp;
    st.top_k[s] = in.top_k;
    st.top_p[s] = in.top_p;
    st.rep[s] = in.rep;
    st.row_seed[s] = in.row_seed;
    st.row_ctr[s] = 0;
    st.lengths[s] = in.length;
  }
  for (int i = threadIdx.x; i < st.hist_len; i += blockDim.x) st.hist[(int64_t)s * st.hist_len + i] = -1;
  const uint4* src = reinterpret_cast<const uint4*>(in.cross_src);
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(st.cross_const) + (int64_t)s * st.cross_elems);
  for (int i = threadIdx.x; i < st.cross_elems / 8; i += blockDim.x) dst[i] = src[i];
}

}  // namespace m3

extern "C" int m3_selftest_timeout(int32_t polls, int32_t* status) {
  M3_REQUIRE(status && polls >= 0 && polls <= (1 << 20), M3_ERR_ARG, "m3_selftest_timeout: polls %d", polls);
  int* d = nullptr;
  M3_CUDA(cudaMalloc(&d, sizeof(int)));
  M3_CUDA(cudaMemset(d, 0, sizeof(int)));
  m3::selftest_timeout_kernel<<<1, 1>>>(polls, d);
  M3_LAUNCHED();
  const cudaError_t e = cudaMemcpy(status, d, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(d);
  M3_CUDA(e);
  return M3_OK;
}

extern "C" const char* m3_last_error(void) { return m3::last_error(); }

extern "C" int m3_version(void) { return 1; }

extern "C" int64_t m3_launch_count(void) { return m3::launch_count(); }

extern "C" int m3_pack_readout(const int64_t* code, const int64_t* cb0, const float* pcm, int64_t* packed,
                               int32_t rows, int32_t spf, m3_stream stream) {
  M3_REQUIRE(code && cb0 && pcm && packed, M3_ERR_ARG, "m3_pack_readout: null argument");
  M3_REQUIRE(spf % 4 == 0 && rows >= 0, M3_ERR_ARG, "m3_pack_readout: spf %d not a multiple of 4", spf);
  if (rows == 0) return M3_OK;
  m3::pack_readout_kernel<<<rows, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(code, cb0, pcm, packed, spf);
  M3_LAUNCHED();
  return M3_OK;
}

extern "C" int m3_slot_reset(const m3_slot_state* st, const m3_slot_init* init, m3_stream stream) {
  M3_REQUIRE(st && init && st->frames && st->min_frames && st->hazard && st->aeos_bias && st->seed && st->ctr &&
                 st->hist && st->temp && st->top_k && st->top_p && st->rep && st->row_seed && st->row_ctr &&
                 st->cross_const && st->lengths && init->cross_src,
             M3_ERR_ARG, "m3_slot_reset: null argument");
  M3_REQUIRE(init->slot >= 0 && init->slot < st->max_slots, M3_ERR_RANGE, "m3_slot_reset: slot %d outside [0, %d)",
             init->slot, st->max_slots);
  M3_REQUIRE(st->hist_len >= 0 && st->cross_elems >= 0 && st->cross_elems % 8 == 0 &&
                 (reinterpret_cast<uintptr_t>(st->cross_const) & 15) == 0 &&
                 (reinterpret_cast<uintptr_t>(init->cross_src) & 15) == 0,
             M3_ERR_ARG, "m3_slot_reset: speaker constant of %d elements must be 16-byte aligned rows",
             st->cross_elems);
  m3::slot_reset_kernel<<<1, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(*st, *init);
  M3_LAUNCHED();
  return M3_OK;
}
