// The engine tick as native calls (replaces the device half of Engine._tick, maya3/engine.py:534-561): gather each
// row's backbone input (a seat's feedback vector, or a prompt token embedding for inline-prefill rows), the backbone
// step, each seat's hidden state, the cb0 sampler, the depth loop, the feedback write-back, the Mimi frame and the
// packed readout, enqueued with no host synchronisation.
//
// The tick has two parts.  The main part (m3_tick_run_main) ends with the feedback write-back, which the next tick
// reads; the codec part (m3_tick_run_codec: Mimi frame + readout) is off that path, so it may run on a second stream
// beside the next tick's main part.  m3_tick_stage_codec hands one tick's outputs over: it copies the stop codes,
// cb0, codes and seat slots into one of two codec input sets, which the main part of the next tick does not touch.
// m3_tick_run is the three in order on one stream.
#include <vector>

#include "common.cuh"

namespace m3 {

int guard_check(const m3_guard_config* c, const m3_guard_state* s);  // guard.cu

// x[r] = feedback[slot[r]] for decode rows (token == kFromFeedback), embed[token[r]] for prefill rows, zero for
// padding rows (token == -1).
constexpr int64_t kFromFeedback = -2;

__global__ void gather_inputs_kernel(const int64_t* __restrict__ slots, const int64_t* __restrict__ tokens,
                                     const bf16* __restrict__ feedback, const bf16* __restrict__ embed,
                                     int64_t vocab, bf16* __restrict__ x, int D, int max_slots, int* status) {
  const int r = blockIdx.x;
  const uint4* src = nullptr;
  if (tokens[r] == kFromFeedback) {
    int64_t s = slots[r];
    if (s < 0 || s > max_slots) {
      report(status, M3_DEV_BAD_SLOT);
      s = max_slots;
    }
    src = reinterpret_cast<const uint4*>(feedback + s * D);
  } else {
    const int64_t t = tokens[r];
    if (t >= vocab) report(status, M3_DEV_BAD_CODE);
    if (t >= 0 && t < vocab) src = reinterpret_cast<const uint4*>(embed + t * D);
  }
  uint4* dst = reinterpret_cast<uint4*>(x + (int64_t)r * D);
  for (int i = threadIdx.x; i < D / 8; i += blockDim.x) dst[i] = src ? src[i] : make_uint4(0, 0, 0, 0);
}

// dst[i] = src[idx[i]] (rows of D bf16)
__global__ void gather_rows_kernel(const bf16* __restrict__ src, const int64_t* __restrict__ idx, int n_src,
                                   bf16* __restrict__ dst, int D) {
  const int i = blockIdx.x;
  int64_t j = idx[i];
  j = j < 0 ? 0 : (j >= n_src ? n_src - 1 : j);
  const uint4* s = reinterpret_cast<const uint4*>(src + j * D);
  uint4* d = reinterpret_cast<uint4*>(dst + (int64_t)i * D);
  for (int k = threadIdx.x; k < D / 8; k += blockDim.x) d[k] = s[k];
}

// dst[idx[i]] = src[i] for the first n rows (feedback[slot] = fb, maya3/engine.py:556)
__global__ void scatter_rows_kernel(const bf16* __restrict__ src, const int64_t* __restrict__ idx, int n,
                                    int max_slots, bf16* __restrict__ dst, int D) {
  const int i = blockIdx.x;
  if (i >= n) return;
  const int64_t j = idx[i];
  if (j < 0 || j > max_slots) return;
  const uint4* s = reinterpret_cast<const uint4*>(src + (int64_t)i * D);
  uint4* d = reinterpret_cast<uint4*>(dst + j * D);
  for (int k = threadIdx.x; k < D / 8; k += blockDim.x) d[k] = s[k];
}

// The codec inputs of one tick: c_code / c_cb0 / c_slot [seats], c_codes [seats, n_q] (one thread per int64).
__global__ void stage_codec_kernel(const int64_t* __restrict__ code, const int64_t* __restrict__ cb0,
                                   const int64_t* __restrict__ codes, const int64_t* __restrict__ s_slot, int seats,
                                   int n_q, int64_t* __restrict__ c_code, int64_t* __restrict__ c_cb0,
                                   int64_t* __restrict__ c_codes, int64_t* __restrict__ c_slot) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < seats * n_q) c_codes[i] = codes[i];
  if (i < seats) {
    c_code[i] = code[i];
    c_cb0[i] = cb0[i];
    c_slot[i] = s_slot[i];
  }
}

}  // namespace m3

using namespace m3;

struct m3_tick {
  m3_tick_config c{};
  void* ws = nullptr;
  bf16 *x = nullptr, *out = nullptr, *h = nullptr, *fb = nullptr;
  int64_t *code = nullptr, *cb0 = nullptr, *codes = nullptr;
  float* pcm = nullptr;
  int* status = nullptr;
  int64_t *c_code[2] = {}, *c_cb0[2] = {}, *c_codes[2] = {}, *c_slot[2] = {};  // the two codec input sets
  bool guard = false;  // m3_tick_set_guard: run the guards after the cb0 sampler
  m3_guard_config gc{};
  m3_guard_state gs{};
};

extern "C" int m3_tick_create(const m3_tick_config* cfg, m3_tick** out) {
  M3_REQUIRE(cfg && out && cfg->bb && cfg->cb0 && cfg->depth && cfg->mimi && cfg->feedback, M3_ERR_ARG,
             "m3_tick_create: null argument");
  M3_REQUIRE(cfg->hidden % 8 == 0 && cfg->spf % 4 == 0, M3_ERR_ARG, "m3_tick_create: sizes");
  auto* t = new m3_tick();
  t->c = *cfg;
  const size_t R = cfg->max_rows, S = cfg->max_seats, D = cfg->hidden;
  size_t bytes = 0;
  auto add = [&](size_t n) { bytes += (n + 255) / 256 * 256; };
  add(R * D * 2); add(R * D * 2); add(S * D * 2); add(S * D * 2); add(S * 8); add(S * 8); add(S * cfg->n_q * 8);
  add(S * cfg->spf * 4); add(256);
  for (int k = 0; k < 2; ++k) {
    add(S * 8); add(S * 8); add(S * cfg->n_q * 8); add(S * 8);
  }
  cudaError_t e = cudaMalloc(&t->ws, bytes);
  if (e != cudaSuccess) {
    delete t;
    set_error("m3_tick_create: cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
    return M3_ERR_CUDA;
  }
  char* p = (char*)t->ws;
  auto carve = [&](size_t n) {
    char* r = p;
    p += (n + 255) / 256 * 256;
    return r;
  };
  t->x = (bf16*)carve(R * D * 2);
  t->out = (bf16*)carve(R * D * 2);
  t->h = (bf16*)carve(S * D * 2);
  t->fb = (bf16*)carve(S * D * 2);
  t->code = (int64_t*)carve(S * 8);
  t->cb0 = (int64_t*)carve(S * 8);
  t->codes = (int64_t*)carve(S * cfg->n_q * 8);
  t->pcm = (float*)carve(S * cfg->spf * 4);
  t->status = (int*)carve(256);
  for (int k = 0; k < 2; ++k) {
    t->c_code[k] = (int64_t*)carve(S * 8);
    t->c_cb0[k] = (int64_t*)carve(S * 8);
    t->c_codes[k] = (int64_t*)carve(S * cfg->n_q * 8);
    t->c_slot[k] = (int64_t*)carve(S * 8);
  }
  cudaMemset(t->status, 0, 256);
  *out = t;
  return M3_OK;
}

extern "C" int m3_tick_destroy(m3_tick* t) {
  if (!t) return M3_OK;
  cudaFree(t->ws);
  delete t;
  return M3_OK;
}

extern "C" int m3_tick_status(m3_tick* t, int32_t* status, int32_t clear) {
  M3_REQUIRE(t && status, M3_ERR_ARG, "m3_tick_status: null argument");
  int32_t s[5] = {0, 0, 0, 0, 0};
  M3_CUDA(cudaMemcpy(&s[0], t->status, 4, cudaMemcpyDeviceToHost));
  M3_TRY(m3_backbone_status(t->c.bb, &s[1], clear));
  M3_TRY(m3_depth_status(t->c.depth, &s[2], clear));
  M3_TRY(m3_mimi_status(t->c.mimi, &s[3], clear));
  M3_TRY(m3_cb0_status(t->c.cb0, &s[4], clear));
  if (clear) M3_CUDA(cudaMemset(t->status, 0, 4));
  *status = 0;
  for (int i = 0; i < 5 && !*status; ++i) *status = s[i];
  return M3_OK;
}

extern "C" int m3_tick_run_main(m3_tick* t, const int64_t* plan, int32_t rows, int32_t seats, int32_t ctx,
                                int32_t apply_rep, int32_t apply_top_p, m3_stream stream) {
  M3_REQUIRE(t && plan, M3_ERR_ARG, "m3_tick_run_main: null argument");
  const m3_tick_config& c = t->c;
  M3_REQUIRE(rows >= 0 && rows <= c.max_rows && seats >= 0 && seats <= c.max_seats, M3_ERR_RANGE,
             "m3_tick_run_main: rows %d seats %d outside the configured maxima", rows, seats);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int D = c.hidden;
  // plan layout (int64): rows x {slot, offset, real, token}, then seats x {slot, row}
  const int64_t* r_slot = plan;
  const int64_t* r_off = plan + rows;
  const int64_t* r_real = plan + 2 * rows;
  const int64_t* r_tok = plan + 3 * rows;
  const int64_t* s_slot = plan + 4 * rows;
  const int64_t* s_row = plan + 4 * rows + seats;
  if (rows > 0) {
    gather_inputs_kernel<<<rows, 128, 0, s>>>(r_slot, r_tok, (const bf16*)c.feedback, (const bf16*)c.embed,
                                              c.vocab, t->x, D, c.max_slots, t->status);
    M3_LAUNCHED();
    M3_TRY(m3_backbone_step(c.bb, r_slot, r_off, r_real, t->x, t->out, rows, ctx, stream));
  }
  if (seats == 0) return M3_OK;
  gather_rows_kernel<<<seats, 128, 0, s>>>(t->out, s_row, rows > 0 ? rows : 1, t->h, D);
  M3_LAUNCHED();
  M3_TRY(m3_cb0_step(c.cb0, t->h, s_slot, t->code, t->cb0, seats, apply_rep, apply_top_p, stream));
  if (t->guard) M3_TRY(m3_guard_step(&t->gc, &t->gs, s_slot, t->code, t->cb0, seats, stream));
  M3_TRY(m3_depth_step(c.depth, s_slot, t->h, t->cb0, t->codes, t->fb, seats, stream));
  scatter_rows_kernel<<<seats, 128, 0, s>>>(t->fb, s_slot, seats, c.max_slots - 1, (bf16*)c.feedback, D);
  M3_LAUNCHED();
  return M3_OK;
}

extern "C" int m3_tick_stage_codec(m3_tick* t, const int64_t* plan, int32_t rows, int32_t seats, int32_t set,
                                   m3_stream stream) {
  M3_REQUIRE(t && plan, M3_ERR_ARG, "m3_tick_stage_codec: null argument");
  const m3_tick_config& c = t->c;
  M3_REQUIRE(rows >= 0 && rows <= c.max_rows && seats >= 0 && seats <= c.max_seats && (set == 0 || set == 1),
             M3_ERR_RANGE, "m3_tick_stage_codec: rows %d seats %d set %d out of range", rows, seats, set);
  if (seats == 0) return M3_OK;
  const int n = seats * c.n_q;
  stage_codec_kernel<<<cdiv(n, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      t->code, t->cb0, t->codes, plan + 4 * rows, seats, c.n_q, t->c_code[set], t->c_cb0[set], t->c_codes[set],
      t->c_slot[set]);
  M3_LAUNCHED();
  return M3_OK;
}

extern "C" int m3_tick_run_codec(m3_tick* t, int32_t seats, int32_t set, int64_t* packed, m3_stream stream) {
  M3_REQUIRE(t && packed, M3_ERR_ARG, "m3_tick_run_codec: null argument");
  const m3_tick_config& c = t->c;
  M3_REQUIRE(seats >= 0 && seats <= c.max_seats && (set == 0 || set == 1), M3_ERR_RANGE,
             "m3_tick_run_codec: seats %d set %d out of range", seats, set);
  if (seats == 0) return M3_OK;
  M3_TRY(m3_mimi_decode(c.mimi, t->c_slot[set], t->c_codes[set], t->pcm, seats, stream));
  M3_TRY(m3_pack_readout(t->c_code[set], t->c_cb0[set], t->pcm, packed, seats, c.spf, stream));
  return M3_OK;
}

extern "C" int m3_tick_run(m3_tick* t, const int64_t* plan, int32_t rows, int32_t seats, int32_t ctx,
                           int32_t apply_rep, int32_t apply_top_p, int64_t* packed, m3_stream stream) {
  M3_REQUIRE(t && plan && packed, M3_ERR_ARG, "m3_tick_run: null argument");
  M3_TRY(m3_tick_run_main(t, plan, rows, seats, ctx, apply_rep, apply_top_p, stream));
  M3_TRY(m3_tick_stage_codec(t, plan, rows, seats, 0, stream));
  return m3_tick_run_codec(t, seats, 0, packed, stream);
}

extern "C" int m3_tick_set_guard(m3_tick* t, const m3_guard_config* cfg, const m3_guard_state* st) {
  M3_REQUIRE(t, M3_ERR_ARG, "m3_tick_set_guard: null handle");
  if (!cfg) {
    t->guard = false;
    return M3_OK;
  }
  M3_TRY(guard_check(cfg, st));
  M3_REQUIRE(cfg->max_slots == t->c.max_slots, M3_ERR_ARG, "m3_tick_set_guard: guard max_slots %d, tick max_slots %d",
             cfg->max_slots, t->c.max_slots);
  t->gc = *cfg;
  t->gs = *st;
  t->guard = true;
  return M3_OK;
}

extern "C" int m3_tick_outputs(m3_tick* t, void** h, int64_t** codes, float** pcm) {
  M3_REQUIRE(t, M3_ERR_ARG, "m3_tick_outputs: null handle");
  if (h) *h = t->h;
  if (codes) *codes = t->codes;
  if (pcm) *pcm = t->pcm;
  return M3_OK;
}
