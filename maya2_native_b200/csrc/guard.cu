// The engine's loop guard and frame cap on the device (maya3/guards.py:49-106, maya3/engine.py:571-617).
//
// The reference evaluates them on the host after each tick's readout: per seat that delivered a frame it shifts the
// frame's cb0 code into a 96-code history, ends the seat at its frame cap, and every second frame from frame 32
// (outside text-derived suspend windows) runs loop_detect -- a 32-frame stall, or a period p in 2..16 with
// c[t] == c[t-p] on >= 70% of the last 64 frames -- whose hit sets an EOS boost on the seat's AEOS logit for the
// following ticks and, if the loop persists 24 frames past the boost, stops the seat.  Here one warp per seat does
// the same right after the cb0 sampler, inside the tick's stream: the history is a per-slot ring, the verdict and
// the boost count ride the stop code into the readout, and the boost lands in the sampler's aeos_bias before the
// next tick reads it.  Integer work on a few hundred bytes per seat: latency-bound, one launch per tick.
#include "common.cuh"

namespace m3 {

constexpr int kGuardHistMax = 128;
constexpr int kGuardWarps = 4;

__global__ void __launch_bounds__(kGuardWarps * 32)
guard_kernel(const m3_guard_config c, const m3_guard_state st, const int64_t* __restrict__ slots,
             int64_t* __restrict__ code, const int64_t* __restrict__ cb0, int seats) {
  __shared__ int win_s[kGuardWarps][kGuardHistMax];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x * kGuardWarps + w;
  if (i >= seats) return;  // warp-uniform
  const int64_t slot = slots[i];
  if (slot < 0 || slot >= c.max_slots) return;  // the padding slot carries no seat
  const int64_t stop = code[i];
  const int nb0 = st.n_boost[slot];
  if (stop != 0) {  // the sampler ended the seat: no frame, no guard (maya3/engine.py:576-578)
    if (lane == 0) code[i] = stop | ((int64_t)nb0 << 16);
    return;
  }
  const int H = c.hist;
  int* ring = st.hist + slot * H;
  const int f = st.frames[slot] + 1;  // this frame's number in the piece
  const int cur = (int)cb0[i];
  // the newest K codes, oldest first; frames before the first are -1 (the reference's empty history)
  const int K = max(c.stall, c.period_win);
  int* win = win_s[w];
  for (int j = lane; j < K; j += 32) {
    const int k = f - K + 1 + j;
    win[j] = k == f ? cur : (k >= 1 ? ring[(k - 1) % H] : -1);
  }
  __syncwarp();

  int verdict = M3_GUARD_NONE, boost_at = st.boost_at[slot], nb = nb0;
  bool set_bias = false, clear_bias = false;
  if (f >= st.cap[slot]) {
    verdict = M3_GUARD_CAP;  // maya3/engine.py:586-593
  } else if (c.loop && f >= c.start && f % c.every == 0) {
    bool inside = false;  // suspend windows (maya3/engine.py:594-596)
    const int nw = min(st.n_windows[slot], c.max_windows);
    for (int k = lane; k < nw; k += 32) {
      const int* ab = st.windows + ((int64_t)slot * c.max_windows + k) * 2;
      inside |= ab[0] <= f && f <= ab[1];
    }
    if (!__any_sync(0xffffffffu, inside)) {
      int kind = 0;  // loop_detect_batch (maya3/guards.py:80-106): stall first, then the smallest period
      if (f >= max(12, c.stall)) {
        const int* tail = win + (K - c.stall);
        bool eq = true;
        for (int j = lane; j < c.stall; j += 32) eq &= tail[j] == tail[0];
        if (__all_sync(0xffffffffu, eq)) {
          kind = M3_GUARD_STALL;
        } else if (f >= max(12, max(c.stall, c.period_win))) {
          const int* pw = win + (K - c.period_win);
          for (int p = c.pmin; p <= c.pmax && !kind; ++p) {
            const int pairs = c.period_win - p;
            int hits = 0;
            for (int j = lane; j < pairs; j += 32) hits += pw[j + p] == pw[j];
            hits = __reduce_add_sync(0xffffffffu, hits);
            if ((double)hits / (double)pairs >= c.period_thr) kind = M3_GUARD_PERIOD;
          }
        }
      }
      if (kind && c.mode == 0) {  // boost mode (maya3/engine.py:606-614)
        if (boost_at < 0) {
          boost_at = f;
          nb += 1;
          set_bias = true;
        }
        if (f - boost_at >= c.backstop) verdict = M3_GUARD_BACKSTOP;
      } else if (kind) {
        verdict = kind;  // stop mode: loop_stall / loop_period
      } else if (boost_at >= 0) {  // the loop cleared: the boost is removed (:615-617)
        boost_at = -1;
        clear_bias = true;
      }
    }
  }
  if (lane == 0) {
    ring[(f - 1) % H] = cur;
    st.frames[slot] = f;
    st.boost_at[slot] = boost_at;
    st.n_boost[slot] = nb;
    if (set_bias) st.aeos_bias[slot] = c.boost;
    if (clear_bias) st.aeos_bias[slot] = 0.f;
    code[i] = ((int64_t)verdict << 8) | ((int64_t)nb << 16);
  }
}

int guard_check(const m3_guard_config* c, const m3_guard_state* s) {
  M3_REQUIRE(c && s, M3_ERR_ARG, "guard: null config or state");
  M3_REQUIRE(c->hist >= 1 && c->hist <= kGuardHistMax && c->stall >= 1 && c->stall <= c->hist &&
                 c->period_win >= 1 && c->period_win <= c->hist,
             M3_ERR_ARG, "guard: hist %d stall %d period_win %d (need stall, period_win <= hist <= %d)", c->hist,
             c->stall, c->period_win, kGuardHistMax);
  M3_REQUIRE(c->pmin >= 1 && c->pmax < c->period_win && c->every >= 1 && (c->mode == 0 || c->mode == 1) &&
                 c->max_windows >= 0 && c->max_slots >= 1,
             M3_ERR_ARG, "guard: pmin %d pmax %d every %d mode %d max_windows %d max_slots %d", c->pmin, c->pmax,
             c->every, c->mode, c->max_windows, c->max_slots);
  M3_REQUIRE(s->frames && s->cap && s->boost_at && s->n_boost && s->hist && s->n_windows && s->aeos_bias &&
                 (s->windows || c->max_windows == 0),
             M3_ERR_ARG, "guard: null state array");
  return M3_OK;
}

}  // namespace m3

using namespace m3;

extern "C" int m3_guard_step(const m3_guard_config* cfg, const m3_guard_state* st, const int64_t* slots,
                             int64_t* code, const int64_t* cb0, int32_t seats, m3_stream stream) {
  M3_TRY(guard_check(cfg, st));
  M3_REQUIRE(slots && code && cb0 && seats >= 0, M3_ERR_ARG, "m3_guard_step: null argument or seats %d", seats);
  if (seats == 0) return M3_OK;
  guard_kernel<<<cdiv(seats, kGuardWarps), kGuardWarps * 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      *cfg, *st, slots, code, cb0, seats);
  M3_LAUNCHED();
  return M3_OK;
}
