// Fused SEANet decoder stages (the long, low-channel end of the Mimi decoder): one kernel per transposed conv and
// one per residual block, on the tensor cores, reading their activations by TMA.  See seanet.cu.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace m3 {

// ELU -> ConvTranspose1d(cin -> cout, kernel 2r, stride r) of one stage, written as a 2-tap causal conv over the
// stage input e = ELU(x) (bf16 [R][L][cin]): output row t (r * cout values = output steps t*r .. t*r + r-1) is
// sum_c e[t-1][c] W[c][:, r + jj] + e[t][c] W[c][:, jj] + bias.  Row t = L is the overlap tail kept for the next
// frame (serve/fast_codec.py:112-126).
struct ConvTFused {
  CUtensorMap amap;          // e as [R][L][cin], box {64 channels, 128 rows, 1}, 128-byte swizzle
  CUtensorMap bmap;          // wc as [r * cout][2 * cin], box {64, BN rows}, 128-byte swizzle
  CUtensorMap smap;          // u as [R][L][r * cout] for the persistent form's stores: box {32, 32, 1}, 64-byte swizzle
  const bf16* wc;            // [r * cout][2 * cin]: row jj*cout + o = [W[:, o, jj + r], W[:, o, jj]]
  const bf16* bias;          // [cout]
  const bf16* tail_in;       // previous frame's tails, [r * cout] per stream at stride in_row (state snapshot)
  int64_t in_row;
  bf16* state;               // slot state rows; the new tail goes to state[slot][tail_off ..]
  int64_t state_row, tail_off;
  const int* slot32;
  bf16* u;                   // output [R][L * r][cout] = [R][L][r * cout]
  int L, r, cin, cout;
};

// ELU -> conv k3 (cout -> hid, causal, 2 history rows) -> ELU -> conv k1 (hid -> cout) -> + u, then the next
// stage's ELU: e = ELU(u + conv(...)) (bf16 [R][Lo][cout]).  The new history (last 2 rows of ELU(u)) goes to the state.
struct ResFused {
  CUtensorMap umap;          // u as [R][Lo][cout], box {64 channels, 130 rows, 1}, 128-byte swizzle
  const bf16* w1;            // [hid][3 * cout] (tap-major, as the unfused path)
  const bf16* b1;            // [hid]
  const bf16* w2;            // [cout][hid]
  const bf16* b2;            // [cout]
  const bf16* hist_in;       // previous frame's ELU'd history rows, [2][cout] per stream at stride in_row
  int64_t in_row;
  bf16* state;
  int64_t state_row, hist_off;
  const int* slot32;
  bf16* e;                   // output [R][Lo][cout]
  int Lo, cout, hid;
};

// Final ELU -> conv (64 channels -> 1, 3 or 7 taps, causal) over the last stage's e = ELU(y) (bf16 [R][L][64]) ->
// fp32 PCM [R][L] = bf16(conv + bias) as the reference's bf16 model rounds it.
struct FinalFused {
  CUtensorMap xmap;          // e as [R][L][64], box {64 channels, 128 + taps - 1 rows, 1}, 128-byte swizzle
  const bf16* w;             // [taps * 64], tap-major
  const bf16* bias;          // [1]
  const bf16* state;         // the taps - 1 ELU'd history rows at state[slot][hist_off ..]
  int64_t state_row, hist_off;
  const int* slot32;
  float* pcm;
  int L, taps;
};
bool final_fused_ok(int channels, int taps);
int launch_final_fused(const FinalFused& p, int R, cudaStream_t s, int* status);

// Kernel shapes supported by the fused forms (other stages use the GEMM + elementwise path), and the transposed
// conv's output columns per CTA (its weight map's box height).
int convt_fused_bn(int N);
// The persistent form (weight slice of 128 columns resident, TMA-store epilogue): its weight box is 128 rows.
bool convt_persistent_ok(int cin, int cout, int r);
bool convt_fused_ok(int cin, int cout, int r);
bool res_fused_ok(int cout, int hid);
size_t convt_fused_smem(int cin, int cout, int r);
size_t res_fused_smem(int cout, int hid);
// Set the kernels' shared-memory limits (once per process and device).
int seanet_fused_init();

// sms: SMs the persistent forms spread over (0 or above the device's count: all of them).
int launch_convt_fused(const ConvTFused& p, int R, cudaStream_t s, int* status, int sms = 0);
// wc[jj*cout + o][k] = k < cin ? wt[(jj + r)*cout + o][k] : wt[jj*cout + o][k - cin], from the transposed conv's
// [2r * cout][cin] repack (element (j*cout + o, c) = W[c, o, j]).
int launch_convt_repack(const bf16* wt, int r, int cout, int cin, bf16* wc, cudaStream_t s);
int launch_res_fused(const ResFused& p, int R, cudaStream_t s, int* status, int sms = 0);

// Snapshot of the stateful rows the fused kernels read (so that they can write the new state in place):
// for each listed region, dst[b][0 .. len) = state[slot32[b]][off .. off + len).
struct StateCopy {
  int n;
  int64_t off[16];
  int len[16];
  int64_t dst_off[16];  // element offset of the region inside one row of the snapshot
};
int launch_state_snapshot(const bf16* state, int64_t state_row, const int* slot32, int R, const StateCopy& c,
                          bf16* snap, int64_t snap_row, cudaStream_t s);

}  // namespace m3
