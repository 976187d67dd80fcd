/* maya3_b200.h -- C ABI of the B200-native Maya3 decode tick.
 *
 * One shared library (libm3b200.so, sm_100a) exports the per-tick hot path of Maya3's streaming TTS engine: the
 * Qwen3 backbone decode over a static per-seat KV cache, the cb0 sampler with controlled stop, the depth
 * transformer's RVQ level loop with top-k sampling, and the one-frame Mimi decoder.  It replaces the reference's
 * serve-side components (serve/fast_backbone.py, serve/fast_depth.py, serve/fast_depth_kernels.py,
 * serve/fast_codec.py and Engine._cb0 in maya3/engine.py) behind the same seat interface.
 *
 * Conventions
 *   - Plain pointers and sizes only.  Every tensor argument is a DEVICE pointer unless marked "host".
 *   - Weights and per-seat state (KV caches, lengths, sampler state, codec state) are owned by the caller and must
 *     outlive the handle; a handle owns only its scratch memory, allocated once by *_create.
 *   - Every call that does device work takes a cudaStream_t (passed as void*) and only enqueues work: no host
 *     synchronisation and no allocation, so a step can be captured into a CUDA graph by the caller.
 *   - Functions return M3_OK (0) or a negative M3_ERR_*; m3_last_error() describes the last failure on the calling
 *     thread.  Problems seen inside kernels (slot or position out of range, a timed-out wait) are recorded in the
 *     handle's device status word and read back with *_status() after the caller's own synchronisation.
 *   - Row arrays (slots, offsets, real, codes) are int64, as the reference's torch.long tensors.
 *   - Slot `max_slots` is the padding ("dummy") slot, as in the reference: bucket padding rows point at it.
 */
#ifndef MAYA3_B200_H
#define MAYA3_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  M3_OK = 0,
  M3_ERR_ARG = -1,         /* bad argument: shape, size, pointer (reference raises ValueError) */
  M3_ERR_CUDA = -2,        /* a CUDA or cuBLAS call failed */
  M3_ERR_RANGE = -3,       /* slot / bucket out of range (reference raises IndexError / ValueError) */
  M3_ERR_UNSUPPORTED = -4  /* geometry this build does not implement */
};

enum { /* device status word values */
  M3_DEV_OK = 0,
  M3_DEV_BAD_SLOT = 1,     /* a row named a slot outside [0, max_slots]; it was redirected to the dummy slot */
  M3_DEV_BAD_POS = 2,      /* a position reached the KV capacity; the row was clamped */
  M3_DEV_BAD_CODE = 3,     /* a code outside [0, n_codes) reached an embedding table; it was clamped */
  M3_DEV_TIMEOUT = 4       /* a bounded wait inside a kernel gave up */
};

typedef void* m3_stream; /* cudaStream_t */

#if defined(__GNUC__)
#define M3_API __attribute__((visibility("default")))
#else
#define M3_API
#endif

M3_API const char* m3_last_error(void);
M3_API int m3_version(void);
/* Number of this library's kernel launches issued by this process so far (a launch captured into a CUDA graph
 * counts once at capture; the difference across a capture is the number of library kernels in the graph). */
M3_API int64_t m3_launch_count(void);
/* Failure-detection self-test: a kernel waits (at most `polls` polls, <= 2^20) on a barrier that never completes and
 * takes the bounded-wait exit every kernel of this library has; *status = the device status it recorded
 * (M3_DEV_TIMEOUT when the wait gave up).  Synchronises with the device; for tests. */
M3_API int m3_selftest_timeout(int32_t polls, int32_t* status);

/* ---------------------------------------------------------------------------------------------- utilities */
/* Y[M,N] = X[M,K] . W[N,K]^T, bf16 inputs, fp32 accumulation, Y bf16 (y_f32 = 0) or fp32 (y_f32 = 1).
 * Row-major with leading dimensions ldx, ldw, ldy (elements).  Replaces F.linear on the serving path
 * (serve/fast_backbone.py:193,200-202; serve/fast_depth.py:150,167,185-191; serve/fast_codec.py:140,168-181).
 * m <= 8 runs this library's GEMV kernel; larger m runs cuBLAS (cublasGemmEx, fp32 compute), as the reference's
 * F.linear does. */
M3_API int m3_gemm_bf16(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int32_t m,
                 int32_t n, int32_t k, int32_t y_f32, m3_stream stream);

/* In place f = bf16(GELU_erf(f)) over n8 groups of 8 bf16 values: the depth and Mimi feed-forward activation
 * (F.gelu on bf16 tensors) as the stages apply it.  For tests. */
M3_API int m3_gelu_bf16(void* f, int64_t n8, m3_stream stream);
/* m3_gemm_bf16 with a feed-forward activation in the GEMV kernel's epilogue (m <= 8, 16-byte aligned rows; other
 * shapes return M3_ERR_UNSUPPORTED): act 1, y = bf16(GELU_erf(bf16(x w^T))) over n columns; act 2, SwiGLU: w holds
 * n = 2F rows (gate rows, then up rows), y is [m, F] = bf16(bf16(silu(g)) * u) of the bf16 gate and up outputs
 * (serve/fast_backbone.py:200-202).  Same bits as the unfused layer followed by its activation pass.  The stages
 * fuse these themselves at small batch; this entry is for tests. */
M3_API int m3_gemm_bf16_act(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int32_t m,
                            int32_t n, int32_t k, int32_t act, m3_stream stream);

/* ---------------------------------------------------------------------------------------------- backbone */
/* Replaces StaticBackbone (serve/fast_backbone.py:111-362): the static-KV Qwen3 decode with per-seat positions. */
typedef struct m3_backbone m3_backbone;

typedef struct {
  int32_t layers, hidden, heads, kv_heads, head_dim, ffn;
  int32_t max_slots;  /* real seats; slot max_slots is the dummy */
  int32_t capacity;   /* KV positions per seat */
  int32_t max_rows;   /* largest row bucket a step may use (decode rows + inline prefill rows) */
  float eps;          /* RMSNorm epsilon */
} m3_backbone_config;

typedef struct {
  /* host arrays of `layers` device pointers; all tensors bf16 row-major */
  const void* const* in_norm;   /* [hidden]                                  input_layernorm.weight */
  const void* const* wqkv;      /* [(heads + 2 kv_heads) head_dim, hidden]   q|k|v proj rows (fast_backbone.py:135) */
  const void* const* q_norm;    /* [head_dim] */
  const void* const* k_norm;    /* [head_dim] */
  const void* const* wo;        /* [hidden, heads head_dim] */
  const void* const* post_norm; /* [hidden] */
  const void* const* wgu;       /* [2 ffn, hidden]  gate rows then up rows (fast_backbone.py:139) */
  const void* const* wdown;     /* [hidden, ffn] */
  const void* final_norm;       /* [hidden] */
  const void* cos;              /* [capacity, head_dim] RoPE tables in the model dtype (fast_backbone.py:152-153) */
  const void* sin;
  void* const* k_cache;         /* per layer [max_slots + 1, kv_heads, capacity, head_dim] (fast_backbone.py:146-148) */
  void* const* v_cache;
  int64_t* lengths;             /* [max_slots + 1] tokens held per slot (fast_backbone.py:149) */
} m3_backbone_weights;

M3_API int m3_backbone_create(const m3_backbone_config* cfg, const m3_backbone_weights* w, m3_backbone** out);
M3_API int m3_backbone_destroy(m3_backbone* bb);
/* One graphed step of StaticBackbone._forward (serve/fast_backbone.py:176-234) over `rows` rows.
 * slots [rows]: the slot of each row (inline-prefill rows repeat their slot, padding rows use the dummy);
 * offsets [rows] or NULL: position offset of each prefill row (0 for decode rows); real [rows] or NULL: 1 for
 * rows that advance their slot's length (NULL = all rows); x [rows, hidden] bf16 input; out [rows, hidden] bf16
 * final-normed hidden state.  ctx: context bucket, at least max(lengths[slot] + offset) + 1 over the rows.
 * Each row attends over keys 0..pos of its slot, pos = lengths[slot] + offset; every row's K/V is written before
 * any row attends, so prefill rows form an exact causal prefill (fast_backbone.py:326-333). */
M3_API int m3_backbone_step(m3_backbone* bb, const int64_t* slots, const int64_t* offsets, const int64_t* real,
                     const void* x, void* out, int32_t rows, int32_t ctx, m3_stream stream);
/* Read (and optionally clear) the device status word; synchronises with the device. */
M3_API int m3_backbone_status(m3_backbone* bb, int32_t* status, int32_t clear);
/* Voice prefix KV (maya3/engine.py:276-280, serve/fast_backbone.py:316-322): copy the first `length` positions of
 * every layer's K and V of `slot` to (save) or from (load) a packed store, bf16 [layers, 2 (K, V), kv_heads, length,
 * head_dim], 16-byte aligned.  Load also sets lengths[slot] = length (the host mirror is the caller's).  One launch
 * each, stream-ordered and capturable.  slot outside [0, max_slots) or length outside (0, capacity]: M3_ERR_RANGE. */
M3_API int m3_backbone_save_prefix(m3_backbone* bb, int32_t slot, void* store, int32_t length, m3_stream stream);
M3_API int m3_backbone_load_prefix(m3_backbone* bb, int32_t slot, const void* store, int32_t length,
                                   m3_stream stream);
/* Measurement hook: re-run layer `layer`'s decode attention (split-KV pass + combine) on the queries, slots and
 * positions the last m3_backbone_step left in the handle's scratch (rows and ctx as that step), to time the kernel
 * on the live cache (rows beyond any step's are rejected with M3_ERR_RANGE).  Overwrites only the handle's attention
 * output scratch. */
M3_API int m3_backbone_attention(m3_backbone* bb, int32_t layer, int32_t rows, int32_t ctx, m3_stream stream);
/* The attention of m3_backbone_attention with every K/V stage barrier expecting 16 bytes more than its copies bring
 * (rows <= 8), so that every wait in the launch runs out: a test of the kernel's bounded waits, which here give up
 * after 1000 polls each.  The launch ends by itself, its output rows are zero, M3_DEV_TIMEOUT is in the handle's
 * status (m3_backbone_status) and the context stays usable. */
M3_API int m3_backbone_attention_selftest(m3_backbone* bb, int32_t layer, int32_t rows, int32_t ctx, m3_stream stream);

/* ---------------------------------------------------------------------------------------------- cb0 sampler */
/* Replaces Engine._cb0 + Backbone.cb0_logits + row_exponential (maya3/engine.py:652-694,
 * tts/model/backbone.py:97, serve/fast_depth_kernels.py:339-355): per-seat temperature, top-k, top-p, presence
 * penalty, controlled stop and the per-request Philox stream. */
typedef struct m3_cb0 m3_cb0;

typedef struct {
  int32_t hidden;
  int32_t n_cls;      /* 2049 = 2048 codes + AEOS */
  int32_t max_slots;
  int32_t max_rows;
  int32_t rep_win;    /* presence-penalty window (frames of cb0 history) */
} m3_cb0_config;

typedef struct {         /* per-slot state tensors of maya3/engine.py:210-223, each [max_slots + 1] */
  const void* head;      /* bf16 [n_cls, hidden]  cb0_head.weight; copied at create (zero-padded to a multiple of 8
                          * rows for the head GEMM), so later writes to it are not seen by the handle */
  int64_t* frames;       /* frames generated by the seat */
  const int64_t* min_frames;
  float* hazard;
  const float* aeos_bias;
  const float* temp;
  const int64_t* top_k;
  const float* top_p;
  const float* rep;
  const int32_t* seed;
  int32_t* ctr;
  int64_t* hist;         /* [max_slots + 1, rep_win] last cb0 codes, -1 = empty */
} m3_cb0_state;

M3_API int m3_cb0_create(const m3_cb0_config* cfg, const m3_cb0_state* st, m3_cb0** out);
M3_API int m3_cb0_destroy(m3_cb0* s);
/* Read (and optionally clear) the handle's device status word (a row whose slot was outside [0, max_slots] was
 * sampled from the padding slot's state: M3_DEV_BAD_SLOT); synchronises with the device.  The reference raises
 * IndexError on the host for such a slot (maya3/engine.py:652-694 indexes its per-slot tensors with it). */
M3_API int m3_cb0_status(m3_cb0* s, int32_t* status, int32_t clear);
/* Inspection: the head output of the handle's last m3_cb0_step (the bf16 logits [rows, n_cls] its sampler read,
 * before temperature and bias) into dst (bf16 [rows, n_cls], dense), stream-ordered.  The reference's counterpart is
 * Backbone.cb0_logits(h) (tts/model/backbone.py:97), which Engine._cb0 calls first (maya3/engine.py:657). */
M3_API int m3_cb0_copy_logits(m3_cb0* s, void* dst, int32_t rows, m3_stream stream);
/* h [rows, hidden] bf16, idx [rows] slot per row -> stop code [rows] (0 or REASONS 2/3/4, maya3/engine.py:46) and
 * cb0 [rows] in [0, 2047]; advances the per-slot state.  apply_rep / apply_top_p mirror the engine's host flags
 * (`cb0_rep_win > 0 and (cb0_rep > 0 or any_rep)`, `_any_top_p`). */
M3_API int m3_cb0_step(m3_cb0* s, const void* h, const int64_t* idx, int64_t* code, int64_t* cb0, int32_t rows,
                int32_t apply_rep, int32_t apply_top_p, m3_stream stream);
/* m3_cb0_step without a handle and without allocating, for callers that must not allocate device memory while
 * they sample: a host that gave this library a fixed device budget up front and forbids any later cudaMalloc, or a
 * latency-critical serving thread on which cudaMalloc / cudaFree would synchronise the device and stall every seat.
 * This entry point has no counterpart in the reference (which samples with eager torch ops that allocate freely).
 * Same arguments and results as m3_cb0_step, with the configuration and per-slot state passed directly; limits:
 * rows <= 8 per call, n_cls <= 4096, hidden <= 3072 (a multiple of 8), h and st->head on 16-byte boundaries; other
 * calls are rejected with M3_ERR_ARG before any device work.
 * Scratch: a 64 KiB static device array inside the library, held by every GPU that loads it until the process
 * exits.  The first call on a device looks up that array's device address, so make it before any stream capture.
 * Every call shares the one array: calls that overlap on the GPU (different streams without ordering) race.
 * Problems seen inside the kernel (a slot outside [0, max_slots], sampled from the padding slot's state) go to a
 * status word in the same array: zero when the library loads, it keeps the first problem of any call until
 * m3_cb0_noalloc_status clears it. */
M3_API int m3_cb0_step_noalloc(const m3_cb0_config* cfg, const m3_cb0_state* st, const void* h, const int64_t* idx,
                               int64_t* code, int64_t* cb0, int32_t rows, int32_t apply_rep, int32_t apply_top_p,
                               m3_stream stream);
/* Read (and optionally clear) the status word of m3_cb0_step_noalloc on the current device; synchronises with the
 * device and allocates nothing. */
M3_API int m3_cb0_noalloc_status(int32_t* status, int32_t clear);
/* The sampler alone on given fp32 logits [rows, n_cls] (the cb0 head output as fp32). */
M3_API int m3_cb0_sample_logits(m3_cb0* s, const float* logits, const int64_t* idx, int64_t* code, int64_t* cb0,
                         int32_t rows, int32_t apply_rep, int32_t apply_top_p, m3_stream stream);

/* ---------------------------------------------------------------------------------------------- depth */
/* Replaces FastDepth (serve/fast_depth.py:32-257) with its fused kernels (serve/fast_depth_kernels.py). */
typedef struct m3_depth m3_depth;

typedef struct {
  int32_t layers, d, heads, ffn;
  int32_t n_q;            /* codebooks per frame: cb0 + n_q - 1 depth levels */
  int32_t n_codes;
  int32_t d_backbone;
  int32_t n_groups;
  int32_t group_of_level[64];  /* level -> weight group; entry 0 unused (tts/model/depth_v2.py:45) */
  int32_t max_slots, max_rows;
  float ln_eps;
  float inv_temp;         /* 1 / sampler temperature, computed in double and rounded once (Triton's fp32 argument) */
  int32_t top_k;
  int32_t greedy;         /* argmax instead of sampling */
} m3_depth_config;

typedef struct {
  const void* in_proj;    /* [d, d_backbone] */
  const void* embed;      /* [n_q - 1, n_codes, d] prefix table code_up(code_lo) + level_emb[1:] (fast_depth.py:49-50) */
  const void* level0;     /* [d] level_emb[0] */
  /* host arrays of n_groups * layers device pointers, index group * layers + layer */
  const void* const* n1_w; const void* const* n1_b;
  const void* const* n2_w; const void* const* n2_b;
  const void* const* qkv;  /* [3d, d] */
  const void* const* o;    /* [d, d] */
  const void* const* f1;   /* [ffn, d] */
  const void* const* f2;   /* [d, ffn] */
  const void* norm_w; const void* norm_b;
  const void* const* heads;   /* host array of n_q - 1 pointers, each [n_codes, d] */
  const void* const* cross_kv; /* host array of `layers` pointers, each [2d, d] (speaker cross-attn kv) */
  const void* const* cross_o;  /* host array of `layers` pointers, each [d, d] */
  const void* audio_table;     /* [n_q n_codes, d_backbone] AudioInputEmbed.table */
  const void* audio_norm;      /* [d_backbone] AudioInputEmbed.norm.weight */
  void* cross_const;           /* [max_slots + 1, layers, d] per-slot speaker constants (fast_depth.py:56) */
  int32_t* row_seed;           /* [max_slots + 1] per-slot Philox seed (fast_depth.py:66) */
  int32_t* row_ctr;            /* [max_slots + 1] per-slot frame counter */
} m3_depth_weights;

M3_API int m3_depth_create(const m3_depth_config* cfg, const m3_depth_weights* w, m3_depth** out);
M3_API int m3_depth_destroy(m3_depth* d);
/* FastDepth.set_speaker (serve/fast_depth.py:72-82): mem [d] bf16, keep = the reference mask (0 or 1). */
M3_API int m3_depth_set_speaker(m3_depth* d, int32_t slot, const void* mem, float keep, m3_stream stream);
/* FastDepth.__call__ (serve/fast_depth.py:241-257): h [rows, d_backbone] bf16, cb0 [rows] -> codes [rows, n_q]
 * int64 and feedback [rows, d_backbone] bf16 (the next backbone input); advances row_ctr of each row's slot. */
M3_API int m3_depth_step(m3_depth* d, const int64_t* slots, const void* h, const int64_t* cb0, int64_t* codes,
                  void* feedback, int32_t rows, m3_stream stream);
/* The level sampler alone (serve/fast_depth_kernels.py:305-336): logits [rows, n] (bf16 if logits_bf16 else
 * fp32), per-row seed/counter -> codes [rows].  inv_temp = 1 / temperature. */
M3_API int m3_topk_sample(const void* logits, int32_t logits_bf16, int32_t rows, int32_t n, const int32_t* seed,
                   const int32_t* ctr, int32_t level, float inv_temp, int32_t top_k, int32_t greedy, int64_t* codes,
                   m3_stream stream);
M3_API int m3_depth_status(m3_depth* d, int32_t* status, int32_t clear);
/* Inspection: with buf set (bf16 [n_q - 1][max_rows][n_codes], 16-byte aligned), every later m3_depth_step (and every
 * step captured into a graph after this call) writes level l's head logits to buf[l - 1] instead of its scratch, so
 * they can be compared with the reference's d.heads[level - 1](y) (serve/fast_depth.py:190-191); NULL restores the
 * scratch.  bytes < the size above -> M3_ERR_ARG. */
M3_API int m3_depth_debug_logits(m3_depth* d, void* buf, int64_t bytes);

/* ---------------------------------------------------------------------------------------------- mimi */
/* Replaces StaticMimi (serve/fast_codec.py:32-277): one 80 ms frame per seat with per-slot streaming state. */
typedef struct m3_mimi m3_mimi;

typedef struct {
  int32_t hidden, n_q, n_semantic, codebook_size, codebook_dim;
  int32_t layers, heads, ffn, window, ring;
  int32_t n_ratios, ratios[8];
  int32_t num_filters, kernel, last_kernel, res_kernel, compress, upsample_stride;
  int32_t max_slots, max_rows;
  float norm_eps;
} m3_mimi_config;

typedef struct {
  const void* codebooks;     /* [n_q, codebook_size, codebook_dim] decoded embeddings (embed_sum / usage) */
  const void* proj_sem;      /* [hidden, codebook_dim] semantic output_proj */
  const void* proj_ac;       /* [hidden, codebook_dim] acoustic output_proj */
  const void* upsample;      /* [hidden, 2 upsample_stride] depthwise ConvTranspose1d weight */
  /* transformer, host arrays of `layers` pointers */
  const void* const* ln1_w; const void* const* ln1_b;
  const void* const* wqkv;   /* [3 hidden, hidden] q|k|v proj rows */
  const void* const* wo;     /* [hidden, hidden] */
  const void* const* ln2_w; const void* const* ln2_b;
  const void* const* fc1;    /* [ffn, hidden] */
  const void* const* fc2;    /* [hidden, ffn] */
  const void* const* ls1;    /* [hidden] self_attn_layer_scale */
  const void* const* ls2;    /* [hidden] mlp_layer_scale */
  const float* inv_freq;     /* [head_dim / 2] fp32 RoPE frequencies, as the model holds them */
  /* SEANet decoder, host arrays; conv weights repacked tap-major: [c_out, k * c_in] with element (o, j c_in + i) =
   * W[o, i, j]; transposed-conv weights [2r c_out, c_in] with element (j c_out + o, i) = W[i, o, j] */
  const void* conv0_w; const void* conv0_b;
  const void* const* convt_w; const void* const* convt_b;     /* n_ratios */
  const void* const* res1_w; const void* const* res1_b;       /* n_ratios: k res_kernel, c -> c / compress */
  const void* const* res2_w; const void* const* res2_b;       /* n_ratios: k 1, c / compress -> c */
  const void* final_w; const void* final_b;                   /* [1, last_kernel num_filters] */
  /* per-slot state, caller-owned (rows = max_slots + 1) */
  void* conv_state;          /* bf16 [rows, m3_mimi_state_elems()] histories and overlap tails, channels-last */
  void* kv;                  /* bf16 [layers, 2, rows, heads, ring, head_dim] keys post-RoPE (fast_codec.py:68) */
  int64_t* key_pos;          /* [rows, ring] absolute key positions, empty = -(1 << 40) */
  int64_t* tokens;           /* [rows] transformer tokens consumed */
} m3_mimi_weights;

/* Elements of one slot's conv_state row for a geometry. */
M3_API int64_t m3_mimi_state_elems(const m3_mimi_config* cfg);
M3_API int m3_mimi_create(const m3_mimi_config* cfg, const m3_mimi_weights* w, m3_mimi** out);
M3_API int m3_mimi_destroy(m3_mimi* m);
/* StaticMimi.reset (serve/fast_codec.py:236-244). */
M3_API int m3_mimi_reset(m3_mimi* m, int32_t slot, int32_t zero_kv, m3_stream stream);
/* StaticMimi.decode (serve/fast_codec.py:246-277): codes [rows, n_q] -> pcm [rows, samples_per_frame] fp32. */
M3_API int m3_mimi_decode(m3_mimi* m, const int64_t* slots, const int64_t* codes, float* pcm, int32_t rows,
                   m3_stream stream);
M3_API int m3_mimi_status(m3_mimi* m, int32_t* status, int32_t clear);
/* How many SMs the handle's persistent SEANet kernels (transposed convs and residual blocks of the fused stages)
 * spread their CTAs over; 0 (the default) or more than the device has: all.  A decoder that runs on a second
 * stream beside other work (the engine's codec part beside the next tick's main part) leaves the other stream
 * room this way: its kernels otherwise take every SM for their duration.  Results do not depend on it.  Takes
 * effect at the next decode; a CUDA graph keeps the grid it was captured with. */
M3_API int m3_mimi_set_sm_budget(m3_mimi* m, int32_t sms);
/* Measurement hook: re-run decoder stage `stage`'s fused transposed conv (a stage of the fused SEANet suffix) over
 * `rows` streams on the activation buffers the last decode left, writing the overlap tails to a scratch row instead
 * of the streams' state; *bytes = its algorithmic bytes (bf16 stage input read + stage output written). */
M3_API int m3_mimi_convt(m3_mimi* m, int32_t stage, int32_t rows, int64_t* bytes, m3_stream stream);

/* ---------------------------------------------------------------------------------------------- tick */
/* The device half of one engine tick (maya3/engine.py:534-561, Engine._tick from the backbone step through the
 * packed readout) as one call over the four stage handles. */
typedef struct m3_tick m3_tick;

typedef struct {
  m3_backbone* bb;
  m3_cb0* cb0;
  m3_depth* depth;
  m3_mimi* mimi;
  const void* embed;   /* [vocab, hidden] bf16 token embeddings read by inline-prefill rows (may be NULL) */
  int64_t vocab;
  void* feedback;      /* [max_slots + 1, hidden] bf16 per-slot next backbone input (maya3/engine.py:211) */
  int32_t hidden, max_rows, max_seats, n_q, spf, max_slots;
} m3_tick_config;

M3_API int m3_tick_create(const m3_tick_config* cfg, m3_tick** out);
M3_API int m3_tick_destroy(m3_tick* t);
/* plan: device int64 [4 rows + 2 seats]: per backbone row (slot, offset, real, source) then per seat (slot, row of
 * the backbone output holding its hidden state).  A row's source is -2 for a decode row (input = feedback[slot]),
 * a prompt token id for an inline-prefill row (input = embed[token]) or -1 for a padding row (zeros).  Runs the
 * backbone over `rows` rows, then cb0, depth, the feedback write-back, Mimi and the readout over `seats` seats;
 * packed receives [seats, 2 + spf / 4] int64 (stop code, cb0, int16 PCM). */
M3_API int m3_tick_run(m3_tick* t, const int64_t* plan, int32_t rows, int32_t seats, int32_t ctx, int32_t apply_rep,
                       int32_t apply_top_p, int64_t* packed, m3_stream stream);
/* m3_tick_run in three parts, so that the codec part of one tick can run on a second stream beside the next tick's
 * main part.  run_main: the backbone through the feedback write-back (the next tick's input); stage_codec: copies
 * this tick's stop codes, cb0, codes and seat slots (plan as for run_main) into codec input set `set` (0 or 1);
 * run_codec: the Mimi frame and the packed readout from set `set`.  The caller orders them: stage_codec after
 * run_main on its stream; run_codec after stage_codec; stage_codec into a set only after the run_codec that last
 * read it; Mimi slot resets (m3_mimi_reset) on the codec part's stream.  The codec part's library GEMMs use the
 * Mimi handle's own workspace.  m3_tick_run = run_main, stage_codec(set 0), run_codec(set 0) on one stream. */
M3_API int m3_tick_run_main(m3_tick* t, const int64_t* plan, int32_t rows, int32_t seats, int32_t ctx,
                            int32_t apply_rep, int32_t apply_top_p, m3_stream stream);
M3_API int m3_tick_stage_codec(m3_tick* t, const int64_t* plan, int32_t rows, int32_t seats, int32_t set,
                               m3_stream stream);
M3_API int m3_tick_run_codec(m3_tick* t, int32_t seats, int32_t set, int64_t* packed, m3_stream stream);
/* Device pointers of the last tick's per-seat hidden states [max_seats, hidden] bf16, codes [max_seats, n_q] and
 * fp32 PCM [max_seats, spf] (any may be NULL). */
M3_API int m3_tick_outputs(m3_tick* t, void** h, int64_t** codes, float** pcm);
/* First non-zero device status word over the tick and its stage handles; synchronises. */
M3_API int m3_tick_status(m3_tick* t, int32_t* status, int32_t clear);

/* ---------------------------------------------------------------------------------------------- guards */
/* The engine's loop guard and frame cap (GuardConfig, maya3/guards.py:49-75; loop_detect_batch, :80-106; the
 * per-seat update after the readout, maya3/engine.py:571-617), run on the device right after the cb0 sampler
 * instead of on the host after the tick's sync.  The text-derived parts (the duration prior behind a seat's cap,
 * the suspend windows of suspend_windows_v2, :128-146) stay on the host and arrive per slot at bind time. */
typedef struct {
  int32_t loop;          /* GuardConfig.enabled && GuardConfig.loop: evaluate the loop rule (the cap always applies) */
  int32_t stall;         /* 32: a stall is the last `stall` codes all equal to the first of them */
  int32_t period_win;    /* 64: window of the period rule */
  double period_thr;     /* 0.7: mean of c[t] == c[t-p] over the window at or above which p is a period */
  int32_t pmin, pmax;    /* 2, 16: periods tried, smallest first; pmax < period_win */
  int32_t start, every;  /* 32, 2: the rule runs on frames f >= start with f % every == 0 */
  int32_t mode;          /* 0 = boost (EOS boost, then backstop), 1 = stop at the first loop */
  float boost;           /* 4.0: AEOS bias while the loop persists */
  int32_t backstop;      /* 24: frames after the boost began at which a persisting loop stops the seat */
  int32_t hist;          /* 96: cb0 codes kept per slot; stall, period_win <= hist <= 128 */
  int32_t max_windows;   /* suspend windows per slot */
  int32_t max_slots;
} m3_guard_config;

typedef struct {         /* per-slot state, each [max_slots + 1] unless stated (row max_slots = padding slot) */
  int32_t* frames;       /* frames delivered in the seat's current piece (_Seat.frames) */
  const int32_t* cap;    /* the piece's frame cap (_Seat.cap) */
  int32_t* boost_at;     /* frame at which the current EOS boost began, -1 = none (_Seat.boost_at) */
  int32_t* n_boost;      /* boosts so far in the piece (_Seat.n_boost) */
  int32_t* hist;         /* [max_slots + 1, hist] cb0 ring: the code of frame f at (f - 1) % hist (_Seat.hist) */
  const int32_t* n_windows;  /* suspend windows in use per slot */
  const int32_t* windows;    /* [max_slots + 1, max_windows, 2] inclusive frame windows (a, b) with no loop action */
  float* aeos_bias;      /* the cb0 sampler's per-slot AEOS bias (m3_cb0_state.aeos_bias, maya3/engine.py:215) */
} m3_guard_state;

/* Guard verdicts: the seat's frame is delivered, then the seat finishes (maya3/engine.py:586-614). */
enum { M3_GUARD_NONE = 0, M3_GUARD_CAP = 1, M3_GUARD_BACKSTOP = 2, M3_GUARD_STALL = 3, M3_GUARD_PERIOD = 4 };

/* One guard update per seat: for a seat whose sampler stop code is 0 (it delivers a frame) the slot's frame count
 * and cb0 ring advance, the cap is checked, and on due frames outside the suspend windows the loop rule runs and the
 * EOS boost is set or cleared in aeos_bias (seen by the next tick's sampler, as the reference's host write is).
 * code: in, the sampler's stop codes [seats]; out, stop | verdict << 8 | n_boost << 16.  Seats on the padding slot
 * are skipped.  Returns M3_ERR_ARG for a configuration outside the limits above. */
M3_API int m3_guard_step(const m3_guard_config* cfg, const m3_guard_state* st, const int64_t* slots, int64_t* code,
                         const int64_t* cb0, int32_t seats, m3_stream stream);
/* Attach guards to a tick (copied; NULL cfg detaches): m3_tick_run then runs m3_guard_step after the cb0 sampler and
 * the readout's stop column carries the packed verdicts.  Call before capturing the tick into a graph. */
M3_API int m3_tick_set_guard(m3_tick* t, const m3_guard_config* cfg, const m3_guard_state* st);

/* ---------------------------------------------------------------------------------------------- slot reset */
/* The device half of binding a request to a slot (maya3/engine.py:420-447, Engine._bind) as one launch: the cb0
 * sampler's per-slot state (frames, minimum frames, hazard, AEOS bias, seed, counter, repetition history set to -1,
 * temperature, top-k, top-p, repetition penalty), the depth sampler's stream seed and counter, the slot's depth
 * speaker constant (copied from cross_src) and its backbone length.  The state pointers are the per-slot tensors the
 * sampler, depth and backbone objects were created with ([max_slots + 1] rows each; hist [max_slots + 1, hist_len],
 * cross_const [max_slots + 1, cross_elems] bf16 with cross_elems a multiple of 8).  The Mimi state has its own reset
 * (m3_mimi_reset). */
typedef struct {
  int64_t *frames, *min_frames;
  float *hazard, *aeos_bias;
  int32_t *seed, *ctr;
  int64_t* hist;
  int32_t hist_len;
  float* temp;
  int64_t* top_k;
  float *top_p, *rep;
  int32_t *row_seed, *row_ctr;
  void* cross_const;
  int32_t cross_elems;
  int64_t* lengths;
  int32_t max_slots;
} m3_slot_state;

typedef struct {
  int32_t slot, seed, row_seed, min_frames;
  int64_t top_k, length;
  float temp, top_p, rep;
  const void* cross_src; /* [cross_elems] bf16 */
} m3_slot_init;

/* slot must lie in [0, max_slots) (the padding slot is never bound); cross_src and cross_const 16-byte aligned. */
M3_API int m3_slot_reset(const m3_slot_state* st, const m3_slot_init* init, m3_stream stream);

/* ---------------------------------------------------------------------------------------------- readout */
/* The engine's per-tick readout (maya3/engine.py:557-561): packed [rows, 2 + spf / 4] int64 rows holding
 * (stop code, cb0, PCM as int16 = round(clamp(pcm, -1, 1) * 32767)). */
M3_API int m3_pack_readout(const int64_t* code, const int64_t* cb0, const float* pcm, int64_t* packed, int32_t rows,
                    int32_t spf, m3_stream stream);

#ifdef __cplusplus
}
#endif
#endif /* MAYA3_B200_H */
