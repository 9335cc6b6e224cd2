/*
 * tabnet_stage.h -- C ABI of the B200 stage engine (libtabnet_stage.so).
 *
 * The engine replaces the stage engine of ce-tabnet, web/inference-worker.js,
 * behind the same three-call contract (web/inference-worker.js:13-19,
 * web/inference.js:9-15):
 *
 *   initStage(spec) -> ctx        tn_stage_init
 *   forward(ctx, req) -> out      tn_stage_forward / tn_stage_forward_batch
 *   freeStage(ctx)                tn_stage_free
 *
 * Plain C types only (no torch, no C++), so a Node-API addon, ctypes, cgo or
 * JNI binding can call it directly.  All calls return 0 or a negative TN_E*
 * status and never abort; tn_last_error() gives the calling thread's message.
 * Calls on one tn_stage are serialised by an internal mutex; stages on
 * different devices may run concurrently from different threads.
 */
#ifndef TABNET_STAGE_H
#define TABNET_STAGE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TN_ABI_VERSION 2

/* ---- status codes ---- */
#define TN_OK 0
#define TN_EINVAL (-1)       /* bad argument (sizes, ids, null pointers) */
#define TN_ENOMEM (-2)       /* host or device allocation failed */
#define TN_ECUDA (-3)        /* a CUDA runtime call failed */
#define TN_EUNSUPPORTED (-4) /* "unsupported quant" (web/inference-worker.js:126,136) */
#define TN_ECAPACITY (-5)    /* max_ctx / max_seqs / max_tokens_per_step / KV pages exceeded */
#define TN_ESTATE (-6)       /* wrong stage role for the call (e.g. ids to a non-first stage) */
#define TN_ETIMEOUT (-7)     /* a bounded device wait ran out */

/* ---- weight formats (web/inference-worker.js:92-137) ---- */
typedef enum {
  TN_QUANT_F32 = 0,
  TN_QUANT_F16 = 1,
  TN_QUANT_Q4_0 = 2, /* 18-byte blocks: f16 d, 16 bytes; byte j = elem 2j (lo), 2j+1 (hi); w=(nib-8)*d */
  TN_QUANT_Q8_0 = 3  /* 34-byte blocks: f16 d, 32 x int8; w = q*d */
} tn_quant;

/* what a non-last stage returns (the reference returns the last position only) */
enum { TN_HOP_LAST = 0, TN_HOP_ALL = 1 };

/* spec flags */
#define TN_FLAG_NO_GRAPHS (1u << 0) /* never capture decode steps in CUDA graphs */
#define TN_FLAG_PROFILE (1u << 1)   /* time every kernel launch with CUDA events (tn_stage_profile) */
#define TN_FLAG_NO_FUSED_DECODE (1u << 2) /* decode steps use the separate norm / matvec / RoPE kernels */
#define TN_FLAG_KV_F16 (1u << 3)          /* KV cache of fp16 rows (half the bytes; the reference keeps f32) */
#define TN_FLAG_KV_F8 (1u << 4)           /* KV cache of fp8 e4m3 rows (a quarter; saturates at +-448, no scale) */

/* One layer's packed buffer, tensors in web/inference-worker.js:142-159 order:
 * attn_norm(f16) wq wk wv wo ffn_norm(f16) w_gate w_up w_down. */
typedef struct {
  int32_t idx;      /* absolute layer index */
  int32_t quant;    /* tn_quant of the matrices */
  const void* buf;  /* packed bytes (host, or device if weights_on_device) */
  uint64_t len;
} tn_layer_weights;

/* initStage({arch, dims, layers:[lo,hi), is_first, is_last, weights, opts}) */
typedef struct {
  uint32_t abi_version; /* TN_ABI_VERSION */
  /* dims (web/inference-worker.js:426-429) */
  int32_t hidden_dim, n_heads, n_kv_heads, vocab;
  int32_t ffn_dim;      /* 0 -> roundFfn(hidden_dim) (web/inference-worker.js:160-163) */
  double rope_theta;
  /* stage slice */
  int32_t layer_lo, layer_hi, is_first, is_last;
  /* weights (web/shard-loader.js:16-22 `weights` object) */
  const tn_layer_weights* layers;
  int32_t n_layers;     /* == layer_hi - layer_lo */
  const void* embed;   uint64_t embed_len;   int32_t embed_quant;   /* first stage */
  const void* norm;    uint64_t norm_len;                          /* last stage, f16 [H] */
  const void* lm_head; uint64_t lm_head_len; int32_t lm_head_quant; /* last stage */
  int32_t weights_on_device; /* 1: every weight pointer above is device memory of `device` */
  /* runtime options (web/inference-worker.js:642 opts.max_ctx) */
  int32_t device;
  int32_t max_ctx;             /* KV rows per sequence; 0 -> 4096 */
  int32_t max_seqs;            /* concurrent sequences with KV; 0 -> 16 */
  int32_t max_tokens_per_step; /* rows fused into one step; 0 -> 512 (longer prompts are chunked) */
  uint32_t flags;
  /* Paged KV (not in the reference, whose KV is one growing array per
   * sequence): 0 keeps max_ctx contiguous rows per sequence slot; else the
   * rows live in a pool of kv_pages pages of kv_page_tokens positions (a power
   * of two in [16, 4096]), a sequence taking pages as it grows and returning
   * them when freed.  max_ctx still bounds one sequence and max_seqs the
   * sequences; kv_pages 0 -> max_seqs * ceil(max_ctx / kv_page_tokens). */
  int32_t kv_page_tokens;
  int32_t kv_pages;
} tn_stage_spec;

typedef struct tn_stage tn_stage;

/* forward(ctx, {seq_id, token_pos, hidden?, token_ids?, temperature?, top_p?}) */
typedef struct {
  uint64_t seq_id;            /* the JS string seq_id mapped to an integer by the binding */
  int32_t token_pos;          /* RoPE position of the first token in this request */
  int32_t n_tokens;           /* positions in this request (>= 1) */
  const int32_t* token_ids;   /* first stage: [n_tokens] */
  const uint16_t* hidden;     /* other stages: [n_tokens * hidden_dim] fp16 bits */
  double temperature;         /* last stage; <= 0 is greedy (web/inference-worker.js:660) */
  double top_p;               /* last stage */
  uint64_t rng_seed;          /* last stage, temperature > 0: seeds the uniform draw */
  int32_t hop_mode;           /* TN_HOP_LAST (reference behaviour) or TN_HOP_ALL */
} tn_fwd_req;

typedef struct {
  uint16_t* hidden;           /* caller-owned, capacity hidden_cap_tokens * hidden_dim */
  int32_t hidden_cap_tokens;
  int32_t n_hidden_tokens;    /* written: positions returned (1 for TN_HOP_LAST) */
  int32_t token_id;           /* written on the last stage */
} tn_fwd_out;

/* web/inference-worker.js:417 initStage.  Copies and repacks every weight;
 * the caller may free its buffers when this returns. */
int tn_stage_init(const tn_stage_spec* spec, tn_stage** out);

/* web/inference-worker.js:471 forward (and :690 forwardSafe for the last
 * stage).  Host buffers in, host buffers out; synchronous. */
int tn_stage_forward(tn_stage* st, const tn_fwd_req* req, tn_fwd_out* out);

/* Several sequences fused into one step (micro-batching; the reference runs
 * them as independent forward calls).  reqs[i] and outs[i] as above. */
int tn_stage_forward_batch(tn_stage* st, const tn_fwd_req* reqs, int32_t n_reqs, tn_fwd_out* outs);

/* Release one sequence's KV slot and, with a paged cache, its pages (no
 * reference counterpart: the reference keeps every sequence's KV until
 * freeStage, web/inference-worker.js:677-684).  Steps of that sequence
 * enqueued with tn_stage_step_async must have finished: the slot and its
 * pages may be handed to the next sequence at once. */
int tn_stage_free_seq(tn_stage* st, uint64_t seq_id);

/* KV rows currently cached for seq_id (0 if unknown). */
int32_t tn_stage_kv_len(tn_stage* st, uint64_t seq_id);

/* web/inference-worker.js:677 freeStage. */
void tn_stage_free(tn_stage* st);

/* Message for the last failing call on this thread ("" if none). */
const char* tn_last_error(void);

/* ---- device-resident decode step (pipeline runner, benchmarks) ----
 * One token per sequence; inputs and outputs are device pointers on the
 * stage's device.  Enqueued on `stream` (NULL: the stage's own stream) and
 * returns without waiting; KV bookkeeping is advanced at enqueue time. */
typedef struct {
  int32_t n_seqs;
  const uint64_t* seq_ids;     /* host [n_seqs] */
  const int32_t* token_pos;    /* host [n_seqs] */
  const int32_t* d_token_ids;  /* first stage: device [n_seqs] */
  const uint16_t* d_hidden_in; /* other stages: device [n_seqs * H] fp16 bits */
  uint16_t* d_hidden_out;      /* non-last stage: device [n_seqs * H] */
  int32_t* d_token_out;        /* last stage: device [n_seqs] */
  double temperature, top_p;
  uint64_t rng_seed;
} tn_step_desc;
int tn_stage_step_async(tn_stage* st, const tn_step_desc* step, void* stream);
/* Waits for the stage's work on `stream` (NULL: the stage stream) and reports
 * what tn_stage_step_async cannot: TN_ETIMEOUT if a kernel's bounded wait on
 * its copy pipeline gave up since the last check or forward call (the outputs
 * of the steps since then are invalid; the stage's split-K counters are reset
 * so later steps run clean), else TN_OK.  The synchronous forward calls do this
 * check themselves.  No counterpart in the reference, whose steps are
 * synchronous. */
int tn_stage_check(tn_stage* st, void* stream);
/* Test hook: marks the stage as if a kernel's bounded wait had given up (the
 * next tn_stage_check or forward returns TN_ETIMEOUT and recovers).  Failure
 * handling is tested this way and with tn_test_bounded_wait, without faulting
 * a GPU. */
int tn_stage_test_raise_kernel_error(tn_stage* st);
/* the stage's own stream (cudaStream_t) */
void* tn_stage_stream(tn_stage* st);

typedef struct {
  uint64_t weight_bytes;   /* device bytes held by repacked weights */
  uint64_t kv_bytes;       /* device bytes of the KV arena */
  uint64_t scratch_bytes;  /* device bytes of activations and partials */
  uint64_t packed_bytes;   /* packed (reference-format) bytes the weights came from */
  int32_t n_layers, head_dim, q_dim, kv_dim, ffn_dim;
  int32_t graphs_captured; /* decode-step CUDA graphs instantiated so far */
  int32_t launches_last_step; /* kernels the last step launched */
} tn_stage_info;
int tn_stage_get_info(tn_stage* st, tn_stage_info* info);

/* Per-kernel device time of the synchronous forward calls since the last
 * reset, for stages created with TN_FLAG_PROFILE: ms[k] and launches[k] for
 * each class k below (arrays of TN_PROF_N). */
enum {
  TN_PROF_MATVEC_QKV = 0, TN_PROF_MATVEC_O, TN_PROF_MATVEC_GATE_UP, TN_PROF_MATVEC_DOWN,
  TN_PROF_MATVEC_LM_HEAD, TN_PROF_ATTENTION, TN_PROF_NORM, TN_PROF_ROPE_KV, TN_PROF_OTHER, TN_PROF_N
};
int tn_stage_profile(tn_stage* st, double* ms, uint64_t* launches, int32_t reset);
/* Turn per-launch timing on or off after init (drops captured graphs, which
 * are re-captured with or without the timing events). */
int tn_stage_set_profile(tn_stage* st, int32_t on);

/* Test hook: copy device state left by the last forward/step call into host
 * memory (synchronises the stage's stream).  what = TN_PEEK_HIDDEN: the f32
 * hidden rows of that step, [rows][hidden_dim]; TN_PEEK_LOGITS (last stage):
 * the f32 logits of its output rows, [n_out][vocab].  Copies min(bytes, size). */
enum { TN_PEEK_HIDDEN = 0, TN_PEEK_LOGITS = 1 };
int tn_stage_peek(tn_stage* st, int32_t what, void* host_out, uint64_t bytes);

/* ---- single-op entry points (tests, microbenchmarks) ---- */

/* A quantised [rows x cols] matrix, repacked on the device from packed bytes
 * laid out as by dequantToF32 (web/inference-worker.js:102-129). */
typedef struct tn_matrix tn_matrix;
int tn_matrix_create(int32_t device, int32_t quant, int32_t rows, int32_t cols, const void* packed,
                     uint64_t len, int32_t on_device, tn_matrix** out);
/* y[t][r] = sum_c W[r][c] * x[t][c] for t < n_tokens (web/inference-worker.js:523-527);
 * device pointers, f32. */
int tn_matrix_matvec(const tn_matrix* m, int32_t n_tokens, const float* d_x, float* d_y, void* stream);
/* the dequantised matrix, [rows][cols] f32 (bit-exact check of repack + decode) */
int tn_matrix_dequant(const tn_matrix* m, float* d_out, void* stream);
uint64_t tn_matrix_device_bytes(const tn_matrix* m);
/* Test hook: the sum of the matrix's cross-CTA arrival and ticket counters,
 * which every completed matvec leaves at zero for the next launch
 * (synchronises the matrix's device). */
int tn_matrix_counter_sum(const tn_matrix* m, int64_t* out);
void tn_matrix_free(tn_matrix* m);

/* GQA attention for query rows over an f32 KV cache laid out
 * [n_slots][n_kv_heads][max_ctx][head_dim] (K and V separately).  Row r uses
 * slot d_slot[r] and cached positions [0, d_len[r]); a row whose slot is
 * outside [0, n_slots) or whose length is < 1 yields zeros, lengths above
 * max_ctx are clamped.  Math of
 * web/inference-worker.js:556-564; d_q, d_out: [n_rows][n_heads*head_dim].
 * d_scratch (device, tn_attention_scratch_bytes() bytes, 256-byte aligned)
 * holds the row table (16 bytes a row) and, when few rows leave SMs idle and
 * each row's positions are split over several CTAs, the splits' arrival
 * counters and partial results (merged on the device in split order, so the
 * output is deterministic).  Any row count that fits the caller's buffers is
 * accepted. */
uint64_t tn_attention_scratch_bytes(int32_t n_rows, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                                    int32_t max_ctx);
int tn_attention(int32_t n_rows, int32_t n_slots, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                 int32_t max_ctx, const float* d_q, const float* d_k, const float* d_v,
                 const int32_t* d_slot, const int32_t* d_len, float* d_out, void* d_scratch,
                 uint64_t scratch_bytes, void* stream);
/* tn_attention over an fp16 KV cache (IEEE binary16 bits, same layout): the
 * cache format of stages created with TN_FLAG_KV_F16.  Scores, softmax and the
 * weighted sum are computed in f32 from the fp16 rows. */
int tn_attention_f16(int32_t n_rows, int32_t n_slots, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                     int32_t max_ctx, const float* d_q, const uint16_t* d_k, const uint16_t* d_v,
                     const int32_t* d_slot, const int32_t* d_len, float* d_out, void* d_scratch,
                     uint64_t scratch_bytes, void* stream);

/* tn_attention over a paged cache, the layout of stages created with
 * kv_page_tokens > 0, one layer: d_k / d_v are pools of n_pages pages
 * [page][kv_head][page_tokens][head_dim] of kv_type elements (0 f32, 1 fp16,
 * 2 fp8 e4m3; 16-byte aligned); row r's positions 0 .. d_len[r] - 1 are
 * position p % page_tokens of page d_pages[r * max_pages + p / page_tokens].
 * page_tokens is a power of two in [16, 4096], max_pages <= 1023.  A row whose
 * used page ids leave [0, n_pages) gives zeros.  Scratch as tn_attention with
 * max_ctx = max_pages * page_tokens. */
int tn_attention_paged(int32_t kv_type, int32_t n_rows, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                       int32_t page_tokens, int32_t max_pages, int32_t n_pages, const float* d_q, const void* d_k,
                       const void* d_v, const int32_t* d_pages, const int32_t* d_len, float* d_out,
                       void* d_scratch, uint64_t scratch_bytes, void* stream);

/* tn_attention over an fp8 e4m3 KV cache (one byte a value, same layout): the
 * cache format of stages created with TN_FLAG_KV_F8.  Computed in f32. */
int tn_attention_f8(int32_t n_rows, int32_t n_slots, int32_t n_heads, int32_t n_kv_heads, int32_t head_dim,
                    int32_t max_ctx, const float* d_q, const uint8_t* d_k, const uint8_t* d_v,
                    const int32_t* d_slot, const int32_t* d_len, float* d_out, void* d_scratch,
                    uint64_t scratch_bytes, void* stream);

/* tn_attention without a scratch argument, for callers that cannot allocate
 * device memory.  This entry point has no counterpart in the reference.
 *
 * Some callers of this library cannot call cudaMalloc: a host whose memory
 * manager owns the whole device and forbids allocations behind its back (a
 * framework caching allocator, or a Node-API addon that only receives buffers
 * from JavaScript), a C binding layer that has no allocator of its own, or a
 * serving loop that must never pay the device-wide synchronisation that
 * cudaMalloc/cudaFree can imply.  This variant takes the same inputs and
 * output as tn_attention but keeps its scratch (row table, split counters and
 * partials) in a fixed array compiled into the library:
 * TN_ATTENTION_STATIC_SCRATCH_BYTES (1 MiB) of device memory, held on every
 * GPU that loads the library until the process exits.  The number of splits
 * per row is reduced until the partials fit; calls whose row table alone
 * exceeds the array (more than 65536 rows) fail with TN_ECAPACITY and launch
 * nothing; nothing here allocates.
 *
 * It runs on the calling thread's current device.  Its first call on a device
 * looks up that device's address of the array (once per device), so make that
 * first call before any stream capture.  All calls share the one array and
 * leave their contents in it; every call writes all it reads, so nothing needs
 * clearing, but calls whose work overlaps on the GPU (other streams, other
 * threads) race on the array and must be serialised by the caller.  The
 * address is kept for the life of the process: after cudaDeviceReset (or a
 * reset of the device's primary context) reload the library before calling
 * this entry point again. */
#define TN_ATTENTION_STATIC_SCRATCH_BYTES (1u << 20)
int tn_attention_static(int32_t n_rows, int32_t n_slots, int32_t n_heads, int32_t n_kv_heads,
                        int32_t head_dim, int32_t max_ctx, const float* d_q, const float* d_k,
                        const float* d_v, const int32_t* d_slot, const int32_t* d_len, float* d_out,
                        void* stream);

/* Test hook: one CTA runs the kernels' bounded mbarrier wait on a barrier
 * that nothing arrives at, with a limit of limit_cycles SM cycles (at most the
 * kernels' own ~2 s).  Returns TN_ETIMEOUT when the wait gave up -- always,
 * by construction -- and leaves the device usable; synchronises the device.
 * No counterpart in the reference. */
int tn_test_bounded_wait(uint64_t limit_cycles);

/* Activation hop codec, bit-exact with f32ToF16 / f16ToF32
 * (web/inference-worker.js:68-88): round half up, subnormal mantissa masked. */
int tn_hop_encode(const float* d_in, uint16_t* d_out, uint64_t n, void* stream);
int tn_hop_decode(const uint16_t* d_in, float* d_out, uint64_t n, void* stream);
uint16_t tn_hop_encode_host(float v);

/* Sampling of web/inference-worker.js:658-672 over [n_rows][vocab] logits.
 * temperature <= 0: greedy (lowest index among maxima).  Otherwise softmax
 * at `temperature`, nucleus `top_p`, and the uniform tn_sample_uniform(seed, row)
 * in place of Math.random(). */
int tn_sample(float* d_logits, int32_t n_rows, int32_t vocab, double temperature, double top_p,
              uint64_t rng_seed, int32_t* d_out, void* stream); /* temperature > 0 overwrites d_logits */
double tn_sample_uniform(uint64_t rng_seed, uint64_t row);

/* ---- synthetic model packs (seeded weights in the reference byte layout) ----
 * Deterministic across host and device: the same seed gives the same bytes. */
typedef struct {
  int32_t hidden_dim, n_heads, n_kv_heads, vocab, ffn_dim;
} tn_dims;
enum { TN_TAG_EMBED = 1, TN_TAG_NORM = 2, TN_TAG_LM_HEAD = 3 };
/* bytes of one packed layer (web/inference-worker.js:142-178) */
uint64_t tn_layer_bytes(const tn_dims* dims, int32_t quant);
/* quantBytesFor (web/inference-worker.js:130-137); 0 for an unknown quant */
uint64_t tn_quant_bytes(uint64_t count, int32_t quant);
/* one packed layer; `out` is host memory, or device memory when on_device */
int tn_synth_layer(uint64_t seed, int32_t layer_idx, const tn_dims* dims, int32_t quant, void* out,
                   int32_t on_device, void* stream);
/* a whole-model tensor: tag TN_TAG_EMBED / TN_TAG_LM_HEAD ([vocab x H] in
 * `quant`) or TN_TAG_NORM ([H] f16) */
int tn_synth_tensor(uint64_t seed, int32_t tag, const tn_dims* dims, int32_t quant, void* out,
                    int32_t on_device, void* stream);

int tn_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* TABNET_STAGE_H */
