/*
 * ref_cpu.h -- ORACLE (test infrastructure only).
 *
 * A C restatement of the ce-tabnet stage engine's CPU path
 * (web/inference-worker.js, the "WASM/CPU fallback"), used as the parity
 * checker for the CUDA stage engine and as the timed CPU baseline.  Nothing in
 * the product links this library; only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py load it.
 *
 * Numeric model (the reference runs in JavaScript): every JS Number is an
 * IEEE double, every Float32Array element is a float (stores round to nearest
 * even).  Accumulators, norms, RoPE and softmax are therefore computed in
 * double and rounded to float where the reference stores into a Float32Array.
 * The build disables FP contraction so a*c - b*s is not fused (JS never fuses).
 * The only known approximation: glibc's exp/pow/cos/sin/log2 versus V8's
 * fdlibm-derived versions may differ by <= 1 ulp in double, which is almost
 * always invisible after the float store.
 *
 * Parity pin: the reference ships no golden vectors or engine tests (its only
 * test, dev/serve.js --selftest, drives a mock engine), and no JavaScript
 * runtime exists on this machine, so this oracle is "parity unpinned" against
 * reference-produced outputs.  It is pinned instead by known-answer tests
 * derived by hand from the reference source (tests/golden/).
 */
#ifndef TABNET_REF_CPU_H
#define TABNET_REF_CPU_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* quant codes (same numbering as the engine's tn_quant) */
enum { REF_F32 = 0, REF_F16 = 1, REF_Q4_0 = 2, REF_Q8_0 = 3 };

/* web/inference-worker.js:74-88 f32ToF16 (literal double-math restatement) */
uint16_t ref_f32_to_f16(double val);
/* web/inference-worker.js:68-73 f16ToF32 */
double ref_f16_to_f32(uint16_t h);
/* array forms (:89-90) with OpenMP over the array; used by exhaustive tests */
void ref_f32_to_f16_array(const float* in, uint16_t* out, int64_t n);
void ref_f32bits_to_f16_range(uint32_t first_bits, uint64_t count, uint16_t* out);

/* web/inference-worker.js:130-137 quantBytesFor; returns -1 on unsupported quant */
int64_t ref_quant_bytes(int64_t count, int quant);
/* web/inference-worker.js:102-129 dequantToF32, restricted to elements
 * [start, start+count) of a tensor whose packed bytes begin at `buf`. */
int ref_dequant_range(const uint8_t* buf, int quant, int64_t start, int64_t count, float* out);

/* web/inference-worker.js:142-163 layerLayout / roundFfn */
int ref_round_ffn(int hidden);
typedef struct {
  int H, nH, nKV, headDim, qDim, kvDim, ffn;
  int64_t off[9];    /* byte offset of attn_norm, wq, wk, wv, wo, ffn_norm, w_gate, w_up, w_down */
  int64_t count[9];  /* element counts */
  int64_t total;     /* packed layer bytes */
} ref_layout;
int ref_layer_layout(int hidden, int n_heads, int n_kv_heads, int ffn_dim, int quant, ref_layout* out);

/* kernels of the CPU path (web/inference-worker.js:516-540) */
void ref_rmsnorm(const float* x, const float* w, int H, float* out);
/* y[r] = sum_c W[r][c] * x[c]; W given as packed bytes of a [rows x cols] tensor */
int ref_matvec_packed(const uint8_t* W, int quant, int rows, int cols, const float* x, float* y,
                      int n_threads);
void ref_rope(float* vec, int n_heads, int head_dim, int pos, double theta);
/* one-query GQA attention over S cached rows (web/inference-worker.js:556-564).
 * K, V: [S][kvDim] rows; q: [nH*hd]; out: [nH*hd] */
void ref_attention(const float* q, const float* K, const float* V, int S, int nH, int nKV, int hd,
                   float* out);
/* web/inference-worker.js:658-672 sample; `u` replaces Math.random() */
int ref_sample(const float* logits, int n, double temperature, double top_p, double u);

/* ---- stage (initStage / forward / freeStage) ---- */
typedef struct {
  int hidden_dim, n_heads, n_kv_heads, vocab, ffn_dim; /* ffn_dim 0 -> roundFfn */
  double rope_theta;
  int layer_lo, layer_hi, is_first, is_last;
  const uint8_t* const* layer_bufs;
  const int* layer_quants;
  int n_layers;
  const uint8_t* embed; int embed_quant;
  const uint8_t* norm;          /* always f16 (web/inference-worker.js:442) */
  const uint8_t* lm_head; int lm_head_quant;
  int n_threads;                /* matvec row parallelism (results independent of it) */
} ref_spec;

typedef struct ref_stage ref_stage;

ref_stage* ref_init(const ref_spec* spec);
/*
 * forward (web/inference-worker.js:471-490, 690-716).  Exactly one of
 * token_ids (first stage; n positions) or hidden (other stages; n positions of
 * fp16 bits, n>1 runs the positions in order) is used.
 * Outputs: out_hidden (fp16 bits of the LAST position, [H]) when !is_last;
 * out_token when is_last; optional out_f32 ([H], the final f32 hidden state of
 * the last position, pre-encode) and out_logits ([vocab], last stage only).
 */
int ref_forward(ref_stage* st, uint64_t seq_id, int token_pos, const int32_t* token_ids,
                const uint16_t* hidden, int n, double temperature, double top_p, double u,
                uint16_t* out_hidden, int32_t* out_token, float* out_f32, float* out_logits);
/* KV rows currently cached for a sequence (0 if unknown) */
int ref_kv_len(ref_stage* st, uint64_t seq_id);
/* copy of the cached K/V row (layer li, row s) */
int ref_kv_row(ref_stage* st, uint64_t seq_id, int li, int s, float* k_out, float* v_out);
/* Not in the reference: store K / V rows rounded (ties to even) to binary16
   (fmt 1) or to fp8 e4m3 saturating at +-448 (fmt 2), the opt-in fp16 / fp8
   KV caches of the GPU stage; fmt 0 keeps f32 rows. */
void ref_set_kv_format(ref_stage* st, int fmt);
/* the rounding ref_set_kv_format applies, for one value */
float ref_round_kv(int fmt, float x);
void ref_free(ref_stage* st);

#ifdef __cplusplus
}
#endif
#endif
