/*
 * ref_cpu.c -- ORACLE (test infrastructure only; see ref_cpu.h).
 *
 * Line-by-line restatement of the ce-tabnet stage engine's CPU path,
 * web/inference-worker.js, in the numeric model of JavaScript: double for
 * every Number, float for every Float32Array element.  Each function cites the
 * reference lines it follows.  Compile with -ffp-contract=off (JS never fuses
 * a multiply into an add).
 */
#include "ref_cpu.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define QK 32 /* web/inference-worker.js:101 */

/* JS Math.round: the integer closest to x, ties toward +Infinity.  Computed
 * without the floor(x + 0.5) double-rounding trap (x - floor(x) is exact). */
static double js_round(double x) {
  double r = floor(x);
  return (x - r >= 0.5) ? r + 1.0 : r;
}

/* web/inference-worker.js:68-73 */
double ref_f16_to_f32(uint16_t h) {
  int s = (h & 0x8000) >> 15, e = (h & 0x7c00) >> 10, f = h & 0x03ff;
  if (e == 0) return (s ? -1.0 : 1.0) * pow(2.0, -14) * (f / 1024.0);
  if (e == 0x1f) return f ? NAN : (s ? -INFINITY : INFINITY);
  return (s ? -1.0 : 1.0) * pow(2.0, e - 15) * (1.0 + f / 1024.0);
}

/* web/inference-worker.js:74-88 (round-half-up; subnormal branch masks m) */
uint16_t ref_f32_to_f16(double val) {
  if (isnan(val)) return 0x7e00;
  uint16_t sign = (val < 0 || (val == 0 && signbit(val))) ? 0x8000 : 0;
  val = fabs(val);
  if (isinf(val)) return sign | 0x7c00;
  if (val == 0) return sign;
  double e = floor(log2(val));
  e = fmax(-25.0, fmin(16.0, e));
  double m;
  if (e < -14) {
    m = js_round(val / pow(2.0, -24));
    return (uint16_t)(sign | ((int64_t)m & 0x3ff));
  }
  m = js_round((val / pow(2.0, e) - 1.0) * 1024.0);
  if (m == 1024) { e += 1; m = 0; }
  if (e > 15) return sign | 0x7c00;
  return (uint16_t)(sign | (((int)e + 15) << 10) | ((int64_t)m & 0x3ff));
}

void ref_f32_to_f16_array(const float* in, uint16_t* out, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; i++) out[i] = ref_f32_to_f16((double)in[i]);
}

void ref_f32bits_to_f16_range(uint32_t first_bits, uint64_t count, uint16_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)count; i++) {
    uint32_t b = first_bits + (uint32_t)i;
    float f;
    memcpy(&f, &b, 4);
    out[i] = ref_f32_to_f16((double)f);
  }
}

/* web/inference-worker.js:130-137 */
int64_t ref_quant_bytes(int64_t count, int quant) {
  if (quant == REF_F32) return count * 4;
  if (quant == REF_F16) return count * 2;
  int64_t nblocks = (count + QK - 1) / QK;
  if (quant == REF_Q8_0) return nblocks * (2 + QK);
  if (quant == REF_Q4_0) return nblocks * (2 + QK / 2);
  return -1;
}

static uint16_t rd_u16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* web/inference-worker.js:102-129, for elements [start, start+count) of the
 * flattened tensor (blocks are laid over the flat tensor, so a row that does
 * not start on a 32-element boundary straddles two blocks). */
int ref_dequant_range(const uint8_t* buf, int quant, int64_t start, int64_t count, float* out) {
  if (quant == REF_F32) {
    memcpy(out, buf + start * 4, (size_t)count * 4);
    return 0;
  }
  if (quant == REF_F16) {
    for (int64_t i = 0; i < count; i++) out[i] = (float)ref_f16_to_f32(rd_u16(buf + (start + i) * 2));
    return 0;
  }
  if (quant != REF_Q8_0 && quant != REF_Q4_0) return -1;
  const int64_t bb = (quant == REF_Q8_0) ? (2 + QK) : (2 + QK / 2);
  for (int64_t i = 0; i < count; i++) {
    const int64_t w = start + i, b = w / QK, j = w % QK;
    const uint8_t* blk = buf + b * bb;
    const double scale = ref_f16_to_f32(rd_u16(blk));
    if (quant == REF_Q8_0) {
      out[i] = (float)((double)(int8_t)blk[2 + j] * scale);           /* :112 */
    } else {
      const uint8_t byte = blk[2 + j / 2];
      const int nib = (j & 1) ? (byte >> 4) : (byte & 0x0f);          /* :119-121 */
      out[i] = (float)((double)(nib - 8) * scale);
    }
  }
  return 0;
}

/* web/inference-worker.js:160-163 */
int ref_round_ffn(int H) {
  int x = (int)floor((8.0 * H) / 3.0);
  return (int)ceil(x / 256.0) * 256;
}

/* web/inference-worker.js:142-159 and the offsets walk of dequantLayer :166-178 */
int ref_layer_layout(int H, int nH, int nKV, int ffn_dim, int quant, ref_layout* L) {
  if (H <= 0 || nH <= 0 || nKV <= 0) return -1;
  L->H = H; L->nH = nH; L->nKV = nKV;
  L->headDim = (int)floor((double)H / nH);
  L->qDim = nH * L->headDim;
  L->kvDim = nKV * L->headDim;
  L->ffn = ffn_dim ? ffn_dim : ref_round_ffn(H);
  const int64_t counts[9] = {H,
                             (int64_t)H * L->qDim,
                             (int64_t)H * L->kvDim,
                             (int64_t)H * L->kvDim,
                             (int64_t)L->qDim * H,
                             H,
                             (int64_t)H * L->ffn,
                             (int64_t)H * L->ffn,
                             (int64_t)L->ffn * H};
  int64_t off = 0;
  for (int t = 0; t < 9; t++) {
    const int eff = (t == 0 || t == 5) ? REF_F16 : quant; /* norms stored f16 (:171-172) */
    const int64_t nb = ref_quant_bytes(counts[t], eff);
    if (nb < 0) return -1;
    L->off[t] = off;
    L->count[t] = counts[t];
    off += nb;
  }
  L->total = off;
  return 0;
}

/* web/inference-worker.js:516-522 */
void ref_rmsnorm(const float* x, const float* w, int H, float* o) {
  double s = 0;
  for (int i = 0; i < H; i++) s += (double)x[i] * (double)x[i];
  const double inv = 1.0 / sqrt(s / H + 1e-5);
  for (int i = 0; i < H; i++) o[i] = (float)((double)x[i] * inv * (double)w[i]);
}

/* web/inference-worker.js:523-527, dequantising each row on the fly (the
 * values are identical to the reference's pre-dequantised f32 tensor: every
 * q*scale product is exact in float). Row-parallel; each row's sum runs in
 * the reference's order, so the result does not depend on n_threads. */
int ref_matvec_packed(const uint8_t* W, int quant, int rows, int cols, const float* x, float* y,
                      int n_threads) {
  if (ref_quant_bytes(1, quant) < 0) return -1;
  if (n_threads <= 0) n_threads = 1;
  int err = 0;
#pragma omp parallel num_threads(n_threads)
  {
    float* row = (float*)malloc(sizeof(float) * (size_t)cols);
    if (!row) {
#pragma omp atomic write
      err = -2;
    }
#pragma omp for schedule(static)
    for (int r = 0; r < rows; r++) {
      if (!row) continue;
      double a = 0;
      if ((quant == REF_Q4_0 || quant == REF_Q8_0) && cols % QK == 0) {
        /* Rows start on a block boundary: the block loop of dequantToF32
         * (web/inference-worker.js:107-124) takes each block's scale once, and
         * every weight is formed and accumulated exactly as below in element
         * order, so the sums are those of the element-wise path. */
        const int64_t bb = (quant == REF_Q8_0) ? (2 + QK) : (2 + QK / 2);
        const uint8_t* blk = W + ((int64_t)r * cols / QK) * bb;
        for (int c0 = 0; c0 < cols; c0 += QK, blk += bb) {
          const double scale = ref_f16_to_f32(rd_u16(blk));
          for (int j = 0; j < QK; j++) {
            float w;
            if (quant == REF_Q8_0) {
              w = (float)((double)(int8_t)blk[2 + j] * scale);
            } else {
              const uint8_t byte = blk[2 + j / 2];
              const int nib = (j & 1) ? (byte >> 4) : (byte & 0x0f);
              w = (float)((double)(nib - 8) * scale);
            }
            a += (double)w * (double)x[c0 + j];
          }
        }
      } else {
        ref_dequant_range(W, quant, (int64_t)r * cols, cols, row);
        for (int c = 0; c < cols; c++) a += (double)row[c] * (double)x[c];
      }
      y[r] = (float)a;
    }
    free(row);
  }
  return err;
}

/* web/inference-worker.js:528-540 */
void ref_rope(float* vec, int nHeads, int headDim, int pos, double theta) {
  const int half = headDim >> 1;
  for (int h = 0; h < nHeads; h++) {
    const int base = h * headDim;
    for (int i = 0; i < half; i++) {
      const double freq = pow(theta, (double)(-2 * i) / headDim);
      const double ang = pos * freq, c = cos(ang), s = sin(ang);
      const double a = vec[base + i], b = vec[base + half + i];
      vec[base + i] = (float)(a * c - b * s);
      vec[base + half + i] = (float)(a * s + b * c);
    }
  }
}

/* web/inference-worker.js:556-564 */
void ref_attention(const float* q, const float* K, const float* V, int S, int nH, int nKV, int hd,
                   float* attnOut) {
  const int kvDim = nKV * hd;
  const double g = (double)nH / nKV;
  const double scale = 1.0 / sqrt((double)hd);
  float* scores = (float*)malloc(sizeof(float) * (size_t)(S > 0 ? S : 1));
  for (int head = 0; head < nH; head++) {
    const int kvh = (int)floor(head / g), qb = head * hd;
    double mx = -INFINITY;
    for (int s = 0; s < S; s++) {
      const float* kk = K + (size_t)s * kvDim;
      const int kb = kvh * hd;
      double dot = 0;
      for (int dd = 0; dd < hd; dd++) dot += (double)q[qb + dd] * (double)kk[kb + dd];
      dot *= scale;
      scores[s] = (float)dot;
      if (dot > mx) mx = dot;
    }
    double den = 0;
    for (int s = 0; s < S; s++) {
      scores[s] = (float)exp((double)scores[s] - mx);
      den += (double)scores[s];
    }
    for (int dd = 0; dd < hd; dd++) {
      double acc = 0;
      for (int s = 0; s < S; s++) acc += (double)scores[s] * (double)V[(size_t)s * kvDim + kvh * hd + dd];
      attnOut[qb + dd] = (float)(acc / den);
    }
  }
  free(scores);
}

/* ---- sampling, web/inference-worker.js:658-672 ---- */
static const float* g_sort_probs; /* qsort has no context pointer in C99 */
static int cmp_prob_desc(const void* pa, const void* pb) {
  const int a = *(const int*)pa, b = *(const int*)pb;
  const double d = (double)g_sort_probs[b] - (double)g_sort_probs[a];
  if (d > 0) return 1;
  if (d < 0) return -1;
  return (a > b) - (a < b); /* V8's Array.prototype.sort is stable */
}

int ref_sample(const float* logits, int n, double temperature, double top_p, double u) {
  if (temperature <= 0) {
    int bi = 0;
    double bv = -INFINITY;
    for (int i = 0; i < n; i++)
      if ((double)logits[i] > bv) { bv = logits[i]; bi = i; }
    return bi;
  }
  double mx = -INFINITY;
  for (int i = 0; i < n; i++)
    if ((double)logits[i] > mx) mx = logits[i];
  float* probs = (float*)malloc(sizeof(float) * (size_t)n);
  int* idx = (int*)malloc(sizeof(int) * (size_t)n);
  double sum = 0;
  for (int i = 0; i < n; i++) {
    const double e = exp(((double)logits[i] - mx) / temperature);
    probs[i] = (float)e;
    sum += e;
  }
  for (int i = 0; i < n; i++) probs[i] = (float)((double)probs[i] / sum);
  for (int i = 0; i < n; i++) idx[i] = i;
  g_sort_probs = probs;
  qsort(idx, (size_t)n, sizeof(int), cmp_prob_desc);
  double cum = 0;
  int cut = n;
  for (int r = 0; r < n; r++) {
    cum += probs[idx[r]];
    if (cum >= top_p) { cut = r + 1; break; }
  }
  const double r = u * cum;
  double acc = 0;
  int out = idx[0];
  for (int j = 0; j < cut; j++) {
    acc += probs[idx[j]];
    if (r <= acc) { out = idx[j]; break; }
  }
  free(probs);
  free(idx);
  return out;
}

/* ---- stage ---- */
typedef struct {
  uint64_t id;
  int len, cap;
  float** K; /* [nLayers] -> [cap][kvDim] */
  float** V;
} ref_seq;

struct ref_stage {
  ref_spec spec;
  ref_layout L;
  int nLayers;
  float** norms;        /* [nLayers*2] attn_norm, ffn_norm as f32 */
  float* embed;         /* [vocab*H] f32 (first stage) */
  float* final_norm;    /* [H] */
  ref_seq* seqs;
  int n_seqs, cap_seqs;
  int kv_fmt; /* not in the reference: KV rows rounded to binary16 (1) or e4m3 (2) when pushed */
};

/* x rounded to the nearest binary16 value (ties to even), as a float: the
   stored value of an fp16 KV cache.  Overflow gives infinity. */
static float round_f16(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  const uint32_t sign = u & 0x80000000u, a = u & 0x7fffffffu;
  if (a >= 0x7f800000u) return x; /* inf, nan */
  if (a >= 0x38800000u) {         /* binary16 normal range: keep 10 mantissa bits */
    uint32_t r = a + 0xfffu + ((a >> 13) & 1u);
    r &= ~0x1fffu;
    if (r >= 0x47800000u) r = 0x7f800000u;
    r |= sign;
    float y;
    memcpy(&y, &r, 4);
    return y;
  }
  /* subnormal range: multiples of 2^-24 (x * 2^24 is exact) */
  return rintf(x * 16777216.0f) * (1.0f / 16777216.0f);
}

/* x rounded to the nearest fp8 e4m3 value (OCP FP8 E4M3: bias 7, 3 mantissa
   bits, largest finite 448, no infinities), ties to even, saturating finite:
   the stored value of an fp8 KV cache.  NaN stays NaN. */
static float round_e4m3(float x) {
  if (isnan(x)) return x;
  const float a = fabsf(x);
  float r;
  if (isinf(a)) {
    r = 448.0f;
  } else if (a >= 0.015625f) { /* normal: 2^e <= a < 2^(e+1), quantum 2^(e-3) */
    int E;
    frexpf(a, &E); /* a = m 2^E, 0.5 <= m < 1, so e = E - 1 */
    r = ldexpf(rintf(ldexpf(a, 4 - E)), E - 4);
    if (r > 448.0f) r = 448.0f;
  } else { /* subnormal: multiples of 2^-9 */
    r = rintf(a * 512.0f) * (1.0f / 512.0f);
  }
  return signbit(x) ? -r : r;
}

static float round_kv(int fmt, float x) { return fmt == 1 ? round_f16(x) : (fmt == 2 ? round_e4m3(x) : x); }

void ref_set_kv_format(ref_stage* st, int fmt) { st->kv_fmt = (fmt == 1 || fmt == 2) ? fmt : 0; }

float ref_round_kv(int fmt, float x) { return round_kv(fmt, x); }

static ref_seq* find_seq(ref_stage* st, uint64_t id, int create) {
  for (int i = 0; i < st->n_seqs; i++)
    if (st->seqs[i].id == id) return &st->seqs[i];
  if (!create) return NULL;
  if (st->n_seqs == st->cap_seqs) {
    int nc = st->cap_seqs ? st->cap_seqs * 2 : 8;
    ref_seq* ns = (ref_seq*)realloc(st->seqs, sizeof(ref_seq) * (size_t)nc);
    if (!ns) return NULL;
    st->seqs = ns;
    st->cap_seqs = nc;
  }
  ref_seq* s = &st->seqs[st->n_seqs++];
  memset(s, 0, sizeof(*s));
  s->id = id;
  s->K = (float**)calloc((size_t)st->nLayers, sizeof(float*));
  s->V = (float**)calloc((size_t)st->nLayers, sizeof(float*));
  return s;
}

static int seq_reserve(ref_stage* st, ref_seq* s, int need) {
  if (need <= s->cap) return 0;
  int nc = s->cap ? s->cap : 16;
  while (nc < need) nc *= 2;
  const size_t kvDim = (size_t)st->L.kvDim;
  for (int l = 0; l < st->nLayers; l++) {
    float* nk = (float*)realloc(s->K[l], sizeof(float) * kvDim * (size_t)nc);
    if (!nk) return -2;
    s->K[l] = nk;
    float* nv = (float*)realloc(s->V[l], sizeof(float) * kvDim * (size_t)nc);
    if (!nv) return -2;
    s->V[l] = nv;
  }
  s->cap = nc;
  return 0;
}

/* web/inference-worker.js:417-466 */
ref_stage* ref_init(const ref_spec* spec) {
  ref_stage* st = (ref_stage*)calloc(1, sizeof(ref_stage));
  if (!st) return NULL;
  st->spec = *spec;
  st->nLayers = spec->layer_hi - spec->layer_lo;
  if (st->nLayers != spec->n_layers) { free(st); return NULL; }
  const int q0 = spec->n_layers > 0 ? spec->layer_quants[0] : REF_Q8_0;
  if (ref_layer_layout(spec->hidden_dim, spec->n_heads, spec->n_kv_heads, spec->ffn_dim, q0, &st->L)) {
    free(st);
    return NULL;
  }
  const int H = spec->hidden_dim;
  st->norms = (float**)calloc((size_t)(2 * st->nLayers + 1), sizeof(float*));
  for (int l = 0; l < st->nLayers; l++) {
    ref_layout Ll;
    if (ref_layer_layout(H, spec->n_heads, spec->n_kv_heads, spec->ffn_dim, spec->layer_quants[l], &Ll)) {
      ref_free(st);
      return NULL;
    }
    st->norms[2 * l] = (float*)malloc(sizeof(float) * (size_t)H);
    st->norms[2 * l + 1] = (float*)malloc(sizeof(float) * (size_t)H);
    ref_dequant_range(spec->layer_bufs[l] + Ll.off[0], REF_F16, 0, H, st->norms[2 * l]);
    ref_dequant_range(spec->layer_bufs[l] + Ll.off[5], REF_F16, 0, H, st->norms[2 * l + 1]);
  }
  if (spec->is_first && spec->embed) {
    st->embed = (float*)malloc(sizeof(float) * (size_t)spec->vocab * H);
    if (!st->embed || ref_dequant_range(spec->embed, spec->embed_quant, 0, (int64_t)spec->vocab * H, st->embed)) {
      ref_free(st);
      return NULL;
    }
  }
  if (spec->is_last && spec->norm) {
    st->final_norm = (float*)malloc(sizeof(float) * (size_t)H);
    ref_dequant_range(spec->norm, REF_F16, 0, H, st->final_norm);
  }
  return st;
}

/* web/inference-worker.js:541-578 (runLayersCpu) */
static int run_layers(ref_stage* st, ref_seq* kv, int pos, float* h) {
  const ref_spec* sp = &st->spec;
  const int H = sp->hidden_dim, nH = sp->n_heads, nKV = sp->n_kv_heads, hd = st->L.headDim;
  const int qDim = nH * hd, kvDim = nKV * hd, ffn = st->L.ffn;
  const int nt = sp->n_threads;
  if (seq_reserve(st, kv, kv->len + 1)) return -2;
  float* xn = (float*)malloc(sizeof(float) * (size_t)H);
  float* q = (float*)malloc(sizeof(float) * (size_t)qDim);
  float* k = (float*)malloc(sizeof(float) * (size_t)kvDim);
  float* v = (float*)malloc(sizeof(float) * (size_t)kvDim);
  float* att = (float*)malloc(sizeof(float) * (size_t)qDim);
  float* proj = (float*)malloc(sizeof(float) * (size_t)H);
  float* gate = (float*)malloc(sizeof(float) * (size_t)ffn);
  float* up = (float*)malloc(sizeof(float) * (size_t)ffn);
  float* act = (float*)malloc(sizeof(float) * (size_t)ffn);
  int rc = 0;
  for (int li = 0; li < st->nLayers && rc == 0; li++) {
    const int quant = sp->layer_quants[li];
    ref_layout Ll;
    ref_layer_layout(H, nH, nKV, sp->ffn_dim, quant, &Ll);
    const uint8_t* b = sp->layer_bufs[li];
    /* attention */
    ref_rmsnorm(h, st->norms[2 * li], H, xn);
    rc |= ref_matvec_packed(b + Ll.off[1], quant, qDim, H, xn, q, nt);
    rc |= ref_matvec_packed(b + Ll.off[2], quant, kvDim, H, xn, k, nt);
    rc |= ref_matvec_packed(b + Ll.off[3], quant, kvDim, H, xn, v, nt);
    ref_rope(q, nH, hd, pos, sp->rope_theta);
    ref_rope(k, nKV, hd, pos, sp->rope_theta);
    if (st->kv_fmt)
      for (int i = 0; i < kvDim; i++) {
        k[i] = round_kv(st->kv_fmt, k[i]);
        v[i] = round_kv(st->kv_fmt, v[i]);
      }
    memcpy(kv->K[li] + (size_t)kv->len * kvDim, k, sizeof(float) * (size_t)kvDim); /* :554 push */
    memcpy(kv->V[li] + (size_t)kv->len * kvDim, v, sizeof(float) * (size_t)kvDim);
    const int S = kv->len + 1;
    ref_attention(q, kv->K[li], kv->V[li], S, nH, nKV, hd, att);
    rc |= ref_matvec_packed(b + Ll.off[4], quant, H, qDim, att, proj, nt);
    for (int i = 0; i < H; i++) h[i] = (float)((double)h[i] + (double)proj[i]); /* :566 */
    /* MLP (SwiGLU) */
    ref_rmsnorm(h, st->norms[2 * li + 1], H, xn);
    rc |= ref_matvec_packed(b + Ll.off[6], quant, ffn, H, xn, gate, nt);
    rc |= ref_matvec_packed(b + Ll.off[7], quant, ffn, H, xn, up, nt);
    for (int i = 0; i < ffn; i++) {
      const double gv = gate[i];
      act[i] = (float)((gv / (1.0 + exp(-gv))) * (double)up[i]);                /* :572 */
    }
    rc |= ref_matvec_packed(b + Ll.off[8], quant, H, ffn, act, proj, nt);
    for (int i = 0; i < H; i++) h[i] = (float)((double)h[i] + (double)proj[i]); /* :574 */
  }
  if (rc == 0) kv->len += 1; /* every layer pushed one row */
  free(xn); free(q); free(k); free(v); free(att); free(proj); free(gate); free(up); free(act);
  return rc;
}

int ref_forward(ref_stage* st, uint64_t seq_id, int token_pos, const int32_t* token_ids,
                const uint16_t* hidden, int n, double temperature, double top_p, double u,
                uint16_t* out_hidden, int32_t* out_token, float* out_f32, float* out_logits) {
  const ref_spec* sp = &st->spec;
  const int H = sp->hidden_dim;
  if (n <= 0) return -1;
  ref_seq* kv = find_seq(st, seq_id, 1);
  if (!kv) return -2;
  float* h = (float*)malloc(sizeof(float) * (size_t)H);
  int rc = 0;
  for (int p = 0; p < n && rc == 0; p++) {
    const int pos = token_pos + p;
    if (sp->is_first) {
      /* embedLookup :509-515 (ids outside [0, vocab) are rejected here; the
       * reference would silently produce a zero or partial row) */
      const int32_t id = token_ids[p];
      if (!st->embed || id < 0 || id >= sp->vocab) { rc = -1; break; }
      memcpy(h, st->embed + (size_t)id * H, sizeof(float) * (size_t)H);
    } else {
      for (int i = 0; i < H; i++) h[i] = (float)ref_f16_to_f32(hidden[(size_t)p * H + i]);
    }
    rc = run_layers(st, kv, pos, h);
  }
  if (rc == 0) {
    if (out_f32) memcpy(out_f32, h, sizeof(float) * (size_t)H);
    if (sp->is_last) {
      /* runLastCpu :579-583, then sample :715 */
      float* hn = (float*)malloc(sizeof(float) * (size_t)H);
      float* logits = (float*)malloc(sizeof(float) * (size_t)sp->vocab);
      ref_rmsnorm(h, st->final_norm, H, hn);
      rc = ref_matvec_packed(sp->lm_head, sp->lm_head_quant, sp->vocab, H, hn, logits, sp->n_threads);
      if (rc == 0) {
        if (out_logits) memcpy(out_logits, logits, sizeof(float) * (size_t)sp->vocab);
        if (out_token) *out_token = ref_sample(logits, sp->vocab, temperature, top_p, u);
      }
      free(hn);
      free(logits);
    } else if (out_hidden) {
      for (int i = 0; i < H; i++) out_hidden[i] = ref_f32_to_f16((double)h[i]);
    }
  }
  free(h);
  return rc;
}

int ref_kv_len(ref_stage* st, uint64_t seq_id) {
  ref_seq* s = find_seq(st, seq_id, 0);
  return s ? s->len : 0;
}

int ref_kv_row(ref_stage* st, uint64_t seq_id, int li, int s_idx, float* k_out, float* v_out) {
  ref_seq* s = find_seq(st, seq_id, 0);
  if (!s || li < 0 || li >= st->nLayers || s_idx < 0 || s_idx >= s->len) return -1;
  const size_t kvDim = (size_t)st->L.kvDim;
  memcpy(k_out, s->K[li] + (size_t)s_idx * kvDim, sizeof(float) * kvDim);
  memcpy(v_out, s->V[li] + (size_t)s_idx * kvDim, sizeof(float) * kvDim);
  return 0;
}

void ref_free(ref_stage* st) {
  if (!st) return;
  for (int i = 0; i < st->n_seqs; i++) {
    for (int l = 0; l < st->nLayers; l++) {
      free(st->seqs[i].K[l]);
      free(st->seqs[i].V[l]);
    }
    free(st->seqs[i].K);
    free(st->seqs[i].V);
  }
  free(st->seqs);
  if (st->norms)
    for (int l = 0; l < 2 * st->nLayers; l++) free(st->norms[l]);
  free(st->norms);
  free(st->embed);
  free(st->final_norm);
  free(st);
}
