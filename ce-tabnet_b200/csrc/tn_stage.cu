// tn_stage.cu -- stage runtime behind the C ABI (initStage / forward / freeStage).
//
// One tn_stage owns a contiguous layer slice [lo, hi) on one GPU
// (web/inference-worker.js:417-466): repacked weights, an f32 KV arena
// [slot][layer][kv_head][ctx][head_dim], activations for up to
// max_tokens_per_step rows, and one CUDA stream.  A forward call turns its
// requests into rows (sequence slot, RoPE position, KV index, attention
// length), uploads them with the inputs, runs the layer stack as one batched
// step (prefill positions and concurrent sequences alike) and reads back the
// fp16 hop rows or the sampled tokens.  Decode-shaped steps (one row per
// sequence) replay CUDA graphs captured per row count.
#include <cmath>
#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "tn_kernels.cuh"

namespace tn {

static thread_local char g_err[1024];
void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}
void clear_error() { g_err[0] = 0; }

// switches to `dev` for the lifetime of the guard
struct DevGuard {
  int prev = -1;
  cudaError_t err = cudaSuccess;
  explicit DevGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) err = cudaSetDevice(dev);
  }
  ~DevGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};
#define TN_ENTER_DEVICE(dev)                                                             \
  DevGuard dev_guard_(dev);                                                              \
  TN_REQUIRE(dev_guard_.err == cudaSuccess, TN_ECUDA, "cudaSetDevice(%d): %s", (int)(dev), \
             cudaGetErrorString(dev_guard_.err))

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

enum { IN_IDS = 0, IN_HIDDEN = 1 };
constexpr int CTL_RING = 8;

struct GraphEntry {
  cudaGraphExec_t exec = nullptr;
  int n_ev = 0, n_launch = 0;  // profiling events and kernel launches of the captured step
};

struct LayerW {
  Matrix qkv, o, gu, down;
  float* attn_norm = nullptr;
  float* ffn_norm = nullptr;
};

}  // namespace tn

using namespace tn;

struct tn_stage {
  std::mutex mu;
  int device = 0;
  cudaStream_t stream = nullptr;
  int H = 0, nH = 0, nKV = 0, hd = 0, qDim = 0, kvDim = 0, F = 0, V = 0;
  double theta = 0;
  int lo = 0, hi = 0, nL = 0;
  bool first = false, last = false;
  int max_ctx = 0, max_seqs = 0, max_T = 0;
  uint32_t flags = 0;
  std::vector<LayerW> layers;
  Matrix embed, lm_head;
  float* final_norm = nullptr;
  // KV arena
  char* kc = nullptr;  // kv_type elements
  char* vc = nullptr;
  int kv_type = KV_F32;
  // split-attention partials and arrival counters (zero between launches)
  float* attn_ws = nullptr;
  int* attn_cnt = nullptr;
  size_t attn_ws_floats = 0, attn_cnt_ints = 0;
  size_t kvh_stride = 0, layer_stride = 0, slot_stride = 0;
  // paged KV (kv_page_tokens > 0): a pool of n_pages pages laid out
  // [page][layer][kv_head][page_tokens][head_dim]; a sequence slot holds
  // seq_pages[slot] of them, listed in its row of the page table
  int page_tokens = 0, page_shift = 0, n_pages = 0, max_pages = 0;
  int* d_pages = nullptr;  // [max_seqs][max_pages] page ids
  int* h_pages = nullptr;  // pinned host copy
  std::vector<int> free_pages, seq_pages;
  KvMap kvmap;
  // activations
  float *h = nullptr, *xn = nullptr, *qkv = nullptr, *q = nullptr, *att = nullptr, *act = nullptr,
        *logits = nullptr;
  uint16_t *hid_in = nullptr, *hid_out = nullptr;
  int *ids = nullptr, *tok_out = nullptr, *err = nullptr;
  int* kerr = nullptr;  // set by a kernel whose bounded wait gave up
  void* gemm_ws = nullptr;  // activation tiles of the dequant-GEMM (steps of many rows)
  size_t gemm_ws_bytes = 0;
  double2* cs = nullptr;
  double* freq = nullptr;
  // control block: rows | outrows | sampler params, uploaded once per step
  char* d_ctl = nullptr;
  size_t ctl_outrows_off = 0, ctl_params_off = 0, ctl_bytes = 0;
  char* h_ctl[CTL_RING] = {};
  cudaEvent_t ctl_ev[CTL_RING] = {};
  int ctl_pos = 0;
  // pinned host staging of the synchronous API
  void* h_in = nullptr;
  void* h_out = nullptr;
  // sequences
  std::unordered_map<uint64_t, int> seq_slot;
  std::vector<int> free_slots;
  std::vector<int> kv_len;
  std::map<std::tuple<int, int, int>, GraphEntry> graphs;
  bool graphs_broken = false;
  // per-launch timing (TN_FLAG_PROFILE): begin/end event pairs of the current step
  bool prof = false;
  std::vector<cudaEvent_t> ev;
  std::vector<int> ev_class;
  int ev_used = 0, step_launches = 0;
  double prof_ms[TN_PROF_N] = {};
  uint64_t prof_launches[TN_PROF_N] = {};
  uint64_t weight_bytes = 0, kv_bytes = 0, scratch_bytes = 0, packed_bytes = 0;
  std::vector<void*> allocs;  // scratch allocations

  ~tn_stage();
};

static void free_ptr(void* p) {
  if (p) cudaFree(p);
}

tn_stage::~tn_stage() {
  for (auto& kv : graphs) cudaGraphExecDestroy(kv.second.exec);
  for (cudaEvent_t e : ev) cudaEventDestroy(e);
  for (auto& L : layers) {
    matrix_free(&L.qkv);
    matrix_free(&L.o);
    matrix_free(&L.gu);
    matrix_free(&L.down);
    free_ptr(L.attn_norm);
    free_ptr(L.ffn_norm);
  }
  matrix_free(&embed);
  matrix_free(&lm_head);
  free_ptr(final_norm);
  free_ptr(kc);
  free_ptr(vc);
  for (void* p : allocs) free_ptr(p);
  for (int i = 0; i < CTL_RING; i++) {
    if (h_ctl[i]) cudaFreeHost(h_ctl[i]);
    if (ctl_ev[i]) cudaEventDestroy(ctl_ev[i]);
  }
  if (h_in) cudaFreeHost(h_in);
  if (h_out) cudaFreeHost(h_out);
  if (h_pages) cudaFreeHost(h_pages);
  if (stream) cudaStreamDestroy(stream);
}

namespace tn {

template <typename T>
static int dalloc(tn_stage* st, T** p, size_t count) {
  const size_t bytes = align256(count * sizeof(T));
  cudaError_t e = cudaMalloc((void**)p, bytes);
  if (e != cudaSuccess) {
    *p = nullptr;
    set_error("cudaMalloc(%zu bytes): %s", bytes, cudaGetErrorString(e));
    return TN_ENOMEM;
  }
  st->allocs.push_back(*p);
  st->scratch_bytes += bytes;
  TN_CHECK_CUDA(cudaMemsetAsync(*p, 0, bytes, st->stream));
  return TN_OK;
}

// device copy of `bytes` of weights: the pointer itself when already on the
// device, else the staging buffer after an upload ordered on the stage stream.
// (A plain cudaMemcpy from pageable memory may return before its DMA lands, and
// the legacy stream does not order the non-blocking stage stream's repack after it.)
static int stage_src(const tn_stage_spec* sp, const void* src, uint64_t bytes, uint8_t* staging,
                     cudaStream_t s, const uint8_t** out) {
  if (sp->weights_on_device) {
    *out = (const uint8_t*)src;
    return TN_OK;
  }
  TN_CHECK_CUDA(cudaMemcpyAsync(staging, src, bytes, cudaMemcpyHostToDevice, s));
  *out = staging;
  return TN_OK;
}

static int load_layer(tn_stage* st, const tn_stage_spec* sp, int li, uint8_t* staging) {
  const tn_layer_weights& lw = sp->layers[li];
  LayerLayout L;
  TN_REQUIRE(layer_layout(st->H, st->nH, st->nKV, sp->ffn_dim, lw.quant, &L), TN_EUNSUPPORTED,
             "layer %d: unsupported quant %d", lw.idx, lw.quant);
  TN_REQUIRE(lw.buf && lw.len >= L.total, TN_EINVAL, "layer %d: buffer of %llu bytes, layout needs %llu",
             lw.idx, (unsigned long long)lw.len, (unsigned long long)L.total);
  const uint8_t* src = nullptr;
  int rc = stage_src(sp, lw.buf, L.total, staging, st->stream, &src);
  if (rc) return rc;
  LayerW& W = st->layers[li];
  const int q = lw.quant;
  // wq | wk | wv fused into one [qDim + 2 kvDim, H] matrix
  if ((rc = matrix_alloc(&W.qkv, q, st->qDim + 2 * st->kvDim, st->H, st->stream, false))) return rc;
  // (q and k rows pair-interleaved per head for the RoPE epilogue: stride -hd)
  if ((rc = matrix_repack(&W.qkv, src + L.off[1], q, st->qDim, 0, -st->hd, st->stream))) return rc;
  if ((rc = matrix_repack(&W.qkv, src + L.off[2], q, st->kvDim, st->qDim, -st->hd, st->stream))) return rc;
  if ((rc = matrix_repack(&W.qkv, src + L.off[3], q, st->kvDim, st->qDim + st->kvDim, 1, st->stream)))
    return rc;
  if ((rc = matrix_alloc(&W.o, q, st->H, st->qDim, st->stream, false))) return rc;
  if ((rc = matrix_repack(&W.o, src + L.off[4], q, st->H, 0, 1, st->stream))) return rc;
  // w_gate / w_up interleaved by row: (2i, 2i+1) = (gate_i, up_i) for the SwiGLU epilogue
  if ((rc = matrix_alloc(&W.gu, q, 2 * st->F, st->H, st->stream, false))) return rc;
  if ((rc = matrix_repack(&W.gu, src + L.off[6], q, st->F, 0, 2, st->stream))) return rc;
  if ((rc = matrix_repack(&W.gu, src + L.off[7], q, st->F, 1, 2, st->stream))) return rc;
  if ((rc = matrix_alloc(&W.down, q, st->H, st->F, st->stream, false))) return rc;
  if ((rc = matrix_repack(&W.down, src + L.off[8], q, st->H, 0, 1, st->stream))) return rc;
  // norms: f16 bits -> f32 (exact)
  TN_CHECK_CUDA(cudaMalloc(&W.attn_norm, align256(st->H * sizeof(float))));
  TN_CHECK_CUDA(cudaMalloc(&W.ffn_norm, align256(st->H * sizeof(float))));
  if ((rc = hop_decode((const uint16_t*)(src + L.off[0]), st->H, W.attn_norm, st->stream))) return rc;
  if ((rc = hop_decode((const uint16_t*)(src + L.off[5]), st->H, W.ffn_norm, st->stream))) return rc;
  // the staging buffer is reused by the next layer: finish this one first
  TN_CHECK_CUDA(cudaStreamSynchronize(st->stream));
  st->weight_bytes += W.qkv.bytes + W.o.bytes + W.gu.bytes + W.down.bytes + 2 * align256(st->H * 4);
  st->packed_bytes += L.total;
  return TN_OK;
}

static int init_impl(const tn_stage_spec* sp, tn_stage* st) {
  TN_REQUIRE(sp->abi_version == TN_ABI_VERSION, TN_EINVAL, "abi_version %u != %d", sp->abi_version,
             TN_ABI_VERSION);
  TN_REQUIRE(sp->hidden_dim > 0 && sp->n_heads > 0 && sp->n_kv_heads > 0 && sp->vocab > 0, TN_EINVAL,
             "dims must be positive");
  TN_REQUIRE(sp->layer_hi >= sp->layer_lo && sp->n_layers == sp->layer_hi - sp->layer_lo, TN_EINVAL,
             "n_layers (%d) != layer_hi - layer_lo (%d)", sp->n_layers, sp->layer_hi - sp->layer_lo);
  TN_REQUIRE(sp->n_layers == 0 || sp->layers, TN_EINVAL, "layers missing");
  st->device = sp->device;
  st->H = sp->hidden_dim;
  st->nH = sp->n_heads;
  st->nKV = sp->n_kv_heads;
  st->hd = st->H / st->nH;
  st->qDim = st->nH * st->hd;
  st->kvDim = st->nKV * st->hd;
  st->F = sp->ffn_dim ? sp->ffn_dim : round_ffn(st->H);
  st->V = sp->vocab;
  st->theta = sp->rope_theta;
  st->lo = sp->layer_lo;
  st->hi = sp->layer_hi;
  st->nL = sp->n_layers;
  st->first = sp->is_first != 0;
  st->last = sp->is_last != 0;
  st->max_ctx = sp->max_ctx > 0 ? sp->max_ctx : 4096;
  st->max_seqs = sp->max_seqs > 0 ? sp->max_seqs : 16;
  st->max_T = sp->max_tokens_per_step > 0 ? sp->max_tokens_per_step : 512;
  st->flags = sp->flags;
  if (sp->kv_page_tokens) {
    const int pt = sp->kv_page_tokens;
    TN_REQUIRE(pt >= 16 && pt <= 4096 && (pt & (pt - 1)) == 0, TN_EINVAL,
               "kv_page_tokens %d: a power of two in [16, 4096]", pt);
    st->page_tokens = pt;
    while ((1 << st->page_shift) < pt) st->page_shift++;
    st->max_pages = (st->max_ctx + pt - 1) / pt;
    TN_REQUIRE(st->max_pages + 1 <= kAttnMaxPages, TN_EINVAL,
               "max_ctx %d needs %d pages of %d positions (at most %d)", st->max_ctx, st->max_pages, pt,
               kAttnMaxPages - 1);
    const int64_t dflt = (int64_t)st->max_seqs * st->max_pages;
    const int64_t np = sp->kv_pages > 0 ? sp->kv_pages : dflt;
    TN_REQUIRE(np <= (1 << 30), TN_EINVAL, "kv_pages %lld", (long long)np);
    st->n_pages = (int)np;
  } else {
    TN_REQUIRE(sp->kv_pages == 0, TN_EINVAL, "kv_pages without kv_page_tokens");
  }
  st->kv_type = (sp->flags & TN_FLAG_KV_F8) ? KV_F8 : ((sp->flags & TN_FLAG_KV_F16) ? KV_F16 : KV_F32);
  TN_REQUIRE(!((sp->flags & TN_FLAG_KV_F8) && (sp->flags & TN_FLAG_KV_F16)), TN_EINVAL,
             "TN_FLAG_KV_F16 and TN_FLAG_KV_F8 exclude each other");
  TN_REQUIRE(st->hd == 32 || st->hd == 64 || st->hd == 128, TN_EUNSUPPORTED,
             "head_dim %d unsupported (32, 64, 128)", st->hd);
  TN_REQUIRE(st->nH % st->nKV == 0 && (st->nH / st->nKV) <= 16 &&
                 ((st->nH / st->nKV) & (st->nH / st->nKV - 1)) == 0,
             TN_EUNSUPPORTED, "n_heads / n_kv_heads must be a power of two <= 16");
  TN_REQUIRE(st->F > 0 && st->F <= 32768 && st->H <= 32768, TN_EUNSUPPORTED, "dims above 32768");
  TN_REQUIRE(!st->first || sp->embed, TN_EINVAL, "first stage needs weights.embed");
  TN_REQUIRE(!st->last || (sp->norm && sp->lm_head), TN_EINVAL, "last stage needs weights.norm and lm_head");

  TN_ENTER_DEVICE(st->device);
  TN_CHECK_CUDA(cudaStreamCreateWithFlags(&st->stream, cudaStreamNonBlocking));

  // staging for host weights
  uint64_t stage_bytes = 0;
  for (int i = 0; i < st->nL; i++) {
    LayerLayout L;
    if (layer_layout(st->H, st->nH, st->nKV, sp->ffn_dim, sp->layers[i].quant, &L))
      stage_bytes = std::max<uint64_t>(stage_bytes, L.total);
  }
  const uint64_t embed_bytes = st->first ? quant_bytes((uint64_t)st->V * st->H, sp->embed_quant) : 0;
  const uint64_t head_bytes = st->last ? quant_bytes((uint64_t)st->V * st->H, sp->lm_head_quant) : 0;
  TN_REQUIRE(!st->first || (embed_bytes && sp->embed_len >= embed_bytes), TN_EINVAL,
             "embed: quant %d, %llu bytes given, %llu needed", sp->embed_quant,
             (unsigned long long)sp->embed_len, (unsigned long long)embed_bytes);
  TN_REQUIRE(!st->last || (head_bytes && sp->lm_head_len >= head_bytes), TN_EINVAL,
             "lm_head: quant %d, %llu bytes given, %llu needed", sp->lm_head_quant,
             (unsigned long long)sp->lm_head_len, (unsigned long long)head_bytes);
  TN_REQUIRE(!st->last || sp->norm_len >= (uint64_t)st->H * 2, TN_EINVAL, "norm: need %d f16 values", st->H);
  stage_bytes = std::max(stage_bytes, std::max(embed_bytes, head_bytes));
  uint8_t* staging = nullptr;
  if (!sp->weights_on_device && stage_bytes) {
    cudaError_t e = cudaMalloc(&staging, stage_bytes);
    TN_REQUIRE(e == cudaSuccess, TN_ENOMEM, "staging cudaMalloc(%llu): %s", (unsigned long long)stage_bytes,
               cudaGetErrorString(e));
  }
  struct StagingFree {
    uint8_t* p;
    ~StagingFree() {
      if (p) cudaFree(p);
    }
  } staging_free{staging};

  int rc;
  st->layers.resize(st->nL);
  for (int i = 0; i < st->nL; i++)
    if ((rc = load_layer(st, sp, i, staging))) return rc;
  const uint8_t* src = nullptr;
  if (st->first) {
    if ((rc = stage_src(sp, sp->embed, embed_bytes, staging, st->stream, &src))) return rc;
    if ((rc = matrix_alloc(&st->embed, sp->embed_quant, st->V, st->H, st->stream, false))) return rc;
    if ((rc = matrix_repack(&st->embed, src, sp->embed_quant, st->V, 0, 1, st->stream))) return rc;
    TN_CHECK_CUDA(cudaStreamSynchronize(st->stream));
    st->weight_bytes += st->embed.bytes;
    st->packed_bytes += embed_bytes;
  }
  if (st->last) {
    if ((rc = stage_src(sp, sp->lm_head, head_bytes, staging, st->stream, &src))) return rc;
    if ((rc = matrix_alloc(&st->lm_head, sp->lm_head_quant, st->V, st->H, st->stream, false))) return rc;
    if ((rc = matrix_repack(&st->lm_head, src, sp->lm_head_quant, st->V, 0, 1, st->stream))) return rc;
    TN_CHECK_CUDA(cudaStreamSynchronize(st->stream));
    if ((rc = stage_src(sp, sp->norm, (uint64_t)st->H * 2, staging, st->stream, &src))) return rc;
    TN_CHECK_CUDA(cudaMalloc(&st->final_norm, align256(st->H * sizeof(float))));
    if ((rc = hop_decode((const uint16_t*)src, st->H, st->final_norm, st->stream))) return rc;
    TN_CHECK_CUDA(cudaStreamSynchronize(st->stream));
    st->weight_bytes += st->lm_head.bytes;
    st->packed_bytes += head_bytes + (uint64_t)st->H * 2;
  }

  // KV arena, K and V: [slot][layer][kv_head][max_ctx][head_dim], or the
  // page pool [page][layer][kv_head][page_tokens][head_dim]
  const int ctx_rows = st->page_tokens ? st->page_tokens : st->max_ctx;
  st->kvh_stride = (size_t)ctx_rows * st->hd;
  st->layer_stride = st->kvh_stride * st->nKV;
  st->slot_stride = st->layer_stride * std::max(1, st->nL);
  const size_t kv_elems = st->slot_stride * (st->page_tokens ? st->n_pages : st->max_seqs);
  if (st->nL > 0) {
    const size_t eb = kv_elem_bytes(st->kv_type);
    cudaError_t e1 = cudaMalloc(&st->kc, kv_elems * eb);
    cudaError_t e2 = e1 == cudaSuccess ? cudaMalloc(&st->vc, kv_elems * eb) : e1;
    TN_REQUIRE(e1 == cudaSuccess && e2 == cudaSuccess, TN_ENOMEM,
               "KV arena of 2 x %zu bytes (%d %s of %d rows): %s", kv_elems * eb,
               st->page_tokens ? st->n_pages : st->max_seqs, st->page_tokens ? "pages" : "slots", ctx_rows,
               cudaGetErrorString(e1 != cudaSuccess ? e1 : e2));
    st->kv_bytes = 2 * kv_elems * eb;
  }
  st->kvmap.slot_stride = st->slot_stride;
  st->kvmap.kvh_stride = st->kvh_stride;
  if (st->page_tokens) {
    TN_CHECK_CUDA(cudaHostAlloc((void**)&st->h_pages, (size_t)st->max_seqs * st->max_pages * sizeof(int),
                                cudaHostAllocDefault));
    if ((rc = dalloc(st, &st->d_pages, (size_t)st->max_seqs * st->max_pages))) return rc;
    st->kvmap.pages = st->d_pages;
    st->kvmap.max_pages = st->max_pages;
    st->kvmap.shift = st->page_shift;
    for (int i = st->n_pages - 1; i >= 0; i--) st->free_pages.push_back(i);
    st->seq_pages.assign(st->max_seqs, 0);
  }

  // activations for max_T rows
  const int T = st->max_T, nout = std::max(1, std::min(st->max_T, st->max_seqs));
  if ((rc = dalloc(st, &st->h, (size_t)T * st->H))) return rc;
  if ((rc = dalloc(st, &st->xn, (size_t)T * st->H))) return rc;
  if ((rc = dalloc(st, &st->qkv, (size_t)T * (st->qDim + 2 * st->kvDim)))) return rc;
  if ((rc = dalloc(st, &st->q, (size_t)T * st->qDim))) return rc;
  if ((rc = dalloc(st, &st->att, (size_t)T * st->qDim))) return rc;
  if ((rc = dalloc(st, &st->act, (size_t)T * st->F))) return rc;
  if (st->last && (rc = dalloc(st, &st->logits, (size_t)nout * st->V))) return rc;
  if ((rc = dalloc(st, &st->hid_in, (size_t)T * st->H))) return rc;
  if ((rc = dalloc(st, &st->hid_out, (size_t)T * st->H))) return rc;
  if ((rc = dalloc(st, &st->ids, (size_t)T))) return rc;
  if ((rc = dalloc(st, &st->tok_out, (size_t)T))) return rc;
  if ((rc = dalloc(st, &st->err, 1))) return rc;
  if ((rc = dalloc(st, &st->kerr, 1))) return rc;
  if ((rc = dalloc(st, &st->cs, (size_t)T * (st->hd / 2)))) return rc;
  if (T >= kGemmMinTokens) {
    // the widest input of any matrix the GEMM may take: hidden, attention output or FFN activation
    const int kmax = std::max(st->H, std::max(st->qDim, st->F));
    st->gemm_ws_bytes = gemm_scratch_bytes(T, kmax);
    if ((rc = dalloc(st, (char**)&st->gemm_ws, st->gemm_ws_bytes))) return rc;
  }
  // one cross-CTA workspace for every decode matvec of the stage (its
  // launches are ordered on the stage stream)
  {
    size_t wsf = 0, cnti = 0;
    std::vector<Matrix*> ms;
    for (auto& L : st->layers) ms.insert(ms.end(), {&L.qkv, &L.o, &L.gu, &L.down});
    if (st->first) ms.push_back(&st->embed);
    if (st->last) ms.push_back(&st->lm_head);
    for (Matrix* m : ms) {
      wsf = std::max(wsf, m->ws_floats);
      cnti = std::max(cnti, m->cnt_ints);
    }
    float* ws = nullptr;
    int* cnt = nullptr;
    if (wsf && (rc = dalloc(st, &ws, wsf))) return rc;
    if (cnti && (rc = dalloc(st, &cnt, cnti))) return rc;
    for (Matrix* m : ms)
      if (m->ws_floats) {
        m->ws = ws;
        m->cnt = cnt;
      }
  }
  // split-attention workspace: the largest over every row count of a step
  {
    size_t wsf = 0, cnti = 0;
    for (int t = 1; t <= T; t++) {
      const AttnPlan p = attn_plan(t, st->nH, st->nKV, st->hd, st->max_ctx, st->kv_type);
      wsf = std::max(wsf, p.ws_floats);
      cnti = std::max(cnti, p.cnt_ints);
    }
    st->attn_ws_floats = wsf;
    st->attn_cnt_ints = cnti;
    if (wsf && (rc = dalloc(st, &st->attn_ws, wsf))) return rc;
    if (cnti && (rc = dalloc(st, &st->attn_cnt, cnti))) return rc;
  }
  if ((rc = dalloc(st, &st->freq, (size_t)(st->hd / 2)))) return rc;
  // RoPE frequencies theta^(-2i/hd) in double (web/inference-worker.js:533)
  std::vector<double> freq(st->hd / 2);
  for (int i = 0; i < st->hd / 2; i++) freq[i] = std::pow(st->theta, (double)(-2 * i) / st->hd);
  TN_CHECK_CUDA(cudaMemcpyAsync(st->freq, freq.data(), freq.size() * sizeof(double), cudaMemcpyHostToDevice,
                                st->stream));
  // control block
  st->ctl_outrows_off = align256((size_t)T * sizeof(RowInfo));
  st->ctl_params_off = st->ctl_outrows_off + align256((size_t)T * sizeof(int));
  st->ctl_bytes = st->ctl_params_off + align256((size_t)T * 3 * sizeof(double));
  if ((rc = dalloc(st, &st->d_ctl, st->ctl_bytes))) return rc;
  for (int i = 0; i < CTL_RING; i++) {
    TN_CHECK_CUDA(cudaHostAlloc((void**)&st->h_ctl[i], st->ctl_bytes, cudaHostAllocDefault));
    TN_CHECK_CUDA(cudaEventCreateWithFlags(&st->ctl_ev[i], cudaEventDisableTiming));
  }
  TN_CHECK_CUDA(cudaHostAlloc(&st->h_in, (size_t)T * st->H * sizeof(uint16_t) + 256, cudaHostAllocDefault));
  TN_CHECK_CUDA(cudaHostAlloc(&st->h_out, (size_t)T * st->H * sizeof(uint16_t) + 256, cudaHostAllocDefault));
  if (st->flags & TN_FLAG_PROFILE) {
    st->prof = true;
    const int pairs = st->nL * 12 + 16;
    st->ev.resize(2 * pairs);
    st->ev_class.resize(pairs);
    for (auto& e : st->ev) TN_CHECK_CUDA(cudaEventCreate(&e));
  }
  st->kv_len.assign(st->max_seqs, 0);
  for (int i = st->max_seqs - 1; i >= 0; i--) st->free_slots.push_back(i);
  TN_CHECK_CUDA(cudaStreamSynchronize(st->stream));
  return TN_OK;
}

// an event record that survives stream capture as a graph node
static void record_event(cudaEvent_t e, cudaStream_t s) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(s, &cs);
  if (cs == cudaStreamCaptureStatusActive) cudaEventRecordWithFlags(e, s, cudaEventRecordExternal);
  else cudaEventRecord(e, s);
}

// record the begin event of a timed launch (no-op unless profiling)
static int prof_begin(tn_stage* st, cudaStream_t s, int cls) {
  if (!st->prof || st->ev_used * 2 + 1 >= (int)st->ev.size()) return -1;
  const int i = st->ev_used++;
  st->ev_class[i] = cls;
  record_event(st->ev[2 * i], s);
  return i;
}
static void prof_end(tn_stage* st, cudaStream_t s, int i) {
  if (i >= 0) record_event(st->ev[2 * i + 1], s);
}
// fold the finished step's event pairs into the per-class totals (stream synchronised)
static void prof_collect(tn_stage* st) {
  if (!st->prof) return;
  for (int i = 0; i < st->ev_used; i++) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, st->ev[2 * i], st->ev[2 * i + 1]) == cudaSuccess) {
      st->prof_ms[st->ev_class[i]] += ms;
      st->prof_launches[st->ev_class[i]] += 1;
    }
  }
  st->ev_used = 0;
}

// launch `expr` (which starts `nk` kernels) as one timed unit of class `cls`
#define TN_STEP_LAUNCH(cls, nk, expr)        \
  do {                                       \
    const int pi_ = prof_begin(st, s, cls);  \
    if ((rc = (expr))) return rc;            \
    prof_end(st, s, pi_);                    \
    st->step_launches += (nk);               \
  } while (0)

// After the stage's work on s has finished: TN_ETIMEOUT if a kernel's
// bounded wait gave up since the last check (its step's outputs are invalid),
// with the split-K arrival counters and workspaces zeroed so that the next
// step starts clean; TN_OK otherwise.
static int recover_kernel_error(tn_stage* st, cudaStream_t s) {
  int kerr = 0;
  TN_CHECK_CUDA(cudaMemcpy(&kerr, st->kerr, sizeof(int), cudaMemcpyDeviceToHost));
  if (!kerr) return TN_OK;
  TN_CHECK_CUDA(cudaMemset(st->kerr, 0, sizeof(int)));
  // a launch that gave up may have left split-K arrival counts behind
  for (LayerW& L : st->layers) {
    matrix_reset_counters(L.qkv, s);
    matrix_reset_counters(L.o, s);
    matrix_reset_counters(L.gu, s);
    matrix_reset_counters(L.down, s);
  }
  matrix_reset_counters(st->lm_head, s);
  if (st->gemm_ws) TN_CHECK_CUDA(cudaMemsetAsync(st->gemm_ws, 0, st->gemm_ws_bytes, s));
  if (st->attn_cnt) TN_CHECK_CUDA(cudaMemsetAsync(st->attn_cnt, 0, st->attn_cnt_ints * sizeof(int), s));
  TN_CHECK_CUDA(cudaStreamSynchronize(s));
  set_error("a kernel's bounded wait on its copy pipeline gave up; the step's outputs are invalid");
  return TN_ETIMEOUT;
}

// the layer stack for T rows already described by the control block
// kernels one matvec / matvec_dec call over T tokens launches (the GEMM: its
// activation prep and the GEMM; the decode matvec: one per 4 tokens)
static int mv_launches(const tn_stage* st, const Matrix& m, int T) {
  if (m.kind != MK_Q4 && m.kind != MK_Q8) return 1;
  return gemm_ok(m, T) && st->gemm_ws ? 2 : (T + 3) / 4;
}

static int run_step(tn_stage* st, int T, int n_out, int input_kind, cudaStream_t s) {
  const RowInfo* rows = (const RowInfo*)st->d_ctl;
  const int* outrows = (const int*)(st->d_ctl + st->ctl_outrows_off);
  const double* params = (const double*)(st->d_ctl + st->ctl_params_off);
  const int H = st->H, ldqkv = st->qDim + 2 * st->kvDim;
  int rc;
  st->ev_used = 0;
  st->step_launches = 0;
  auto mvl = [&](const Matrix& m, int rows) { return mv_launches(st, m, rows); };
  if (input_kind == IN_IDS)
    TN_STEP_LAUNCH(TN_PROF_OTHER, 1, embed_rows(st->embed, st->ids, T, st->h, H, st->err, s));
  else
    TN_STEP_LAUNCH(TN_PROF_OTHER, 1, hop_decode(st->hid_in, (uint64_t)T * H, st->h, s));
  TN_STEP_LAUNCH(TN_PROF_ROPE_KV, 1, rope_table(rows, st->freq, st->hd / 2, T, st->cs, s));
  const AttnPlan ap = attn_plan(T, st->nH, st->nKV, st->hd, st->max_ctx, st->kv_type, st->attn_ws_floats);
  const size_t eb = kv_elem_bytes(st->kv_type);
  for (int l = 0; l < st->nL; l++) {
    LayerW& L = st->layers[l];
    char* kc = st->kc + (size_t)l * st->layer_stride * eb;
    char* vc = st->vc + (size_t)l * st->layer_stride * eb;
    // decode-sized steps use the fused decode matvec (RMSNorm prologue,
    // RoPE + KV epilogue, programmatic dependent launches); other steps and
    // matrix formats it does not cover run the separate kernels
    const bool fuse = !(st->flags & TN_FLAG_NO_FUSED_DECODE);
    if (fuse && matvec_dec_ok(L.qkv, T)) {
      MvFuse f;
      f.norm_w = L.attn_norm;
      f.rinfo = rows;
      f.cs = st->cs;
      f.q_out = st->q;
      f.kc = kc;
      f.vc = vc;
      f.kv_type = st->kv_type;
      f.kv = st->kvmap;
      f.q_dim = st->qDim;
      f.kv_dim = st->kvDim;
      f.hd = st->hd;
      TN_STEP_LAUNCH(TN_PROF_MATVEC_QKV, mvl(L.qkv, T), matvec_dec(L.qkv, T, st->h, H, st->qkv, ldqkv, EPI_QKV_ROPE, f, st->kerr, s));
    } else {
      TN_STEP_LAUNCH(TN_PROF_NORM, 1, rmsnorm(st->h, H, nullptr, L.attn_norm, st->xn, H, H, T, s));
      TN_STEP_LAUNCH(TN_PROF_MATVEC_QKV, mvl(L.qkv, T), matvec(L.qkv, T, st->xn, H, st->qkv, ldqkv, EPI_STORE, st->kerr, st->gemm_ws, st->gemm_ws_bytes, s));
      TN_STEP_LAUNCH(TN_PROF_ROPE_KV, 1,
                     rope_kv(st->qkv, ldqkv, rows, st->cs, st->q, kc, vc, st->kv_type, st->kvmap, st->nH,
                             st->nKV, st->hd, T, s));
    }
    TN_STEP_LAUNCH(TN_PROF_ATTENTION, 1,
                   attention(st->q, st->qDim, kc, vc, st->kv_type, st->kvmap, rows, T, st->nH, st->nKV, st->hd, ap,
                             st->att, st->qDim, st->attn_ws, st->attn_cnt, s));
    if (fuse && matvec_dec_ok(L.o, T))
      TN_STEP_LAUNCH(TN_PROF_MATVEC_O, mvl(L.o, T), matvec_dec(L.o, T, st->att, st->qDim, st->h, H, EPI_RESID, MvFuse(), st->kerr, s));
    else
      TN_STEP_LAUNCH(TN_PROF_MATVEC_O, mvl(L.o, T), matvec(L.o, T, st->att, st->qDim, st->h, H, EPI_RESID, st->kerr, st->gemm_ws, st->gemm_ws_bytes, s));
    if (fuse && matvec_dec_ok(L.gu, T)) {
      MvFuse f;
      f.norm_w = L.ffn_norm;
      TN_STEP_LAUNCH(TN_PROF_MATVEC_GATE_UP, mvl(L.gu, T), matvec_dec(L.gu, T, st->h, H, st->act, st->F, EPI_SWIGLU, f, st->kerr, s));
    } else {
      TN_STEP_LAUNCH(TN_PROF_NORM, 1, rmsnorm(st->h, H, nullptr, L.ffn_norm, st->xn, H, H, T, s));
      TN_STEP_LAUNCH(TN_PROF_MATVEC_GATE_UP, mvl(L.gu, T), matvec(L.gu, T, st->xn, H, st->act, st->F, EPI_SWIGLU, st->kerr, st->gemm_ws, st->gemm_ws_bytes, s));
    }
    if (fuse && matvec_dec_ok(L.down, T))
      TN_STEP_LAUNCH(TN_PROF_MATVEC_DOWN, mvl(L.down, T), matvec_dec(L.down, T, st->act, st->F, st->h, H, EPI_RESID, MvFuse(), st->kerr, s));
    else
      TN_STEP_LAUNCH(TN_PROF_MATVEC_DOWN, mvl(L.down, T), matvec(L.down, T, st->act, st->F, st->h, H, EPI_RESID, st->kerr, st->gemm_ws, st->gemm_ws_bytes, s));
  }
  if (st->last) {
    if (!(st->flags & TN_FLAG_NO_FUSED_DECODE) && matvec_dec_ok(st->lm_head, n_out)) {
      MvFuse f;
      f.norm_w = st->final_norm;
      f.rowsel = outrows;
      TN_STEP_LAUNCH(TN_PROF_MATVEC_LM_HEAD, mvl(st->lm_head, n_out),
                     matvec_dec(st->lm_head, n_out, st->h, H, st->logits, st->V, EPI_STORE, f, st->kerr, s));
    } else {
      TN_STEP_LAUNCH(TN_PROF_NORM, 1, rmsnorm(st->h, H, outrows, st->final_norm, st->xn, H, H, n_out, s));
      TN_STEP_LAUNCH(TN_PROF_MATVEC_LM_HEAD, mvl(st->lm_head, n_out),
                     matvec(st->lm_head, n_out, st->xn, H, st->logits, st->V, EPI_STORE, st->kerr, st->gemm_ws, st->gemm_ws_bytes, s));
    }
    TN_STEP_LAUNCH(TN_PROF_OTHER, 1, sample_rows(st->logits, n_out, st->V, params, st->tok_out, s));
  } else {
    TN_STEP_LAUNCH(TN_PROF_OTHER, 1, hop_encode_rows(st->h, H, outrows, n_out, H, st->hid_out, s));
  }
  return TN_OK;
}

// run a step, through a cached CUDA graph when the shape is decode-like
static int launch_step(tn_stage* st, int T, int n_out, int input_kind, bool graphable, cudaStream_t s) {
  if (!graphable || (st->flags & TN_FLAG_NO_GRAPHS) || st->graphs_broken)
    return run_step(st, T, n_out, input_kind, s);
  const auto key = std::make_tuple(T, n_out, input_kind);
  auto it = st->graphs.find(key);
  if (it == st->graphs.end()) {
    cudaGraph_t g = nullptr;
    TN_CHECK_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    const int rc = run_step(st, T, n_out, input_kind, s);
    const cudaError_t ce = cudaStreamEndCapture(s, &g);
    if (rc) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    if (ce != cudaSuccess || !g) {
      cudaGetLastError();
      st->graphs_broken = true;
      return run_step(st, T, n_out, input_kind, s);
    }
    GraphEntry ge;
    ge.n_ev = st->ev_used;
    ge.n_launch = st->step_launches;
    const cudaError_t ie = cudaGraphInstantiate(&ge.exec, g, 0);
    cudaGraphDestroy(g);
    if (ie != cudaSuccess) {
      cudaGetLastError();
      st->graphs_broken = true;
      return run_step(st, T, n_out, input_kind, s);
    }
    it = st->graphs.emplace(key, ge).first;
  }
  TN_CHECK_CUDA(cudaGraphLaunch(it->second.exec, s));
  st->ev_used = it->second.n_ev;
  st->step_launches = it->second.n_launch;
  return TN_OK;
}

// next pinned control buffer (waits until its previous upload has been consumed)
static char* next_ctl(tn_stage* st, int* idx) {
  const int i = st->ctl_pos;
  st->ctl_pos = (st->ctl_pos + 1) % CTL_RING;
  cudaEventSynchronize(st->ctl_ev[i]);
  *idx = i;
  return st->h_ctl[i];
}

static int upload_ctl(tn_stage* st, int idx, cudaStream_t s) {
  TN_CHECK_CUDA(cudaMemcpyAsync(st->d_ctl, st->h_ctl[idx], st->ctl_bytes, cudaMemcpyHostToDevice, s));
  TN_CHECK_CUDA(cudaEventRecord(st->ctl_ev[idx], s));
  return TN_OK;
}

// a freed sequence slot's pages go back to the pool
static void release_pages(tn_stage* st, int slot) {
  if (!st->page_tokens) return;
  for (int j = st->seq_pages[slot] - 1; j >= 0; j--)
    st->free_pages.push_back(st->h_pages[(size_t)slot * st->max_pages + j]);
  st->seq_pages[slot] = 0;
}

// slots for the requests' sequences and pages for their new rows; new slots
// and pages are released again on failure
struct SlotTxn {
  tn_stage* st;
  std::vector<uint64_t> created;
  std::vector<std::pair<int, int>> taken;  // (slot, page) in order
  bool committed = false;
  ~SlotTxn() {
    if (committed) return;
    for (auto it = taken.rbegin(); it != taken.rend(); ++it) {
      st->seq_pages[it->first]--;
      st->free_pages.push_back(it->second);
    }
    for (uint64_t id : created) {
      auto it = st->seq_slot.find(id);
      if (it != st->seq_slot.end()) {
        st->kv_len[it->second] = 0;
        st->free_slots.push_back(it->second);
        st->seq_slot.erase(it);
      }
    }
  }
  // pages for rows [0, rows) of the slot's sequence, their page-table
  // entries copied to the device on s ahead of the step's kernels.  (The
  // copy reads the pinned host entries when it runs; an entry changes only
  // when its slot is reused, after tn_stage_free_seq, which callers may not
  // issue while that sequence's steps are in flight.)
  int grow(int slot, int rows, cudaStream_t s) {
    if (!st->page_tokens) return TN_OK;
    const int need = (rows + st->page_tokens - 1) >> st->page_shift, j0 = st->seq_pages[slot];
    if (need <= j0) return TN_OK;
    TN_REQUIRE((int)st->free_pages.size() >= need - j0, TN_ECAPACITY,
               "KV page pool exhausted: %d pages needed, %zu of %d free", need - j0, st->free_pages.size(),
               st->n_pages);
    int* row = st->h_pages + (size_t)slot * st->max_pages;
    for (int j = j0; j < need; j++) {
      row[j] = st->free_pages.back();
      st->free_pages.pop_back();
      st->seq_pages[slot]++;
      taken.emplace_back(slot, row[j]);
    }
    TN_CHECK_CUDA(cudaMemcpyAsync(st->d_pages + (size_t)slot * st->max_pages + j0, row + j0,
                                  (size_t)(need - j0) * sizeof(int), cudaMemcpyHostToDevice, s));
    return TN_OK;
  }
  int get(uint64_t id, int* slot) {
    auto it = st->seq_slot.find(id);
    if (it != st->seq_slot.end()) {
      *slot = it->second;
      return TN_OK;
    }
    TN_REQUIRE(!st->free_slots.empty(), TN_ECAPACITY, "all %d sequence slots in use (max_seqs)", st->max_seqs);
    *slot = st->free_slots.back();
    st->free_slots.pop_back();
    st->kv_len[*slot] = 0;
    st->seq_slot[id] = *slot;
    created.push_back(id);
    return TN_OK;
  }
};

double sample_uniform(uint64_t seed, uint64_t row) {
  const uint64_t h = mix64(seed ^ mix64(row + 0x632BE59BD9B4E019ull));
  return (double)(h >> 11) * (1.0 / 9007199254740992.0);
}

static int forward_impl(tn_stage* st, const tn_fwd_req* reqs, int n, tn_fwd_out* outs) {
  TN_REQUIRE(reqs && outs && n > 0, TN_EINVAL, "forward: no requests");
  TN_REQUIRE(n <= st->max_seqs, TN_ECAPACITY, "forward: %d sequences in one batch > max_seqs %d", n, st->max_seqs);
  const int H = st->H;
  {
    std::unordered_set<uint64_t> seen;
    for (int i = 0; i < n; i++) {
      const tn_fwd_req& r = reqs[i];
      TN_REQUIRE(seen.insert(r.seq_id).second, TN_EINVAL, "forward: seq_id %llu twice in one batch",
                 (unsigned long long)r.seq_id);
      TN_REQUIRE(r.n_tokens >= 1, TN_EINVAL, "forward: n_tokens must be >= 1");
      TN_REQUIRE(r.hop_mode == TN_HOP_LAST || r.hop_mode == TN_HOP_ALL, TN_EINVAL, "forward: bad hop_mode");
      if (st->first) {
        TN_REQUIRE(r.token_ids, TN_ESTATE, "first stage: token_ids required");
        for (int p = 0; p < r.n_tokens; p++)
          TN_REQUIRE(r.token_ids[p] >= 0 && r.token_ids[p] < st->V, TN_EINVAL,
                     "token id %d outside [0, %d)", r.token_ids[p], st->V);
      } else {
        TN_REQUIRE(r.hidden, TN_ESTATE, "stage %d: hidden input required", st->lo);
      }
      if (!st->last) {
        const int need = r.hop_mode == TN_HOP_ALL ? r.n_tokens : 1;
        TN_REQUIRE(outs[i].hidden && outs[i].hidden_cap_tokens >= need, TN_EINVAL,
                   "forward: output buffer for %d tokens needed", need);
      }
    }
  }
  SlotTxn txn{st};
  std::vector<int> slot(n);
  int rc;
  for (int i = 0; i < n; i++) {
    if ((rc = txn.get(reqs[i].seq_id, &slot[i]))) return rc;
    TN_REQUIRE(st->kv_len[slot[i]] + reqs[i].n_tokens <= st->max_ctx, TN_ECAPACITY,
               "seq %llu: %d cached + %d new rows > max_ctx %d", (unsigned long long)reqs[i].seq_id,
               st->kv_len[slot[i]], reqs[i].n_tokens, st->max_ctx);
    if ((rc = txn.grow(slot[i], st->kv_len[slot[i]] + reqs[i].n_tokens, st->stream))) return rc;
  }
  // global row list
  struct RowRef {
    int req, p;
  };
  std::vector<RowRef> refs;
  std::vector<RowInfo> rows;
  for (int i = 0; i < n; i++)
    for (int p = 0; p < reqs[i].n_tokens; p++) {
      const int kvi = st->kv_len[slot[i]] + p;
      rows.push_back(RowInfo{slot[i], reqs[i].token_pos + p, kvi, kvi + 1});
      refs.push_back(RowRef{i, p});
    }
  const int R = (int)rows.size();
  auto is_out = [&](int r) {
    const tn_fwd_req& q = reqs[refs[r].req];
    const bool last_row = refs[r].p == q.n_tokens - 1;
    return st->last ? last_row : (q.hop_mode == TN_HOP_ALL || last_row);
  };
  const bool decode_shape = R == n;  // one row per sequence
  cudaStream_t s = st->stream;
  for (int r0 = 0; r0 < R; r0 += st->max_T) {
    const int T = std::min(st->max_T, R - r0);
    int ci;
    char* ctl = next_ctl(st, &ci);
    RowInfo* crow = (RowInfo*)ctl;
    int* cout = (int*)(ctl + st->ctl_outrows_off);
    double* cpar = (double*)(ctl + st->ctl_params_off);
    std::vector<int> out_global;
    for (int k = 0; k < T; k++) {
      crow[k] = rows[r0 + k];
      if (is_out(r0 + k)) {
        const int o = (int)out_global.size();
        const tn_fwd_req& q = reqs[refs[r0 + k].req];
        cout[o] = k;
        cpar[3 * o] = q.temperature;
        cpar[3 * o + 1] = q.top_p;
        cpar[3 * o + 2] = sample_uniform(q.rng_seed, (uint64_t)(uint32_t)(q.token_pos + refs[r0 + k].p));
        out_global.push_back(r0 + k);
      }
    }
    const int n_out = (int)out_global.size();
    if ((rc = upload_ctl(st, ci, s))) return rc;
    if (st->first) {
      int* hin = (int*)st->h_in;
      for (int k = 0; k < T; k++) hin[k] = reqs[refs[r0 + k].req].token_ids[refs[r0 + k].p];
      TN_CHECK_CUDA(cudaMemcpyAsync(st->ids, hin, (size_t)T * sizeof(int), cudaMemcpyHostToDevice, s));
    } else {
      uint16_t* hin = (uint16_t*)st->h_in;
      for (int k = 0; k < T; k++)
        std::memcpy(hin + (size_t)k * H, reqs[refs[r0 + k].req].hidden + (size_t)refs[r0 + k].p * H,
                    (size_t)H * sizeof(uint16_t));
      TN_CHECK_CUDA(cudaMemcpyAsync(st->hid_in, hin, (size_t)T * H * sizeof(uint16_t), cudaMemcpyHostToDevice, s));
    }
    if (n_out == 0) {
      if ((rc = run_step(st, T, 0, st->first ? IN_IDS : IN_HIDDEN, s))) return rc;
      if (st->prof) {
        TN_CHECK_CUDA(cudaStreamSynchronize(s));
        prof_collect(st);
      }
      continue;
    }
    if ((rc = launch_step(st, T, n_out, st->first ? IN_IDS : IN_HIDDEN, decode_shape, s))) return rc;
    if (st->last)
      TN_CHECK_CUDA(cudaMemcpyAsync(st->h_out, st->tok_out, (size_t)n_out * sizeof(int), cudaMemcpyDeviceToHost, s));
    else
      TN_CHECK_CUDA(cudaMemcpyAsync(st->h_out, st->hid_out, (size_t)n_out * H * sizeof(uint16_t),
                                    cudaMemcpyDeviceToHost, s));
    TN_CHECK_CUDA(cudaStreamSynchronize(s));
    prof_collect(st);
    for (int o = 0; o < n_out; o++) {
      const RowRef& rr = refs[out_global[o]];
      tn_fwd_out& out = outs[rr.req];
      if (st->last) {
        out.token_id = ((const int*)st->h_out)[o];
      } else {
        const tn_fwd_req& q = reqs[rr.req];
        const int dst = q.hop_mode == TN_HOP_ALL ? rr.p : 0;
        std::memcpy(out.hidden + (size_t)dst * H, (const uint16_t*)st->h_out + (size_t)o * H,
                    (size_t)H * sizeof(uint16_t));
        out.n_hidden_tokens = q.hop_mode == TN_HOP_ALL ? q.n_tokens : 1;
      }
    }
  }
  TN_CHECK_CUDA(cudaStreamSynchronize(s));
  if ((rc = recover_kernel_error(st, s))) return rc;
  for (int i = 0; i < n; i++) {
    st->kv_len[slot[i]] += reqs[i].n_tokens;
    if (st->last) outs[i].n_hidden_tokens = 0;
  }
  txn.committed = true;
  return TN_OK;
}

static int step_async_impl(tn_stage* st, const tn_step_desc* d, cudaStream_t s) {
  const int n = d->n_seqs;
  TN_REQUIRE(n >= 1 && n <= std::min(st->max_T, st->max_seqs), TN_ECAPACITY,
             "step: %d sequences (max %d)", n, std::min(st->max_T, st->max_seqs));
  TN_REQUIRE(d->seq_ids && d->token_pos, TN_EINVAL, "step: seq_ids and token_pos required");
  TN_REQUIRE(st->first ? d->d_token_ids != nullptr : d->d_hidden_in != nullptr, TN_ESTATE,
             "step: input pointer for this stage role missing");
  TN_REQUIRE(st->last ? d->d_token_out != nullptr : d->d_hidden_out != nullptr, TN_ESTATE,
             "step: output pointer for this stage role missing");
  SlotTxn txn{st};
  std::vector<int> slot(n);
  for (int i = 0; i < n; i++) {
    int rc = txn.get(d->seq_ids[i], &slot[i]);
    if (rc) return rc;
    TN_REQUIRE(st->kv_len[slot[i]] + 1 <= st->max_ctx, TN_ECAPACITY, "seq %llu: max_ctx %d reached",
               (unsigned long long)d->seq_ids[i], st->max_ctx);
    for (int j = 0; j < i; j++)
      TN_REQUIRE(slot[j] != slot[i], TN_EINVAL, "step: seq_id twice in one step");
    if ((rc = txn.grow(slot[i], st->kv_len[slot[i]] + 1, s))) return rc;
  }
  int ci;
  char* ctl = next_ctl(st, &ci);
  RowInfo* crow = (RowInfo*)ctl;
  int* cout = (int*)(ctl + st->ctl_outrows_off);
  double* cpar = (double*)(ctl + st->ctl_params_off);
  for (int i = 0; i < n; i++) {
    const int kvi = st->kv_len[slot[i]];
    crow[i] = RowInfo{slot[i], d->token_pos[i], kvi, kvi + 1};
    cout[i] = i;
    cpar[3 * i] = d->temperature;
    cpar[3 * i + 1] = d->top_p;
    cpar[3 * i + 2] = sample_uniform(d->rng_seed, (uint64_t)(uint32_t)d->token_pos[i]);
  }
  int rc;
  if ((rc = upload_ctl(st, ci, s))) return rc;
  if (st->first)
    TN_CHECK_CUDA(cudaMemcpyAsync(st->ids, d->d_token_ids, (size_t)n * sizeof(int), cudaMemcpyDeviceToDevice, s));
  else
    TN_CHECK_CUDA(cudaMemcpyAsync(st->hid_in, d->d_hidden_in, (size_t)n * st->H * sizeof(uint16_t),
                                  cudaMemcpyDeviceToDevice, s));
  if ((rc = launch_step(st, n, n, st->first ? IN_IDS : IN_HIDDEN, true, s))) return rc;
  if (st->last)
    TN_CHECK_CUDA(cudaMemcpyAsync(d->d_token_out, st->tok_out, (size_t)n * sizeof(int), cudaMemcpyDeviceToDevice, s));
  else
    TN_CHECK_CUDA(cudaMemcpyAsync(d->d_hidden_out, st->hid_out, (size_t)n * st->H * sizeof(uint16_t),
                                  cudaMemcpyDeviceToDevice, s));
  for (int i = 0; i < n; i++) st->kv_len[slot[i]] += 1;
  txn.committed = true;
  return TN_OK;
}

}  // namespace tn

// ===================================================================== C ABI
extern "C" const char* tn_last_error(void) { return g_err; }
extern "C" int tn_abi_version(void) { return TN_ABI_VERSION; }

extern "C" int tn_stage_init(const tn_stage_spec* spec, tn_stage** out) {
  clear_error();
  TN_REQUIRE(spec && out, TN_EINVAL, "tn_stage_init: null argument");
  *out = nullptr;
  tn_stage* st = new (std::nothrow) tn_stage();
  TN_REQUIRE(st, TN_ENOMEM, "tn_stage_init: out of host memory");
  const int rc = init_impl(spec, st);
  if (rc) {
    std::string msg = tn_last_error();
    {
      DevGuard g(st->device);
      delete st;
    }
    set_error("%s", msg.c_str());
    return rc;
  }
  *out = st;
  return TN_OK;
}

extern "C" int tn_stage_forward_batch(tn_stage* st, const tn_fwd_req* reqs, int32_t n_reqs, tn_fwd_out* outs) {
  clear_error();
  TN_REQUIRE(st, TN_EINVAL, "null stage");
  std::lock_guard<std::mutex> lk(st->mu);
  TN_ENTER_DEVICE(st->device);
  return forward_impl(st, reqs, n_reqs, outs);
}

extern "C" int tn_stage_forward(tn_stage* st, const tn_fwd_req* req, tn_fwd_out* out) {
  return tn_stage_forward_batch(st, req, 1, out);
}

extern "C" int tn_stage_step_async(tn_stage* st, const tn_step_desc* step, void* stream) {
  clear_error();
  TN_REQUIRE(st && step, TN_EINVAL, "null argument");
  std::lock_guard<std::mutex> lk(st->mu);
  TN_ENTER_DEVICE(st->device);
  return step_async_impl(st, step, stream ? (cudaStream_t)stream : st->stream);
}

extern "C" void* tn_stage_stream(tn_stage* st) { return st ? (void*)st->stream : nullptr; }

extern "C" int tn_stage_check(tn_stage* st, void* stream) {
  clear_error();
  TN_REQUIRE(st, TN_EINVAL, "null stage");
  std::lock_guard<std::mutex> lk(st->mu);
  TN_ENTER_DEVICE(st->device);
  const cudaStream_t s = stream ? (cudaStream_t)stream : st->stream;
  TN_CHECK_CUDA(cudaStreamSynchronize(s));
  return recover_kernel_error(st, s);
}

extern "C" int tn_stage_test_raise_kernel_error(tn_stage* st) {
  clear_error();
  TN_REQUIRE(st, TN_EINVAL, "null stage");
  std::lock_guard<std::mutex> lk(st->mu);
  TN_ENTER_DEVICE(st->device);
  TN_CHECK_CUDA(cudaMemsetAsync(st->kerr, 1, sizeof(int), st->stream));
  return TN_OK;
}

extern "C" int tn_stage_free_seq(tn_stage* st, uint64_t seq_id) {
  clear_error();
  TN_REQUIRE(st, TN_EINVAL, "null stage");
  std::lock_guard<std::mutex> lk(st->mu);
  auto it = st->seq_slot.find(seq_id);
  TN_REQUIRE(it != st->seq_slot.end(), TN_EINVAL, "unknown seq_id %llu", (unsigned long long)seq_id);
  st->kv_len[it->second] = 0;
  release_pages(st, it->second);
  st->free_slots.push_back(it->second);
  st->seq_slot.erase(it);
  return TN_OK;
}

extern "C" int32_t tn_stage_kv_len(tn_stage* st, uint64_t seq_id) {
  if (!st) return 0;
  std::lock_guard<std::mutex> lk(st->mu);
  auto it = st->seq_slot.find(seq_id);
  return it == st->seq_slot.end() ? 0 : st->kv_len[it->second];
}

extern "C" int tn_stage_get_info(tn_stage* st, tn_stage_info* info) {
  clear_error();
  TN_REQUIRE(st && info, TN_EINVAL, "null argument");
  std::lock_guard<std::mutex> lk(st->mu);
  info->weight_bytes = st->weight_bytes;
  info->kv_bytes = st->kv_bytes;
  info->scratch_bytes = st->scratch_bytes;
  info->packed_bytes = st->packed_bytes;
  info->n_layers = st->nL;
  info->head_dim = st->hd;
  info->q_dim = st->qDim;
  info->kv_dim = st->kvDim;
  info->ffn_dim = st->F;
  info->graphs_captured = (int32_t)st->graphs.size();
  info->launches_last_step = st->step_launches;
  return TN_OK;
}

extern "C" int tn_stage_profile(tn_stage* st, double* ms, uint64_t* launches, int32_t reset) {
  clear_error();
  TN_REQUIRE(st, TN_EINVAL, "null stage");
  std::lock_guard<std::mutex> lk(st->mu);
  TN_REQUIRE(st->prof, TN_ESTATE, "stage was created without TN_FLAG_PROFILE");
  for (int k = 0; k < TN_PROF_N; k++) {
    if (ms) ms[k] = st->prof_ms[k];
    if (launches) launches[k] = st->prof_launches[k];
    if (reset) {
      st->prof_ms[k] = 0;
      st->prof_launches[k] = 0;
    }
  }
  return TN_OK;
}

extern "C" int tn_stage_set_profile(tn_stage* st, int32_t on) {
  clear_error();
  TN_REQUIRE(st, TN_EINVAL, "null stage");
  std::lock_guard<std::mutex> lk(st->mu);
  TN_ENTER_DEVICE(st->device);
  TN_CHECK_CUDA(cudaStreamSynchronize(st->stream));
  if (on && st->ev.empty()) {
    const int pairs = st->nL * 12 + 16;
    st->ev.resize(2 * pairs);
    st->ev_class.resize(pairs);
    for (auto& e : st->ev) TN_CHECK_CUDA(cudaEventCreate(&e));
  }
  if ((bool)on != st->prof) {
    for (auto& kv : st->graphs) cudaGraphExecDestroy(kv.second.exec);
    st->graphs.clear();
  }
  st->prof = on != 0;
  st->ev_used = 0;
  return TN_OK;
}

extern "C" int tn_stage_peek(tn_stage* st, int32_t what, void* host_out, uint64_t bytes) {
  clear_error();
  TN_REQUIRE(st && host_out, TN_EINVAL, "null argument");
  std::lock_guard<std::mutex> lk(st->mu);
  TN_ENTER_DEVICE(st->device);
  TN_REQUIRE(what == TN_PEEK_HIDDEN || (what == TN_PEEK_LOGITS && st->last), TN_EINVAL, "peek: bad target %d", what);
  const void* src = what == TN_PEEK_HIDDEN ? (const void*)st->h : (const void*)st->logits;
  const uint64_t cap = what == TN_PEEK_HIDDEN ? (uint64_t)st->max_T * st->H * 4
                                              : (uint64_t)std::max(1, std::min(st->max_T, st->max_seqs)) * st->V * 4;
  TN_CHECK_CUDA(cudaStreamSynchronize(st->stream));
  TN_CHECK_CUDA(cudaMemcpy(host_out, src, std::min(bytes, cap), cudaMemcpyDeviceToHost));
  return TN_OK;
}

extern "C" void tn_stage_free(tn_stage* st) {
  if (!st) return;
  {
    DevGuard g(st->device);
    cudaStreamSynchronize(st->stream);
    delete st;
  }
}
