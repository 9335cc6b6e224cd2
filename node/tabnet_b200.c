/*
 * tabnet_b200.c -- Node-API addon over libtabnet_stage.so (include/tabnet_stage.h).
 *
 * Exports the engine contract of web/inference-worker.js:13-19 with the same
 * argument meaning, defaults and errors:
 *
 *   initStage(spec)  -> Promise<ctx>                        (:417-466)
 *   forward(ctx, req) -> Promise<{hidden: Uint16Array} | {token_id}>  (:471-490, :690-716)
 *   freeStage(ctx)                                          (:677-684)
 *
 * Each engine call runs on the libuv thread pool (napi_async_work), so the
 * event loop never waits for the GPU.  Weight buffers are borrowed for the
 * duration of init only (tn_stage_init copies and repacks them).  An
 * activation frame is read as its uint16 bit patterns: on runtimes with a
 * native Float16Array the reference's polyfill (:60-62) is absent, and the
 * element values of such an array are not the bits forward expects.
 * String seq_ids map to the engine's 64-bit handles by FNV-1a.
 *
 * Build: node-gyp rebuild (binding.gyp beside this file), with
 * libtabnet_stage.so built by ce-tabnet_b200/build.py.
 * Untested here: this image has no Node.js and no node_api.h.
 */
#include <node_api.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "tabnet_stage.h"

#define NAPI_OK(call)                                      \
  do {                                                     \
    if ((call) != napi_ok) {                               \
      napi_throw_error(env, NULL, "tabnet_b200: " #call);  \
      return NULL;                                         \
    }                                                      \
  } while (0)

/* ---------------------------------------------------------------- helpers */
typedef struct {
  tn_stage* st;
  int32_t hidden_dim, vocab, is_first, is_last;
  int freed;
} stage_ctx;

static void ctx_finalize(napi_env env, void* data, void* hint) {
  stage_ctx* c = (stage_ctx*)data;
  (void)env;
  (void)hint;
  if (!c->freed && c->st) tn_stage_free(c->st);
  free(c);
}

static int has(napi_env env, napi_value obj, const char* key) {
  bool b = false;
  napi_valuetype t;
  napi_value v;
  if (napi_has_named_property(env, obj, key, &b) != napi_ok || !b) return 0;
  if (napi_get_named_property(env, obj, key, &v) != napi_ok) return 0;
  if (napi_typeof(env, v, &t) != napi_ok) return 0;
  return t != napi_undefined && t != napi_null;
}

static napi_value prop(napi_env env, napi_value obj, const char* key) {
  napi_value v = NULL;
  napi_get_named_property(env, obj, key, &v);
  return v;
}

static double num(napi_env env, napi_value obj, const char* key, double dflt) {
  double d = dflt;
  if (has(env, obj, key)) napi_get_value_double(env, prop(env, obj, key), &d);
  return d;
}

static int truthy(napi_env env, napi_value obj, const char* key) {
  bool b = false;
  napi_value v;
  if (!has(env, obj, key)) return 0;
  if (napi_coerce_to_bool(env, prop(env, obj, key), &v) != napi_ok) return 0;
  napi_get_value_bool(env, v, &b);
  return b ? 1 : 0;
}

/* "q4_0" -> TN_QUANT_Q4_0; -1 is "unsupported quant" (web/inference-worker.js:126, :136) */
static int quant_code(napi_env env, napi_value s) {
  char b[16] = {0};
  size_t n = 0;
  if (napi_get_value_string_utf8(env, s, b, sizeof b, &n) != napi_ok) return -1;
  if (!strcmp(b, "f32")) return TN_QUANT_F32;
  if (!strcmp(b, "f16")) return TN_QUANT_F16;
  if (!strcmp(b, "q4_0")) return TN_QUANT_Q4_0;
  if (!strcmp(b, "q8_0")) return TN_QUANT_Q8_0;
  return -1;
}

/* bytes of an ArrayBuffer, a TypedArray or a DataView */
static int bytes_of(napi_env env, napi_value v, void** data, size_t* len) {
  bool is = false;
  if (napi_is_arraybuffer(env, v, &is) == napi_ok && is)
    return napi_get_arraybuffer_info(env, v, data, len) == napi_ok;
  if (napi_is_typedarray(env, v, &is) == napi_ok && is) {
    napi_typedarray_type t;
    size_t n, off;
    napi_value ab;
    void* base;
    if (napi_get_typedarray_info(env, v, &t, &n, &base, &ab, &off) != napi_ok) return 0;
    size_t el = 1;
    switch (t) {
      case napi_int16_array:
      case napi_uint16_array: el = 2; break;
      case napi_int32_array:
      case napi_uint32_array:
      case napi_float32_array: el = 4; break;
      case napi_float64_array:
      case napi_bigint64_array:
      case napi_biguint64_array: el = 8; break;
      default: el = 1;
    }
    *data = base;
    *len = n * el;
    return 1;
  }
  if (napi_is_dataview(env, v, &is) == napi_ok && is) {
    napi_value ab;
    size_t off;
    return napi_get_dataview_info(env, v, len, data, &ab, &off) == napi_ok;
  }
  return 0;
}

static napi_value make_error(napi_env env, const char* msg) {
  napi_value m, e;
  napi_create_string_utf8(env, msg, NAPI_AUTO_LENGTH, &m);
  napi_create_error(env, NULL, m, &e);
  return e;
}

static uint64_t seq_key(napi_env env, napi_value v) {
  /* FNV-1a over the string form of seq_id */
  char buf[256];
  size_t n = 0;
  napi_value s;
  uint64_t h = 1469598103934665603ull;
  if (napi_coerce_to_string(env, v, &s) != napi_ok) return h;
  napi_get_value_string_utf8(env, s, buf, sizeof buf, &n);
  for (size_t i = 0; i < n; i++) h = (h ^ (uint8_t)buf[i]) * 1099511628211ull;
  return h;
}

/* ---------------------------------------------------------------- initStage */
typedef struct {
  napi_async_work work;
  napi_deferred deferred;
  napi_ref keep; /* the spec object, so its buffers outlive the worker thread's reads */
  tn_stage_spec spec;
  tn_layer_weights* layers;
  tn_stage* st;
  int rc;
  char err[512];
} init_job;

static void init_exec(napi_env env, void* p) {
  init_job* j = (init_job*)p;
  (void)env;
  j->rc = tn_stage_init(&j->spec, &j->st);
  if (j->rc) {
    strncpy(j->err, tn_last_error(), sizeof j->err - 1);
    j->err[sizeof j->err - 1] = 0;
  }
}

static void init_done(napi_env env, napi_status status, void* p) {
  init_job* j = (init_job*)p;
  napi_value v;
  if (status != napi_ok || j->rc) {
    napi_reject_deferred(env, j->deferred, make_error(env, j->rc ? j->err : "initStage cancelled"));
  } else {
    stage_ctx* c = (stage_ctx*)calloc(1, sizeof *c);
    c->st = j->st;
    c->hidden_dim = j->spec.hidden_dim;
    c->vocab = j->spec.vocab;
    c->is_first = j->spec.is_first;
    c->is_last = j->spec.is_last;
    napi_create_external(env, c, ctx_finalize, NULL, &v);
    napi_resolve_deferred(env, j->deferred, v);
  }
  napi_delete_reference(env, j->keep);
  napi_delete_async_work(env, j->work);
  free(j->layers);
  free(j);
}

static napi_value js_initStage(napi_env env, napi_callback_info info) {
  size_t argc = 1;
  napi_value argv[1], promise, name;
  NAPI_OK(napi_get_cb_info(env, info, &argc, argv, NULL, NULL));
  if (argc < 1) {
    napi_throw_type_error(env, NULL, "initStage(spec)");
    return NULL;
  }
  napi_value spec = argv[0];
  napi_value dims = prop(env, spec, "dims"), w = prop(env, spec, "weights");
  napi_value opts = has(env, spec, "opts") ? prop(env, spec, "opts") : NULL;
  init_job* j = (init_job*)calloc(1, sizeof *j);
  tn_stage_spec* s = &j->spec;
  s->abi_version = TN_ABI_VERSION;
  s->hidden_dim = (int32_t)num(env, dims, "hidden_dim", 0);
  s->n_heads = (int32_t)num(env, dims, "n_heads", 0);
  s->n_kv_heads = (int32_t)num(env, dims, "n_kv_heads", 0);
  s->vocab = (int32_t)num(env, dims, "vocab", 0);
  s->ffn_dim = (int32_t)num(env, dims, "ffn_dim", 0); /* 0 -> roundFfn (:160-163) */
  s->rope_theta = num(env, dims, "rope_theta", 10000.0);
  napi_value lr = prop(env, spec, "layers"), e0, e1;
  napi_get_element(env, lr, 0, &e0);
  napi_get_element(env, lr, 1, &e1);
  double lo = 0, hi = 0;
  napi_get_value_double(env, e0, &lo);
  napi_get_value_double(env, e1, &hi);
  s->layer_lo = (int32_t)lo;
  s->layer_hi = (int32_t)hi;
  s->is_first = truthy(env, spec, "is_first");
  s->is_last = truthy(env, spec, "is_last");
  /* weights.quant is the default of every per-layer and whole-model quant;
   * embedQuant / lmHeadQuant fall back to it, then to "q4_0" (:465-466) */
  int dflt = TN_QUANT_Q4_0;
  if (has(env, w, "quant") && (dflt = quant_code(env, prop(env, w, "quant"))) < 0) goto unsupported;
  {
    napi_value wl = prop(env, w, "layers");
    uint32_t n = 0;
    napi_get_array_length(env, wl, &n);
    j->layers = (tn_layer_weights*)calloc(n ? n : 1, sizeof(tn_layer_weights));
    for (uint32_t i = 0; i < n; i++) {
      napi_value l;
      napi_get_element(env, wl, i, &l);
      if (!has(env, l, "buf")) { /* multi-part layers: the reference reads only `buf` (:434) */
        napi_throw_error(env, NULL, "multi-part layers are not supported");
        goto fail;
      }
      void* data;
      size_t len;
      if (!bytes_of(env, prop(env, l, "buf"), &data, &len)) {
        napi_throw_type_error(env, NULL, "weights.layers[i].buf must be an ArrayBuffer or a typed array");
        goto fail;
      }
      int q = has(env, l, "quant") ? quant_code(env, prop(env, l, "quant")) : dflt;
      if (q < 0) goto unsupported;
      j->layers[i].idx = (int32_t)num(env, l, "idx", s->layer_lo + (double)i);
      j->layers[i].quant = q;
      j->layers[i].buf = data;
      j->layers[i].len = len;
    }
    s->layers = j->layers;
    s->n_layers = (int32_t)n;
  }
  if (s->is_first && has(env, w, "embed")) {
    void* data;
    size_t len;
    if (!bytes_of(env, prop(env, w, "embed"), &data, &len)) goto badbuf;
    s->embed = data;
    s->embed_len = len;
    s->embed_quant = has(env, w, "embedQuant") ? quant_code(env, prop(env, w, "embedQuant")) : dflt;
    if (s->embed_quant < 0) goto unsupported;
  }
  if (s->is_last) {
    void* data;
    size_t len;
    if (has(env, w, "norm")) {
      if (!bytes_of(env, prop(env, w, "norm"), &data, &len)) goto badbuf;
      s->norm = data;
      s->norm_len = len;
    }
    if (has(env, w, "lm_head")) {
      if (!bytes_of(env, prop(env, w, "lm_head"), &data, &len)) goto badbuf;
      s->lm_head = data;
      s->lm_head_len = len;
      s->lm_head_quant = has(env, w, "lmHeadQuant") ? quant_code(env, prop(env, w, "lmHeadQuant")) : dflt;
      if (s->lm_head_quant < 0) goto unsupported;
    }
  }
  s->max_ctx = opts ? (int32_t)num(env, opts, "max_ctx", 4096) : 4096; /* :642 */
  s->max_seqs = opts ? (int32_t)num(env, opts, "max_seqs", 16) : 16;
  s->device = opts ? (int32_t)num(env, opts, "device", 0) : 0;
  s->kv_page_tokens = opts ? (int32_t)num(env, opts, "kv_page_tokens", 0) : 0; /* 0: contiguous KV */
  s->kv_pages = opts ? (int32_t)num(env, opts, "kv_pages", 0) : 0;
  NAPI_OK(napi_create_reference(env, spec, 1, &j->keep));
  NAPI_OK(napi_create_promise(env, &j->deferred, &promise));
  napi_create_string_utf8(env, "tabnet_b200.initStage", NAPI_AUTO_LENGTH, &name);
  NAPI_OK(napi_create_async_work(env, NULL, name, init_exec, init_done, j, &j->work));
  NAPI_OK(napi_queue_async_work(env, j->work));
  return promise;
unsupported:
  napi_throw_error(env, NULL, "unsupported quant");
  goto fail;
badbuf:
  napi_throw_type_error(env, NULL, "weights buffers must be ArrayBuffers or typed arrays");
fail:
  free(j->layers);
  free(j);
  return NULL;
}

/* ---------------------------------------------------------------- forward */
typedef struct {
  napi_async_work work;
  napi_deferred deferred;
  napi_ref ctx_ref;
  stage_ctx* c;
  tn_fwd_req req;
  tn_fwd_out out;
  int32_t* ids;      /* copied token ids */
  uint16_t* hidden;  /* copied input frame bits */
  uint16_t* result;  /* output frame (non-last stage) */
  int rc;
  char err[512];
} fwd_job;

static void fwd_exec(napi_env env, void* p) {
  fwd_job* j = (fwd_job*)p;
  (void)env;
  j->rc = tn_stage_forward(j->c->st, &j->req, &j->out);
  if (j->rc) {
    strncpy(j->err, tn_last_error(), sizeof j->err - 1);
    j->err[sizeof j->err - 1] = 0;
  }
}

static void fwd_done(napi_env env, napi_status status, void* p) {
  fwd_job* j = (fwd_job*)p;
  if (status != napi_ok || j->rc) {
    napi_reject_deferred(env, j->deferred, make_error(env, j->rc ? j->err : "forward cancelled"));
  } else {
    napi_value obj, v;
    napi_create_object(env, &obj);
    if (j->c->is_last) {
      napi_create_int32(env, j->out.token_id, &v);
      napi_set_named_property(env, obj, "token_id", v);
    } else {
      /* a fresh Uint16Array owned by the caller (the reference returns a new array, :486) */
      const size_t n = (size_t)j->out.n_hidden_tokens * (size_t)j->c->hidden_dim;
      void* data;
      napi_value ab;
      napi_create_arraybuffer(env, n * 2, &data, &ab);
      memcpy(data, j->result, n * 2);
      napi_create_typedarray(env, napi_uint16_array, n, ab, 0, &v);
      napi_set_named_property(env, obj, "hidden", v);
    }
    napi_resolve_deferred(env, j->deferred, obj);
  }
  napi_delete_reference(env, j->ctx_ref);
  napi_delete_async_work(env, j->work);
  free(j->ids);
  free(j->hidden);
  free(j->result);
  free(j);
}

static napi_value js_forward(napi_env env, napi_callback_info info) {
  size_t argc = 2;
  napi_value argv[2], promise, name;
  NAPI_OK(napi_get_cb_info(env, info, &argc, argv, NULL, NULL));
  stage_ctx* c = NULL;
  if (argc < 2 || napi_get_value_external(env, argv[0], (void**)&c) != napi_ok || !c) {
    napi_throw_type_error(env, NULL, "forward(ctx, req)");
    return NULL;
  }
  if (c->freed) {
    napi_throw_error(env, NULL, "stage has been freed");
    return NULL;
  }
  napi_value req = argv[1];
  fwd_job* j = (fwd_job*)calloc(1, sizeof *j);
  j->c = c;
  j->req.seq_id = seq_key(env, prop(env, req, "seq_id"));
  j->req.token_pos = (int32_t)num(env, req, "token_pos", 0);
  j->req.temperature = num(env, req, "temperature", 0.7); /* :715 `temperature ?? 0.7` */
  j->req.top_p = num(env, req, "top_p", 0.95);
  j->req.rng_seed = (uint64_t)num(env, req, "rng_seed", 0);
  j->req.hop_mode = TN_HOP_LAST; /* the reference returns the last position only (:486) */
  if (c->is_first) {
    /* ids = token_ids || [token_id] (:480) */
    uint32_t n = 0;
    if (has(env, req, "token_ids")) napi_get_array_length(env, prop(env, req, "token_ids"), &n);
    if (n == 0) {
      if (!has(env, req, "token_id")) {
        napi_throw_error(env, NULL, "first stage: token_ids or token_id required");
        free(j);
        return NULL;
      }
      j->ids = (int32_t*)malloc(sizeof(int32_t));
      j->ids[0] = (int32_t)num(env, req, "token_id", 0);
      n = 1;
    } else {
      napi_value arr = prop(env, req, "token_ids"), e;
      j->ids = (int32_t*)malloc(sizeof(int32_t) * n);
      for (uint32_t i = 0; i < n; i++) {
        double d = 0;
        napi_get_element(env, arr, i, &e);
        napi_get_value_double(env, e, &d);
        j->ids[i] = (int32_t)d;
      }
    }
    j->req.token_ids = j->ids;
    j->req.n_tokens = (int32_t)n;
  } else {
    void* data;
    size_t len;
    if (!has(env, req, "hidden") || !bytes_of(env, prop(env, req, "hidden"), &data, &len) ||
        len % ((size_t)c->hidden_dim * 2) != 0 || len == 0) {
      napi_throw_type_error(env, NULL, "hidden must be a Uint16Array (fp16 bits) of n * hidden_dim values");
      free(j);
      return NULL;
    }
    j->hidden = (uint16_t*)malloc(len);
    memcpy(j->hidden, data, len);
    j->req.hidden = j->hidden;
    j->req.n_tokens = (int32_t)(len / ((size_t)c->hidden_dim * 2));
  }
  if (!c->is_last) {
    j->result = (uint16_t*)malloc((size_t)c->hidden_dim * 2);
    j->out.hidden = j->result;
    j->out.hidden_cap_tokens = 1;
  }
  NAPI_OK(napi_create_reference(env, argv[0], 1, &j->ctx_ref)); /* the stage lives while the call runs */
  NAPI_OK(napi_create_promise(env, &j->deferred, &promise));
  napi_create_string_utf8(env, "tabnet_b200.forward", NAPI_AUTO_LENGTH, &name);
  NAPI_OK(napi_create_async_work(env, NULL, name, fwd_exec, fwd_done, j, &j->work));
  NAPI_OK(napi_queue_async_work(env, j->work));
  return promise;
}

/* ---------------------------------------------------------------- freeStage */
static napi_value js_freeStage(napi_env env, napi_callback_info info) {
  size_t argc = 1;
  napi_value argv[1];
  NAPI_OK(napi_get_cb_info(env, info, &argc, argv, NULL, NULL));
  stage_ctx* c = NULL;
  if (argc < 1 || napi_get_value_external(env, argv[0], (void**)&c) != napi_ok || !c) return NULL;
  /* tn_stage_free waits for the stage's stream; a forward still queued on the
   * thread pool holds a reference to ctx, so the caller awaits it first (the
   * reference frees only between steps, web/tabnet-node.js:187, :202) */
  if (!c->freed) {
    tn_stage_free(c->st);
    c->st = NULL;
    c->freed = 1;
  }
  return NULL;
}

static napi_value init_module(napi_env env, napi_value exports) {
  napi_property_descriptor d[] = {
      {"initStage", NULL, js_initStage, NULL, NULL, NULL, napi_default, NULL},
      {"forward", NULL, js_forward, NULL, NULL, NULL, napi_default, NULL},
      {"freeStage", NULL, js_freeStage, NULL, NULL, NULL, napi_default, NULL},
  };
  NAPI_OK(napi_define_properties(env, exports, sizeof d / sizeof d[0], d));
  return exports;
}

NAPI_MODULE(NODE_GYP_MODULE_NAME, init_module)
