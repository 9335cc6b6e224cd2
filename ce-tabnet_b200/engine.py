"""Host mirror of the reference stage-engine API over the C ABI.

Same names, argument meaning and error behaviour as web/inference-worker.js:
  initStage(spec) -> StageCtx                       (:417)
  forward(ctx, req) -> {"hidden": u16[H]} | {"token_id": int}   (:471, :690)
  freeStage(ctx)                                    (:677)
  sample(logits, temperature=0.7, top_p=0.95)       (:658)
Buffers are numpy arrays or bytes (ArrayBuffer); fp16 activations travel as
uint16 bit patterns, as the reference's Float16Array polyfill carries them
(:56-62).  Every call runs on the GPU through libtabnet_stage.so; there is no
CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import itertools
import os
from dataclasses import dataclass, field

import numpy as np

from . import _lib
from .pack import quant_bytes, round_ffn


def _quant_code(q: str) -> int:
    if q not in _lib.QUANT:
        raise _lib.TnError(_lib.TN_EUNSUPPORTED, f"unsupported quant {q}")  # :126, :136
    return _lib.QUANT[q]


def _as_u8(buf):
    """Host bytes as a uint8 array; a device tensor (weights already in GPU
    memory) passes through with data_ptr()/nbytes."""
    if hasattr(buf, "data_ptr"):
        return _DevBuf(buf.data_ptr(), buf.numel() * buf.element_size())
    if isinstance(buf, np.ndarray):
        return np.ascontiguousarray(buf).view(np.uint8).reshape(-1)
    return np.frombuffer(memoryview(buf), dtype=np.uint8)


class _DevBuf:
    """Minimal stand-in exposing .ctypes.data / .nbytes for a device pointer."""

    class _Ptr:
        def __init__(self, p):
            self.data = p

    def __init__(self, ptr: int, nbytes: int):
        self.ctypes = self._Ptr(ptr)
        self.nbytes = nbytes


@dataclass
class StageCtx:
    """Opaque stage context (the reference's ctx, web/inference-worker.js:422-431)."""
    handle: C.c_void_p
    dims: dict
    layers: tuple
    is_first: bool
    is_last: bool
    hidden_dim: int
    nLayers: int
    backend: str = "cuda"
    ready: bool = True
    hop_mode: int = _lib.TN_HOP_LAST
    _seq_ids: dict = field(default_factory=dict)
    _next_seq: itertools.count = field(default_factory=lambda: itertools.count(1))
    _seed: int = field(default_factory=lambda: int.from_bytes(os.urandom(8), "little"))

    def seq_key(self, seq_id) -> int:
        """Map the reference's string seq_id onto the engine's u64 handle."""
        if seq_id not in self._seq_ids:
            self._seq_ids[seq_id] = next(self._next_seq)
        return self._seq_ids[seq_id]

    def peek(self, what: str, rows: int) -> np.ndarray:
        """Test hook: f32 hidden rows ("hidden") or logits ("logits") of the last step."""
        width = self.hidden_dim if what == "hidden" else int(self.dims["vocab"])
        out = np.zeros((rows, width), dtype=np.float32)
        code = 0 if what == "hidden" else 1
        _lib.check(_lib.load().tn_stage_peek(self.handle, code, out.ctypes.data, out.nbytes))
        return out

    def profile(self, reset: bool = False) -> dict:
        """{kernel class: (ms, launches)} of synchronous calls (opts.profile stages)."""
        n = len(_lib.PROF_CLASSES)
        ms = (C.c_double * n)()
        cnt = (C.c_uint64 * n)()
        _lib.check(_lib.load().tn_stage_profile(self.handle, ms, cnt, int(reset)))
        return {k: (ms[i], int(cnt[i])) for i, k in enumerate(_lib.PROF_CLASSES)}

    def info(self) -> dict:
        inf = _lib.StageInfo()
        _lib.check(_lib.load().tn_stage_get_info(self.handle, C.byref(inf)))
        return {k: getattr(inf, k) for k, _ in _lib.StageInfo._fields_}


def initStage(spec: dict) -> StageCtx:
    """initStage (web/inference-worker.js:417-466).

    spec = {arch, dims:{hidden_dim, n_heads, n_kv_heads, vocab, rope_theta, ffn_dim?},
            layers:[lo, hi], is_first, is_last,
            weights:{layers:[{idx, buf, quant}], embed?, norm?, lm_head?, embedQuant?, lmHeadQuant?, quant?},
            opts?:{max_ctx, max_seqs, max_tokens_per_step, device, hop_mode, no_graphs,
                   kv_dtype: "f32" (default, the reference's rows) | "f16" (half-size KV cache)
                             | "f8" (e4m3, quarter-size),
                   kv_page_tokens: 0 (contiguous max_ctx rows per sequence) | positions per KV page,
                   kv_pages: pages in the pool (0: max_seqs x max_ctx worth)}}
    """
    lib = _lib.load()
    dims, (lo, hi), w = spec["dims"], spec["layers"], spec["weights"]
    opts = spec.get("opts") or {}
    H = int(dims["hidden_dim"])
    keep = []  # buffers referenced by the spec until tn_stage_init returns
    wl = w.get("layers", [])
    arr = (_lib.LayerWeights * max(1, len(wl)))()
    for i, l in enumerate(wl):
        if "buf" not in l:
            raise _lib.TnError(_lib.TN_EUNSUPPORTED, "multi-part layers are not supported")  # :434
        b = _as_u8(l["buf"])
        keep.append(b)
        arr[i] = _lib.LayerWeights(int(l["idx"]), _quant_code(l.get("quant", w.get("quant", "q4_0"))),
                                   b.ctypes.data, b.nbytes)
    s = _lib.StageSpec()
    s.abi_version = _lib.TN_ABI_VERSION
    s.hidden_dim, s.n_heads, s.n_kv_heads = H, int(dims["n_heads"]), int(dims["n_kv_heads"])
    s.vocab = int(dims["vocab"])
    s.ffn_dim = int(dims.get("ffn_dim") or 0)
    s.rope_theta = float(dims["rope_theta"])
    s.layer_lo, s.layer_hi = int(lo), int(hi)
    s.is_first, s.is_last = int(bool(spec.get("is_first"))), int(bool(spec.get("is_last")))
    s.layers, s.n_layers = arr, len(wl)
    if spec.get("is_first") and w.get("embed") is not None:
        e = _as_u8(w["embed"])
        keep.append(e)
        s.embed, s.embed_len = e.ctypes.data, e.nbytes
        s.embed_quant = _quant_code(w.get("embedQuant") or w.get("quant") or "q4_0")  # :465
    if spec.get("is_last"):
        if w.get("norm") is not None:
            n = _as_u8(w["norm"])
            keep.append(n)
            s.norm, s.norm_len = n.ctypes.data, n.nbytes
        if w.get("lm_head") is not None:
            h = _as_u8(w["lm_head"])
            keep.append(h)
            s.lm_head, s.lm_head_len = h.ctypes.data, h.nbytes
            s.lm_head_quant = _quant_code(w.get("lmHeadQuant") or w.get("quant") or "q4_0")  # :466
    s.weights_on_device = int(bool(w.get("on_device", False)))
    s.device = int(opts.get("device", 0))
    s.max_ctx = int(opts.get("max_ctx", 4096))  # :642
    s.max_seqs = int(opts.get("max_seqs", 16))
    s.max_tokens_per_step = int(opts.get("max_tokens_per_step", 512))
    kv_dtype = opts.get("kv_dtype", "f32")
    if kv_dtype not in ("f32", "f16", "f8"):
        raise ValueError(f"opts.kv_dtype must be 'f32', 'f16' or 'f8', not {kv_dtype!r}")
    s.kv_page_tokens = int(opts.get("kv_page_tokens") or 0)
    s.kv_pages = int(opts.get("kv_pages") or 0)
    s.flags = (_lib.TN_FLAG_NO_GRAPHS if opts.get("no_graphs") else 0) | \
        (_lib.TN_FLAG_PROFILE if opts.get("profile") else 0) | \
        (_lib.TN_FLAG_NO_FUSED_DECODE if opts.get("fused_decode") is False else 0) | \
        (_lib.TN_FLAG_KV_F16 if kv_dtype == "f16" else 0) | \
        (_lib.TN_FLAG_KV_F8 if kv_dtype == "f8" else 0)
    handle = C.c_void_p()
    _lib.check(lib.tn_stage_init(C.byref(s), C.byref(handle)))
    return StageCtx(handle=handle, dims=dict(dims), layers=(lo, hi), is_first=bool(spec.get("is_first")),
                    is_last=bool(spec.get("is_last")), hidden_dim=H, nLayers=hi - lo,
                    hop_mode=_lib.TN_HOP_ALL if opts.get("hop_mode") == "all" else _lib.TN_HOP_LAST)


def _build_req(ctx: StageCtx, req: dict, keep: list):
    r = _lib.FwdReq()
    r.seq_id = ctx.seq_key(req["seq_id"])
    if ctx.is_first:
        ids = req.get("token_ids")
        if ids is None or len(ids) == 0:
            if req.get("token_id") is None:
                raise _lib.TnError(_lib.TN_ESTATE, "first stage: token_ids or token_id required")
            ids = [req["token_id"]]  # :480
        a = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
        keep.append(a)
        r.token_ids = a.ctypes.data_as(C.POINTER(C.c_int32))
        r.n_tokens = int(a.size)
        r.token_pos = int(req.get("token_pos") or 0)  # :483
    else:
        hid = np.asarray(req["hidden"])
        hid = np.ascontiguousarray(hid.view(np.uint16) if hid.dtype == np.float16 else hid.astype(np.uint16, copy=False))
        keep.append(hid)
        if hid.size % ctx.hidden_dim:
            raise _lib.TnError(_lib.TN_EINVAL, f"hidden of {hid.size} values is not a multiple of {ctx.hidden_dim}")
        r.hidden = hid.ctypes.data_as(C.POINTER(C.c_uint16))
        r.n_tokens = hid.size // ctx.hidden_dim
        r.token_pos = int(req["token_pos"])
    t = req.get("temperature")
    p = req.get("top_p")
    r.temperature = 0.7 if t is None else float(t)  # :715 `?? 0.7`
    r.top_p = 0.95 if p is None else float(p)
    r.rng_seed = int(req.get("rng_seed", ctx._seed)) & (2**64 - 1)
    hop = req.get("hop_mode")
    r.hop_mode = ctx.hop_mode if hop is None else (_lib.TN_HOP_ALL if hop == "all" else _lib.TN_HOP_LAST)
    return r


def forward_batch(ctx: StageCtx, reqs: list) -> list:
    """Several sequences' requests fused into one engine step."""
    if not ctx.ready:
        raise _lib.TnError(_lib.TN_ESTATE, "stage has been freed")
    keep = []
    n = len(reqs)
    creqs = (_lib.FwdReq * n)()
    outs = (_lib.FwdOut * n)()
    bufs = []
    for i, q in enumerate(reqs):
        creqs[i] = _build_req(ctx, q, keep)
        if not ctx.is_last:
            cap = creqs[i].n_tokens if creqs[i].hop_mode == _lib.TN_HOP_ALL else 1
            b = np.zeros(cap * ctx.hidden_dim, dtype=np.uint16)
            bufs.append(b)
            outs[i].hidden = b.ctypes.data_as(C.POINTER(C.c_uint16))
            outs[i].hidden_cap_tokens = cap
        else:
            bufs.append(None)
    _lib.check(_lib.load().tn_stage_forward_batch(ctx.handle, creqs, n, outs))
    res = []
    for i in range(n):
        if ctx.is_last:
            res.append({"token_id": int(outs[i].token_id)})
        else:
            k = outs[i].n_hidden_tokens
            h = bufs[i][: k * ctx.hidden_dim]
            res.append({"hidden": h if k == 1 else h.reshape(k, ctx.hidden_dim)})
    return res


def forward(ctx: StageCtx, req: dict) -> dict:
    """forward (web/inference-worker.js:471-490; last stage :690-716)."""
    return forward_batch(ctx, [req])[0]


forwardSafe = forward
forwardLast = forward


def freeStage(ctx: StageCtx) -> None:
    """freeStage (web/inference-worker.js:677-684)."""
    if ctx is None or not ctx.ready:
        return
    _lib.load().tn_stage_free(ctx.handle)
    ctx.handle = C.c_void_p()
    ctx._seq_ids.clear()
    ctx.ready = False


def free_seq(ctx: StageCtx, seq_id) -> None:
    """Drop one sequence's KV (the reference has no per-sequence free)."""
    key = ctx._seq_ids.pop(seq_id, None)
    if key is not None:
        _lib.check(_lib.load().tn_stage_free_seq(ctx.handle, key))


def kv_len(ctx: StageCtx, seq_id) -> int:
    key = ctx._seq_ids.get(seq_id)
    return 0 if key is None else int(_lib.load().tn_stage_kv_len(ctx.handle, key))


def sample(logits, temperature: float = 0.7, top_p: float = 0.95, rng_seed: int = 0) -> int:
    """sample (web/inference-worker.js:658-672) on the GPU; the uniform draw is
    tn_sample_uniform(rng_seed, 0) in place of Math.random()."""
    import torch  # device memory only

    x = torch.as_tensor(np.ascontiguousarray(np.asarray(logits, dtype=np.float32))).cuda()
    out = torch.zeros(1, dtype=torch.int32, device=x.device)
    _lib.check(_lib.load().tn_sample(x.data_ptr(), 1, x.numel(), float(temperature), float(top_p),
                                     int(rng_seed), out.data_ptr(), torch.cuda.current_stream().cuda_stream))
    return int(out.item())
