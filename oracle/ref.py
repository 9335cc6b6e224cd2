"""ORACLE (test infrastructure only): ctypes wrapper of oracle/libref_cpu.so.

libref_cpu.so restates the reference engine's CPU path
(web/inference-worker.js:68-178, 417-583, 658-716) in C with JavaScript's
numeric model (double accumulators, float storage).  Only tests/,
__graft_entry__.smoke() and bench.py's CPU baseline legs use it, as the checker
or the timed CPU baseline -- never as part of the engine.

Parity pin: the reference has no golden vectors or engine tests and no
JavaScript runtime exists on this machine, so the oracle is "parity unpinned"
against reference-produced outputs; it is pinned by hand-derived known-answer
tests (tests/golden/kat_*.json).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "libref_cpu.so"
QUANT = {"f32": 0, "f16": 1, "q4_0": 2, "q8_0": 3}
KV_FORMAT = {"f32": 0, "f16": 1, "f8": 2}
_lib = None


class RefSpec(C.Structure):
    _fields_ = [
        ("hidden_dim", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int), ("vocab", C.c_int),
        ("ffn_dim", C.c_int), ("rope_theta", C.c_double),
        ("layer_lo", C.c_int), ("layer_hi", C.c_int), ("is_first", C.c_int), ("is_last", C.c_int),
        ("layer_bufs", C.POINTER(C.c_void_p)), ("layer_quants", C.POINTER(C.c_int)), ("n_layers", C.c_int),
        ("embed", C.c_void_p), ("embed_quant", C.c_int), ("norm", C.c_void_p),
        ("lm_head", C.c_void_p), ("lm_head_quant", C.c_int), ("n_threads", C.c_int),
    ]


def load() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
        lib = C.CDLL(str(LIB))
        lib.ref_f32_to_f16.restype = C.c_uint16
        lib.ref_f32_to_f16.argtypes = [C.c_double]
        lib.ref_f16_to_f32.restype = C.c_double
        lib.ref_f16_to_f32.argtypes = [C.c_uint16]
        lib.ref_f32_to_f16_array.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
        lib.ref_f32bits_to_f16_range.argtypes = [C.c_uint32, C.c_uint64, C.c_void_p]
        lib.ref_quant_bytes.restype = C.c_int64
        lib.ref_quant_bytes.argtypes = [C.c_int64, C.c_int]
        lib.ref_dequant_range.argtypes = [C.c_void_p, C.c_int, C.c_int64, C.c_int64, C.c_void_p]
        lib.ref_round_ffn.argtypes = [C.c_int]
        lib.ref_rmsnorm.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
        lib.ref_matvec_packed.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int]
        lib.ref_rope.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_double]
        lib.ref_attention.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                      C.c_void_p]
        lib.ref_sample.argtypes = [C.c_void_p, C.c_int, C.c_double, C.c_double, C.c_double]
        lib.ref_init.restype = C.c_void_p
        lib.ref_init.argtypes = [C.POINTER(RefSpec)]
        lib.ref_forward.argtypes = [C.c_void_p, C.c_uint64, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_double,
                                    C.c_double, C.c_double, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        lib.ref_kv_len.argtypes = [C.c_void_p, C.c_uint64]
        lib.ref_kv_row.argtypes = [C.c_void_p, C.c_uint64, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        lib.ref_free.argtypes = [C.c_void_p]
        lib.ref_set_kv_format.argtypes = [C.c_void_p, C.c_int]
        lib.ref_round_kv.argtypes = [C.c_int, C.c_float]
        lib.ref_round_kv.restype = C.c_float
        _lib = lib
    return _lib


def threads() -> int:
    return int(os.environ.get("TABNET_ORACLE_THREADS", os.cpu_count() or 1))


def f32_to_f16(v: float) -> int:
    return int(load().ref_f32_to_f16(float(v)))


def f32_to_f16_array(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.empty(x.size, dtype=np.uint16)
    load().ref_f32_to_f16_array(x.ctypes.data, out.ctypes.data, x.size)
    return out


def f32bits_to_f16(first: int, count: int) -> np.ndarray:
    out = np.empty(count, dtype=np.uint16)
    load().ref_f32bits_to_f16_range(first, count, out.ctypes.data)
    return out


def f16_to_f32(h: int) -> float:
    return float(load().ref_f16_to_f32(int(h)))


def quant_bytes(count: int, quant: str) -> int:
    return int(load().ref_quant_bytes(count, QUANT[quant]))


def dequant(buf: np.ndarray, quant: str, count: int, start: int = 0) -> np.ndarray:
    buf = np.ascontiguousarray(buf, dtype=np.uint8)
    out = np.empty(count, dtype=np.float32)
    if load().ref_dequant_range(buf.ctypes.data, QUANT[quant], start, count, out.ctypes.data) != 0:
        raise ValueError(f"unsupported quant {quant}")
    return out


def matvec(buf: np.ndarray, quant: str, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    buf = np.ascontiguousarray(buf, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(rows, dtype=np.float32)
    if load().ref_matvec_packed(buf.ctypes.data, QUANT[quant], rows, cols, x.ctypes.data, y.ctypes.data,
                                threads()) != 0:
        raise ValueError("matvec failed")
    return y


def rmsnorm(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    load().ref_rmsnorm(x.ctypes.data, w.ctypes.data, x.size, out.ctypes.data)
    return out


def rope(vec: np.ndarray, n_heads: int, head_dim: int, pos: int, theta: float) -> np.ndarray:
    v = np.array(vec, dtype=np.float32, copy=True)
    load().ref_rope(v.ctypes.data, n_heads, head_dim, pos, theta)
    return v


def attention(q: np.ndarray, K: np.ndarray, V: np.ndarray, n_heads: int, n_kv: int, head_dim: int) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.float32)
    K = np.ascontiguousarray(K, dtype=np.float32)
    V = np.ascontiguousarray(V, dtype=np.float32)
    out = np.empty(n_heads * head_dim, dtype=np.float32)
    load().ref_attention(q.ctypes.data, K.ctypes.data, V.ctypes.data, K.shape[0], n_heads, n_kv, head_dim,
                         out.ctypes.data)
    return out


def sample(logits: np.ndarray, temperature: float, top_p: float, u: float) -> int:
    x = np.ascontiguousarray(logits, dtype=np.float32)
    return int(load().ref_sample(x.ctypes.data, x.size, temperature, top_p, u))


class RefStage:
    """initStage / forward / freeStage of the reference CPU path."""

    def __init__(self, dims: dict, lo: int, hi: int, is_first: bool, is_last: bool, weights: dict,
                 n_threads: int | None = None, kv_dtype: str = "f32"):
        lib = load()
        self.H = int(dims["hidden_dim"])
        self.vocab = int(dims["vocab"])
        self.is_first, self.is_last = is_first, is_last
        self._keep = []
        layers = weights["layers"]
        bufs = (C.c_void_p * max(1, len(layers)))()
        quants = (C.c_int * max(1, len(layers)))()
        for i, l in enumerate(layers):
            b = np.ascontiguousarray(l["buf"], dtype=np.uint8)
            self._keep.append(b)
            bufs[i] = b.ctypes.data
            quants[i] = QUANT[l["quant"]]
        s = RefSpec()
        s.hidden_dim, s.n_heads, s.n_kv_heads = self.H, int(dims["n_heads"]), int(dims["n_kv_heads"])
        s.vocab, s.ffn_dim, s.rope_theta = self.vocab, int(dims.get("ffn_dim") or 0), float(dims["rope_theta"])
        s.layer_lo, s.layer_hi, s.is_first, s.is_last = lo, hi, int(is_first), int(is_last)
        s.layer_bufs, s.layer_quants, s.n_layers = bufs, quants, len(layers)

        def ptr(key):
            if weights.get(key) is None:
                return None
            a = np.ascontiguousarray(weights[key], dtype=np.uint8)
            self._keep.append(a)
            return a.ctypes.data

        s.embed = ptr("embed") if is_first else None
        s.embed_quant = QUANT[weights.get("embedQuant") or weights.get("quant") or "q4_0"]
        s.norm = ptr("norm") if is_last else None
        s.lm_head = ptr("lm_head") if is_last else None
        s.lm_head_quant = QUANT[weights.get("lmHeadQuant") or weights.get("quant") or "q4_0"]
        s.n_threads = n_threads or threads()
        self._spec = s
        self.h = lib.ref_init(C.byref(s))
        if not self.h:
            raise ValueError("ref_init failed")
        # not part of the reference: K / V rows stored as binary16 or fp8 e4m3,
        # the opt-in cache formats of the GPU stage (TN_FLAG_KV_F16 / _F8)
        if kv_dtype != "f32":
            lib.ref_set_kv_format(self.h, KV_FORMAT[kv_dtype])

    def forward(self, seq_id: int, token_pos: int, token_ids=None, hidden=None, temperature: float = 0.0,
                top_p: float = 0.95, u: float = 0.0) -> dict:
        lib = load()
        if self.is_first:
            ids = np.ascontiguousarray(np.asarray(token_ids, dtype=np.int32))
            n, ids_p, hid_p = ids.size, ids.ctypes.data, None
        else:
            hid = np.ascontiguousarray(np.asarray(hidden, dtype=np.uint16).reshape(-1))
            n, ids_p, hid_p = hid.size // self.H, None, hid.ctypes.data
        out_h = np.zeros(self.H, dtype=np.uint16)
        out_f = np.zeros(self.H, dtype=np.float32)
        logits = np.zeros(self.vocab, dtype=np.float32) if self.is_last else None
        tok = C.c_int32(-1)
        rc = lib.ref_forward(self.h, seq_id, token_pos, ids_p, hid_p, n, temperature, top_p, u,
                             out_h.ctypes.data, C.byref(tok), out_f.ctypes.data,
                             logits.ctypes.data if logits is not None else None)
        if rc != 0:
            raise ValueError(f"ref_forward failed ({rc})")
        res = {"hidden_f32": out_f}
        if self.is_last:
            res["token_id"] = int(tok.value)
            res["logits"] = logits
        else:
            res["hidden"] = out_h
        return res

    def kv_len(self, seq_id: int) -> int:
        return int(load().ref_kv_len(self.h, seq_id))

    def kv_row(self, seq_id: int, layer: int, s: int, kv_dim: int):
        k = np.zeros(kv_dim, dtype=np.float32)
        v = np.zeros(kv_dim, dtype=np.float32)
        if load().ref_kv_row(self.h, seq_id, layer, s, k.ctypes.data, v.ctypes.data) != 0:
            raise IndexError("no such KV row")
        return k, v

    def free(self) -> None:
        if self.h:
            load().ref_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
