"""Model-pack layout and seeded synthetic packs.

Layout math restates web/inference-worker.js:130-163 (quantBytesFor,
layerLayout, roundFfn).  Synthetic weights come from the engine library's
counter-based generator (tn_synth_*), which writes the reference byte layout
on the host or directly in device memory with identical bytes; the reference
itself ships no quantiser or runnable pack (tools/shard-model.js:5-7).
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field

import numpy as np

from . import _lib

QK = 32  # web/inference-worker.js:101
NORM_TENSORS = ("attn_norm", "ffn_norm")
TENSORS = ("attn_norm", "wq", "wk", "wv", "wo", "ffn_norm", "w_gate", "w_up", "w_down")


def quant_bytes(count: int, quant: str) -> int:
    """quantBytesFor (web/inference-worker.js:130-137)."""
    if quant == "f32":
        return count * 4
    if quant == "f16":
        return count * 2
    nblocks = -(-count // QK)
    if quant == "q8_0":
        return nblocks * (2 + QK)
    if quant == "q4_0":
        return nblocks * (2 + QK // 2)
    raise ValueError(f"unsupported quant {quant}")


def round_ffn(hidden: int) -> int:
    """roundFfn (web/inference-worker.js:160-163)."""
    x = (8 * hidden) // 3
    return -(-x // 256) * 256


@dataclass(frozen=True)
class ModelDims:
    hidden_dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    vocab: int
    ffn_dim: int
    rope_theta: float
    quant: str
    embed_quant: str
    lm_head_quant: str
    seed: int
    name: str = ""

    @property
    def head_dim(self) -> int:
        return self.hidden_dim // self.n_heads

    def dims(self) -> dict:
        """The reference's `dims` object (web/inference-worker.js:30)."""
        return {"hidden_dim": self.hidden_dim, "n_heads": self.n_heads, "n_kv_heads": self.n_kv_heads,
                "vocab": self.vocab, "rope_theta": self.rope_theta, "ffn_dim": self.ffn_dim}

    def c_dims(self) -> _lib.Dims:
        return _lib.Dims(self.hidden_dim, self.n_heads, self.n_kv_heads, self.vocab, self.ffn_dim)


# The workloads the engine is measured on (seeded synthetic weights):
#  tiny: 256-dim, 4 layers, 8/2 heads, SwiGLU 688, vocab 4096, q8_0, f32 embeddings
#  llama8b: Llama-3-8B shape, q4_0;  llama70b: Llama-3-70B shape, q4_0
MODELS = {
    "tiny": ModelDims(256, 4, 8, 2, 4096, 688, 10000.0, "q8_0", "f32", "q8_0", 0, "tiny"),
    "llama8b": ModelDims(4096, 32, 32, 8, 128256, 14336, 500000.0, "q4_0", "q4_0", "q4_0", 1, "llama8b"),
    "llama70b": ModelDims(8192, 80, 64, 8, 128256, 28672, 500000.0, "q4_0", "q4_0", "q4_0", 2, "llama70b"),
}


def layer_layout(m: ModelDims, quant: str | None = None) -> dict:
    """layerLayout + the offsets walk of dequantLayer (web/inference-worker.js:142-178)."""
    quant = quant or m.quant
    H, nH, nKV = m.hidden_dim, m.n_heads, m.n_kv_heads
    hd = H // nH
    q_dim, kv_dim = nH * hd, nKV * hd
    ffn = m.ffn_dim or round_ffn(H)
    counts = [H, H * q_dim, H * kv_dim, H * kv_dim, q_dim * H, H, H * ffn, H * ffn, ffn * H]
    off, offs = 0, {}
    for name, count in zip(TENSORS, counts):
        eff = "f16" if name in NORM_TENSORS else quant
        offs[name] = (off, count, eff)
        off += quant_bytes(count, eff)
    return {"H": H, "nH": nH, "nKV": nKV, "headDim": hd, "qDim": q_dim, "kvDim": kv_dim, "ffn": ffn,
            "tensors": offs, "total": off}


def synth_layer(m: ModelDims, layer_idx: int, quant: str | None = None) -> np.ndarray:
    """One packed layer (host bytes) of the seeded synthetic model."""
    quant = quant or m.quant
    lib = _lib.load()
    n = layer_layout(m, quant)["total"]
    buf = np.empty(n, dtype=np.uint8)
    d = m.c_dims()
    _lib.check(lib.tn_synth_layer(m.seed, layer_idx, C.byref(d), _lib.QUANT[quant], buf.ctypes.data, 0, None))
    return buf


def synth_tensor(m: ModelDims, tag: str) -> np.ndarray:
    """embed / lm_head ([vocab x H] in their quant) or the final norm ([H] f16)."""
    lib = _lib.load()
    code = {"embed": _lib.TN_TAG_EMBED, "norm": _lib.TN_TAG_NORM, "lm_head": _lib.TN_TAG_LM_HEAD}[tag]
    quant = {"embed": m.embed_quant, "norm": "f16", "lm_head": m.lm_head_quant}[tag]
    count = m.hidden_dim if tag == "norm" else m.vocab * m.hidden_dim
    buf = np.empty(quant_bytes(count, quant), dtype=np.uint8)
    d = m.c_dims()
    _lib.check(lib.tn_synth_tensor(m.seed, code, C.byref(d), _lib.QUANT[quant], buf.ctypes.data, 0, None))
    return buf


def synth_device(m: ModelDims, what: str | int, out_ptr: int, stream: int | None = None) -> None:
    """Write a layer (int index) or a whole-model tensor directly into device memory."""
    lib = _lib.load()
    d = m.c_dims()
    if isinstance(what, int):
        _lib.check(lib.tn_synth_layer(m.seed, what, C.byref(d), _lib.QUANT[m.quant], out_ptr, 1, stream))
    else:
        code = {"embed": _lib.TN_TAG_EMBED, "norm": _lib.TN_TAG_NORM, "lm_head": _lib.TN_TAG_LM_HEAD}[what]
        quant = {"embed": m.embed_quant, "norm": "f16", "lm_head": m.lm_head_quant}[what]
        _lib.check(lib.tn_synth_tensor(m.seed, code, C.byref(d), _lib.QUANT[quant], out_ptr, 1, stream))


def tensor_bytes(m: ModelDims, what: str | int) -> int:
    if isinstance(what, int):
        return layer_layout(m)["total"]
    if what == "norm":
        return 2 * m.hidden_dim
    quant = m.embed_quant if what == "embed" else m.lm_head_quant
    return quant_bytes(m.vocab * m.hidden_dim, quant)


def synth_weights(m: ModelDims, lo: int, hi: int, is_first: bool, is_last: bool) -> dict:
    """The reference `weights` object (web/shard-loader.js:16-22) for layers [lo, hi)."""
    w = {"arch": "llama", "dims": m.dims(), "quant": m.quant,
         "layers": [{"idx": i, "buf": synth_layer(m, i), "quant": m.quant} for i in range(lo, hi)]}
    if is_first:
        w["embed"] = synth_tensor(m, "embed")
        w["embedQuant"] = m.embed_quant
    if is_last:
        w["norm"] = synth_tensor(m, "norm")
        w["lm_head"] = synth_tensor(m, "lm_head")
        w["lmHeadQuant"] = m.lm_head_quant
    return w


def synth_prompt(m: ModelDims, n: int, seed: int | None = None) -> list[int]:
    """Uniform random token ids in [0, vocab) from the model seed."""
    rng = np.random.default_rng(m.seed if seed is None else seed)
    return [int(t) for t in rng.integers(0, m.vocab, size=n)]


def layer_weight_bytes(m: ModelDims) -> int:
    return layer_layout(m)["total"]


def model_bytes(m: ModelDims) -> int:
    """Packed bytes streamed by a whole-model decode step (layers + lm_head)."""
    return m.n_layers * layer_weight_bytes(m) + quant_bytes(m.vocab * m.hidden_dim, m.lm_head_quant)
