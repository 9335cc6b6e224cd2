"""ctypes binding of libtabnet_stage.so (declarations mirror include/tabnet_stage.h).

Loading the library needs no GPU; every compute call does.  There is no CPU
fallback: if the shared library is missing, loading raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libtabnet_stage.so"

TN_ABI_VERSION = 2
TN_OK, TN_EINVAL, TN_ENOMEM, TN_ECUDA, TN_EUNSUPPORTED, TN_ECAPACITY, TN_ESTATE, TN_ETIMEOUT = (
    0, -1, -2, -3, -4, -5, -6, -7)
STATUS_NAMES = {0: "TN_OK", -1: "TN_EINVAL", -2: "TN_ENOMEM", -3: "TN_ECUDA", -4: "TN_EUNSUPPORTED",
                -5: "TN_ECAPACITY", -6: "TN_ESTATE", -7: "TN_ETIMEOUT"}
QUANT = {"f32": 0, "f16": 1, "q4_0": 2, "q8_0": 3}
TN_HOP_LAST, TN_HOP_ALL = 0, 1
TN_FLAG_NO_GRAPHS = 1
TN_FLAG_PROFILE = 2
TN_FLAG_NO_FUSED_DECODE = 4
TN_FLAG_KV_F16 = 8
TN_FLAG_KV_F8 = 16
PROF_CLASSES = ["matvec_qkv", "matvec_o", "matvec_gate_up", "matvec_down", "matvec_lm_head", "attention",
                "rmsnorm", "rope_kv", "other"]
TN_TAG_EMBED, TN_TAG_NORM, TN_TAG_LM_HEAD = 1, 2, 3


class TnError(RuntimeError):
    """A failing tn_* call: `code` is the TN_E* status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


class LayerWeights(C.Structure):
    _fields_ = [("idx", C.c_int32), ("quant", C.c_int32), ("buf", C.c_void_p), ("len", C.c_uint64)]


class StageSpec(C.Structure):
    _fields_ = [
        ("abi_version", C.c_uint32),
        ("hidden_dim", C.c_int32), ("n_heads", C.c_int32), ("n_kv_heads", C.c_int32), ("vocab", C.c_int32),
        ("ffn_dim", C.c_int32),
        ("rope_theta", C.c_double),
        ("layer_lo", C.c_int32), ("layer_hi", C.c_int32), ("is_first", C.c_int32), ("is_last", C.c_int32),
        ("layers", C.POINTER(LayerWeights)), ("n_layers", C.c_int32),
        ("embed", C.c_void_p), ("embed_len", C.c_uint64), ("embed_quant", C.c_int32),
        ("norm", C.c_void_p), ("norm_len", C.c_uint64),
        ("lm_head", C.c_void_p), ("lm_head_len", C.c_uint64), ("lm_head_quant", C.c_int32),
        ("weights_on_device", C.c_int32),
        ("device", C.c_int32), ("max_ctx", C.c_int32), ("max_seqs", C.c_int32),
        ("max_tokens_per_step", C.c_int32),
        ("flags", C.c_uint32),
        ("kv_page_tokens", C.c_int32), ("kv_pages", C.c_int32),
    ]


class FwdReq(C.Structure):
    _fields_ = [
        ("seq_id", C.c_uint64), ("token_pos", C.c_int32), ("n_tokens", C.c_int32),
        ("token_ids", C.POINTER(C.c_int32)), ("hidden", C.POINTER(C.c_uint16)),
        ("temperature", C.c_double), ("top_p", C.c_double), ("rng_seed", C.c_uint64),
        ("hop_mode", C.c_int32),
    ]


class FwdOut(C.Structure):
    _fields_ = [("hidden", C.POINTER(C.c_uint16)), ("hidden_cap_tokens", C.c_int32),
                ("n_hidden_tokens", C.c_int32), ("token_id", C.c_int32)]


class StepDesc(C.Structure):
    _fields_ = [
        ("n_seqs", C.c_int32), ("seq_ids", C.POINTER(C.c_uint64)), ("token_pos", C.POINTER(C.c_int32)),
        ("d_token_ids", C.c_void_p), ("d_hidden_in", C.c_void_p), ("d_hidden_out", C.c_void_p),
        ("d_token_out", C.c_void_p),
        ("temperature", C.c_double), ("top_p", C.c_double), ("rng_seed", C.c_uint64),
    ]


class StageInfo(C.Structure):
    _fields_ = [("weight_bytes", C.c_uint64), ("kv_bytes", C.c_uint64), ("scratch_bytes", C.c_uint64),
                ("packed_bytes", C.c_uint64), ("n_layers", C.c_int32), ("head_dim", C.c_int32),
                ("q_dim", C.c_int32), ("kv_dim", C.c_int32), ("ffn_dim", C.c_int32),
                ("graphs_captured", C.c_int32), ("launches_last_step", C.c_int32)]


class Dims(C.Structure):
    _fields_ = [("hidden_dim", C.c_int32), ("n_heads", C.c_int32), ("n_kv_heads", C.c_int32),
                ("vocab", C.c_int32), ("ffn_dim", C.c_int32)]


# (name, restype, argtypes) of every exported symbol of include/tabnet_stage.h
SIGNATURES = [
    ("tn_stage_init", C.c_int, [C.POINTER(StageSpec), C.POINTER(C.c_void_p)]),
    ("tn_stage_forward", C.c_int, [C.c_void_p, C.POINTER(FwdReq), C.POINTER(FwdOut)]),
    ("tn_stage_forward_batch", C.c_int, [C.c_void_p, C.POINTER(FwdReq), C.c_int32, C.POINTER(FwdOut)]),
    ("tn_stage_free_seq", C.c_int, [C.c_void_p, C.c_uint64]),
    ("tn_stage_kv_len", C.c_int32, [C.c_void_p, C.c_uint64]),
    ("tn_stage_free", None, [C.c_void_p]),
    ("tn_last_error", C.c_char_p, []),
    ("tn_stage_step_async", C.c_int, [C.c_void_p, C.POINTER(StepDesc), C.c_void_p]),
    ("tn_stage_stream", C.c_void_p, [C.c_void_p]),
    ("tn_stage_check", C.c_int, [C.c_void_p, C.c_void_p]),
    ("tn_stage_test_raise_kernel_error", C.c_int, [C.c_void_p]),
    ("tn_test_bounded_wait", C.c_int, [C.c_uint64]),
    ("tn_stage_get_info", C.c_int, [C.c_void_p, C.POINTER(StageInfo)]),
    ("tn_stage_peek", C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_uint64]),
    ("tn_stage_profile", C.c_int, [C.c_void_p, C.POINTER(C.c_double), C.POINTER(C.c_uint64), C.c_int32]),
    ("tn_stage_set_profile", C.c_int, [C.c_void_p, C.c_int32]),
    ("tn_matrix_create", C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_uint64,
                                   C.c_int32, C.POINTER(C.c_void_p)]),
    ("tn_matrix_matvec", C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p]),
    ("tn_matrix_dequant", C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p]),
    ("tn_matrix_device_bytes", C.c_uint64, [C.c_void_p]),
    ("tn_matrix_counter_sum", C.c_int, [C.c_void_p, C.POINTER(C.c_int64)]),
    ("tn_matrix_free", None, [C.c_void_p]),
    ("tn_attention_scratch_bytes", C.c_uint64, [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32]),
    ("tn_attention", C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                               C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                               C.c_void_p, C.c_uint64, C.c_void_p]),
    ("tn_attention_paged", C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                     C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                     C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint64, C.c_void_p]),
    ("tn_attention_f8", C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                  C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                  C.c_void_p, C.c_uint64, C.c_void_p]),
    ("tn_attention_f16", C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                   C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                   C.c_void_p, C.c_uint64, C.c_void_p]),
    ("tn_attention_static", C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                      C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                      C.c_void_p]),
    ("tn_hop_encode", C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.c_void_p]),
    ("tn_hop_decode", C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.c_void_p]),
    ("tn_hop_encode_host", C.c_uint16, [C.c_float]),
    ("tn_sample", C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_double, C.c_double, C.c_uint64,
                            C.c_void_p, C.c_void_p]),
    ("tn_sample_uniform", C.c_double, [C.c_uint64, C.c_uint64]),
    ("tn_layer_bytes", C.c_uint64, [C.POINTER(Dims), C.c_int32]),
    ("tn_quant_bytes", C.c_uint64, [C.c_uint64, C.c_int32]),
    ("tn_synth_layer", C.c_int, [C.c_uint64, C.c_int32, C.POINTER(Dims), C.c_int32, C.c_void_p, C.c_int32,
                                 C.c_void_p]),
    ("tn_synth_tensor", C.c_int, [C.c_uint64, C.c_int32, C.POINTER(Dims), C.c_int32, C.c_void_p, C.c_int32,
                                  C.c_void_p]),
    ("tn_abi_version", C.c_int, []),
]

_lib = None


def load() -> C.CDLL:
    """Load libtabnet_stage.so once; raises if it has not been built."""
    global _lib
    if _lib is None:
        path = Path(os.environ.get("TABNET_STAGE_LIB", LIB_PATH))
        if not path.exists():
            raise OSError(f"{path} not found: build it with `python __graft_entry__.py` "
                          "(the stage engine has no CPU fallback)")
        lib = C.CDLL(str(path))
        for name, res, args in SIGNATURES:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.tn_abi_version() != TN_ABI_VERSION:
            raise OSError(f"{path}: ABI version {lib.tn_abi_version()} != {TN_ABI_VERSION}")
        _lib = lib
    return _lib


def check(rc: int) -> None:
    if rc != TN_OK:
        raise TnError(rc, load().tn_last_error().decode(errors="replace"))
