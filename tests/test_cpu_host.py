"""CPU tests of the host side: the C ABI library loads and exports every
symbol include/tabnet_stage.h declares; host-side codecs, layout math and the
synthetic pack writer agree with the oracle (no GPU needed)."""
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def header_symbols():
    text = (ROOT / "include" / "tabnet_stage.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tn_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg._lib.load()
    syms = header_symbols()
    assert len(syms) >= 25
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing
    bound = {name for name, _, _ in pkg._lib.SIGNATURES}
    assert set(syms) == bound, set(syms) ^ bound


def test_abi_version(pkg):
    assert pkg._lib.load().tn_abi_version() == 2


def test_layout_matches_oracle_and_library(pkg, ref):
    import ctypes as C

    lib = pkg._lib.load()
    for name in ("tiny", "llama8b", "llama70b"):
        m = pkg.pack.MODELS[name]
        for q in ("q4_0", "q8_0", "f16", "f32"):
            L = pkg.pack.layer_layout(m, q)
            d = m.c_dims()
            assert L["total"] == lib.tn_layer_bytes(C.byref(d), pkg._lib.QUANT[q])
    # packed layer bytes of each workload (web/inference-worker.js:142-159 layout with each model's dims)
    assert pkg.pack.layer_layout(pkg.pack.MODELS["tiny"])["total"] == 736_512
    assert pkg.pack.layer_layout(pkg.pack.MODELS["llama8b"])["total"] == 122_699_776
    assert pkg.pack.layer_layout(pkg.pack.MODELS["llama70b"])["total"] == 481_329_152
    for n in (1, 31, 32, 33, 688, 4096 * 4096):
        for q in ("q4_0", "q8_0", "f16", "f32"):
            assert pkg.pack.quant_bytes(n, q) == ref.quant_bytes(n, q) == lib.tn_quant_bytes(n, pkg._lib.QUANT[q])
    for H in (256, 2048, 4096, 8192, 100):
        assert pkg.pack.round_ffn(H) == ref.load().ref_round_ffn(H)


def _interesting_f32_bits(rng, n_random):
    """Every exponent with edge mantissas (ties, carries, masks) plus random patterns."""
    out = []
    for e in range(256):
        for mant in (0, 1, 0x1000, 0x0fff, 0x1001, 0x2000, 0x3000, 0x7fe000, 0x7ff000, 0x7fefff, 0x7fffff,
                     0x400000, 0x200000, 0x7ff800):
            for s in (0, 1):
                out.append((s << 31) | (e << 23) | mant)
    out.extend(rng.integers(0, 2**32, n_random, dtype=np.uint64).tolist())
    return np.array(out, dtype=np.uint64).astype(np.uint32)


def test_host_hop_encoder_matches_oracle(pkg, ref):
    lib = pkg._lib.load()
    bits = _interesting_f32_bits(np.random.default_rng(0), 200_000)
    f = bits.view(np.float32)
    want = ref.f32_to_f16_array(f)
    got = np.array([lib.tn_hop_encode_host(float(v)) for v in f[:20000]], dtype=np.uint16)
    assert np.array_equal(got, want[:20000])


def test_synth_deterministic_and_quantised(pkg, ref):
    m = pkg.pack.MODELS["tiny"]
    a = pkg.pack.synth_layer(m, 1)
    b = pkg.pack.synth_layer(m, 1)
    assert np.array_equal(a, b)
    assert not np.array_equal(a, pkg.pack.synth_layer(m, 2))
    L = pkg.pack.layer_layout(m)
    off, count, q = L["tensors"]["wq"]
    w = ref.dequant(a[off:], q, count)
    assert abs(float(w.std()) - 0.02) < 0.002 and abs(float(w.mean())) < 1e-3
    off, count, q = L["tensors"]["attn_norm"]
    nrm = ref.dequant(a[off:], q, count)
    assert abs(float(nrm.mean()) - 1.0) < 0.01
