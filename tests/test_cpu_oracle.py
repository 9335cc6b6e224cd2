"""The oracle against the hand-derived known-answer fixtures of tests/golden/
(the reference has no golden vectors of its own), plus CPU self-consistency
checks of the restatement (no GPU)."""
import json
import struct
from pathlib import Path

import numpy as np
import pytest

GOLD = Path(__file__).resolve().parent / "golden"


def bits_to_f32(s: str) -> float:
    return struct.unpack("<f", struct.pack("<I", int(s, 16)))[0]


def test_f32_to_f16_kats(ref, pkg):
    kat = json.loads((GOLD / "kat_f16.json").read_text())
    lib = pkg._lib.load()
    for src, want, why in kat["f32_to_f16"]:
        v = bits_to_f32(src)
        assert ref.f32_to_f16(v) == int(want, 16), (src, why)
        assert lib.tn_hop_encode_host(v) == int(want, 16), (src, why)


def test_f16_to_f32_kats(ref):
    kat = json.loads((GOLD / "kat_f16.json").read_text())
    for src, want, why in kat["f16_to_f32"]:
        got = np.float32(ref.f16_to_f32(int(src, 16))).view(np.uint32)
        assert int(got) == int(want, 16), (src, why)


def test_quant_kats(ref):
    kat = json.loads((GOLD / "kat_quant.json").read_text())
    for q in ("q4_0", "q8_0"):
        k = kat[q]
        got = ref.dequant(np.array(k["bytes"], dtype=np.uint8), q, k["count"])
        assert got.tolist() == k["expected"], k["derivation"]
    s = kat["straddle"]
    buf = np.array(s["bytes"], dtype=np.uint8)
    got = ref.dequant(buf, s["quant"], s["cols"], start=s["cols"])
    assert got.tolist() == s["expected_row1"], s["derivation"]
    # a matvec over straddling rows reads exactly those values
    x = np.ones(s["cols"], dtype=np.float32)
    y = ref.matvec(buf, s["quant"], s["rows"], s["cols"], x)
    assert y[1] == np.float32(sum(s["expected_row1"]))


def test_sizes_kats(ref, pkg):
    kat = json.loads((GOLD / "kat_quant.json").read_text())["sizes"]
    for n, q, want in kat["quant_bytes"]:
        assert ref.quant_bytes(n, q) == want
    for H, want in kat["round_ffn"]:
        assert ref.load().ref_round_ffn(H) == want
    for name, want in kat["layer_bytes"].items():
        assert pkg.pack.layer_layout(pkg.pack.MODELS[name])["total"] == want


def test_sample_kats(ref):
    for k in json.loads((GOLD / "kat_sample.json").read_text()):
        got = ref.sample(np.array(k["logits"], dtype=np.float32), k["temperature"], k["top_p"], k["u"])
        assert got == k["expected"], k["derivation"]


def test_rope_position_zero_is_identity(ref):
    v = np.random.default_rng(0).standard_normal(4 * 64).astype(np.float32)
    assert np.array_equal(ref.rope(v, 4, 64, 0, 10000.0), v)


def test_rope_rotates_pairs(ref):
    """Half-split pairing (i, i + hd/2) with angle pos * theta^(-2i/hd)."""
    hd, pos, theta = 8, 3, 10000.0
    v = np.arange(1, hd + 1, dtype=np.float32)
    out = ref.rope(v, 1, hd, pos, theta)
    for i in range(hd // 2):
        ang = pos * theta ** (-2 * i / hd)
        a, b = float(v[i]), float(v[i + hd // 2])
        assert out[i] == np.float32(a * np.cos(ang) - b * np.sin(ang))
        assert out[i + hd // 2] == np.float32(a * np.sin(ang) + b * np.cos(ang))


def test_single_position_attention_returns_v(ref):
    rng = np.random.default_rng(1)
    nH, nKV, hd = 8, 2, 32
    q = rng.standard_normal(nH * hd).astype(np.float32)
    K = rng.standard_normal((1, nKV * hd)).astype(np.float32)
    V = rng.standard_normal((1, nKV * hd)).astype(np.float32)
    out = ref.attention(q, K, V, nH, nKV, hd)
    for h in range(nH):
        kvh = h // (nH // nKV)
        assert np.array_equal(out[h * hd:(h + 1) * hd], V[0, kvh * hd:(kvh + 1) * hd])


def test_stage_split_equals_whole_model_without_hops(ref, pkg):
    """Two oracle stages joined by hidden states must reproduce a single stage
    up to the fp16 hop rounding (the hop is the only extra rounding)."""
    m = pkg.pack.MODELS["tiny"]
    w = pkg.pack.synth_weights(m, 0, m.n_layers, True, True)
    whole = ref.RefStage(m.dims(), 0, 4, True, True, w)
    wa = dict(w, layers=w["layers"][:2])
    wb = dict(w, layers=w["layers"][2:])
    a = ref.RefStage(m.dims(), 0, 2, True, False, wa)
    b = ref.RefStage(m.dims(), 2, 4, False, True, wb)
    prompt = pkg.pack.synth_prompt(m, 6)
    for p, t in enumerate(prompt):
        hw = whole.forward(1, p, token_ids=[t])
        ha = a.forward(1, p, token_ids=[t])
        hb = b.forward(1, p, hidden=ha["hidden"])
        err = np.max(np.abs(hw["hidden_f32"] - hb["hidden_f32"])) / np.max(np.abs(hw["hidden_f32"]))
        assert err < 1e-2, (p, err)


def test_tiny_greedy_fixture_matches_oracle(ref, pkg):
    g = json.loads((GOLD / "tiny_greedy.json").read_text())
    m = pkg.pack.MODELS["tiny"]
    assert g["prompt"] == pkg.pack.synth_prompt(m, 32)
    w = pkg.pack.synth_weights(m, 0, m.n_layers, True, True)
    st = ref.RefStage(m.dims(), 0, 4, True, True, w)
    r = st.forward(1, 0, token_ids=g["prompt"])
    toks = [r["token_id"]]
    for s in range(8):
        toks.append(st.forward(1, 32 + s, token_ids=[toks[-1]])["token_id"])
    assert toks == g["tokens"][:9]


def test_oracle_fp16_kv_rows_are_rounded_f32_rows(ref, pkg):
    """The oracle's fp16-cache mode (the GPU stage's opt-in TN_FLAG_KV_F16
    format; the reference keeps f32) stores each K / V value rounded to the
    nearest binary16, ties to even -- numpy's float16 conversion.  Layer 0 of
    position 0 sees identical inputs in both modes, so its rows compare
    exactly; the sampled token of a short prompt stays the same."""
    m = pkg.pack.MODELS["tiny"]
    w = pkg.pack.synth_weights(m, 0, m.n_layers, True, True)
    kv_dim = m.n_kv_heads * (m.hidden_dim // m.n_heads)
    full = ref.RefStage(m.dims(), 0, m.n_layers, True, True, w)
    half = ref.RefStage(m.dims(), 0, m.n_layers, True, True, w, kv_dtype="f16")
    prompt = pkg.pack.synth_prompt(m, 5)
    a = full.forward(1, 0, token_ids=prompt)
    b = half.forward(1, 0, token_ids=prompt)
    for s in range(len(prompt)):
        k32, v32 = full.kv_row(1, 0, s, kv_dim)
        k16, v16 = half.kv_row(1, 0, s, kv_dim)
        if s == 0:
            assert np.array_equal(k16, k32.astype(np.float16).astype(np.float32))
            assert np.array_equal(v16, v32.astype(np.float16).astype(np.float32))
        assert np.array_equal(k16, k16.astype(np.float16).astype(np.float32))  # every row holds fp16 values
    assert b["token_id"] == a["token_id"]
    assert float(np.max(np.abs(b["logits"] - a["logits"])) / np.max(np.abs(a["logits"]))) < 1e-2


def test_oracle_e4m3_rounding_matches_torch(ref):
    """The oracle's fp8 e4m3 rounding (the GPU stage's opt-in TN_FLAG_KV_F8
    cache format) against torch's float8_e4m3fn conversion: nearest, ties to
    even, subnormals down to 2^-9, saturating to +-448 (torch is given the
    clipped value; it does not saturate)."""
    import torch
    lib = ref.load()
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.standard_normal(4000).astype(np.float32) * s for s in (1e-3, 1e-2, 0.1, 1, 10, 100)])
    edge = [0.0, -0.0, 2.0 ** -6, 2.0 ** -7, 2.0 ** -9, 2.0 ** -10, 1.5 * 2 ** -10, 2.5 * 2 ** -9, 3.5 * 2 ** -9,
            1.0625, 1.1875, 447.0, 448.0, 449.0, 463.9, 464.0, 480.0, 1e6, -1e6]
    x = np.concatenate([x, np.array(edge, np.float32)])
    got = np.array([lib.ref_round_kv(2, float(v)) for v in x], np.float32)
    want = torch.from_numpy(np.clip(x, -448, 448)).to(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(got, want)
    assert lib.ref_round_kv(2, float("inf")) == 448.0 and np.isnan(lib.ref_round_kv(2, float("nan")))


def test_oracle_fp8_kv_rows_are_e4m3_values(ref, pkg):
    """With the fp8-cache mode every stored K / V value is an e4m3 value and
    layer 0 of position 0 holds exactly the rounded f32 rows."""
    import torch
    m = pkg.pack.MODELS["tiny"]
    w = pkg.pack.synth_weights(m, 0, m.n_layers, True, True)
    kv_dim = m.n_kv_heads * (m.hidden_dim // m.n_heads)
    full = ref.RefStage(m.dims(), 0, m.n_layers, True, True, w)
    q8 = ref.RefStage(m.dims(), 0, m.n_layers, True, True, w, kv_dtype="f8")
    prompt = pkg.pack.synth_prompt(m, 5)
    full.forward(1, 0, token_ids=prompt)
    q8.forward(1, 0, token_ids=prompt)

    def e4m3(a):
        return torch.from_numpy(np.clip(a, -448, 448)).to(torch.float8_e4m3fn).float().numpy()

    for s in range(len(prompt)):
        k32, v32 = full.kv_row(1, 0, s, kv_dim)
        k8, v8 = q8.kv_row(1, 0, s, kv_dim)
        if s == 0:
            assert np.array_equal(k8, e4m3(k32)) and np.array_equal(v8, e4m3(v32))
        assert np.array_equal(k8, e4m3(k8)) and np.array_equal(v8, e4m3(v8))
