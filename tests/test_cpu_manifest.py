"""Model packs (models/README.md): objects `<base>.<cid>.bin` + manifest.json
as tools/shard-model.js writes them, read back into initStage's weights object
as web/shard-loader.js assembles it, with SHA-256 cid verification."""
import hashlib
import json

import numpy as np
import pytest


@pytest.fixture(scope="module")
def tiny(pkg):
    m = pkg.pack.MODELS["tiny"]
    return m, pkg.pack.synth_weights(m, 0, m.n_layers, True, True)


def _split(pkg, m, buf):
    cut = pkg.pack.layer_layout(m)["tensors"]["ffn_norm"][0]  # attention tensors, then the MLP's
    return [("attn", buf[:cut]), ("mlp", buf[cut:])]


@pytest.fixture(scope="module")
def packdir(pkg, tiny, tmp_path_factory):
    m, w = tiny
    d = tmp_path_factory.mktemp("pack")
    layers = [l["buf"] for l in w["layers"]]
    layers[1] = _split(pkg, m, layers[1])
    man = pkg.manifest.write_pack(d, "tiny", m.dims(), layers, embed=w["embed"], norm=w["norm"], lm_head=w["lm_head"],
                                  quant=m.quant, embed_quant=m.embed_quant, lm_head_quant=m.lm_head_quant,
                                  ffn_dim=m.ffn_dim)
    return d, man


def test_normalize_cid(pkg):
    h = "ab" * 32
    nc = pkg.manifest.normalize_cid
    assert nc(h) == h and nc(h.upper()) == h
    assert nc("sha256:" + h) == h and nc("SHA-256-" + h) == h and nc("sha256-" + h) == h
    assert nc("bafybeigdyrzt5sfp7udm7hu76uh7y26nf3efuylqabf3oclgtqy55fbzdi") is None
    assert nc(h[:-1]) is None and nc("sha512:" + h) is None


def test_written_pack_layout(pkg, tiny, packdir):
    m, w = tiny
    d, man = packdir
    text = (d / "manifest.json").read_text()
    assert text.startswith('{\n  "model_id": "tiny",\n  "arch": "llama",\n  "n_layers": 4,\n  "hidden_dim": 256,')
    assert '\n  "rope_theta": 10000,\n' in text  # a JS number, not 10000.0
    parsed = json.loads(text)
    assert list(parsed) == ["model_id", "arch", "n_layers", "hidden_dim", "n_heads", "n_kv_heads", "vocab",
                            "rope_theta", "quant", "layers", "embed", "norm", "lm_head", "approx_weight_bytes",
                            "ffn_dim"]
    assert pkg.frame.js_stringify(parsed, 2) == text
    assert list(parsed["layers"][0]) == ["idx", "quant", "cid", "file", "bytes"]
    assert list(parsed["layers"][1]) == ["idx", "quant", "parts", "bytes"]
    assert [p["role"] for p in parsed["layers"][1]["parts"]] == ["attn", "mlp"]
    for L in parsed["layers"]:
        for o in L.get("parts", [L]):
            data = (d / o["file"]).read_bytes()
            assert hashlib.sha256(data).hexdigest() == o["cid"] and len(data) == o["bytes"]
            assert o["file"].endswith(f".{o['cid']}.bin")
    assert parsed["layers"][1]["bytes"] == len(w["layers"][1]["buf"])
    assert parsed["approx_weight_bytes"] == sum(len(l["buf"]) for l in w["layers"]) + \
        len(w["embed"]) + len(w["lm_head"]) + len(w["norm"])


def test_load_stage_bytes(pkg, tiny, packdir):
    m, w = tiny
    d, _ = packdir
    got = pkg.manifest.load_stage(d, 0, m.n_layers, need_embed=True, need_lm_head=True)
    assert [l["idx"] for l in got["layers"]] == list(range(m.n_layers))
    for a, b in zip(got["layers"], w["layers"]):
        assert np.array_equal(a["buf"], np.frombuffer(bytes(b["buf"]), dtype=np.uint8)) and a["quant"] == m.quant
    for k in ("embed", "norm", "lm_head"):
        assert np.array_equal(got[k], np.frombuffer(bytes(w[k]), dtype=np.uint8)), k
    assert got["embedQuant"] == m.embed_quant and got["lmHeadQuant"] == m.lm_head_quant
    assert got["dims"] == m.dims()
    mid = pkg.manifest.load_stage(d, 1, 3)
    assert [l["idx"] for l in mid["layers"]] == [1, 2] and "embed" not in mid and "lm_head" not in mid


def test_loaded_pack_runs_like_memory(pkg, ref, tiny, packdir):
    m, w = tiny
    d, _ = packdir
    got = pkg.manifest.load_stage(d, 0, m.n_layers, need_embed=True, need_lm_head=True)
    a = ref.RefStage(m.dims(), 0, m.n_layers, True, True, w)
    b = ref.RefStage(got["dims"], 0, m.n_layers, True, True, got)
    prompt = pkg.pack.synth_prompt(m, 6, seed=5)
    ta = a.forward(1, 0, token_ids=prompt)["token_id"]
    tb = b.forward(1, 0, token_ids=prompt)["token_id"]
    assert ta == tb
    for s in range(4):
        ta2 = a.forward(1, 6 + s, token_ids=[ta])["token_id"]
        tb2 = b.forward(1, 6 + s, token_ids=[tb])["token_id"]
        assert ta2 == tb2, s
        ta, tb = ta2, tb2


def test_integrity_and_errors(pkg, tiny, packdir, tmp_path):
    m, w = tiny
    d, man = packdir
    M = pkg.manifest
    # a corrupted object fails verification, and loads with verify=False
    bad = tmp_path / "bad"
    bad.mkdir()
    for f in d.iterdir():
        (bad / f.name).write_bytes(f.read_bytes())
    victim = bad / man["layers"][2]["file"]
    data = bytearray(victim.read_bytes())
    data[100] ^= 1
    victim.write_bytes(bytes(data))
    with pytest.raises(M.PackError, match="integrity check failed"):
        M.load_stage(bad, 2, 3)
    assert len(M.load_stage(bad, 2, 3, verify=False)["layers"][0]["buf"]) == len(data)
    with pytest.raises(M.PackError, match="out of bounds"):
        M.load_stage(d, 3, 5)
    with pytest.raises(M.PackError, match="empty layer range"):
        M.load_stage(d, 2, 2)
    # a non-hash cid scheme is trusted; byte_range selects [first, last] of a packed file
    blob = tmp_path / "two.bin"
    l0, l3 = bytes(w["layers"][0]["buf"]), bytes(w["layers"][3]["buf"])
    blob.write_bytes(l0 + l3)
    man2 = {"layers": [{"idx": 0, "quant": m.quant, "cid": "bafy-not-a-hash", "file": "two.bin",
                        "byte_range": [0, len(l0) - 1]},
                       {"idx": 1, "quant": m.quant, "cid": hashlib.sha256(l3).hexdigest(), "file": "two.bin",
                        "byte_range": [len(l0), len(l0) + len(l3) - 1]}]}
    got = M.load_stage((man2, tmp_path), 0, 2)
    assert bytes(got["layers"][0]["buf"]) == l0 and bytes(got["layers"][1]["buf"]) == l3
    with pytest.raises(M.PackError, match="no cid"):
        M.load_stage(({"layers": [{"idx": 0, "file": "two.bin"}]}, tmp_path), 0, 1)
