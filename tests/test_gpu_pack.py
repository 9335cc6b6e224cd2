"""initStage from a model pack on disk (manifest.json + content-addressed
objects, one layer split into attention / MLP parts): the same greedy tokens
as the stage built from the in-memory weights."""
import pytest

pytestmark = pytest.mark.gpu


def test_stage_from_pack_matches_memory(pkg, tmp_path):
    m = pkg.pack.MODELS["tiny"]
    w = pkg.pack.synth_weights(m, 0, m.n_layers, True, True)
    layers = [l["buf"] for l in w["layers"]]
    cut = pkg.pack.layer_layout(m)["tensors"]["ffn_norm"][0]
    layers[2] = [("attn", layers[2][:cut]), ("mlp", layers[2][cut:])]
    pkg.manifest.write_pack(tmp_path, "tiny", m.dims(), layers, embed=w["embed"], norm=w["norm"],
                            lm_head=w["lm_head"], quant=m.quant, embed_quant=m.embed_quant,
                            lm_head_quant=m.lm_head_quant, ffn_dim=m.ffn_dim)
    loaded = pkg.manifest.load_stage(tmp_path, 0, m.n_layers, need_embed=True, need_lm_head=True)
    opts = {"max_ctx": 64, "max_seqs": 1, "device": 0}
    spec = {"arch": "llama", "dims": m.dims(), "layers": [0, m.n_layers], "is_first": True, "is_last": True}
    a = pkg.initStage({**spec, "weights": w, "opts": opts})
    b = pkg.initStage({**spec, "dims": loaded["dims"], "weights": loaded, "opts": opts})
    prompt = pkg.pack.synth_prompt(m, 10, seed=8)
    ta = pkg.forward(a, {"seq_id": 0, "token_pos": 0, "token_ids": prompt, "temperature": 0})["token_id"]
    tb = pkg.forward(b, {"seq_id": 0, "token_pos": 0, "token_ids": prompt, "temperature": 0})["token_id"]
    assert ta == tb
    for s in range(8):
        ta = pkg.forward(a, {"seq_id": 0, "token_pos": 10 + s, "token_ids": [ta], "temperature": 0})["token_id"]
        tb = pkg.forward(b, {"seq_id": 0, "token_pos": 10 + s, "token_ids": [tb], "temperature": 0})["token_id"]
        assert ta == tb, s
    pkg.freeStage(a)
    pkg.freeStage(b)
