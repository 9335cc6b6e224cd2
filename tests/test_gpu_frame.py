"""B200 stages on the reference's activation frames (web/protocol.js:101-120,
web/tabnet-node.js:140-193): three stages of the tiny model hop frames and
must return what direct forward calls on the hidden arrays return -- the same
payload bits, the same frame meta, the same greedy tokens."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny(pkg):
    m = pkg.pack.MODELS["tiny"]
    return m, pkg.pack.synth_weights(m, 0, m.n_layers, True, True)


def _stage(pkg, m, w, lo, hi, first, last):
    sub = {k: v for k, v in w.items() if k != "layers"}
    sub["layers"] = [l for l in w["layers"] if lo <= l["idx"] < hi]
    return pkg.initStage({"arch": "llama", "dims": m.dims(), "layers": [lo, hi], "is_first": first,
                          "is_last": last, "weights": sub, "opts": {"max_ctx": 128, "max_seqs": 2, "device": 0}})


def test_frame_hops_match_direct_forward(pkg, tiny):
    m, w = tiny
    fr = pkg.frame
    cuts = [(0, 1, True, False), (1, 3, False, False), (3, m.n_layers, False, True)]
    via_frames = [_stage(pkg, m, w, *c) for c in cuts]
    direct = [_stage(pkg, m, w, *c) for c in cuts]
    H = m.hidden_dim
    prompt = pkg.pack.synth_prompt(m, 12, seed=11)
    pos = len(prompt) - 1
    # stage 0 prefills and frames the last position (web/tabnet-node.js:167-169)
    h0 = pkg.forward(via_frames[0], {"seq_id": "s", "token_pos": 0, "token_ids": prompt})["hidden"]
    d0 = pkg.forward(direct[0], {"seq_id": "s", "token_pos": 0, "token_ids": prompt})["hidden"]
    assert np.array_equal(h0, d0)
    for step in range(6):
        frame0 = fr.encode_activation(fr.activation_meta("run1", "tab-0", "s", pos, 0, 1, H), h0)
        frame1 = fr.forward_frame(via_frames[1], frame0, node="b200-1", stage=1)
        msg = fr.forward_frame(via_frames[2], frame1, node="b200-2", stage=2, temperature=0)
        d1 = pkg.forward(direct[1], {"seq_id": "s", "token_pos": pos, "hidden": d0})["hidden"]
        tok = pkg.forward(direct[2], {"seq_id": "s", "token_pos": pos, "hidden": d1, "temperature": 0})["token_id"]
        meta1, payload1 = fr.decode_activation(frame1)
        assert meta1 == fr.activation_meta("run1", "b200-1", "s", pos, 1, 2, H), step
        assert payload1 == d1.astype("<u2").tobytes(), step
        assert msg == fr.token_message("run1", "b200-2", "s", pos, tok), step
        # stage 0 embeds the sampled token at the next position (:173-182)
        pos += 1
        h0 = pkg.forward(via_frames[0], {"seq_id": "s", "token_pos": pos, "token_ids": [msg["token_id"]]})["hidden"]
        d0 = pkg.forward(direct[0], {"seq_id": "s", "token_pos": pos, "token_ids": [tok]})["hidden"]
        assert np.array_equal(h0, d0), step
    for c in via_frames + direct:
        pkg.freeStage(c)


def test_frame_rejects_other_dtypes(pkg, tiny):
    m, w = tiny
    fr = pkg.frame
    ctx = _stage(pkg, m, w, 1, 3, False, False)
    bad = fr.encode_activation({"seq_id": "s", "token_pos": 0, "dtype": "f32", "shape": [m.hidden_dim]},
                               np.zeros(m.hidden_dim, dtype=np.float32))
    with pytest.raises(ValueError):
        fr.forward_frame(ctx, bad, node="n", stage=1)
    pkg.freeStage(ctx)
