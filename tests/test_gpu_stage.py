"""Stage-engine parity on the GPU through the C ABI (initStage / forward /
freeStage), against the oracle on identical seeded weights and prompts.

Greedy tokens must be identical; hidden states (fp16 hop frames, decoded)
within max|a-b| / max|b| <= 1e-3.
"""
import base64
import json
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HIDDEN_TOL = 1e-3
LOGIT_TOL = 1e-4  # max |a - b| / max |b| of a logits row (f32 accumulation vs the oracle's f64)


def f16(bits):
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def maxrel(a, b):
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


@pytest.fixture(scope="module")
def tiny(pkg):
    m = pkg.pack.MODELS["tiny"]
    return m, pkg.pack.synth_weights(m, 0, m.n_layers, True, True)


def _stage(pkg, m, w, lo, hi, first, last, **opts):
    sub = {k: v for k, v in w.items() if k != "layers"}
    sub["layers"] = [l for l in w["layers"] if lo <= l["idx"] < hi]
    o = {"max_ctx": 256, "max_seqs": 8, "device": 0}
    o.update(opts)
    return pkg.initStage({"arch": "llama", "dims": m.dims(), "layers": [lo, hi], "is_first": first,
                          "is_last": last, "weights": sub, "opts": o}), sub


@pytest.mark.parametrize("fused", [True, False])
def test_tiny_single_stage_greedy_64(pkg, ref, tiny, fused):
    m, w = tiny
    ctx, _ = _stage(pkg, m, w, 0, m.n_layers, True, True, fused_decode=fused)
    oracle = ref.RefStage(m.dims(), 0, m.n_layers, True, True, w)
    prompt = pkg.pack.synth_prompt(m, 32)
    got = pkg.forward(ctx, {"seq_id": "a", "token_pos": 0, "token_ids": prompt, "temperature": 0})["token_id"]
    want = oracle.forward(1, 0, token_ids=prompt)
    assert got == want["token_id"]
    toks = [got]
    assert maxrel(ctx.peek("logits", 1)[0], want["logits"]) <= LOGIT_TOL
    for s in range(64):
        pos = 32 + s
        got = pkg.forward(ctx, {"seq_id": "a", "token_pos": pos, "token_ids": [toks[-1]], "temperature": 0})
        want = oracle.forward(1, pos, token_ids=[toks[-1]])
        lg = np.sort(want["logits"])[::-1]
        assert got["token_id"] == want["token_id"], (s, "top-2 gap", lg[0] - lg[1])
        # every step's logits, not only their argmax (the greedy map of this
        # tiny model settles on a fixed point after a dozen steps)
        err = maxrel(ctx.peek("logits", 1)[0], want["logits"])
        assert err <= LOGIT_TOL, (s, err)
        toks.append(got["token_id"])
    assert pkg.kv_len(ctx, "a") == 32 + 64 == oracle.kv_len(1)
    pkg.freeStage(ctx)


# An fp8 cache value is one of 16 per binade, so an f32 K / V value that the
# GPU and the oracle compute a few ulps apart can land on either side of a
# rounding midpoint and differ by one e4m3 step (6 %); logits move by far
# less than this bound when that happens.
KV_LOGIT_TOL = {"f16": LOGIT_TOL, "f8": 2e-3}


@pytest.mark.parametrize("kv", ["f16", "f8"])
@pytest.mark.parametrize("fused", [True, False])
def test_tiny_kv_lowp_greedy_vs_oracle(pkg, ref, tiny, fused, kv):
    """The opt-in fp16 / fp8 e4m3 KV caches (TN_FLAG_KV_F16 / _F8; the
    reference keeps f32 rows) against the oracle storing the same rounded
    rows: greedy tokens identical and per-step logits within tolerance over
    32 steps, on the fused RoPE + KV-append epilogue and on the separate
    kernels.  The cache takes a half / a quarter of the f32 one's bytes."""
    m, w = tiny
    ctx, _ = _stage(pkg, m, w, 0, m.n_layers, True, True, fused_decode=fused, kv_dtype=kv)
    ref32, _ = _stage(pkg, m, w, 0, m.n_layers, True, True)
    assert ctx.info()["kv_bytes"] * (2 if kv == "f16" else 4) == ref32.info()["kv_bytes"]
    pkg.freeStage(ref32)
    tol = KV_LOGIT_TOL[kv]
    oracle = ref.RefStage(m.dims(), 0, m.n_layers, True, True, w, kv_dtype=kv)
    prompt = pkg.pack.synth_prompt(m, 24, seed=77)
    got = pkg.forward(ctx, {"seq_id": "h", "token_pos": 0, "token_ids": prompt, "temperature": 0})["token_id"]
    want = oracle.forward(1, 0, token_ids=prompt)
    assert got == want["token_id"]
    assert maxrel(ctx.peek("logits", 1)[0], want["logits"]) <= tol
    tok = got
    for s in range(32):
        pos = 24 + s
        got = pkg.forward(ctx, {"seq_id": "h", "token_pos": pos, "token_ids": [tok], "temperature": 0})
        want = oracle.forward(1, pos, token_ids=[tok])
        assert got["token_id"] == want["token_id"], s
        err = maxrel(ctx.peek("logits", 1)[0], want["logits"])
        assert err <= tol, (s, err)
        tok = got["token_id"]
    pkg.freeStage(ctx)


@pytest.mark.parametrize("fused", [True, False])
def test_tiny_paged_kv_matches_contiguous(pkg, ref, tiny, fused):
    """A paged KV cache (16-position pages from a shared pool) against the
    contiguous arena: three sequences decoded interleaved so that their pages
    interleave in the pool, one freed half way and its pages reused by a
    fourth.  Every step's logits are bitwise those of the contiguous stage
    (the same rows in the same order, only their addresses differ) and the
    greedy tokens those of the oracle."""
    m, w = tiny
    paged, _ = _stage(pkg, m, w, 0, m.n_layers, True, True, fused_decode=fused, kv_page_tokens=16, kv_pages=40)
    flat, _ = _stage(pkg, m, w, 0, m.n_layers, True, True, fused_decode=fused)
    assert paged.info()["kv_bytes"] * 256 * 8 == flat.info()["kv_bytes"] * 40 * 16
    oracles = {}
    toks, pos = {}, {}
    for i, sid in enumerate(["a", "b", "c"]):
        prompt = pkg.pack.synth_prompt(m, 5 + 9 * i, seed=40 + i)
        oracles[sid] = ref.RefStage(m.dims(), 0, m.n_layers, True, True, w)
        outs = []
        for ctx in (paged, flat):
            outs.append(pkg.forward(ctx, {"seq_id": sid, "token_pos": 0, "token_ids": prompt, "temperature": 0}))
            outs[-1]["logits"] = ctx.peek("logits", 1)[0].copy()
        assert np.array_equal(outs[0]["logits"], outs[1]["logits"])
        want = oracles[sid].forward(1, 0, token_ids=prompt)
        assert outs[0]["token_id"] == want["token_id"]
        toks[sid], pos[sid] = outs[0]["token_id"], len(prompt)
    for step in range(40):
        if step == 20:
            for ctx in (paged, flat):
                pkg.free_seq(ctx, "b")
            del toks["b"]
            prompt = pkg.pack.synth_prompt(m, 30, seed=99)
            oracles["d"] = ref.RefStage(m.dims(), 0, m.n_layers, True, True, w)
            for ctx in (paged, flat):
                r = pkg.forward(ctx, {"seq_id": "d", "token_pos": 0, "token_ids": prompt, "temperature": 0})
            assert r["token_id"] == oracles["d"].forward(1, 0, token_ids=prompt)["token_id"]
            toks["d"], pos["d"] = r["token_id"], len(prompt)
        for sid in list(toks):
            got = []
            for ctx in (paged, flat):
                got.append(pkg.forward(ctx, {"seq_id": sid, "token_pos": pos[sid], "token_ids": [toks[sid]],
                                             "temperature": 0})["token_id"])
                got.append(ctx.peek("logits", 1)[0].copy())
            assert np.array_equal(got[1], got[3]), (step, sid)
            want = oracles[sid].forward(1, pos[sid], token_ids=[toks[sid]])
            assert got[0] == got[2] == want["token_id"], (step, sid)
            assert maxrel(got[1], want["logits"]) <= LOGIT_TOL
            toks[sid], pos[sid] = got[0], pos[sid] + 1
    for sid in toks:
        assert pkg.kv_len(paged, sid) == pkg.kv_len(flat, sid) == pos[sid]
    pkg.freeStage(paged)
    pkg.freeStage(flat)


def test_tiny_paged_kv_pool_exhaustion(pkg, tiny):
    """A forward that needs more pages than the pool has left fails with
    TN_ECAPACITY and takes nothing: the pages of its new sequence and of a
    grown one go back, and freeing a sequence makes room again."""
    m, w = tiny
    ctx, _ = _stage(pkg, m, w, 0, m.n_layers, True, True, kv_page_tokens=16, kv_pages=4)
    pkg.forward(ctx, {"seq_id": "x", "token_pos": 0, "token_ids": pkg.pack.synth_prompt(m, 40), "temperature": 0})
    with pytest.raises(pkg._lib.TnError) as e:  # 3 pages held, 2 more needed
        pkg.forward(ctx, {"seq_id": "y", "token_pos": 0, "token_ids": pkg.pack.synth_prompt(m, 20, seed=2),
                          "temperature": 0})
    assert e.value.code == pkg._lib.TN_ECAPACITY
    assert pkg.kv_len(ctx, "y") == 0
    with pytest.raises(pkg._lib.TnError):  # one sequence growing past the pool, alongside a new one
        pkg.forward_batch(ctx, [{"seq_id": "x", "token_pos": 40, "token_ids": [1] * 9, "temperature": 0},
                                {"seq_id": "z", "token_pos": 0, "token_ids": [2], "temperature": 0}])
    assert pkg.kv_len(ctx, "x") == 40 and pkg.kv_len(ctx, "z") == 0
    pkg.forward(ctx, {"seq_id": "y", "token_pos": 0, "token_ids": [3] * 16, "temperature": 0})  # the 4th page
    pkg.free_seq(ctx, "x")
    pkg.forward(ctx, {"seq_id": "z", "token_pos": 0, "token_ids": [2] * 48, "temperature": 0})  # x's 3 pages
    assert pkg.kv_len(ctx, "z") == 48
    pkg.freeStage(ctx)


def test_tiny_two_stages_reference_hops(pkg, ref, tiny):
    """The reference runtime's hop semantics: prefill hops only the last
    position (web/tabnet-node.js:167-169), so stage 1's KV starts at one row."""
    m, w = tiny
    a, wa = _stage(pkg, m, w, 0, 2, True, False)
    b, wb = _stage(pkg, m, w, 2, 4, False, True)
    oa = ref.RefStage(m.dims(), 0, 2, True, False, wa)
    ob = ref.RefStage(m.dims(), 2, 4, False, True, wb)
    prompt = pkg.pack.synth_prompt(m, 24, seed=3)
    ha = pkg.forward(a, {"seq_id": "s", "token_pos": 0, "token_ids": prompt})["hidden"]
    ra = oa.forward(7, 0, token_ids=prompt)
    assert maxrel(f16(ha), f16(ra["hidden"])) <= HIDDEN_TOL
    pos = len(prompt) - 1
    tok = pkg.forward(b, {"seq_id": "s", "token_pos": pos, "hidden": ha, "temperature": 0})["token_id"]
    assert tok == ob.forward(7, pos, hidden=ha)["token_id"]
    for step in range(16):
        pos = len(prompt) + step
        ha = pkg.forward(a, {"seq_id": "s", "token_pos": pos, "token_ids": [tok]})["hidden"]
        ra = oa.forward(7, pos, token_ids=[tok])
        assert maxrel(f16(ha), f16(ra["hidden"])) <= HIDDEN_TOL, step
        tok2 = pkg.forward(b, {"seq_id": "s", "token_pos": pos, "hidden": ha, "temperature": 0})["token_id"]
        assert tok2 == ob.forward(7, pos, hidden=ha)["token_id"], step
        tok = tok2
    pkg.freeStage(a)
    pkg.freeStage(b)


def test_tiny_two_stages_hop_all(pkg, ref, tiny):
    """hop_mode all: every prompt position crosses the stage boundary, so the
    pipeline computes what one stage over all layers computes."""
    m, w = tiny
    a, wa = _stage(pkg, m, w, 0, 2, True, False, hop_mode="all")
    b, wb = _stage(pkg, m, w, 2, 4, False, True)
    oa = ref.RefStage(m.dims(), 0, 2, True, False, wa)
    ob = ref.RefStage(m.dims(), 2, 4, False, True, wb)
    prompt = pkg.pack.synth_prompt(m, 20, seed=4)
    hs = pkg.forward(a, {"seq_id": 9, "token_pos": 0, "token_ids": prompt})["hidden"]
    assert hs.shape == (20, m.hidden_dim)
    want = np.stack([oa.forward(9, p, token_ids=[prompt[p]])["hidden"] for p in range(20)])
    for p in range(20):
        assert maxrel(f16(hs[p]), f16(want[p])) <= HIDDEN_TOL, p
    tok = pkg.forward(b, {"seq_id": 9, "token_pos": 0, "hidden": hs, "temperature": 0})["token_id"]
    assert tok == ob.forward(9, 0, hidden=hs)["token_id"]
    assert pkg.kv_len(b, 9) == 20
    pkg.freeStage(a)
    pkg.freeStage(b)


@pytest.mark.parametrize("n_seqs", [2, 4, 6, 8])
def test_batch_equals_individual(pkg, ref, tiny, n_seqs):
    m, w = tiny
    one, _ = _stage(pkg, m, w, 0, m.n_layers, True, True)
    many, _ = _stage(pkg, m, w, 0, m.n_layers, True, True)
    prompts = [pkg.pack.synth_prompt(m, 5 + 3 * i, seed=10 + i) for i in range(n_seqs)]
    solo = [pkg.forward(one, {"seq_id": i, "token_pos": 0, "token_ids": p, "temperature": 0})["token_id"]
            for i, p in enumerate(prompts)]
    batch = pkg.forward_batch(many, [{"seq_id": i, "token_pos": 0, "token_ids": p, "temperature": 0}
                                     for i, p in enumerate(prompts)])
    assert [r["token_id"] for r in batch] == solo
    toks = list(solo)
    for step in range(12):
        reqs = [{"seq_id": i, "token_pos": len(prompts[i]) + step, "token_ids": [toks[i]], "temperature": 0}
                for i in range(n_seqs)]
        b = [r["token_id"] for r in pkg.forward_batch(many, reqs)]
        s = [pkg.forward(one, r)["token_id"] for r in reqs]
        assert b == s, step
        toks = b
    assert many.info()["graphs_captured"] >= 1
    pkg.freeStage(one)
    pkg.freeStage(many)


def test_chunked_prefill_matches(pkg, ref, tiny):
    """A prompt longer than max_tokens_per_step runs in several steps."""
    m, w = tiny
    ctx, _ = _stage(pkg, m, w, 0, m.n_layers, True, True, max_tokens_per_step=16)
    oracle = ref.RefStage(m.dims(), 0, m.n_layers, True, True, w)
    prompt = pkg.pack.synth_prompt(m, 45, seed=6)
    got = pkg.forward(ctx, {"seq_id": "c", "token_pos": 0, "token_ids": prompt, "temperature": 0})["token_id"]
    assert got == oracle.forward(1, 0, token_ids=prompt)["token_id"]
    pkg.freeStage(ctx)


def test_temperature_sampling_matches_oracle_draw(pkg, ref, tiny):
    m, w = tiny
    ctx, _ = _stage(pkg, m, w, 0, m.n_layers, True, True)
    oracle = ref.RefStage(m.dims(), 0, m.n_layers, True, True, w)
    lib = pkg._lib.load()
    prompt = pkg.pack.synth_prompt(m, 12, seed=8)
    seed = 4242
    got = pkg.forward(ctx, {"seq_id": "t", "token_pos": 0, "token_ids": prompt, "temperature": 0.8,
                            "top_p": 0.9, "rng_seed": seed})["token_id"]
    u = lib.tn_sample_uniform(seed, len(prompt) - 1)
    want = oracle.forward(1, 0, token_ids=prompt, temperature=0.8, top_p=0.9, u=u)["token_id"]
    assert got == want
    pkg.freeStage(ctx)


@pytest.mark.parametrize("page", [0, 16])
def test_device_step_matches_forward(pkg, ref, tiny, torch_cuda, page):
    """tn_stage_step_async (device token ids in and out) against forward; with
    16-position KV pages the steps cross into each sequence's second page,
    taken and copied to the device table on the step's stream."""
    torch = torch_cuda
    m, w = tiny
    lib = pkg._lib.load()
    import ctypes as C

    a, _ = _stage(pkg, m, w, 0, m.n_layers, True, True)
    b, _ = _stage(pkg, m, w, 0, m.n_layers, True, True, kv_page_tokens=page)
    prompts = [pkg.pack.synth_prompt(m, 6, seed=20 + i) for i in range(3)]
    toks = [pkg.forward(a, {"seq_id": i, "token_pos": 0, "token_ids": p, "temperature": 0})["token_id"]
            for i, p in enumerate(prompts)]
    for i, p in enumerate(prompts):
        pkg.forward(b, {"seq_id": i, "token_pos": 0, "token_ids": p, "temperature": 0})
    ids = (C.c_uint64 * 3)(*[b.seq_key(i) for i in range(3)])
    cur = list(toks)
    for step in range(12):
        pos = (C.c_int32 * 3)(*[6 + step] * 3)
        din = torch.tensor(cur, dtype=torch.int32, device="cuda")
        dout = torch.zeros(3, dtype=torch.int32, device="cuda")
        d = pkg._lib.StepDesc(n_seqs=3, seq_ids=ids, token_pos=pos, d_token_ids=din.data_ptr(),
                              d_token_out=dout.data_ptr(), temperature=0.0, top_p=0.95, rng_seed=0)
        pkg._lib.check(lib.tn_stage_step_async(b.handle, C.byref(d), None))
        torch.cuda.synchronize()
        want = [pkg.forward(a, {"seq_id": i, "token_pos": 6 + step, "token_ids": [cur[i]], "temperature": 0})
                ["token_id"] for i in range(3)]
        got = dout.cpu().tolist()
        assert got == want, step
        cur = got
    pkg.freeStage(a)
    pkg.freeStage(b)


def test_device_step_three_stages(pkg, tiny, torch_cuda):
    """The device-buffer step API (what the multi-GPU pipeline drives) on a
    first, a middle and a last stage: fp16 frames and tokens identical to the
    host API on a twin chain of stages."""
    torch = torch_cuda
    m, w = tiny
    lib = pkg._lib.load()
    import ctypes as C

    cuts = [(0, 1, True, False), (1, 3, False, False), (3, m.n_layers, False, True)]
    host = [_stage(pkg, m, w, *c)[0] for c in cuts]
    dev = [_stage(pkg, m, w, *c)[0] for c in cuts]
    prompt = pkg.pack.synth_prompt(m, 9, seed=31)
    pos = len(prompt) - 1
    for chain in (host, dev):  # prefill: stage 0 hops its last position (web/tabnet-node.js:167-169)
        h = pkg.forward(chain[0], {"seq_id": 5, "token_pos": 0, "token_ids": prompt})["hidden"]
        h = pkg.forward(chain[1], {"seq_id": 5, "token_pos": pos, "hidden": h})["hidden"]
        tok = pkg.forward(chain[2], {"seq_id": 5, "token_pos": pos, "hidden": h, "temperature": 0})["token_id"]
    H = m.hidden_dim
    d_tok = torch.tensor([tok], dtype=torch.int32, device="cuda")
    d_h1 = torch.zeros(H, dtype=torch.float16, device="cuda")
    d_h2 = torch.zeros(H, dtype=torch.float16, device="cuda")
    d_out = torch.zeros(1, dtype=torch.int32, device="cuda")
    chain_stream = torch.cuda.Stream()  # not the legacy default stream, whose handle 0 means "the stage's own"
    stream = chain_stream.cuda_stream
    torch.cuda.synchronize()  # the buffers above were filled on the default stream
    for step in range(6):
        pos += 1
        h1 = pkg.forward(host[0], {"seq_id": 5, "token_pos": pos, "token_ids": [tok]})["hidden"]
        h2 = pkg.forward(host[1], {"seq_id": 5, "token_pos": pos, "hidden": h1})["hidden"]
        tok = pkg.forward(host[2], {"seq_id": 5, "token_pos": pos, "hidden": h2, "temperature": 0})["token_id"]
        p = (C.c_int32 * 1)(pos)
        for i, ctx in enumerate(dev):
            ids = (C.c_uint64 * 1)(ctx.seq_key(5))
            d = pkg._lib.StepDesc(n_seqs=1, seq_ids=ids, token_pos=p, temperature=0.0, top_p=0.95, rng_seed=0)
            if i == 0:
                d.d_token_ids, d.d_hidden_out = d_tok.data_ptr(), d_h1.data_ptr()
            elif i == 1:
                d.d_hidden_in, d.d_hidden_out = d_h1.data_ptr(), d_h2.data_ptr()
            else:
                d.d_hidden_in, d.d_token_out = d_h2.data_ptr(), d_out.data_ptr()
            # one stream for the chain, so each stage reads the frame the previous one wrote
            pkg._lib.check(lib.tn_stage_step_async(ctx.handle, C.byref(d), C.c_void_p(stream)))
        torch.cuda.synchronize()
        assert np.array_equal(d_h1.cpu().numpy().view(np.uint16), h1), step
        assert np.array_equal(d_h2.cpu().numpy().view(np.uint16), h2), step
        assert int(d_out.item()) == tok, step
        with torch.cuda.stream(chain_stream):
            d_tok.copy_(d_out)
    for c in host + dev:
        pkg.freeStage(c)


def test_errors(pkg, tiny):
    m, w = tiny
    ctx, _ = _stage(pkg, m, w, 0, m.n_layers, True, True, max_ctx=16, max_seqs=2)
    E = pkg._lib.TnError
    with pytest.raises(E) as e:
        pkg.forward(ctx, {"seq_id": 1, "token_pos": 0, "token_ids": [m.vocab]})
    assert e.value.code == pkg._lib.TN_EINVAL
    with pytest.raises(E) as e:
        pkg.forward(ctx, {"seq_id": 1, "token_pos": 0, "token_ids": list(range(17))})
    assert e.value.code == pkg._lib.TN_ECAPACITY
    assert pkg.kv_len(ctx, 1) == 0  # a failed call leaves no KV behind
    pkg.forward(ctx, {"seq_id": 1, "token_pos": 0, "token_ids": [1], "temperature": 0})
    pkg.forward(ctx, {"seq_id": 2, "token_pos": 0, "token_ids": [1], "temperature": 0})
    with pytest.raises(E) as e:
        pkg.forward(ctx, {"seq_id": 3, "token_pos": 0, "token_ids": [1], "temperature": 0})
    assert e.value.code == pkg._lib.TN_ECAPACITY
    pkg.free_seq(ctx, 2)
    pkg.forward(ctx, {"seq_id": 3, "token_pos": 0, "token_ids": [1], "temperature": 0})
    with pytest.raises(E) as e:
        pkg.forward(ctx, {"seq_id": 1, "token_pos": 1, "hidden": np.zeros(m.hidden_dim, np.uint16)})
    assert e.value.code == pkg._lib.TN_ESTATE
    pkg.freeStage(ctx)
    bad = dict(w)
    bad["layers"] = [dict(l, quant="q5_1") for l in w["layers"]]
    with pytest.raises(E) as e:
        _stage(pkg, m, bad, 0, m.n_layers, True, True)
    assert "unsupported quant q5_1" in str(e.value)


@pytest.mark.parametrize("name,lo,hi,first,last", [("llama8b", 0, 2, True, False), ("llama70b", 40, 41, False, False)])
def test_large_shape_slices(pkg, ref, name, lo, hi, first, last):
    """Layer slices of the 8B and 70B shapes: stage output hidden states
    against the oracle over a short prefill."""
    m = pkg.pack.MODELS[name]
    w = {"arch": "llama", "dims": m.dims(), "quant": m.quant,
         "layers": [{"idx": i, "buf": pkg.pack.synth_layer(m, i), "quant": m.quant} for i in range(lo, hi)]}
    if first:
        w["embed"] = pkg.pack.synth_tensor(m, "embed")
        w["embedQuant"] = m.embed_quant
    ctx = pkg.initStage({"arch": "llama", "dims": m.dims(), "layers": [lo, hi], "is_first": first,
                         "is_last": last, "weights": w,
                         "opts": {"max_ctx": 64, "max_seqs": 2, "device": 0, "hop_mode": "all"}})
    oracle = ref.RefStage(m.dims(), lo, hi, first, last, w)
    n = 6
    if first:
        prompt = pkg.pack.synth_prompt(m, n, seed=9)
        got = pkg.forward(ctx, {"seq_id": 0, "token_pos": 0, "token_ids": prompt})["hidden"]
        want = [oracle.forward(1, p, token_ids=[prompt[p]])["hidden"] for p in range(n)]
    else:
        rng = np.random.default_rng(11)
        hid = rng.standard_normal((n, m.hidden_dim)).astype(np.float16).view(np.uint16)
        got = pkg.forward(ctx, {"seq_id": 0, "token_pos": 0, "hidden": hid})["hidden"]
        want = [oracle.forward(1, p, hidden=hid[p])["hidden"] for p in range(n)]
    for p in range(n):
        assert maxrel(f16(got[p]), f16(want[p])) <= HIDDEN_TOL, p
    # single-token decode steps (the fused decode kernels) continue the sequence
    for step in range(3):
        pos = n + step
        if first:
            tok = int((step * 7919 + 11) % m.vocab)
            got = pkg.forward(ctx, {"seq_id": 0, "token_pos": pos, "token_ids": [tok]})["hidden"]
            want = oracle.forward(1, pos, token_ids=[tok])["hidden"]
        else:
            h1 = (np.random.default_rng(pos).standard_normal(m.hidden_dim)).astype(np.float16).view(np.uint16)
            got = pkg.forward(ctx, {"seq_id": 0, "token_pos": pos, "hidden": h1})["hidden"]
            want = oracle.forward(1, pos, hidden=h1)["hidden"]
        assert maxrel(f16(got), f16(want)) <= HIDDEN_TOL, ("decode", step)
    pkg.freeStage(ctx)
    oracle.free()


def _device_weights(pkg, torch, m):
    """The seeded packed model written straight into device memory (the same
    bytes as the host writer, tests/test_gpu_kernels.py checks that)."""
    w = {"layers": [], "on_device": True, "quant": m.quant, "embedQuant": m.embed_quant,
         "lmHeadQuant": m.lm_head_quant}
    for i in range(m.n_layers):
        t = torch.empty(pkg.pack.tensor_bytes(m, i), dtype=torch.uint8, device="cuda")
        pkg.pack.synth_device(m, i, t.data_ptr())
        w["layers"].append({"idx": i, "buf": t, "quant": m.quant})
    for k in ("embed", "norm", "lm_head"):
        w[k] = torch.empty(pkg.pack.tensor_bytes(m, k), dtype=torch.uint8, device="cuda")
        pkg.pack.synth_device(m, k, w[k].data_ptr())
    torch.cuda.synchronize()
    return w


def test_llama8b_greedy_64_vs_oracle_fixture(pkg, torch_cuda):
    """The whole Llama-3-8B-shaped q4_0 model as one stage (32 layers, 128256
    vocab lm_head): a 32-token prompt prefill, then 64 decode steps, against
    the oracle's run stored in tests/golden/llama8b_greedy.json (made by
    tests/golden/make_llama8b_greedy.py).  Two sequences: greedy (argmax fed
    back; the fixture's 65 tokens are all distinct, so the bar is not met at a
    fixed point) and teacher-forced (fixed inputs).  Every step: identical
    token, final hidden state (every 32nd element) within HIDDEN_TOL, the
    oracle's 16 largest logits within HIDDEN_TOL of the largest."""
    torch = torch_cuda
    fx = json.loads((Path(__file__).parent / "golden" / "llama8b_greedy.json").read_text())
    assert fx["greedy_distinct"] >= 16 and fx["forced_distinct"] >= 16
    m = pkg.pack.MODELS["llama8b"]
    w = _device_weights(pkg, torch, m)
    ctx = pkg.initStage({"arch": "llama", "dims": m.dims(), "layers": [0, m.n_layers], "is_first": True,
                         "is_last": True, "weights": w, "opts": {"max_ctx": 128, "max_seqs": 2, "device": 0}})
    del w
    torch.cuda.empty_cache()
    stride, prompt = fx["hidden_stride"], fx["prompt"]

    def check(rec, got_tok, rows, where):
        assert got_tok == rec["token"], (where, got_tok, rec["token"], "oracle top-2 gap", rec["gap"])
        h = ctx.peek("hidden", rows)[rows - 1][::stride]
        want_h = np.frombuffer(base64.b64decode(rec["hidden_sub"]), dtype="<f4")
        assert maxrel(h, want_h) <= HIDDEN_TOL, (where, maxrel(h, want_h))
        lg = ctx.peek("logits", 1)[0]
        tv = np.asarray(rec["top_val"], dtype=np.float64)
        err = float(np.max(np.abs(lg[rec["top_idx"]] - tv)) / np.max(np.abs(tv)))
        assert err <= HIDDEN_TOL, (where, err)

    for run, seq in (("greedy", "g"), ("forced", "f")):
        steps = fx[run]
        tok = pkg.forward(ctx, {"seq_id": seq, "token_pos": 0, "token_ids": prompt, "temperature": 0})["token_id"]
        check(steps[0], tok, len(prompt), (run, "prefill"))
        for s in range(64):
            inp = tok if run == "greedy" else fx["forced_inputs"][s]
            tok = pkg.forward(ctx, {"seq_id": seq, "token_pos": len(prompt) + s, "token_ids": [inp],
                                    "temperature": 0})["token_id"]
            check(steps[s + 1], tok, 1, (run, s))
    pkg.freeStage(ctx)
