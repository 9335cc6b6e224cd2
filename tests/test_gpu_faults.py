"""Failure handling on the GPU without faulting it: a bounded device wait
made to run out on purpose (a barrier that nothing arrives at, a short
limit) returns TN_ETIMEOUT and leaves the context usable; a stage whose
kernel reported a given-up wait returns TN_ETIMEOUT from the next forward or
check, resets its split-K state and then runs on correctly; the pipeline
runner turns that report into PipelineError."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _maxrel(a, b):
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


def test_bounded_wait_runs_out_and_device_stays_usable(pkg, ref, torch_cuda):
    torch = torch_cuda
    lib = pkg._lib.load()
    assert lib.tn_test_bounded_wait(2_000_000) == pkg._lib.TN_ETIMEOUT  # ~1 ms at 2 GHz
    assert b"gave up" in lib.tn_last_error()
    assert lib.tn_test_bounded_wait(0) == pkg._lib.TN_EINVAL
    # a kernel with the same waits runs correctly afterwards
    rows, cols = 512, 1024
    m = pkg.pack.ModelDims(cols, 1, 1, 1, rows, 0, 1e4, "q4_0", "q4_0", "q4_0", 9)
    d = m.c_dims()
    buf = np.empty(pkg.pack.quant_bytes(rows * cols, "q4_0"), dtype=np.uint8)
    pkg._lib.check(lib.tn_synth_tensor(9, pkg._lib.TN_TAG_EMBED, C.byref(d), pkg._lib.QUANT["q4_0"],
                                       buf.ctypes.data, 0, None))
    h = C.c_void_p()
    pkg._lib.check(lib.tn_matrix_create(0, pkg._lib.QUANT["q4_0"], rows, cols, buf.ctypes.data, buf.nbytes, 0,
                                        C.byref(h)))
    try:
        x = np.random.default_rng(1).standard_normal(cols).astype(np.float32)
        dx = torch.from_numpy(x).cuda()
        dy = torch.zeros(rows, device="cuda")
        pkg._lib.check(lib.tn_matrix_matvec(h, 1, dx.data_ptr(), dy.data_ptr(), None))
        torch.cuda.synchronize()
        assert _maxrel(dy.cpu().numpy(), ref.matvec(buf, "q4_0", rows, cols, x)) < 1e-4
    finally:
        lib.tn_matrix_free(h)


def _tiny_stage(pkg, **opts):
    m = pkg.pack.MODELS["tiny"]
    w = pkg.pack.synth_weights(m, 0, m.n_layers, True, True)
    o = {"max_ctx": 128, "max_seqs": 4, "device": 0}
    o.update(opts)
    ctx = pkg.initStage({"arch": "llama", "dims": m.dims(), "layers": [0, m.n_layers], "is_first": True,
                         "is_last": True, "weights": w, "opts": o})
    return m, w, ctx


def test_stage_reports_and_recovers_from_kernel_wait_failure(pkg, ref):
    m, w, ctx = _tiny_stage(pkg)
    lib = pkg._lib.load()
    oracle = ref.RefStage(m.dims(), 0, m.n_layers, True, True, w)
    prompt = pkg.pack.synth_prompt(m, 8, seed=3)
    tok = pkg.forward(ctx, {"seq_id": 1, "token_pos": 0, "token_ids": prompt, "temperature": 0})["token_id"]
    assert tok == oracle.forward(1, 0, token_ids=prompt)["token_id"]
    assert lib.tn_stage_check(ctx.handle, None) == pkg._lib.TN_OK
    pkg._lib.check(lib.tn_stage_test_raise_kernel_error(ctx.handle))
    with pytest.raises(pkg._lib.TnError) as ei:
        pkg.forward(ctx, {"seq_id": 1, "token_pos": 8, "token_ids": [tok], "temperature": 0})
    assert ei.value.code == pkg._lib.TN_ETIMEOUT
    assert pkg.kv_len(ctx, 1) == 8  # the failed step committed nothing
    # the same step again: correct, the stage recovered
    got = pkg.forward(ctx, {"seq_id": 1, "token_pos": 8, "token_ids": [tok], "temperature": 0})["token_id"]
    assert got == oracle.forward(1, 8, token_ids=[tok])["token_id"]
    # an async check reports it the same way, once
    pkg._lib.check(lib.tn_stage_test_raise_kernel_error(ctx.handle))
    assert lib.tn_stage_check(ctx.handle, None) == pkg._lib.TN_ETIMEOUT
    assert lib.tn_stage_check(ctx.handle, None) == pkg._lib.TN_OK
    pkg.freeStage(ctx)


def test_pipeline_surfaces_kernel_wait_failure(pkg, torch_cuda):
    torch = torch_cuda
    m, w, ctx = _tiny_stage(pkg)
    lib = pkg._lib.load()
    prompts = [pkg.pack.synth_prompt(m, 6, seed=10 + i) for i in range(2)]
    first = pkg.pipeline.prefill(ctx, 0, 1, prompts, m.hidden_dim)
    pipe = pkg.pipeline.Pipeline(pkg.pipeline.DeviceStage(ctx, 2), 0, 1, 2, m.hidden_dim, deadline_s=60)
    pipe.pos = [[6], [6]]
    pipe.tok[:, 0] = torch.tensor(first, dtype=torch.int32)
    pipe.rounds(2)
    pkg._lib.check(lib.tn_stage_test_raise_kernel_error(ctx.handle))
    with pytest.raises(pkg.pipeline.PipelineError) as ei:
        pipe.rounds(1)
    assert ei.value.code == pkg._lib.TN_ETIMEOUT and ei.value.tick == -1
    pipe.rounds(1)  # recovered
    pkg.freeStage(ctx)
