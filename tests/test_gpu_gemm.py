"""The tcgen05 dequant-GEMM (steps of 16 or more tokens) against the oracle,
through the C ABI (tn_matrix_matvec routes those token counts to it).

Each token row of the product is compared with the oracle's matvec of the
same packed bytes (web/inference-worker.js:523-527, f64 accumulation):
max |a - b| / max |b| within MATVEC_TOL, the bar of the single-matvec tests.
The three-product fp16 split keeps the measured error near f32 rounding.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MATVEC_TOL = 1e-4


def _synth(pkg, rows, cols, quant, seed):
    m = pkg.pack.ModelDims(cols, 1, 1, 1, rows, 0, 1e4, quant, quant, quant, seed)
    d = m.c_dims()
    buf = np.empty(pkg.pack.quant_bytes(rows * cols, quant), dtype=np.uint8)
    pkg._lib.check(pkg._lib.load().tn_synth_tensor(seed, pkg._lib.TN_TAG_EMBED, C.byref(d), pkg._lib.QUANT[quant],
                                                   buf.ctypes.data, 0, None))
    return buf


def _run(pkg, ref, torch, quant, rows, cols, T, seed, scale=1.0, check_every=1):
    lib = pkg._lib.load()
    buf = _synth(pkg, rows, cols, quant, seed)
    h = C.c_void_p()
    pkg._lib.check(lib.tn_matrix_create(0, pkg._lib.QUANT[quant], rows, cols, buf.ctypes.data, buf.nbytes, 0,
                                        C.byref(h)))
    try:
        rng = np.random.default_rng(seed)
        x = (rng.standard_normal((T, cols)) * scale).astype(np.float32)
        dx = torch.from_numpy(x).cuda()
        dy = torch.full((T, rows), float("nan"), dtype=torch.float32, device="cuda")
        pkg._lib.check(lib.tn_matrix_matvec(h, T, dx.data_ptr(), dy.data_ptr(), None))
        torch.cuda.synchronize()
        got = dy.cpu().numpy()
        assert np.isfinite(got).all()
        worst = 0.0
        for t in sorted(set(range(0, T, check_every)) | {T - 1}):
            want = ref.matvec(buf, quant, rows, cols, x[t])
            err = float(np.max(np.abs(got[t] - want)) / max(float(np.max(np.abs(want))), 1e-30))
            worst = max(worst, err)
            assert err < MATVEC_TOL, (t, err)
        return worst
    finally:
        lib.tn_matrix_free(h)


@pytest.mark.parametrize("quant,rows,cols,T", [
    ("q4_0", 128, 64, 16),     # one CTA, one K slice
    ("q8_0", 128, 64, 16),
    ("q4_0", 40, 128, 21),     # a partial M tile, a partial N tile
    ("q8_0", 24, 192, 17),
    ("q4_0", 300, 4096, 33),   # one N tile of 48 (T rounded up to 16)
    ("q4_0", 64, 28672, 16),   # the longest K (70B down): 112 chunks of accumulation
    ("q8_0", 1000, 8192, 64),
    ("q4_0", 4096, 4096, 128),
])
def test_gemm_small_and_medium(pkg, ref, torch_cuda, quant, rows, cols, T):
    _run(pkg, ref, torch_cuda, quant, rows, cols, T, seed=rows + cols + T)


@pytest.mark.parametrize("quant,rows,cols,T", [
    ("q4_0", 14336, 4096, 512),   # 8B gate / up, a full prefill chunk: 4 N tiles of 128
    ("q4_0", 4096, 14336, 200),   # 8B down: 2 N tiles of 112
    ("q8_0", 4096, 4096, 512),
    ("q4_0", 128256, 4096, 16),   # the lm_head over 16 rows
])
def test_gemm_large(pkg, ref, torch_cuda, quant, rows, cols, T):
    _run(pkg, ref, torch_cuda, quant, rows, cols, T, seed=rows ^ cols ^ T, check_every=max(1, T // 12))


@pytest.mark.parametrize("quant,rows,cols,T", [
    ("q4_0", 4096, 14336, 16),   # 32 M tiles: K split 5 ways
    ("q4_0", 128, 8192, 16),     # one M tile: K split 16 ways
    ("q8_0", 1024, 4096, 200),   # 8 M tiles x 2 N tiles, split 8 ways
])
def test_gemm_split_k_deterministic(pkg, ref, torch_cuda, quant, rows, cols, T):
    """Matrices with too few 128-row tiles to fill the GPU split K over
    several CTAs; the last to arrive sums the partials in split order.  Three
    launches back to back (no synchronisation between them) give identical
    bits, and match the oracle."""
    torch = torch_cuda
    lib = pkg._lib.load()
    buf = _synth(pkg, rows, cols, quant, 41)
    h = C.c_void_p()
    pkg._lib.check(lib.tn_matrix_create(0, pkg._lib.QUANT[quant], rows, cols, buf.ctypes.data, buf.nbytes, 0,
                                        C.byref(h)))
    try:
        x = np.random.default_rng(42).standard_normal((T, cols)).astype(np.float32)
        dx = torch.from_numpy(x).cuda()
        outs = [torch.full((T, rows), float("nan"), dtype=torch.float32, device="cuda") for _ in range(3)]
        for dy in outs:
            pkg._lib.check(lib.tn_matrix_matvec(h, T, dx.data_ptr(), dy.data_ptr(), None))
        torch.cuda.synchronize()
        got = [o.cpu().numpy() for o in outs]
        assert np.array_equal(got[0], got[1]) and np.array_equal(got[0], got[2])
        for t in sorted({0, T // 2, T - 1}):
            want = ref.matvec(buf, quant, rows, cols, x[t])
            assert float(np.max(np.abs(got[0][t] - want)) / np.max(np.abs(want))) < MATVEC_TOL
    finally:
        lib.tn_matrix_free(h)


def test_gemm_activation_range(pkg, ref, torch_cuda):
    """Rows of very different magnitudes (each token row is scaled by its own
    power of two before the fp16 split)."""
    torch = torch_cuda
    for scale in (1e-6, 1e4):
        _run(pkg, ref, torch, "q4_0", 512, 1024, 24, seed=3, scale=scale)
