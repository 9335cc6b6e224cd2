"""tn_attention_static: attention for callers that cannot allocate device memory.

Some callers of this library cannot call cudaMalloc (a host whose own memory
manager owns the device, a binding layer with no allocator, a serving loop
that must not stall on allocation), so this entry point keeps its scratch in a
fixed array inside the library instead of taking it from the caller.  The test
drives it through the C ABI and checks it against tn_attention, which takes
caller scratch, on two calls in a row (the second runs over whatever the first
left in the shared array).  This file is collected last so a failure here
leaves every other test already run; it also passes on its own.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATTN_TOL = 1e-5  # the attention tolerance of tests/test_gpu_kernels.py


def _case(torch, rng, n_slots, nH, nKV, hd, max_ctx, lens, slots):
    K = rng.standard_normal((n_slots, nKV, max_ctx, hd)).astype(np.float32)
    V = rng.standard_normal((n_slots, nKV, max_ctx, hd)).astype(np.float32)
    q = rng.standard_normal((len(lens), nH * hd)).astype(np.float32)
    return {"K": torch.from_numpy(K).cuda(), "V": torch.from_numpy(V).cuda(), "q": torch.from_numpy(q).cuda(),
            "slot": torch.tensor(slots, dtype=torch.int32, device="cuda"),
            "len": torch.tensor(lens, dtype=torch.int32, device="cuda"),
            "dims": (len(lens), n_slots, nH, nKV, hd, max_ctx)}


def _with_caller_scratch(pkg, torch, c):
    lib = pkg._lib.load()
    n, n_slots, nH, nKV, hd, max_ctx = c["dims"]
    out = torch.zeros((n, nH * hd), dtype=torch.float32, device="cuda")
    nbytes = lib.tn_attention_scratch_bytes(n, nH, nKV, hd, max_ctx)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    pkg._lib.check(lib.tn_attention(n, n_slots, nH, nKV, hd, max_ctx, c["q"].data_ptr(), c["K"].data_ptr(),
                                    c["V"].data_ptr(), c["slot"].data_ptr(), c["len"].data_ptr(), out.data_ptr(),
                                    scratch.data_ptr(), nbytes, None))
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _with_static_scratch(pkg, torch, c):
    lib = pkg._lib.load()
    n, n_slots, nH, nKV, hd, max_ctx = c["dims"]
    out = torch.full((n, nH * hd), float("nan"), dtype=torch.float32, device="cuda")
    pkg._lib.check(lib.tn_attention_static(n, n_slots, nH, nKV, hd, max_ctx, c["q"].data_ptr(), c["K"].data_ptr(),
                                           c["V"].data_ptr(), c["slot"].data_ptr(), c["len"].data_ptr(),
                                           out.data_ptr(), None))
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_static_scratch_attention_matches_caller_scratch(pkg, torch_cuda):
    torch = torch_cuda
    rng = np.random.default_rng(2024)
    cases = [
        _case(torch, rng, 3, 64, 8, 128, 1100, [1, 9, 1024, 300], [0, 1, 2, 0]),  # 70B heads, long contexts
        _case(torch, rng, 2, 8, 2, 32, 96, [5, 96, 40], [1, 0, 1]),             # tiny heads, more rows
    ]
    for i, c in enumerate(cases):  # two calls in a row over the one shared array
        want = _with_caller_scratch(pkg, torch, c)
        got = _with_static_scratch(pkg, torch, c)
        assert np.isfinite(got).all(), i
        err = float(np.max(np.abs(got - want)) / max(float(np.max(np.abs(want))), 1e-30))
        assert err <= ATTN_TOL, (i, err)


def test_static_scratch_row_limit_boundary(pkg, torch_cuda):
    """65536 rows fill the fixed array exactly and run (rows are not bounded
    by the grid's y / z limits); the result equals the caller-scratch entry
    point's.  65537 rows are refused before anything is launched."""
    torch = torch_cuda
    lib = pkg._lib.load()
    rng = np.random.default_rng(65536)
    n = 1 << 16
    lens = [1 + (r % 4) for r in range(n)]
    c = _case(torch, rng, 2, 8, 2, 32, 4, lens, [r % 2 for r in range(n)])
    assert lib.tn_attention_scratch_bytes(n, 8, 2, 32, 4) == (1 << 20)
    want = _with_caller_scratch(pkg, torch, c)
    got = _with_static_scratch(pkg, torch, c)
    assert np.isfinite(got).all()
    err = float(np.max(np.abs(got - want)) / max(float(np.max(np.abs(want))), 1e-30))
    assert err <= ATTN_TOL, err
    n1 = n + 1
    dummy = torch.zeros(16, dtype=torch.float32, device="cuda")
    idx = torch.zeros(n1, dtype=torch.int32, device="cuda")
    rc = lib.tn_attention_static(n1, 1, 8, 2, 32, 4, dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(),
                                 idx.data_ptr(), idx.data_ptr(), dummy.data_ptr(), None)
    assert rc == pkg._lib.TN_ECAPACITY
    # a refused call leaves nothing behind: the next call runs
    got2 = _with_static_scratch(pkg, torch, c)
    assert np.array_equal(got2, got)


def test_static_scratch_rejects_oversized_calls(pkg, torch_cuda):
    torch = torch_cuda
    lib = pkg._lib.load()
    n, nH, nKV, hd, max_ctx = 70000, 64, 8, 128, 4096  # the fixed array holds 65536 rows
    assert lib.tn_attention_scratch_bytes(n, nH, nKV, hd, max_ctx) > (1 << 20)
    dummy = torch.zeros(16, dtype=torch.float32, device="cuda")
    idx = torch.zeros(n, dtype=torch.int32, device="cuda")
    rc = lib.tn_attention_static(n, 1, nH, nKV, hd, max_ctx, dummy.data_ptr(), dummy.data_ptr(),
                                 dummy.data_ptr(), idx.data_ptr(), idx.data_ptr(), dummy.data_ptr(), None)
    assert rc == pkg._lib.TN_ECAPACITY
    assert "scratch" in lib.tn_last_error().decode()
