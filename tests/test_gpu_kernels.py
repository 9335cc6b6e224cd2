"""Single-kernel parity on the GPU, through the C ABI, against the oracle.

Bit-exact: synthetic pack bytes (device vs host writer), weight repack +
decode, the activation hop encoder.  Within f32-accumulate tolerance: the
dequant-matvec and the GQA attention (max |a-b| / max |b|).
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MATVEC_TOL = 1e-4  # max-relative error of f32 accumulation vs the oracle's double
ATTN_TOL = 1e-5


def _synth_matrix(pkg, rows, cols, quant, seed):
    """A seeded [rows x cols] tensor in the reference byte layout (the embed
    generator over a (vocab=rows, hidden=cols) shape)."""
    m = pkg.pack.ModelDims(cols, 1, 1, 1, rows, 0, 1e4, quant, quant, quant, seed)
    d = m.c_dims()
    buf = np.empty(pkg.pack.quant_bytes(rows * cols, quant), dtype=np.uint8)
    pkg._lib.check(pkg._lib.load().tn_synth_tensor(seed, pkg._lib.TN_TAG_EMBED, C.byref(d), pkg._lib.QUANT[quant],
                                                   buf.ctypes.data, 0, None))
    return buf


class Mat:
    def __init__(self, pkg, quant, rows, cols, buf):
        self.lib = pkg._lib.load()
        self.h = C.c_void_p()
        pkg._lib.check(self.lib.tn_matrix_create(0, pkg._lib.QUANT[quant], rows, cols, buf.ctypes.data, buf.nbytes, 0,
                                                 C.byref(self.h)))

    def __del__(self):
        self.lib.tn_matrix_free(self.h)


def test_device_synth_matches_host(pkg, torch_cuda):
    torch = torch_cuda
    for name, layers in (("tiny", range(4)), ("llama8b", [0, 31])):
        m = pkg.pack.MODELS[name]
        for what in list(layers) + ["norm", "embed", "lm_head"]:
            if name != "tiny" and what in ("embed", "lm_head"):
                continue
            n = pkg.pack.tensor_bytes(m, what)
            dev = torch.empty(n, dtype=torch.uint8, device="cuda")
            pkg.pack.synth_device(m, what, dev.data_ptr())
            torch.cuda.synchronize()
            host = pkg.pack.synth_layer(m, what) if isinstance(what, int) else pkg.pack.synth_tensor(m, what)
            assert np.array_equal(dev.cpu().numpy(), host), (name, what)


@pytest.mark.parametrize("quant,rows,cols", [
    ("q4_0", 64, 256), ("q8_0", 64, 256),
    ("q4_0", 16, 688), ("q8_0", 256, 688),   # rows that straddle blocks (688 % 32 != 0)
    ("q4_0", 13, 96), ("f16", 40, 100), ("f32", 24, 72),
])
def test_dequant_bit_exact(pkg, ref, torch_cuda, quant, rows, cols):
    torch = torch_cuda
    buf = _synth_matrix(pkg, rows, cols, quant, seed=7)
    mat = Mat(pkg, quant, rows, cols, buf)
    out = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
    pkg._lib.check(mat.lib.tn_matrix_dequant(mat.h, out.data_ptr(), None))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    want = ref.dequant(buf, quant, rows * cols)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def _maxrel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


@pytest.mark.parametrize("quant,rows,cols", [
    ("q4_0", 4096, 4096), ("q4_0", 14336, 4096), ("q4_0", 4096, 14336), ("q8_0", 4096, 4096),
    ("q8_0", 1000, 8192), ("q4_0", 8, 28672), ("q8_0", 256, 688), ("f16", 300, 200), ("f32", 77, 96),
])
@pytest.mark.parametrize("T", [1, 2, 3, 5, 8, 11])
def test_matvec_vs_oracle(pkg, ref, torch_cuda, quant, rows, cols, T):
    torch = torch_cuda
    buf = _synth_matrix(pkg, rows, cols, quant, seed=rows + cols)
    mat = Mat(pkg, quant, rows, cols, buf)
    rng = np.random.default_rng(T)
    x = rng.standard_normal((T, cols)).astype(np.float32)
    dx = torch.from_numpy(x).cuda()
    dy = torch.full((T, rows), float("nan"), dtype=torch.float32, device="cuda")
    pkg._lib.check(mat.lib.tn_matrix_matvec(mat.h, T, dx.data_ptr(), dy.data_ptr(), None))
    torch.cuda.synchronize()
    got = dy.cpu().numpy()
    for t in range(T):
        want = ref.matvec(buf, quant, rows, cols, x[t])
        assert _maxrel(got[t], want) < MATVEC_TOL, (t, _maxrel(got[t], want))


@pytest.mark.parametrize("quant,rows,cols,T", [
    ("q4_0", 4096, 4096, 4), ("q4_0", 4096, 4096, 16), ("q4_0", 4096, 4096, 64), ("q4_0", 4096, 4096, 512),
    ("q4_0", 14336, 4096, 16), ("q4_0", 14336, 4096, 64), ("q8_0", 4096, 14336, 16), ("q8_0", 4096, 4096, 64),
    ("q4_0", 128256, 4096, 4),  # the 8B lm_head
])
def test_matvec_token_sweep(pkg, ref, torch_cuda, quant, rows, cols, T):
    """The matvec microbench's token counts (4 .. 512) on its weight shapes:
    token rows against the oracle (all up to 16 tokens, a spread past that)."""
    torch = torch_cuda
    buf = _synth_matrix(pkg, rows, cols, quant, seed=rows ^ cols ^ T)
    mat = Mat(pkg, quant, rows, cols, buf)
    rng = np.random.default_rng(1000 + T)
    x = rng.standard_normal((T, cols)).astype(np.float32)
    dx = torch.from_numpy(x).cuda()
    dy = torch.full((T, rows), float("nan"), dtype=torch.float32, device="cuda")
    pkg._lib.check(mat.lib.tn_matrix_matvec(mat.h, T, dx.data_ptr(), dy.data_ptr(), None))
    torch.cuda.synchronize()
    got = dy.cpu().numpy()
    assert np.isfinite(got).all()
    step = max(1, T // 16)  # past 16 tokens the oracle checks every step-th one and the last
    for t in sorted(set(range(0, T, step)) | {T - 1}):
        want = ref.matvec(buf, quant, rows, cols, x[t])
        assert _maxrel(got[t], want) < MATVEC_TOL, (t, _maxrel(got[t], want))


def test_matvec_back_to_back_same_matrix(pkg, ref, torch_cuda):
    """One pool-eligible matrix (the 8B lm_head: whole tiles taken by ticket)
    launched repeatedly on one stream with no synchronisation in between,
    alternating one, two and three tokens (three = a two-token and a one-token
    launch) with fresh x each time: every output row matches the oracle, and
    the per-tile arrival and per-chunk ticket counters read back as zero."""
    torch = torch_cuda
    rows, cols, quant = 128256, 4096, "q4_0"
    buf = _synth_matrix(pkg, rows, cols, quant, seed=77)
    mat = Mat(pkg, quant, rows, cols, buf)
    rng = np.random.default_rng(78)
    runs = []
    for T in (1, 2, 1, 3, 2, 1):
        x = rng.standard_normal((T, cols)).astype(np.float32)
        dx = torch.from_numpy(x).cuda()
        dy = torch.full((T, rows), float("nan"), dtype=torch.float32, device="cuda")
        runs.append((x, dx, dy))
    torch.cuda.synchronize()
    for x, dx, dy in runs:  # enqueued back to back
        pkg._lib.check(mat.lib.tn_matrix_matvec(mat.h, x.shape[0], dx.data_ptr(), dy.data_ptr(), None))
    torch.cuda.synchronize()
    for i, (x, _, dy) in enumerate(runs):
        got = dy.cpu().numpy()
        for t in range(x.shape[0]):
            want = ref.matvec(buf, quant, rows, cols, x[t])
            assert _maxrel(got[t], want) < MATVEC_TOL, (i, t, _maxrel(got[t], want))
    total = C.c_int64(-1)
    pkg._lib.check(mat.lib.tn_matrix_counter_sum(mat.h, C.byref(total)))
    assert total.value == 0


def _kv_cache(torch, K, V, kv):
    """Device copies of the cache in format kv, and the values the oracle sees
    (an fp16 or fp8 e4m3 cache holds the f32 values rounded to nearest even)."""
    if kv == "f8":
        K8 = torch.from_numpy(K).to(torch.float8_e4m3fn)
        V8 = torch.from_numpy(V).to(torch.float8_e4m3fn)
        return (K8.view(torch.uint8).cuda(), V8.view(torch.uint8).cuda(), K8.float().numpy(),
                V8.float().numpy())
    if kv == "f16":
        K, V = K.astype(np.float16), V.astype(np.float16)
        return torch.from_numpy(K).cuda(), torch.from_numpy(V).cuda(), K.astype(np.float32), V.astype(np.float32)
    return torch.from_numpy(K).cuda(), torch.from_numpy(V).cuda(), K, V


def _attn_call(pkg, lib, kv, *args):
    fn = {"f32": lib.tn_attention, "f16": lib.tn_attention_f16, "f8": lib.tn_attention_f8}[kv]
    pkg._lib.check(fn(*args))


@pytest.mark.parametrize("kv", ["f32", "f16", "f8"])
@pytest.mark.parametrize("hd,nH,nKV", [(128, 32, 8), (128, 64, 8), (32, 8, 2), (64, 64, 4)])
def test_attention_vs_oracle(pkg, ref, torch_cuda, hd, nH, nKV, kv):
    """Rows of 1 .. 2100 positions; an fp16 or fp8 cache is compared with the
    oracle on the same rounded values (only the storage format differs)."""
    torch = torch_cuda
    lib = pkg._lib.load()
    max_ctx, n_slots = 2100, 3
    rng = np.random.default_rng(hd + nH)
    K = rng.standard_normal((n_slots, nKV, max_ctx, hd)).astype(np.float32)
    V = rng.standard_normal((n_slots, nKV, max_ctx, hd)).astype(np.float32)
    lens = [1, 7, 33, 2048, 517, 2100]
    slots = [0, 1, 2, 0, 1, 2]
    q = rng.standard_normal((len(lens), nH * hd)).astype(np.float32)
    dK, dV, K, V = _kv_cache(torch, K, V, kv)
    dq = torch.from_numpy(q).cuda()
    dslot = torch.tensor(slots, dtype=torch.int32, device="cuda")
    dlen = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = torch.zeros((len(lens), nH * hd), dtype=torch.float32, device="cuda")
    nbytes = lib.tn_attention_scratch_bytes(len(lens), nH, nKV, hd, max_ctx)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    _attn_call(pkg, lib, kv, len(lens), n_slots, nH, nKV, hd, max_ctx, dq.data_ptr(), dK.data_ptr(), dV.data_ptr(),
               dslot.data_ptr(), dlen.data_ptr(), out.data_ptr(), scratch.data_ptr(), nbytes, None)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for r, (L, s) in enumerate(zip(lens, slots)):
        # the oracle's cache rows are [pos][kvDim] with kvDim = nKV * hd
        Kr = K[s, :, :L, :].transpose(1, 0, 2).reshape(L, nKV * hd)
        Vr = V[s, :, :L, :].transpose(1, 0, 2).reshape(L, nKV * hd)
        want = ref.attention(q[r], Kr, Vr, nH, nKV, hd)
        assert _maxrel(got[r], want) < ATTN_TOL, (r, L, _maxrel(got[r], want))


@pytest.mark.parametrize("kv,page", [("f32", 16), ("f32", 64), ("f16", 256), ("f8", 64), ("f32", 4096)])
def test_attention_paged_vs_oracle(pkg, ref, torch_cuda, kv, page):
    """tn_attention_paged: each row's positions scattered over a shuffled page
    pool (page boundaries inside warp steps and splits), lengths 1 .. 5000,
    against the oracle on the rows gathered back in order; a row naming a page
    outside the pool gives zeros."""
    torch = torch_cuda
    lib = pkg._lib.load()
    hd, nH, nKV = 128, 32, 8
    lens = [1, page - 1, page, page + 1, 7, 2100, 5000, 3 * page + 5]
    n = len(lens)
    max_pages = -(-max(lens) // page)
    rng = np.random.default_rng(page)
    need = sum(-(-L // page) for L in lens)
    n_pages = need + 5
    perm = rng.permutation(n_pages)
    table = np.full((n + 1, max_pages), -1, np.int32)
    k = 0
    for r, L in enumerate(lens):
        for j in range(-(-L // page)):
            table[r, j] = perm[k]
            k += 1
    table[n, 0] = n_pages  # the extra row: a page id outside the pool
    lens = lens + [5]
    K = rng.standard_normal((n_pages, nKV, page, hd)).astype(np.float32)
    V = rng.standard_normal((n_pages, nKV, page, hd)).astype(np.float32)
    dK, dV, K, V = _kv_cache(torch, K, V, kv)
    q = rng.standard_normal((n + 1, nH * hd)).astype(np.float32)
    dq = torch.from_numpy(q).cuda()
    dtab = torch.from_numpy(table).cuda()
    dlen = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = torch.full((n + 1, nH * hd), 7.0, dtype=torch.float32, device="cuda")
    nbytes = lib.tn_attention_scratch_bytes(n + 1, nH, nKV, hd, max_pages * page)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    code = {"f32": 0, "f16": 1, "f8": 2}[kv]
    pkg._lib.check(lib.tn_attention_paged(code, n + 1, nH, nKV, hd, page, max_pages, n_pages, dq.data_ptr(),
                                          dK.data_ptr(), dV.data_ptr(), dtab.data_ptr(), dlen.data_ptr(),
                                          out.data_ptr(), scratch.data_ptr(), nbytes, None))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for r in range(n):
        L = lens[r]
        pos = np.arange(L)
        pg = table[r, pos // page]
        Kr = K[pg, :, pos % page, :].reshape(L, nKV * hd)
        Vr = V[pg, :, pos % page, :].reshape(L, nKV * hd)
        want = ref.attention(q[r], Kr, Vr, nH, nKV, hd)
        assert _maxrel(got[r], want) < ATTN_TOL, (r, L, _maxrel(got[r], want))
    assert not got[n].any()


@pytest.mark.parametrize("L,n_rows,n_slots,kv", [
    (512, 1, 1, "f32"), (1024, 1, 1, "f32"), (2048, 8, 8, "f32"), (2048, 64, 16, "f32"), (8192, 1, 1, "f32"),
    (8192, 8, 4, "f32"), (8192, 64, 8, "f32"), (32768, 1, 1, "f32"), (32768, 8, 2, "f32"), (32768, 64, 8, "f32"),
    (1024, 1, 1, "f16"), (8192, 8, 4, "f16"), (32768, 1, 1, "f16"), (32768, 8, 2, "f16"),
    (1024, 1, 1, "f8"), (8192, 8, 4, "f8"), (32768, 1, 1, "f8"), (32768, 64, 8, "f8"),
])
def test_attention_context_sweep(pkg, ref, torch_cuda, L, n_rows, n_slots, kv):
    """The GQA decode-attention sweep (32 query / 8 KV heads x 128, contexts
    512 .. 32768, 1 .. 64 concurrent rows, f32, fp16 and fp8 caches) against the
    oracle.  Few rows split every row's positions over many CTAs; two
    launches back to back give identical bits (the merge runs in split order
    and the last CTA resets the arrival counters)."""
    torch = torch_cuda
    lib = pkg._lib.load()
    hd, nH, nKV = 128, 32, 8
    rng = np.random.default_rng(L + n_rows)
    K = rng.standard_normal((n_slots, nKV, L, hd), dtype=np.float32)
    V = rng.standard_normal((n_slots, nKV, L, hd), dtype=np.float32)
    lens = [L - (r % 3) for r in range(n_rows)]
    slots = [r % n_slots for r in range(n_rows)]
    q = rng.standard_normal((n_rows, nH * hd), dtype=np.float32)
    dK, dV, K, V = _kv_cache(torch, K, V, kv)
    dq = torch.from_numpy(q).cuda()
    dslot = torch.tensor(slots, dtype=torch.int32, device="cuda")
    dlen = torch.tensor(lens, dtype=torch.int32, device="cuda")
    outs = [torch.zeros((n_rows, nH * hd), dtype=torch.float32, device="cuda") for _ in range(2)]
    nbytes = lib.tn_attention_scratch_bytes(n_rows, nH, nKV, hd, L)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    for out in outs:
        _attn_call(pkg, lib, kv, n_rows, n_slots, nH, nKV, hd, L, dq.data_ptr(), dK.data_ptr(), dV.data_ptr(),
                   dslot.data_ptr(), dlen.data_ptr(), out.data_ptr(), scratch.data_ptr(), nbytes, None)
    torch.cuda.synchronize()
    got = outs[0].cpu().numpy()
    assert np.isfinite(got).all()
    assert np.array_equal(got, outs[1].cpu().numpy())
    step = max(1, n_rows // 4) if L >= 8192 else 1  # long contexts: the oracle checks a spread of rows
    for r in sorted(set(range(0, n_rows, step)) | {n_rows - 1}):
        s, n = slots[r], lens[r]
        Kr = K[s, :, :n, :].transpose(1, 0, 2).reshape(n, nKV * hd)
        Vr = V[s, :, :n, :].transpose(1, 0, 2).reshape(n, nKV * hd)
        want = ref.attention(q[r], Kr, Vr, nH, nKV, hd)
        assert _maxrel(got[r], want) < ATTN_TOL, (r, n, _maxrel(got[r], want))


def test_hop_encode_exhaustive(pkg, ref, torch_cuda):
    """Every f32 bit pattern through the device encoder equals the oracle's
    literal restatement of f32ToF16 (web/inference-worker.js:74-88)."""
    torch = torch_cuda
    lib = pkg._lib.load()
    chunk = 1 << 28
    out = torch.empty(chunk, dtype=torch.int16, device="cuda")
    for c in range((1 << 32) // chunk):
        first = c * chunk
        bits = torch.arange(first, first + chunk, dtype=torch.int64, device="cuda")
        f32 = torch.where(bits >= 2**31, bits - 2**32, bits).to(torch.int32).view(torch.float32)
        pkg._lib.check(lib.tn_hop_encode(f32.data_ptr(), out.data_ptr(), chunk, None))
        torch.cuda.synchronize()
        got = out.cpu().numpy().view(np.uint16)
        want = ref.f32bits_to_f16(first, chunk)
        bad = np.nonzero(got != want)[0]
        assert bad.size == 0, [(hex(first + int(i)), hex(got[i]), hex(want[i])) for i in bad[:5]]


def test_hop_decode_exhaustive(pkg, ref, torch_cuda):
    torch = torch_cuda
    lib = pkg._lib.load()
    h = torch.arange(0, 65536, dtype=torch.int32, device="cuda").to(torch.int16)
    out = torch.empty(65536, dtype=torch.float32, device="cuda")
    pkg._lib.check(lib.tn_hop_decode(h.data_ptr(), out.data_ptr(), 65536, None))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for i in range(65536):
        w = ref.f16_to_f32(i)
        g = float(got[i])
        assert (np.isnan(w) and np.isnan(g)) or (w == g and np.signbit(w) == np.signbit(g)), i


def test_sample_vs_oracle(pkg, ref, torch_cuda):
    torch = torch_cuda
    lib = pkg._lib.load()
    rng = np.random.default_rng(5)
    V = 128256
    for trial, (temp, top_p) in enumerate([(0.0, 0.95), (-1.0, 0.5), (0.7, 0.95), (1.0, 0.5), (0.3, 1.0),
                                           (2.0, 0.99)]):
        logits = (rng.standard_normal(V) * 2).astype(np.float32)
        logits[rng.integers(0, V, 3)] = logits.max()  # ties at the max: lowest index wins
        seed = 1000 + trial
        d = torch.from_numpy(logits).cuda()
        out = torch.zeros(1, dtype=torch.int32, device="cuda")
        pkg._lib.check(lib.tn_sample(d.data_ptr(), 1, V, temp, top_p, seed, out.data_ptr(), None))
        got = int(out.item())
        want = ref.sample(logits, temp, top_p, lib.tn_sample_uniform(seed, 0))
        assert got == want, (trial, got, want)
