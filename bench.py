#!/usr/bin/env python
"""Decode throughput of the B200 stage engine: Llama-3-70B-shaped q4_0 model,
8 one-sequence micro-batches in flight, 1024-token prompts.

Each GPU holds one contiguous layer stage (the planner's ranges; one stage of
all 80 layers at N=1).  A stage runs one micro-batch per tick, and a bench
step is one round in which every micro-batch advances by one token (at N=1:
the 8 micro-batches back to back on one GPU; at N>1: a pipeline whose
activations hop over NCCL send/recv).  `value` is tokens per second of the
whole job with inputs resident in HBM; `e2e` drives the same rounds through
the host-buffer API (tn_stage_forward), host<->device copies included.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  (N>1: python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N)

Kernel sweeps (one GPU, one JSON line with a point per configuration):

  python bench.py --micro matvec [--shape 4096x4096,...] [--quant q4_0,q8_0] [--tokens 1,4,16,64,512]
  python bench.py --micro attn [--ctx 512,...] [--seqs 1,8,64]

The matvec sweep covers the dequant-matvec / dequant-GEMM weight shapes
(4096x4096, 14336x4096, 4096x14336, 128256x4096; q4_0 and q8_0; 1 .. 512
tokens), the attention sweep the GQA decode attention (32 query / 8 KV heads x
128, f32 KV; 512 .. 32768 cached positions; 1, 8, 64 rows).  Every launch reads
another copy of its inputs, and the copies together exceed the 126 MB L2, so
each launch streams from HBM.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s (70B-shape q4_0, 8 one-sequence micro-batches in flight)"
SCALING = "strong"  # total work (8 micro-batches x steps) is fixed as N grows


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=8, help="timed rounds (every micro-batch +1 token)")
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--model", default="llama70b")
    p.add_argument("--microbatches", type=int, default=8)
    p.add_argument("--prompt", type=int, default=1024)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-fused", action="store_true", help="skip the fused M-row decode measurement (N=1)")
    p.add_argument("--micro", choices=["matvec", "attn"], default=None, help="kernel sweep instead of decode")
    p.add_argument("--shape", default=None, help="matvec sweep: rows x cols list, e.g. 57344x8192,4096x4096")
    p.add_argument("--quant", default="q4_0,q8_0", help="matvec sweep: weight formats")
    p.add_argument("--tokens", default="1,4,16,64,512", help="matvec sweep: token counts")
    p.add_argument("--ctx", default="512,2048,8192,32768", help="attention sweep: cached positions")
    p.add_argument("--seqs", default="1,8,64", help="attention sweep: concurrent rows")
    p.add_argument("--kv", default="f32,f16,f8", help="attention sweep: KV cache element types")
    p.add_argument("--heads", default="32,8", help="attention sweep: query heads, KV heads")
    p.add_argument("--page-tokens", type=int, default=0,
                   help="attention sweep: paged cache with pages of this many positions (0: contiguous)")
    p.add_argument("--kv-cache", choices=["f32", "f16", "f8"], default="f32",
                   help="decode: KV cache element type (f32 = the reference's rows; f16 / f8 opt in)")
    p.add_argument("--kv-page-tokens", type=int, default=0,
                   help="decode: paged KV cache with pages of this many positions (0: contiguous per sequence)")
    p.add_argument("--reps", type=int, default=20, help="kernel sweeps: timed launches per point")
    return p.parse_args(argv)


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def workload_config(args, world: int) -> dict:
    return {"workload": f"{args.model} q4_0 decode: {args.microbatches} micro-batches x 1 sequence in flight, "
                        f"{args.prompt}-token prompts, one micro-batch per stage step",
            "model": args.model, "microbatches": args.microbatches, "seqs_per_microbatch": 1,
            "prompt_len": args.prompt, "stages": world, "parallelism": f"pp{world}", "kv_cache": args.kv_cache,
            "kv_page_tokens": args.kv_page_tokens,
            "l2": "weights (39 GB at N=1) exceed the 126 MB L2 every step; no flush needed",
            "sampling": "greedy (temperature 0)",
            "weights": "seeded synthetic: Irwin-Hall(4) approximation of N(0, 0.02) per element, quantised "
                       "to q4_0 per 32-element block (no checkpoint: shapes and format of the named model)"}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=self.file,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9 and f[1].replace(".", "").isdigit():
                rows.append(f)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


def physical_gpu(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].strip().isdigit():
            return int(ids[local_rank])
    return local_rank


def measured_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def measured_tensor_peak() -> tuple[float, str]:
    """Dense bf16 TFLOP/s: the burst figure (kernels timed alone)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


L2_BYTES = 126e6


def _ints(text: str) -> list[int]:
    return [int(v) for v in text.split(",") if v.strip()]


def micro_matvec(args):
    """The dequant-matvec sweep: each (shape, format, tokens) point timed over
    args.reps launches with CUDA events, rotating over enough copies of the
    matrix that each launch reads its weights from HBM."""
    import torch

    import __graft_entry__ as g

    pkg = g.load_package()
    lib, P = pkg._lib.load(), pkg._lib
    torch.cuda.set_device(0)
    shapes = ([tuple(int(v) for v in sh.split("x")) for sh in args.shape.split(",")] if args.shape
              else [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)])
    hbm, hbm_kind = measured_peaks()
    tc, tc_kind = measured_tensor_peak()
    ridge = tc * 1e12 / (hbm * 1e9)  # FLOP per byte where the two roofs meet
    clocks = ClockSampler(physical_gpu(0))
    clocks.start()
    points = []
    for rows, cols in shapes:
        for quant in args.quant.split(","):
            nbytes = pkg.pack.quant_bytes(rows * cols, quant)
            copies = max(1, int(2 * L2_BYTES // nbytes) + 1) if nbytes < 2 * L2_BYTES else 1
            m = pkg.pack.ModelDims(cols, 1, 1, 1, rows, 0, 1e4, quant, quant, quant, 5)
            src = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
            d = m.c_dims()
            P.check(lib.tn_synth_tensor(5, P.TN_TAG_EMBED, C.byref(d), P.QUANT[quant], src.data_ptr(), 1, None))
            torch.cuda.synchronize()
            mats = []
            for _ in range(copies):
                h = C.c_void_p()
                P.check(lib.tn_matrix_create(0, P.QUANT[quant], rows, cols, src.data_ptr(), nbytes, 1, C.byref(h)))
                mats.append(h)
            del src
            for T in _ints(args.tokens):
                x = torch.randn(T, cols, device="cuda")
                y = torch.empty(T, rows, device="cuda")
                # every copy once (the first call of a copy with a new token count
                # sizes its GEMM scratch), then the warm-up launches
                for i in range(copies + max(3, args.warmup)):
                    P.check(lib.tn_matrix_matvec(mats[i % copies], T, x.data_ptr(), y.data_ptr(), None))
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for i in range(args.reps):
                    P.check(lib.tn_matrix_matvec(mats[i % copies], T, x.data_ptr(), y.data_ptr(), None))
                e1.record()
                torch.cuda.synchronize()
                us = e0.elapsed_time(e1) / args.reps * 1e3
                byts = nbytes + 4 * T * (rows + cols)
                flops = 2 * T * rows * cols
                gbs, tfs = byts / us / 1e3, flops / us / 1e6
                tensor = flops / byts >= ridge
                roof = ({"bound": "tensor", "achieved": round(tfs, 2), "peak": tc, "unit": "TFLOP/s",
                         "frac": round(tfs / tc, 4), "peak_source": tc_kind}
                        if tensor else
                        {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(gbs / hbm, 4), "peak_source": hbm_kind})
                points.append({"shape": f"{rows}x{cols}", "quant": quant, "tokens": T, "us": round(us, 2),
                               "GB_s": round(gbs, 1), "TFLOP_s": round(tfs, 3), "roofline": roof,
                               "copies": copies})
                print(f"# {rows}x{cols} {quant} T={T}: {us:.1f} us, {gbs:.0f} GB/s, {tfs:.2f} TFLOP/s",
                      file=sys.stderr, flush=True)
            for h in mats:
                lib.tn_matrix_free(h)
    clk = clocks.stop()
    print(json.dumps({"micro": "matvec", "metric": "dequant-matvec HBM GB/s (TFLOP/s past the ridge)",
                      "unit": "GB/s", "points": points, "clocks": clk, "reps": args.reps,
                      "config": {"l2": "launches rotate over copies of the matrix totalling > 2 x L2",
                                 "x": "f32 N(0,1)", "weights": "seeded Irwin-Hall(4) approximation of N(0, 0.02), "
                                 "quantised per block"}}), flush=True)
    return 0


def micro_attn(args):
    """The GQA decode-attention sweep: tn_attention over seqs rows of ctx
    cached positions, each launch on other sequence slots of an arena larger
    than twice the L2 (or, with --page-tokens, on the same rows as pages of a
    shuffled pool).  Device time per call from a CUDA graph of `reps` calls:
    each the row-table kernel and the attention kernel."""
    import torch

    import __graft_entry__ as g

    pkg = g.load_package()
    lib, P = pkg._lib.load(), pkg._lib
    torch.cuda.set_device(0)
    nH, nKV = _ints(args.heads)
    hd = 128
    hbm, hbm_kind = measured_peaks()
    clocks = ClockSampler(physical_gpu(0))
    clocks.start()
    points = []
    stream = torch.cuda.Stream()
    for kv, ctx, seqs in [(k, c, n) for k in args.kv.split(",") for c in _ints(args.ctx) for n in _ints(args.seqs)]:
        eb = {"f32": 4, "f16": 2, "f8": 1}[kv]
        slot_bytes = 2 * nKV * ctx * hd * eb
        groups = max(1, int(2 * L2_BYTES // (slot_bytes * seqs)) + 1)
        n_slots = groups * seqs
        gen = torch.Generator(device="cuda").manual_seed(ctx + seqs)
        dt = {"f32": torch.float32, "f16": torch.float16, "f8": torch.float8_e4m3fn}[kv]
        K = torch.randn((n_slots, nKV, ctx, hd), device="cuda", generator=gen)
        V = torch.randn((n_slots, nKV, ctx, hd), device="cuda", generator=gen)
        if args.page_tokens:
            # the same rows as pages of a pool: slot s's positions in ctx / pt
            # pages, handed out in a shuffled order
            pt = args.page_tokens
            per = ctx // pt
            K = K.view(n_slots, nKV, per, pt, hd).transpose(1, 2).reshape(n_slots * per, nKV, pt, hd)
            V = V.view(n_slots, nKV, per, pt, hd).transpose(1, 2).reshape(n_slots * per, nKV, pt, hd)
            perm = torch.randperm(n_slots * per, generator=torch.Generator().manual_seed(ctx)).to(torch.int32)
            K[perm.long().cuda()] = K.clone()
            V[perm.long().cuda()] = V.clone()
            tables = [perm.view(n_slots, per)[g0 * seqs:(g0 + 1) * seqs].contiguous().cuda() for g0 in range(groups)]
        K, V = K.to(dt), V.to(dt)
        fn = {"f32": lib.tn_attention, "f16": lib.tn_attention_f16, "f8": lib.tn_attention_f8}[kv]
        q = torch.randn((seqs, nH * hd), device="cuda", generator=gen)
        out = torch.empty_like(q)
        lens = torch.full((seqs,), ctx, dtype=torch.int32, device="cuda")
        slots = [torch.arange(g0 * seqs, (g0 + 1) * seqs, dtype=torch.int32, device="cuda") for g0 in range(groups)]
        nbytes = lib.tn_attention_scratch_bytes(seqs, nH, nKV, hd, ctx)
        scratch = torch.empty(max(nbytes, 256), dtype=torch.uint8, device="cuda")

        if args.page_tokens:
            code = {"f32": 0, "f16": 1, "f8": 2}[kv]

            def call(i):
                P.check(lib.tn_attention_paged(code, seqs, nH, nKV, hd, pt, per, n_slots * per, q.data_ptr(),
                                               K.data_ptr(), V.data_ptr(), tables[i % groups].data_ptr(),
                                               lens.data_ptr(), out.data_ptr(), scratch.data_ptr(), nbytes,
                                               stream.cuda_stream))
        else:
            def call(i):
                P.check(fn(seqs, n_slots, nH, nKV, hd, ctx, q.data_ptr(), K.data_ptr(), V.data_ptr(),
                           slots[i % groups].data_ptr(), lens.data_ptr(), out.data_ptr(), scratch.data_ptr(),
                           nbytes, stream.cuda_stream))

        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            for i in range(max(3, args.warmup)):
                call(i)
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for i in range(args.reps):
                    call(i)
            for _ in range(3):
                graph.replay()
            stream.synchronize()
            e0.record(stream)
            graph.replay()
            e1.record(stream)
            stream.synchronize()
        us = e0.elapsed_time(e1) / args.reps * 1e3
        del graph
        byts = seqs * ctx * 2 * nKV * hd * eb + 2 * seqs * nH * hd * 4
        gbs = byts / us / 1e3
        points.append({"kv": kv, "ctx": ctx, "seqs": seqs, "page_tokens": args.page_tokens, "us": round(us, 2),
                       "GB_s": round(gbs, 1),
                       "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                                    "frac": round(gbs / hbm, 4), "peak_source": hbm_kind},
                       "arena_MB": round(n_slots * slot_bytes / 1e6, 1)})
        print(f"# attn kv={kv} heads={nH}/{nKV} ctx={ctx} seqs={seqs} page={args.page_tokens}: {us:.1f} us, "
              f"{gbs:.0f} GB/s", file=sys.stderr, flush=True)
        del K, V
        torch.cuda.empty_cache()
    clk = clocks.stop()
    print(json.dumps({"micro": "attn", "metric": f"GQA decode attention HBM GB/s ({nH}/{nKV} heads x 128)",
                      "unit": "GB/s", "points": points, "clocks": clk, "reps": args.reps,
                      "config": {"l2": "launches rotate over sequence slots of an arena > 2 x L2",
                                 "values": "q f32, K / V N(0,1) stored as the point's kv type"}}), flush=True)
    return 0


# ------------------------------------------------------------------ oracle CPU timing
def oracle_token_time(pkg, m, n_threads: int, layer_reps: int) -> dict:
    """The reference CPU path (oracle) on one decode token: `layer_reps`
    single-layer steps and one final-norm + lm_head step, extrapolated to the
    whole model: s/token = n_layers * t_layer + t_head."""
    from oracle import ref

    layer = pkg.pack.synth_layer(m, 0)
    w = {"layers": [{"idx": 0, "buf": layer, "quant": m.quant}], "quant": m.quant}
    mid = ref.RefStage(m.dims(), 0, 1, False, False, w, n_threads)
    rng = np.random.default_rng(0)
    hid = (rng.standard_normal(m.hidden_dim) * 0.5).astype(np.float16).view(np.uint16)
    times = []
    for r in range(layer_reps):
        t0 = time.perf_counter()
        mid.forward(1, r, hidden=hid)
        times.append(time.perf_counter() - t0)
    mid.free()
    del layer
    head = pkg.pack.synth_tensor(m, "lm_head")
    x = rng.standard_normal(m.hidden_dim).astype(np.float32)
    t0 = time.perf_counter()
    ref.matvec(head, m.lm_head_quant, m.vocab, m.hidden_dim, x)
    t_head = time.perf_counter() - t0
    t_layer = statistics.mean(times)
    s_tok = m.n_layers * t_layer + t_head
    return {"tok_s": 1.0 / s_tok, "t_layer_s": t_layer, "t_head_s": t_head, "layer_times": times,
            "sample": f"EXTRAPOLATED: {layer_reps} single-token steps through one {m.name} layer (positions "
                      f"0..{layer_reps - 1}) + one lm_head matvec, scaled to {m.n_layers} layers; "
                      f"{n_threads} oracle thread(s)"}


def run_reference(args):
    """The reference CPU implementation of the path (the oracle's C
    restatement of web/inference-worker.js), all host threads."""
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    import __graft_entry__ as g

    pkg = g.load_package()
    m = pkg.pack.MODELS[args.model]
    n_threads = os.cpu_count() or 1
    os.environ["TABNET_ORACLE_THREADS"] = str(n_threads)
    warm = oracle_token_time(pkg, m, n_threads, max(1, args.warmup))
    res = oracle_token_time(pkg, m, n_threads, max(1, args.steps))
    # the reference engine is single-threaded JavaScript: the same sample on one thread
    os.environ["TABNET_ORACLE_THREADS"] = "1"
    one = oracle_token_time(pkg, m, 1, 2)
    os.environ["TABNET_ORACLE_THREADS"] = str(n_threads)
    # one reference "step" = one round: every micro-batch's sequence +1 token,
    # run one after another as the reference engine does
    s_round = args.microbatches / res["tok_s"]
    value = res["tok_s"]
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": s_round * 1e3, "higher_is_better": True, "scaling": SCALING,
            "vs_baseline": None, "dtype": "f64 accumulate, f32 storage (q4_0 weights)", "data": "synthetic",
            "impl": "reference", "config": workload_config(args, world),
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": n_threads, "kind": "port",
                             "sample": res["sample"], "extrapolated": True,
                             "single_thread": {"value": one["tok_s"], "unit": "tok/s", "cores": 1,
                                               "sample": one["sample"], "extrapolated": True}},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "detail": {"t_layer_s": res["t_layer_s"], "t_head_s": res["t_head_s"], "warm_tok_s": warm["tok_s"],
                       "single_thread_t_layer_s": one["t_layer_s"]}}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ our engine
def device_weights(pkg, torch, m, lo, hi, first, last):
    """Seeded packed weights written straight into device memory."""
    pack = pkg.pack
    bufs = {"layers": []}
    for i in range(lo, hi):
        t = torch.empty(pack.tensor_bytes(m, i), dtype=torch.uint8, device="cuda")
        pack.synth_device(m, i, t.data_ptr())
        bufs["layers"].append({"idx": i, "buf": t, "quant": m.quant})
    if first:
        bufs["embed"] = torch.empty(pack.tensor_bytes(m, "embed"), dtype=torch.uint8, device="cuda")
        pack.synth_device(m, "embed", bufs["embed"].data_ptr())
        bufs["embedQuant"] = m.embed_quant
    if last:
        for k in ("norm", "lm_head"):
            bufs[k] = torch.empty(pack.tensor_bytes(m, k), dtype=torch.uint8, device="cuda")
            pack.synth_device(m, k, bufs[k].data_ptr())
        bufs["lmHeadQuant"] = m.lm_head_quant
    bufs["on_device"] = True
    bufs["quant"] = m.quant
    torch.cuda.synchronize()
    return bufs


def matvec_bytes(pkg, m, cls: str, T: int = 1) -> int:
    """Algorithmic bytes of one matvec launch: packed weights + f32 x + f32 y
    (read and written again for the residual epilogues)."""
    from_pack = pkg.pack
    H, F, V = m.hidden_dim, m.ffn_dim, m.vocab
    hd = H // m.n_heads
    q, kv = m.n_heads * hd, m.n_kv_heads * hd
    qb = lambda n: from_pack.quant_bytes(n, m.quant)
    if cls == "matvec_qkv":
        return qb((q + 2 * kv) * H) + 4 * T * (H + q + 2 * kv)
    if cls == "matvec_o":
        return qb(H * q) + 4 * T * (q + 2 * H)
    if cls == "matvec_gate_up":
        return qb(2 * F * H) + 4 * T * (H + F)
    if cls == "matvec_down":
        return qb(H * F) + 4 * T * (F + 2 * H)
    if cls == "matvec_lm_head":
        return from_pack.quant_bytes(V * H, m.lm_head_quant) + 4 * T * (H + V)
    raise KeyError(cls)


def run_ours(args):
    rank, world, local = dist_env()
    import torch

    torch.cuda.set_device(local)
    import __graft_entry__ as g

    pkg = g.load_package()
    lib = pkg._lib.load()
    m = pkg.pack.MODELS[args.model]
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    M = args.microbatches
    assert M >= world, "need at least one micro-batch per stage"
    L = pkg.pack.layer_layout(m)["total"]
    hd = m.hidden_dim // m.n_heads
    kv_layer = pkg.planner.kv_bytes_per_layer(m.n_kv_heads, hd, args.prompt + 64, 4) * M
    plan = pkg.planner.plan_gpus(m.n_layers, world, L, kv_layer, pkg.pack.tensor_bytes(m, "embed"),
                                 pkg.pack.tensor_bytes(m, "lm_head"))
    st = plan[rank]
    lo, hi = st["layers"]
    # decode positions: pipeline warm-up + timed + e2e + profiled rounds, then
    # the fused pass (warm-up + timed + e2e)
    n_decode = 2 * max(3, args.warmup) + 6 * args.steps + 12
    t_init = time.perf_counter()
    w = device_weights(pkg, torch, m, lo, hi, st["is_first"], st["is_last"])
    ctx = pkg.initStage({"arch": "llama", "dims": m.dims(), "layers": [lo, hi], "is_first": st["is_first"],
                         "is_last": st["is_last"], "weights": w,
                         "opts": {"device": local, "max_ctx": args.prompt + n_decode + 4, "max_seqs": M,
                                  "max_tokens_per_step": 512, "kv_dtype": args.kv_cache,
                                  "kv_page_tokens": args.kv_page_tokens}})
    del w
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    t_init = time.perf_counter() - t_init
    prompts = [pkg.pack.synth_prompt(m, args.prompt, seed=100 + mb) for mb in range(M)]
    t_pre = time.perf_counter()
    first_tok = pkg.pipeline.prefill(ctx, rank, world, prompts, m.hidden_dim)
    torch.cuda.synchronize()
    t_pre = time.perf_counter() - t_pre
    pipe = pkg.pipeline.Pipeline(pkg.pipeline.DeviceStage(ctx, M), rank, world, M, m.hidden_dim, deadline_s=900)
    pipe.pos = [[args.prompt] for _ in range(M)]
    if rank == 0:
        pipe.tok.copy_(torch.tensor(first_tok, dtype=torch.int32).view(M, 1))

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            import torch.distributed as dist

            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        import torch.distributed as dist

        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # warm-up (captures the decode-step CUDA graph)
    pipe.rounds(args.warmup)
    barrier()
    # ---- timed: device-resident inputs, CUDA events on the stage stream
    clocks = ClockSampler(physical_gpu(local))
    clocks.start()
    time.sleep(0.3)
    barrier()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    # K rounds in the pipeline's steady state: with several stages the call
    # runs one round before and one after them (the fill and the drain), and
    # each rank's events bracket its own K x M steps
    lead = 1 if world > 1 else 0
    torch.cuda.nvtx.range_push("decode_timed")  # (profilers: --nvtx-include decode_timed/)
    pipe.rounds(lead + args.steps + lead, wait=False, marks={lead * M: ev0, (lead + args.steps) * M: ev1})
    torch.cuda.nvtx.range_pop()
    barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    clk = clocks.stop()
    info = ctx.info()
    tokens = args.steps * M
    value = tokens / (ms / 1e3)
    launches = info["launches_last_step"] * tokens
    # ---- e2e: the host-buffer API (tn_stage_forward) for every micro-batch step
    # (same schedule; a step's input frame comes to the host from the receive
    # slot and its output goes back to the send slot, so the stages still work
    # on different micro-batches at once)
    barrier()
    tm = {lead * M: None, (lead + args.steps) * M: None}
    pipe.rounds_host(ctx, lead + args.steps + lead, marks=tm)
    e2e_s = max_over_ranks(tm[(lead + args.steps) * M] - tm[lead * M])
    e2e_val = tokens / e2e_s
    # per round: token ids in (rank 0) and out (last rank), one fp16 frame into
    # and one out of the host API at each of the world - 1 stage boundaries
    h2d = d2h = 4 * M + 2 * m.hidden_dim * M * (world - 1)
    # ---- profiled pass: per-kernel device time (CUDA events around each launch)
    pkg._lib.check(lib.tn_stage_set_profile(ctx.handle, 1))
    ctx.profile(reset=True)
    if world == 1:
        pipe.rounds_host(ctx, args.steps)
    prof = ctx.profile() if world == 1 else {}
    pkg._lib.check(lib.tn_stage_set_profile(ctx.handle, 0))
    fused = None
    if world == 1 and not args.no_fused:
        fused = fused_decode(pkg, torch, ctx, pipe, args)
    peak, peak_kind = measured_peaks()
    mv = [k for k in prof if k.startswith("matvec") and prof[k][1] > 0]
    roof = None
    if mv:
        # dominant kernel: the tensor-core matvec k_mmv; its gate/up launches
        # carry 55% of a layer's weight bytes, so the roofline is quoted on them
        tot_bytes = sum(matvec_bytes(pkg, m, k) * prof[k][1] for k in mv)
        tot_ms = sum(prof[k][0] for k in mv)
        n_launch = sum(prof[k][1] for k in mv)
        dom = "matvec_gate_up" if "matvec_gate_up" in mv else max(mv, key=lambda k: prof[k][0])
        dom_bytes = matvec_bytes(pkg, m, dom)
        dom_us = prof[dom][0] / prof[dom][1] * 1e3
        achieved = dom_bytes / (dom_us / 1e6) / 1e9
        traffic = None
        tf = ROOT / "profiles" / "k_mmv_gate_up_70b_traffic.json"
        if tf.exists():
            traffic = json.loads(tf.read_text()).get("dram_bytes_per_launch")
        roof = {"kernel": f"k_mmv ({m.quant} tensor-core matvec, mma.m16n8k32 s8, 1 token), {dom} launches",
                "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                "algorithmic_bytes_per_launch": int(dom_bytes), "launches": prof[dom][1],
                "avg_launch_us": round(dom_us, 2),
                "all_matvecs": {"achieved": round(tot_bytes / (tot_ms / 1e3) / 1e9, 1), "launches": n_launch,
                                "share_of_step_time": round(tot_ms / sum(v[0] for v in prof.values()), 4)},
                # every matvec class of the step: average launch time and GB/s
                "per_class": {k: {"avg_launch_us": round(prof[k][0] / prof[k][1] * 1e3, 2),
                                  "achieved": round(matvec_bytes(pkg, m, k) / (prof[k][0] / prof[k][1] / 1e3) / 1e9,
                                                    1),
                                  "frac": round(matvec_bytes(pkg, m, k) / (prof[k][0] / prof[k][1] / 1e3) / 1e9
                                                / peak, 4)} for k in mv},
                "timing": "CUDA events around each launch on the stage stream (profiled pass after the timed one)"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        n_threads = os.cpu_count() or 1
        os.environ["TABNET_ORACLE_THREADS"] = str(n_threads)
        o = oracle_token_time(pkg, m, n_threads, 3)
        cpu = {"value": o["tok_s"], "unit": "tok/s", "cores": n_threads, "kind": "port", "sample": o["sample"],
               "extrapolated": True}
    step_bytes = pkg.pack.model_bytes(m) + M * m.n_layers * 2 * (args.prompt + args.warmup + args.steps) * \
        m.n_kv_heads * hd * 4
    line = {"metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": SCALING, "vs_baseline": None, "dtype": "f32 (q4_0 weights, f32 activations and accumulate)",
            "data": "synthetic (seeded weights and prompts)", "config": workload_config(args, world),
            "e2e": {"value": round(e2e_val, 3) if e2e_val else None, "unit": "tok/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": launches, "clocks": clk, "roofline": roof, "cpu_baseline": cpu, "fused": fused,
            "detail": {"weight_roofline_tok_s": round(peak * 1e9 / pkg.pack.model_bytes(m) * world, 1),
                       "step_bytes_whole_model": step_bytes, "init_s": round(t_init, 1), "prefill_s": round(t_pre, 1),
                       "prefill_tok_s": round(M * args.prompt / t_pre, 1),
                       "profile_ms": {k: [round(v[0], 3), v[1]] for k, v in prof.items()}}}
    if rank == 0:
        print(json.dumps(line), flush=True)
    pkg.freeStage(ctx)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def fused_decode(pkg, torch, ctx, pipe, args) -> dict:
    """One GPU: the M micro-batches' decode steps fused into one M-row step
    per token (the stage batches concurrent sequences), timed like the
    pipeline rounds -- device-resident token ids, CUDA events on the stage
    stream -- and end to end through the host-buffer batch API."""
    lib, P, M = pipe.stage.lib, pkg._lib, pipe.M
    ids = (C.c_uint64 * M)(*[ctx.seq_key(mb) for mb in range(M)])
    tok = pipe.tok.view(-1)

    def step():
        pos = (C.c_int32 * M)(*[p[0] for p in pipe.pos])
        d = P.StepDesc(n_seqs=M, seq_ids=ids, token_pos=pos, d_token_ids=tok.data_ptr(),
                       d_token_out=tok.data_ptr(), temperature=0.0, top_p=0.95, rng_seed=0)
        P.check(lib.tn_stage_step_async(ctx.handle, C.byref(d), pipe.stage.stream_ptr))
        for mb in range(M):
            pipe.pos[mb][0] += 1

    with torch.cuda.stream(pipe.stream):
        for _ in range(max(3, args.warmup)):
            step()
    torch.cuda.synchronize()
    clocks = ClockSampler(physical_gpu(torch.cuda.current_device()))
    clocks.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(pipe.stream):
        ev0.record(pipe.stream)
        for _ in range(args.steps):
            step()
        ev1.record(pipe.stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    launches = ctx.info()["launches_last_step"]
    # end to end: one forward_batch call (token ids in, sampled ids out) per step
    toks = tok.cpu().tolist()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        out = pkg.forward_batch(ctx, [{"seq_id": mb, "token_pos": pipe.pos[mb][0], "token_ids": [toks[mb]],
                                       "temperature": 0} for mb in range(M)])
        toks = [o["token_id"] for o in out]
        for mb in range(M):
            pipe.pos[mb][0] += 1
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    # a profiled pass of two steps: device time per launch class
    P.check(lib.tn_stage_set_profile(ctx.handle, 1))
    ctx.profile(reset=True)
    for _ in range(2):
        out = pkg.forward_batch(ctx, [{"seq_id": mb, "token_pos": pipe.pos[mb][0], "token_ids": [toks[mb]],
                                       "temperature": 0} for mb in range(M)])
        toks = [o["token_id"] for o in out]
        for mb in range(M):
            pipe.pos[mb][0] += 1
    prof = {k: [round(v[0] / 2, 3), v[1] // 2] for k, v in ctx.profile().items() if v[1]}
    P.check(lib.tn_stage_set_profile(ctx.handle, 0))
    n_tok = args.steps * M
    return {"value": round(n_tok / (ms / 1e3), 3), "unit": "tok/s", "rows_per_step": M,
            "profile_ms_per_step": prof,
            "ms_per_step": round(ms / args.steps, 4), "steps": args.steps, "gpu_launches": launches * args.steps,
            "clocks": clk,
            "e2e": {"value": round(n_tok / e2e_s, 3), "unit": "tok/s", "h2d_bytes_per_step": 4 * M,
                    "d2h_bytes_per_step": 4 * M},
            "schedule": f"all {M} sequences' next tokens as one {M}-row step (matvecs in groups of up to "
                        "4 token columns); value above is the micro-batch schedule"}


def main(argv=None):
    args = parse_args(argv)
    if args.micro == "matvec":
        return micro_matvec(args)
    if args.micro == "attn":
        return micro_attn(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
