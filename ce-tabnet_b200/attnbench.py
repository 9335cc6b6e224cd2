"""Single-kernel microbenchmark of decode attention (one query row).

70B head shapes (64 query heads, 8 KV heads, head_dim 128) at a given cached
length; every launch reads another sequence slot of a KV arena larger than the
126 MB L2, so K / V rows come from HBM as in the decode step.  Times `reps`
tn_attention calls with CUDA events and prints microseconds per call and the
K / V bytes read per second.  This is the small case attention profiles are
taken on:

    python ce-tabnet_b200/attnbench.py [cached_len] [reps]
"""
from __future__ import annotations

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

N_HEADS, N_KV, HEAD_DIM = 64, 8, 128


def main() -> None:
    import torch

    import __graft_entry__ as ge

    pkg = ge.load_package()
    lib, P = pkg._lib.load(), pkg._lib
    L = int(sys.argv[1]) if len(sys.argv) > 1 else 1057
    reps = int(sys.argv[2]) if len(sys.argv) > 2 else 20
    max_ctx = L
    slot_bytes = 2 * N_KV * max_ctx * HEAD_DIM * 4
    n_slots = max(2, int(2 * 126e6 // slot_bytes) + 1)  # arena > 2 x L2
    g = torch.Generator(device="cuda").manual_seed(7)
    K = torch.randn((n_slots, N_KV, max_ctx, HEAD_DIM), device="cuda", generator=g)
    V = torch.randn((n_slots, N_KV, max_ctx, HEAD_DIM), device="cuda", generator=g)
    q = torch.randn((1, N_HEADS * HEAD_DIM), device="cuda", generator=g)
    out = torch.empty_like(q)
    lens = torch.tensor([L], dtype=torch.int32, device="cuda")
    slots = [torch.tensor([s], dtype=torch.int32, device="cuda") for s in range(n_slots)]
    nbytes = lib.tn_attention_scratch_bytes(1, N_HEADS, N_KV, HEAD_DIM, max_ctx)
    scratch = torch.empty(max(nbytes, 256), dtype=torch.uint8, device="cuda")

    def call(i):
        P.check(lib.tn_attention(1, n_slots, N_HEADS, N_KV, HEAD_DIM, max_ctx, q.data_ptr(), K.data_ptr(),
                                 V.data_ptr(), slots[i % n_slots].data_ptr(), lens.data_ptr(), out.data_ptr(),
                                 scratch.data_ptr(), nbytes, None))

    for i in range(3):
        call(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(reps):
        call(3 + i)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / reps * 1e3
    kv = 2 * N_KV * L * HEAD_DIM * 4
    print(f"attention 1 row, {N_HEADS}/{N_KV} heads x {HEAD_DIM}, {L} cached: {us:.1f} us/call, "
          f"{kv / us / 1e3:.0f} GB/s of K/V ({n_slots} slots, {n_slots * slot_bytes / 1e6:.0f} MB arena)", flush=True)


if __name__ == "__main__":
    main()
