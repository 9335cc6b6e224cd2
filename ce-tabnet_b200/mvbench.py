"""Single-matrix microbenchmark of the decode matvec (one token).

Builds one seeded q4_0 / q8_0 matrix on the device, times `reps` launches of
tn_matrix_matvec with CUDA events and prints microseconds per launch and the
weight bytes streamed per second.  This is the small case that kernel
profiles are taken on (one matrix of a few hundred MB, larger than the L2):

    python ce-tabnet_b200/mvbench.py 57344x8192 [reps] [q4_0|q8_0]
"""
from __future__ import annotations

import ctypes as C
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

# the 70B layer shapes: fused QKV, attention output, fused gate/up, down
SHAPES = [(10240, 8192), (8192, 8192), (57344, 8192), (8192, 28672)]


def main() -> None:
    import torch

    import __graft_entry__ as ge

    pkg = ge.load_package()
    lib, P = pkg._lib.load(), pkg._lib
    only = sys.argv[1] if len(sys.argv) > 1 else None
    reps = int(sys.argv[2]) if len(sys.argv) > 2 else 20
    quant = sys.argv[3] if len(sys.argv) > 3 else "q4_0"
    shapes = SHAPES if not only else [tuple(int(v) for v in only.split("x"))]
    for rows, cols in shapes:
        m = pkg.pack.ModelDims(cols, 1, 1, 1, rows, 0, 1e4, quant, quant, quant, 5)
        nbytes = pkg.pack.quant_bytes(rows * cols, quant)
        src = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        d = m.c_dims()
        P.check(lib.tn_synth_tensor(5, P.TN_TAG_EMBED, C.byref(d), P.QUANT[quant], src.data_ptr(), 1, None))
        torch.cuda.synchronize()
        h = C.c_void_p()
        P.check(lib.tn_matrix_create(0, P.QUANT[quant], rows, cols, src.data_ptr(), nbytes, 1, C.byref(h)))
        del src
        x = torch.randn(1, cols, device="cuda")
        y = torch.empty(1, rows, device="cuda")
        for _ in range(3):
            P.check(lib.tn_matrix_matvec(h, 1, x.data_ptr(), y.data_ptr(), None))
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            P.check(lib.tn_matrix_matvec(h, 1, x.data_ptr(), y.data_ptr(), None))
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) / reps * 1e3
        note = "" if nbytes > 126e6 else " (fits in L2: repeated launches read it from there)"
        print(f"{rows}x{cols} {quant}: {us:.1f} us/launch, {nbytes / us / 1e3:.0f} GB/s of weights{note}", flush=True)
        lib.tn_matrix_free(h)


if __name__ == "__main__":
    main()
