"""Multi-GPU decode pipeline over the stage engine: one process per GPU, one
contiguous layer slice (stage) per rank, activations hopping between ranks
as fp16 [rows, H] frames.

This is the runner the reference builds from its mesh of stage workers (each
worker runs initStage / forward for its slice, web/inference-worker.js:417-490,
and hands the hidden frame to the next one, web/tabnet-node.js:154-185).  Here
the ranks of one node exchange frames over NCCL point-to-point (NVLink /
NVSwitch); gloo on CPU runs the same code for the host-logic tests.

Schedule.  planner.pipeline_tick: at tick tau rank r steps micro-batch step
j = tau - r; the frame of step j arrives from rank r - 1 at the start of the
tick and the output of step j - 1 leaves for rank r + 1; the last rank's
sampled tokens return to rank 0 for the micro-batch's next step (n_micro >=
world keeps them in time).  All point-to-point operations of a tick are
posted together.

Ordering without host waits.  Every NCCL operation is issued while the stage
stream is the current stream: the NCCL stream first waits for the stage's
earlier work (the step that wrote the frame being sent, or the step that read
the buffer being received into), and work.wait() makes the stage stream wait
for the transfer -- device-side, the host only enqueues.  Each micro-batch has
its own input / output frame slots, so a frame is received while other
micro-batches compute.  The host blocks once per call, on an event after the
last tick, with a deadline.

Failure detection (the reference's heartbeat / stale sweep,
web/mesh-coordinator.js:96-113, for ranks of one job): a rank that dies or
stalls leaves its peers' transfers incomplete.  On gloo, each transfer's host
wait carries the remaining deadline; on NCCL, the final event is polled until
the deadline.  Either way the call raises PipelineError with code TN_ETIMEOUT
(TN_ESTATE when the transport reports a lost peer) after aborting the process
group's communicators (ncclCommAbort under ProcessGroupNCCL), so no NCCL
kernel is left waiting for a peer that will not come.  Create the NCCL group
with nccl_group_options() for a non-blocking communicator.
"""
from __future__ import annotations

import ctypes as C
import datetime
import time

import numpy as np

from . import _lib, planner


class PipelineError(_lib.TnError):
    """A pipeline call that could not complete: code TN_ETIMEOUT when a peer's
    transfer did not finish within the deadline (a stalled or dead rank),
    TN_ESTATE when the transport reported the peer lost.  `rank` is this
    process's rank and `tick` the schedule tick (-1: the final drain)."""

    def __init__(self, code: int, msg: str, rank: int, tick: int):
        super().__init__(code, msg)
        self.rank, self.tick = rank, tick


def nccl_group_options():
    """ProcessGroupNCCL options for the pipeline's group: a non-blocking
    communicator, so that an abort after a missed deadline returns instead
    of waiting on a peer."""
    from torch.distributed import ProcessGroupNCCL

    o = ProcessGroupNCCL.Options()
    o.config.blocking = 0
    return o


class DeviceStage:
    """A StageCtx stepped on device buffers through tn_stage_step_async (no
    host copies): micro-batch mb holds `rows` sequences, seq ids mb * rows + i."""

    def __init__(self, ctx, n_micro: int, rows: int = 1):
        self.ctx, self.rows = ctx, rows
        self.lib = _lib.load()
        self.is_first, self.is_last = ctx.is_first, ctx.is_last
        self.stream_ptr = self.lib.tn_stage_stream(ctx.handle)
        self._ids = [(C.c_uint64 * rows)(*[ctx.seq_key(mb * rows + i) for i in range(rows)]) for mb in range(n_micro)]

    def step(self, mb: int, pos: list[int], tok_in, hid_in, tok_out, hid_out) -> None:
        d = _lib.StepDesc(n_seqs=len(pos), seq_ids=self._ids[mb], token_pos=(C.c_int32 * len(pos))(*pos),
                          temperature=0.0, top_p=0.95, rng_seed=0)
        if self.is_first:
            d.d_token_ids = tok_in.data_ptr()
        else:
            d.d_hidden_in = hid_in.data_ptr()
        if self.is_last:
            d.d_token_out = tok_out.data_ptr()
        else:
            d.d_hidden_out = hid_out.data_ptr()
        _lib.check(self.lib.tn_stage_step_async(self.ctx.handle, C.byref(d), self.stream_ptr))

    def check(self) -> None:
        """Raise TnError(TN_ETIMEOUT) if a kernel's bounded wait gave up in a
        step since the last check (tn_stage_check; the stage recovers)."""
        _lib.check(self.lib.tn_stage_check(self.ctx.handle, self.stream_ptr))


class Pipeline:
    """One rank of the decode pipeline.

    stage: DeviceStage (or any object with is_first, is_last and
      step(mb, pos, tok_in, hid_in, tok_out, hid_out) enqueueing one step;
      `stream_ptr` when it runs on a CUDA stream).
    Frame slots (per micro-batch, on `device`): tok [M, rows] int32 -- rank 0's
    input tokens, refilled by the last rank's samples; hin / hout [M, rows, H]
    fp16 -- the received and the produced hidden frames; tok_out [M, rows] --
    the last rank's samples on their way back.  pos[mb][i] is the next
    position of sequence i of micro-batch mb.
    """

    def __init__(self, stage, rank: int, world: int, n_micro: int, hidden: int, *, rows: int = 1,
                 device=None, group=None, deadline_s: float = 120.0):
        import torch

        if n_micro < world:
            raise _lib.TnError(_lib.TN_EINVAL, f"{n_micro} micro-batches for {world} stages: need at least one each")
        self.torch, self.stage = torch, stage
        self.rank, self.world, self.M, self.H, self.rows = rank, world, n_micro, hidden, rows
        self.group, self.deadline_s = group, deadline_s
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        z = lambda *shape, dt: torch.zeros(shape, dtype=dt, device=self.device)
        self.tok = z(n_micro, rows, dt=torch.int32)
        self.tok_out = z(n_micro, rows, dt=torch.int32)
        self.hin = z(n_micro, rows, hidden, dt=torch.float16)
        self.hout = z(n_micro, rows, hidden, dt=torch.float16)
        self.pos = [[0] * rows for _ in range(n_micro)]
        sp = getattr(stage, "stream_ptr", None)
        self.stream = torch.cuda.ExternalStream(sp) if (sp and self.device.type == "cuda") else None

    # -------------------------------------------------------------- helpers
    def _stream_ctx(self):
        import contextlib

        return self.torch.cuda.stream(self.stream) if self.stream is not None else contextlib.nullcontext()

    def _step(self, mb: int) -> None:
        p = self.pos[mb]
        tok_out = self.tok if self.world == 1 else self.tok_out  # one stage: samples feed its own next step
        self.stage.step(mb, list(p), self.tok[mb], self.hin[mb], tok_out[mb], self.hout[mb])
        self.pos[mb] = [x + 1 for x in p]

    def _fail(self, tick: int, err: Exception | None, timed_out: bool):
        self.abort()
        code = _lib.TN_ETIMEOUT if timed_out or err is None or "timeout" in str(err).lower() \
            or "timed out" in str(err).lower() else _lib.TN_ESTATE
        what = f"{type(err).__name__}: {err}" if err is not None else f"no completion within {self.deadline_s:g} s"
        raise PipelineError(code, f"rank {self.rank}, tick {tick}: a peer's transfer did not complete ({what})",
                            self.rank, tick) from err

    def abort(self) -> None:
        """Abort the group's communicators (outstanding NCCL kernels return)."""
        import torch.distributed as dist

        if self.world == 1 or not dist.is_initialized():
            return
        try:
            pg = self.group or dist.distributed_c10d._get_default_group()
            pg.abort()
        except Exception:
            pass

    # ------------------------------------------------------------ schedule
    def rounds(self, n_rounds: int, wait: bool = True, marks: dict | None = None) -> None:
        """n_rounds x M micro-batch steps on this rank, fill and drain
        included.  wait: return when this rank's work is complete (or raise
        PipelineError at the deadline); else return once it is enqueued.
        marks: {j: CUDA event} recorded on the stage stream just before this
        rank's j-th step of the call (j = n_rounds x M: after its last), so a
        caller can time whole rounds in the pipeline's steady state."""
        import torch.distributed as dist

        torch, W, M, r = self.torch, self.world, self.M, self.rank
        n = n_rounds * M
        t_end = time.monotonic() + self.deadline_s
        gloo = self.device.type != "cuda"
        bufs = {"recv_token": self.tok, "recv_hidden": self.hin, "send_hidden": self.hout,
                "send_token": self.tok_out}
        def mark(j):
            if marks and j in marks:
                marks[j].record(self.stream if self.stream is not None else torch.cuda.current_stream())

        with self._stream_ctx():
            if W == 1:
                for j in range(n):
                    mark(j)
                    self._step(j % M)
                mark(n)
            else:
                j_local = 0
                for tau in range(planner.pipeline_ticks(W, n)):
                    sched, mb = planner.pipeline_tick(r, W, M, n, tau)
                    ops = [dist.P2POp(dist.irecv if kind.startswith("recv") else dist.isend, bufs[kind][b], peer,
                                      group=self.group)
                           for kind, b, peer in sched]
                    if ops:
                        try:
                            works = dist.batch_isend_irecv(ops)
                            for w in works:
                                if gloo:
                                    left = t_end - time.monotonic()
                                    if left <= 0:
                                        self._fail(tau, None, True)
                                    w.wait(timeout=datetime.timedelta(seconds=left))
                                else:
                                    w.wait()  # the stage stream waits for the transfer
                        except PipelineError:
                            raise
                        except Exception as e:  # a lost peer or a transport timeout
                            self._fail(tau, e, False)
                    if mb is not None:
                        mark(j_local)
                        self._step(mb)
                        j_local += 1
                mark(n)
        if wait:
            self._drain(t_end)

    def _drain(self, t_end: float) -> None:
        torch = self.torch
        if self.device.type != "cuda":
            return
        ev = torch.cuda.Event()
        ev.record(self.stream if self.stream is not None else torch.cuda.current_stream())
        while not ev.query():
            if time.monotonic() > t_end:
                self._fail(-1, None, True)
            time.sleep(0.0002)
        check = getattr(self.stage, "check", None)
        if check is not None:
            try:
                check()
            except _lib.TnError as e:  # a device-side bounded wait gave up in one of the steps
                raise PipelineError(e.code, f"rank {self.rank}: {e}", self.rank, -1) from e

    # ----------------------------------------------------------- host API
    def rounds_host(self, ctx, n_rounds: int, marks: dict | None = None) -> None:
        """The same schedule with every stage step through the host-buffer API
        (tn_stage_forward): a step's input frame comes to the host from the
        receive slot and its output frame goes back to the send slot, so the
        end-to-end path of a caller holding host buffers is timed.  marks:
        {j: None}, filled with time.perf_counter() just before this rank's
        j-th step of the call (j = n_rounds x M: after its last)."""
        import torch.distributed as dist

        from . import engine

        torch, W, M, r = self.torch, self.world, self.M, self.rank
        n = n_rounds * M
        bufs = {"recv_token": self.tok, "recv_hidden": self.hin, "send_hidden": self.hout,
                "send_token": self.tok_out}
        j_local = 0

        def mark(j):
            if marks is not None and j in marks:
                marks[j] = time.perf_counter()

        for tau in range(planner.pipeline_ticks(W, n) if W > 1 else n):
            if W == 1:
                sched, mb = [], tau % M
            else:
                sched, mb = planner.pipeline_tick(r, W, M, n, tau)
            ops = [dist.P2POp(dist.irecv if kind.startswith("recv") else dist.isend, bufs[kind][b], peer,
                              group=self.group)
                   for kind, b, peer in sched]
            if ops:
                for w in dist.batch_isend_irecv(ops):
                    w.wait()
            if mb is None:
                continue
            mark(j_local)
            j_local += 1
            reqs = []
            for i in range(self.rows):
                req = {"seq_id": mb * self.rows + i, "token_pos": self.pos[mb][i], "temperature": 0}
                if ctx.is_first:
                    req["token_ids"] = [int(self.tok[mb, i].item())]
                else:
                    req["hidden"] = self.hin[mb, i].cpu().numpy().view(np.uint16)
                reqs.append(req)
            outs = engine.forward_batch(ctx, reqs)
            for i, out in enumerate(outs):
                if ctx.is_last:
                    (self.tok if W == 1 else self.tok_out)[mb, i] = out["token_id"]
                else:
                    self.hout[mb, i].copy_(torch.from_numpy(out["hidden"].view(np.float16)))
            self.pos[mb] = [x + 1 for x in self.pos[mb]]
        mark(j_local)
        if self.device.type == "cuda":
            torch.cuda.synchronize()

    def frame_bytes_per_round(self) -> int:
        """Host bytes in and out per round of rounds_host on this rank."""
        per = 4 * self.rows if (self.rank == 0 or self.rank == self.world - 1) else 0
        return self.M * (per + (2 * self.H * self.rows if self.world > 1 else 0))


def prefill(ctx, rank: int, world: int, prompts: list[list[int]], hidden: int, group=None) -> list[int] | None:
    """Prompt prefill through the host API, one micro-batch of one sequence
    per prompt (seq id = prompt index): rank 0 embeds the prompts, every
    position's hidden frame hops to the next rank (hop mode all, so each
    stage's KV covers the prompt), and the last rank's first sampled tokens
    return to rank 0.  Returns them on rank 0 (and the last rank)."""
    import torch
    import torch.distributed as dist

    from . import engine

    M, L = len(prompts), len(prompts[0])
    if rank == 0:
        reqs = [{"seq_id": mb, "token_pos": 0, "token_ids": prompts[mb], "temperature": 0, "hop_mode": "all"}
                for mb in range(M)]
    else:
        buf = torch.empty((M, L, hidden), dtype=torch.float16, device="cuda")
        dist.recv(buf, rank - 1, group=group)
        hid = buf.cpu().numpy().view(np.uint16)
        reqs = [{"seq_id": mb, "token_pos": 0, "hidden": hid[mb], "temperature": 0, "hop_mode": "all"}
                for mb in range(M)]
    out = engine.forward_batch(ctx, reqs)
    if ctx.is_last:
        first = [o["token_id"] for o in out]
        if world > 1:
            dist.send(torch.tensor(first, dtype=torch.int32, device="cuda"), 0, group=group)
        return first
    hs = np.stack([o["hidden"] for o in out]).astype(np.uint16)
    dist.send(torch.from_numpy(hs.view(np.float16)).cuda(), rank + 1, group=group)
    if rank == 0:
        t = torch.empty(M, dtype=torch.int32, device="cuda")
        dist.recv(t, world - 1, group=group)
        return t.cpu().tolist()
    return None
