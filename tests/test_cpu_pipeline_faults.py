"""The pipeline runner (ce-tabnet_b200/pipeline.py) on CPU gloo ranks with a
toy stage per rank: a full run reproduces a sequential pass of the same
stages, and a rank that dies or stalls part way makes its peer's call end
with PipelineError at the deadline instead of waiting for ever.  The failure
is made on the host (a process that exits, a step that sleeps); nothing here
touches a GPU.  The NCCL path differs only in how the deadline is observed
(an event polled on the stage stream) and in the abort reaching
ncclCommAbort."""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

H = 4


def _first(tok, pos):
    return [(tok * 7 + pos + i) % 251 for i in range(H)]


def _mid(h, rank, pos):
    return [(2 * v + rank + pos) % 251 for v in h]


def _last(h, pos):
    return (sum(h) * 31 + pos) % 1009


def _sequential(world, n_mb, n_steps, first_tokens):
    out = []
    for j in range(n_steps):
        mb, pos = j % n_mb, j // n_mb
        tok = first_tokens[mb] if j < n_mb else out[j - n_mb]
        h = _first(tok, pos)
        for r in range(1, world - 1):
            h = _mid(h, r, pos)
        out.append(_last(h, pos))
    return out


class ToyStage:
    """A stage of the toy model on CPU tensors (one sequence per micro-batch),
    with an optional host-side fault at this rank's k-th step."""

    def __init__(self, rank, world, fault=None):
        self.rank, self.world = rank, world
        self.is_first, self.is_last = rank == 0, rank == world - 1
        self.fault, self.n = fault, 0
        self.seen = []  # (mb, pos, token) of the first stage's inputs

    def step(self, mb, pos, tok_in, hid_in, tok_out, hid_out):
        if self.fault and self.n == self.fault[1]:
            if self.fault[0] == "exit":
                os._exit(3)  # the rank dies between steps
            time.sleep(self.fault[2])  # the rank stalls
        self.n += 1
        p = pos[0]
        if self.is_first:
            self.seen.append((mb, p, int(tok_in[0])))
            h = _first(int(tok_in[0]), p)
        else:
            h = [int(v) for v in hid_in[0].tolist()]
            if not self.is_last:
                h = _mid(h, self.rank, p)
        if self.is_last:
            tok_out[0] = _last(h, p)
        else:
            hid_out[0] = torch.tensor(h, dtype=torch.float16)


def _rank_main(rank, world, port, n_mb, n_rounds, first_tokens, fault, deadline, result):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    import __graft_entry__ as ge

    pkg = ge.load_package()
    torch.set_num_threads(1)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    stage = ToyStage(rank, world, fault if fault and fault[-1] == rank else None)
    pipe = pkg.pipeline.Pipeline(stage, rank, world, n_mb, H, device="cpu", deadline_s=deadline)
    if rank == 0:
        pipe.tok[:, 0] = torch.tensor(first_tokens, dtype=torch.int32)
    t0 = time.monotonic()
    try:
        pipe.rounds(n_rounds)
        result[rank] = ("ok", stage.seen if rank == 0 else None, time.monotonic() - t0)
    except pkg.pipeline.PipelineError as e:
        result[rank] = ("error", e.code, time.monotonic() - t0)
        os._exit(0)  # peers may be gone: leave without the group's teardown
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, n_mb, n_rounds, first_tokens, fault=None, deadline=60.0, join_s=90):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        result = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank_main,
                             args=(r, world, port, n_mb, n_rounds, first_tokens, fault, deadline, result))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(join_s)
        codes = [p.exitcode for p in procs]
        for p in procs:
            if p.is_alive():
                p.kill()
        return codes, dict(result)


@pytest.mark.parametrize("world,n_mb", [(2, 2), (3, 4)])
def test_pipeline_runner_matches_sequential(world, n_mb):
    n_rounds = 3
    first = [11 * (i + 1) for i in range(n_mb)]
    codes, res = _run(world, n_mb, n_rounds, first)
    assert codes == [0] * world, codes
    assert all(res[r][0] == "ok" for r in range(world))
    want = _sequential(world, n_mb, n_rounds * n_mb, first)
    # rank 0's input token of step j (j >= n_mb) is the last stage's output of step j - n_mb
    for mb, pos, tok in res[0][1]:
        j = pos * n_mb + mb
        assert tok == (first[mb] if j < n_mb else want[j - n_mb]), (mb, pos)


def test_pipeline_dead_rank_ends_peer_call():
    """Rank 1 exits at its 3rd step: rank 0's call ends with PipelineError
    (TN_ESTATE for the lost connection or TN_ETIMEOUT at the deadline)."""
    codes, res = _run(2, 2, 4, [5, 6], fault=("exit", 2, 1), deadline=8.0)
    assert codes[1] == 3
    assert res[0][0] == "error", res
    assert res[0][1] in (-6, -7)  # TN_ESTATE, TN_ETIMEOUT
    assert res[0][2] < 30


def test_pipeline_stalled_rank_times_out():
    """Rank 1 sleeps 25 s at its 2nd step: rank 0 gives up at its 3 s
    deadline with TN_ETIMEOUT; rank 1 then finds its peer gone."""
    codes, res = _run(2, 2, 4, [5, 6], fault=("stall", 1, 25, 1), deadline=3.0, join_s=60)
    assert res[0][0] == "error", res
    assert res[0][1] == -7  # TN_ETIMEOUT
    assert 2.5 < res[0][2] < 15
