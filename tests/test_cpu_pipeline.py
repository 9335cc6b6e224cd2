"""The multi-GPU decode pipeline's host logic on CPU: gloo ranks run the tick
schedule of planner.pipeline_tick (the one bench.py drives over NCCL) with a
toy stage per rank, and rank 0 checks every token that comes back against a
sequential run of the same stages.  This exercises the P2P pairing (no tick
may leave a send without its receive), the fill / drain, and the feedback of
the last stage's token to rank 0 for the micro-batch's next step."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

H = 4  # toy hidden width


def _stage_first(tok: int, pos: int) -> list[int]:
    return [tok * 7 + pos + i for i in range(H)]


def _stage_mid(h: list[int], rank: int, pos: int) -> list[int]:
    return [2 * v + rank + pos for v in h]


def _stage_last(h: list[int], pos: int) -> int:
    return (sum(h) * 31 + pos) % 1009


def _sequential(world: int, n_mb: int, n_steps: int, first_tokens: list[int]) -> list[int]:
    out = []
    for j in range(n_steps):
        mb, pos = j % n_mb, j // n_mb
        tok = first_tokens[mb] if j < n_mb else out[j - n_mb]
        h = _stage_first(tok, pos)
        for r in range(1, world - 1):
            h = _stage_mid(h, r, pos)
        out.append(_stage_last(h, pos))
    return out


def _rank_main(rank, world, port, n_mb, n_steps, first_tokens, result):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    import __graft_entry__ as ge

    planner = ge.load_package().planner
    torch.set_num_threads(1)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    tok = torch.tensor([[t] for t in first_tokens], dtype=torch.int64)
    tok_out = torch.zeros((n_mb, 1), dtype=torch.int64)
    hin = torch.zeros((n_mb, H), dtype=torch.int64)
    hout = torch.zeros((n_mb, H), dtype=torch.int64)
    bufs = {"recv_token": tok, "recv_hidden": hin, "send_hidden": hout, "send_token": tok_out}
    pos = [0] * n_mb
    got = {}
    for tick in range(planner.pipeline_ticks(world, n_steps)):
        sched, mb = planner.pipeline_tick(rank, world, n_mb, n_steps, tick)
        ops = [dist.P2POp(dist.irecv if k.startswith("recv") else dist.isend, bufs[k][b], peer)
               for k, b, peer in sched]
        if ops:
            for w in dist.batch_isend_irecv(ops):
                w.wait()
        for k, b, _ in sched:
            if rank == 0 and k == "recv_token":
                got[tick - world] = int(tok[b, 0])  # the token of step tick - world
        if mb is None:
            continue
        p = pos[mb]
        if rank == 0:
            h = _stage_first(int(tok[mb, 0]), p)
        else:
            h = [int(v) for v in hin[mb]]
            if rank < world - 1:
                h = _stage_mid(h, rank, p)
        if rank < world - 1:
            hout[mb] = torch.tensor(h, dtype=torch.int64)
        else:
            tok_out[mb, 0] = _stage_last(h, p)
        pos[mb] += 1
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        result.update(got)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,n_mb", [(2, 2), (2, 4), (3, 3), (3, 5)])
def test_pipeline_schedule_gloo(world, n_mb):
    n_steps = 4 * n_mb
    first_tokens = [11 * (i + 1) for i in range(n_mb)]
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        result = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank_main, args=(r, world, port, n_mb, n_steps, first_tokens, result))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        codes = [p.exitcode for p in procs]
        for p in procs:
            if p.is_alive():
                p.kill()
        assert codes == [0] * world, codes
        want = _sequential(world, n_mb, n_steps, first_tokens)
        got = dict(result)
    # rank 0 receives the token of every step whose micro-batch steps again
    assert sorted(got) == list(range(n_steps - n_mb))
    assert [got[j] for j in range(n_steps - n_mb)] == want[: n_steps - n_mb]


def test_pipeline_tick_pairs_every_send():
    """Pure schedule check: at every tick each send has the matching receive."""
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    import __graft_entry__ as ge

    planner = ge.load_package().planner
    for world in (2, 3, 4, 8):
        for n_mb in (world, world + 3):
            n = 5 * n_mb
            steps = [0] * world
            for tick in range(planner.pipeline_ticks(world, n)):
                sends, recvs = set(), set()
                for r in range(world):
                    ops, mb = planner.pipeline_tick(r, world, n_mb, n, tick)
                    for k, b, peer in ops:
                        if k.startswith("send"):
                            sends.add((r, peer, k.split("_")[1], b))
                        else:
                            recvs.add((peer, r, k.split("_")[1], b))
                    steps[r] += mb is not None
                assert sends == recvs, (world, n_mb, tick)
            assert steps == [n] * world
