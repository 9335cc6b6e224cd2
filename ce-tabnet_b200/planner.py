"""Stage planner: contiguous layer ranges onto GPUs.

Restates the reference's planning math -- web/model-config.js:41-84
(tabsNeeded, defaultStagePlan, equalStages) and models/plan.js:55-89, 364-432
(tabWeightBudget, perLayerBytes, kvBytesPerLayer, distributeLayers,
largestRemainder) -- and applies it to GPUs of one box, whose budgets are
their free HBM times a weight fraction.
"""
from __future__ import annotations

import math

GiB = 1024 ** 3
MiB = 1024 ** 2
PER_TAB_WEIGHT_BYTES = 1.0 * GiB          # web/model-config.js:7


def tabs_needed(approx_weight_bytes: int, per_tab_bytes: float = PER_TAB_WEIGHT_BYTES) -> int:
    """web/model-config.js:41-45."""
    return max(1, math.ceil(approx_weight_bytes / per_tab_bytes))


def equal_stages(n_layers: int, n_stages: int) -> list[dict]:
    """web/model-config.js:77-84."""
    plan, per = [], math.ceil(n_layers / n_stages)
    stage, lo = 0, 0
    while lo < n_layers:
        plan.append({"stage": stage, "layers": [lo, min(n_layers, lo + per)]})
        stage += 1
        lo += per
    return plan


def default_stage_plan(n_layers: int, approx_weight_bytes: int, budgets: list[float] | None) -> list[dict]:
    """Greedy memory-weighted contiguous plan (web/model-config.js:50-75)."""
    per_layer = approx_weight_bytes / n_layers
    if not budgets:
        return equal_stages(n_layers, tabs_needed(approx_weight_bytes))
    srt = sorted(budgets, reverse=True)
    plan, lo, stage, ti = [], 0, 0, 0
    while lo < n_layers:
        budget = srt[min(ti, len(srt) - 1)]
        can_hold = max(1, math.floor(budget / per_layer))
        hi = min(n_layers, lo + can_hold)
        plan.append({"stage": stage, "layers": [lo, hi]})
        lo, stage, ti = hi, stage + 1, ti + 1
    return plan


def kv_bytes_per_layer(n_kv_heads: int, head_dim: int, ctx: int, bytes_per_elem: int = 2) -> int:
    """models/plan.js:85-89 (fp16 there; the engine's KV is f32, bytes_per_elem=4)."""
    return 2 * ctx * n_kv_heads * head_dim * bytes_per_elem


def largest_remainder(floats: list[float], total: int) -> list[int]:
    """models/plan.js:419-429."""
    out = [math.floor(f) for f in floats]
    rem = total - sum(out)
    order = sorted(range(len(floats)), key=lambda i: floats[i] - math.floor(floats[i]), reverse=True)
    for i in order:
        if rem <= 0:
            break
        out[i] += 1
        rem -= 1
    return out


def distribute_layers(n_layers: int, budgets: list[float], layer_bytes: int, kv_per_layer: int,
                      embed_bytes: int = 0, lm_head_bytes: int = 0) -> list[list[int]]:
    """Budget-proportional contiguous ranges with capacity clamps
    (models/plan.js:364-408); holders are taken in the given order."""
    H = len(budgets)
    if H == 0:
        return []
    per_layer_cost = layer_bytes + kv_per_layer
    cap = []
    for i, b in enumerate(budgets):
        reserve = (embed_bytes if i == 0 else 0) + (lm_head_bytes if i == H - 1 else 0)
        cap.append(max(0, math.floor((b - reserve) / per_layer_cost)))
    total = sum(budgets) or 1
    want = largest_remainder([b / total * n_layers for b in budgets], n_layers)
    want = [min(w, c) for w, c in zip(want, cap)]
    deficit, guard = n_layers - sum(want), 0
    while deficit > 0 and guard < n_layers * 2:
        guard += 1
        moved = False
        for i in range(H):
            if deficit > 0 and want[i] < cap[i]:
                want[i] += 1
                deficit -= 1
                moved = True
        if not moved:
            break
    ranges, lo = [], 0
    for cnt in want:
        if cnt <= 0 or lo >= n_layers:
            continue
        hi = min(n_layers, lo + cnt)
        ranges.append([lo, hi])
        lo = hi
    return ranges


def plan_gpus(n_layers: int, n_gpus: int, layer_bytes: int, kv_per_layer: int, embed_bytes: int,
              lm_head_bytes: int, free_bytes: list[float] | None = None,
              weight_fraction: float = 0.9) -> list[dict]:
    """Contiguous stages over n_gpus GPUs of one box: embed on the first,
    lm_head on the last.  Equal GPUs give equal stages (80 layers on 8 GPUs:
    8 x 10).  Raises if the model does not fit."""
    if free_bytes is None:
        free_bytes = [180e9] * n_gpus
    budgets = [f * weight_fraction for f in free_bytes[:n_gpus]]
    ranges = distribute_layers(n_layers, budgets, layer_bytes, kv_per_layer, embed_bytes, lm_head_bytes)
    if not ranges or ranges[-1][1] != n_layers or len(ranges) != n_gpus:
        raise ValueError(f"{n_layers} layers do not fit {n_gpus} GPUs with budgets {budgets}")
    return [{"stage": i, "layers": r, "is_first": i == 0, "is_last": i == len(ranges) - 1, "device_rank": i}
            for i, r in enumerate(ranges)]


def pipeline_tick(rank: int, world: int, n_mb: int, n_steps: int, tick: int) -> tuple[list[tuple], int | None]:
    """The decode pipeline's schedule at one tick, for one stage (rank).

    Stages run one micro-batch step per tick: rank r runs step j = tick - r
    (micro-batch j % n_mb).  At the start of the tick it receives the input of
    step j from rank r - 1 and sends the output of step j - 1 to rank r + 1, so
    every send meets its receive in the same tick on the peer.  The last rank's
    sampled token of step j goes back to rank 0, arriving at tick j + world, and
    feeds step j + n_mb (n_mb >= world keeps that arrival in time).

    Returns (ops, mb): ops are ("recv_hidden" | "recv_token" | "send_hidden" |
    "send_token", micro-batch, peer) to post together before the step, and mb is
    the micro-batch this rank steps at this tick, or None.
    """
    assert n_mb >= world, "need at least as many micro-batches as stages"
    j = tick - rank
    ops: list[tuple] = []
    if rank == 0:
        jt = tick - world  # the token of step jt arrives now, for step jt + n_mb
        if world > 1 and 0 <= jt < n_steps and jt + n_mb < n_steps:
            ops.append(("recv_token", jt % n_mb, world - 1))
    elif 0 <= j < n_steps:
        ops.append(("recv_hidden", j % n_mb, rank - 1))
    if world > 1 and 1 <= j <= n_steps:  # output of step j - 1
        if rank < world - 1:
            ops.append(("send_hidden", (j - 1) % n_mb, rank + 1))
        elif j - 1 + n_mb < n_steps:
            ops.append(("send_token", (j - 1) % n_mb, 0))
    return ops, (j % n_mb if 0 <= j < n_steps else None)


def pipeline_ticks(world: int, n_steps: int) -> int:
    """Ticks for n_steps micro-batch steps per stage, fill and drain included."""
    return n_steps + world
