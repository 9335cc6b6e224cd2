"""B200 stage engine for ce-tabnet: a drop-in for web/inference-worker.js.

The directory name is not a Python identifier, so the package is imported
under the name `ce_tabnet_b200` by `load_package()` (see __graft_entry__.py).
"""
from . import _lib, frame, manifest, pack, pipeline, planner
from .engine import (StageCtx, forward, forward_batch, forwardLast, forwardSafe, freeStage, free_seq,
                     initStage, kv_len, sample)

__all__ = ["StageCtx", "initStage", "forward", "forward_batch", "forwardSafe", "forwardLast", "freeStage",
           "free_seq", "kv_len", "sample", "frame", "manifest", "pack", "pipeline", "planner", "_lib"]
