"""Generate tests/golden/llama8b_greedy.json: the oracle on the whole
Llama-3-8B-shaped q4_0 model (32 layers, one stage: first and last), seeded
synthetic weights (seed 1), a 32-token uniform prompt, then 64 decode steps.

Two runs, each a separate sequence of the same oracle stage:
  greedy: every step feeds back the argmax (the 64-step greedy bar);
  forced: every step feeds a predetermined uniform token instead (teacher
          forcing), so each step's argmax depends on a different input and the
          comparison cannot sit at a fixed point of the greedy map.
Per step the fixture keeps the argmax token, the top-2 logit gap, the 16
largest logits (index, value) and every 32nd element of the f32 hidden state
that enters the final norm (base64 of little-endian float32).

The oracle is the C restatement of the reference CPU path
(web/inference-worker.js:471-583, 658-716); this script is test
infrastructure, run once on a CPU host:

    python tests/golden/make_llama8b_greedy.py   (about 15 minutes on 8 cores)
"""
from __future__ import annotations

import base64
import json
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

PROMPT, STEPS, HIDDEN_STRIDE, TOPK = 32, 64, 32, 16


def _b64(a: np.ndarray) -> str:
    return base64.b64encode(np.ascontiguousarray(a, dtype="<f4").tobytes()).decode()


def _record(res: dict) -> dict:
    lg = res["logits"]
    top = np.argsort(-lg, kind="stable")[:TOPK]
    return {"token": int(res["token_id"]), "gap": float(lg[top[0]] - lg[top[1]]),
            "top_idx": [int(i) for i in top], "top_val": [float(lg[i]) for i in top],
            "hidden_sub": _b64(res["hidden_f32"][::HIDDEN_STRIDE])}


def main() -> None:
    import __graft_entry__ as g
    from oracle import ref

    pkg = g.load_package()
    m = pkg.pack.MODELS["llama8b"]
    t0 = time.time()
    w = pkg.pack.synth_weights(m, 0, m.n_layers, True, True)
    oracle = ref.RefStage(m.dims(), 0, m.n_layers, True, True, w)
    prompt = pkg.pack.synth_prompt(m, PROMPT)
    forced_inputs = pkg.pack.synth_prompt(m, STEPS, seed=4242)
    out = {"model": "llama8b", "seed": m.seed, "quant": m.quant, "prompt": prompt, "hidden_stride": HIDDEN_STRIDE,
           "topk": TOPK, "forced_inputs": forced_inputs}
    for run, seq in (("greedy", 1), ("forced", 2)):
        res = oracle.forward(seq, 0, token_ids=prompt, temperature=0.0)
        steps = [_record(res)]
        tok = res["token_id"]
        for s in range(STEPS):
            inp = tok if run == "greedy" else forced_inputs[s]
            res = oracle.forward(seq, PROMPT + s, token_ids=[inp], temperature=0.0)
            steps.append(_record(res))
            tok = res["token_id"]
            print(f"{run} step {s}: token {tok} gap {steps[-1]['gap']:.4f} ({time.time() - t0:.0f} s)",
                  flush=True)
        out[run] = steps
        out[run + "_distinct"] = len({st["token"] for st in steps})
    oracle.free()
    dst = Path(__file__).with_name("llama8b_greedy.json")
    dst.write_text(json.dumps(out, indent=0) + "\n")
    print(f"wrote {dst}: greedy {out['greedy_distinct']} distinct tokens, forced {out['forced_distinct']}")


if __name__ == "__main__":
    main()
