"""Model packs: a directory of content-addressed objects plus manifest.json
(models/README.md), written as tools/shard-model.js writes them and read into
the `weights` object of initStage as web/shard-loader.js assembles it.

Object files are `<base>.<cid>.bin` with cid = lower-case hex SHA-256 of the
bytes (tools/shard-model.js:181-187).  A layer is one object or a list of
`parts` ({role, cid, file, bytes}, attention then MLP).  On load every object
whose cid is a SHA-256 (64 hex digits, optionally `sha256:` / `sha-256-`) is
verified; other cid schemes are trusted, as in the reference
(web/shard-loader.js:271-283).  Objects resolve to `file` in the pack
directory, else `<cid>.bin`, optionally a `byte_range` [first, last] of it
(:204-221); fetching over the network is the reference's job, not this
module's.

Deliberate differences from the reference loader: the parts of a split layer
are joined into the layer buffer (the reference's initStage reads only `buf`,
web/inference-worker.js:434, so split layers do not load there); the weights
object carries the pack's quant types (`quant`, and `embedQuant` /
`lmHeadQuant` from the embed / lm_head objects' `quant` when present) and
`ffn_dim` when the manifest has it -- the reference loader passes neither, so
its initStage falls back to q4_0 and to roundFfn(hidden_dim).
"""
from __future__ import annotations

import concurrent.futures as cf
import hashlib
import hmac
import json
import os
import re
from pathlib import Path

import numpy as np

from .frame import js_stringify

__all__ = ["normalize_cid", "verify_cid", "write_pack", "read_manifest", "load_stage", "PackError"]

_CID = re.compile(r"^(?:sha-?256[:\-])?([0-9a-f]{64})$")


class PackError(ValueError):
    pass


def normalize_cid(cid) -> str | None:
    """normalizeCidToHex (web/shard-loader.js:278-282): the SHA-256 hex of a
    hash cid, or None for another cid scheme."""
    m = _CID.match(str(cid).lower())
    return m.group(1) if m else None


def verify_cid(buf, cid) -> bool:
    """verifyCid (web/shard-loader.js:271-276)."""
    want = normalize_cid(cid)
    if want is None:
        return True
    return hmac.compare_digest(hashlib.sha256(memoryview(buf)).hexdigest(), want)


def _as_bytes(b) -> memoryview:
    if isinstance(b, np.ndarray):
        return memoryview(np.ascontiguousarray(b).view(np.uint8).reshape(-1))
    return memoryview(b).cast("B")


def _emit(out: Path, base: str, data) -> dict:
    mv = _as_bytes(data)
    cid = hashlib.sha256(mv).hexdigest()
    name = f"{base}.{cid}.bin"
    with open(out / name, "wb") as f:
        f.write(mv)
    return {"cid": cid, "file": name, "bytes": mv.nbytes}


def write_pack(out_dir, model_id: str, dims: dict, layers: list, *, embed=None, norm=None, lm_head=None,
               quant: str = "q4_0", arch: str = "llama", approx_weight_bytes: int | None = None,
               embed_quant: str | None = None, lm_head_quant: str | None = None,
               ffn_dim: int | None = None) -> dict:
    """Write a pack the way buildManifest does (tools/shard-model.js:189-236):
    objects `<base>.<cid>.bin`, then manifest.json as JSON.stringify(manifest,
    null, 2).  `layers[i]` is the layer's bytes, or a list of (role, bytes)
    parts.  embed_quant / lm_head_quant / ffn_dim add fields the reference
    packer does not write (read back by load_stage)."""
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    manifest = {"model_id": model_id, "arch": arch, "n_layers": len(layers), "hidden_dim": int(dims["hidden_dim"]),
                "n_heads": int(dims["n_heads"]), "n_kv_heads": int(dims["n_kv_heads"]), "vocab": int(dims["vocab"]),
                "rope_theta": float(dims["rope_theta"]), "quant": quant, "layers": []}

    def emit_one(base, o):
        if isinstance(o, (list, tuple)) and o and isinstance(o[0], (list, tuple)):
            parts = []
            for role, data in o:
                r = _emit(out, f"{base}.{role}", data)
                parts.append({"role": role, "cid": r["cid"], "file": r["file"], "bytes": r["bytes"]})
            return {"parts": parts}
        return _emit(out, base, o)

    for key, obj, q in (("embed", embed, embed_quant), ("norm", norm, None), ("lm_head", lm_head, lm_head_quant)):
        if obj is not None:
            manifest[key] = emit_one(key, obj)
            if q is not None:
                manifest[key]["quant"] = q
    total = 0
    for i, layer in enumerate(layers):
        emitted = emit_one(f"layer_{i:03d}", layer)
        entry = {"idx": i, "quant": quant, **emitted}
        entry["bytes"] = sum(p["bytes"] for p in emitted["parts"]) if "parts" in emitted else emitted["bytes"]
        manifest["layers"].append(entry)
        total += entry["bytes"]
    extra = sum(manifest[k]["bytes"] for k in ("embed", "lm_head", "norm") if k in manifest and "bytes" in manifest[k])
    manifest["approx_weight_bytes"] = int(approx_weight_bytes) if approx_weight_bytes else total + extra
    if ffn_dim is not None:
        manifest["ffn_dim"] = int(ffn_dim)
    (out / "manifest.json").write_text(js_stringify(manifest, 2), encoding="utf-8")
    return manifest


def read_manifest(pack_dir, name: str = "manifest.json") -> dict:
    return json.loads((Path(pack_dir) / name).read_text(encoding="utf-8"))


def _object_path(base: Path, obj: dict, cid: str) -> Path:
    url = obj.get("url")
    if url is not None:
        if "://" in str(url) and not str(url).startswith("file://"):
            raise PackError(f"object {cid}: fetching {url} is not done here (put the file in the pack directory)")
        return Path(str(url)[len("file://"):] if str(url).startswith("file://") else base / str(url))
    return base / str(obj.get("file") or f"{cid}.bin")


def _read_one(base: Path, obj: dict, verify: bool) -> np.ndarray:
    """fetchOne (web/shard-loader.js:174-201) for a local pack."""
    cid = obj.get("cid", obj.get("id"))
    if not cid:
        raise PackError("object has no cid (content addressing is required)")
    path = _object_path(base, obj, cid)
    br = obj.get("byte_range")
    if isinstance(br, (list, tuple)):
        first, last = int(br[0]), int(br[1])
        with open(path, "rb") as f:
            f.seek(first)
            buf = np.frombuffer(f.read(last - first + 1), dtype=np.uint8)
    else:
        buf = np.fromfile(path, dtype=np.uint8)
    if verify and not verify_cid(buf, cid):
        raise PackError(f"integrity check failed for {cid} (got {hashlib.sha256(buf).hexdigest()})")
    return buf


def _read_object(base: Path, obj: dict, verify: bool) -> np.ndarray:
    """fetchObjectFull (:163-172); parts are joined in manifest order."""
    parts = obj.get("parts")
    if isinstance(parts, list) and parts:
        return np.concatenate([_read_one(base, p, verify) for p in parts])
    return _read_one(base, obj, verify)


def load_stage(pack, lo: int, hi: int, *, need_embed: bool = False, need_lm_head: bool = False,
               verify: bool = True, threads: int | None = None) -> dict:
    """load (web/shard-loader.js:56-140) from a local pack directory (or a
    (manifest, directory) pair): the weights object of a stage holding layers
    [lo, hi), with the embedding for a first stage and norm + lm_head for a
    last one.  Objects are read (and hashed) on a thread pool."""
    if isinstance(pack, tuple):
        manifest, base = pack[0], Path(pack[1])
    else:
        base = Path(pack)
        manifest = read_manifest(base)
    layers = manifest.get("layers")
    if not isinstance(layers, list):
        raise PackError("manifest missing layers[]")
    if not hi > lo:
        raise PackError(f"empty layer range [{lo},{hi})")
    if lo < 0 or hi > len(layers):
        raise PackError(f"stage range [{lo},{hi}) out of bounds for {len(layers)}-layer model")
    plan = []
    for i in range(lo, hi):
        if not layers[i]:
            raise PackError(f"manifest missing layer {i}")
        plan.append(("layer", i, layers[i]))
    if need_embed:
        if not manifest.get("embed"):
            raise PackError("needEmbed but manifest has no embed object")
        plan.append(("embed", None, manifest["embed"]))
    if need_lm_head:
        if not manifest.get("lm_head") or not manifest.get("norm"):
            raise PackError("needLmHead but manifest lacks lm_head/norm")
        plan.append(("lm_head", None, manifest["lm_head"]))
        plan.append(("norm", None, manifest["norm"]))
    with cf.ThreadPoolExecutor(max_workers=threads or min(8, os.cpu_count() or 1)) as ex:
        data = list(ex.map(lambda p: _read_object(base, p[2], verify), plan))
    quant = manifest.get("quant", "q4_0")
    dims = {k: manifest[k] for k in ("hidden_dim", "n_heads", "n_kv_heads", "vocab", "rope_theta") if k in manifest}
    if manifest.get("ffn_dim"):
        dims["ffn_dim"] = manifest["ffn_dim"]
    out = {"arch": manifest.get("arch"), "dims": dims, "quant": quant, "layers": []}
    for (kind, idx, obj), buf in zip(plan, data):
        if kind == "layer":
            out["layers"].append({"idx": idx, "buf": buf, "quant": obj.get("quant", quant)})
        else:
            out[kind] = buf
            if kind == "embed":
                out["embedQuant"] = obj.get("quant", quant)
            elif kind == "lm_head":
                out["lmHeadQuant"] = obj.get("quant", quant)
    return out
