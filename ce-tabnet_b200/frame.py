"""Activation wire frame of the reference (web/protocol.js:101-120) and a
stage's frame hop (web/tabnet-node.js:140-153, :186-193).

Frame = 4-byte little-endian header length, the UTF-8 JSON header (the
activation meta without `data`), then the raw payload bytes (fp16 bits of the
hidden state, little endian).  The header is serialised exactly as
JavaScript's JSON.stringify writes it (`js_stringify`), so frames built here
are byte-identical to the reference's for the same meta and payload, and a
B200 stage can sit in a pipeline of reference stages.

Payload note: encodeActivation sends `payload.buffer`, i.e. the whole
ArrayBuffer behind a typed array.  Here the payload is the bytes of the array
given; the two agree whenever the typed array owns its buffer, as the hidden
state `forward` returns does (web/tabnet-node.js:192).
"""
from __future__ import annotations

import json
import math
import re
import struct

import numpy as np

__all__ = ["UNDEFINED", "js_stringify", "encode_activation", "decode_activation", "activation_meta",
           "token_message", "forward_frame"]


class _Undefined:
    """JavaScript's `undefined`: dropped from objects, `null` in arrays."""

    def __repr__(self) -> str:
        return "UNDEFINED"


UNDEFINED = _Undefined()

_ARRAY_INDEX = re.compile(r"^(0|[1-9][0-9]*)$")
_ESC = {'"': '\\"', "\\": "\\\\", "\b": "\\b", "\f": "\\f", "\n": "\\n", "\r": "\\r", "\t": "\\t"}


def _js_number(x) -> str:
    """Number::toString (ECMA-262 6.1.6.1.20) for a finite double, as JSON.stringify uses it."""
    if isinstance(x, bool):
        raise TypeError("bool is not a number here")
    x = float(x)
    if not math.isfinite(x):
        return "null"
    if x == 0.0:
        return "0"  # also -0
    sign = "-" if x < 0 else ""
    # shortest round-trip digits s (no leading / trailing zeros) and n with x = 0.s * 10^n
    mant, _, exp = repr(abs(x)).partition("e")
    e10 = int(exp) if exp else 0
    ip, _, fp = mant.partition(".")
    digits = (ip + fp).lstrip("0")
    lead_zeros = len(ip + fp) - len((ip + fp).lstrip("0"))
    n = len(ip) - lead_zeros + e10
    digits = digits.rstrip("0") or "0"
    k = len(digits)
    if k <= n <= 21:
        return sign + digits + "0" * (n - k)
    if 0 < n <= 21:
        return sign + digits[:n] + "." + digits[n:]
    if -6 < n <= 0:
        return sign + "0." + "0" * (-n) + digits
    e = n - 1
    es = ("+" if e >= 0 else "-") + str(abs(e))
    return sign + digits[0] + ("." + digits[1:] if k > 1 else "") + "e" + es


def _js_string(s: str) -> str:
    out = ['"']
    for ch in s:
        o = ord(ch)
        if ch in _ESC:
            out.append(_ESC[ch])
        elif o < 0x20 or 0xD800 <= o <= 0xDFFF:  # controls and lone surrogates: \\u escapes (lower case)
            out.append("\\u%04x" % o)
        else:
            out.append(ch)
    out.append('"')
    return "".join(out)


def _js_value(v, in_array: bool, gap: str = "", indent: str = ""):
    if v is UNDEFINED or callable(v):
        return "null" if in_array else None
    if v is None:
        return "null"
    if v is True or (isinstance(v, np.bool_) and bool(v)):
        return "true"
    if v is False or isinstance(v, np.bool_):
        return "false"
    if isinstance(v, (int, float, np.integer, np.floating)):
        return _js_number(v)
    if isinstance(v, str):
        return _js_string(v)
    inner = indent + gap
    sep = ",\n" + inner if gap else ","
    if isinstance(v, dict):
        keys = [str(k) for k in v]
        if len(set(keys)) != len(keys):
            raise ValueError("duplicate keys after string conversion")
        vals = dict(zip(keys, v.values()))
        # own property order: array-index keys ascending, then the rest in insertion order
        idx = sorted((k for k in keys if _ARRAY_INDEX.match(k) and int(k) < 2**32 - 1), key=int)
        order = idx + [k for k in keys if k not in set(idx)]
        parts = []
        for k in order:
            s = _js_value(vals[k], False, gap, inner)
            if s is not None:
                parts.append(_js_string(k) + (": " if gap else ":") + s)
        if not parts:
            return "{}"
        return "{\n" + inner + sep.join(parts) + "\n" + indent + "}" if gap else "{" + sep.join(parts) + "}"
    if isinstance(v, (list, tuple)):
        items = [_js_value(x, True, gap, inner) for x in v]
        if not items:
            return "[]"
        return "[\n" + inner + sep.join(items) + "\n" + indent + "]" if gap else "[" + sep.join(items) + "]"
    if isinstance(v, np.ndarray):
        return _js_value(v.tolist(), in_array, gap, indent)
    raise TypeError(f"cannot serialise {type(v).__name__}")


def js_stringify(value, space: int = 0) -> str:
    """JSON.stringify(value, null, space) for JSON-shaped Python values (dict,
    list, str, int, float, bool, None, UNDEFINED); space is the indent width
    (0: none, at most 10 as in JavaScript)."""
    s = _js_value(value, False, " " * max(0, min(10, int(space))), "")
    if s is None:
        raise ValueError("JSON.stringify(undefined) is not a string")
    return s


def _payload_bytes(payload) -> bytes:
    if isinstance(payload, (bytes, bytearray, memoryview)):
        return bytes(payload)
    a = np.asarray(payload)
    if a.dtype.byteorder == ">":
        a = a.astype(a.dtype.newbyteorder("<"))
    return np.ascontiguousarray(a).tobytes()


def encode_activation(meta: dict, payload) -> bytes:
    """encodeActivation (web/protocol.js:104-113)."""
    header = js_stringify({**meta, "data": UNDEFINED}).encode("utf-8")
    return struct.pack("<I", len(header)) + header + _payload_bytes(payload)


def _reject_constant(name):
    raise ValueError(f"JSON.parse does not accept {name}")


def _parse_int(text: str):
    # JSON.parse yields doubles: integers past 2^53 keep only a double's precision
    v = int(text)
    return v if abs(v) <= 2**53 else float(v)


def decode_activation(frame) -> tuple[dict, bytes]:
    """decodeActivation (web/protocol.js:114-120): (meta, payload bytes).
    Raises ValueError where the reference throws (short frame, header past the
    end, header that is not JSON)."""
    buf = bytes(frame)
    if len(buf) < 4:
        raise ValueError("frame shorter than its length word")
    (hlen,) = struct.unpack_from("<I", buf, 0)
    if 4 + hlen > len(buf):
        raise ValueError(f"header of {hlen} bytes runs past a {len(buf)}-byte frame")
    text = buf[4:4 + hlen].decode("utf-8", errors="replace")  # TextDecoder: U+FFFD for bad bytes
    if text.startswith("\ufeff"):
        text = text[1:]  # TextDecoder drops a leading byte-order mark
    try:
        meta = json.loads(text, parse_constant=_reject_constant, parse_int=_parse_int)
    except json.JSONDecodeError as e:
        raise ValueError(f"header is not JSON: {e}") from None
    return meta, buf[4 + hlen:]


def activation_meta(run, node, seq_id, token_pos, from_stage, to_stage, n) -> dict:
    """The meta a stage sends with its hidden state (web/tabnet-node.js:189-190)."""
    return {"run": run, "node": node, "seq_id": seq_id, "token_pos": token_pos, "from_stage": from_stage,
            "to_stage": to_stage, "dtype": "f16", "shape": [n]}


def token_message(run, node, seq_id, token_pos, token_id, text="", done=False) -> dict:
    """token() (web/protocol.js:33-34): what the last stage sends the coordinator."""
    return {"t": "token", "run": run, "node": node, "seq_id": seq_id, "token_pos": token_pos,
            "token_id": token_id, "text": text, "done": done}


def forward_frame(ctx, frame, *, node, stage: int, run=None, temperature=None, top_p=None, rng_seed=None):
    """A stage's hop on an activation frame (_onActivation,
    web/tabnet-node.js:140-153): run this stage on the frame's fp16 payload at
    the frame's (seq_id, token_pos); a first or middle stage returns the frame
    for stage + 1 (meta of :189-190), the last stage returns the token message.

    The payload is read as the fp16 bits the sender encoded (f32ToF16 output);
    the reference reads it through a Float16Array, whose element values are
    not the bit patterns its forward expects."""
    from . import engine

    meta, payload = decode_activation(frame)
    if meta.get("dtype", "f16") != "f16":
        raise ValueError(f"activation dtype {meta.get('dtype')!r}: fp16 frames only")
    if len(payload) % 2:
        raise ValueError("fp16 payload of odd length")
    hidden = np.frombuffer(payload, dtype="<u2")
    req = {"seq_id": meta["seq_id"], "token_pos": meta["token_pos"], "hidden": hidden}
    for k, v in (("temperature", temperature), ("top_p", top_p), ("rng_seed", rng_seed)):
        if v is not None:
            req[k] = v
    out = engine.forward(ctx, req)
    run = meta.get("run") if run is None else run
    if ctx.is_last:
        return token_message(run, node, meta["seq_id"], meta["token_pos"], out["token_id"])
    h = out["hidden"]
    return encode_activation(activation_meta(run, node, meta["seq_id"], meta["token_pos"], stage, stage + 1,
                                             int(h.size)), h)
