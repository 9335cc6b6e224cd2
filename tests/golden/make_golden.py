"""Writes the known-answer fixtures of tests/golden/.

The reference ships no golden vectors for its engine, so these are derived by
hand from web/inference-worker.js -- each expected value carries the reasoning
that produced it -- and pin the oracle (tests/test_cpu_oracle.py).  The only
fixture computed by a program is tiny_greedy.json, produced by the oracle
itself once the KATs hold, so GPU runs can compare without re-running it.

    python tests/golden/make_golden.py            # KAT fixtures only
    python tests/golden/make_golden.py --greedy   # also tiny_greedy.json (runs the oracle)
"""
from __future__ import annotations

import json
import struct
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def f32bits(x: float) -> str:
    return "0x%08x" % struct.unpack("<I", struct.pack("<f", x))[0]


# f32ToF16 (web/inference-worker.js:74-88): e = clamp(floor(log2 v), -25, 16);
# normal branch m = Math.round((v/2^e - 1)*1024) (ties up), carry m==1024 -> e+1,
# e > 15 -> inf; subnormal branch (e < -14) m = Math.round(v/2^-24) & 0x3ff.
F32_TO_F16 = [
    # (f32 bit pattern, expected fp16 bits, derivation)
    ("0x3f800000", "0x3c00", "1.0: e=0, m=0"),
    ("0xc0000000", "0xc000", "-2.0: sign, e=1, m=0"),
    ("0x477fe000", "0x7bff", "65504: e=15, m=round(0.99902*1024)=1023"),
    ("0x477fefff", "0x7bff", "65519.996: m=round(1023.4999)=1023"),
    ("0x477ff000", "0x7c00", "65520: m=round(1023.5)=1024 -> e=16 > 15 -> inf"),
    ("0x47800000", "0x7c00", "65536: e=16 > 15 -> inf"),
    ("0x7f7fffff", "0x7c00", "f32 max: e clamped to 16 -> inf"),
    ("0x3f801000", "0x3c01", "1+2^-11: m=round(0.5)=1 (ties up; RNE gives 0x3c00)"),
    ("0x3f803000", "0x3c02", "1+3*2^-11: m=round(1.5)=2"),
    ("0x47001000", "0x7801", "32768+16: m=round(0.5)=1 (RNE gives 0x7800)"),
    ("0x3dcccccd", "0x2e66", "0.1: e=-4, m=round(614.40002)=614"),
    ("0x38800000", "0x0400", "2^-14: e=-14 (normal branch), m=0"),
    ("0x38c00000", "0x0600", "1.5*2^-14: m=512"),
    ("0x33800000", "0x0001", "2^-24: subnormal, m=round(1)=1"),
    ("0x33000000", "0x0001", "2^-25: m=round(0.5)=1 (RNE gives 0)"),
    ("0x33400000", "0x0001", "1.5*2^-25: m=round(0.75)=1"),
    ("0x32800000", "0x0000", "2^-26: e clamped to -25, m=round(0.25)=0"),
    ("0x34200000", "0x0003", "2.5*2^-24: m=round(2.5)=3 (RNE gives 2)"),
    ("0x387fe000", "0x0000", "2^-14-2^-25: m=round(1023.5)=1024, &0x3ff -> 0 (RNE gives 0x0400)"),
    ("0x387fc000", "0x03ff", "2^-14-2^-24: m=1023"),
    ("0x80000000", "0x8000", "-0: Object.is(val,-0) keeps the sign"),
    ("0x00000000", "0x0000", "+0"),
    ("0x00000001", "0x0000", "smallest f32 subnormal: m=round(tiny)=0"),
    ("0x80000001", "0x8000", "negative f32 subnormal: sign kept, m=0"),
    ("0x7f800000", "0x7c00", "+inf"),
    ("0xff800000", "0xfc00", "-inf"),
    ("0x7fc00000", "0x7e00", "NaN -> 0x7e00"),
    ("0xffc00001", "0x7e00", "negative NaN -> 0x7e00, no sign"),
    ("0xbf801000", "0xbc01", "-(1+2^-11): magnitude rounds up"),
]

# f16ToF32 (web/inference-worker.js:68-73)
F16_TO_F32 = [
    ("0x3c00", "0x3f800000", "1.0"),
    ("0x0001", "0x33800000", "2^-14 * 1/1024 = 2^-24"),
    ("0x03ff", "0x387fc000", "2^-14 * 1023/1024"),
    ("0x7bff", "0x477fe000", "2^15 * (1+1023/1024) = 65504"),
    ("0xfc00", "0xff800000", "-inf"),
    ("0x8000", "0x80000000", "-0 -> (-1)*2^-14*0 = -0"),
]

# q4_0 / q8_0 blocks (web/inference-worker.js:109-124): a q4_0 block is an fp16
# scale then 16 bytes; byte j holds element 2j in its LOW nibble and 2j+1 in
# its HIGH nibble; w = (nib - 8) * scale.  q8_0: fp16 scale, 32 int8, w = q*scale.
def q4_block(scale_bits: int, nib_pairs: list[tuple[int, int]]) -> list[int]:
    out = [scale_bits & 0xFF, scale_bits >> 8]
    for lo, hi in nib_pairs:
        out.append(lo | (hi << 4))
    return out


Q4_NIBS = [(j % 16, 15 - (j % 16)) for j in range(16)]  # byte j = (lo=j, hi=15-j)
Q4_KAT = {
    "quant": "q4_0",
    "bytes": q4_block(0x4000, Q4_NIBS),  # scale 2.0
    "count": 32,
    # element 2j = (j - 8) * 2, element 2j+1 = (15 - j - 8) * 2
    "expected": [v for j in range(16) for v in ((j - 8) * 2.0, (7 - j) * 2.0)],
    "derivation": "scale 0x4000 = 2.0; byte j = j | (15-j)<<4 -> elements 2j=(j-8)*2, 2j+1=(7-j)*2",
}
Q8_KAT = {
    "quant": "q8_0",
    "bytes": [0x00, 0x38] + [(q if q >= 0 else 256 + q) for q in range(-16, 16)],  # scale 0.5
    "count": 32,
    "expected": [q * 0.5 for q in range(-16, 16)],
    "derivation": "scale 0x3800 = 0.5; int8 q = -16..15 -> q*0.5",
}
# A [2 x 48] q8_0 tensor: 96 elements = 3 blocks laid over the FLAT tensor, so
# row 1 (elements 48..95) starts at element 16 of block 1.
_blocks = []
for b, scale in enumerate((0x3c00, 0x4000, 0x4200)):  # 1.0, 2.0, 3.0
    _blocks += [scale & 0xFF, scale >> 8] + [((b * 32 + i) % 100) for i in range(32)]
STRADDLE_KAT = {
    "quant": "q8_0", "rows": 2, "cols": 48, "bytes": _blocks,
    "expected_row1": [((32 + i) % 100) * 2.0 for i in range(16, 32)] + [((64 + i) % 100) * 3.0 for i in range(32)],
    "derivation": "row 1 = block 1 elements 16..31 (scale 2) then block 2 elements 0..31 (scale 3)",
}

# quantBytesFor (:130-137) and the packed layer sizes of layerLayout (:142-159)
SIZES = {
    "quant_bytes": [[32, "q4_0", 18], [33, "q4_0", 36], [32, "q8_0", 34], [688, "q8_0", 22 * 34],
                    [10, "f16", 20], [10, "f32", 40]],
    "round_ffn": [[256, 768], [4096, 11008], [8192, 22016]],
    # attn_norm(f16) wq wk wv wo ffn_norm(f16) w_gate w_up w_down
    "layer_bytes": {"tiny": 736512, "llama8b": 122699776, "llama70b": 481329152},
}

# sample (:658-672).  logits [2, 1, 0, 1], temperature 1: e = [1, e^-1, e^-2,
# e^-1], sum 1.8711, probs ~ [0.5344, 0.1966, 0.0723, 0.1966]; sorted by prob
# desc (stable): [0, 1, 3, 2]; running sums 0.5344, 0.7311, 0.9277, 1.0.
SAMPLE_KAT = [
    {"logits": [2.0, 1.0, 0.0, 1.0], "temperature": 0.0, "top_p": 0.95, "u": 0.5, "expected": 0,
     "derivation": "greedy: first strictly greater"},
    {"logits": [1.0, 3.0, 3.0, 2.0], "temperature": -1.0, "top_p": 0.95, "u": 0.5, "expected": 1,
     "derivation": "greedy tie: lowest index"},
    {"logits": [2.0, 1.0, 0.0, 1.0], "temperature": 1.0, "top_p": 0.5, "u": 0.99, "expected": 0,
     "derivation": "cum 0.5344 >= 0.5 after idx 0 -> cut 1 -> always idx 0"},
    {"logits": [2.0, 1.0, 0.0, 1.0], "temperature": 1.0, "top_p": 0.9, "u": 0.7, "expected": 1,
     "derivation": "cut 3 (0,1,3), cum 0.9277; r=0.6494: 0.5344 < r <= 0.7311 -> idx 1"},
    {"logits": [2.0, 1.0, 0.0, 1.0], "temperature": 1.0, "top_p": 0.9, "u": 0.9, "expected": 3,
     "derivation": "r=0.8349 > 0.7311 -> idx 3 (tie with idx 1 keeps index order)"},
    {"logits": [2.0, 1.0, 0.0, 1.0], "temperature": 1.0, "top_p": 0.9, "u": 0.0, "expected": 0,
     "derivation": "r=0 <= first acc -> idx 0"},
]


def write_kats():
    (HERE / "kat_f16.json").write_text(json.dumps({"f32_to_f16": F32_TO_F16, "f16_to_f32": F16_TO_F32}, indent=1))
    (HERE / "kat_quant.json").write_text(json.dumps(
        {"q4_0": Q4_KAT, "q8_0": Q8_KAT, "straddle": STRADDLE_KAT, "sizes": SIZES}, indent=1))
    (HERE / "kat_sample.json").write_text(json.dumps(SAMPLE_KAT, indent=1))


def write_greedy():
    """Oracle greedy tokens of the tiny model: 32-token prompt, 64 decode steps."""
    root = HERE.parent.parent
    sys.path.insert(0, str(root))
    import __graft_entry__ as g
    from oracle import ref

    pkg = g.load_package()
    m = pkg.pack.MODELS["tiny"]
    w = pkg.pack.synth_weights(m, 0, m.n_layers, True, True)
    st = ref.RefStage(m.dims(), 0, m.n_layers, True, True, w)
    prompt = pkg.pack.synth_prompt(m, 32)
    r = st.forward(1, 0, token_ids=prompt)
    toks, gaps = [r["token_id"]], []
    for s in range(64):
        lg = sorted(r["logits"].tolist(), reverse=True)
        gaps.append(lg[0] - lg[1])
        r = st.forward(1, 32 + s, token_ids=[toks[-1]])
        toks.append(r["token_id"])
    (HERE / "tiny_greedy.json").write_text(json.dumps(
        {"model": "tiny", "seed": m.seed, "prompt": prompt, "tokens": toks,
         "top2_gaps": [round(x, 6) for x in gaps]}, indent=1))


if __name__ == "__main__":
    write_kats()
    if "--greedy" in sys.argv:
        write_greedy()
