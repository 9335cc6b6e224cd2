"""The activation wire frame (web/protocol.js:101-120): byte layout, the
JSON.stringify header, decode errors.  The first case is the reference's own
selftest frame (dev/serve.js:133-139) with its bytes written out from the
format: u32 LE header length, the header as JSON.stringify writes it (object
literal key order, no whitespace, `data` dropped), then the payload bytes."""
import json
import math
import struct

import numpy as np
import pytest


@pytest.fixture(scope="module")
def fr(pkg):
    return pkg.frame


def test_reference_selftest_frame_bytes(fr):
    meta = {"run": "demo", "node": "n0", "seq_id": "s1", "token_pos": 3, "from_stage": 0, "to_stage": 1,
            "dtype": "f16", "shape": [8]}
    payload = np.arange(1, 9, dtype=np.uint16)
    header = b'{"run":"demo","node":"n0","seq_id":"s1","token_pos":3,"from_stage":0,"to_stage":1,"dtype":"f16","shape":[8]}'
    want = struct.pack("<I", len(header)) + header + b"".join(struct.pack("<H", i) for i in range(1, 9))
    frame = fr.encode_activation(meta, payload)
    assert frame == want
    dec_meta, dec_payload = fr.decode_activation(frame)
    # the selftest's own assertions (dev/serve.js:138-139)
    assert dec_meta["seq_id"] == "s1" and dec_meta["to_stage"] == 1
    u16 = np.frombuffer(dec_payload, dtype="<u2")
    assert len(u16) == 8 and u16[7] == 8
    assert dec_meta == meta


def test_data_key_is_dropped(fr):
    meta = {"run": "r", "data": [1, 2, 3], "seq_id": "x"}
    frame = fr.encode_activation(meta, b"\x00\x3c")
    (hlen,) = struct.unpack_from("<I", frame)
    assert frame[4:4 + hlen] == b'{"run":"r","seq_id":"x"}'
    assert frame[4 + hlen:] == b"\x00\x3c"


@pytest.mark.parametrize("x,want", [
    (0.1, "0.1"), (1.5, "1.5"), (-2.5, "-2.5"), (100, "100"), (-0.0, "0"), (3, "3"),
    (123.456, "123.456"), (1e-6, "0.000001"), (1.2e-6, "0.0000012"), (1e-7, "1e-7"),
    (1.23e-18, "1.23e-18"), (-2.5e-10, "-2.5e-10"), (1e20, "100000000000000000000"),
    (1.2345678901234568e20, "123456789012345680000"), (1e21, "1e+21"),
    (1.7976931348623157e308, "1.7976931348623157e+308"), (5e-324, "5e-324"),
    (2**53 + 1, "9007199254740992"), (float("nan"), "null"), (float("inf"), "null"),
])
def test_number_formatting(fr, x, want):
    # Number::toString, ECMA-262 6.1.6.1.20 (what JSON.stringify writes)
    assert fr.js_stringify(x) == want


def test_key_order_undefined_and_escapes(fr):
    u = fr.UNDEFINED
    assert fr.js_stringify({"b": 1, "2": 2, "a": 3, "1": 4, "u": u, "l": [u, None, True, False]}) == \
        '{"1":4,"2":2,"b":1,"a":3,"l":[null,null,true,false]}'
    assert fr.js_stringify("\x01\n\"\\é \ud800") == '"\\u0001\\n\\"\\\\é \\ud800"'
    assert fr.js_stringify({"s": [1.5, {"k": "v"}], "e": []}) == '{"s":[1.5,{"k":"v"}],"e":[]}'
    with pytest.raises(ValueError):
        fr.js_stringify(u)


def test_decode_errors_and_text_decoding(fr):
    with pytest.raises(ValueError):
        fr.decode_activation(b"\x01\x00")
    with pytest.raises(ValueError):
        fr.decode_activation(struct.pack("<I", 10) + b"{}")
    with pytest.raises(ValueError):
        fr.decode_activation(struct.pack("<I", 3) + b"{x}")
    with pytest.raises(ValueError):  # JSON.parse rejects NaN
        fr.decode_activation(struct.pack("<I", 9) + b'{"a":NaN}')
    bom = b"\xef\xbb\xbf" + b'{"a":1}'
    assert fr.decode_activation(struct.pack("<I", len(bom)) + bom) == ({"a": 1}, b"")
    bad = b'{"a":"\xff"}'
    meta, _ = fr.decode_activation(struct.pack("<I", len(bad)) + bad + b"zz")
    assert meta == {"a": "�"}


def test_random_round_trips(fr):
    rng = np.random.default_rng(7)
    alphabet = ["a", "Z", "0", " ", "é", "中", "\U0001f600", "\n", '"', "\\", "\x7f"]
    for _ in range(200):
        meta = {
            "run": "".join(rng.choice(alphabet, size=rng.integers(0, 8))),
            "seq_id": int(rng.integers(-2**31, 2**31)),
            "token_pos": int(rng.integers(0, 1 << 20)),
            "f": float(rng.standard_normal() * 10.0 ** int(rng.integers(-30, 30))),
            "shape": [int(rng.integers(1, 9000))],
            "nested": {"x": [True, None, 1.25]},
        }
        payload = rng.integers(0, 65536, size=int(rng.integers(0, 64)), dtype=np.uint16)
        frame = fr.encode_activation(meta, payload)
        m2, p2 = fr.decode_activation(frame)
        assert m2 == meta and p2 == payload.astype("<u2").tobytes()
        # the header is valid JSON whose re-serialisation is stable
        (hlen,) = struct.unpack_from("<I", frame)
        hdr = frame[4:4 + hlen].decode()
        assert fr.js_stringify(json.loads(hdr)) == hdr
        assert not math.isnan(m2["f"])


def test_activation_meta_and_token_message(fr):
    meta = fr.activation_meta("run1", "gpu-0", "s", 41, 2, 3, 8192)
    assert list(meta) == ["run", "node", "seq_id", "token_pos", "from_stage", "to_stage", "dtype", "shape"]
    assert meta["shape"] == [8192] and meta["dtype"] == "f16"
    tok = fr.token_message("run1", "gpu-0", "s", 41, 17)
    assert fr.js_stringify(tok) == \
        '{"t":"token","run":"run1","node":"gpu-0","seq_id":"s","token_pos":41,"token_id":17,"text":"","done":false}'
