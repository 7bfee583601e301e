"""Generate tests/golden/known_answers.json: the known-answer cases of the
reference's own quant tests, restated.

The blocks are built with Python restatements of the reference's test
builders (makeQ8_0Block, dot_test.go:12-22; f32ToF16, dot_test.go:25-49,
which truncates the mantissa and flushes subnormals; makeQ5_KBlock,
dot_q5k_test.go:13-81) and the Q6_K block of dot_q6k_test.go:65-96.  The
expected values are the answers those tests state, not oracle outputs.

    python tests/golden/make_golden.py
"""
import json
import math
import os
import struct

HERE = os.path.dirname(os.path.abspath(__file__))


def f32_to_f16_test(f: float) -> int:
    """dot_test.go:25-49 (test helper: truncates, flushes subnormals)."""
    bits = struct.unpack("<I", struct.pack("<f", f))[0]
    sign, exp, mant = (bits >> 31) & 1, (bits >> 23) & 0xFF, bits & 0x7FFFFF
    if exp == 0:
        return sign << 15
    if exp == 0xFF:
        return (sign << 15) | 0x7C00 | (mant >> 13)
    ne = exp - 127 + 15
    if ne >= 31:
        return (sign << 15) | 0x7C00
    if ne <= 0:
        return sign << 15
    return (sign << 15) | (ne << 10) | (mant >> 13)


def make_q8_0_block(scale: float, quants) -> bytes:
    h = f32_to_f16_test(scale)
    return bytes([h & 0xFF, h >> 8]) + bytes((q & 0xFF) for q in quants)


def make_q5_k_block(d, dmin, sub_scales, sub_mins, quants) -> bytes:
    b = bytearray(176)
    hd, hm = f32_to_f16_test(d), f32_to_f16_test(dmin)
    b[0:4] = bytes([hd & 0xFF, hd >> 8, hm & 0xFF, hm >> 8])
    sc = b[4:16]
    for i in range(4):
        sc[i] = sub_scales[i] & 63
        sc[i + 4] = sub_mins[i] & 63
    for i in range(4, 8):
        s, m = sub_scales[i], sub_mins[i]
        sc[i + 4] = (s & 0xF) | ((m & 0xF) << 4)
        sc[i - 4] |= (s >> 4) << 6
        sc[i] |= (m >> 4) << 6
    b[4:16] = sc
    qh = bytearray(32)
    qs = bytearray(128)
    q_off, sub = 0, 0
    for j in range(0, 256, 64):
        for l in range(32):
            q = quants[j + l]
            qs[q_off + l] = (qs[q_off + l] & 0xF0) | (q & 0xF)
            if q & 0x10:
                qh[l] |= 1 << sub
        sub += 1
        for l in range(32):
            q = quants[j + 32 + l]
            qs[q_off + l] = (qs[q_off + l] & 0x0F) | ((q & 0xF) << 4)
            if q & 0x10:
                qh[l] |= 1 << sub
        sub += 1
        q_off += 32
    b[16:48] = qh
    b[48:176] = qs
    return bytes(b)


def cases():
    out = []
    # dot_test.go:120-148: scale 1.0, quants 1, x = 1 -> 32.0
    out.append({"name": "q8_0_all_ones", "type": 8, "n": 32, "block": make_q8_0_block(1.0, [1] * 32).hex(),
                "x": 1.0, "dot": 32.0, "values": {"all": 1.0}})
    # dot_test.go:150-176: scale 0.5, quants -1, x = 2 -> -32.0
    out.append({"name": "q8_0_negative", "type": 8, "n": 32, "block": make_q8_0_block(0.5, [-1] * 32).hex(),
                "x": 2.0, "dot": -32.0, "values": {"all": -0.5}})
    ones = [1] * 8
    zeros = [0] * 8
    # dot_q5k_test.go:84-108: all quants 15, d=1, scales 1 -> 15.0
    out.append({"name": "q5_k_all_15", "type": 13, "n": 256,
                "block": make_q5_k_block(1.0, 0.0, ones, zeros, [15] * 256).hex(), "x": 1.0, "dot": 15.0 * 256,
                "values": {"all": 15.0}})
    # dot_q5k_test.go:111-136: all quants 16 (high bit only) -> 16.0
    out.append({"name": "q5_k_all_16", "type": 13, "n": 256,
                "block": make_q5_k_block(1.0, 0.0, ones, zeros, [16] * 256).hex(), "x": 1.0, "dot": 16.0 * 256,
                "values": {"all": 16.0}})
    # dot_q5k_test.go:138-174: alternating 0/31, d=.5 dmin=.25 sc=2 m=1 -> -0.25 / 30.75
    alt = [0 if i % 2 == 0 else 31 for i in range(256)]
    out.append({"name": "q5_k_alternating", "type": 13, "n": 256,
                "block": make_q5_k_block(0.5, 0.25, [2] * 8, [1] * 8, alt).hex(), "x": 1.0,
                "dot": 128 * -0.25 + 128 * 30.75, "values": {"even": -0.25, "odd": 30.75}})
    # dot_q5k_test.go:176-222: element 0 of every sub-group has only the high bit
    hb = [0] * 256
    for i in range(0, 256, 32):
        hb[i] = 16
    out.append({"name": "q5_k_high_bit_positions", "type": 13, "n": 256,
                "block": make_q5_k_block(1.0, 0.0, ones, zeros, hb).hex(), "x": 1.0, "dot": 16.0 * 8,
                "values": {"index_multiple_of_32": 16.0, "other": 0.0}})
    # dot_q6k_test.go:59-104: ql=0x11, qh=0, scales 10+5i, d=1.0 (0x3C00), x=1
    b = bytearray(210)
    b[0:128] = b"\x11" * 128
    for i in range(16):
        b[192 + i] = (10 + 5 * i) & 0xFF
    b[208], b[209] = 0x00, 0x3C
    scales = [10 + 5 * i for i in range(16)]
    out.append({"name": "q6_k_distinct_scales", "type": 14, "n": 256, "block": bytes(b).hex(), "x": 1.0,
                "dot": float(sum(-31 * s * 16 for s in scales)),
                "values": {"per16": [float(-31 * s) for s in scales]}})
    return out


if __name__ == "__main__":
    path = os.path.join(HERE, "known_answers.json")
    with open(path, "w") as f:
        json.dump({"source": "restated known-answer tests of dbrushchenko/llm-embed internal/ggml/*_test.go",
                   "cases": cases()}, f, indent=1)
    print(path)
    assert math.isclose(cases()[-1]["dot"], -376960.0)
