"""Golden vectors of the reference's weight dequantization
(pkg/quant/dequant.go:9-393) for every type its Dequantize accepts.

A plain-Python restatement, written separately from the C oracle
(oracle/oracle.c) and from the device decoder (gollama_b200/csrc/
quant_formats.cuh): fp16ToFp32 with the reference's shift loop, then each
format's loops in the reference's order with numpy.float32 scalars, so every
product and sum rounds once to float32 like Go's (no fused multiply-add on
amd64).  Blocks hold random bytes; the half-precision scales come from a list
that covers zero, both signs, subnormals, the largest finite half and
ordinary values.  tests/test_quant.py checks the oracle against these
vectors bit for bit.

    python tests/golden/make_quant_golden.py     # rewrites dequant.json
"""
import json
from pathlib import Path

import numpy as np

OUT = Path(__file__).with_name("dequant.json")
f32 = np.float32

# type code: (elements per block, bytes per block)  pkg/gguf/format.go:117-149
FORMATS = {0: (1, 4), 1: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 12: (256, 144),
           14: (256, 210)}
SCALES = [0x0000, 0x8000, 0x0001, 0x03FF, 0x8200, 0x0400, 0x2E66, 0x211F, 0xA11F, 0x3C00, 0x7BFF, 0xFBFF, 0x1C00,
          0x3555]


def fp16_to_fp32(h: int) -> f32:
    """dequant.go:9-41."""
    sign = (h >> 15) & 1
    exp = (h >> 10) & 0x1F
    mant = h & 0x3FF
    if exp == 0:
        if mant == 0:
            f = sign << 31
        else:
            exp = 1
            while (mant & 0x400) == 0:
                mant <<= 1
                exp -= 1
            mant &= 0x3FF
            f = (sign << 31) | (((exp + 127 - 15) & 0xFFFFFFFF) << 23) | (mant << 13)
    elif exp == 31:
        f = (sign << 31) | 0x7F800000 | (mant << 13)
    else:
        f = (sign << 31) | ((exp + 127 - 15) << 23) | (mant << 13)
    return np.array([f & 0xFFFFFFFF], np.uint32).view(np.float32)[0]


def u16(d: bytes, o: int) -> int:
    return d[o] | (d[o + 1] << 8)


def u32(d: bytes, o: int) -> int:
    return u16(d, o) | (u16(d, o + 2) << 16)


def i8(x: int) -> int:
    x &= 0xFF
    return x - 256 if x >= 128 else x


def dequantize(data: bytes, n: int, t: int) -> np.ndarray:
    out = np.zeros(n, np.float32)
    if t == 0:
        return np.frombuffer(data[: 4 * n], np.float32).copy()
    if t == 1:
        for i in range(n):
            out[i] = fp16_to_fp32(u16(data, 2 * i))
        return out
    be, bb = FORMATS[t]
    for b in range(n // be):
        o = b * bb
        if t == 8:  # :68-85
            scale = fp16_to_fp32(u16(data, o))
            for i in range(32):
                out[b * 32 + i] = scale * f32(i8(data[o + 2 + i]))
        elif t == 2:  # :99-119
            scale = fp16_to_fp32(u16(data, o))
            for i in range(16):
                q = data[o + 2 + i]
                out[b * 32 + 2 * i] = scale * f32((q & 0x0F) - 8)
                out[b * 32 + 2 * i + 1] = scale * f32((q >> 4) - 8)
        elif t == 3:  # :141-163
            scale, mn = fp16_to_fp32(u16(data, o)), fp16_to_fp32(u16(data, o + 2))
            for i in range(16):
                q = data[o + 4 + i]
                out[b * 32 + 2 * i] = scale * f32(q & 0x0F) + mn
                out[b * 32 + 2 * i + 1] = scale * f32(q >> 4) + mn
        elif t == 6:  # :167-199
            scale = fp16_to_fp32(u16(data, o))
            qh = u32(data, o + 2)
            for i in range(16):
                q = data[o + 6 + i]
                q0, q1 = q & 0x0F, q >> 4
                if (qh >> (i * 2)) & 1:
                    q0 |= 0x10
                if (qh >> (i * 2 + 1)) & 1:
                    q1 |= 0x10
                out[b * 32 + 2 * i] = scale * f32(q0 - 16)
                out[b * 32 + 2 * i + 1] = scale * f32(q1 - 16)
        elif t == 7:  # :203-233
            scale, mn = fp16_to_fp32(u16(data, o)), fp16_to_fp32(u16(data, o + 2))
            qh = u32(data, o + 4)
            for i in range(16):
                q = data[o + 8 + i]
                q0, q1 = q & 0x0F, q >> 4
                if (qh >> (i * 2)) & 1:
                    q0 |= 0x10
                if (qh >> (i * 2 + 1)) & 1:
                    q1 |= 0x10
                out[b * 32 + 2 * i] = scale * f32(q0) + mn
                out[b * 32 + 2 * i + 1] = scale * f32(q1) + mn
        elif t == 12:  # :237-300
            d, dmin = fp16_to_fp32(u16(data, o)), fp16_to_fp32(u16(data, o + 2))
            s = data[o + 4 : o + 16]
            qs = data[o + 16 : o + 144]
            sc = [s[0] & 63, s[1] & 63, s[2] & 63, s[3] & 63,
                  (s[8] & 0xF) | ((s[0] >> 6) << 4), (s[8] >> 4) | ((s[1] >> 6) << 4),
                  (s[9] & 0xF) | ((s[2] >> 6) << 4), (s[9] >> 4) | ((s[3] >> 6) << 4)]
            m = [s[4] & 63, s[5] & 63, s[6] & 63, s[7] & 63,
                 (s[10] & 0xF) | ((s[4] >> 6) << 4), (s[10] >> 4) | ((s[5] >> 6) << 4),
                 (s[11] & 0xF) | ((s[6] >> 6) << 4), (s[11] >> 4) | ((s[7] >> 6) << 4)]
            for j in range(8):
                scale_val = d * f32(sc[j])
                min_val = dmin * f32(m[j])
                for i in range(16):
                    q = qs[j * 16 + i]
                    out[b * 256 + j * 32 + i * 2] = scale_val * f32(q & 0x0F) - min_val
                    out[b * 256 + j * 32 + i * 2 + 1] = scale_val * f32(q >> 4) - min_val
        elif t == 14:  # :304-344
            ql, qh, scales = data[o : o + 128], data[o + 128 : o + 192], data[o + 192 : o + 208]
            d = fp16_to_fp32(u16(data, o + 208))
            for j in range(16):
                scale_val = d * f32(i8(scales[j]))
                for i in range(16):
                    idx = j * 16 + i
                    q = (ql[idx // 2] & 0x0F) if idx % 2 == 0 else (ql[idx // 2] >> 4)
                    q_high = (qh[idx // 4] >> ((idx % 4) * 2)) & 0x03
                    q6 = i8(q | (q_high << 4)) - 32
                    out[b * 256 + idx] = scale_val * f32(q6)
    return out


def random_blocks(t: int, nblocks: int, rng) -> bytes:
    be, bb = FORMATS[t]
    raw = bytearray(rng.integers(0, 256, nblocks * bb, dtype=np.uint8).tobytes())
    if t in (0, 1):
        if t == 0:  # finite float32 values only: a NaN's payload is not part of the format
            v = rng.standard_normal(nblocks).astype(np.float32)
            return v.tobytes()
        return bytes(raw)
    # half fields from the list (every one at its offset)
    half_offsets = {2: [0], 3: [0, 2], 6: [0], 7: [0, 2], 8: [0], 12: [0, 2], 14: [208]}[t]
    for b in range(nblocks):
        for ho in half_offsets:
            h = SCALES[int(rng.integers(0, len(SCALES)))]
            raw[b * bb + ho] = h & 0xFF
            raw[b * bb + ho + 1] = h >> 8
    return bytes(raw)


def main() -> None:
    rng = np.random.default_rng(20250612)
    data = {}
    for t, (be, bb) in FORMATS.items():
        nblocks = {1: 64, 32: 12, 256: 3}[be] if t != 0 else 32
        if t == 1:  # every fp16 class: random codes plus the scale list
            raw = random_blocks(t, nblocks, rng) + b"".join(h.to_bytes(2, "little") for h in SCALES)
            n = nblocks + len(SCALES)
        else:
            raw = random_blocks(t, nblocks, rng)
            n = nblocks * be
        out = dequantize(raw, n, t)
        data[str(t)] = {"n": n, "hex": raw.hex(), "bits": [int(x) for x in out.view(np.uint32)]}
    OUT.write_text(json.dumps(data, separators=(",", ":")))
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
