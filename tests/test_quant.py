"""Frozen quantized weights (pkg/quant/dequant.go): the oracle's restatement
pinned by values worked out by hand and by numpy's IEEE half conversion.

The reference has no tests for these formats, so the fixtures are the
build's own: every fp16 code, hand-made Q8_0 and Q4_0 blocks (including the
reference's nibble order: element 2i is the low nibble, element 2i+1 the
high one), and random blocks against an independent numpy decoder."""
import ctypes as C

import numpy as np
import pytest

from oracle.oracle import lib

F32, F16, Q4_0, Q8_0 = 0, 1, 2, 8


def orc_dequant(data: bytes, n: int, qtype: int) -> np.ndarray:
    src = np.frombuffer(data, np.uint8).copy()
    out = np.empty(n, np.float32)
    rc = lib().orc_dequantize(src.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p), C.c_int64(n), qtype)
    assert rc == 0
    return out


def expected_half_bits(h: np.ndarray) -> np.ndarray:
    """fp16ToFp32 by the IEEE definition: numpy for numbers, payload << 13 for NaN."""
    f = h.view(np.float16).astype(np.float32).view(np.uint32)
    nan = ((h >> 10) & 0x1F == 31) & (h & 0x3FF != 0)
    f[nan] = ((h[nan].astype(np.uint32) >> 15) << 31) | 0x7F800000 | ((h[nan].astype(np.uint32) & 0x3FF) << 13)
    return f


def test_fp16_every_code():
    fn = lib().orc_fp16_to_fp32
    fn.restype = C.c_float
    fn.argtypes = [C.c_uint16]
    codes = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    # bit for bit through the array path (signalling NaNs keep their payload)
    assert np.array_equal(orc_dequant(codes.tobytes(), 65536, F16).view(np.uint32), expected_half_bits(codes))
    # the scalar entry point on every non-NaN code (a float returned through
    # ctypes is widened to a Python float, which would quiet a signalling NaN)
    num = codes[~(((codes >> 10) & 0x1F == 31) & (codes & 0x3FF != 0))]
    got = np.array([fn(int(h)) for h in num], np.float32).view(np.uint32)
    assert np.array_equal(got, expected_half_bits(num))


def test_q8_0_hand_block():
    # scale 0.5 (fp16 0x3800), codes -128..127 in steps of 8
    codes = np.arange(-128, 128, 8, dtype=np.int8)
    blk = np.uint16(0x3800).tobytes() + codes.tobytes()
    assert len(blk) == 34
    want = np.array([0.5 * c for c in range(-128, 128, 8)], np.float32)
    assert np.array_equal(orc_dequant(blk, 32, Q8_0), want)


def test_q4_0_hand_block_nibble_order():
    # scale 2.0 (fp16 0x4000); byte i = (hi << 4) | lo with lo = i, hi = 15 - i
    qs = bytes(((15 - i) << 4) | i for i in range(16))
    blk = np.uint16(0x4000).tobytes() + qs
    assert len(blk) == 18
    want = []
    for i in range(16):
        want += [2.0 * (i - 8), 2.0 * ((15 - i) - 8)]  # element 2i: low nibble; 2i+1: high nibble
    assert np.array_equal(orc_dequant(blk, 32, Q4_0), np.array(want, np.float32))


def numpy_dequant(data: bytes, n: int, qtype: int) -> np.ndarray:
    a = np.frombuffer(data, np.uint8)
    if qtype == F16:
        return a.view(np.float16).astype(np.float32)
    bsz = 34 if qtype == Q8_0 else 18
    blocks = a.reshape(n // 32, bsz)
    scale = blocks[:, :2].copy().view(np.float16).astype(np.float32)
    if qtype == Q8_0:
        q = blocks[:, 2:].view(np.int8).astype(np.float32)
    else:
        b = blocks[:, 2:]
        q = np.empty((n // 32, 32), np.float32)
        q[:, 0::2] = (b & 0x0F).astype(np.float32) - 8
        q[:, 1::2] = (b >> 4).astype(np.float32) - 8
    return (scale * q).astype(np.float32).reshape(-1)


def random_weight(qtype: int, rows: int, cols: int, seed: int) -> bytes:
    """Rows of `cols` elements: fp16 scales U(0.005, 0.02), uniform random codes."""
    r = np.random.default_rng(seed)
    n = rows * cols
    if qtype == F16:
        return r.standard_normal(n).astype(np.float16).tobytes()
    nb = n // 32
    scale = r.uniform(0.005, 0.02, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    codes = r.integers(0, 256, (nb, 32 if qtype == Q8_0 else 16), dtype=np.uint8)
    return np.concatenate([scale, codes], axis=1).tobytes()


@pytest.mark.parametrize("qtype", [F16, Q4_0, Q8_0])
def test_random_blocks_match_numpy(qtype):
    data = random_weight(qtype, 64, 256, 3 + qtype)
    n = 64 * 256
    assert np.array_equal(orc_dequant(data, n, qtype), numpy_dequant(data, n, qtype))


@pytest.mark.parametrize("qtype", [Q4_0, Q8_0])
def test_oracle_linear_bwd_dx_q(qtype):
    """The oracle's dX = dY . deq(W) (dA loop of MatMulGrad on the dequantized weight)."""
    M, K, N = 8, 64, 32
    r = np.random.default_rng(9)
    dy = r.standard_normal((M, N)).astype(np.float32)
    data = random_weight(qtype, N, K, 4)
    src = np.frombuffer(data, np.uint8).copy()
    dx = np.zeros((M, K), np.float32)
    rc = lib().orc_linear_bwd_dx_q(dy.ctypes.data_as(C.c_void_p), src.ctypes.data_as(C.c_void_p), qtype,
                                   dx.ctypes.data_as(C.c_void_p), M, K, N)
    assert rc == 0
    w = numpy_dequant(data, N * K, qtype).reshape(N, K)
    np.testing.assert_allclose(dx, dy.astype(np.float64) @ w.astype(np.float64), rtol=1e-5, atol=1e-6)
