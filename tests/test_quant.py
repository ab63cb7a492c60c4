"""Frozen quantized weights (pkg/quant/dequant.go): the oracle's restatement
pinned by values worked out by hand and by numpy's IEEE half conversion.

The reference has no tests for these formats, so the fixtures are the
build's own: every fp16 code, hand-made Q8_0 and Q4_0 blocks (including the
reference's nibble order: element 2i is the low nibble, element 2i+1 the
high one), random blocks against an independent numpy decoder, and golden
vectors of every format the reference's Dequantize accepts from a separate
plain-Python restatement (tests/golden/make_quant_golden.py).  The device
decoder (gollama_b200/csrc/quant_formats.cuh) is compiled for the host here
and must reproduce the oracle bit for bit on random blocks, including NaN,
infinite and subnormal half scales."""
import ctypes as C
import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle.oracle import lib

F32, F16, Q4_0, Q8_0 = 0, 1, 2, 8
Q4_1, Q5_0, Q5_1, Q4_K, Q6_K = 3, 6, 7, 12, 14
ALL_TYPES = [F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K, Q6_K]
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22), Q5_1: (32, 24), Q8_0: (32, 34),
         Q4_K: (256, 144), Q6_K: (256, 210)}
HERE = Path(__file__).parent
GOLDEN = json.loads((HERE / "golden" / "dequant.json").read_text())


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


@pytest.mark.parametrize("qtype", ALL_TYPES)
def test_oracle_matches_dequant_golden(qtype):
    g = GOLDEN[str(qtype)]
    got = orc_dequant(bytes.fromhex(g["hex"]), g["n"], qtype)
    assert np.array_equal(got.view(np.uint32), np.array(g["bits"], np.uint32))


def test_q4_k_hand_block():
    """Sub-block 5 (scale and min from the packed high bits) of a Q4_K block:
    d = 1, dmin = 0.5; scales[9] = 0x3A (sc[6] low = 0xA, sc[7] low = 3),
    scales[1] = 0x80 (sc[5] high = 2 << 4), scales[8] = 0x70 (sc[5] low = 7)."""
    blk = bytearray(144)
    blk[0:2] = (0x3C00).to_bytes(2, "little")  # d = 1
    blk[2:4] = (0x3800).to_bytes(2, "little")  # dmin = 0.5
    s = blk[4:16]
    s[1] = 0x80  # sc[1] = 0, high bits 2 -> sc[5] += 32
    s[8] = 0x70  # sc[4] low 0, sc[5] low 7
    s[5] = 0xC5  # m[1] = 5, high bits 3 -> m[5] += 48
    s[10] = 0x90  # m[4] low 0, m[5] low 9
    blk[4:16] = s
    for i in range(16):
        blk[16 + 5 * 16 + i] = (15 - i) << 4 | i  # sub-block 5: element 2i = i, 2i+1 = 15 - i
    out = orc_dequant(bytes(blk), 256, Q4_K)
    sc5, m5 = 7 | 32, 9 | 48
    want = []
    for i in range(16):
        want += [np.float32(sc5) * np.float32(i) - np.float32(0.5 * m5),
                 np.float32(sc5) * np.float32(15 - i) - np.float32(0.5 * m5)]
    assert np.array_equal(out[160:192], np.array(want, np.float32))


@pytest.fixture(scope="module")
def host_decoder():
    """quant_formats.cuh built as a host library (test harness only)."""
    out = HERE / "native" / "_build" / "quant_host.so"
    out.parent.mkdir(exist_ok=True)
    src = HERE / "native" / "quant_host.cpp"
    hdr = HERE.parent / "gollama_b200" / "csrc" / "quant_formats.cuh"
    if not out.exists() or out.stat().st_mtime < max(src.stat().st_mtime, hdr.stat().st_mtime):
        subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-shared", "-fPIC", str(src), "-o", str(out)],
                       check=True)
    h = C.CDLL(str(out))
    h.qf_dequantize_host.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int64]
    h.qf_dequantize_host.restype = C.c_int
    return h


def random_format_bytes(qtype, nblocks, seed):
    """Random bytes for every field, scales included (NaN, infinite and
    subnormal halves among them)."""
    be, bb = BLOCK[qtype]
    raw = np.random.default_rng(seed).integers(0, 256, nblocks * bb, dtype=np.uint8)
    return raw.tobytes(), nblocks * be


@pytest.mark.parametrize("qtype", ALL_TYPES)
def test_device_decoder_matches_oracle_on_host(host_decoder, qtype):
    for seed in range(3):
        nblocks = {1: 4096, 32: 512, 256: 64}[BLOCK[qtype][0]]
        data, n = random_format_bytes(qtype, nblocks, 100 * qtype + seed)
        want = orc_dequant(data, n, qtype)
        src = np.frombuffer(data, np.uint8).copy()
        got = np.empty(n, np.float32)
        assert host_decoder.qf_dequantize_host(src.ctypes.data_as(C.c_void_p), qtype,
                                               got.ctypes.data_as(C.c_void_p), n) == 0
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), qtype
    g = GOLDEN[str(qtype)]
    src = np.frombuffer(bytes.fromhex(g["hex"]), np.uint8).copy()
    n = g["n"] - g["n"] % 4
    got = np.empty(n, np.float32)
    assert host_decoder.qf_dequantize_host(src.ctypes.data_as(C.c_void_p), qtype, got.ctypes.data_as(C.c_void_p),
                                           n) == 0
    assert np.array_equal(got.view(np.uint32), np.array(g["bits"][:n], np.uint32))


def test_host_decoder_rejects_partial_blocks(host_decoder):
    buf = np.zeros(1024, np.uint8)
    out = np.zeros(256, np.float32)
    assert host_decoder.qf_dequantize_host(buf.ctypes.data_as(C.c_void_p), Q4_K, out.ctypes.data_as(C.c_void_p),
                                           128) == -1
    assert host_decoder.qf_dequantize_host(buf.ctypes.data_as(C.c_void_p), 9, out.ctypes.data_as(C.c_void_p),
                                           32) == -1  # Q8_1: not in the reference's Dequantize


HALF_OFFSETS = {Q4_0: [0], Q4_1: [0, 2], Q5_0: [0], Q5_1: [0, 2], Q8_0: [0], Q4_K: [0, 2], Q6_K: [208]}


def sane_format_weight(qtype, rows, cols, seed):
    """rows x cols elements of any block format: half scales U(0.005, 0.02)
    (positive, finite), every other byte random."""
    if qtype in (F16, Q4_0, Q8_0):
        return random_weight(qtype, rows, cols, seed)
    be, bb = BLOCK[qtype]
    nb = rows * cols // be
    r = np.random.default_rng(seed)
    raw = r.integers(0, 256, (nb, bb), dtype=np.uint8)
    for off in HALF_OFFSETS[qtype]:
        raw[:, off : off + 2] = r.uniform(0.005, 0.02, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return raw.tobytes()


@pytest.mark.parametrize("qtype", [Q4_1, Q5_0, Q5_1, Q4_K, Q6_K])
def test_oracle_linear_bwd_dx_q_more_formats(qtype):
    M, K, N = 4, 256, 8
    r = np.random.default_rng(19)
    dy = r.standard_normal((M, N)).astype(np.float32)
    data = sane_format_weight(qtype, N, K, 6)
    src = np.frombuffer(data, np.uint8).copy()
    dx = np.zeros((M, K), np.float32)
    assert lib().orc_linear_bwd_dx_q(dy.ctypes.data_as(C.c_void_p), src.ctypes.data_as(C.c_void_p), qtype,
                                     dx.ctypes.data_as(C.c_void_p), M, K, N) == 0
    w = orc_dequant(data, N * K, qtype).reshape(N, K)
    assert np.all(np.isfinite(w))
    np.testing.assert_allclose(dx, dy.astype(np.float64) @ w.astype(np.float64), rtol=1e-5, atol=1e-5)
