"""Frozen quantized weights on the GPU against the oracle: glc_dequantize bit
for bit (every fp16 code, random blocks of every format with extreme scales), and
glc_linear_bwd_dx_q (dX = dY . deq(W), MatMulGrad's dA on the dequantized
weight) within the TF32 bar of the other GEMMs (relative Frobenius error
2e-3)."""
import ctypes as C

import numpy as np
import pytest

from oracle.oracle import lib as orc_lib
from tests.helpers import rel_fro
from tests.test_quant import (F16, Q4_0, Q4_1, Q4_K, Q5_0, Q5_1, Q6_K, Q8_0, orc_dequant, random_format_bytes,
                              random_weight, sane_format_weight)

pytestmark = pytest.mark.gpu
TOL = 2e-3


def gpu_dequant(ctx, data: bytes, n: int, qtype: int) -> np.ndarray:
    src = ctx.from_numpy(np.frombuffer(data, np.uint8).copy())
    out = ctx.empty((n,))
    ctx.call("glc_dequantize", qtype, src.ptr, out.ptr, n)
    ctx.sync()
    return out.numpy()


def test_dequant_f16_every_code(ctx):
    codes = np.arange(65536, dtype=np.uint32).astype(np.uint16).tobytes()
    got = gpu_dequant(ctx, codes, 65536, F16)
    assert np.array_equal(got.view(np.uint32), orc_dequant(codes, 65536, F16).view(np.uint32))


@pytest.mark.parametrize("qtype", [Q4_0, Q8_0])
def test_dequant_blocks_bit_exact(ctx, qtype):
    data = bytearray(random_weight(qtype, 96, 512, 21 + qtype))
    bsz = 34 if qtype == Q8_0 else 18
    # extreme scales in the first blocks: subnormal, largest, infinity, NaN, -0
    for i, h in enumerate([0x0001, 0x03FF, 0x7BFF, 0x7C00, 0x7E01, 0x8000]):
        data[bsz * i : bsz * i + 2] = np.uint16(h).tobytes()
    data = bytes(data)
    n = 96 * 512
    got, want = gpu_dequant(ctx, data, n, qtype), orc_dequant(data, n, qtype)
    # a product that is NaN (NaN scale, infinity times code 0) carries the
    # multiplier's NaN encoding (canonical on the GPU, x86's on the host):
    # NaN for NaN there, identical bits everywhere else
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


def test_dequant_rejects_ragged_blocks(ctx):
    from gollama_b200.device import GlcError

    src, out = ctx.empty((64,)), ctx.empty((48,))
    with pytest.raises(GlcError):
        ctx.call("glc_dequantize", Q8_0, src.ptr, out.ptr, 48)
    with pytest.raises(GlcError):
        ctx.call("glc_dequantize", 9, src.ptr, out.ptr, 32)  # Q8_1: not in the reference's Dequantize
    with pytest.raises(GlcError):
        ctx.call("glc_dequantize", Q4_K, src.ptr, out.ptr, 32)  # a partial 256-element super-block


@pytest.mark.parametrize("qtype", [Q4_1, Q5_0, Q5_1, Q4_K, Q6_K])
def test_dequant_more_formats_bit_exact(ctx, qtype):
    """Random bytes in every field (NaN, infinite and subnormal scales among
    them): identical bits except NaN encodings, as above."""
    data, n = random_format_bytes(qtype, 512 if qtype in (Q4_K, Q6_K) else 4096, 77 + qtype)
    got, want = gpu_dequant(ctx, data, n, qtype), orc_dequant(data, n, qtype)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


@pytest.mark.parametrize("qtype", [F16, Q4_0, Q8_0, Q4_1, Q5_0, Q5_1, Q4_K, Q6_K])
@pytest.mark.parametrize("M,K,N,acc", [(64, 256, 96, 0), (300, 512, 1376, 1), (512, 2048, 704, 0)])
def test_linear_bwd_dx_q(ctx, qtype, M, K, N, acc):
    r = np.random.default_rng(M + K + N + qtype)
    dy = r.standard_normal((M, N)).astype(np.float32)
    dx0 = r.standard_normal((M, K)).astype(np.float32) if acc else np.zeros((M, K), np.float32)
    data = sane_format_weight(qtype, N, K, 31 + qtype)
    src = np.frombuffer(data, np.uint8).copy()
    want = dx0.astype(np.float64).copy()
    rc = orc_lib().orcd_linear_bwd_dx_q(dy.astype(np.float64).ctypes.data_as(C.c_void_p), src.ctypes.data_as(C.c_void_p),
                                        qtype, want.ctypes.data_as(C.c_void_p), M, K, N)
    assert rc == 0
    d_dy, d_w, d_dx = ctx.from_numpy(dy), ctx.from_numpy(src), ctx.from_numpy(dx0)
    ctx.call("glc_linear_bwd_dx_q", d_dy.ptr, d_w.ptr, qtype, d_dx.ptr, M, K, N, acc)
    ctx.sync()
    assert rel_fro(d_dx.numpy(), want) < TOL


@pytest.mark.parametrize("qtype", [F16, Q4_0, Q8_0, Q4_1, Q5_0, Q5_1, Q4_K, Q6_K])
@pytest.mark.parametrize("M,K,N,acc", [(64, 256, 96, 0), (300, 512, 1376, 1), (512, 2048, 704, 0), (130, 768, 36, 1)])
def test_linear_bwd_dx_q_fused_decode(ctx, qtype, M, K, N, acc):
    """glc_set_quant_path(2): the blocks decoded inside the GEMM's operand load
    give the oracle's dX within the TF32 bar and agree with the dequantize +
    GEMM path (both round W to TF32 the same way)."""
    r = np.random.default_rng(M + K + N + qtype + 1)
    dy = r.standard_normal((M, N)).astype(np.float32)
    dx0 = r.standard_normal((M, K)).astype(np.float32) if acc else np.zeros((M, K), np.float32)
    data = sane_format_weight(qtype, N, K, 61 + qtype)
    src = np.frombuffer(data, np.uint8).copy()
    want = dx0.astype(np.float64).copy()
    assert orc_lib().orcd_linear_bwd_dx_q(dy.astype(np.float64).ctypes.data_as(C.c_void_p),
                                          src.ctypes.data_as(C.c_void_p), qtype, want.ctypes.data_as(C.c_void_p), M,
                                          K, N) == 0
    outs = []
    try:
        for path in (1, 2):
            ctx.call("glc_set_quant_path", path)
            d_dy, d_w, d_dx = ctx.from_numpy(dy), ctx.from_numpy(src), ctx.from_numpy(dx0)
            ctx.call("glc_linear_bwd_dx_q", d_dy.ptr, d_w.ptr, qtype, d_dx.ptr, M, K, N, acc)
            ctx.sync()
            outs.append(d_dx.numpy())
    finally:
        ctx.call("glc_set_quant_path", 0)
    assert rel_fro(outs[1], want) < TOL
    assert rel_fro(outs[1], outs[0].astype(np.float64)) < 1e-6
