"""GGUF tensors on the device: LoadTensor (loadTensor,
pkg/model/transformer.go:285-303, with the dequantization on the GPU) gives
the oracle's values bit for bit for every format, and a tensor's stored
bytes uploaded as they are feed glc_linear_bwd_dx_q directly."""
import ctypes as C

import numpy as np
import pytest

from gollama_b200 import gguf
from gollama_b200.device import GlcError
from oracle.oracle import lib as orc_lib
from tests import gguf_writer as W
from tests.helpers import rel_fro
from tests.test_quant import ALL_TYPES, F32, Q4_K, Q8_0, orc_dequant, sane_format_weight

pytestmark = pytest.mark.gpu


def weight_bytes(qtype, rows, cols, seed):
    if qtype == F32:
        return np.random.default_rng(seed).standard_normal(rows * cols).astype(np.float32).tobytes()
    return sane_format_weight(qtype, rows, cols, seed)


def test_load_tensor_every_format(ctx, tmp_path):
    rows, cols = 8, 512
    tensors = [(f"w{t}", [cols, rows], t, weight_bytes(t, rows, cols, 40 + t)) for t in ALL_TYPES]
    blob, *_ = W.gguf_bytes([("general.architecture", W.STRING, "llama")], tensors)
    path = tmp_path / "w.gguf"
    path.write_bytes(blob)
    with gguf.Open(path) as r:
        for name, dims, t, data in tensors:
            got = r.LoadTensor(ctx, name).numpy()
            assert got.shape == (rows, cols)
            want = orc_dequant(data, rows * cols, t).reshape(rows, cols)
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), name


@pytest.mark.parametrize("qtype", [Q8_0, Q4_K])
def test_uploaded_weight_feeds_linear_bwd_dx_q(ctx, tmp_path, qtype):
    M, K, N = 64, 512, 96  # W [N out][K in], GGUF dims [K, N]
    data = weight_bytes(qtype, N, K, 5)
    blob, *_ = W.gguf_bytes([], [("blk.0.ffn_down.weight", [K, N], qtype, data)])
    path = tmp_path / "q.gguf"
    path.write_bytes(blob)
    r = np.random.default_rng(3)
    dy = r.standard_normal((M, N)).astype(np.float32)
    want = np.zeros((M, K), np.float64)
    src = np.frombuffer(data, np.uint8).copy()
    assert orc_lib().orcd_linear_bwd_dx_q(dy.astype(np.float64).ctypes.data_as(C.c_void_p),
                                          src.ctypes.data_as(C.c_void_p), qtype, want.ctypes.data_as(C.c_void_p), M,
                                          K, N) == 0
    with gguf.Open(path) as g:
        wq = g.UploadTensor(ctx, "blk.0.ffn_down.weight")
        assert np.array_equal(wq.numpy(), src)
        d_dy, d_dx = ctx.from_numpy(dy), ctx.zeros((M, K))
        ctx.call("glc_linear_bwd_dx_q", d_dy.ptr, wq.ptr, qtype, d_dx.ptr, M, K, N, 0)
        ctx.sync()
    assert rel_fro(d_dx.numpy(), want) < 2e-3


def test_load_tensor_refusals(ctx, tmp_path):
    tensors = [("odd", [33], 2, bytes(36)), ("bf16", [8], 30, bytes(16))]
    blob, *_ = W.gguf_bytes([], tensors)
    path = tmp_path / "o.gguf"
    path.write_bytes(blob)
    with gguf.Open(path) as r:
        with pytest.raises(GlcError):
            r.LoadTensor(ctx, "odd")  # not a whole number of blocks
        with pytest.raises(GlcError):
            r.LoadTensor(ctx, "bf16")  # not in the reference's Dequantize (panics there)
