"""The isolated backward-op sweep and the quantized-weight dX at their full
sizes, against the oracle (oracle/oracle.c) or an fp64 product of the same fp32
inputs.

Sizes: linear layers with M = 32768 tokens for (K, N) in (2048, 2048),
(2048, 5632), (5632, 2048); RMSNorm backward 32768 x 2048; causal attention
with 32 query / 4 KV heads, head_dim 64, batch 4, sequences of 1024 and 2048;
softmax cross-entropy on 32768 x 32000 logits N(0, 2) with uniform targets;
dX = dY . deq(W) with W 5632 x 2048 stored as Q8_0 and Q4_0 and dY 16384 x 5632.

The large operands are drawn on the device (torch's seeded generator) and the
checks use sampled rows and columns where the full product would take the
host minutes: a GEMM output is compared on 64 rows (64 x 48 entries of dW);
attention at sequence 2048 on two of the four sequences; the CE loss on every
row and its gradient on 256 rows.  Bars: 2e-3 relative Frobenius error for
tensor-core results (TF32 operands, fp32 accumulation), 2e-5 for fp32
CUDA-core kernels, 1e-5 relative for the CE loss."""
import ctypes as C

import numpy as np
import pytest

from oracle.oracle import Oracle
from oracle.oracle import lib as orc_lib
from tests.helpers import FP32_RTOL, rel_fro, threads
from tests.test_ops_gpu import ATTN_TOL, tf32
from tests.test_quant import Q4_0, Q8_0, random_weight

pytestmark = pytest.mark.gpu

TOL = 2e-3
M_SWEEP = 32768


@pytest.fixture(scope="module")
def torch_cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device visible to torch")
    return torch


@pytest.fixture(scope="module")
def orc():
    return Oracle(threads=threads())


def dev_randn(torch, shape, seed, std=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    t = torch.randn(*shape, generator=g, device="cuda", dtype=torch.float32)
    return t.mul_(std) if std != 1.0 else t


def ptr(t):
    return C.c_void_p(t.data_ptr())


def sample(n, k, seed):
    return np.sort(np.random.default_rng(seed).choice(n, size=min(k, n), replace=False))


@pytest.mark.parametrize("K,N", [(2048, 2048), (2048, 5632), (5632, 2048)])
def test_linear_sweep_m32768(ctx, torch_cuda, K, N):
    """Y = X.W^T, dX = dY.W and dW = dY^T.X (MatMulGrad, pkg/tensor/grad.go:
    81-152) at M = 32768, each checked on sampled rows against fp64."""
    torch, M = torch_cuda, M_SWEEP
    X = dev_randn(torch, (M, K), 11 + K)
    W = dev_randn(torch, (N, K), 12 + N)
    dY = dev_randn(torch, (M, N), 13 + K + N)
    Y = torch.empty((M, N), device="cuda")
    dX = torch.empty((M, K), device="cuda")
    dW = torch.empty((N, K), device="cuda")
    torch.cuda.synchronize()
    ctx.call("glc_linear_fwd", ptr(X), ptr(W), ptr(Y), M, K, N, None)
    ctx.call("glc_linear_bwd_dx", ptr(dY), ptr(W), ptr(dX), M, K, N, 0)
    ctx.call("glc_linear_bwd_dw", ptr(dY), ptr(X), ptr(dW), M, K, N, 0)
    ctx.sync()
    rows = sample(M, 64, K + N)
    ridx = torch.as_tensor(rows, device="cuda")
    Wh = W.cpu().numpy().astype(np.float64)
    xr = X.index_select(0, ridx).cpu().numpy().astype(np.float64)
    gr = dY.index_select(0, ridx).cpu().numpy().astype(np.float64)
    assert rel_fro(Y.index_select(0, ridx).cpu().numpy(), xr @ Wh.T) < TOL
    assert rel_fro(dX.index_select(0, ridx).cpu().numpy(), gr @ Wh) < TOL
    # dW[n, k] sums over all M tokens: sampled output rows n and columns k
    ns, ks = sample(N, 64, N + 1), sample(K, 48, K + 2)
    gcols = dY.index_select(1, torch.as_tensor(ns, device="cuda")).cpu().numpy().astype(np.float64)
    xcols = X.index_select(1, torch.as_tensor(ks, device="cuda")).cpu().numpy().astype(np.float64)
    got = dW.cpu().numpy()[np.ix_(ns, ks)]
    assert rel_fro(got, gcols.T @ xcols) < TOL


def test_rmsnorm_bwd_sweep_32768x2048(ctx, orc, torch_cuda):
    """RMSNorm backward (exact gradient) at 32768 x 2048 against the oracle's
    (pkg/train/trainer.go:141-203 with the full RMSNorm derivative)."""
    torch = torch_cuda
    rows, cols = M_SWEEP, 2048
    x = dev_randn(torch, (rows, cols), 21)
    dy = dev_randn(torch, (rows, cols), 22)
    w = (1 + 0.1 * dev_randn(torch, (cols,), 23)).contiguous()
    xh, dyh, wh = x.cpu().numpy(), dy.cpu().numpy(), w.cpu().numpy()
    _, rms = orc.rmsnorm_fwd(xh, wh, 1e-5)
    ref_dx, ref_dw = orc.rmsnorm_bwd(xh, wh, rms, dyh, 1)
    d_rms = torch.as_tensor(rms, device="cuda")
    dx = torch.zeros((rows, cols), device="cuda")
    dxr = torch.empty((rows, cols), device="cuda")
    dw = torch.zeros((cols,), device="cuda")
    torch.cuda.synchronize()
    ctx.call("glc_rmsnorm_bwd", ptr(x), ptr(w), ptr(d_rms), ptr(dy), ptr(dx), ptr(dxr), ptr(dw), rows, cols, 1, 0, 0)
    ctx.sync()
    assert rel_fro(dx.cpu().numpy(), ref_dx) < FP32_RTOL
    assert rel_fro(dw.cpu().numpy(), ref_dw) < FP32_RTOL


@pytest.mark.parametrize("S,check_seqs", [(1024, (0, 1, 2, 3)), (2048, (0, 3))])
def test_attention_sweep_b4_h32_kv4(ctx, orc, S, check_seqs):
    """Causal attention forward and backward with grouped KV heads
    (pkg/train/trainer.go:323-389 with the head map of
    pkg/model/attention.go:118,149) at batch 4, 32/4 heads, head_dim 64."""
    B, H, Hkv, hd = 4, 32, 4, 64
    T = B * S
    r = np.random.default_rng(S + 5)
    q = tf32(r.standard_normal((T, H * hd), dtype=np.float32))
    k = tf32(r.standard_normal((T, Hkv * hd), dtype=np.float32))
    v = tf32(r.standard_normal((T, Hkv * hd), dtype=np.float32))
    dO = tf32(r.standard_normal((T, H * hd), dtype=np.float32))
    bq, bk, bv, bdo = ctx.from_numpy(q), ctx.from_numpy(k), ctx.from_numpy(v), ctx.from_numpy(dO)
    bo, blse = ctx.empty((T, H * hd)), ctx.empty((B, H, S))
    bdq, bdk, bdv = ctx.empty(q.shape), ctx.empty(k.shape), ctx.empty(v.shape)
    ctx.call("glc_attention_fwd", bq.ptr, bk.ptr, bv.ptr, bo.ptr, blse.ptr, B, S, H, Hkv, hd, 0)
    ctx.call("glc_attention_bwd", bq.ptr, bk.ptr, bv.ptr, bo.ptr, blse.ptr, bdo.ptr, bdq.ptr, bdk.ptr, bdv.ptr,
             B, S, H, Hkv, hd, 0)
    ctx.sync()
    sel = np.concatenate([np.arange(b * S, (b + 1) * S) for b in check_seqs])
    ref_o = orc.attention_fwd(q[sel], k[sel], v[sel], S, H, Hkv, hd)
    ref_dq, ref_dk, ref_dv = orc.attention_bwd(q[sel], k[sel], v[sel], dO[sel], S, H, Hkv, hd)
    errs = [rel_fro(bo.numpy()[sel], ref_o), rel_fro(bdq.numpy()[sel], ref_dq), rel_fro(bdk.numpy()[sel], ref_dk),
            rel_fro(bdv.numpy()[sel], ref_dv)]
    assert max(errs) < ATTN_TOL, errs


def test_softmax_ce_sweep_32768x32000(ctx, orc, torch_cuda):
    """SoftmaxCrossEntropyGrad (pkg/tensor/grad.go:210-280) on 32768 x 32000
    logits N(0, 2), uniform targets: the loss over every row, the gradient
    (p - onehot) / rows on 256 sampled rows."""
    torch = torch_cuda
    rows, V = M_SWEEP, 32000
    logits = dev_randn(torch, (rows, V), 31, std=2.0)
    g = torch.Generator(device="cuda").manual_seed(32)
    tg = torch.randint(0, V, (rows,), generator=g, device="cuda", dtype=torch.int64)
    lh, th = logits.cpu().numpy(), tg.cpu().numpy()
    logp = torch.empty((rows,), device="cuda")
    loss = torch.empty((1,), device="cuda")
    scale = np.float32(1.0) / np.float32(rows)
    torch.cuda.synchronize()
    ctx.call("glc_softmax_ce", ptr(logits), ptr(tg), rows, V, C.c_float(scale), ptr(logp), ptr(loss), 1, 0)
    ctx.sync()
    # the oracle's mean loss over chunks of rows, recombined into the mean over all
    chunk = 4096
    total = 0.0
    for r0 in range(0, rows, chunk):
        total += orc.softmax_ce(lh[r0 : r0 + chunk], th[r0 : r0 + chunk]) * min(chunk, rows - r0)
    ref_loss = total / rows
    got_loss = float(loss.cpu().numpy()[0])
    assert abs(got_loss - ref_loss) <= 1e-5 * abs(ref_loss), (got_loss, ref_loss)
    sel = sample(rows, 256, 33)
    _, probs = orc.softmax_ce(lh[sel], th[sel], want_probs=True)
    ref_g = probs.astype(np.float64) * float(scale)
    ref_g[np.arange(len(sel)), th[sel]] -= float(scale)
    got_g = logits.index_select(0, torch.as_tensor(sel, device="cuda")).cpu().numpy()
    assert rel_fro(got_g, ref_g) < 1e-5


def _quant_dx_full_size(ctx, torch, qtype, path):
    """dX[16384, 2048] = dY[16384, 5632] . deq(W[5632, 2048]) on the device;
    returns (dX sampled rows, the oracle's dequantize-then-matmul of them)."""
    M, K, N = 16384, 2048, 5632
    data = random_weight(qtype, N, K, 41 + qtype)
    src = np.frombuffer(data, np.uint8).copy()
    dY = dev_randn(torch, (M, N), 42 + qtype)
    dX = torch.empty((M, K), device="cuda")
    d_w = ctx.from_numpy(src)
    torch.cuda.synchronize()
    try:
        ctx.call("glc_set_quant_path", path)
        ctx.call("glc_linear_bwd_dx_q", ptr(dY), d_w.ptr, qtype, ptr(dX), M, K, N, 0)
        ctx.sync()
    finally:
        ctx.call("glc_set_quant_path", 0)
    rows = sample(M, 64, 43 + qtype)
    ridx = torch.as_tensor(rows, device="cuda")
    dyr = dY.index_select(0, ridx).cpu().numpy().astype(np.float64)
    want = np.zeros((len(rows), K), np.float64)
    # the reference's DequantizeQ8_0/Q4_0 (pkg/quant/dequant.go:68-137), then dA of MatMulGrad
    assert orc_lib().orcd_linear_bwd_dx_q(dyr.ctypes.data_as(C.c_void_p), src.ctypes.data_as(C.c_void_p), qtype,
                                          want.ctypes.data_as(C.c_void_p), len(rows), K, N) == 0
    return dX.index_select(0, ridx).cpu().numpy(), want


@pytest.mark.parametrize("qtype", [Q8_0, Q4_0], ids=["Q8_0", "Q4_0"])
def test_quant_dx_full_size(ctx, torch_cuda, qtype):
    got, want = _quant_dx_full_size(ctx, torch_cuda, qtype, 1)
    assert rel_fro(got, want) < TOL


@pytest.mark.parametrize("qtype", [Q8_0, Q4_0], ids=["Q8_0", "Q4_0"])
def test_quant_dx_full_size_fused_decode(ctx, torch_cuda, qtype):
    got, want = _quant_dx_full_size(ctx, torch_cuda, qtype, 2)
    assert rel_fro(got, want) < TOL
