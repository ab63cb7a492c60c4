"""tcgen05 TF32 GEMM (the three linear-layer products of MatMulGrad,
pkg/tensor/grad.go:81-152) against an fp64 numpy reference of the same fp32
inputs.  Tolerance: relative Frobenius error 2e-3 (TF32 operands, fp32
accumulation)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-3


def rel_fro(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


SHAPES = [
    (128, 32, 256),
    (256, 64, 512),
    (200, 72, 100),      # ragged in every dimension
    (64, 128, 344),      # tiny-config FFN width
    (512, 344, 128),     # K not a multiple of 32
    (1024, 512, 1376),
    (4096, 2048, 256),   # TinyLlama K/V projection (GQA)
]


@pytest.mark.parametrize("M,K,N", SHAPES)
def test_linear_fwd(ctx, M, K, N):
    rng = np.random.default_rng(M * 7 + K * 3 + N)
    X = rng.standard_normal((M, K), dtype=np.float32)
    W = rng.standard_normal((N, K), dtype=np.float32)
    dX, dW, dY = ctx.from_numpy(X), ctx.from_numpy(W), ctx.empty((M, N))
    ctx.call("glc_linear_fwd", dX.ptr, dW.ptr, dY.ptr, M, K, N, None)
    ctx.sync()
    ref = X.astype(np.float64) @ W.astype(np.float64).T
    assert rel_fro(dY.numpy(), ref) < TOL


@pytest.mark.parametrize("M,K,N", SHAPES)
def test_linear_fwd_residual(ctx, M, K, N):
    rng = np.random.default_rng(11 + M)
    X = rng.standard_normal((M, K), dtype=np.float32)
    W = rng.standard_normal((N, K), dtype=np.float32)
    R = rng.standard_normal((M, N), dtype=np.float32) * 10
    dX, dW, dR, dY = ctx.from_numpy(X), ctx.from_numpy(W), ctx.from_numpy(R), ctx.empty((M, N))
    ctx.call("glc_linear_fwd", dX.ptr, dW.ptr, dY.ptr, M, K, N, dR.ptr)
    ctx.sync()
    ref = X.astype(np.float64) @ W.astype(np.float64).T + R
    assert rel_fro(dY.numpy(), ref) < TOL


@pytest.mark.parametrize("M,K,N", SHAPES)
@pytest.mark.parametrize("accumulate", [0, 1])
def test_linear_bwd_dx(ctx, M, K, N, accumulate):
    rng = np.random.default_rng(5 + M + N)
    G = rng.standard_normal((M, N), dtype=np.float32)
    W = rng.standard_normal((N, K), dtype=np.float32)
    D0 = rng.standard_normal((M, K), dtype=np.float32)
    dG, dW, dD = ctx.from_numpy(G), ctx.from_numpy(W), ctx.from_numpy(D0)
    ctx.call("glc_linear_bwd_dx", dG.ptr, dW.ptr, dD.ptr, M, K, N, accumulate)
    ctx.sync()
    ref = G.astype(np.float64) @ W.astype(np.float64) + (D0 if accumulate else 0)
    assert rel_fro(dD.numpy(), ref) < TOL


@pytest.mark.parametrize("M,K,N", SHAPES)
@pytest.mark.parametrize("accumulate", [0, 1])
def test_linear_bwd_dw(ctx, M, K, N, accumulate):
    rng = np.random.default_rng(9 + K)
    G = rng.standard_normal((M, N), dtype=np.float32)
    X = rng.standard_normal((M, K), dtype=np.float32)
    D0 = rng.standard_normal((N, K), dtype=np.float32)
    dG, dX, dD = ctx.from_numpy(G), ctx.from_numpy(X), ctx.from_numpy(D0)
    ctx.call("glc_linear_bwd_dw", dG.ptr, dX.ptr, dD.ptr, M, K, N, accumulate)
    ctx.sync()
    ref = G.astype(np.float64).T @ X.astype(np.float64) + (D0 if accumulate else 0)
    assert rel_fro(dD.numpy(), ref) < TOL


def test_gemm_mn_major_a_k_major_b(ctx):
    """The fourth operand-major combination (A MN-major, B K-major)."""
    M, N, K = 300, 260, 96
    rng = np.random.default_rng(3)
    At = rng.standard_normal((K, M), dtype=np.float32)  # A stored [K][M]
    B = rng.standard_normal((N, K), dtype=np.float32)
    dA, dB, dC = ctx.from_numpy(At), ctx.from_numpy(B), ctx.empty((M, N))
    ctx.call("glc_gemm_tf32", dA.ptr, M, 1, dB.ptr, K, 0, dC.ptr, N, M, N, K, 0, None, 0, 0)
    ctx.sync()
    ref = At.T.astype(np.float64) @ B.astype(np.float64).T
    assert rel_fro(dC.numpy(), ref) < TOL


def test_tf32_operand_rounding_probe(ctx):
    """Records how the tensor core treats fp32 bits below the TF32 mantissa:
    A = 1 + 0.75 ulp(tf32) is seen as 1 (truncation) or 1 + 2^-10 (rounding)."""
    M, N, K = 128, 256, 32
    a = np.float32(1.0 + 3 * 2.0**-12)
    A = np.full((M, K), a, np.float32)
    B = np.ones((N, K), np.float32)
    dA, dB, dC = ctx.from_numpy(A), ctx.from_numpy(B), ctx.empty((M, N))
    ctx.call("glc_linear_fwd", dA.ptr, dB.ptr, dC.ptr, M, K, N, None)
    ctx.sync()
    v = float(dC.numpy()[0, 0])
    assert v in (32.0, 32.0 * (1 + 2.0**-10)), v
    print(f"\nTF32 operand handling: {'truncation' if v == 32.0 else 'round-to-nearest'} (C = {v!r})")


def test_gemm_rejects_misaligned(ctx):
    from gollama_b200.device import GlcError

    X = ctx.empty((4, 6))
    W = ctx.empty((4, 6))
    Y = ctx.empty((4, 4))
    with pytest.raises(GlcError):
        ctx.call("glc_linear_fwd", X.ptr, W.ptr, Y.ptr, 4, 6, 4, None)


@pytest.mark.parametrize("M,K,N", [(4096, 2048, 256), (200, 72, 100), (1024, 512, 1376)])
def test_linear_bwd_grouped(ctx, M, K, N):
    """dX and dW of one MatMulGrad GradFn in one grouped launch."""
    rng = np.random.default_rng(M + K)
    G = rng.standard_normal((M, N), dtype=np.float32)
    X = rng.standard_normal((M, K), dtype=np.float32)
    W = rng.standard_normal((N, K), dtype=np.float32)
    dX0 = rng.standard_normal((M, K), dtype=np.float32)
    dG, dXa, dWa = ctx.from_numpy(G), ctx.from_numpy(X), ctx.from_numpy(W)
    ddx, ddw = ctx.from_numpy(dX0), ctx.empty((N, K))
    ctx.call("glc_linear_bwd", dG.ptr, dXa.ptr, dWa.ptr, ddx.ptr, ddw.ptr, M, K, N, 1, 0)
    ctx.sync()
    G64 = G.astype(np.float64)
    assert rel_fro(ddx.numpy(), G64 @ W.astype(np.float64) + dX0) < TOL
    assert rel_fro(ddw.numpy(), G64.T @ X.astype(np.float64)) < TOL


@pytest.mark.parametrize("variant", [1, 2])
@pytest.mark.parametrize("M,K,N", [(64, 96, 200), (200, 72, 100), (384, 256, 640), (1024, 512, 1376)])
def test_gemm_variants_all_majors(ctx, variant, M, K, N):
    """Single-CTA (1) and CTA-pair (2) tiles on the forward, dX and dW
    products, with ragged edges and with row counts that leave the second CTA
    of a pair without rows."""
    rng = np.random.default_rng(variant * 1000 + M + K + N)
    X = rng.standard_normal((M, K), dtype=np.float32)
    W = rng.standard_normal((N, K), dtype=np.float32)
    G = rng.standard_normal((M, N), dtype=np.float32)
    D0 = rng.standard_normal((M, K), dtype=np.float32)
    dX, dW, dG = ctx.from_numpy(X), ctx.from_numpy(W), ctx.from_numpy(G)
    Y, gX, gW = ctx.empty((M, N)), ctx.from_numpy(D0), ctx.empty((N, K))
    ctx.call("glc_set_gemm_variant", variant)
    try:
        ctx.call("glc_linear_fwd", dX.ptr, dW.ptr, Y.ptr, M, K, N, None)
        ctx.call("glc_linear_bwd", dG.ptr, dX.ptr, dW.ptr, gX.ptr, gW.ptr, M, K, N, 1, 0)
        ctx.sync()
    finally:
        ctx.call("glc_set_gemm_variant", 0)
    X64, W64, G64 = X.astype(np.float64), W.astype(np.float64), G.astype(np.float64)
    assert rel_fro(Y.numpy(), X64 @ W64.T) < TOL
    assert rel_fro(gX.numpy(), G64 @ W64 + D0) < TOL
    assert rel_fro(gW.numpy(), G64.T @ X64) < TOL


def test_gemm_variant_rejects_unknown(ctx):
    from gollama_b200.device import GlcError

    with pytest.raises(GlcError):
        ctx.call("glc_set_gemm_variant", 3)


@pytest.mark.parametrize("variant", [0, 1])
@pytest.mark.parametrize("M,K,F", [(64, 64, 344), (256, 128, 344), (300, 256, 1376), (4096, 2048, 5632)])
def test_linear_fwd_swiglu_matches_separate_ops(ctx, variant, M, K, F):
    """glc_linear_fwd_swiglu (SwiGLU in the GEMM epilogue on CTA pairs; GEMM then
    the SwiGLU kernel otherwise) equals glc_linear_fwd followed by
    glc_swiglu_fwd bit for bit."""
    rng = np.random.default_rng(M + K + F)
    X = rng.standard_normal((M, K), dtype=np.float32)
    W = (rng.standard_normal((2 * F, K), dtype=np.float32) * 0.1).astype(np.float32)
    dX, dW = ctx.from_numpy(X), ctx.from_numpy(W)
    gu, h = ctx.empty((M, 2 * F)), ctx.empty((M, F))
    ctx.call("glc_set_gemm_variant", variant)
    try:
        ctx.call("glc_linear_fwd_swiglu", dX.ptr, dW.ptr, gu.ptr, h.ptr, M, K, F, 1)
        y = ctx.empty((M, 2 * F))
        ctx.call("glc_linear_fwd", dX.ptr, dW.ptr, y.ptr, M, K, 2 * F, None)
        ctx.sync()
    finally:
        ctx.call("glc_set_gemm_variant", 0)
    ref_gu = y.numpy()
    assert np.array_equal(gu.numpy().view(np.uint32), ref_gu.view(np.uint32))
    g, u = ctx.from_numpy(np.ascontiguousarray(ref_gu[:, :F])), ctx.from_numpy(np.ascontiguousarray(ref_gu[:, F:]))
    h2 = ctx.empty((M, F))
    ctx.call("glc_swiglu_fwd", g.ptr, u.ptr, h2.ptr, M * F, 1)
    ctx.sync()
    assert np.array_equal(h.numpy().view(np.uint32), h2.numpy().view(np.uint32))


@pytest.mark.parametrize("M,K,N", [(384, 256, 640), (1024, 512, 1376), (4096, 2048, 2560), (4096, 5632, 2048),
                                   (300, 72, 100)])
def test_gemm_dynamic_order_bit_identical(ctx, M, K, N):
    """glc_set_gemm_schedule(2): CTA pairs take tiles from a counter; the
    forward, the grouped dX + dW launch and a SwiGLU-epilogue launch give
    the same bits as the fixed order, over more launches than one pass of
    the counter ring would need to be cleared."""
    rng = np.random.default_rng(M + 3 * K + N)
    X = rng.standard_normal((M, K), dtype=np.float32)
    W = rng.standard_normal((N, K), dtype=np.float32)
    G = rng.standard_normal((M, N), dtype=np.float32)
    D0 = rng.standard_normal((M, K), dtype=np.float32)
    dX, dW, dG = ctx.from_numpy(X), ctx.from_numpy(W), ctx.from_numpy(G)
    outs = []
    try:
        ctx.call("glc_set_gemm_variant", 2)
        for mode in (1, 2):
            ctx.call("glc_set_gemm_schedule", mode)
            Y, gX, gW = ctx.empty((M, N)), ctx.from_numpy(D0), ctx.empty((N, K))
            ctx.call("glc_linear_fwd", dX.ptr, dW.ptr, Y.ptr, M, K, N, None)
            ctx.call("glc_linear_bwd", dG.ptr, dX.ptr, dW.ptr, gX.ptr, gW.ptr, M, K, N, 1, 0)
            if mode == 2:
                for _ in range(3):  # wrap the ring of tile counters (1024 launches) once
                    for _ in range(400):
                        ctx.call("glc_linear_fwd", dX.ptr, dW.ptr, Y.ptr, M, K, N, None)
                    ctx.sync()
            ctx.sync()
            outs.append([a.numpy().view(np.uint32) for a in (Y, gX, gW)])
    finally:
        ctx.call("glc_set_gemm_schedule", 0)
        ctx.call("glc_set_gemm_variant", 0)
    for a, b in zip(*outs):
        assert np.array_equal(a, b)
