"""Each CUDA op through the C ABI against the oracle's restatement of the
reference op (oracle/oracle.c), on seeded inputs."""
import ctypes as C

import numpy as np
import pytest

from oracle.oracle import Oracle
from tests.helpers import FP32_RTOL, rel_fro, threads

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def orc():
    return Oracle(threads=threads())


def rng(seed):
    return np.random.default_rng(seed)


@pytest.mark.parametrize("rows,cols", [(1, 128), (257, 128), (1000, 512), (4096, 2048), (3, 8192)])
def test_rmsnorm_fwd(ctx, orc, rows, cols):
    r = rng(rows + cols)
    x = r.standard_normal((rows, cols), dtype=np.float32)
    w = (1 + 0.1 * r.standard_normal(cols)).astype(np.float32)
    ref_y, ref_rms = orc.rmsnorm_fwd(x, w, 1e-5)
    dx, dw, dy, drms = ctx.from_numpy(x), ctx.from_numpy(w), ctx.empty((rows, cols)), ctx.empty((rows,))
    ctx.call("glc_rmsnorm_fwd", dx.ptr, dw.ptr, dy.ptr, drms.ptr, rows, cols, C.c_float(1e-5), 0)
    ctx.sync()
    assert rel_fro(drms.numpy(), ref_rms) < 1e-6
    assert rel_fro(dy.numpy(), ref_y) < 1e-6


@pytest.mark.parametrize("full", [0, 1])
@pytest.mark.parametrize("rows,cols", [(5, 128), (300, 512), (2048, 2048)])
def test_rmsnorm_bwd(ctx, orc, rows, cols, full):
    r = rng(rows * 3 + full)
    x = r.standard_normal((rows, cols), dtype=np.float32)
    w = (1 + 0.1 * r.standard_normal(cols)).astype(np.float32)
    g = r.standard_normal((rows, cols), dtype=np.float32)
    dx0 = r.standard_normal((rows, cols), dtype=np.float32)
    dw0 = r.standard_normal(cols).astype(np.float32)
    _, rms = orc.rmsnorm_fwd(x, w, 1e-5)
    ref_dx, ref_dw = orc.rmsnorm_bwd(x, w, rms, g, full, dx=dx0.copy(), dw=dw0.copy())
    bx, bw, brms, bg = ctx.from_numpy(x), ctx.from_numpy(w), ctx.from_numpy(rms), ctx.from_numpy(g)
    bdx, bdw, bdxr = ctx.from_numpy(dx0), ctx.from_numpy(dw0), ctx.empty((rows, cols))
    ctx.call("glc_rmsnorm_bwd", bx.ptr, bw.ptr, brms.ptr, bg.ptr, bdx.ptr, bdxr.ptr, bdw.ptr, rows, cols, full, 1, 1)
    ctx.sync()
    out_dx = bdx.numpy()
    assert rel_fro(out_dx, ref_dx) < FP32_RTOL
    assert rel_fro(bdw.numpy(), ref_dw) < FP32_RTOL
    # the rounded copy is dx rounded to TF32 (10 mantissa bits)
    assert np.max(np.abs(bdxr.numpy() - out_dx) / (np.abs(out_dx) + 1e-30)) <= 2.0**-11


@pytest.mark.parametrize("variant", [1, 3])
@pytest.mark.parametrize("acc", [0, 1])
@pytest.mark.parametrize("rows,cols", [(5, 128), (300, 512), (3, 1028), (4096, 2048), (1000, 2052), (9, 2048)])
def test_rmsnorm_bwd_exact_variants(ctx, orc, rows, cols, acc, variant):
    """The exact backward through the row-by-row kernel (1) and the
    bulk-copy pipeline (3, the default for the exact gradient; more rows per
    block than its four stages, partial last blocks, rows wider than it
    takes fall back) against the oracle."""
    r = rng(rows * 7 + cols + acc)
    x = r.standard_normal((rows, cols), dtype=np.float32)
    w = (1 + 0.1 * r.standard_normal(cols)).astype(np.float32)
    g = r.standard_normal((rows, cols), dtype=np.float32)
    dx0 = r.standard_normal((rows, cols), dtype=np.float32) if acc else np.zeros((rows, cols), np.float32)
    _, rms = orc.rmsnorm_fwd(x, w, 1e-5)
    ref_dx, ref_dw = orc.rmsnorm_bwd(x, w, rms, g, 1, dx=dx0.copy())
    try:
        ctx.call("glc_set_rmsnorm_variant", variant)
        bx, bw, brms, bg = ctx.from_numpy(x), ctx.from_numpy(w), ctx.from_numpy(rms), ctx.from_numpy(g)
        bdx, bdw, bdxr = ctx.from_numpy(dx0), ctx.zeros((cols,)), ctx.empty((rows, cols))
        ctx.call("glc_rmsnorm_bwd", bx.ptr, bw.ptr, brms.ptr, bg.ptr, bdx.ptr, bdxr.ptr, bdw.ptr, rows, cols, 1, acc, 0)
        ctx.sync()
    finally:
        ctx.call("glc_set_rmsnorm_variant", 0)
    out_dx = bdx.numpy()
    assert rel_fro(out_dx, ref_dx) < FP32_RTOL
    assert rel_fro(bdw.numpy(), ref_dw) < FP32_RTOL
    assert np.max(np.abs(bdxr.numpy() - out_dx) / (np.abs(out_dx) + 1e-30)) <= 2.0**-11


@pytest.mark.parametrize("full,acc", [(0, 0), (1, 1), (1, 0)])
@pytest.mark.parametrize("rows,cols", [(5, 128), (300, 512), (4096, 2048), (1000, 2052)])
def test_rmsnorm_bwd_pipelined_bit_identical(ctx, rows, cols, full, acc):
    """glc_set_rmsnorm_variant(2) (cp.async-pipelined rows) returns the same
    bits as the row-by-row kernel; 2052 columns fall back to it."""
    r = rng(rows + cols + full)
    x = r.standard_normal((rows, cols), dtype=np.float32)
    w = (1 + 0.1 * r.standard_normal(cols)).astype(np.float32)
    g = r.standard_normal((rows, cols), dtype=np.float32)
    dx0 = r.standard_normal((rows, cols), dtype=np.float32)
    dw0 = r.standard_normal(cols).astype(np.float32)
    rms = np.sqrt((x.astype(np.float64) ** 2).mean(1) + 1e-5).astype(np.float32)
    outs = []
    try:
        for variant in (1, 2):
            ctx.call("glc_set_rmsnorm_variant", variant)
            bx, bw, brms, bg = ctx.from_numpy(x), ctx.from_numpy(w), ctx.from_numpy(rms), ctx.from_numpy(g)
            bdx, bdw, bdxr = ctx.from_numpy(dx0), ctx.from_numpy(dw0), ctx.empty((rows, cols))
            ctx.call("glc_rmsnorm_bwd", bx.ptr, bw.ptr, brms.ptr, bg.ptr, bdx.ptr, bdxr.ptr, bdw.ptr, rows, cols, full,
                     acc, 1)
            ctx.sync()
            outs.append([a.numpy().view(np.uint32) for a in (bdx, bdxr, bdw)])
    finally:
        ctx.call("glc_set_rmsnorm_variant", 0)
    for a, b in zip(*outs):
        assert np.array_equal(a, b)


def test_rmsnorm_simplified_matches_reference_formula(ctx):
    """Reference-mode backward is exactly dx = dy*w/rms, dw = sum dy*x/rms (trainer.go:186-198)."""
    rows, cols = 64, 128
    r = rng(1)
    x = r.standard_normal((rows, cols), dtype=np.float32)
    w = r.standard_normal(cols).astype(np.float32)
    g = r.standard_normal((rows, cols), dtype=np.float32)
    rms = np.sqrt((x.astype(np.float64) ** 2).mean(1) + 1e-5).astype(np.float32)
    bx, bw, brms, bg = ctx.from_numpy(x), ctx.from_numpy(w), ctx.from_numpy(rms), ctx.from_numpy(g)
    bdx, bdw = ctx.zeros((rows, cols)), ctx.zeros((cols,))
    ctx.call("glc_rmsnorm_bwd", bx.ptr, bw.ptr, brms.ptr, bg.ptr, bdx.ptr, None, bdw.ptr, rows, cols, 0, 0, 0)
    ctx.sync()
    ref_dx = (g * w[None, :]) / rms[:, None]
    assert np.array_equal(bdx.numpy(), ref_dx.astype(np.float32))


@pytest.mark.parametrize("n", [4, 4096, 1 << 20])
def test_swiglu_fwd_bit_exact(ctx, orc, n):
    """silu(g)*u with the reference's exp32 must be bit-identical to the oracle."""
    r = rng(n)
    g = (r.standard_normal(n) * 4).astype(np.float32)
    g[:4] = [0.0, -88.5, 90.0, -20.0][: min(4, n)]
    u = r.standard_normal(n).astype(np.float32)
    gs, sig = orc.silu_fwd(g)
    ref = gs * u
    bg, bu, bh = ctx.from_numpy(g), ctx.from_numpy(u), ctx.empty((n,))
    ctx.call("glc_swiglu_fwd", bg.ptr, bu.ptr, bh.ptr, n, 0)
    ctx.sync()
    assert np.array_equal(bh.numpy(), ref)


@pytest.mark.parametrize("n", [4096, 1 << 20])
def test_swiglu_bwd_bit_exact(ctx, orc, n):
    r = rng(n + 1)
    g = (r.standard_normal(n) * 4).astype(np.float32)
    u = r.standard_normal(n).astype(np.float32)
    dh = r.standard_normal(n).astype(np.float32)
    gs, sig = orc.silu_fwd(g)
    # product node then SiLU, as in the reference's reverse topological order
    dgs = dh * u
    dup = dh * gs
    dgate = orc.silu_bwd(g, sig, dgs)
    bg, bu, bdh = ctx.from_numpy(g), ctx.from_numpy(u), ctx.from_numpy(dh)
    bdg, bdu = ctx.empty((n,)), ctx.empty((n,))
    ctx.call("glc_swiglu_bwd", bg.ptr, bu.ptr, bdh.ptr, bdg.ptr, bdu.ptr, n, 0, 0)
    ctx.sync()
    assert np.array_equal(bdu.numpy(), dup)
    assert np.array_equal(bdg.numpy(), dgate)


@pytest.mark.parametrize("rows,V", [(7, 256), (512, 32000), (64, 1000), (33, 8196), (300, 16384), (7, 16388),
                                    (16, 40000)])
@pytest.mark.parametrize("write_grad", [0, 1])
@pytest.mark.parametrize("variant", [0, 2])
def test_softmax_ce(ctx, orc, rows, V, write_grad, variant):
    """glc_set_ce_variant: 0 (automatic: one-shot clusters for the reference's
    arithmetic) and 2 (rows streamed through persistent CTAs, 8192 < V <=
    32768), both against the oracle; at or below V = 8192, and above 32768,
    the variants share a kernel."""
    if variant and not 8192 < V <= 32768:
        pytest.skip("one kernel for both variants at this vocabulary")
    r = rng(rows + V)
    logits = (r.standard_normal((rows, V)) * 2).astype(np.float32)
    tg = r.integers(0, V, rows).astype(np.int64)
    tg[0] = -1          # ignored target: no loss, still counted in the mean
    if rows > 1:
        tg[1] = V + 5   # out of range: ignored too
    ref_loss, probs = orc.softmax_ce(logits, tg, want_probs=True)
    bl, bt = ctx.from_numpy(logits), ctx.from_numpy(tg)
    blogp, bloss = ctx.empty((rows,)), ctx.empty((1,))
    scale = np.float32(1.0) / np.float32(rows)
    try:
        ctx.call("glc_set_ce_variant", variant)
        ctx.call("glc_softmax_ce", bl.ptr, bt.ptr, rows, V, C.c_float(scale), blogp.ptr, bloss.ptr, write_grad, 0)
        ctx.sync()
    finally:
        ctx.call("glc_set_ce_variant", 0)
    loss = float(bloss.numpy()[0])
    assert abs(loss - ref_loss) <= 1e-5 * abs(ref_loss)
    if write_grad:
        ref_g = orc.softmax_ce_grad(probs, tg)
        assert rel_fro(bl.numpy(), ref_g) < 1e-5
        # rows of the CE gradient sum to zero when the target is valid
        assert np.abs(bl.numpy()[2:].sum(1)).max() < 1e-5


@pytest.mark.parametrize("rows,V", [(7, 256), (512, 32000), (33, 8196), (7, 16388), (16, 40000)])
@pytest.mark.parametrize("variant", [0, 1])
@pytest.mark.parametrize("round_out", [0, 1])
def test_softmax_ce_llama(ctx, rows, V, variant, round_out):
    """glc_softmax_ce_llama (expf/logf, reciprocal multiply: the Llama-mode
    step's loss) against float64 softmax cross-entropy, with an ignored and
    an out-of-range target; round_out=1 rounds the gradient to TF32."""
    if variant and not 8192 < V <= 32768:
        pytest.skip("one kernel for both variants at this vocabulary")
    r = rng(3 * rows + V)
    logits = (r.standard_normal((rows, V)) * 2).astype(np.float32)
    tg = r.integers(0, V, rows).astype(np.int64)
    tg[0] = -1
    tg[1] = V + 5
    x = logits.astype(np.float64)
    e = np.exp(x - x.max(1, keepdims=True))
    p = e / e.sum(1, keepdims=True)
    ok = (tg >= 0) & (tg < V)
    idx = np.arange(rows)[ok]
    scale = np.float32(1.0) / np.float32(rows)
    ref_loss = -np.log(p[idx, tg[ok]] + 1e-10).sum() / rows
    ref_g = p * float(scale)
    ref_g[idx, tg[ok]] -= float(scale)
    bl, bt = ctx.from_numpy(logits), ctx.from_numpy(tg)
    blogp, bloss = ctx.empty((rows,)), ctx.empty((1,))
    try:
        ctx.call("glc_set_ce_variant", variant)
        ctx.call("glc_softmax_ce_llama", bl.ptr, bt.ptr, rows, V, C.c_float(scale), blogp.ptr, bloss.ptr, 1, round_out)
        ctx.sync()
    finally:
        ctx.call("glc_set_ce_variant", 0)
    loss = float(bloss.numpy()[0])
    assert abs(loss - ref_loss) <= 2e-5 * abs(ref_loss), (loss, ref_loss)
    g = bl.numpy()
    assert rel_fro(g, ref_g) < (1e-3 if round_out else 1e-5)
    if round_out:
        assert not np.any(g.view(np.uint32) & 0x1FFF)


def test_rope_matches_oracle_and_inverts(ctx, orc):
    T, S, nh, hd = 256, 64, 4, 64
    r = rng(2)
    x = r.standard_normal((T, nh * hd), dtype=np.float32)
    ct, st = orc.rope_table(hd, S, 10000.0)
    ch, sh = np.zeros_like(ct), np.zeros_like(st)
    assert ctx.lib.glc_rope_table(hd, S, C.c_float(10000.0), ch.ctypes.data_as(C.c_void_p),
                                  sh.ctypes.data_as(C.c_void_p)) == 0
    assert np.array_equal(ch, ct) and np.array_equal(sh, st)
    bx, bc, bs = ctx.from_numpy(x), ctx.from_numpy(ct), ctx.from_numpy(st)
    ctx.call("glc_rope", bx.ptr, T, S, nh, hd, bc.ptr, bs.ptr, 0, 0)
    ctx.sync()
    ref = orc.rope_apply(x, S, nh, hd, ct, st)
    assert np.array_equal(bx.numpy(), ref)
    ctx.call("glc_rope", bx.ptr, T, S, nh, hd, bc.ptr, bs.ptr, 1, 0)
    ctx.sync()
    ref_inv = orc.rope_apply(ref, S, nh, hd, ct, st, inverse=True)
    assert np.array_equal(bx.numpy(), ref_inv)
    assert rel_fro(bx.numpy(), x) < 1e-6


def tf32(x):
    """Round to the nearest TF32 value (ties away from zero), as the kernels
    that produce tensor-core operands do."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((b + np.uint32(0x1000)) & np.uint32(0xFFFFE000)).view(np.float32)


ATTN_TOL = 2e-3  # TF32 tensor-core attention (P and dS rounded to TF32) vs the fp32 oracle


@pytest.mark.parametrize("B,S,H,Hkv,hd", [(2, 64, 4, 4, 32), (1, 100, 4, 2, 64), (2, 256, 8, 4, 64), (1, 130, 2, 1, 32),
                                          (1, 1024, 4, 1, 64), (3, 200, 2, 2, 64)])
def test_attention_fwd_bwd(ctx, orc, B, S, H, Hkv, hd):
    T = B * S
    r = rng(T + H)
    q = tf32(r.standard_normal((T, H * hd), dtype=np.float32))
    k = tf32(r.standard_normal((T, Hkv * hd), dtype=np.float32))
    v = tf32(r.standard_normal((T, Hkv * hd), dtype=np.float32))
    dO = tf32(r.standard_normal((T, H * hd), dtype=np.float32))
    ref_o = orc.attention_fwd(q, k, v, S, H, Hkv, hd)
    ref_dq, ref_dk, ref_dv = orc.attention_bwd(q, k, v, dO, S, H, Hkv, hd)
    bq, bk, bv, bdo = ctx.from_numpy(q), ctx.from_numpy(k), ctx.from_numpy(v), ctx.from_numpy(dO)
    bo, blse = ctx.empty((T, H * hd)), ctx.empty((B, H, S))
    ctx.call("glc_attention_fwd", bq.ptr, bk.ptr, bv.ptr, bo.ptr, blse.ptr, B, S, H, Hkv, hd, 0)
    bdq, bdk, bdv = ctx.empty(q.shape), ctx.empty(k.shape), ctx.empty(v.shape)
    ctx.call("glc_attention_bwd", bq.ptr, bk.ptr, bv.ptr, bo.ptr, blse.ptr, bdo.ptr, bdq.ptr, bdk.ptr, bdv.ptr,
             B, S, H, Hkv, hd, 0)
    ctx.sync()
    errs = [rel_fro(bo.numpy(), ref_o), rel_fro(bdq.numpy(), ref_dq), rel_fro(bdk.numpy(), ref_dk),
            rel_fro(bdv.numpy(), ref_dv)]
    assert max(errs) < ATTN_TOL, errs


@pytest.mark.parametrize("B,S,H,Hkv,hd", [(1, 128, 2, 1, 64), (2, 300, 4, 2, 64), (4, 1024, 32, 4, 64),
                                          (3, 257, 3, 3, 32), (1, 2048, 8, 8, 64)])
def test_attention_fwd_persistent_bit_identical(ctx, B, S, H, Hkv, hd):
    """glc_set_attention_fwd_variant(2) (one persistent CTA per SM, pipelines
    running across work items) returns the grid kernel's O and LSE bit for bit."""
    T = B * S
    r = rng(T + H + hd)
    q = tf32(r.standard_normal((T, H * hd), dtype=np.float32))
    k = tf32(r.standard_normal((T, Hkv * hd), dtype=np.float32))
    v = tf32(r.standard_normal((T, Hkv * hd), dtype=np.float32))
    bq, bk, bv = ctx.from_numpy(q), ctx.from_numpy(k), ctx.from_numpy(v)
    outs = []
    try:
        for variant in (1, 2):
            ctx.call("glc_set_attention_fwd_variant", variant)
            bo, blse = ctx.empty((T, H * hd)), ctx.empty((B, H, S))
            ctx.call("glc_attention_fwd", bq.ptr, bk.ptr, bv.ptr, bo.ptr, blse.ptr, B, S, H, Hkv, hd, 0)
            ctx.sync()
            outs.append((bo.numpy().view(np.uint32), blse.numpy().view(np.uint32)))
    finally:
        ctx.call("glc_set_attention_fwd_variant", 0)
    assert np.array_equal(outs[0][0], outs[1][0])
    assert np.array_equal(outs[0][1], outs[1][1])


@pytest.mark.parametrize("B,S,H,Hkv,hd", [(1, 128, 2, 1, 64), (2, 300, 4, 2, 64), (4, 1024, 32, 4, 64),
                                          (3, 257, 3, 3, 32)])
def test_attention_dq_persistent_bit_identical(ctx, B, S, H, Hkv, hd):
    """glc_set_attention_dq_variant(2) and (3): dQ bit for bit as the grid kernel's
    (dK and dV come from the unchanged kernel)."""
    T = B * S
    r = rng(T + 2 * H + hd)
    q = tf32(r.standard_normal((T, H * hd), dtype=np.float32))
    k = tf32(r.standard_normal((T, Hkv * hd), dtype=np.float32))
    v = tf32(r.standard_normal((T, Hkv * hd), dtype=np.float32))
    dO = tf32(r.standard_normal((T, H * hd), dtype=np.float32))
    bq, bk, bv, bdo = ctx.from_numpy(q), ctx.from_numpy(k), ctx.from_numpy(v), ctx.from_numpy(dO)
    bo, blse = ctx.empty((T, H * hd)), ctx.empty((B, H, S))
    ctx.call("glc_attention_fwd", bq.ptr, bk.ptr, bv.ptr, bo.ptr, blse.ptr, B, S, H, Hkv, hd, 0)
    outs = []
    try:
        for variant in (1, 2, 3):
            ctx.call("glc_set_attention_dq_variant", variant)
            bdq, bdk, bdv = ctx.empty(q.shape), ctx.empty(k.shape), ctx.empty(v.shape)
            ctx.call("glc_attention_bwd", bq.ptr, bk.ptr, bv.ptr, bo.ptr, blse.ptr, bdo.ptr, bdq.ptr, bdk.ptr, bdv.ptr,
                     B, S, H, Hkv, hd, 0)
            ctx.sync()
            outs.append([a.numpy().view(np.uint32) for a in (bdq, bdk, bdv)])
    finally:
        ctx.call("glc_set_attention_dq_variant", 0)
    for other in outs[1:]:
        for a, b_ in zip(outs[0], other):
            assert np.array_equal(a, b_)


@pytest.mark.parametrize("B,S,H,Hkv,hd,split", [(1, 128, 2, 1, 64, 0), (2, 300, 4, 2, 64, 0), (4, 1024, 32, 4, 64, 0),
                                                (4, 1024, 32, 4, 64, 1), (3, 257, 3, 3, 32, 0), (1, 64, 2, 2, 64, 0),
                                                (2, 200, 8, 2, 32, 4)])
def test_attention_dkdv_two_groups_bit_identical(ctx, B, S, H, Hkv, hd, split):
    """glc_set_attention_dkdv_variant(2): dK and dV bit for bit as the
    one-group kernel's, for every split of the query-head group (split 0:
    automatic) and a single-step CTA (S = 64: the second group idles)."""
    T = B * S
    r = rng(T + 3 * H + hd + split)
    q = tf32(r.standard_normal((T, H * hd), dtype=np.float32))
    k = tf32(r.standard_normal((T, Hkv * hd), dtype=np.float32))
    v = tf32(r.standard_normal((T, Hkv * hd), dtype=np.float32))
    dO = tf32(r.standard_normal((T, H * hd), dtype=np.float32))
    bq, bk, bv, bdo = ctx.from_numpy(q), ctx.from_numpy(k), ctx.from_numpy(v), ctx.from_numpy(dO)
    bo, blse = ctx.empty((T, H * hd)), ctx.empty((B, H, S))
    ctx.call("glc_attention_fwd", bq.ptr, bk.ptr, bv.ptr, bo.ptr, blse.ptr, B, S, H, Hkv, hd, 0)
    outs = []
    try:
        ctx.call("glc_set_attention_split", split)
        for variant in (1, 2):
            ctx.call("glc_set_attention_dkdv_variant", variant)
            bdq, bdk, bdv = ctx.empty(q.shape), ctx.empty(k.shape), ctx.empty(v.shape)
            ctx.call("glc_attention_bwd", bq.ptr, bk.ptr, bv.ptr, bo.ptr, blse.ptr, bdo.ptr, bdq.ptr, bdk.ptr, bdv.ptr,
                     B, S, H, Hkv, hd, 0)
            ctx.sync()
            outs.append([a.numpy().view(np.uint32) for a in (bdq, bdk, bdv)])
    finally:
        ctx.call("glc_set_attention_dkdv_variant", 0)
        ctx.call("glc_set_attention_split", 0)
    for a, b_ in zip(*outs):
        assert np.array_equal(a, b_)


@pytest.mark.parametrize("nsplit", [1, 2, 4, 3])
def test_attention_bwd_group_splits(ctx, orc, nsplit):
    """dK/dV with the 4 query heads of each KV head over 1, 2 or 4 CTAs (3 is
    not a divisor and falls back to the automatic choice): every split
    against the oracle, and dq unchanged bit for bit."""
    B, S, H, Hkv, hd = 2, 384, 8, 2, 64
    T = B * S
    r = rng(77)
    q = tf32(r.standard_normal((T, H * hd), dtype=np.float32))
    k = tf32(r.standard_normal((T, Hkv * hd), dtype=np.float32))
    v = tf32(r.standard_normal((T, Hkv * hd), dtype=np.float32))
    dO = tf32(r.standard_normal((T, H * hd), dtype=np.float32))
    ref_dq, ref_dk, ref_dv = orc.attention_bwd(q, k, v, dO, S, H, Hkv, hd)
    bq, bk, bv, bdo = ctx.from_numpy(q), ctx.from_numpy(k), ctx.from_numpy(v), ctx.from_numpy(dO)
    bo, blse = ctx.empty((T, H * hd)), ctx.empty((B, H, S))
    ctx.call("glc_attention_fwd", bq.ptr, bk.ptr, bv.ptr, bo.ptr, blse.ptr, B, S, H, Hkv, hd, 0)
    outs = []
    try:
        for split in (0, nsplit):
            ctx.call("glc_set_attention_split", split)
            bdq, bdk, bdv = ctx.empty(q.shape), ctx.empty(k.shape), ctx.empty(v.shape)
            ctx.call("glc_attention_bwd", bq.ptr, bk.ptr, bv.ptr, bo.ptr, blse.ptr, bdo.ptr, bdq.ptr, bdk.ptr,
                     bdv.ptr, B, S, H, Hkv, hd, 0)
            ctx.sync()
            outs.append((bdq.numpy(), bdk.numpy(), bdv.numpy()))
    finally:
        ctx.call("glc_set_attention_split", 0)
    dq, dk, dv = outs[1]
    errs = [rel_fro(dq, ref_dq), rel_fro(dk, ref_dk), rel_fro(dv, ref_dv)]
    assert max(errs) < ATTN_TOL, errs
    assert np.array_equal(dq, outs[0][0])
    assert rel_fro(dk, outs[0][1]) < 1e-5 and rel_fro(dv, outs[0][2]) < 1e-5


def test_embedding_fwd_bwd(ctx):
    V, d, B, S = 50, 64, 3, 20
    T = B * S
    r = rng(9)
    E = r.standard_normal((V, d), dtype=np.float32)
    P = r.standard_normal((S, d), dtype=np.float32)
    tok = r.integers(0, V, T).astype(np.int64)
    tok[3], tok[7] = -2, V + 1  # clamped to id 0 (trainer.go:280-282)
    clamped = np.where((tok < 0) | (tok >= V), 0, tok)
    bt, bE, bP, bo = ctx.from_numpy(tok), ctx.from_numpy(E), ctx.from_numpy(P), ctx.empty((T, d))
    ctx.call("glc_embed_fwd", bt.ptr, bE.ptr, bP.ptr, bo.ptr, T, S, d, V)
    ctx.sync()
    ref = E[clamped] + P[np.arange(T) % S]
    assert np.array_equal(bo.numpy(), ref)
    dh = r.standard_normal((T, d), dtype=np.float32)
    dE0 = r.standard_normal((V, d), dtype=np.float32)
    bdh, bdE = ctx.from_numpy(dh), ctx.from_numpy(dE0)
    ctx.call("glc_embed_bwd", tok.ctypes.data_as(C.c_void_p), T, bdh.ptr, bdE.ptr, d, V)
    ctx.sync()
    want = dE0.copy()
    for t in range(T):  # dE[tok] += dh[t], t ascending
        want[clamped[t]] += dh[t]
    assert np.array_equal(bdE.numpy(), want)


@pytest.mark.parametrize("d", [2048, 2052])
def test_embedding_bwd_hot_ids(ctx, d):
    """Zipf-like ids: one id holds 301 rows (a ragged tail of 8-row batches),
    rows of d/4 float4 columns spread over several column blocks; the sum per
    id stays in ascending t, bit for bit."""
    V, T = 4000, 1200
    r = rng(10)
    tok = r.integers(0, V, T).astype(np.int64)
    tok[r.choice(T, 301, replace=False)] = 17
    tok[r.choice(np.flatnonzero(tok != 17), 9, replace=False)] = 3
    dh = r.standard_normal((T, d), dtype=np.float32)
    dE0 = r.standard_normal((V, d), dtype=np.float32)
    bdh, bdE = ctx.from_numpy(dh), ctx.from_numpy(dE0)
    ctx.call("glc_embed_bwd", tok.ctypes.data_as(C.c_void_p), T, bdh.ptr, bdE.ptr, d, V)
    ctx.sync()
    want = dE0.copy()
    for t in range(T):
        want[tok[t]] += dh[t]
    assert np.array_equal(bdE.numpy(), want)


@pytest.mark.parametrize("V,T,hot", [(256, 1, False), (256, 5000, True), (32000, 4096, True), (70000, 3001, False),
                                     (40, 2049, True), (2, 1024, False)])
def test_embedding_bwd_device_segments_bit_identical(ctx, V, T, hot):
    """glc_embed_bwd_device sorts the positions by id on the device (one to
    three radix passes here, partial last tiles, out-of-range ids clamped to
    0): the scatter is bit-identical to glc_embed_bwd's host-built segments."""
    d = 64
    r = rng(V + T)
    tok = r.integers(-3, V + 3, T).astype(np.int64)
    if hot:
        tok[r.choice(T, T // 3, replace=False)] = 7 % V
    dh = r.standard_normal((T, d), dtype=np.float32)
    dE0 = r.standard_normal((V, d), dtype=np.float32)
    outs = []
    for name in ("glc_embed_bwd", "glc_embed_bwd_device"):
        bt, bdh, bdE = ctx.from_numpy(tok), ctx.from_numpy(dh), ctx.from_numpy(dE0)
        src = tok.ctypes.data_as(C.c_void_p) if name == "glc_embed_bwd" else bt.ptr
        ctx.call(name, src, T, bdh.ptr, bdE.ptr, d, V)
        ctx.sync()
        outs.append(bdE.numpy().view(np.uint32))
    assert np.array_equal(outs[0], outs[1])
    if T <= 2049:
        clamped = np.where((tok < 0) | (tok >= V), 0, tok)
        want = dE0.copy()
        for t in range(T):  # dE[tok] += dh[t], t ascending
            want[clamped[t]] += dh[t]
        assert np.array_equal(outs[1], want.view(np.uint32))


def test_round_tf32(ctx):
    x = np.array([1.0 + 3 * 2.0**-12, 1.0 + 2.0**-12, -(1.0 + 3 * 2.0**-12), 3.0e-39, 1.0e30], np.float32)
    x = np.concatenate([x, np.zeros(3, np.float32)])
    bx, by = ctx.from_numpy(x), ctx.empty(x.shape)
    ctx.call("glc_round_tf32", bx.ptr, by.ptr, x.size)
    ctx.sync()
    y = by.numpy()
    assert y[0] == np.float32(1.0 + 2.0**-10)
    assert y[2] == -np.float32(1.0 + 2.0**-10)
    bits = y.view(np.uint32)
    assert np.all(bits & 0x1FFF == 0)


def adamw_reference(p, g, m, v, lr, b1, b2, eps, wd, step, scale):
    """AdamW.Step (pkg/train/optimizer.go:37-76) in numpy with Go's types:
    float32 moments and parameters, float64 bias correction and update."""
    f32 = np.float32
    if scale != 1.0:
        g = (g * f32(scale)).astype(f32)
    m = f32(b1) * m + (f32(1) - f32(b1)) * g
    v = f32(b2) * v + ((f32(1) - f32(b2)) * g) * g
    bc1 = 1.0 - np.float64(f32(b1)) ** step
    bc2 = 1.0 - np.float64(f32(b2)) ** step
    upd = (m.astype(np.float64) / bc1 / (np.sqrt(v.astype(np.float64) / bc2) + np.float64(f32(eps)))).astype(f32)
    p = p - f32(lr) * (upd + f32(wd) * p)
    return p, g, m, v


@pytest.mark.parametrize("step", [1, 7])
def test_clip_and_adamw_bit_exact(ctx, step):
    n = 1 << 22
    r = rng(step)
    p = (r.standard_normal(n) * 0.02).astype(np.float32)
    g = (r.standard_normal(n) * np.exp(r.uniform(-12, 2, n))).astype(np.float32)
    g[:16] = 0.0
    m = (r.standard_normal(n) * 1e-3).astype(np.float32) if step > 1 else np.zeros(n, np.float32)
    v = (np.abs(r.standard_normal(n)) * 1e-6).astype(np.float32) if step > 1 else np.zeros(n, np.float32)
    segs = np.array([0, n // 2, n // 2 + 64, n // 2 - 64], np.int64)  # two segments, a 64-float hole
    bp, bg, bm, bv, bs = ctx.from_numpy(p), ctx.from_numpy(g), ctx.from_numpy(m), ctx.from_numpy(v), ctx.empty((n,))
    dnorm, dscale = ctx.empty((1,), np.float64), ctx.empty((1,))
    ctx.call("glc_grad_clip_norm", bg.ptr, segs.ctypes.data_as(C.c_void_p), 2, C.c_float(1.0), dnorm.ptr, dscale.ptr)
    ctx.call("glc_adamw_step", bp.ptr, bg.ptr, bm.ptr, bv.ptr, bs.ptr, segs.ctypes.data_as(C.c_void_p), 2, dscale.ptr,
             C.c_float(3e-4), C.c_float(0.9), C.c_float(0.95), C.c_float(1e-8), C.c_float(0.1), step)
    ctx.sync()
    sel = np.r_[0 : n // 2, n // 2 + 64 : n]
    norm = float(np.sqrt(np.sum(g[sel].astype(np.float64) ** 2)))
    assert abs(dnorm.numpy()[0] - norm) <= 1e-12 * norm
    scale = np.float32(1.0 / norm) if np.float32(norm) > 1.0 else np.float32(1.0)
    assert dscale.numpy()[0] == scale
    rp, rg, rm, rv = adamw_reference(p[sel], g[sel], m[sel], v[sel], 3e-4, 0.9, 0.95, 1e-8, 0.1, step, float(scale))
    out_p, out_g, out_m, out_v = bp.numpy(), bg.numpy(), bm.numpy(), bv.numpy()
    assert np.array_equal(out_m[sel], rm) and np.array_equal(out_v[sel], rv)
    assert np.array_equal(out_g[sel], rg)
    assert np.array_equal(out_p[sel], rp)
    hole = slice(n // 2, n // 2 + 64)
    assert np.array_equal(out_p[hole], p[hole]) and np.array_equal(out_g[hole], g[hole])
    sh = bs.numpy()[sel]
    assert np.all(sh.view(np.uint32) & 0x1FFF == 0)
    assert np.max(np.abs(sh - rp) / np.maximum(np.abs(rp), 1e-30)) <= 2.0**-11


def test_exp32_bit_exact_against_oracle(ctx):
    """The device exp32 equals the oracle's restatement of the reference's
    exp32 bit for bit: a strided sweep over every float bit pattern in
    [-88.5, 88.5], random arguments, and the edges (subnormal results,
    saturation, infinities, zeros).  The reference's _exp keeps only two
    polynomial terms (exp32(1) = 2.718261, not e), so a more accurate
    exponential would fail here."""
    from oracle.oracle import lib

    top = np.float32(88.5).view(np.uint32)
    pos = np.arange(0, int(top), 97, dtype=np.uint32)
    sweep = np.concatenate([pos, pos | np.uint32(0x80000000)]).view(np.float32)
    rnd = np.random.default_rng(7).uniform(-90.0, 90.0, 1 << 22).astype(np.float32)
    edges = np.array([0.0, -0.0, -87.0, np.nextafter(np.float32(-87.0), np.float32(-100)), 88.0,
                      np.nextafter(np.float32(88.0), np.float32(100)), -88.0,
                      np.nextafter(np.float32(-88.0), np.float32(-100)), -100.0, 100.0, 1e-30, -1e-30, 1e-45,
                      -1e-45, np.inf, -np.inf, 0.6931472, -0.6931472, 1.0, -1.0], dtype=np.float32)
    x = np.ascontiguousarray(np.concatenate([sweep, rnd, edges]))
    want = np.empty_like(x)
    lib().orc_exp32_array(x.ctypes.data_as(C.c_void_p), want.ctypes.data_as(C.c_void_p), C.c_int64(x.size))
    dx, dy = ctx.from_numpy(x), ctx.empty(x.shape)
    ctx.call("glc_exp32", dx.ptr, dy.ptr, x.size)
    ctx.sync()
    got = dy.numpy()
    bad = np.nonzero(got.view(np.uint32) != want.view(np.uint32))[0]
    assert bad.size == 0, f"{bad.size} mismatches, first x={x[bad[:5]]} got={got[bad[:5]]} want={want[bad[:5]]}"
