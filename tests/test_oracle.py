"""The CPU oracle (oracle/oracle.c) checked on its own.

The reference ships no golden vectors, so the restatement is pinned by:
known answers read off the Go source, closed forms, bit-identity between the
reference-structured (literal) loops and the fast loops, and finite
differences of the Llama-mode backward in float64.
"""
import math

import numpy as np
import pytest

from gollama_b200 import synthetic as syn
from oracle.oracle import Config, Oracle, OptimState, TrainState
from tests.helpers import oracle_config, oracle_optim, rel_fro


@pytest.fixture(scope="module")
def o32():
    return Oracle(double=False, threads=4)


@pytest.fixture(scope="module")
def o64():
    return Oracle(double=True, threads=4)


# ------------------------------------------------------------------ GEMMs
@pytest.mark.parametrize("M,K,N", [(1, 13, 9), (7, 19, 5), (33, 64, 17), (16, 40, 24)])
def test_matmul_literal_and_fast_loops_bit_identical(M, K, N):
    r = np.random.default_rng(M * K * N)
    a = r.standard_normal((M, K), dtype=np.float32)
    b = r.standard_normal((N, K), dtype=np.float32)
    dc = r.standard_normal((M, N), dtype=np.float32)
    lit = Oracle(threads=1, literal=True)
    fast = Oracle(threads=3, literal=False)
    assert np.array_equal(lit.matmul_transpose_b(a, b), fast.matmul_transpose_b(a, b))
    da0 = r.standard_normal((M, K), dtype=np.float32)
    assert np.array_equal(lit.matmul_grad_da(dc, b, da0.copy()), fast.matmul_grad_da(dc, b, da0.copy()))
    db0 = r.standard_normal((N, K), dtype=np.float32)
    assert np.array_equal(lit.matmul_grad_db(dc, a, db0.copy()), fast.matmul_grad_db(dc, a, db0.copy()))


def test_matmul_transpose_b_uses_eight_partial_sums(o32):
    """dotProduct (matmul.go:237-259): sums 8 strided partials, then s0+...+s7, then the tail."""
    K = 19
    r = np.random.default_rng(0)
    a = r.standard_normal((1, K), dtype=np.float32)
    b = r.standard_normal((1, K), dtype=np.float32)
    s = [np.float32(0)] * 8
    k = 0
    while k <= K - 8:
        for j in range(8):
            s[j] = np.float32(s[j] + np.float32(a[0, k + j] * b[0, k + j]))
        k += 8
    tot = np.float32(0)
    for j in range(8):
        tot = np.float32(tot + s[j]) if j else s[0]
    for kk in range(k, K):
        tot = np.float32(tot + np.float32(a[0, kk] * b[0, kk]))
    assert o32.matmul_transpose_b(a, b)[0, 0] == tot


def test_matmul_grads_match_numpy(o64):
    r = np.random.default_rng(1)
    dc, b, a = r.standard_normal((9, 7)), r.standard_normal((7, 5)), r.standard_normal((9, 5))
    assert np.allclose(o64.matmul_grad_da(dc, b), dc @ b)
    assert np.allclose(o64.matmul_grad_db(dc, a), dc.T @ a)


# ------------------------------------------------------------------ exp / log of grad.go
def test_go_exp_known_answers(o32):
    L = o32.L
    assert L.orc_go_exp(0.0) == 1.0
    assert L.orc_exp32(-88.5) == 0.0              # grad.go:285-287
    assert L.orc_exp32(88.5) == np.float32(3.4e38)  # grad.go:288-290
    xs = np.linspace(-20, 20, 4001)
    rel = max(abs(L.orc_go_exp(float(x)) - math.exp(x)) / math.exp(x) for x in xs)
    # the reference's polynomial is truncated and one coefficient has the
    # wrong sign: its relative error is about 1.4e-5, not ~1e-16
    assert 5e-6 < rel < 3e-5, rel


def test_go_log_accuracy(o32):
    L = o32.L
    xs = np.geomspace(1e-10, 4.0, 2000)
    err = max(abs(L.orc_go_log(float(x)) - math.log(x)) for x in xs)
    assert err < 1e-6, err
    assert L.orc_go_log(0.0) == -1e100 and L.orc_go_log(-1.0) == -1e100


# ------------------------------------------------------------------ RMSNorm
def test_rmsnorm_forward_formula(o32):
    r = np.random.default_rng(2)
    x = r.standard_normal((5, 16), dtype=np.float32)
    w = r.standard_normal(16).astype(np.float32)
    y, rms = o32.rmsnorm_fwd(x, w, 1e-5)
    ss = np.zeros(5, np.float32)
    for j in range(16):
        ss = (ss + x[:, j] * x[:, j]).astype(np.float32)
    want_rms = np.sqrt(ss.astype(np.float64) / 16 + np.float64(np.float32(1e-5))).astype(np.float32)
    assert np.array_equal(rms, want_rms)
    assert np.array_equal(y, (x / want_rms[:, None]) * w[None, :])


def test_rmsnorm_simplified_backward_is_reference_formula(o32):
    r = np.random.default_rng(3)
    x = r.standard_normal((4, 8), dtype=np.float32)
    w = r.standard_normal(8).astype(np.float32)
    g = r.standard_normal((4, 8), dtype=np.float32)
    _, rms = o32.rmsnorm_fwd(x, w)
    dx, dw = o32.rmsnorm_bwd(x, w, rms, g, full=False)
    assert np.array_equal(dx, (g * w) / rms[:, None])


def test_rmsnorm_full_backward_finite_differences(o64):
    r = np.random.default_rng(4)
    x = r.standard_normal((3, 12))
    w = r.standard_normal(12)
    g = r.standard_normal((3, 12))
    _, rms = o64.rmsnorm_fwd(x, w)
    dx, dw = o64.rmsnorm_bwd(x, w, rms, g, full=True)
    f = lambda xx, ww: float((o64.rmsnorm_fwd(xx, ww)[0] * g).sum())
    h = 1e-6
    for i, j in [(0, 0), (1, 5), (2, 11)]:
        xp, xm = x.copy(), x.copy()
        xp[i, j] += h
        xm[i, j] -= h
        assert abs((f(xp, w) - f(xm, w)) / (2 * h) - dx[i, j]) < 1e-6
    for j in [0, 7]:
        wp, wm = w.copy(), w.copy()
        wp[j] += h
        wm[j] -= h
        assert abs((f(x, wp) - f(x, wm)) / (2 * h) - dw[j]) < 1e-6


# ------------------------------------------------------------------ softmax CE
def test_softmax_ce_rows_and_ignored_targets(o32):
    r = np.random.default_rng(5)
    logits = (r.standard_normal((6, 30)) * 2).astype(np.float32)
    tg = np.array([1, 2, -1, 40, 0, 29], np.int64)
    loss, p = o32.softmax_ce(logits, tg, want_probs=True)
    assert np.allclose(p.sum(1), 1, atol=1e-6)
    valid = [0, 1, 4, 5]
    ref = -np.log(p[valid, tg[valid]].astype(np.float64) + 1e-10).sum() / 6  # ignored rows count in N
    assert abs(loss - ref) < 1e-5 * abs(ref)
    g = o32.softmax_ce_grad(p, tg)
    assert np.allclose(g[valid].sum(1), 0, atol=1e-7)
    assert np.allclose(g[[2, 3]], p[[2, 3]] / 6)  # no onehot for ignored targets


# ------------------------------------------------------------------ RoPE
def test_rope_consecutive_pairs_and_inverse(o64):
    T, S, nh, hd = 6, 3, 2, 8
    r = np.random.default_rng(6)
    x = r.standard_normal((T, nh * hd))
    c, s = o64.rope_table(hd, S, 10000.0)
    y = o64.rope_apply(x, S, nh, hd, c, s)
    z = x.reshape(T, nh, hd // 2, 2)
    cz = z[..., 0] + 1j * z[..., 1]
    pos = np.arange(T) % S
    ang = pos[:, None] * (1.0 / 10000.0 ** (2 * np.arange(hd // 2) / hd))[None, :]
    want = cz * np.exp(1j * ang)[:, None, :]
    got = y.reshape(T, nh, hd // 2, 2)
    assert np.allclose(got[..., 0] + 1j * got[..., 1], want)
    assert np.allclose(o64.rope_apply(y, S, nh, hd, c, s, inverse=True), x)


# ------------------------------------------------------------------ attention
def softmax_attention_ref(q, k, v, S, H, Hkv, hd):
    T = q.shape[0]
    B = T // S
    out = np.zeros_like(q)
    for b in range(B):
        for h in range(H):
            kh = h // (H // Hkv)
            Q = q[b * S:(b + 1) * S, h * hd:(h + 1) * hd]
            K = k[b * S:(b + 1) * S, kh * hd:(kh + 1) * hd]
            Vv = v[b * S:(b + 1) * S, kh * hd:(kh + 1) * hd]
            s = Q @ K.T / math.sqrt(hd)
            s += np.triu(np.full((S, S), -np.inf), 1)
            p = np.exp(s - s.max(1, keepdims=True))
            p /= p.sum(1, keepdims=True)
            out[b * S:(b + 1) * S, h * hd:(h + 1) * hd] = p @ Vv
    return out


def test_attention_forward_gqa(o64):
    B, S, H, Hkv, hd = 2, 7, 4, 2, 8
    r = np.random.default_rng(7)
    q, k, v = (r.standard_normal((B * S, n * hd)) for n in (H, Hkv, Hkv))
    assert np.allclose(o64.attention_fwd(q, k, v, S, H, Hkv, hd), softmax_attention_ref(q, k, v, S, H, Hkv, hd))


def test_attention_backward_finite_differences(o64):
    B, S, H, Hkv, hd = 1, 5, 4, 2, 4
    r = np.random.default_rng(8)
    q, k, v = (r.standard_normal((B * S, n * hd)) for n in (H, Hkv, Hkv))
    g = r.standard_normal((B * S, H * hd))
    dq, dk, dv = o64.attention_bwd(q, k, v, g, S, H, Hkv, hd)
    f = lambda qq, kk, vv: float((o64.attention_fwd(qq, kk, vv, S, H, Hkv, hd) * g).sum())
    h = 1e-6
    for arr, grad in ((q, dq), (k, dk), (v, dv)):
        for idx in [(0, 0), (3, 5), (4, arr.shape[1] - 1)]:
            a0 = arr[idx]
            arr[idx] = a0 + h
            fp = f(q, k, v)
            arr[idx] = a0 - h
            fm = f(q, k, v)
            arr[idx] = a0
            assert abs((fp - fm) / (2 * h) - grad[idx]) < 1e-6


# ------------------------------------------------------------------ optimizer
def test_adamw_first_step_closed_form(o32):
    """Step 1: m^ = g, v^ = g^2, so update = g/(|g|+eps) (optimizer.go:58-73)."""
    shape = syn.TINY.with_(layers=1, vocab=16, hidden=8, heads=2, inter=8, seq=4, batch=1)
    cfg = oracle_config(shape)
    n = o32.param_total(cfg)
    r = np.random.default_rng(9)
    p0 = r.standard_normal(n).astype(np.float32)
    g = r.standard_normal(n).astype(np.float32)
    st = TrainState.create(p0, len(o32.param_layout(cfg)), oracle_optim())
    st.has_grad[:] = 1
    st.opt.lr = np.float32(1e-3)
    import ctypes as C
    o32.fn("adamw_step")(st.params.ctypes.data_as(C.c_void_p), g.ctypes.data_as(C.c_void_p),
                         st.has_grad.ctypes.data_as(C.c_void_p), st.m.ctypes.data_as(C.c_void_p),
                         st.v.ctypes.data_as(C.c_void_p), C.byref(cfg), C.byref(st.opt))
    upd = (g.astype(np.float64) / (np.abs(g.astype(np.float64)) + 1e-8))
    want = p0 - np.float32(1e-3) * (upd.astype(np.float32) + np.float32(0.1) * p0)
    assert np.allclose(st.params, want, rtol=0, atol=1e-6)


def test_lr_schedule(o32):
    st = OptimState(initial_lr=np.float32(3e-4), warmup_steps=100, total_steps=1000)
    assert o32.get_lr(st, 0) == 0.0
    assert o32.get_lr(st, 50) == np.float32(np.float32(3e-4) * np.float32(50)) / np.float32(100)
    assert abs(o32.get_lr(st, 100) - 3e-4) < 1e-10
    assert abs(o32.get_lr(st, 550) - 3e-4 * 0.5) < 1e-9


# ------------------------------------------------------------------ whole model
MICRO = syn.ModelShape("micro", 2, 16, 4, 2, 24, 20, 6, 2, mode=1)


@pytest.mark.parametrize("mode", [0, 1])
def test_model_fp32_matches_fp64(o32, o64, mode):
    shape = MICRO.with_(mode=mode, kv_heads=2 if mode else 4)
    cfg = oracle_config(shape)
    p = syn.init_params(shape, 3).astype(np.float64) * 5
    p[np.isclose(syn.init_params(shape, 3), 1.0)] = 1.0
    inp, tg = syn.batch(shape, 3)
    l32, g32, h32 = o32.forward_backward(cfg, p.astype(np.float32), inp, tg)
    l64, g64, h64 = o64.forward_backward(cfg, p, inp, tg)
    assert np.array_equal(h32, h64)
    assert abs(l32 - l64) < 1e-5 * abs(l64)
    assert rel_fro(g32, g64) < 1e-4


def test_llama_mode_gradients_finite_differences(o64):
    shape = MICRO
    cfg = oracle_config(shape)
    p = syn.init_params(shape, 11).astype(np.float64)
    scale = np.where(p == 1.0, 1.0, 10.0)  # larger weights so every path matters
    p = np.where(p == 1.0, 1.0 + 0.1 * np.sin(np.arange(p.size)), p * scale)
    inp, tg = syn.batch(shape, 11)
    loss, g, has = o64.forward_backward(cfg, p, inp, tg)
    assert has.all()
    layout = o64.param_layout(cfg)
    r = np.random.default_rng(0)
    h = 1e-6
    for off, rows, cols in layout:
        for i in r.choice(rows * cols, size=min(3, rows * cols), replace=False):
            j = off + int(i)
            pp, pm = p.copy(), p.copy()
            pp[j] += h
            pm[j] -= h
            fd = (o64.forward_backward(cfg, pp, inp, tg, backward=False)[0]
                  - o64.forward_backward(cfg, pm, inp, tg, backward=False)[0]) / (2 * h)
            assert abs(fd - g[j]) < 1e-6 + 1e-5 * abs(fd), (off, rows, cols, i, fd, g[j])


def test_reference_mode_token_embedding_grad_rows_equal(o32):
    """Ones seed (grad.go:45-50) + tied head: dE = ones^T . hF, every row identical."""
    shape = MICRO.with_(mode=0, kv_heads=4)
    cfg = oracle_config(shape)
    p = syn.init_params(shape, 2)
    inp, tg = syn.batch(shape, 2)
    _, g, has = o32.forward_backward(cfg, p, inp, tg)
    off, V, d = o32.param_layout(cfg)[0]
    dE = g[off:off + V * d].reshape(V, d)
    assert np.array_equal(dE, np.broadcast_to(dE[0], dE.shape))


@pytest.mark.parametrize("mode", [0, 1])
def test_data_parallel_sum_equals_global_batch(o64, mode):
    """Splitting the batch over W ranks and summing their gradients gives the
    single-process gradient: ones seed sums (reference), the CE mean needs a
    1/W factor per rank (Llama: each rank seeds 1/(W*T_rank))."""
    shape = MICRO.with_(mode=mode, kv_heads=2 if mode else 4, batch=4)
    cfg = oracle_config(shape)
    p = syn.init_params(shape, 4).astype(np.float64)
    inp, tg = syn.batch(shape, 4)
    _, g_all, _ = o64.forward_backward(cfg, p, inp, tg)
    W = 2
    acc = np.zeros_like(g_all)
    for rk in range(W):
        sl = slice(rk * 2, rk * 2 + 2)
        _, g, _ = o64.forward_backward(cfg, p, inp[sl], tg[sl])
        acc += g / (W if mode == 1 else 1)
    assert rel_fro(acc, g_all) < 1e-12


def test_train_step_state(o32):
    shape = MICRO.with_(mode=0, kv_heads=4)
    cfg = oracle_config(shape)
    p = syn.init_params(shape, 6)
    inp, tg = syn.batch(shape, 6)
    st = TrainState.create(p, len(o32.param_layout(cfg)), oracle_optim())
    loss, norm = o32.train_step(cfg, st, inp, tg)
    assert st.opt.trainer_step == 1 and st.opt.adam_step == 1
    assert norm > 1.0  # ones-seeded gradients are large: clipping is active
    clipped = float(np.sqrt(np.sum(st.grads.astype(np.float64) ** 2)))
    assert abs(clipped - 1.0) < 1e-4
    assert math.isfinite(loss)


@pytest.mark.parametrize("shape", [syn.TINY, syn.TINY_LLAMA_MODE], ids=lambda s: s.name)
def test_scalar_build_bit_identical(shape):
    """oracle/liboracle_scalar.so (built like Go's amd64 code, which the CPU
    baseline times) computes the same bits as the test build: a whole step in
    reference-structured (literal) threading, loss, gradients and weights."""
    params = syn.init_params(shape, 4)
    inputs, targets = syn.batch(shape, 4)
    outs = []
    for scalar in (False, True):
        orc = Oracle(threads=2, literal=True, scalar=scalar)
        cfg = oracle_config(shape)
        st = TrainState.create(params, len(orc.param_layout(cfg)), oracle_optim())
        loss, norm = orc.train_step(cfg, st, inputs, targets)
        outs.append((loss, norm, st.grads.copy(), st.params.copy()))
    (l0, n0, g0, p0), (l1, n1, g1, p1) = outs
    assert l0 == l1 and n0 == n1
    assert np.array_equal(g0.view(np.uint32), g1.view(np.uint32))
    assert np.array_equal(p0.view(np.uint32), p1.view(np.uint32))
