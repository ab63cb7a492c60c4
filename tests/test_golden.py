"""The oracle against golden vectors of the reference's own arithmetic: the
float32 exponential and logarithm (pkg/tensor/grad.go:283-381), the linear
layer's products (pkg/tensor/matmul.go:145-259, grad.go:81-152), RoPE
(pkg/model/rope.go), SiLU
(grad.go:417-449), RMSNorm with its simplified gradient
(pkg/train/trainer.go:141-203), softmax cross-entropy (grad.go:210-280),
AdamW's cast sequence (pkg/train/optimizer.go:37-76) and one whole TrainStep
in reference semantics (pkg/train/trainer.go:462-505) on a micro model.

tests/golden/go_arith.json is written by tests/golden/make_golden.py, a
plain-Python restatement of the reference's `_exp` / `_log` made separately
from the C oracle (oracle/oracle.c) and the device code.  The oracle must
reproduce every vector bit for bit (the device code is checked against the
oracle on a sweep in tests/test_ops_gpu.py)."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle.oracle import lib

GOLDEN = json.loads((Path(__file__).parent / "golden" / "go_arith.json").read_text())


def f32(bits: int) -> np.float32:
    return np.array([bits], np.uint32).view(np.float32)[0]


def b32(v: float) -> int:
    return int(np.array([v], np.float32).view(np.uint32)[0])


@pytest.mark.parametrize("kind", ["exp32", "log32"])
def test_oracle_matches_golden_bits(kind):
    fn = getattr(lib(), "orc_" + kind)
    bad = [(hex(x), hex(y), hex(b32(fn(float(f32(x)))))) for x, y in GOLDEN[kind] if b32(fn(float(f32(x)))) != y]
    assert not bad, bad[:5]
    assert len(GOLDEN[kind]) > 2000


def test_oracle_go_exp_float64_matches_golden():
    fn = lib().orc_go_exp
    for x, y in GOLDEN["go_exp"]:
        assert fn(x) == y, (x, fn(x), y)


def test_oracle_adamw_matches_golden_bits():
    """Five AdamW.Step calls (optimizer.go:37-76) on 96 parameters padded into
    a micro model's arena: p, m and v bit for bit after every step."""
    import ctypes as C

    from gollama_b200 import synthetic as syn
    from oracle.oracle import Oracle, TrainState
    from tests.helpers import oracle_config, oracle_optim

    gd = GOLDEN["adamw"]
    o = Oracle(threads=1)
    shape = syn.TINY.with_(layers=1, vocab=16, hidden=8, heads=2, inter=8, seq=4, batch=1)
    cfg = oracle_config(shape)
    n_all = o.param_total(cfg)
    n = len(gd["p0"])
    assert n_all >= n
    p0 = np.zeros(n_all, np.float32)
    p0[:n] = np.array(gd["p0"], np.uint32).view(np.float32)
    st = TrainState.create(p0, len(o.param_layout(cfg)), oracle_optim())
    st.has_grad[:] = 1
    st.opt.lr, st.opt.beta1, st.opt.beta2 = np.float32(gd["lr"]), np.float32(gd["beta1"]), np.float32(gd["beta2"])
    st.opt.eps, st.opt.weight_decay = np.float32(gd["eps"]), np.float32(gd["weight_decay"])
    for g_bits, want in zip(gd["grads"], gd["after"]):
        g = np.zeros(n_all, np.float32)
        g[:n] = np.array(g_bits, np.uint32).view(np.float32)
        o.fn("adamw_step")(st.params.ctypes.data_as(C.c_void_p), g.ctypes.data_as(C.c_void_p),
                           st.has_grad.ctypes.data_as(C.c_void_p), st.m.ctypes.data_as(C.c_void_p),
                           st.v.ctypes.data_as(C.c_void_p), C.byref(cfg), C.byref(st.opt))
        for key, arr in (("p", st.params), ("m", st.m), ("v", st.v)):
            assert np.array_equal(arr[:n].view(np.uint32), np.array(want[key], np.uint32)), key


def arr(key_bits, shape=None):
    a = np.array(key_bits, np.uint32).view(np.float32)
    return a.reshape(shape) if shape else a


def same(a, b_bits):
    return np.array_equal(np.ascontiguousarray(a, np.float32).reshape(-1).view(np.uint32), np.array(b_bits, np.uint32))


@pytest.mark.parametrize("literal", [True, False])
def test_oracle_matmul_matches_golden_bits(literal):
    """MatMulTransposeB with dotProduct's eight partial sums and MatMulGrad's
    dA/dB loops, in the oracle's reference-structured and fast loops."""
    from oracle.oracle import Oracle

    o, gd = Oracle(threads=3, literal=literal), GOLDEN["matmul"]
    a, b, dc = arr(gd["a"], (5, 21)), arr(gd["b"], (7, 21)), arr(gd["dc"], (5, 7))
    assert same(o.matmul_transpose_b(a, b), gd["c"])
    assert same(o.matmul_grad_da(dc, b, arr(gd["da0"], (5, 21)).copy()), gd["da"])
    assert same(o.matmul_grad_db(dc, a, arr(gd["db0"], (7, 21)).copy()), gd["db"])


def test_oracle_rope_matches_golden_bits():
    """RoPE tables and the consecutive-pair rotation (pkg/model/rope.go)."""
    from oracle.oracle import Oracle

    o, gd = Oracle(threads=1), GOLDEN["rope"]
    ct, st = o.rope_table(gd["dim"], gd["max_seq"], gd["theta"])
    assert same(ct, gd["cos"]) and same(st, gd["sin"])
    y = o.rope_apply(arr(gd["x"], (12, 24)), gd["max_seq"], gd["heads"], gd["dim"], ct, st)
    assert same(y, gd["y"])


def test_oracle_gqa_attention_forward_matches_golden_bits():
    """The trainer's attention arithmetic (trainer.go:329-382) with the KV-head
    map of pkg/model/attention.go:118,149."""
    from oracle.oracle import Oracle

    o, gd = Oracle(threads=2), GOLDEN["attention_gqa"]
    q, k, v = arr(gd["q"], (12, 16)), arr(gd["k"], (12, 8)), arr(gd["v"], (12, 8))
    assert same(o.attention_fwd(q, k, v, gd["S"], gd["H"], gd["Hkv"], gd["hd"]), gd["o"])


def test_oracle_silu_matches_golden_bits():
    from oracle.oracle import Oracle

    o, gd = Oracle(threads=1), GOLDEN["silu"]
    x = arr(gd["x"])
    y, sig = o.silu_fwd(x)
    assert same(y, gd["y"])
    assert same(o.silu_bwd(x, sig, arr(gd["dy"])), gd["dx"])


def test_oracle_rmsnorm_matches_golden_bits():
    from oracle.oracle import Oracle

    o, gd = Oracle(threads=1), GOLDEN["rmsnorm"]
    x, w = arr(gd["x"], (6, 64)), arr(gd["w"])
    y, rms = o.rmsnorm_fwd(x, w, gd["eps"])
    assert same(y, gd["y"]) and same(rms, gd["rms"])
    dx, dw = o.rmsnorm_bwd(x, w, rms, arr(gd["dout"], (6, 64)), 0)
    assert same(dx, gd["dx"]) and same(dw, gd["dw"])


def test_oracle_softmax_ce_matches_golden_bits():
    from oracle.oracle import Oracle

    o, gd = Oracle(threads=1), GOLDEN["softmax_ce"]
    lg = arr(gd["logits"], (6, 100))
    loss, probs = o.softmax_ce(lg, gd["targets"], want_probs=True)
    assert b32(loss) == gd["loss"]
    assert same(o.softmax_ce_grad(probs, gd["targets"]), gd["grad"])


def test_oracle_reference_train_step_matches_golden_bits():
    """TrainStep in reference semantics on a micro model (2 layers, d 8, 2
    heads, FFN 12, vocab 11, two sequences of 5 with out-of-range ids and
    ignored targets): the loss, which parameters have a gradient, every
    clipped gradient, every weight and AdamW moment after the step, bit for
    bit against the separate restatement (tests/golden/ref_step.py)."""
    from oracle.oracle import Config, Oracle, OptimState, TrainState

    gd = GOLDEN["ref_step"]
    c, hp = gd["config"], gd["hparams"]
    cfg = Config(vocab=c["vocab"], hidden=c["hidden"], layers=c["layers"], heads=c["heads"], kv_heads=c["heads"],
                 inter=c["inter"], max_seq=c["seq"], norm_eps=c["norm_eps"], rope_theta=10000.0, mode=0)
    o = Oracle(threads=2)
    layout = o.param_layout(cfg)
    assert [(r_, c_) for _, r_, c_ in layout] == [tuple(s) for s in gd["shapes"]]
    params = np.concatenate([arr(p) for p in gd["params"]])
    opt = OptimState(lr=0.0, beta1=hp["beta1"], beta2=hp["beta2"], eps=hp["eps"], weight_decay=hp["wd"], adam_step=0,
                     initial_lr=hp["lr"], warmup_steps=hp["warmup"], total_steps=hp["total_steps"],
                     grad_clip=hp["clip"], trainer_step=0)
    st = TrainState.create(params, len(layout), opt)
    loss, _ = o.train_step(cfg, st, np.array(gd["inputs"]), np.array(gd["targets"]))
    assert b32(loss) == gd["loss"]
    for i, (off, r_, c_) in enumerate(layout):
        sl = slice(off, off + r_ * c_)
        assert bool(st.has_grad[i]) == (gd["grads"][i] is not None), i
        if gd["grads"][i] is not None:
            assert same(st.grads[sl], gd["grads"][i]), ("grad", i)
        assert same(st.params[sl], gd["after"][i]), ("param", i)
        assert same(st.m[sl], gd["m"][i]) and same(st.v[sl], gd["v"][i]), ("moments", i)


def test_golden_clamps_and_known_values():
    ex = {f32(x): f32(y) for x, y in GOLDEN["exp32"]}
    assert ex[np.float32(0.0)] == np.float32(1.0)
    assert ex[np.float32(88.5)] == np.float32(3.4e38) and ex[np.float32(-88.5)] == 0.0  # grad.go:285-290
    # the truncated polynomial: exp32(1) is 2.718261, not e = 2.7182817
    assert abs(float(ex[np.float32(1.0)]) - 2.718261) < 1e-6
    lg = {f32(x): f32(y) for x, y in GOLDEN["log32"]}
    assert lg[np.float32(1.0)] == 0.0 and np.isneginf(lg[np.float32(0.0)])
