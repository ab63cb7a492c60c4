"""Trainer.TrainStep (pkg/train/trainer.go:462-505) on the GPU against the
oracle's step on identical seeded parameters and tokens.

Bars (tests/helpers.py): loss within 1e-4 relative; every parameter gradient
(as TrainStep leaves it: after clipping) and every post-step weight within
2e-3 relative Frobenius error; the set of parameters that have a gradient
(Go's `Grad != nil`) identical."""
import numpy as np
import pytest

from gollama_b200 import synthetic as syn
from gollama_b200.train import NewTrainableModel, NewTrainer, config_for
from oracle.oracle import Oracle, TrainState
from tests.helpers import GRAD_RFRO, LOSS_RTOL, STEP_HPARAMS, WEIGHT_RFRO, oracle_config, oracle_optim, rel_fro, threads

pytestmark = pytest.mark.gpu

# The TinyLlama-1.1B widths (d 2048, 32 query / 4 KV heads, FFN 5632, vocab
# 32000, sequences of 1024) with 2 of its 22 layers and 2 sequences: the
# north-star shape at a size the oracle steps through in about a minute.
TINYLLAMA_WIDTH = syn.TINYLLAMA.with_(name="tinyllama-width-2l-b2", layers=2, batch=2)
SHAPES = [syn.TINY, syn.TINY_LLAMA_MODE, syn.SMALL, syn.SMALL_LLAMA_MODE, TINYLLAMA_WIDTH]


def run_oracle(shape, params, inputs, targets, steps=1):
    orc = Oracle(threads=threads())
    ocfg = oracle_config(shape)
    st = TrainState.create(params, len(orc.param_layout(ocfg)), oracle_optim())
    losses = []
    for s in range(steps):
        loss, norm = orc.train_step(ocfg, st, inputs[s], targets[s])
        losses.append(loss)
    return losses, st, orc.param_layout(ocfg)


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: s.name)
def test_train_step_parity(ctx, shape):
    seed = 1234
    params = syn.init_params(shape, seed)
    inputs, targets = syn.batch(shape, seed)
    (oloss,), st, layout = run_oracle(shape, params, [inputs], [targets])

    model = NewTrainableModel(config_for(shape, **STEP_HPARAMS), ctx)
    model.set_params(params)
    tr = NewTrainer(model)
    loss = tr.TrainStep(inputs, targets)
    assert tr.last_launches() > 0

    assert abs(loss - oloss) <= LOSS_RTOL * abs(oloss), (loss, oloss)
    got_p = model.Params()
    assert [p.has_grad for p in got_p] == [bool(h) for h in st.has_grad]
    grads, weights = model.get_grads(), model.get_params()
    worst = []
    for p, (off, r, c) in zip(got_p, layout):
        n = r * c
        assert (p.offset, p.shape) == (off, (r, c))
        if p.has_grad:
            e = rel_fro(grads[off : off + n], st.grads[off : off + n])
            worst.append((e, p.index))
            assert e < GRAD_RFRO, f"grad of param {p.index} {p.shape}: rel-fro {e:.3e}"
        e = rel_fro(weights[off : off + n], st.params[off : off + n])
        assert e < WEIGHT_RFRO, f"weight of param {p.index}: rel-fro {e:.3e}"
    worst.sort(reverse=True)
    print(f"\n{shape.name}: loss {loss:.6f} (oracle {oloss:.6f}); worst grad rel-fro {worst[:3]}")


def test_reference_mode_gradient_set(ctx):
    """Reference semantics: attention has no GradFn (trainer.go:335-337) and
    the embedding none either (:290-291), so WQ/WK/WV, every AttnNorm and
    PosEmbed never get a gradient; AdamW leaves them untouched (optimizer.go:45)."""
    shape = syn.TINY
    params = syn.init_params(shape, 5)
    inputs, targets = syn.batch(shape, 5)
    model = NewTrainableModel(config_for(shape, **STEP_HPARAMS), ctx)
    model.set_params(params)
    NewTrainer(model).TrainStep(inputs, targets)
    names = [n for n, _ in syn.param_shapes(shape)]
    after = model.get_params()
    for p, name in zip(model.Params(), names):
        frozen = name == "PosEmbed" or name.endswith((".WQ", ".WK", ".WV", ".AttnNorm"))
        assert p.has_grad == (not frozen), name
        seg = slice(p.offset, p.offset + p.shape[0] * p.shape[1])
        if frozen:
            assert np.array_equal(after[seg], params[seg]), name


def test_multi_step_loss_curve(ctx):
    """Small Llama-mode decoder: 5 steps track the oracle's loss curve."""
    shape = syn.SMALL_LLAMA_MODE.with_(layers=2)
    params = syn.init_params(shape, 77)
    batches = [syn.batch(shape, 100 + s) for s in range(5)]
    olosses, st, _ = run_oracle(shape, params, [b[0] for b in batches], [b[1] for b in batches], steps=5)
    model = NewTrainableModel(config_for(shape, **STEP_HPARAMS), ctx)
    model.set_params(params)
    tr = NewTrainer(model)
    losses = [tr.TrainStep(i, t) for i, t in batches]
    for a, b in zip(losses, olosses):
        assert abs(a - b) <= 1e-3 * abs(b), (losses, olosses)
    assert rel_fro(model.get_params(), st.params) < WEIGHT_RFRO


@pytest.mark.parametrize("shape", [syn.TINY, syn.TINY_LLAMA_MODE], ids=lambda s: s.name)
def test_second_step_norm_grads_weights(ctx, shape):
    """Two steps (the second with every gradient already allocated, AdamW
    moments non-zero): each step's clip norm, and the second step's clipped
    gradients and weights, against the oracle's."""
    params = syn.init_params(shape, 31)
    batches = [syn.batch(shape, 40 + s) for s in range(2)]
    orc = Oracle(threads=threads())
    ocfg = oracle_config(shape)
    st = TrainState.create(params, len(orc.param_layout(ocfg)), oracle_optim())
    onorms = [orc.train_step(ocfg, st, i, t)[1] for i, t in batches]
    model = NewTrainableModel(config_for(shape, **STEP_HPARAMS), ctx)
    model.set_params(params)
    tr = NewTrainer(model)
    norms = []
    for i, t in batches:
        tr.TrainStep(i, t)
        norms.append(tr.last_stats()[0])
    for a, b in zip(norms, onorms):
        assert abs(a - b) <= 2e-3 * abs(b), (norms, onorms)
    grads, weights = model.get_grads(), model.get_params()
    for p in model.Params():
        seg = slice(p.offset, p.offset + p.shape[0] * p.shape[1])
        if p.has_grad:
            assert rel_fro(grads[seg], st.grads[seg]) < GRAD_RFRO, p.index
        assert rel_fro(weights[seg], st.params[seg]) < WEIGHT_RFRO, p.index


def test_context_closes_its_models_and_trainers():
    """Models and trainers use their context's stream: closing the context
    closes them first (trainers, then models), and a later close is a no-op."""
    from gollama_b200.device import Context

    with Context(0) as c:
        model = NewTrainableModel(config_for(syn.TINY, **STEP_HPARAMS), c)
        model.set_params(syn.init_params(syn.TINY, 3))
        tr = NewTrainer(model)
        tr.TrainStep(*syn.batch(syn.TINY, 3))
    assert tr.h is None and model.h is None
    tr.close()
    model.close()


@pytest.mark.parametrize("shape", [syn.TINY_LLAMA_MODE, syn.SMALL_LLAMA_MODE.with_(layers=2)], ids=lambda s: s.name)
def test_fused_swiglu_epilogue_bit_identical(ctx, shape):
    """With Llama semantics the SwiGLU forward may run in the gate/up GEMM's
    epilogue; the step is bit-identical to the default separate kernel."""
    params = syn.init_params(shape, 21)
    inputs, targets = syn.batch(shape, 21)
    out = []
    try:
        for fused in (1, 0):
            ctx.call("glc_set_fused_swiglu", fused)
            model = NewTrainableModel(config_for(shape, **STEP_HPARAMS), ctx)
            model.set_params(params)
            loss = NewTrainer(model).TrainStep(inputs, targets)
            out.append((loss, model.get_grads(), model.get_params()))
            model.close()
    finally:
        ctx.call("glc_set_fused_swiglu", 0)
    (l1, g1, w1), (l0, g0, w0) = out
    assert l1 == l0
    assert np.array_equal(g1.view(np.uint32), g0.view(np.uint32))
    assert np.array_equal(w1.view(np.uint32), w0.view(np.uint32))


@pytest.mark.parametrize("shape", [syn.TINY, syn.TINY_LLAMA_MODE, syn.SMALL_LLAMA_MODE.with_(layers=2)],
                         ids=lambda s: s.name)
def test_clip_norm_covers_every_gradient_once(ctx, shape):
    """On one GPU the clip norm's squares come from the dW GEMM epilogues plus
    a pass over the gradients no GEMM stores.  With a threshold that never
    clips, the reported norm equals the float64 norm of the returned
    gradients: a gradient counted twice or missed would show far above
    float64 rounding."""
    hp = dict(STEP_HPARAMS, GradClipNorm=1e30)
    params = syn.init_params(shape, 8)
    model = NewTrainableModel(config_for(shape, **hp), ctx)
    model.set_params(params)
    tr = NewTrainer(model)
    for s in range(2):  # the first step allocates the gradients, the second reuses them
        tr.TrainStep(*syn.batch(shape, 50 + s))
        norm = tr.last_stats()[0]
        g = model.get_grads().astype(np.float64)
        has = np.zeros(g.size, bool)
        for p in model.Params():
            if p.has_grad:
                has[p.offset : p.offset + p.shape[0] * p.shape[1]] = True
        ref = float(np.sqrt(np.sum(g[has] ** 2)))
        assert abs(norm - ref) <= 1e-10 * ref, (s, norm, ref)


def test_tracing_ranges_leave_the_step_unchanged(ctx):
    """glc_set_tracing(1) adds NVTX ranges around the step's phases (host
    calls only): the step's results are the same bits."""
    shape = syn.TINY_LLAMA_MODE
    params = syn.init_params(shape, 29)
    inputs, targets = syn.batch(shape, 29)
    out = []
    try:
        for on in (0, 1):
            ctx.call("glc_set_tracing", on)
            model = NewTrainableModel(config_for(shape, **STEP_HPARAMS), ctx)
            model.set_params(params)
            loss = NewTrainer(model).TrainStep(inputs, targets)
            out.append((loss, model.get_params()))
            model.close()
    finally:
        ctx.call("glc_set_tracing", 0)
    assert out[0][0] == out[1][0]
    assert np.array_equal(out[0][1].view(np.uint32), out[1][1].view(np.uint32))


@pytest.mark.parametrize("shape", [syn.TINY_LLAMA_MODE, syn.TINY], ids=lambda s: s.name)
def test_programmatic_dependent_launch_step_bit_identical(ctx, shape):
    """glc_set_pdl(1) (the default): kernels launch while their predecessor
    finishes and wait for it at entry; two steps give the same bits as
    ordinary launches (glc_set_pdl(0))."""
    params = syn.init_params(shape, 37)
    batches = [syn.batch(shape, 37 + s) for s in range(2)]
    out = []
    try:
        for on in (0, 1):
            ctx.call("glc_set_pdl", on)
            model = NewTrainableModel(config_for(shape, **STEP_HPARAMS), ctx)
            model.set_params(params)
            tr = NewTrainer(model)
            losses = [tr.TrainStep(*b) for b in batches]
            out.append((losses, model.get_grads(), model.get_params()))
            tr.close()
            model.close()
    finally:
        ctx.call("glc_set_pdl", 1)  # the default
    (l0, g0, w0), (l1, g1, w1) = out
    assert l0 == l1
    assert np.array_equal(g0.view(np.uint32), g1.view(np.uint32))
    assert np.array_equal(w0.view(np.uint32), w1.view(np.uint32))


VARIANTS = ["glc_set_attention_fwd_variant", "glc_set_attention_dq_variant", "glc_set_attention_dkdv_variant",
            "glc_set_rmsnorm_variant",
            "glc_set_gemm_schedule"]


@pytest.mark.parametrize("shape", [syn.TINY_LLAMA_MODE, syn.SMALL_LLAMA_MODE.with_(layers=2)], ids=lambda s: s.name)
def test_opt_in_variants_step_bit_identical(ctx, shape):
    """A whole step (RoPE in the dQ epilogue included) with the persistent
    attention kernels and the pipelined RMSNorm backward equals the default
    step bit for bit."""
    params = syn.init_params(shape, 23)
    inputs, targets = syn.batch(shape, 23)
    out = []
    try:
        for v in (1, 2):
            for name in VARIANTS:
                ctx.call(name, v)
            model = NewTrainableModel(config_for(shape, **STEP_HPARAMS), ctx)
            model.set_params(params)
            loss = NewTrainer(model).TrainStep(inputs, targets)
            out.append((loss, model.get_grads(), model.get_params()))
            model.close()
    finally:
        for name in VARIANTS:
            ctx.call(name, 0)
    (l1, g1, w1), (l2, g2, w2) = out
    assert l1 == l2
    assert np.array_equal(g1.view(np.uint32), g2.view(np.uint32))
    assert np.array_equal(w1.view(np.uint32), w2.view(np.uint32))
