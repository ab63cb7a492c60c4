"""Checkpoints of device-resident trainers.

SaveCheckpoint (pkg/train/trainer.go:554-584) writes the parameters the GPU
holds, in the reference's text format, to <SavePath>/checkpoint_<step>.bin;
reading the file back gives the device parameters bit for bit.  The binary
state file resumes a trainer: a fresh model and trainer that load it take
the next step exactly as the saved trainer does (same loss, gradients,
weights and AdamW moments, bit for bit: the step is deterministic)."""
import numpy as np
import pytest

from gollama_b200 import synthetic as syn
from gollama_b200.checkpoint import read_checkpoint
from gollama_b200.device import GlcError
from gollama_b200.train import NewTrainableModel, NewTrainer, config_for
from tests.helpers import STEP_HPARAMS

pytestmark = pytest.mark.gpu

SHAPES = [syn.TINY, syn.TINY_LLAMA_MODE]


def bits(a):
    return a.view(np.uint32)


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: s.name)
def test_save_checkpoint_holds_the_device_parameters(ctx, shape, tmp_path):
    cfg = config_for(shape, **STEP_HPARAMS, SavePath=str(tmp_path))
    model = NewTrainableModel(cfg, ctx)
    model.set_params(syn.init_params(shape, 3))
    tr = NewTrainer(model)
    for s in range(2):
        tr.TrainStep(*syn.batch(shape, 60 + s))
    path = tr.SaveCheckpoint()
    assert path == f"{tmp_path}/checkpoint_2.bin"
    step, flat = read_checkpoint(path, cfg)
    assert step == 2
    assert np.array_equal(bits(flat), bits(model.get_params()))
    other = NewTrainableModel(config_for(shape, **STEP_HPARAMS, Seed=7), ctx)
    assert other.LoadCheckpoint(path) == 2
    assert np.array_equal(bits(other.get_params()), bits(flat))
    other.close()
    tr.close()
    model.close()


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: s.name)
def test_state_resume_is_bit_identical(ctx, shape, tmp_path):
    params = syn.init_params(shape, 4)
    batches = [syn.batch(shape, 70 + s) for s in range(3)]
    a = NewTrainableModel(config_for(shape, **STEP_HPARAMS), ctx)
    a.set_params(params)
    ta = NewTrainer(a)
    for b in batches[:2]:
        ta.TrainStep(*b)
    state = tmp_path / "trainer.glcstate"
    ta.SaveState(state)
    loss_a = ta.TrainStep(*batches[2])

    b = NewTrainableModel(config_for(shape, **STEP_HPARAMS, Seed=99), ctx)
    tb = NewTrainer(b)
    tb.LoadState(state)
    assert tb.last_stats()[2] == 2
    loss_b = tb.TrainStep(*batches[2])
    assert loss_a == loss_b
    assert ta.last_stats()[1:] == tb.last_stats()[1:]  # learning rate and step
    assert np.array_equal(bits(a.get_params()), bits(b.get_params()))
    assert np.array_equal(bits(a.get_grads()), bits(b.get_grads()))
    for x, y in zip(a.get_moments(), b.get_moments()):
        assert np.array_equal(bits(x), bits(y))
    for o in (tb, b, ta, a):
        o.close()


def test_load_state_refuses_another_model(ctx, tmp_path):
    a = NewTrainableModel(config_for(syn.TINY, **STEP_HPARAMS), ctx)
    ta = NewTrainer(a)
    state = tmp_path / "tiny.glcstate"
    ta.SaveState(state)
    b = NewTrainableModel(config_for(syn.TINY_LLAMA_MODE, **STEP_HPARAMS), ctx)
    tb = NewTrainer(b)
    before = b.get_params()
    with pytest.raises(GlcError) as e:
        tb.LoadState(state)
    assert e.value.code == -1 and "num_kv_heads" in str(e.value)
    assert np.array_equal(bits(b.get_params()), bits(before))
    for o in (tb, b, ta, a):
        o.close()
