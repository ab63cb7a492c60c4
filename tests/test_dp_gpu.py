"""Data-parallel TrainStep on two GPUs (one process each, NCCL over NVLink)
against the oracle's step on the global batch.

Each rank trains on its half of the batch with world_size 2; the gradient
buckets are summed while the backward runs.  After one step both ranks must
hold the same gradients and weights, equal to the oracle's step on the whole
batch within the single-GPU bars (tests/helpers.py).  Skipped on a box with
fewer than two GPUs."""
import ctypes as C
import datetime
import os
import socket
import tempfile

import numpy as np
import pytest

from gollama_b200 import synthetic as syn
from tests.helpers import GRAD_RFRO, LOSS_RTOL, STEP_HPARAMS, WEIGHT_RFRO, oracle_config, oracle_optim, rel_fro, threads

pytestmark = pytest.mark.gpu
WORLD = 2


def _gpus() -> int:
    import torch

    return torch.cuda.device_count()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port, shape_name, out_dir, steps=1):
    import torch.distributed as dist

    from gollama_b200.device import Context
    from gollama_b200.train import NewTrainableModel, NewTrainer, config_for

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120))
    try:
        shape = syn.SHAPES[shape_name]
        with Context(rank) as ctx:
            uid = (C.c_ubyte * 128)()
            if rank == 0:
                assert ctx.lib.glc_dp_unique_id(uid) == 0
            obj = [bytes(uid)]
            dist.broadcast_object_list(obj, src=0)
            uid = (C.c_ubyte * 128).from_buffer_copy(obj[0])
            ctx.call("glc_dp_init", rank, WORLD, uid, 120000)
            params = syn.init_params(shape, 1234)
            model = NewTrainableModel(config_for(shape, WorldSize=WORLD, **STEP_HPARAMS), ctx)
            model.set_params(params)
            tr = NewTrainer(model)
            norms = []
            for step in range(steps):
                inputs, targets = syn.batch(shape, 1234 + step)
                rows = np.array_split(np.arange(inputs.shape[0]), WORLD)[rank]
                loss = tr.TrainStep(inputs[rows], targets[rows])
                norms.append(tr.last_stats()[0])
            np.savez(os.path.join(out_dir, f"rank{rank}.npz"), loss=loss, grads=model.get_grads(),
                     weights=model.get_params(), has=np.array([p.has_grad for p in model.Params()]),
                     norms=np.array(norms))
            ctx.call("glc_dp_destroy")
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(_gpus() < WORLD, reason="needs two GPUs")
@pytest.mark.parametrize("shape", [syn.TINY, syn.TINY_LLAMA_MODE, syn.SMALL_LLAMA_MODE], ids=lambda s: s.name)
def test_two_gpu_step_matches_global_batch(shape):
    import torch.multiprocessing as mp

    from oracle.oracle import Oracle, TrainState

    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main, args=(_free_port(), shape.name, d), nprocs=WORLD, start_method="spawn")
        r = [np.load(os.path.join(d, f"rank{i}.npz")) for i in range(WORLD)]
    # replicas stay identical
    assert np.array_equal(r[0]["grads"], r[1]["grads"])
    assert np.array_equal(r[0]["weights"], r[1]["weights"])

    orc = Oracle(threads=threads())
    ocfg = oracle_config(shape)
    layout = orc.param_layout(ocfg)
    st = TrainState.create(syn.init_params(shape, 1234), len(layout), oracle_optim())
    inputs, targets = syn.batch(shape, 1234)
    oloss, _ = orc.train_step(ocfg, st, inputs, targets)
    # llama: per-rank losses are means over equal halves; reference: sums of means
    loss = float(np.mean([x["loss"] for x in r]))
    assert abs(loss - oloss) <= LOSS_RTOL * abs(oloss), (loss, oloss)
    assert list(r[0]["has"]) == [bool(h) for h in st.has_grad]
    for i, (off, rows, cols) in enumerate(layout):
        n = rows * cols
        if st.has_grad[i]:
            e = rel_fro(r[0]["grads"][off : off + n], st.grads[off : off + n])
            assert e < GRAD_RFRO, f"grad of param {i}: rel-fro {e:.3e}"
        e = rel_fro(r[0]["weights"][off : off + n], st.params[off : off + n])
        assert e < WEIGHT_RFRO, f"weight of param {i}: rel-fro {e:.3e}"


@pytest.mark.skipif(_gpus() < WORLD, reason="needs two GPUs")
@pytest.mark.parametrize("shape", [syn.TINY_LLAMA_MODE, syn.TINY], ids=lambda s: s.name)
def test_two_gpu_three_steps_match_global_batch(shape):
    """Three data-parallel steps: from the second on, the clip norm comes from
    the per-bucket sums taken after each allreduce.  Every step's clip norm,
    and the third step's gradients and weights, against the oracle's steps on
    the global batches."""
    import torch.multiprocessing as mp

    from oracle.oracle import Oracle, TrainState

    steps = 3
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main, args=(_free_port(), shape.name, d, steps), nprocs=WORLD, start_method="spawn")
        r = [np.load(os.path.join(d, f"rank{i}.npz")) for i in range(WORLD)]
    assert np.array_equal(r[0]["weights"], r[1]["weights"])
    assert np.array_equal(r[0]["norms"], r[1]["norms"])
    orc = Oracle(threads=threads())
    ocfg = oracle_config(shape)
    layout = orc.param_layout(ocfg)
    st = TrainState.create(syn.init_params(shape, 1234), len(layout), oracle_optim())
    onorms = []
    for step in range(steps):
        inputs, targets = syn.batch(shape, 1234 + step)
        onorms.append(orc.train_step(ocfg, st, inputs, targets)[1])
    for a, b in zip(r[0]["norms"], onorms):
        assert abs(a - b) <= 2e-3 * abs(b), (list(r[0]["norms"]), onorms)
    for i, (off, rows, cols) in enumerate(layout):
        n = rows * cols
        if st.has_grad[i]:
            assert rel_fro(r[0]["grads"][off : off + n], st.grads[off : off + n]) < GRAD_RFRO, i
        assert rel_fro(r[0]["weights"][off : off + n], st.params[off : off + n]) < WEIGHT_RFRO, i
