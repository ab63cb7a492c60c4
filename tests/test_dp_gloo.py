"""Data-parallel host logic on CPU (world_size 2, 4 and 8, gloo).

The GPU path sums each gradient bucket with NCCL as soon as the backward has
written it (glc_dp_bucket_plan gives the buckets).  What that path relies on
is checked here without a GPU:
  * the bucket plan covers the gradient arena exactly, on parameter
    boundaries, one bucket per layer plus the embedding and the output norm;
  * summing per-rank gradients bucket by bucket, in the order the backward
    completes them, reproduces the gradients of the global batch: in
    reference mode the loss seed is ones, so the rank gradients add; in llama
    mode the cross-entropy mean is over the global batch, so each rank's mean
    is weighted by its share of the tokens before the sum.
Each rank runs the oracle on its share of the batch in its own process.
"""
import ctypes as C
import datetime
import os
import socket
import tempfile

import numpy as np
import pytest

from gollama_b200 import _lib
from gollama_b200 import synthetic as syn
from gollama_b200.train import config_for
from tests.helpers import oracle_config, rel_fro

WORLD = 2


def bucket_plan(shape):
    lib = _lib.load()
    cfg = config_for(shape).to_c()
    n = C.c_int()
    assert lib.glc_dp_bucket_plan(C.byref(cfg), None, None, 0, C.byref(n)) == 0
    begin, end = (C.c_int64 * n.value)(), (C.c_int64 * n.value)()
    assert lib.glc_dp_bucket_plan(C.byref(cfg), begin, end, n.value, C.byref(n)) == 0
    return list(zip(begin, end))


@pytest.mark.parametrize("shape", [syn.TINY, syn.TINY_LLAMA_MODE, syn.SMALL, syn.TINYLLAMA], ids=lambda s: s.name)
def test_bucket_plan_covers_the_arena(shape):
    from oracle.oracle import Oracle

    orc = Oracle()
    cfg = oracle_config(shape)
    buckets = bucket_plan(shape)
    assert len(buckets) == shape.layers + 2
    assert buckets[0][0] == 0 and buckets[-1][1] == orc.param_total(cfg)
    for (b0, e0), (b1, _) in zip(buckets, buckets[1:]):
        assert e0 == b1 and e0 > b0
    offsets = {off for off, _, _ in orc.param_layout(cfg)} | {orc.param_total(cfg)}
    for b, e in buckets:
        assert b in offsets and e in offsets


def test_bucket_plan_rejects_bad_config():
    lib = _lib.load()
    cfg = config_for(syn.TINY).to_c()
    cfg.num_heads = 3  # does not divide hidden 128
    n = C.c_int()
    assert lib.glc_dp_bucket_plan(C.byref(cfg), None, None, 0, C.byref(n)) != 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port, shape_name, out_path, world=WORLD, batch=None):
    import torch
    import torch.distributed as dist

    from oracle.oracle import Oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        shape = syn.SHAPES[shape_name]
        if batch:
            shape = shape.with_(batch=batch)
        orc = Oracle(threads=2)
        cfg = oracle_config(shape)
        params = syn.init_params(shape, seed=11)
        inputs, targets = syn.batch(shape, seed=12)
        rows = np.array_split(np.arange(inputs.shape[0]), world)[rank]
        _, grads, _ = orc.forward_backward(cfg, params, inputs[rows], targets[rows])
        if shape.mode == 1:  # llama: the loss is the mean over the global batch
            grads *= np.float32(len(rows) / inputs.shape[0])
        # buckets summed in the order the backward finishes them (last layer first)
        for b, e in reversed(bucket_plan(shape)):
            t = torch.from_numpy(grads[b:e])
            dist.all_reduce(t)
        if rank == 0:
            _, full, _ = orc.forward_backward(cfg, params, inputs, targets)
            np.savez(out_path, summed=grads, full=full)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("shape_name", ["tiny", "tiny-llama"])
def test_rank_bucket_sum_equals_global_batch(shape_name, world):
    """world 8 (the largest single-box run) takes the tiny shapes at batch 8,
    one sequence per rank."""
    import torch.multiprocessing as mp

    batch = max(world, syn.SHAPES[shape_name].batch)
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "grads.npz")
        mp.start_processes(_rank_main, args=(_free_port(), shape_name, out, world, batch), nprocs=world,
                           start_method="spawn")
        r = np.load(out)
        # the ranks' shares add in a different fp32 order than the full batch
        assert rel_fro(r["summed"], r["full"]) < 1e-5
