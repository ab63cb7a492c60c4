"""The barrier protocol of the CTA-pair GEMM (gemm_tf32_pair_kernel in
gollama_b200/csrc/gemm_tf32.cu), simulated on the CPU (tests/protocol_sim.py):
both tile orders, tiles with fewer, as many and more k-blocks than the six
stages, random completion orders; no deadlock, no early wake, no stage,
accumulator or ring slot reused before its readers finished."""
import random

import pytest

from tests import protocol_sim as sim


@pytest.mark.parametrize("seed", range(25))
def test_pair_gemm_static_order(seed):
    rnd = random.Random(seed)
    k_blocks = [rnd.choice([1, 2, 5, 6, 7, 13]) for _ in range(rnd.randrange(1, 9))]
    assert sim.pair_gemm(k_blocks, seed) == list(range(len(k_blocks)))


@pytest.mark.parametrize("seed", range(25))
def test_pair_gemm_dynamic_order(seed):
    rnd = random.Random(1000 + seed)
    k_blocks = [rnd.choice([1, 3, 6, 8]) for _ in range(5)]
    total = rnd.randrange(1, 40)
    got = sim.pair_gemm(k_blocks, seed, dyn=True, total_tiles=total, skip=rnd.choice([0.0, 0.5, 0.9]))
    assert got == sorted(set(got)) and all(0 <= t < total for t in got)


def test_pair_gemm_dynamic_order_with_no_tile_left():
    """A pair that finds the counter already past the last tile reads only the
    end marker and leaves."""
    assert sim.pair_gemm([4], 3, dyn=True, total_tiles=0) == []


def test_simulator_catches_a_missing_epilogue_arrival():
    """With one epilogue warp fewer counted on tempty, the issuer may write an
    accumulator a warp of the pair still reads."""
    with pytest.raises(AssertionError):
        for seed in range(200):
            sim.pair_gemm([1] * 6, seed, counts={"tempty": 7})


def test_simulator_catches_a_missing_ring_reader():
    """With one reader fewer counted on ring_empty, the leader may publish the
    next index into a slot a reader of the pair has not taken yet."""
    with pytest.raises(AssertionError):
        for seed in range(200):
            sim.pair_gemm([1], seed, dyn=True, total_tiles=40, counts={"ring_empty": 9})
