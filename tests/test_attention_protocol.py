"""The barrier protocols of the persistent attention kernels, simulated on the
CPU (tests/protocol_sim.py): random shapes, grid sizes and completion orders,
no deadlock, no early wake, no buffer reused before its reader finished."""
import random

import pytest

from tests import protocol_sim as sim


@pytest.mark.parametrize("seed", range(40))
def test_forward_protocol(seed):
    r = random.Random(seed)
    H, B, n_qt = r.randint(1, 4), r.randint(1, 3), r.randint(1, 5)
    grid = r.randint(1, H * B * n_qt)
    for cta in range(grid):
        sim.forward(H, B, n_qt, grid, cta, seed * 131 + cta)


@pytest.mark.parametrize("groups", [1, 2])
@pytest.mark.parametrize("seed", range(40))
def test_dq_protocol(seed, groups):
    r = random.Random(seed)
    H, B, n_qt = r.randint(1, 4), r.randint(1, 3), r.randint(1, 5)
    S = r.randint((n_qt - 1) * 128 + 1, n_qt * 128)
    grid = r.randint(1, H * B * n_qt)
    for cta in range(grid):
        sim.dq(H, B, n_qt, S, grid, cta, seed * 7919 + cta, groups)


def test_simulator_catches_a_wrong_parity():
    """A planted mistake: waiting for the wrong phase of a reused barrier."""
    bar = sim.Bar("x", 1)
    bar.arrive()  # phase 0 completes
    bar.arrive()  # phase 1 completes
    w = sim._wait(bar, 0, 0)  # parity 0 ready again only after phase 2: the wait must block
    with pytest.raises(StopIteration):
        next(sim._wait(bar, 1, 1))
    assert next(w, "blocked") is None


@pytest.mark.parametrize("groups", [1, 2])
@pytest.mark.parametrize("seed", range(40))
def test_dkdv_protocol(seed, groups):
    r = random.Random(seed)
    sim.dkdv(r.randint(1, 4), r.randint(1, 16), seed, groups)
