"""CPU model of the bulk-copy ring of rmsnorm_bwd_full_tma_kernel (the exact
RMSNorm backward, gollama_b200/csrc/rmsnorm.cu).

Transcribed: the launcher's split of the rows over blocks, and per block
thread 0 issuing row k into stage k % TMA_STAGES (one mbarrier per stage,
arrive + expect_tx for the row's two or three copies, each landing later),
the block waiting for row k with the parity (k / TMA_STAGES) & 1, and thread 0
issuing the next row into the stage just read after the row's first block
barrier.  Copies land in random order.  Checked: each wait wakes on its own
row's phase, no stage is refilled before its row was read, every row is read
exactly once, the shared memory of two blocks fits an SM; and on an abort (a
wait that gives up) the drain waits only on phases that are still the
stage's outstanding one, so none of its bounded waits names a phase that can
no longer complete."""
import random
import re
from pathlib import Path

import pytest

SRC = (Path(__file__).resolve().parents[1] / "gollama_b200" / "csrc" / "rmsnorm.cu").read_text()
STAGES = int(re.search(r"constexpr int TMA_STAGES = (\d+);", SRC).group(1))
SMEM_PER_SM = 233472  # 228 KiB of shared memory per SM on sm_100
STATIC_BYTES = 32 * 4 + 4 + 1024  # red[32], the abort flag, and the runtime's reserve per block


def sizing(rows, num_sms=148):
    """rmsnorm_bwd's split of the rows for the bulk-copy kernel."""
    nblocks = min(2 * num_sms, rows)
    rpb = (rows + nblocks - 1) // nblocks
    return (rows + rpb - 1) // rpb, rpb


class Stage:
    def __init__(self):
        self.completed, self.pending_arrival, self.tx = 0, 1, 0

    def arrive_expect_tx(self, n):
        self.pending_arrival -= 1
        self.tx += n
        self._maybe()

    def complete_tx(self, n):
        self.tx -= n
        self._maybe()

    def _maybe(self):
        assert self.pending_arrival >= 0 and self.tx >= 0
        if self.pending_arrival == 0 and self.tx == 0:
            self.completed += 1
            self.pending_arrival = 1

    def ready(self, parity):
        return (self.completed & 1) != parity


def run_block(row0, row1, cols, accumulate, rng, abort_at=None, drain_from_start=False):
    """One block's rows [row0, row1).  abort_at: the local row whose wait gives
    up (its copies, and later ones, may still be in flight).  Returns the rows
    read."""
    row_bytes = cols * 4
    ncopies = 3 if accumulate else 2
    stages = [Stage() for _ in range(STAGES)]
    owner = [None] * STAGES
    read = []
    inflight = []  # (stage, bytes)

    def issue(k):
        st = k % STAGES
        assert owner[st] is None or owner[st] in read, f"stage {st} refilled with row {k} before row {owner[st]} was read"
        owner[st] = k
        stages[st].arrive_expect_tx(ncopies * row_bytes)
        for _ in range(ncopies):
            assert row_bytes % 16 == 0
            inflight.append((st, row_bytes))

    def land_some():
        for _ in range(rng.randrange(len(inflight) + 1)):
            st, n = inflight.pop(rng.randrange(len(inflight)))
            stages[st].complete_tx(n)

    n = row1 - row0
    issued = 0
    while issued < STAGES and issued < n:
        issue(issued)
        issued += 1
    k = 0
    while k < n:
        st, parity = k % STAGES, (k // STAGES) & 1
        if k == abort_at:
            land_some()   # some copies land, the awaited one perhaps not: the wait gives up
            break
        while not stages[st].ready(parity):
            assert inflight, f"row {k} waits on a copy that was never issued"
            s, b = inflight.pop(rng.randrange(len(inflight)))
            stages[s].complete_tx(b)
        assert stages[st].completed == k // STAGES + 1 and owner[st] == k
        read.append(k)
        if issued < n:   # after the row's first block barrier
            issue(issued)
            issued += 1
        k += 1
    if abort_at is None:
        assert issued == n
        return read
    land_some()
    # thread 0's drain: every row it waits on must still be its stage's outstanding phase
    for r in range(0 if drain_from_start else k, issued):
        assert stages[r % STAGES].completed <= r // STAGES + 1, f"drain of row {r} names a phase already passed"
    return read


@pytest.mark.parametrize("rows,cols", [(4096, 2048), (32768, 2048), (7, 2048), (300, 512), (1, 1024), (1000, 2044)])
@pytest.mark.parametrize("accumulate", [False, True])
def test_rmsnorm_ring_protocol(rows, cols, accumulate):
    nblocks, rpb = sizing(rows)
    smem = 4 * STAGES * 3 * cols + 8 * STAGES
    assert 2 * (smem + STATIC_BYTES) <= SMEM_PER_SM    # two blocks per SM
    assert (4 * STAGES * 3 * cols) % 8 == 0           # the barriers after the stages are 8-byte aligned
    rng = random.Random(rows + cols)
    seen = []
    for b in range(nblocks):
        row0, row1 = b * rpb, min(rows, (b + 1) * rpb)
        seen += [row0 + k for k in run_block(row0, row1, cols, accumulate, rng)]
    assert sorted(seen) == list(range(rows))


@pytest.mark.parametrize("seed", range(20))
def test_rmsnorm_ring_abort_drain(seed):
    rng = random.Random(seed)
    n = rng.randrange(1, 30)
    run_block(0, n, 2048, seed % 2 == 1, rng, abort_at=rng.randrange(n))


def test_ring_model_catches_a_drain_from_the_first_row():
    """Draining from the block's first row, as an earlier build did, waits on
    phases of stages that have since been refilled and landed."""
    with pytest.raises(AssertionError, match="already passed"):
        for seed in range(50):
            rng = random.Random(seed)
            run_block(0, 20, 2048, False, rng, abort_at=12, drain_from_start=True)
