"""CPU model of the bulk-copy ring of ce_stream_kernel (softmax cross-entropy
with streamed rows, gollama_b200/csrc/ce.cu).

The host's sizing (chunk size, slots, grid) and the kernel's loops are
transcribed: thread 0 issues chunk q of the CTA's rows into slot q % nslots
(one mbarrier per slot, arrive + expect_tx, the copy completing its bytes
later), the threads wait for the chunks of a row in order with the parity
(q / nslots) & 1, and after the row's first block barrier thread 0 issues
chunks up to (k + 1) * CHUNKS + nslots.  Copies complete in random order.
Checked: every wait wakes on the phase of its own chunk (never an older or a
newer one), no slot is refilled before its chunk was consumed, no wait can
spin on a copy never issued, each copy is 16-byte aligned and inside the
logits, and every logit of every row is read exactly once."""
import random
import re
from pathlib import Path

import pytest

SRC = (Path(__file__).resolve().parents[1] / "gollama_b200" / "csrc" / "ce.cu").read_text()


def const(name):
    m = re.search(rf"constexpr (?:int|size_t) {name} = ([0-9 *]+);", SRC)
    assert m, name
    return eval(m.group(1))  # a product of integer literals


THREADS, CHUNKS, MAX_SLOTS, SMEM = (const(n) for n in ("CE_ST_THREADS", "CE_ST_CHUNKS", "CE_ST_MAX_SLOTS",
                                                      "CE_ST_SMEM_BYTES"))
SMEM_PER_BLOCK = 232448  # 227 KiB: the opt-in dynamic + static shared memory of one CTA on sm_100


def sizing(rows, V, num_sms=148):
    """softmax_ce's launch of ce_stream_kernel."""
    nc = V // 4
    cf4 = (nc + CHUNKS - 1) // CHUNKS
    nslots = min(MAX_SLOTS, SMEM // (cf4 * 16))
    return nc, cf4, nslots, min(rows, num_sms)


class Slot:
    """mbarrier with arrival count 1: a phase completes when the arrival and
    every expected transaction byte are in."""

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


def run_cta(rows, V, cta, rng, refill_slack=0):
    nc, cf4, nslots, grid = sizing(rows, V)
    nrows = (rows - 1 - cta) // grid + 1 if cta < rows else 0
    nq = nrows * CHUNKS
    slots = [Slot() for _ in range(nslots)]
    owner = [None] * nslots          # chunk last issued into each slot
    consumed = set()
    inflight = []                    # (slot, bytes) copies not yet landed
    seen = {}                        # row -> the float4 column ranges read from it

    def issue(q):
        j, row = q % CHUNKS, cta + (q // CHUNKS) * grid
        assert row < rows
        cnt = min(cf4, nc - j * cf4)
        assert cnt > 0
        src = (row * V + j * cf4 * 4) * 4          # byte offset into the logits
        nbytes = cnt * 16
        assert src % 16 == 0 and nbytes % 16 == 0 and src + nbytes <= rows * V * 4
        s = q % nslots
        assert owner[s] is None or owner[s] in consumed, f"slot {s} refilled with chunk {q} before {owner[s]} was read"
        owner[s] = q
        slots[s].arrive_expect_tx(nbytes)
        inflight.append((s, nbytes))

    issued = 0
    while issued < nq and issued < nslots:
        issue(issued)
        issued += 1
    slot, ph = 0, 0
    for k in range(nrows):
        row = cta + k * grid
        for j in range(CHUNKS):
            q = k * CHUNKS + j
            assert (slot, ph) == (q % nslots, (q // nslots) & 1)
            while not slots[slot].ready(ph):
                assert inflight, f"chunk {q} waits on a copy that was never issued"
                s, n = inflight.pop(rng.randrange(len(inflight)))
                slots[s].complete_tx(n)
            # woke on this chunk's phase: exactly q // nslots + 1 phases of the slot are complete
            assert slots[slot].completed == q // nslots + 1 and owner[slot] == q
            cnt = cf4 if j + 1 < CHUNKS else nc - j * cf4
            assert (cnt - 1) // THREADS < 2             # entry e: thread e % THREADS, register e // THREADS
            seen.setdefault(row, []).append((j * cf4, cnt))
            slot += 1
            if slot == nslots:
                slot, ph = 0, ph ^ 1
        consumed.update(range(k * CHUNKS, (k + 1) * CHUNKS))  # the row's first block barrier
        lim = min(nq, (k + 1) * CHUNKS + nslots + refill_slack)
        while issued < lim:
            issue(issued)
            issued += 1
    assert issued == nq and not inflight
    return seen, nc


@pytest.mark.parametrize("rows,V", [(4096, 32000), (37, 32000), (33, 8196), (7, 16388), (300, 16384), (1, 32768),
                                    (150, 12000)])
def test_ce_ring_protocol(rows, V):
    nc, cf4, nslots, grid = sizing(rows, V)
    assert 2048 < nc <= CHUNKS * 2 * THREADS            # the launcher's range for this kernel
    assert CHUNKS <= nslots <= MAX_SLOTS                 # a whole row fits the ring
    assert nslots * cf4 * 16 + 1024 <= SMEM_PER_BLOCK    # ring + static barriers and partials
    rng = random.Random(rows * 131 + V)
    covered = set()
    for cta in range(grid):
        seen, _ = run_cta(rows, V, cta, rng)
        for row, ranges in seen.items():
            assert row not in covered
            covered.add(row)
            pos = 0
            for start, cnt in sorted(ranges):           # the chunks tile the row's columns exactly once
                assert start == pos
                pos += cnt
            assert pos == nc
    assert covered == set(range(rows))


def test_ring_model_catches_an_early_refill():
    """Refilling one slot more than the row barrier frees overwrites a chunk
    the threads have not read yet."""
    with pytest.raises(AssertionError, match="refilled"):
        run_cta(4096, 32000, 0, random.Random(1), refill_slack=1)
