"""The oracle against golden vectors of the reference's own float32
exponential and logarithm (pkg/tensor/grad.go:283-381).

tests/golden/go_exp32_log32.json is written by tests/golden/make_golden.py, a
plain-Python restatement of the reference's `_exp` / `_log` made separately
from the C oracle (oracle/oracle.c) and the device code.  The oracle must
reproduce every vector bit for bit (the device code is checked against the
oracle on a sweep in tests/test_ops_gpu.py)."""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle.oracle import lib

GOLDEN = json.loads((Path(__file__).parent / "golden" / "go_exp32_log32.json").read_text())


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


def test_golden_clamps_and_known_values():
    ex = {f32(x): f32(y) for x, y in GOLDEN["exp32"]}
    assert ex[np.float32(0.0)] == np.float32(1.0)
    assert ex[np.float32(88.5)] == np.float32(3.4e38) and ex[np.float32(-88.5)] == 0.0  # grad.go:285-290
    # the truncated polynomial: exp32(1) is 2.718261, not e = 2.7182817
    assert abs(float(ex[np.float32(1.0)]) - 2.718261) < 1e-6
    lg = {f32(x): f32(y) for x, y in GOLDEN["log32"]}
    assert lg[np.float32(1.0)] == 0.0 and np.isneginf(lg[np.float32(0.0)])
