"""Tile lists of grouped CTA-pair GEMM launches (host logic, no GPU).

The dX and dW products of one linear layer share a launch; their tiles take
different times (different reduction lengths), so instead of the fixed
rotation tile = cluster + i * clusters the host hands tiles out in order to
the cluster that frees first.  Checked here through glc_gemm_tile_lists: every
tile appears exactly once, each cluster walks its tiles in ascending order,
the lists are used only where they beat the rotation's estimate by 1 %, and
the shapes of the TinyLlama step get them (except the attention output
projection, where the estimate ties)."""
import ctypes as C

import pytest

from gollama_b200 import _lib

PAIRS = 74  # SM pairs of a B200 (148 SMs)


def tiles(M, N):
    return -(-M // 256) * -(-N // 256)


def kblocks(K):
    return -(-K // 32)


def lists(t0, kb0, t1, kb1, clusters=PAIRS):
    lib = _lib.load()
    used = C.c_int()
    cap = clusters + 1 + t0 + t1
    out = (C.c_int * cap)()
    assert lib.glc_gemm_tile_lists(t0, kb0, t1, kb1, clusters, out, cap, C.byref(used)) == 0
    if not used.value:
        return None
    off = list(out[: clusters + 1])
    ids = list(out[clusters + 1 :])
    return [ids[off[c] : off[c + 1]] for c in range(clusters)]


def estimate(per_cluster, t0, kb0, kb1):
    return max(sum((kb0 if t < t0 else kb1) + 2 for t in lst) for lst in per_cluster)


# (dW first when its reduction is longer, as the launcher orders them): tokens T = 4096
STEP = {
    "qkv": ((tiles(2560, 2048), kblocks(4096)), (tiles(4096, 2048), kblocks(2560))),
    "gate_up": ((tiles(4096, 2048), kblocks(11264)), (tiles(11264, 2048), kblocks(4096))),
    "down": ((tiles(2048, 5632), kblocks(4096)), (tiles(4096, 5632), kblocks(2048))),
    "lm_head": ((tiles(4096, 2048), kblocks(32000)), (tiles(32000, 2048), kblocks(4096))),
}


@pytest.mark.parametrize("name", sorted(STEP))
def test_step_shapes_get_greedy_lists(name):
    (t0, kb0), (t1, kb1) = STEP[name]
    per = lists(t0, kb0, t1, kb1)
    assert per is not None
    flat = sorted(t for lst in per for t in lst)
    assert flat == list(range(t0 + t1))
    assert all(lst == sorted(lst) for lst in per)
    rotation = [list(range(c, t0 + t1, PAIRS)) for c in range(PAIRS)]
    assert 100 * estimate(per, t0, kb0, kb1) <= 99 * estimate(rotation, t0, kb0, kb1)


def test_attention_output_keeps_the_rotation():
    # dW 2048x2048 (64 tiles, K = 4096) with dX 4096x2048 (128 tiles, K = 2048): the estimates tie
    assert lists(tiles(2048, 2048), kblocks(4096), tiles(4096, 2048), kblocks(2048)) is None


def test_equal_tiles_keep_the_rotation():
    assert lists(100, 64, 100, 64) is None


@pytest.mark.parametrize("clusters", [1, 3, 200])
def test_lists_cover_any_cluster_count(clusters):
    per = lists(10, 200, 50, 20, clusters)
    if per is not None:
        assert sorted(t for lst in per for t in lst) == list(range(60))


def test_bad_arguments():
    lib = _lib.load()
    used = C.c_int()
    assert lib.glc_gemm_tile_lists(0, 1, 0, 1, 4, None, 0, C.byref(used)) != 0
    assert lib.glc_gemm_tile_lists(4, 1, 4, 1, 0, None, 0, C.byref(used)) != 0
    # lists wanted but no room for them
    assert lib.glc_gemm_tile_lists(*STEP["qkv"][0], *STEP["qkv"][1], PAIRS, None, 0, C.byref(used)) != 0
