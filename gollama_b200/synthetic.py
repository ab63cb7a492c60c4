"""Seeded synthetic inputs: weights, token ids and the named model shapes.

The reference initialises weights from Go's math/rand (pkg/train/trainer.go:
207,259-266) and draws batches from a tokenized corpus (pkg/train/dataset.go:
39-55).  Neither is reproducible without Go, and no corpus ships, so every
input here comes from one documented generator instead:

  splitmix64(seed, i)  -> 64-bit word i of stream `seed`
  uniform(seed, i)     = (word >> 11) * 2^-53                  in [0, 1)
  normal(seed, i)      = Box-Muller on (uniform(2i), uniform(2i+1)), cosine branch
  zipf(seed, i, V, s)  = inverse CDF of P(k) ~ 1/k^s over k = 1..V, id = k-1

Weight matrices are N(0, 0.02); RMSNorm weights start at 1 like
NewRMSNormTrainable (trainer.go:129-133).  Token sequences are drawn as B rows
of S+1 ids; inputs are [:, :S] and targets [:, 1:], the shift-by-one slicing
of Dataset.GetBatch (dataset.go:50-51).
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import numpy as np

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def splitmix64(seed: int, n: int, start: int = 0) -> np.ndarray:
    with np.errstate(over="ignore"):
        x = (np.uint64(seed) * np.uint64(0x9E3779B97F4A7C15)) + np.uint64(0x9E3779B97F4A7C15) * (
            np.arange(start, start + n, dtype=np.uint64) + np.uint64(1)
        )
        z = x
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return z


def uniform(seed: int, n: int, start: int = 0) -> np.ndarray:
    return (splitmix64(seed, n, start) >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)


def normal(seed: int, n: int, std: float = 1.0) -> np.ndarray:
    u = uniform(seed, 2 * n)
    u1 = 1.0 - u[0::2]  # (0, 1]
    u2 = u[1::2]
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    return (z * std).astype(np.float32)


def uniform_tokens(seed: int, shape, vocab: int) -> np.ndarray:
    n = int(np.prod(shape))
    return np.minimum((uniform(seed, n) * vocab).astype(np.int64), vocab - 1).reshape(shape)


def zipf_tokens(seed: int, shape, vocab: int, s: float = 1.1) -> np.ndarray:
    n = int(np.prod(shape))
    w = 1.0 / np.arange(1, vocab + 1, dtype=np.float64) ** s
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    ids = np.searchsorted(cdf, uniform(seed, n), side="right")
    return np.minimum(ids, vocab - 1).astype(np.int64).reshape(shape)


@dataclass(frozen=True)
class ModelShape:
    """A decoder shape plus the batch it is trained on (one GPU's share)."""

    name: str
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    inter: int
    vocab: int
    seq: int
    batch: int
    mode: int  # 0 reference semantics, 1 Llama semantics
    zipf: bool = False
    rope_theta: float = 10000.0
    norm_eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def tokens(self) -> int:
        return self.batch * self.seq

    def with_(self, **kw) -> "ModelShape":
        return replace(self, **kw)


# Tiny decoder (2 layers, d 128, 4 heads, FFN 344, byte vocab, seq 64, batch 4).
TINY = ModelShape("tiny", 2, 128, 4, 4, 344, 256, 64, 4, mode=0)
TINY_LLAMA_MODE = TINY.with_(name="tiny-llama", kv_heads=2, mode=1)
# Small decoder (6 layers, d 512, 8 heads, FFN 1376, vocab 32000, seq 256, batch 8, Zipf ids).
SMALL = ModelShape("small", 6, 512, 8, 8, 1376, 32000, 256, 8, mode=0, zipf=True)
SMALL_LLAMA_MODE = SMALL.with_(name="small-llama", kv_heads=4, mode=1)
# TinyLlama-1.1B shape (22 layers, d 2048, 32/4 heads, FFN 5632, vocab 32000, seq 1024, batch 4 per GPU).
TINYLLAMA = ModelShape("tinyllama-1.1b", 22, 2048, 32, 4, 5632, 32000, 1024, 4, mode=1, zipf=True)

SHAPES = {s.name: s for s in (TINY, TINY_LLAMA_MODE, SMALL, SMALL_LLAMA_MODE, TINYLLAMA)}


def param_shapes(shape: ModelShape) -> list[tuple[str, tuple[int, int]]]:
    """Params() order of the reference (trainer.go:217,242-247,253); Llama mode
    drops PosEmbed and narrows WK/WV to kv_heads*head_dim rows."""
    d, F, V = shape.hidden, shape.inter, shape.vocab
    kvd = (shape.kv_heads if shape.mode == 1 else shape.heads) * shape.head_dim
    out = [("TokenEmbed", (V, d))]
    if shape.mode == 0:
        out.append(("PosEmbed", (shape.seq, d)))
    for l in range(shape.layers):
        out += [
            (f"L{l}.AttnNorm", (1, d)),
            (f"L{l}.WQ", (d, d)),
            (f"L{l}.WK", (kvd, d)),
            (f"L{l}.WV", (kvd, d)),
            (f"L{l}.WO", (d, d)),
            (f"L{l}.FFNNorm", (1, d)),
            (f"L{l}.WGate", (F, d)),
            (f"L{l}.WUp", (F, d)),
            (f"L{l}.WDown", (d, F)),
        ]
    out.append(("OutputNorm", (1, d)))
    return out


def init_params(shape: ModelShape, seed: int, std: float = 0.02) -> np.ndarray:
    """Flat float32 parameter vector in Params() order."""
    shapes = param_shapes(shape)
    total = sum(r * c for _, (r, c) in shapes)
    out = np.empty(total, np.float32)
    off = 0
    for i, (name, (r, c)) in enumerate(shapes):
        n = r * c
        if name.endswith("Norm"):
            out[off : off + n] = 1.0
        else:
            out[off : off + n] = normal(seed * 1000003 + i, n, std)
        off += n
    return out


def batch(shape: ModelShape, seed: int) -> tuple[np.ndarray, np.ndarray]:
    """(inputs, targets) of shape [batch, seq], int64."""
    B, S = shape.batch, shape.seq
    if shape.zipf:
        seqs = zipf_tokens(seed, (B, S + 1), shape.vocab)
    else:
        seqs = uniform_tokens(seed, (B, S + 1), shape.vocab)
    return np.ascontiguousarray(seqs[:, :S]), np.ascontiguousarray(seqs[:, 1:])
