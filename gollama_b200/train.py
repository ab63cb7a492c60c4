"""Host-side mirror of the reference's trainer interface (pkg/train).

Names follow the Go API so code and tests read like the reference's:
TrainConfig / DefaultTrainConfig (trainer.go:15-69), NewTrainableModel
(:206-256) with Params() (:429-431), NewTrainer (:447-459) and
Trainer.TrainStep (:462-505).  Everything runs through libgollama_cuda's C ABI
on the GPU; nothing here computes.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, fields

import numpy as np

from . import _lib
from .device import Context, GlcError

SEMANTICS_REFERENCE = 0
SEMANTICS_LLAMA = 1


@dataclass
class TrainConfig:
    VocabSize: int = 32000
    HiddenSize: int = 512
    NumLayers: int = 8
    NumHeads: int = 8
    IntermediateSize: int = 1408
    MaxSeqLen: int = 512
    BatchSize: int = 4
    BlockSize: int = 256
    LearningRate: float = 3e-4
    WeightDecay: float = 0.01
    WarmupSteps: int = 100
    MaxSteps: int = 10000
    GradClipNorm: float = 1.0
    # AdamW fields (NewAdamW defaults, optimizer.go:24-34)
    Beta1: float = 0.9
    Beta2: float = 0.999
    Epsilon: float = 1e-8
    # extensions
    NumKVHeads: int = 0
    Semantics: int = SEMANTICS_REFERENCE
    NormEps: float = 1e-5
    RopeTheta: float = 10000.0
    InitStd: float = 0.02
    Seed: int = 42
    WorldSize: int = 1
    # host-only fields (not in glc_train_config): logging and checkpoint cadence
    # and SaveCheckpoint's directory (trainer.go:33-36, defaults :62-65)
    SavePath: str = "./checkpoints"
    LogInterval: int = 10
    SaveInterval: int = 1000

    def to_c(self) -> _lib.TrainConfigC:
        c = _lib.TrainConfigC()
        names = [f[0] for f in _lib.TrainConfigC._fields_]
        vals = [getattr(self, f.name) for f in fields(self)][: len(names)]
        for n, v in zip(names, vals):
            setattr(c, n, v)
        return c


def DefaultTrainConfig() -> TrainConfig:
    return TrainConfig()


def config_for(shape, **overrides) -> TrainConfig:
    """TrainConfig of a gollama_b200.synthetic.ModelShape."""
    cfg = TrainConfig(
        VocabSize=shape.vocab,
        HiddenSize=shape.hidden,
        NumLayers=shape.layers,
        NumHeads=shape.heads,
        IntermediateSize=shape.inter,
        MaxSeqLen=shape.seq,
        BatchSize=shape.batch,
        BlockSize=shape.seq,
        NumKVHeads=shape.kv_heads,
        Semantics=shape.mode,
        RopeTheta=shape.rope_theta,
        NormEps=shape.norm_eps,
    )
    for k, v in overrides.items():
        setattr(cfg, k, v)
    return cfg


@dataclass
class Param:
    index: int
    offset: int
    shape: tuple
    has_grad: bool


class TrainableModel:
    """NewTrainableModel: device-resident parameters in Params() order."""

    def __init__(self, cfg: TrainConfig, ctx: Context | None = None):
        self.ctx = ctx or Context(0)
        self.Config = cfg
        self._c = cfg.to_c()
        h = C.c_void_p()
        self.ctx.check(self.ctx.lib.glc_model_create(self.ctx.h, C.byref(self._c), C.byref(h)), "glc_model_create")
        self.h = h
        self.ctx.adopt(self, 1)
        n, tot = C.c_int(), C.c_int64()
        self.ctx.check(self.ctx.lib.glc_model_num_params(self.h, C.byref(n), C.byref(tot)), "glc_model_num_params")
        self.num_params = n.value
        self.total = tot.value

    def Params(self) -> list[Param]:
        out = []
        for i in range(self.num_params):
            off, r, c, hg = C.c_int64(), C.c_int64(), C.c_int64(), C.c_int()
            self.ctx.check(
                self.ctx.lib.glc_model_param_info(self.h, i, C.byref(off), C.byref(r), C.byref(c), C.byref(hg)),
                "glc_model_param_info",
            )
            out.append(Param(i, off.value, (r.value, c.value), bool(hg.value)))
        return out

    def set_params(self, flat: np.ndarray) -> None:
        flat = np.ascontiguousarray(flat, np.float32)
        assert flat.size == self.total
        self.ctx.check(self.ctx.lib.glc_model_set_params(self.h, flat.ctypes.data_as(C.c_void_p), flat.size),
                       "glc_model_set_params")

    def _get(self, fn: str) -> np.ndarray:
        out = np.empty(self.total, np.float32)
        self.ctx.check(getattr(self.ctx.lib, fn)(self.h, out.ctypes.data_as(C.c_void_p), out.size), fn)
        return out

    def get_params(self) -> np.ndarray:
        return self._get("glc_model_get_params")

    def get_grads(self) -> np.ndarray:
        return self._get("glc_model_get_grads")

    def get_moments(self) -> tuple[np.ndarray, np.ndarray]:
        m = np.empty(self.total, np.float32)
        v = np.empty(self.total, np.float32)
        self.ctx.check(
            self.ctx.lib.glc_model_get_moments(self.h, m.ctypes.data_as(C.c_void_p), v.ctypes.data_as(C.c_void_p),
                                               m.size),
            "glc_model_get_moments",
        )
        return m, v

    def LoadCheckpoint(self, path) -> int:
        """Loads the parameters of a SaveCheckpoint text file (trainer.go:554-584)
        and returns its step.  The file's dimensions must match this model."""
        from .checkpoint import read_checkpoint

        step, flat = read_checkpoint(path, self.Config)
        self.set_params(flat)
        return step

    def close(self) -> None:
        # a model whose context is already gone was closed with it
        if getattr(self, "h", None) and getattr(self.ctx, "h", None):
            self.ctx.lib.glc_model_destroy(self.h)
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def NewTrainableModel(cfg: TrainConfig, ctx: Context | None = None) -> TrainableModel:
    return TrainableModel(cfg, ctx)


class Trainer:
    """NewTrainer: AdamW + warmup/cosine LRScheduler + TrainStep."""

    def __init__(self, model: TrainableModel, cfg: TrainConfig | None = None):
        self.Model = model
        self.Config = cfg or model.Config
        self.ctx = model.ctx
        h = C.c_void_p()
        self.ctx.check(self.ctx.lib.glc_trainer_create(model.h, C.byref(h)), "glc_trainer_create")
        self.h = h
        self.ctx.adopt(self, 0)

    totalLoss = np.float32(0)  # loss tracking of TrainStep (trainer.go:441-442, :501-502)
    lossCount = 0

    def TrainStep(self, inputs, targets) -> float:
        inp = np.ascontiguousarray(inputs, np.int64)
        tgt = np.ascontiguousarray(targets, np.int64)
        if inp.ndim != 2 or inp.shape != tgt.shape:
            raise ValueError("inputs and targets must be [batch, seq] arrays of the same shape")
        B, S = inp.shape
        loss = C.c_float()
        self.ctx.check(
            self.ctx.lib.glc_train_step(self.h, inp.ctypes.data_as(C.c_void_p), tgt.ctypes.data_as(C.c_void_p), B, S,
                                        C.byref(loss)),
            "glc_train_step",
        )
        self.totalLoss = np.float32(self.totalLoss + np.float32(loss.value))
        self.lossCount += 1
        return float(loss.value)

    @property
    def step(self) -> int:
        return self.last_stats()[2]

    def Train(self, dataLoader, log=print) -> None:
        """Trainer.Train (trainer.go:508-551): TrainStep until MaxSteps, a log
        line every LogInterval steps, SaveCheckpoint every SaveInterval steps
        and once at the end."""
        train_loop(self, dataLoader, log)

    def last_stats(self) -> tuple[float, float, int]:
        n, lr, st = C.c_double(), C.c_float(), C.c_int()
        self.ctx.check(self.ctx.lib.glc_trainer_last_stats(self.h, C.byref(n), C.byref(lr), C.byref(st)),
                       "glc_trainer_last_stats")
        return n.value, lr.value, st.value

    def last_launches(self) -> int:
        n = C.c_uint64()
        self.ctx.check(self.ctx.lib.glc_trainer_last_launches(self.h, C.byref(n)), "glc_trainer_last_launches")
        return n.value

    def SaveCheckpoint(self) -> str:
        """Trainer.SaveCheckpoint (trainer.go:554-584): writes
        <Config.SavePath>/checkpoint_<step>.bin in the reference's text format
        and returns the path."""
        buf = C.create_string_buffer(4096)
        self.ctx.check(self.ctx.lib.glc_trainer_save_checkpoint(self.h, str(self.Config.SavePath).encode(), buf, 4096),
                       "glc_trainer_save_checkpoint")
        return buf.value.decode()

    def SaveState(self, path) -> None:
        """Binary resume file: parameters, AdamW m/v and step, scheduler step."""
        self.ctx.check(self.ctx.lib.glc_trainer_save_state(self.h, str(path).encode()), "glc_trainer_save_state")

    def LoadState(self, path) -> None:
        """Restores a SaveState file into this trainer and its model; the next
        TrainStep continues as the saved trainer's next step would."""
        self.ctx.check(self.ctx.lib.glc_trainer_load_state(self.h, str(path).encode()), "glc_trainer_load_state")

    def close(self) -> None:
        if getattr(self, "h", None) and getattr(self.ctx, "h", None):
            self.ctx.lib.glc_trainer_destroy(self.h)
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def NewTrainer(model: TrainableModel, cfg: TrainConfig | None = None) -> Trainer:
    return Trainer(model, cfg)


def train_loop(t, dataLoader, log=print) -> None:
    """The loop of Trainer.Train (trainer.go:508-551) over any trainer with
    TrainStep, step, last_stats, SaveCheckpoint, Config, totalLoss and
    lossCount.  Unlike the reference, an empty batch raises instead of
    looping forever (trainer.go:521-524 `continue`s without advancing)."""
    import os
    import time

    cfg = t.Config
    start = time.monotonic()
    os.makedirs(cfg.SavePath, exist_ok=True)
    log(f"Starting training: {cfg.MaxSteps} steps, batch_size={cfg.BatchSize}, lr={cfg.LearningRate:.2e}")
    while t.step < cfg.MaxSteps:
        inputs, targets = dataLoader.NextBatch()
        if inputs is None:
            raise ValueError("Train: the data loader returned an empty batch")
        loss = t.TrainStep(inputs, targets)
        step = t.step
        if step % cfg.LogInterval == 0:
            avg = np.float32(t.totalLoss) / np.float32(t.lossCount)
            steps_per_sec = step / max(time.monotonic() - start, 1e-9)
            lr = t.last_stats()[1]
            log(f"step {step} | loss: {loss:.4f} (avg: {avg:.4f}) | lr: {lr:.2e} | {steps_per_sec:.1f} steps/sec")
            t.totalLoss, t.lossCount = np.float32(0), 0
        if step % cfg.SaveInterval == 0:
            t.SaveCheckpoint()
    log(f"Training complete! Final step: {t.step}")
    t.SaveCheckpoint()


class Dataset:
    """Dataset (pkg/train/dataset.go:13-52): one token stream, training
    examples are windows of BlockSize tokens and their shift by one."""

    def __init__(self, tokens, blockSize: int):
        self.Tokens = np.asarray(tokens, np.int64)
        self.BlockSize = blockSize

    def Len(self) -> int:
        return 0 if len(self.Tokens) <= self.BlockSize else len(self.Tokens) - self.BlockSize

    def GetBatch(self, batchSize: int, rng: np.random.Generator):
        """Random window starts in [0, len - BlockSize - 1) (dataset.go:39-52);
        (None, None) when the stream is too short.  Go's math/rand stream is
        not reproduced: the starts come from numpy's generator, and a stream
        of exactly BlockSize + 1 tokens returns (None, None) where Go's
        rand.Intn(0) would panic."""
        max_start = len(self.Tokens) - self.BlockSize - 1
        if max_start <= 0:
            return None, None
        starts = rng.integers(0, max_start, batchSize)
        idx = starts[:, None] + np.arange(self.BlockSize)[None, :]
        return self.Tokens[idx], self.Tokens[idx + 1]


def NewDataset(tokens, blockSize: int) -> Dataset:
    return Dataset(tokens, blockSize)


class DataLoader:
    """DataLoader (dataset.go:55-75): batches of random windows from a seeded generator."""

    def __init__(self, dataset: Dataset, batchSize: int, shuffle: bool = True, seed: int = 0):
        self.Dataset, self.BatchSize, self.Shuffle = dataset, batchSize, shuffle
        self.rng = np.random.default_rng(seed)

    def NextBatch(self):
        return self.Dataset.GetBatch(self.BatchSize, self.rng)


def NewDataLoader(dataset: Dataset, batchSize: int, shuffle: bool = True, seed: int = 0) -> DataLoader:
    return DataLoader(dataset, batchSize, shuffle, seed)


__all__ = [
    "Dataset",
    "NewDataset",
    "DataLoader",
    "NewDataLoader",
    "train_loop",
    "TrainConfig",
    "DefaultTrainConfig",
    "config_for",
    "TrainableModel",
    "NewTrainableModel",
    "Trainer",
    "NewTrainer",
    "GlcError",
    "SEMANTICS_REFERENCE",
    "SEMANTICS_LLAMA",
]
