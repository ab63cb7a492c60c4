"""Shared helpers for the parity tests: tolerances, oracle configs, comparisons."""
from __future__ import annotations

import os

import numpy as np

from gollama_b200.synthetic import ModelShape
from oracle.oracle import Config, OptimState

# Bars (written here, used by every parity test):
LOSS_RTOL = 1e-4        # loss, relative
GRAD_RFRO = 2e-3        # every parameter gradient, relative Frobenius error
WEIGHT_RFRO = 2e-3      # every post-step weight, relative Frobenius error
FP32_RTOL = 2e-5        # fp32 CUDA-core kernels (reduction order differs from the oracle)


def rel_fro(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    nb = np.linalg.norm(b)
    if nb == 0:
        return float(np.linalg.norm(a))
    return float(np.linalg.norm(a - b) / nb)


def oracle_config(shape: ModelShape) -> Config:
    return Config(
        vocab=shape.vocab,
        hidden=shape.hidden,
        layers=shape.layers,
        heads=shape.heads,
        kv_heads=shape.kv_heads if shape.mode == 1 else shape.heads,
        inter=shape.inter,
        max_seq=shape.seq,
        norm_eps=shape.norm_eps,
        rope_theta=shape.rope_theta,
        mode=shape.mode,
    )


# one fwd+bwd+AdamW step: lr 3e-4, betas 0.9/0.95, wd 0.1, clip 1.0, no warmup
STEP_HPARAMS = dict(LearningRate=3e-4, WeightDecay=0.1, Beta1=0.9, Beta2=0.95, Epsilon=1e-8, WarmupSteps=0,
                    MaxSteps=10000, GradClipNorm=1.0)


def oracle_optim() -> OptimState:
    h = STEP_HPARAMS
    return OptimState(lr=0.0, beta1=h["Beta1"], beta2=h["Beta2"], eps=h["Epsilon"], weight_decay=h["WeightDecay"],
                      adam_step=0, initial_lr=h["LearningRate"], warmup_steps=h["WarmupSteps"],
                      total_steps=h["MaxSteps"], grad_clip=h["GradClipNorm"], trainer_step=0)


def threads() -> int:
    return max(1, min(64, os.cpu_count() or 1))
