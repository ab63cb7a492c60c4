#!/usr/bin/env python
"""Training throughput of the TinyLlama-1.1B-shaped decoder on B200.

One step = Trainer.TrainStep (pkg/train/trainer.go:462-505) in Llama
semantics: forward, softmax cross-entropy, backward, (data-parallel gradient
allreduce), gradient clipping and AdamW, for batch 4 x seq 1024 per GPU
(4096 tokens), 22 layers, d 2048, 32 query / 4 KV heads, FFN 5632, vocab
32000, random N(0, 0.02) weights and Zipf(1.1) token ids from a seed.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs one process per GPU under torch.distributed.run (RANK, LOCAL_RANK,
WORLD_SIZE from the environment); gradients are summed with NCCL.  Rank 0
prints one JSON line.

  value     tokens/s of the whole job, token ids resident in HBM, K steps timed
            with CUDA events on the compute stream, max over ranks
  e2e       the same through glc_train_step with token ids copied from pinned
            host memory every step and the loss read back every step
  roofline  the tcgen05 GEMM (the dominant kernel) timed per launch with CUDA
            events during extra profiled steps, against the TF32 peak
  cpu_baseline  the oracle (reference threading structure) on the host cores
            on a bounded sample of the same workload, extrapolated per token
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "train tokens/sec (fwd+bwd+AdamW)"
UNIT = "tokens/s"
PROF_NAMES = ["gemm_tf32", "attention_fwd", "attention_bwd", "rmsnorm", "swiglu", "softmax_ce", "adamw", "other"]
HPARAMS = dict(LearningRate=3e-4, WeightDecay=0.1, Beta1=0.9, Beta2=0.95, Epsilon=1e-8, WarmupSteps=0,
               MaxSteps=10000, GradClipNorm=1.0, Seed=1234)


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--profile-steps", type=int, default=2)
    ap.add_argument("--sample-tokens", type=int, default=2, help="tokens per CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--light", action="store_true",
                    help="skip the CPU baseline, the TF32 peak measurement and the profiled steps (for ncu launch lists)")
    ap.add_argument("--set", action="append", default=[], metavar="NAME=VALUE",
                    help="kernel variant switch glc_set_NAME(ctx, VALUE) before the run, e.g. rmsnorm_variant=2, "
                         "attention_fwd_variant=2 (repeatable; recorded in the JSON line's config)")
    a = ap.parse_args()
    for kv in a.set:
        name, _, val = kv.partition("=")
        if not name.isidentifier() or not val.lstrip("-").isdigit():
            ap.error(f"--set wants NAME=INTEGER, got {kv!r}")
    if a.light:
        a.no_cpu_baseline = True
        a.profile_steps = 0
    return a


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def workload_config(n_gpus: int):
    from gollama_b200 import synthetic as syn

    s = syn.TINYLLAMA
    return {
        "workload": "tinyllama-1.1b-shape train step",
        "model": "TinyLlama-1.1B-shaped decoder: 22 layers, d 2048, 32 query / 4 KV heads (GQA, head_dim 64), "
                 "SwiGLU FFN 5632, vocab 32000, RoPE, tied LM head",
        "semantics": "llama (RoPE, GQA, full backward)",
        "global_batch": s.batch * n_gpus,
        "batch_per_gpu": s.batch,
        "seq_len": s.seq,
        "tokens_per_gpu": s.tokens,
        "parallelism": f"dp{n_gpus}",
        "optimizer": "AdamW lr 3e-4 betas 0.9/0.95 wd 0.1, clip 1.0",
        "l2": "no flush needed: every step streams 4.1 GB of weights and ~20 GB of activations, far above the 126 MB L2",
    }


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, n_gpus: int = 1):
        self.proc = None
        self.path = None
        # only this job's GPUs: polling every GPU of a shared box takes driver
        # locks on all of them, and with data parallelism a stall on any rank
        # holds up every rank's next gradient sum
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "").strip()
        ids = [x.strip() for x in vis.split(",") if x.strip()] if vis else [str(i) for i in range(n_gpus)]
        self.ids = ",".join(ids[:n_gpus])

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.ids, f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        self.f.close()
        lines = Path(self.path).read_text().splitlines()
        os.unlink(self.path)
        return self.summarize(lines)

    @staticmethod
    def summarize(lines):
        """The clocks record of the timed region from nvidia-smi's CSV lines
        (QUERY's columns, no header, no units): median SM clock, the highest
        max clock, every throttle reason seen active, the sample count."""
        rows = []
        for line in lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": sorted(reasons),
            "samples": len(rows),
        }


# --------------------------------------------------------------------------- peaks
def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def measure_tf32_peak(device: int, seconds: float = 2.0):
    """cuBLAS TF32 GEMM 8192^3 back to back (sustained), the TF32 roofline denominator."""
    try:
        import torch

        torch.backends.cuda.matmul.allow_tf32 = True
        dev = torch.device("cuda", device)
        a = torch.randn(8192, 8192, device=dev)
        b = torch.randn(8192, 8192, device=dev)
        for _ in range(3):
            a @ b
        torch.cuda.synchronize(dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = 0
        s.record()
        t0 = time.time()
        while time.time() - t0 < seconds:
            for _ in range(20):
                a @ b
            n += 20
        e.record()
        torch.cuda.synchronize(dev)
        ms = s.elapsed_time(e)
        del a, b
        torch.cuda.empty_cache()
        return 2.0 * 8192**3 * n / (ms * 1e-3) / 1e12
    except Exception:
        return None


# --------------------------------------------------------------------------- CPU baseline
class CpuSampler:
    """The oracle with the reference's loop nests and threading (row-parallel
    forward GEMMs, single-threaded dA loop, N-parallel dB loop, everything
    else single-threaded), built like Go's amd64 code (oracle/
    liboracle_scalar.so: -O2, no vectorisation), on the host cores.

    A full TinyLlama-shape step takes the CPU hours, so one sample measures
    (a) forward + backward of the whole 22-layer model on one sequence of
    `sample_tokens` tokens (every GEMM, norm, SwiGLU and the 32000-wide LM head
    scale with the token count), and (b) one query head's causal attention
    forward + backward over a full 1024-token sequence (what (a) runs at a
    sequence of `sample_tokens` only); clip + AdamW is timed once on a 2-layer
    model of the same widths.  Per step (extrapolated):
        4096 / sample_tokens * (a) + (4 sequences * 32 heads * 22 layers) * (b)
        + clip/AdamW per parameter * 1.03e9.
    It also measures whole reference-semantics TrainSteps of the tiny
    configuration (2 layers, d 128, vocab 256, 4 x 64 tokens), end to end."""

    def __init__(self, sample_tokens: int):
        from gollama_b200 import synthetic as syn
        from oracle.oracle import Config, Oracle

        self.syn = syn
        s = self.shape = syn.TINYLLAMA
        self.sample_tokens = sample_tokens
        self.threads = os.cpu_count() or 1
        self.orc = Oracle(threads=self.threads, literal=True, scalar=True)
        self.cfg = Config(vocab=s.vocab, hidden=s.hidden, layers=s.layers, heads=s.heads, kv_heads=s.kv_heads,
                          inter=s.inter, max_seq=s.seq, norm_eps=s.norm_eps, rope_theta=s.rope_theta, mode=1)
        n = self.n_params = self.orc.param_total(self.cfg)
        rng = np.random.default_rng(0)
        self.params = rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)
        for off, r, c in self.orc.param_layout(self.cfg):
            if r == 1:
                self.params[off:off + c] = 1.0
        self.inp = syn.zipf_tokens(7, (1, sample_tokens), s.vocab)
        self.tgt = syn.zipf_tokens(8, (1, sample_tokens), s.vocab)
        hd = s.head_dim
        self.q1 = rng.standard_normal((s.seq, hd), dtype=np.float32)
        self.k1 = rng.standard_normal((s.seq, hd), dtype=np.float32)
        self.v1 = rng.standard_normal((s.seq, hd), dtype=np.float32)
        self.do1 = rng.standard_normal((s.seq, hd), dtype=np.float32)
        # gradient buffers of the whole model, allocated and touched once (the
        # reference allocates its gradients once and ZeroGrad clears them every
        # step: a per-step cost, timed here as zero_s, not a per-token one)
        self.grads = np.zeros(n, np.float32)
        self.has = np.zeros(len(self.orc.param_layout(self.cfg)), np.uint8)
        self.grads.fill(0.0)  # first touch
        t0 = time.perf_counter()
        self.grads.fill(0.0)
        self.zero_s = time.perf_counter() - t0
        self.opt_s = self._optimizer_seconds()
        self.tiny = self._tiny_step()

    def _optimizer_seconds(self) -> float:
        from oracle.oracle import Config, OptimState, TrainState

        s = self.shape
        small = Config(vocab=s.vocab, hidden=s.hidden, layers=2, heads=s.heads, kv_heads=s.kv_heads, inter=s.inter,
                       max_seq=s.seq, norm_eps=s.norm_eps, rope_theta=s.rope_theta, mode=1)
        orc = self.orc
        ns = orc.param_total(small)
        st = TrainState.create(np.full(ns, 0.01, np.float32), len(orc.param_layout(small)),
                               OptimState(beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, lr=3e-4, grad_clip=1.0))
        st.grads[:] = 1e-3
        st.has_grad[:] = 1
        t0 = time.perf_counter()
        orc.fn("grad_clip")(st.grads.ctypes.data_as(C.c_void_p), st.has_grad.ctypes.data_as(C.c_void_p),
                            C.byref(small), C.c_float(1.0))
        orc.fn("adamw_step")(st.params.ctypes.data_as(C.c_void_p), st.grads.ctypes.data_as(C.c_void_p),
                             st.has_grad.ctypes.data_as(C.c_void_p), st.m.ctypes.data_as(C.c_void_p),
                             st.v.ctypes.data_as(C.c_void_p), C.byref(small), C.byref(st.opt))
        return (time.perf_counter() - t0) / ns * self.n_params

    def _tiny_step(self) -> dict:
        """Whole TrainSteps (reference semantics, pkg/train/trainer.go:462-505)
        of the tiny configuration, timed end to end."""
        from oracle.oracle import Config, OptimState, TrainState

        shape = self.syn.TINY
        params = self.syn.init_params(shape, 1)
        inp, tgt = self.syn.batch(shape, 1)
        ocfg = Config(vocab=shape.vocab, hidden=shape.hidden, layers=shape.layers, heads=shape.heads,
                      kv_heads=shape.heads, inter=shape.inter, max_seq=shape.seq, norm_eps=shape.norm_eps,
                      rope_theta=shape.rope_theta, mode=0)
        opt = OptimState(lr=0.0, beta1=HPARAMS["Beta1"], beta2=HPARAMS["Beta2"], eps=HPARAMS["Epsilon"],
                         weight_decay=HPARAMS["WeightDecay"], adam_step=0, initial_lr=HPARAMS["LearningRate"],
                         warmup_steps=HPARAMS["WarmupSteps"], total_steps=HPARAMS["MaxSteps"],
                         grad_clip=HPARAMS["GradClipNorm"], trainer_step=0)
        st = TrainState.create(params, len(self.orc.param_layout(ocfg)), opt)
        self.orc.train_step(ocfg, st, inp, tgt)  # warm-up
        times = []
        for _ in range(3):
            t0 = time.perf_counter()
            self.orc.train_step(ocfg, st, inp, tgt)
            times.append(time.perf_counter() - t0)
        sec = statistics.median(times)
        return {"config": "tiny: 2 layers, d 128, 4 heads, FFN 344, vocab 256, batch 4 x seq 64, reference semantics",
                "s_per_step": sec, "tokens_per_s": shape.tokens / sec, "measured": "3 whole steps, median"}

    def sample(self) -> tuple[float, float]:
        """One sample: (a) seconds, (b) seconds."""
        t0 = time.perf_counter()
        self.orc.fn("forward_backward")(C.byref(self.cfg), self.params.ctypes.data_as(C.c_void_p),
                                        self.grads.ctypes.data_as(C.c_void_p), self.has.ctypes.data_as(C.c_void_p),
                                        self.inp.ctypes.data_as(C.c_void_p), self.tgt.ctypes.data_as(C.c_void_p), 1,
                                        self.sample_tokens, 1)
        a = time.perf_counter() - t0
        S, hd = self.shape.seq, self.shape.head_dim
        t0 = time.perf_counter()
        self.orc.attention_fwd(self.q1, self.k1, self.v1, S, 1, 1, hd)
        self.orc.attention_bwd(self.q1, self.k1, self.v1, self.do1, S, 1, 1, hd)
        b = time.perf_counter() - t0
        return a, b

    def step_seconds(self, a: float, b: float) -> float:
        s = self.shape
        return (s.tokens / self.sample_tokens) * a + (s.batch * s.heads * s.layers) * b + self.zero_s + self.opt_s

    def baseline(self, samples) -> dict:
        a = statistics.mean(x[0] for x in samples)
        b = statistics.mean(x[1] for x in samples)
        sec = self.step_seconds(a, b)
        return {
            "value": self.shape.tokens / sec,
            "unit": UNIT,
            "cores": self.threads,
            "kind": "port",
            "sample": (f"extrapolated: the oracle with the reference's loop nests and threading, built like Go's amd64 "
                       f"code (-O2, no vectorisation), {len(samples)} sample(s): forward+backward of the 22-layer "
                       f"TinyLlama-shape model on 1 sequence x {self.sample_tokens} tokens ({a:.2f} s) and one query "
                       f"head's causal attention fwd+bwd over 1024 tokens ({b:.3f} s); ZeroGrad of 1.03e9 gradients "
                       f"({self.zero_s:.1f} s) and clip+AdamW over them from a 2-layer model ({self.opt_s:.1f} s); "
                       f"per step = {self.shape.tokens}/{self.sample_tokens} x (a) + 2816 x (b) + ZeroGrad + "
                       f"optimizer = {sec:.0f} s"),
            "measured_tiny_step": self.tiny,
        }


# --------------------------------------------------------------------------- reference arm
def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    from gollama_b200 import synthetic as syn

    tokens_per_step = syn.TINYLLAMA.tokens
    W, K = max(0, args.warmup), max(1, args.steps)
    sampler = CpuSampler(args.sample_tokens)
    samples = [sampler.sample() for _ in range(W + K)][W:]
    base = sampler.baseline(samples)
    v = base["value"]
    out = {
        "impl": "reference",
        "metric": METRIC,
        "value": v,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": tokens_per_step / v * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded Zipf(1.1) token ids, random N(0,0.02) weights)",
        "config": workload_config(args.gpus),
        "cpu_baseline": base,
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("the reference is pure Go and no Go toolchain exists here; this arm times the C restatement of its "
                 "trainer (oracle/) with the reference's threading structure on the host cores"),
    }
    print(json.dumps(out), flush=True)
    return 0


# --------------------------------------------------------------------------- our arm
def run_ours(args):
    rank, world, local = dist_env()
    if world != args.gpus:
        world = max(world, 1)
    from gollama_b200 import synthetic as syn
    from gollama_b200.device import Context
    from gollama_b200.train import NewTrainableModel, NewTrainer, config_for

    ctx = Context(local)
    lib = ctx.lib
    for kv in args.set:
        name, _, val = kv.partition("=")
        ctx.call(f"glc_set_{name}", int(val))
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("gloo", init_method="env://", timeout=datetime.timedelta(seconds=300))
        pg = dist
        uid = (C.c_ubyte * 128)()
        if rank == 0:
            assert lib.glc_dp_unique_id(uid) == 0, "ncclGetUniqueId failed"
        obj = [bytes(uid)]
        dist.broadcast_object_list(obj, src=0)
        uid = (C.c_ubyte * 128).from_buffer_copy(obj[0])
        ctx.call("glc_dp_init", rank, world, uid, 300000)

    shape = syn.TINYLLAMA
    cfg = config_for(shape, WorldSize=world, **HPARAMS)
    model = NewTrainableModel(cfg, ctx)
    tr = NewTrainer(model)
    B, S, T = shape.batch, shape.seq, shape.tokens
    K, W, P = args.steps, args.warmup, args.profile_steps
    nb = max(1, K)
    batches = [syn.batch(shape, 1_000_003 * rank + 17 * i + 5) for i in range(nb)]
    dev_in = [ctx.from_numpy(b[0]) for b in batches]
    dev_tg = [ctx.from_numpy(b[1]) for b in batches]
    loss = C.c_float()

    def step_device(i):
        j = i % nb
        ctx.check(lib.glc_train_step_device(tr.h, dev_in[j].ptr, dev_tg[j].ptr, B, S, C.byref(loss)),
                  "glc_train_step_device")

    # pinned host staging for the end-to-end measurement
    nbytes = T * 8
    pin = C.c_void_p()
    ctx.call("glc_host_alloc", 2 * nb * nbytes, C.byref(pin))
    pin_base = pin.value
    for i, (bi, bt) in enumerate(batches):
        C.memmove(pin_base + (2 * i) * nbytes, bi.ctypes.data, nbytes)
        C.memmove(pin_base + (2 * i + 1) * nbytes, bt.ctypes.data, nbytes)

    def step_e2e(i):
        j = i % nb
        ctx.check(lib.glc_train_step(tr.h, C.c_void_p(pin_base + 2 * j * nbytes), C.c_void_p(pin_base + (2 * j + 1) * nbytes),
                                     B, S, C.byref(loss)), "glc_train_step")

    def barrier():
        if world > 1:
            ctx.call("glc_dp_barrier")

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        v = C.c_double(x)
        ctx.call("glc_dp_allreduce_max_host", C.byref(v))
        return v.value

    for i in range(W):
        step_device(i)
    ctx.sync()
    # the sampler starts (and settles) before the barrier, so every rank's
    # timer starts together
    sampler = ClockSampler(world) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier()
    l0 = ctx.launches()
    ms = C.c_float()
    ctx.call("glc_timer_start")
    for i in range(K):
        step_device(i)
    ctx.call("glc_timer_stop", C.byref(ms))
    launches = ctx.launches() - l0
    clocks = sampler.stop() if sampler else None
    t_dev = max_over_ranks(ms.value)
    last_loss = loss.value

    barrier()
    e2e_ms = C.c_float()
    ctx.call("glc_timer_start")
    for i in range(K):
        step_e2e(i)
    ctx.call("glc_timer_stop", C.byref(e2e_ms))
    t_e2e = max_over_ranks(e2e_ms.value)

    barrier()
    counts = (C.c_uint64 * 8)()
    tms = (C.c_double * 8)()
    work = (C.c_double * 8)()
    ctx.call("glc_profile_begin")
    for i in range(P):
        step_device(i)
    ctx.call("glc_profile_end", 8, counts, tms, work)
    grad_norm, lr, nstep = tr.last_stats()
    if world > 1:
        barrier()
        ctx.call("glc_dp_destroy")
        pg.destroy_process_group()
    if rank != 0:
        return 0

    peaks, peak_src = measured_peaks()
    # The GEMMs run kind::tf32, whose dense rate is half the bf16 rate; they are
    # timed inside a long step, so the denominator is half the sustained bf16
    # figure.  cuBLAS's own TF32 GEMM is measured alongside for context.
    tc_peak = peaks["bf16_tflops_sustained"] / 2
    tc_src = (f"{peak_src}: bf16_tflops_sustained {peaks['bf16_tflops_sustained']} / 2 "
              f"(dense TF32 runs at half the bf16 rate)")
    cublas_tf32 = None if args.light else measure_tf32_peak(local)
    prof_ms_step = {n: tms[i] / max(P, 1) for i, n in enumerate(PROF_NAMES)}
    tot_prof = sum(tms) or 1.0
    kernels = {}
    for i, n in enumerate(PROF_NAMES):
        if counts[i] == 0:
            continue
        d = {"launches_per_step": counts[i] / max(P, 1), "ms_per_step": prof_ms_step[n], "share": tms[i] / tot_prof}
        if tms[i] > 0 and work[i] > 0:
            if i in (0, 1, 2):
                d["tflops"] = work[i] / (tms[i] * 1e-3) / 1e12
            else:
                d["gbs"] = work[i] / (tms[i] * 1e-3) / 1e9
        kernels[n] = d
    gemm_avg_ms = tms[0] / max(counts[0], 1)
    gemm_flops_per_launch = work[0] / max(counts[0], 1)
    achieved = gemm_flops_per_launch / (gemm_avg_ms * 1e-3) / 1e12 if gemm_avg_ms > 0 else 0.0
    traffic = None
    tfile = ROOT / "profiles" / "gemm_tf32_traffic.txt"
    if tfile.exists():
        for line in tfile.read_text().splitlines():
            if line.startswith("bytes_per_launch_tinyllama_step_avg:"):
                traffic = float(line.split(":", 1)[1])
    roofline = {
        "kernel": "gemm_tf32 (tcgen05.mma kind::tf32, TMA, TMEM), all linear-layer forward/dX/dW GEMMs of the step",
        "bound": "tensor",
        "achieved": achieved,
        "peak": tc_peak,
        "unit": "TFLOP/s",
        "frac": achieved / tc_peak if tc_peak else None,
        "traffic": traffic,
        "peak_source": tc_src,
        "cublas_tf32_tflops": cublas_tf32,
        "traffic_source": ("profiles/gemm_tf32_traffic.txt (ncu, one bounded capture per GEMM shape of the step, "
                           "weighted by its launches per step)"),
        "flops_per_launch_avg": gemm_flops_per_launch,
        "avg_launch_ms": gemm_avg_ms,
        "launches_per_step": counts[0] / max(P, 1),
    }
    value = world * T * K / (t_dev * 1e-3)
    e2e_value = world * T * K / (t_e2e * 1e-3)
    out = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": t_dev / K,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "tf32",
        "data": "synthetic (seeded Zipf(1.1) token ids, random N(0,0.02) weights)",
        "config": dict(workload_config(world), **({"variants": dict(kv.split("=", 1) for kv in args.set)}
                                                   if args.set else {})),
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": 2 * T * 8, "d2h_bytes_per_step": 16,
                "ms_per_step": t_e2e / K},
        "roofline": roofline,
        "gpu_launches": int(launches),
        "clocks": clocks,
        "kernels": kernels,
        "last_loss": last_loss,
        "grad_norm": grad_norm,
        "hbm_peak_gbs": peaks.get("hbm_gbs"),
        "peaks_source": peak_src,
    }
    if world == 1 and not args.no_cpu_baseline:
        sampler = CpuSampler(args.sample_tokens)
        out["cpu_baseline"] = sampler.baseline([sampler.sample()])
    print(json.dumps(out), flush=True)
    return 0


def main():
    args = parse_args()
    # rank 0's stdout must be exactly one JSON line: NCCL's log (its version
    # banner included, printed at level WARN) goes to stderr
    os.environ.setdefault("NCCL_DEBUG", "WARN")
    os.environ["NCCL_DEBUG_FILE"] = "/dev/stderr"
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
