"""Microbenchmarks of single kernels at the TinyLlama training shapes.

    python -m gollama_b200.microbench CASE [--iters N] [--warmup W]

Each case allocates its operands once (seeded normal values, rounded to TF32
where the training step feeds the tensor cores rounded operands), runs the
kernel W times untimed and N times timed with CUDA events on the library's
compute stream, and prints one line: case, shape, ms per launch, and TFLOP/s
(tensor-core kernels) or GB/s (bandwidth kernels) of algorithmic work.  Used
for ncu captures of one kernel on a bounded case.
"""
from __future__ import annotations

import argparse
import ctypes as C

import numpy as np

from .device import Context

T, D, F, H, HKV, HD, S, V = 4096, 2048, 5632, 32, 4, 64, 1024, 32000


def _tf32(x: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((b + np.uint32(0x1000)) & np.uint32(0xFFFFE000)).view(np.float32)


def _rand(ctx, shape, seed, scale=1.0, tf32=True):
    x = (np.random.default_rng(seed).standard_normal(shape, dtype=np.float32) * np.float32(scale))
    return ctx.from_numpy(_tf32(x) if tf32 else x)


def _time(ctx, fn, iters, warmup):
    for _ in range(warmup):
        fn()
    ctx.sync()
    ms = C.c_float()
    ctx.call("glc_timer_start")
    for _ in range(iters):
        fn()
    ctx.call("glc_timer_stop", C.byref(ms))
    ctx.sync()
    return ms.value / max(iters, 1)


def case_gemm(ctx, kind, M, K, N, iters, warmup):
    """kind: fwd Y=X.W^T, dx dX=dY.W, dw dW=dY^T.X, bwd (dx and dw grouped)."""
    X, W, G = _rand(ctx, (M, K), 1), _rand(ctx, (N, K), 2), _rand(ctx, (M, N), 3)
    Y, dX, dW = ctx.empty((M, N)), ctx.empty((M, K)), ctx.empty((N, K))
    calls = {
        "fwd": lambda: ctx.call("glc_linear_fwd", X.ptr, W.ptr, Y.ptr, M, K, N, None),
        "dx": lambda: ctx.call("glc_linear_bwd_dx", G.ptr, W.ptr, dX.ptr, M, K, N, 0),
        "dw": lambda: ctx.call("glc_linear_bwd_dw", G.ptr, X.ptr, dW.ptr, M, K, N, 0),
        "bwd": lambda: ctx.call("glc_linear_bwd", G.ptr, X.ptr, W.ptr, dX.ptr, dW.ptr, M, K, N, 0, 0),
    }
    ms = _time(ctx, calls[kind], iters, warmup)
    flops = 2.0 * M * N * K * (2 if kind == "bwd" else 1)
    return f"gemm_{kind} M={M} K={K} N={N}", ms, flops / (ms * 1e-3) / 1e12, "TFLOP/s"


def case_gemm_majors(ctx, iters, warmup, M=16384, N=2048, K=2048):
    """C[M,N] = A . B^T through glc_gemm_tf32 with each operand K- or MN-major."""
    out = []
    A_k, A_m = _rand(ctx, (M, K), 21), _rand(ctx, (K, M), 22)
    B_k, B_m = _rand(ctx, (N, K), 23), _rand(ctx, (K, N), 24)
    Cm = ctx.empty((M, N))
    for am in (0, 1):
        for bm in (0, 1):
            A, lda = (A_m, M) if am else (A_k, K)
            B, ldb = (B_m, N) if bm else (B_k, K)
            f = lambda: ctx.call("glc_gemm_tf32", A.ptr, lda, am, B.ptr, ldb, bm, Cm.ptr, N, M, N, K, 0, None, 0, 0)
            ms = _time(ctx, f, iters, warmup)
            out.append((f"gemm A{'mn' if am else 'k'} B{'mn' if bm else 'k'} M={M} N={N} K={K}", ms,
                        2.0 * M * N * K / (ms * 1e-3) / 1e12, "TFLOP/s"))
    return out


def case_linear_sweep(ctx, iters, warmup):
    """Linear-layer sweep: M in {4096, 16384, 32768} x (K, N) in {(2048, 2048),
    (2048, 5632), (5632, 2048)}, forward, dX and dW separately."""
    out = []
    for M in (4096, 16384, 32768):
        for K, N in ((2048, 2048), (2048, 5632), (5632, 2048)):
            for kind in ("fwd", "dx", "dw"):
                out.append(case_gemm(ctx, kind, M, K, N, iters, warmup))
    return out


def case_attention(ctx, kind, iters, warmup, B=4, S=S):
    Tq = B * S
    q, k, v = _rand(ctx, (Tq, H * HD), 4), _rand(ctx, (Tq, HKV * HD), 5), _rand(ctx, (Tq, HKV * HD), 6)
    dO = _rand(ctx, (Tq, H * HD), 7)
    o, lse = ctx.empty((Tq, H * HD)), ctx.empty((B, H, S))
    dq, dk, dv = ctx.empty((Tq, H * HD)), ctx.empty((Tq, HKV * HD)), ctx.empty((Tq, HKV * HD))
    fwd = lambda: ctx.call("glc_attention_fwd", q.ptr, k.ptr, v.ptr, o.ptr, lse.ptr, B, S, H, HKV, HD, 1)
    fwd()
    ctx.sync()
    bwd = lambda: ctx.call("glc_attention_bwd", q.ptr, k.ptr, v.ptr, o.ptr, lse.ptr, dO.ptr, dq.ptr, dk.ptr, dv.ptr,
                           B, S, H, HKV, HD, 1)
    causal = 0.5 * S * (S + 1)
    if kind == "fwd":
        ms, flops = _time(ctx, fwd, iters, warmup), 4.0 * B * H * causal * HD
    else:
        ms, flops = _time(ctx, bwd, iters, warmup), 8.0 * B * H * causal * HD
    return f"attention_{kind} B={B} S={S} H={H}/{HKV} hd={HD}", ms, flops / (ms * 1e-3) / 1e12, "TFLOP/s"


def case_quant_dx(ctx, qtype, iters, warmup, M=16384, K=D, N=F):
    """dX [M, K] = dY [M, N] . deq(W) with W [N, K] stored as Q8_0 (8), Q4_0 (2),
    Q4_K (12) or Q6_K (14): fp16 scales U(0.005, 0.02), every other byte random."""
    r = np.random.default_rng(qtype)
    be, bb, halves = {8: (32, 34, [0]), 2: (32, 18, [0]), 12: (256, 144, [0, 2]), 14: (256, 210, [208])}[qtype]
    nb = N * K // be
    raw = r.integers(0, 256, (nb, bb), dtype=np.uint8)
    for off in halves:
        raw[:, off : off + 2] = r.uniform(0.005, 0.02, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    w = ctx.from_numpy(raw.reshape(-1))
    dy, dx = _rand(ctx, (M, N), 15), ctx.empty((M, K))
    ms = _time(ctx, lambda: ctx.call("glc_linear_bwd_dx_q", dy.ptr, w.ptr, qtype, dx.ptr, M, K, N, 0), iters, warmup)
    name = {8: "Q8_0", 2: "Q4_0", 12: "Q4_K", 14: "Q6_K"}[qtype]
    return f"linear_bwd_dx_q {name} M={M} K={K} N={N}", ms, 2.0 * M * N * K / (ms * 1e-3) / 1e12, "TFLOP/s"


def case_gateup_swiglu(ctx, iters, warmup, M=T, K=D, F=F):
    """Gate/up projection with the SwiGLU epilogue (one launch) against the
    GEMM alone."""
    X, W = _rand(ctx, (M, K), 25), _rand(ctx, (2 * F, K), 26, 0.05)
    GU, Hh = ctx.empty((M, 2 * F)), ctx.empty((M, F))
    ms = _time(ctx, lambda: ctx.call("glc_linear_fwd_swiglu", X.ptr, W.ptr, GU.ptr, Hh.ptr, M, K, F, 1), iters, warmup)
    return f"gate/up GEMM + SwiGLU M={M} K={K} F={F}", ms, 2.0 * M * 2 * F * K / (ms * 1e-3) / 1e12, "TFLOP/s"


def case_swiglu(ctx, iters, warmup):
    gu = _rand(ctx, (T, 2 * F), 8, tf32=False)
    dh = _rand(ctx, (T, F), 9, tf32=False)
    dgu = ctx.empty((T, 2 * F))
    n = T * F
    ms = _time(ctx, lambda: ctx.call("glc_swiglu_bwd", gu.ptr, C.c_void_p(gu.addr + 4 * n), dh.ptr, dgu.ptr,
                                     C.c_void_p(dgu.addr + 4 * n), n, 0, 1), iters, warmup)
    return f"swiglu_bwd n={n}", ms, 20.0 * n / (ms * 1e-3) / 1e9, "GB/s"


def case_rmsnorm(ctx, iters, warmup, T=T):
    x, w, dy = _rand(ctx, (T, D), 10, tf32=False), _rand(ctx, (D,), 11, tf32=False), _rand(ctx, (T, D), 12, tf32=False)
    y, rms = ctx.empty((T, D)), ctx.empty((T,))
    ctx.call("glc_rmsnorm_fwd", x.ptr, w.ptr, y.ptr, rms.ptr, T, D, C.c_float(1e-5), 1)
    dx, dxr, dw = ctx.zeros((T, D)), ctx.empty((T, D)), ctx.zeros((D,))
    ms = _time(ctx, lambda: ctx.call("glc_rmsnorm_bwd", x.ptr, w.ptr, rms.ptr, dy.ptr, dx.ptr, dxr.ptr, dw.ptr, T, D,
                                     1, 1, 1), iters, warmup)
    return f"rmsnorm_bwd {T}x{D}", ms, 5.0 * 4 * T * D / (ms * 1e-3) / 1e9, "GB/s"


def case_rmsnorm_fwd(ctx, iters, warmup):
    x, w = _rand(ctx, (T, D), 10, tf32=False), _rand(ctx, (D,), 11, tf32=False)
    y, rms = ctx.empty((T, D)), ctx.empty((T,))
    ms = _time(ctx, lambda: ctx.call("glc_rmsnorm_fwd", x.ptr, w.ptr, y.ptr, rms.ptr, T, D, C.c_float(1e-5), 1),
               iters, warmup)
    return f"rmsnorm_fwd {T}x{D}", ms, 2.0 * 4 * T * D / (ms * 1e-3) / 1e9, "GB/s"


def case_optimizer(ctx, iters, warmup, n=1 << 28):
    """Clip norm and AdamW over one 2^28-parameter segment (5 fp32 arenas,
    5.4 GB), clip scale 0.5 so the clipped gradient is written back:
    norm 4 B/parameter, AdamW 36 B/parameter."""
    r = np.random.default_rng(15)
    p = ctx.from_numpy((r.standard_normal(n, dtype=np.float32) * np.float32(0.02)))
    g = ctx.from_numpy((r.standard_normal(n, dtype=np.float32) * np.float32(1e-3)))
    m, v, sh = ctx.zeros((n,)), ctx.zeros((n,)), ctx.empty((n,))
    segs = np.array([0, n], np.int64)
    sp = segs.ctypes.data_as(C.c_void_p)
    norm, nscale = ctx.empty((2,)), ctx.empty((1,))  # a float64 and a float32
    scale = ctx.from_numpy(np.array([0.5], np.float32))
    ms_n = _time(ctx, lambda: ctx.call("glc_grad_clip_norm", g.ptr, sp, 1, C.c_float(1.0), norm.ptr, nscale.ptr),
                 iters, warmup)
    ms_a = _time(ctx, lambda: ctx.call("glc_adamw_step", p.ptr, g.ptr, m.ptr, v.ptr, sh.ptr, sp, 1, scale.ptr,
                                       C.c_float(3e-4), C.c_float(0.9), C.c_float(0.95), C.c_float(1e-8),
                                       C.c_float(0.1), 1), iters, warmup)
    return [(f"grad_clip_norm n={n}", ms_n, 4.0 * n / (ms_n * 1e-3) / 1e9, "GB/s"),
            (f"adamw n={n} (clipped)", ms_a, 36.0 * n / (ms_a * 1e-3) / 1e9, "GB/s")]


def case_ce(ctx, iters, warmup, T=T):
    logits = _rand(ctx, (T, V), 13, 2.0, tf32=False)
    tg = ctx.from_numpy(np.random.default_rng(14).integers(0, V, T).astype(np.int64))
    logp, loss = ctx.empty((T,)), ctx.empty((1,))
    ms = _time(ctx, lambda: ctx.call("glc_softmax_ce", logits.ptr, tg.ptr, T, V, C.c_float(1.0 / T), logp.ptr,
                                     loss.ptr, 0, 0), iters, warmup)
    return f"softmax_ce {T}x{V}", ms, 4.0 * T * V / (ms * 1e-3) / 1e9, "GB/s"


def case_ce_grad(ctx, iters, warmup, T=T):
    """The loss and the gradient written over the logits (8 B per logit); the
    later iterations take the earlier gradients as logits."""
    logits = _rand(ctx, (T, V), 13, 2.0, tf32=False)
    tg = ctx.from_numpy(np.random.default_rng(14).integers(0, V, T).astype(np.int64))
    logp, loss = ctx.empty((T,)), ctx.empty((1,))
    ms = _time(ctx, lambda: ctx.call("glc_softmax_ce", logits.ptr, tg.ptr, T, V, C.c_float(1.0 / T), logp.ptr,
                                     loss.ptr, 1, 1), iters, warmup)
    return f"softmax_ce + gradient {T}x{V}", ms, 8.0 * T * V / (ms * 1e-3) / 1e9, "GB/s"


def case_ce_llama(ctx, iters, warmup, T=T):
    """The Llama-mode step's call: expf, the gradient written over the logits
    and rounded to TF32."""
    logits = _rand(ctx, (T, V), 13, 2.0, tf32=False)
    tg = ctx.from_numpy(np.random.default_rng(14).integers(0, V, T).astype(np.int64))
    logp, loss = ctx.empty((T,)), ctx.empty((1,))
    ms = _time(ctx, lambda: ctx.call("glc_softmax_ce_llama", logits.ptr, tg.ptr, T, V, C.c_float(1.0 / T), logp.ptr,
                                     loss.ptr, 1, 1), iters, warmup)
    return f"softmax_ce_llama + gradient {T}x{V}", ms, 8.0 * T * V / (ms * 1e-3) / 1e9, "GB/s"


def case_config4_sweep(ctx, iters, warmup):
    """The isolated backward-op sweep at its stated sizes: linear grads for M in
    {4096, 16384, 32768} x (K, N) in {(2048, 2048), (2048, 5632), (5632, 2048)};
    RMSNorm backward 32768 x 2048; causal attention backward B 4, 32 heads,
    head_dim 64, seq 2048; softmax-CE backward on 32768 x 32000 logits N(0, 2)."""
    out = list(case_linear_sweep(ctx, iters, warmup))
    out.append(case_rmsnorm(ctx, iters, warmup, T=32768))
    out.append(case_attention(ctx, "bwd", iters, warmup, B=4, S=2048))
    out.append(case_ce(ctx, iters, warmup, T=32768))
    return out


CASES = {
    "gemm_fwd": lambda c, i, w: case_gemm(c, "fwd", T, D, D, i, w),
    "gemm_dx": lambda c, i, w: case_gemm(c, "dx", T, D, D, i, w),
    "gemm_dw": lambda c, i, w: case_gemm(c, "dw", T, D, D, i, w),
    "gemm_bwd": lambda c, i, w: case_gemm(c, "bwd", T, D, D, i, w),
    "gemm_fwd_gateup": lambda c, i, w: case_gemm(c, "fwd", T, D, 2 * F, i, w),
    "gemm_fwd_lmhead": lambda c, i, w: case_gemm(c, "fwd", T, D, V, i, w),
    "gemm_fwd_8192": lambda c, i, w: case_gemm(c, "fwd", 8192, 8192, 8192, i, w),
    "gemm_dx_lmhead": lambda c, i, w: case_gemm(c, "dx", T, D, V, i, w),
    "gemm_dw_lmhead": lambda c, i, w: case_gemm(c, "dw", T, D, V, i, w),
    "gemm_bwd_lmhead": lambda c, i, w: case_gemm(c, "bwd", T, D, V, i, w),
    "gemm_bwd_down": lambda c, i, w: case_gemm(c, "bwd", T, F, D, i, w),
    "gemm_fwd_down": lambda c, i, w: case_gemm(c, "fwd", T, F, D, i, w),
    "gemm_fwd_qkv": lambda c, i, w: case_gemm(c, "fwd", T, D, D + 2 * D // 8, i, w),
    "gemm_bwd_qkv": lambda c, i, w: case_gemm(c, "bwd", T, D, D + 2 * D // 8, i, w),
    "gemm_bwd_gateup": lambda c, i, w: case_gemm(c, "bwd", T, D, 2 * F, i, w),
    "linear_sweep": case_linear_sweep,
    "gemm_majors": case_gemm_majors,
    "attention_fwd": lambda c, i, w: case_attention(c, "fwd", i, w),
    "attention_bwd": lambda c, i, w: case_attention(c, "bwd", i, w),
    "attention_fwd_s2048": lambda c, i, w: case_attention(c, "fwd", i, w, S=2048),
    "attention_bwd_s2048": lambda c, i, w: case_attention(c, "bwd", i, w, S=2048),
    "attention_fwd_s256": lambda c, i, w: case_attention(c, "fwd", i, w, B=16, S=256),
    "attention_bwd_s256": lambda c, i, w: case_attention(c, "bwd", i, w, B=16, S=256),
    "swiglu_bwd": case_swiglu,
    "gateup_swiglu": case_gateup_swiglu,
    "quant_dx_q8_0": lambda c, i, w: case_quant_dx(c, 8, i, w),
    "quant_dx_q4_0": lambda c, i, w: case_quant_dx(c, 2, i, w),
    "quant_dx_q4_k": lambda c, i, w: case_quant_dx(c, 12, i, w),
    "quant_dx_q6_k": lambda c, i, w: case_quant_dx(c, 14, i, w),
    "rmsnorm_bwd": case_rmsnorm,
    "config4_sweep": case_config4_sweep,
    "rmsnorm_fwd": case_rmsnorm_fwd,
    "optimizer": case_optimizer,
    "softmax_ce": case_ce,
    "softmax_ce_grad": case_ce_grad,
    "softmax_ce_llama": case_ce_llama,
}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("cases", nargs="+", choices=sorted(CASES) + ["all"])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--variant", type=int, default=0, choices=[0, 1, 2],
                    help="GEMM tiles: 0 automatic, 1 single-CTA 128x256, 2 CTA-pair 256x256")
    ap.add_argument("--attn-split", type=int, default=0,
                    help="attention backward: dK/dV CTAs per KV head (0 automatic, else a divisor of H/Hkv)")
    ap.add_argument("--rmsnorm-variant", type=int, default=0, choices=[0, 1, 2, 3],
                    help="RMSNorm backward: 0 automatic, 1 row by row, 2 cp.async-pipelined rows, 3 bulk-copied rows")
    ap.add_argument("--attn-fwd-variant", type=int, default=0, choices=[0, 1, 2],
                    help="attention forward: 0 automatic, 1 a CTA per query tile, 2 persistent CTAs")
    ap.add_argument("--attn-dq-variant", type=int, default=0, choices=[0, 1, 2, 3],
                    help="attention backward dQ: 0 automatic, 1 a CTA per query tile, 2 persistent CTAs, "
                         "3 persistent with two groups of softmax warps")
    ap.add_argument("--attn-dkdv-variant", type=int, default=0, choices=[0, 1, 2],
                    help="attention backward dK/dV: 0 automatic, 1 one group of softmax warps, 2 two groups")
    ap.add_argument("--ce-variant", type=int, default=0, choices=[0, 1, 2],
                    help="softmax-CE above V = 8192: 0 automatic, 1 one-shot clusters, 2 streamed rows")
    ap.add_argument("--pdl", type=int, default=0, choices=[0, 1],
                    help="programmatic dependent launch between the library's kernels")
    ap.add_argument("--gemm-schedule", type=int, default=0, choices=[0, 1, 2],
                    help="CTA-pair GEMM tile order: 0 automatic, 1 fixed, 2 dynamic (a tile counter)")
    ap.add_argument("--quant-path", type=int, default=0, choices=[0, 1, 2],
                    help="quantized dX: 0 automatic, 1 dequantize + GEMM, 2 decode inside the GEMM")
    a = ap.parse_args(argv)
    names = sorted(CASES) if "all" in a.cases else a.cases
    with Context(0) as ctx:
        ctx.call("glc_set_gemm_variant", a.variant)
        ctx.call("glc_set_attention_split", a.attn_split)
        ctx.call("glc_set_rmsnorm_variant", a.rmsnorm_variant)
        ctx.call("glc_set_ce_variant", a.ce_variant)
        ctx.call("glc_set_quant_path", a.quant_path)
        ctx.call("glc_set_gemm_schedule", a.gemm_schedule)
        ctx.call("glc_set_pdl", a.pdl)
        ctx.call("glc_set_attention_fwd_variant", a.attn_fwd_variant)
        ctx.call("glc_set_attention_dq_variant", a.attn_dq_variant)
        ctx.call("glc_set_attention_dkdv_variant", a.attn_dkdv_variant)
        for n in names:
            res = CASES[n](ctx, a.iters, a.warmup)
            for desc, ms, rate, unit in (res if isinstance(res, list) else [res]):
                print(f"{n:18s} {desc:44s} {ms:9.4f} ms  {rate:9.1f} {unit}", flush=True)


if __name__ == "__main__":
    main()
