"""Golden vectors of the reference's own arithmetic: its float32 exponential
and logarithm, the linear layer's products, SiLU, RMSNorm, softmax
cross-entropy and AdamW.

The reference (pkg/tensor/grad.go:283-381) computes exp32/log32 with its own
float64 polynomials instead of the standard library: `_exp` reduces x to
r = x - k*ln2 with k truncated toward zero from x*log2(e) +- 0.5, evaluates a
truncated rational polynomial and scales by 2^k with repeated doubling or
halving; `_log` halves or doubles x into [1, 2) and evaluates a polynomial in
s = f/(2+f).  exp32 clamps at -88 / 88 before that.

This script restates both in plain Python: Python floats are IEEE float64
and every operation below maps to one float64 operation in the same order
(Go on amd64 does not fuse multiply-add), and numpy.float32 rounds to nearest
like Go's float32() conversion.  It is independent of the C oracle
(oracle/oracle.c) and of the device code, which restate the same functions
separately; tests/test_golden.py checks the oracle against these vectors bit
for bit, and the GPU tests check the device code against the oracle.

The linear layer's products (matmul.go:145-259, grad.go:81-152), SiLU
(grad.go:417-449), RMSNorm with its simplified gradient
(pkg/train/trainer.go:141-203), softmax cross-entropy (grad.go:210-280) and
AdamW.Step (pkg/train/optimizer.go:37-76) are restated the same way, with
float32 sums in the reference's order; ref_step.py restates one whole
TrainStep in reference semantics on a micro model.

    python tests/golden/make_golden.py     # rewrites go_arith.json
"""
import json
import math
from pathlib import Path

import numpy as np

OUT = Path(__file__).with_name("go_arith.json")

LN2_HI = 6.93147180369123816490e-01
LN2_LO = 1.90821492927058770002e-10
LOG2E = 1.44269504088896338700e00
EXP_OVERFLOW = 7.09782712893383973096e02
EXP_UNDERFLOW = -7.45133219101941108420e02


def go_exp(x: float) -> float:
    """grad.go:310-352."""
    if x > EXP_OVERFLOW:
        return 1.7976931348623157e308
    if x < EXP_UNDERFLOW:
        return 0.0
    k = int(x * LOG2E + 0.5) if x >= 0 else int(x * LOG2E - 0.5)  # int() truncates toward zero, as Go's
    r = x - float(k) * LN2_HI - float(k) * LN2_LO
    r2 = r * r
    p = r - r2 * (0.16666666666666602 + r2 * (0.0027777777777015593 + r2 * 6.613756321437934e-05))
    result = 1 - (r * p / (p - 2) - r)
    if k > 0:
        for _ in range(k):
            result *= 2
    else:
        for _ in range(-k):
            result /= 2
    return result


def go_log(x: float) -> float:
    """grad.go:354-381."""
    if x <= 0:
        return -1e100
    k = 0
    while x >= 2:
        x /= 2
        k += 1
    while x < 1:
        x *= 2
        k -= 1
    f = x - 1
    s = f / (2 + f)
    s2 = s * s
    s4 = s2 * s2
    t1 = s2 * (0.6666666666666735 + s4 * (0.2857142874366239 + s4 * 0.1818357216161805))
    t2 = s4 * (0.3999999999940942 + s4 * 0.22222198432149784)
    big_r = t1 + t2
    return float(k) * 0.6931471805599453 + f - s * (f - big_r)


def exp32(x32: np.float32) -> np.float32:
    """grad.go:283-293."""
    if x32 < np.float32(-88):
        return np.float32(0)
    if x32 > np.float32(88):
        return np.float32(3.4e38)
    return np.float32(go_exp(float(x32)))


def log32(x32: np.float32) -> np.float32:
    """grad.go:295-298 (float32(-1e100), the result for x <= 0, is -Inf)."""
    with np.errstate(over="ignore"):
        return np.float32(go_log(float(x32)))


def adamw_steps(p, grads, lr, b1, b2, eps, wd):
    """AdamW.Step (pkg/train/optimizer.go:37-76) over a float32 vector for each
    gradient in turn: float32 moments in Go's evaluation order, float64 bias
    corrections, estimates and update, float32 casts.  1 - beta^t uses C's
    pow (the oracle's), not Go's math.Pow, which squares repeatedly and can
    differ in the last place.  Returns (p, m, v) after every step."""
    f32 = np.float32
    lr, b1, b2, eps, wd = f32(lr), f32(b1), f32(b2), f32(eps), f32(wd)
    m = np.zeros_like(p)
    v = np.zeros_like(p)
    out = []
    for step, g in enumerate(grads, start=1):
        bc1 = 1.0 - math.pow(float(b1), float(step))
        bc2 = 1.0 - math.pow(float(b2), float(step))
        m = b1 * m + (f32(1) - b1) * g
        v = b2 * v + (f32(1) - b2) * g * g
        mhat = m.astype(np.float64) / bc1
        vhat = v.astype(np.float64) / bc2
        update = (mhat / (np.sqrt(vhat) + float(eps))).astype(np.float32)
        p = p - lr * (update + wd * p)
        out.append((p.copy(), m.copy(), v.copy()))
    return out


def silu(xs):
    """SiLUGrad forward (grad.go:424-428): s = 1/(1+exp32(-v)), y = v*s."""
    f32 = np.float32
    s = [f32(1) / (f32(1) + exp32(-v)) for v in xs]
    return np.array(s, np.float32), np.array([v * si for v, si in zip(xs, s)], np.float32)


def silu_grad(xs, s, dy):
    """SiLUGrad's GradFn (grad.go:440-445) onto a zero gradient: dy * s*(1 + v*(1-s))."""
    f32 = np.float32
    return np.array([f32(0) + d * (si * (f32(1) + v * (f32(1) - si))) for v, si, d in zip(xs, s, dy)], np.float32)


def rmsnorm(x, w, eps):
    """RMSNormTrainable.Forward (trainer.go:141-167): float32 sum of squares in
    column order, float64 sqrt, (x / rms) * w."""
    f32 = np.float32
    rows, cols = x.shape
    rms = np.zeros(rows, np.float32)
    y = np.zeros_like(x)
    for i in range(rows):
        ss = f32(0)
        for j in range(cols):
            ss = ss + x[i, j] * x[i, j]
        rms[i] = f32(math.sqrt(float(ss) / float(cols) + float(f32(eps))))
        for j in range(cols):
            y[i, j] = (x[i, j] / rms[i]) * w[j]
    return y, rms


def rmsnorm_grad(x, w, rms, dout):
    """Its simplified GradFn (trainer.go:182-199) onto zero gradients:
    dw[j] += dout*x/rms over the rows in order, dx = dout*w/rms."""
    f32 = np.float32
    rows, cols = x.shape
    dw = np.zeros(cols, np.float32)
    dx = np.zeros_like(x)
    for i in range(rows):
        for j in range(cols):
            dw[j] = dw[j] + dout[i, j] * x[i, j] / rms[i]
            dx[i, j] = f32(0) + dout[i, j] * w[j] / rms[i]
    return dx, dw


def softmax_ce(logits, targets):
    """SoftmaxCrossEntropyGrad (grad.go:210-280): per row the max, exp32 of the
    differences summed in order, probabilities, the loss over valid targets
    divided by the row count, and the GradFn onto a zero gradient."""
    f32 = np.float32
    rows, vocab = logits.shape
    probs = np.zeros_like(logits)
    total = f32(0)
    for b in range(rows):
        mx = logits[b, 0]
        for v in range(1, vocab):
            if logits[b, v] > mx:
                mx = logits[b, v]
        se = f32(0)
        for v in range(vocab):
            probs[b, v] = exp32(logits[b, v] - mx)
            se = se + probs[b, v]
        for v in range(vocab):
            probs[b, v] = probs[b, v] / se
        t = targets[b]
        if 0 <= t < vocab:
            total = total - log32(probs[b, t] + f32(1e-10))
    loss = total / f32(rows)
    scale = f32(1) / f32(rows)
    grad = np.zeros_like(logits)
    for b in range(rows):
        for v in range(vocab):
            gv = probs[b, v] * scale
            if v == targets[b]:
                gv = gv - scale
            grad[b, v] = f32(0) + gv
    return loss, grad


def dot8(a, b):
    """dotProduct (pkg/tensor/matmul.go:237-259): eight float32 partial sums
    over blocks of 8, added left to right, then the remainder."""
    f32 = np.float32
    K = a.size
    s = [f32(0)] * 8
    k = 0
    while k <= K - 8:
        for u in range(8):
            s[u] = s[u] + a[k + u] * b[k + u]
        k += 8
    total = s[0] + s[1] + s[2] + s[3] + s[4] + s[5] + s[6] + s[7]
    while k < K:
        total = total + a[k] * b[k]
        k += 1
    return total


def matmul_grads(a, b, dc, da0, db0):
    """MatMulTransposeB (matmul.go:145-234) C = A . B^T by dotProduct, and
    MatMulGrad's GradFn (grad.go:94-152): dA[m,k] += sum_n dC[m,n]*B[n,k] and
    dB[n,k] += sum_m dC[m,n]*A[m,k], each sum float32 from zero in index order."""
    f32 = np.float32
    M, K = a.shape
    N = b.shape[0]
    c = np.array([[dot8(a[i], b[j]) for j in range(N)] for i in range(M)], np.float32)
    da = da0.copy()
    for m in range(M):
        for k in range(K):
            s = f32(0)
            for n in range(N):
                s = s + dc[m, n] * b[n, k]
            da[m, k] = da[m, k] + s
    db = db0.copy()
    for n in range(N):
        for k in range(K):
            s = f32(0)
            for m in range(M):
                s = s + dc[m, n] * a[m, k]
            db[n, k] = db[n, k] + s
    return c, da, db


def ref_step_fixture(r):
    """Parameters in Params() order (trainer.go:217-253): TokenEmbed [V, d],
    PosEmbed [S, d], per layer AttnNorm, WQ, WK, WV, WO, FFNNorm, WGate, WUp,
    WDown, then OutputNorm; one TrainStep on two sequences of five tokens."""
    import ref_step

    cfg = {"layers": 2, "hidden": 8, "heads": 2, "inter": 12, "vocab": 11, "seq": 5, "norm_eps": 1e-5}
    hp = {"lr": 3e-4, "warmup": 0, "total_steps": 10000, "beta1": 0.9, "beta2": 0.95, "eps": 1e-8, "wd": 0.1,
          "clip": 1.0}
    d, F, V, S = cfg["hidden"], cfg["inter"], cfg["vocab"], cfg["seq"]
    shapes = [(V, d), (S, d)]
    for _ in range(cfg["layers"]):
        shapes += [(1, d), (d, d), (d, d), (d, d), (d, d), (1, d), (F, d), (F, d), (d, F)]
    shapes.append((1, d))
    params = [(1 + 0.1 * r.standard_normal(sh)).astype(np.float32) if sh[0] == 1
              else (r.standard_normal(sh) * 0.3).astype(np.float32) for sh in shapes]
    inputs = r.integers(0, V, (2, S))
    inputs[0, 1], inputs[1, 3] = -1, V + 2        # out-of-range ids embed token 0 (trainer.go:280-282)
    targets = r.integers(0, V, (2, S))
    targets[0, 0], targets[1, 4] = -1, V + 3      # ignored targets (grad.go:239-243)
    loss, grads, after, ms, vs = ref_step.train_step(params, cfg, hp, inputs, targets)
    return {"config": cfg, "hparams": hp, "shapes": shapes, "inputs": inputs.tolist(), "targets": targets.tolist(),
            "params": [bitlist(p) for p in params], "loss": bits(loss),
            "grads": [None if g is None else bitlist(g) for g in grads],
            "after": [bitlist(p) for p in after], "m": [bitlist(m) for m in ms], "v": [bitlist(v) for v in vs]}


def rope(dim, max_seq, theta, x, seq_len, heads):
    """RoPE (pkg/model/rope.go): the tables (precomputeFreqs, :33-48) in
    float64 cast to float32 — with C's pow/cos/sin, the oracle's; Go's may
    differ in a float64's last place — and apply3D (:96-126) with consecutive
    pairs on rows of `heads` heads, position = row % seq_len."""
    half = dim // 2
    cos_t = np.zeros((max_seq, half), np.float32)
    sin_t = np.zeros((max_seq, half), np.float32)
    for pos in range(max_seq):
        for i in range(half):
            freq = 1.0 / math.pow(float(np.float32(theta)), float(2 * i) / float(dim))
            angle = float(pos) * freq
            cos_t[pos, i] = np.float32(math.cos(angle))
            sin_t[pos, i] = np.float32(math.sin(angle))
    y = x.copy()
    for t in range(x.shape[0]):
        pos = t % seq_len
        for h in range(heads):
            base = h * dim
            for i in range(half):
                c, s = cos_t[pos, i], sin_t[pos, i]
                x0, x1 = x[t, base + 2 * i], x[t, base + 2 * i + 1]
                y[t, base + 2 * i] = x0 * c - x1 * s
                y[t, base + 2 * i + 1] = x0 * s + x1 * c
    return cos_t, sin_t, y


def bits(v: np.float32) -> int:
    return int(np.array([v], np.float32).view(np.uint32)[0])


def bitlist(a: np.ndarray) -> list:
    return np.ascontiguousarray(a, np.float32).reshape(-1).view(np.uint32).tolist()


def main() -> None:
    r = np.random.default_rng(20251201)
    xs = np.concatenate([
        np.array([0.0, -0.0, 1.0, -1.0, 0.5, -0.5, 88.0, -88.0, 87.99, -87.99, 88.5, -88.5, 1e-30, -1e-30,
                  0.693147, -0.693147, 20.0, -20.0], np.float32),
        np.linspace(-90, 90, 721, dtype=np.float32),
        r.uniform(-88, 88, 2000).astype(np.float32),
        (r.standard_normal(1000) * 4).astype(np.float32),
    ])
    ls = np.concatenate([
        np.array([1.0, 2.0, 0.5, 1e-10, 1e-10 + 1e-16, 3.0, 1.5, 1e30, 1e-38, 0.0, -1.0], np.float32),
        np.geomspace(1e-12, 1e4, 1500).astype(np.float32),
        r.uniform(0, 1, 1000).astype(np.float32),
    ])
    data = {
        "source": "pkg/tensor/grad.go:283-381 restated in plain Python (tests/golden/make_golden.py)",
        "exp32": [[bits(x), bits(exp32(x))] for x in xs],
        "log32": [[bits(x), bits(log32(x))] for x in ls],
        "go_exp": [[float(x), go_exp(float(x))] for x in np.linspace(-30, 30, 241)],
    }
    # linear layer: C = A . B^T and both gradients onto existing ones; K = 21 (two blocks of 8 + 5)
    a = r.standard_normal((5, 21)).astype(np.float32)
    b = r.standard_normal((7, 21)).astype(np.float32)
    dc = r.standard_normal((5, 7)).astype(np.float32)
    da0 = r.standard_normal((5, 21)).astype(np.float32)
    db0 = r.standard_normal((7, 21)).astype(np.float32)
    c, da, db = matmul_grads(a, b, dc, da0, db0)
    data["matmul"] = {"a": bitlist(a), "b": bitlist(b), "dc": bitlist(dc), "da0": bitlist(da0), "db0": bitlist(db0),
                      "c": bitlist(c), "da": bitlist(da), "db": bitlist(db)}
    # SiLU: special values and a spread of magnitudes
    xs = np.concatenate([np.array([0.0, -0.0, 1.0, -1.0, 88.0, -88.0, 89.0, -89.0, 20.0, -20.0], np.float32),
                         (r.standard_normal(500) * 6).astype(np.float32)])
    sg, y = silu(xs)
    dy = r.standard_normal(xs.size).astype(np.float32)
    data["silu"] = {"x": bitlist(xs), "y": bitlist(y), "dy": bitlist(dy), "dx": bitlist(silu_grad(xs, sg, dy))}
    # RMSNorm: 6 rows of 64, eps 1e-5
    x = r.standard_normal((6, 64)).astype(np.float32)
    w = (1 + 0.1 * r.standard_normal(64)).astype(np.float32)
    yr, rms = rmsnorm(x, w, 1e-5)
    dout = r.standard_normal((6, 64)).astype(np.float32)
    dxr, dwr = rmsnorm_grad(x, w, rms, dout)
    data["rmsnorm"] = {"eps": 1e-5, "x": bitlist(x), "w": bitlist(w), "y": bitlist(yr), "rms": bitlist(rms),
                       "dout": bitlist(dout), "dx": bitlist(dxr), "dw": bitlist(dwr)}
    # softmax-CE: 6 rows of 100 logits N(0, 2); one ignored and one out-of-range target
    lg = (r.standard_normal((6, 100)) * 2).astype(np.float32)
    tg = r.integers(0, 100, 6)
    tg[0], tg[1] = -1, 105
    loss, gce = softmax_ce(lg, tg)
    data["softmax_ce"] = {"logits": bitlist(lg), "targets": tg.tolist(), "loss": bits(loss), "grad": bitlist(gce)}
    # RoPE: head dim 8, 3 heads, rows of 2 sequences x 6 positions, theta 10000
    xr = r.standard_normal((12, 24)).astype(np.float32)
    ct, stb, yr_ = rope(8, 6, 10000.0, xr, 6, 3)
    data["rope"] = {"dim": 8, "max_seq": 6, "theta": 10000.0, "heads": 3, "x": bitlist(xr), "cos": bitlist(ct),
                    "sin": bitlist(stb), "y": bitlist(yr_)}
    # grouped-query attention forward: 4 query heads over 2 KV heads, head dim 4, 2 sequences of 6
    import ref_step

    qa = r.standard_normal((12, 16)).astype(np.float32)
    ka = r.standard_normal((12, 8)).astype(np.float32)
    va = r.standard_normal((12, 8)).astype(np.float32)
    oa = ref_step.attention(ref_step.Node(qa), ref_step.Node(ka), ref_step.Node(va), 6, 4, 2).data
    data["attention_gqa"] = {"S": 6, "H": 4, "Hkv": 2, "hd": 4, "q": bitlist(qa), "k": bitlist(ka), "v": bitlist(va),
                             "o": bitlist(oa)}
    # TrainStep in reference semantics on a micro model (ref_step.py)
    data["ref_step"] = ref_step_fixture(r)
    # AdamW: 96 parameters, 5 steps, the trainer's defaults (lr 3e-4, betas 0.9/0.95, eps 1e-8, wd 0.1)
    p0 = (r.standard_normal(96) * 0.02).astype(np.float32)
    grads = [(r.standard_normal(96) * 10.0 ** r.uniform(-4, 0)).astype(np.float32) for _ in range(5)]
    steps = adamw_steps(p0, grads, 3e-4, 0.9, 0.95, 1e-8, 0.1)
    data["adamw"] = {"lr": 3e-4, "beta1": 0.9, "beta2": 0.95, "eps": 1e-8, "weight_decay": 0.1,
                     "p0": bitlist(p0), "grads": [bitlist(g) for g in grads],
                     "after": [{"p": bitlist(p), "m": bitlist(m), "v": bitlist(v)} for p, m, v in steps]}
    OUT.write_text(json.dumps(data, separators=(",", ":")))
    print(f"wrote {OUT} ({len(data['exp32'])} exp32, {len(data['log32'])} log32 pairs)")


if __name__ == "__main__":
    main()
