"""Trainer.TrainStep in reference semantics (pkg/train/trainer.go:462-505)
restated in plain Python on a micro model, for golden vectors.

The restatement follows the reference's structure rather than the C oracle's:
a small tape of nodes (data, gradient or None, parents, GradFn) built by the
forward exactly as pkg/train/trainer.go:271-426 builds it, Backward() seeding
the logits with ones and running GradFns in reverse depth-first topological
order over Parents (pkg/tensor/grad.go:43-76), then GradientClipping and
AdamW.Step (pkg/train/optimizer.go).  Every float32 sum runs in the
reference's loop order with numpy float32 scalars (one rounding per
operation, no fused multiply-add, as Go on amd64); exp32/log32 come from
make_golden.py.  math.exp and math.cos are C's (the oracle's as well); Go's
math.Exp/Cos may differ from them in the last place of a float64, which a
float32 cast almost always hides.
"""
import math

import numpy as np

f32 = np.float32


class Node:
    """GradTensor (pkg/tensor/grad.go:9-15): data, Grad (None = nil), RequireGrad, Parents, GradFn."""

    def __init__(self, data, require_grad=False, parents=(), grad_fn=None):
        self.data = np.ascontiguousarray(data, np.float32)
        self.grad = None
        self.require_grad = require_grad
        self.parents = list(parents)
        self.grad_fn = grad_fn

    def zero_grad_like(self):
        if self.grad is None:
            self.grad = np.zeros_like(self.data)


def dot8(a, b):
    from make_golden import dot8 as d8  # the same restatement as the linear-layer vectors

    return d8(a, b)


def matmul_grad(a: Node, b: Node) -> Node:
    """MatMulGrad (grad.go:81-155): C = A . B^T with dotProduct; GradFn dA, dB."""
    A, B = a.data, b.data
    M, K = A.shape
    N = B.shape[0]
    out = Node(np.array([[dot8(A[i], B[j]) for j in range(N)] for i in range(M)], np.float32),
               a.require_grad or b.require_grad, [a, b])

    def fn():
        if out.grad is None:
            return
        dC = out.grad
        if a.require_grad:
            a.zero_grad_like()
            for m in range(M):
                for k in range(K):
                    s = f32(0)
                    for n in range(N):
                        s = s + dC[m, n] * B[n, k]
                    a.grad[m, k] = a.grad[m, k] + s
        if b.require_grad:
            b.zero_grad_like()
            for n in range(N):
                for k in range(K):
                    s = f32(0)
                    for m in range(M):
                        s = s + dC[m, n] * A[m, k]
                    b.grad[n, k] = b.grad[n, k] + s

    out.grad_fn = fn
    return out


def add_grad(a: Node, b: Node) -> Node:
    """AddGrad (grad.go:158-197) on equal shapes."""
    out = Node(a.data + b.data, a.require_grad or b.require_grad, [a, b])

    def fn():
        if out.grad is None:
            return
        for t in (a, b):
            if t.require_grad:
                t.zero_grad_like()
                t.grad = t.grad + out.grad

    out.grad_fn = fn
    return out


def silu_grad(x: Node) -> Node:
    """SiLUGrad (grad.go:417-449)."""
    from make_golden import exp32

    flat = x.data.reshape(-1)
    sig = np.array([f32(1) / (f32(1) + exp32(-v)) for v in flat], np.float32)
    out = Node((flat * sig).reshape(x.data.shape), x.require_grad, [x])

    def fn():
        if not x.require_grad or out.grad is None:
            return
        x.zero_grad_like()
        g = x.grad.reshape(-1)
        dy = out.grad.reshape(-1)
        for i, v in enumerate(flat):
            s = sig[i]
            g[i] = g[i] + dy[i] * (s * (f32(1) + v * (f32(1) - s)))

    out.grad_fn = fn
    return out


def product(gate: Node, up: Node) -> Node:
    """The SwiGLU product node (trainer.go:400-422)."""
    out = Node(gate.data * up.data, True, [gate, up])

    def fn():
        if out.grad is None:
            return
        gate.zero_grad_like()
        up.zero_grad_like()
        gate.grad = gate.grad + out.grad * up.data
        up.grad = up.grad + out.grad * gate.data

    out.grad_fn = fn
    return out


def rmsnorm(x: Node, w: Node, eps: float) -> Node:
    """RMSNormTrainable.Forward and its simplified GradFn (trainer.go:141-203)."""
    X, W = x.data, w.data.reshape(-1)
    rows, cols = X.shape
    rms = np.zeros(rows, np.float32)
    y = np.zeros_like(X)
    for i in range(rows):
        ss = f32(0)
        for j in range(cols):
            ss = ss + X[i, j] * X[i, j]
        rms[i] = f32(math.sqrt(float(ss) / float(cols) + float(f32(eps))))
        for j in range(cols):
            y[i, j] = (X[i, j] / rms[i]) * W[j]
    out = Node(y, x.require_grad or w.require_grad, [x, w])

    def fn():
        if out.grad is None:
            return
        if x.require_grad:
            x.zero_grad_like()
        if w.require_grad:
            w.zero_grad_like()
        for i in range(rows):
            for j in range(cols):
                dout = out.grad[i, j]
                if w.require_grad:
                    w.grad.reshape(-1)[j] = w.grad.reshape(-1)[j] + dout * X[i, j] / rms[i]
                if x.require_grad:
                    x.grad[i, j] = x.grad[i, j] + dout * W[j] / rms[i]

    out.grad_fn = fn
    return out


def attention(q: Node, k: Node, v: Node, seq_len: int, heads: int, kv_heads: int = 0) -> Node:
    """forwardAttention's score/softmax/sum (trainer.go:329-382): no GradFn.
    With kv_heads < heads, query head h reads KV head h / (heads / kv_heads)
    (pkg/model/attention.go:118,149) from k/v rows of kv_heads heads."""
    Q, Kd, V = q.data, k.data, v.data
    T, d = Q.shape
    hd = d // heads
    kvh = kv_heads or heads
    group = heads // kvh
    scale = f32(1.0 / math.sqrt(float(hd)))
    att = np.zeros_like(Q)
    for i in range(T):
        pos, b = i % seq_len, i // seq_len
        for h in range(heads):
            o = h * hd
            ko = (h // group) * hd
            scores = []
            mx = f32(-1e10)
            for j in range(pos + 1):
                jj = b * seq_len + j
                dot = f32(0)
                for e in range(hd):
                    dot = dot + Q[i, o + e] * Kd[jj, ko + e]
                sc = dot * scale
                scores.append(sc)
                if sc > mx:
                    mx = sc
            se = f32(0)
            for j in range(len(scores)):
                scores[j] = f32(math.exp(float(scores[j] - mx)))
                se = se + scores[j]
            for j in range(len(scores)):
                scores[j] = scores[j] / se
            for e in range(hd):
                s = f32(0)
                for j in range(pos + 1):
                    s = s + scores[j] * V[b * seq_len + j, ko + e]
                att[i, o + e] = s
    return Node(att, True, [q, k, v])


def backward(root: Node) -> None:
    """Backward (grad.go:43-76): ones seed, DFS topological order, GradFns reversed."""
    if root.grad is None:
        root.grad = np.ones_like(root.data)
    visited, order = set(), []

    def topo(t):
        if id(t) in visited:
            return
        visited.add(id(t))
        for p in t.parents:
            topo(p)
        order.append(t)

    topo(root)
    for t in reversed(order):
        if t.grad_fn is not None:
            t.grad_fn()


def train_step(params, cfg, hp, inputs, targets):
    """One TrainStep; params is the list of arrays in Params() order.  Returns
    (loss, per-parameter gradient or None after clipping, params after AdamW,
    m, v)."""
    from make_golden import adamw_steps, softmax_ce

    L, heads, eps = cfg["layers"], cfg["heads"], cfg["norm_eps"]
    B, S = inputs.shape
    V, d = params[0].shape
    nodes = [Node(p.copy(), True) for p in params]
    tok_embed, pos_embed = nodes[0], nodes[1]
    # Forward (trainer.go:271-305): token + position embedding, no GradFn
    h = np.zeros((B * S, d), np.float32)
    for b in range(B):
        for s in range(S):
            t = int(inputs[b, s])
            t = 0 if t < 0 or t >= V else t
            h[b * S + s] = tok_embed.data[t] + pos_embed.data[s]
    x = Node(h, True, [tok_embed, pos_embed])
    for layer in range(L):
        an, wq, wk, wv, wo, fn_, wg, wu, wd = nodes[2 + 9 * layer: 2 + 9 * layer + 9]
        normed = rmsnorm(x, an, eps)
        q, k, v = matmul_grad(normed, wq), matmul_grad(normed, wk), matmul_grad(normed, wv)
        x = add_grad(x, matmul_grad(attention(q, k, v, S, heads), wo))
        normed = rmsnorm(x, fn_, eps)
        gate, up = matmul_grad(normed, wg), matmul_grad(normed, wu)
        x = add_grad(x, matmul_grad(product(silu_grad(gate), up), wd))
    logits = matmul_grad(rmsnorm(x, nodes[-1], eps), tok_embed)  # tied head (trainer.go:252,302)
    loss, _ = softmax_ce(logits.data, targets.reshape(-1))
    backward(logits)  # TrainStep seeds the logits with ones (trainer.go:488-491)
    # GradientClipping (optimizer.go:169-196)
    total = 0.0
    for n in nodes:
        if n.grad is not None:
            for g in n.grad.reshape(-1):
                total += float(g) * float(g)
    total = math.sqrt(total)
    if f32(total) > f32(hp["clip"]):
        scale = f32(float(f32(hp["clip"])) / total)
        for n in nodes:
            if n.grad is not None:
                n.grad = n.grad * scale
    # GetLR (optimizer.go:157-166) at step 1, then AdamW.Step on the parameters that have a gradient
    warm, total_steps = hp["warmup"], hp["total_steps"]
    if 1 < warm:
        lr = f32(hp["lr"]) * f32(1) / f32(warm)
    else:
        progress = float(1 - warm) / float(total_steps - warm)
        lr = f32(hp["lr"]) * f32(0.5 * (1 + math.cos(math.pi * progress)))
    after, ms, vs = [], [], []
    for n in nodes:
        if n.grad is None:
            after.append(n.data.copy())
            ms.append(np.zeros_like(n.data))
            vs.append(np.zeros_like(n.data))
            continue
        (p1, m1, v1), = adamw_steps(n.data.reshape(-1), [n.grad.reshape(-1)], lr, hp["beta1"], hp["beta2"],
                                     hp["eps"], hp["wd"])
        after.append(p1.reshape(n.data.shape))
        ms.append(m1.reshape(n.data.shape))
        vs.append(v1.reshape(n.data.shape))
    return loss, [n.grad for n in nodes], after, ms, vs
