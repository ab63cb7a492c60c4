// Host side of the training hot path above the C ABI: a C++ restatement of
// the reference's autograd tape (pkg/tensor/grad.go), its trainable model
// (pkg/train/trainer.go) and its optimizer / clipping / LR schedule
// (pkg/train/optimizer.go).  The structure follows the reference — GradTensor
// nodes with parents and closures, Backward() running GradFns in reverse DFS
// topological order, TrainStep's call order — but every GradFn enqueues
// sm_100a kernels on the context stream and every tensor lives on the device.
//
// Two semantics share the code (glc_train_config.semantics):
//   reference: learned position embedding, attention without a GradFn,
//              simplified RMSNorm backward, Backward() seeded with ones on the
//              logits (what TrainStep does, trainer.go:488-491);
//   llama:     RoPE, grouped KV heads, attention backward, exact RMSNorm
//              backward, embedding-gradient scatter, backward seeded by the
//              softmax-cross-entropy GradFn.
//
// Precision: every GEMM operand is rounded to TF32 (round to nearest) where it
// is produced — activations by the kernel that writes them, residual-stream
// gradients by the RMSNorm backward, weights through a rounded shadow copy
// refreshed by AdamW — because the tensor core truncates fp32 operands.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <deque>
#include <functional>
#include <memory>
#include <optional>
#include <string>
#include <unordered_set>
#include <vector>

#include "glc_internal.h"

namespace glc {

// ---------------------------------------------------------------- host helpers
void rope_table_host(int dim, int max_seq, float theta, float* cos_t, float* sin_t) {
  const int half = dim / 2;
  for (int pos = 0; pos < max_seq; ++pos)
    for (int i = 0; i < half; ++i) {
      const double freq = 1.0 / std::pow(static_cast<double>(theta), static_cast<double>(2 * i) / static_cast<double>(dim));
      const double angle = static_cast<double>(pos) * freq;
      cos_t[pos * half + i] = static_cast<float>(std::cos(angle));
      sin_t[pos * half + i] = static_cast<float>(std::sin(angle));
    }
}

void embed_segments_host(const int64_t* tok, int T, int V, std::vector<int>& seg_tok, std::vector<int>& seg_start,
                         std::vector<int>& order) {
  order.resize(T);
  for (int t = 0; t < T; ++t) order[t] = t;
  auto id = [&](int t) {
    int64_t v = tok[t];
    return (v < 0 || v >= V) ? 0 : static_cast<int>(v);
  };
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return id(a) < id(b); });
  seg_tok.clear();
  seg_start.clear();
  for (int i = 0; i < T; ++i) {
    if (i == 0 || id(order[i]) != id(order[i - 1])) {
      seg_tok.push_back(id(order[i]));
      seg_start.push_back(i);
    }
  }
  seg_start.push_back(T);
}

namespace {

// ---------------------------------------------------------------- device arena
// Bump allocator for one step's activations and gradients.  The first step
// discovers the size; afterwards one block serves every step.
class Arena {
 public:
  ~Arena() { release(); }
  void release() {
    for (auto& b : blocks_) cudaFree(b.ptr);
    blocks_.clear();
  }
  // Frees everything of the previous step (the stream is ordered, so memory
  // of the previous step may be reused by kernels enqueued after it).
  int reset(cudaStream_t s) {
    if (blocks_.size() > 1) {  // consolidate into one block sized for a full step
      size_t total = 0;
      for (auto& b : blocks_) total += b.used;
      cudaError_t e = cudaStreamSynchronize(s);
      if (e != cudaSuccess) return -1;
      release();
      if (grow(total + total / 8 + (size_t(64) << 20)) != 0) return -1;
    }
    for (auto& b : blocks_) b.used = 0;
    return 0;
  }
  float* alloc_floats(size_t n) { return static_cast<float*>(alloc(n * sizeof(float))); }
  void* alloc(size_t bytes) {
    bytes = (bytes + 255) & ~size_t(255);
    if (bytes == 0) bytes = 256;
    if (blocks_.empty() || blocks_.back().used + bytes > blocks_.back().size) {
      if (grow(std::max(bytes, size_t(256) << 20)) != 0) return nullptr;
    }
    Block& b = blocks_.back();
    void* p = static_cast<char*>(b.ptr) + b.used;
    b.used += bytes;
    return p;
  }
  size_t capacity() const {
    size_t c = 0;
    for (auto& b : blocks_) c += b.size;
    return c;
  }

 private:
  struct Block {
    void* ptr;
    size_t size;
    size_t used;
  };
  int grow(size_t bytes) {
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return -1;
    blocks_.push_back({p, bytes, 0});
    return 0;
  }
  std::vector<Block> blocks_;
};

struct StepError {
  int code;
};

inline void ck(int rc) {
  if (rc != 0) throw StepError{rc};
}

}  // namespace

// ---------------------------------------------------------------- tape
// GradTensor (pkg/tensor/grad.go:9-15).  `grad == nullptr` is Go's Grad == nil.
struct Node {
  float* data = nullptr;
  int64_t rows = 0, cols = 0;
  float* grad = nullptr;
  bool grad_live = false;           // grad allocated and holding this step's value
  float* grad_round = nullptr;      // TF32-rounded copy of grad (GEMM operand), or nullptr
  const float* gemm_data = nullptr; // TF32-rounded data for GEMMs (nullptr: data is not a GEMM operand)
  bool require_grad = false;
  std::function<void()> grad_fn;
  std::vector<Node*> parents;
  int param = -1;
  // A view over several adjacent parameters (WQ|WK|WV, WGate|WUp): one GEMM
  // operand whose gradient is the gradients of all of them.
  std::vector<int> group;
  int64_t numel() const { return rows * cols; }
};

struct Model;

class Tape {
 public:
  Tape(Context* ctx, Model* model) : ctx_(ctx), model_(model) {}
  Context* ctx() const { return ctx_; }
  cudaStream_t stream() const { return ctx_->stream; }
  Arena& arena() { return arena_; }

  void reset() {
    nodes_.clear();
    if (arena_.reset(ctx_->stream) != 0) throw StepError{GLC_ERR_NOMEM};
  }
  Node* make(int64_t rows, int64_t cols) {
    nodes_.emplace_back();
    Node* n = &nodes_.back();
    n->rows = rows;
    n->cols = cols;
    n->data = alloc(rows * cols);
    return n;
  }
  float* alloc(int64_t n) {
    float* p = arena_.alloc_floats(static_cast<size_t>(n));
    if (!p) {
      ctx_->last_error = "step arena: cudaMalloc failed";
      throw StepError{GLC_ERR_NOMEM};
    }
    return p;
  }

  // Makes n's gradient writable; returns true when the GradFn must accumulate
  // (`+=` onto an existing gradient), false when it may overwrite.
  bool prepare_grad(Node* n);
  // TF32-rounded gradient of n for use as a GEMM operand.
  const float* gemm_grad(Node* n) {
    if (n->grad_round) return n->grad_round;
    float* r = alloc(n->numel());
    ck(round_copy(ctx_, n->grad, r, static_cast<size_t>(n->numel()), stream()));
    n->grad_round = r;
    return r;
  }

  // Backward (pkg/tensor/grad.go:43-76): seed ones when the root has no
  // gradient, DFS topological order over Parents, GradFns in reverse.
  // seed_in_place reuses the root's data buffer for the ones (the caller
  // guarantees nothing reads it afterwards).
  // `before` sees the GradFn order before any runs; `after` is called once
  // each GradFn has been enqueued (its gradients are final on the stream).
  using OrderHook = std::function<void(const std::vector<Node*>&)>;
  using NodeHook = std::function<void(Node*)>;
  void backward(Node* root, bool seed_in_place, const OrderHook& before = nullptr, const NodeHook& after = nullptr) {
    if (!root->grad_live) {
      if (!root->grad) root->grad = seed_in_place ? root->data : alloc(root->numel());
      ck(fill(ctx_, root->grad, 1.0f, static_cast<size_t>(root->numel()), stream()));
      root->grad_live = true;
      root->grad_round = root->grad;  // ones are exact in TF32
    }
    std::vector<Node*> order;
    seen_.clear();
    topo(root, order);
    std::vector<Node*> run;
    for (auto it = order.rbegin(); it != order.rend(); ++it)
      if ((*it)->grad_fn) run.push_back(*it);
    if (before) before(run);
    for (Node* n : run) {
      n->grad_fn();
      if (after) after(n);
    }
  }

 private:
  void topo(Node* t, std::vector<Node*>& order) {
    if (seen_.count(t)) return;
    seen_.insert(t);
    for (Node* p : t->parents) topo(p, order);
    order.push_back(t);
  }
  Context* ctx_;
  Model* model_;
  Arena arena_;
  std::deque<Node> nodes_;
  std::unordered_set<const Node*> seen_;
  friend struct Model;
};

// ---------------------------------------------------------------- model
enum { P_ATTN_NORM = 0, P_WQ, P_WK, P_WV, P_WO, P_FFN_NORM, P_WGATE, P_WUP, P_WDOWN, P_PER_LAYER };

struct Model {
  Context* ctx = nullptr;
  glc_train_config cfg{};
  bool llama = false;
  int hd = 0, kvh = 0;
  // parameter layout (Params() order, trainer.go:217,242-247,253)
  std::vector<int64_t> offset, rows, cols;
  int64_t total = 0;
  // device arenas with the same layout
  float *params = nullptr, *grads = nullptr, *m = nullptr, *v = nullptr, *shadow = nullptr;
  // Go's `Grad != nil` per parameter, and "holds this step's value"
  std::vector<char> grad_allocated, grad_live;
  float *cos_t = nullptr, *sin_t = nullptr;  // RoPE tables [max_seq][hd/2]
  // After a step the gradients hold the unclipped values and pending_scale
  // (one device float) the clip scale; reading them applies it first, so the
  // step does not write the clipped gradients back (4 bytes per parameter).
  float* pending_scale = nullptr;
  bool scale_pending = false;
  // Clip norm from the GEMM epilogues (one GPU): a weight's gradient is final
  // once the last GradFn reading the weight has run, and that GradFn's dW
  // GEMM stores it, so its epilogue adds the squares of what it stores into
  // float64 slots; a small pass covers the gradients no such GEMM stores (the
  // tied embedding, which the scatter also writes, and the RMSNorm weights),
  // and one kernel adds every slot in order.  norm_slots holds norm_slot_cap
  // GEMM slots, then room for that pass's partials.
  double* norm_slots = nullptr;
  long long norm_slot_cap = 0, norm_slot_used = 0;
  double* norm_lvl = nullptr;  // inside norm_slots: the finishing sum's first level
  long long norm_lvl_cap = 0;
  bool norm_fused = false;                 // this step
  std::vector<const Node*> last_consumer;  // this step: the last GradFn reading each parameter
  std::vector<char> norm_covered;          // this step: parameters a GEMM epilogue measured
  std::vector<Node> param_nodes;
  std::vector<Node> qkv_view, gu_view;  // per layer: WQ|WK|WV and WGate|WUp

  int num_params() const { return static_cast<int>(offset.size()); }
  // Gradient buckets for the data-parallel sum, contiguous in the arena: the
  // front parameters (embedding, and positions in reference mode), one per
  // layer, and the output norm.  bucket_of[i] is parameter i's bucket.
  std::vector<int64_t> bucket_begin, bucket_end;
  std::vector<int> bucket_of;
  void plan_buckets() {
    bucket_begin.clear();
    bucket_end.clear();
    bucket_of.assign(num_params(), -1);
    auto add = [&](int first, int last) {  // parameters [first, last]
      for (int i = first; i <= last; ++i) bucket_of[i] = static_cast<int>(bucket_begin.size());
      bucket_begin.push_back(offset[first]);
      bucket_end.push_back(offset[last] + rows[last] * cols[last]);
    };
    add(0, front() - 1);
    for (int l = 0; l < cfg.num_layers; ++l) add(lp(l, 0), lp(l, P_PER_LAYER - 1));
    add(out_norm(), out_norm());
  }
  int front() const { return llama ? 1 : 2; }
  int lp(int layer, int which) const { return front() + layer * P_PER_LAYER + which; }
  int out_norm() const { return num_params() - 1; }

  ~Model() {
    for (float* p : {params, grads, m, v, shadow, cos_t, sin_t, pending_scale})
      if (p) cudaFree(p);
    if (norm_slots) cudaFree(norm_slots);
  }

  bool layout(const glc_train_config& conf);
  int init(Context* c, const glc_train_config& conf);
  void bind_param_nodes() {
    param_nodes.assign(num_params(), Node());
    for (int i = 0; i < num_params(); ++i) {
      Node& n = param_nodes[i];
      n.data = params + offset[i];
      n.rows = rows[i];
      n.cols = cols[i];
      n.grad = grads + offset[i];
      n.gemm_data = shadow + offset[i];
      n.require_grad = true;
      n.param = i;
    }
  }
  Node* P(int i) { return &param_nodes[i]; }
  void bind_views() {
    auto view = [&](int first, int count) {
      Node n;
      n.data = params + offset[first];
      n.grad = grads + offset[first];
      n.gemm_data = shadow + offset[first];
      n.cols = cols[first];
      for (int i = 0; i < count; ++i) {
        n.rows += rows[first + i];
        n.group.push_back(first + i);
      }
      n.require_grad = true;
      return n;
    };
    qkv_view.clear();
    gu_view.clear();
    for (int l = 0; l < cfg.num_layers; ++l) {
      qkv_view.push_back(view(lp(l, P_WQ), 3));
      gu_view.push_back(view(lp(l, P_WGATE), 2));
    }
  }

  // ------------------------------------------------------------ tape ops
  // MatMulGrad (grad.go:81-155): out = a . w^T; with `residual`, the AddGrad
  // that follows it in forwardLayer (trainer.go:312,317; grad.go:158-197) is
  // fused: out = residual + a . w^T, and its GradFn passes the gradient
  // through to `residual` before the two GEMM gradients.
  // round_out: the output is a tensor-core operand (q, k, v feed attention);
  // round_dx: the input gradient is one (the attention output's gradient).
  // swiglu_h: when set, w is a [gate F | up F] view and the same launch also
  // writes h = silu(gate) * up (TF32-rounded) there; the SwiGLU node then
  // adopts that buffer instead of running its own forward.
  Node* matmul(Tape& tp, Node* a, Node* w, Node* residual, bool round_out = false, bool round_dx = false,
               float* swiglu_h = nullptr) {
    const int M = static_cast<int>(a->rows), K = static_cast<int>(a->cols), N = static_cast<int>(w->rows);
    Node* out = tp.make(M, N);
    out->require_grad = a->require_grad || w->require_grad || (residual && residual->require_grad);
    if (residual) out->parents = {residual, a, w};
    else out->parents = {a, w};
    GemmSpec fwd{{a->gemm_data, K, false}, {w->gemm_data, K, false}, out->data, N, M, N, K, false,
                 residual ? residual->data : nullptr, N, round_out};
    if (swiglu_h) {
      fwd.glu = N / 2;
      fwd.glu_h = swiglu_h;
      fwd.ld_glu = N / 2;
      fwd.glu_round = true;
      fwd.glu_fast = llama;
    }
    ck(gemm_tf32_group(ctx, &fwd, 1, tp.stream()));
    if (round_out) out->gemm_data = out->data;
    Tape* t = &tp;
    out->grad_fn = [this, t, out, a, w, residual, M, K, N, round_dx]() {
      if (!out->grad_live) return;
      if (residual && residual->require_grad) {
        if (!residual->grad_live && residual->param < 0) {
          // first contribution: the gradient passes through unchanged, so the
          // buffer is shared instead of copied
          residual->grad = out->grad;
          residual->grad_live = true;
          residual->grad_round = out->grad_round;
        } else {
          const bool acc = t->prepare_grad(residual);
          if (acc) ck(add_inplace(ctx, residual->grad, out->grad, static_cast<size_t>(out->numel()), t->stream()));
          else ck(cudaMemcpyAsync(residual->grad, out->grad, sizeof(float) * out->numel(), cudaMemcpyDeviceToDevice, t->stream()) == cudaSuccess ? 0 : GLC_ERR_CUDA);
        }
      }
      const float* dY = t->gemm_grad(out);
      // dA = dC . B and dB = dC^T . A (grad.go:102-152) in one grouped launch
      GemmSpec g[2];
      int n = 0;
      if (a->require_grad) {
        const bool acc = t->prepare_grad(a);
        const bool rnd = round_dx && !acc;
        g[n++] = GemmSpec{{dY, N, false}, {w->gemm_data, K, true}, a->grad, K, M, K, N, acc, nullptr, 0, rnd};
        if (rnd) a->grad_round = a->grad;
      }
      if (w->require_grad) {
        const bool acc = t->prepare_grad(w);
        g[n] = GemmSpec{{dY, N, true}, {a->gemm_data, K, true}, w->grad, K, N, K, M, acc, nullptr, 0, false};
        claim_norm_slots(w, out, N, K, g[n]);
        ++n;
      }
      if (n) ck(gemm_tf32_group(ctx, g, n, t->stream()));
    };
    return out;
  }

  // When the clip norm comes from the GEMM epilogues and `consumer` is the
  // last GradFn reading every parameter of w, the dW GEMM into w's gradient
  // sums the squares of the final values into the next free slots.
  void claim_norm_slots(const Node* w, const Node* consumer, int rows, int cols, GemmSpec& g) {
    if (!norm_fused) return;
    std::vector<int> ps;
    if (w->param >= 0) ps.push_back(w->param);
    for (int i : w->group) ps.push_back(i);
    if (ps.empty()) return;
    for (int i : ps)
      if (last_consumer[i] != consumer) return;
    const long long need = gemm_sumsq_slots(rows, cols);
    if (norm_slot_used + need > norm_slot_cap) return;
    g.sumsq = norm_slots + norm_slot_used;
    g.sumsq_cap = need;
    norm_slot_used += need;
    for (int i : ps) norm_covered[i] = 1;
  }

  // RMSNormTrainable.Forward and its GradFn (trainer.go:141-203).
  Node* rmsnorm(Tape& tp, Node* x, Node* w) {
    const int R = static_cast<int>(x->rows), Cc = static_cast<int>(x->cols);
    Node* out = tp.make(R, Cc);
    out->require_grad = x->require_grad || w->require_grad;
    out->parents = {x, w};
    float* rms = tp.alloc(R);
    ck(rmsnorm_fwd(ctx, x->data, w->data, out->data, rms, R, Cc, cfg.norm_eps, true, tp.stream()));
    out->gemm_data = out->data;
    Tape* t = &tp;
    const bool full = llama;
    out->grad_fn = [this, t, out, x, w, rms, R, Cc, full]() {
      if (!out->grad_live) return;
      const bool xacc = t->prepare_grad(x);
      const bool wacc = t->prepare_grad(w);
      float* xr = t->alloc(x->numel());
      ck(rmsnorm_bwd(ctx, x->data, w->data, rms, out->grad, x->grad, xr, w->grad, R, Cc, full, xacc, wacc, nullptr,
                     0, t->stream()));
      x->grad_round = xr;
    };
    return out;
  }

  // forwardAttention (trainer.go:323-389) without its projections, on the
  // fused projection output qkv = [q | k | v] ([T, H*hd + 2*Hkv*hd]); Llama
  // semantics add RoPE on q and k (in place) and a GradFn.
  Node* attention(Tape& tp, Node* qkv, int B, int S) {
    const int H = cfg.num_heads, Hkv = kvh, T = B * S;
    const int ld = static_cast<int>(qkv->cols), qw = H * hd, kw = Hkv * hd;
    if (llama) {
      // q and k are adjacent in each row: H + Hkv heads rotated by one launch
      ck(rope(ctx, qkv->data, ld, T, S, H + Hkv, hd, cos_t, sin_t, false, true, tp.stream()));
    }
    Node* out = tp.make(T, qw);
    out->require_grad = true;
    out->parents = {qkv};
    float* lse = tp.alloc(static_cast<int64_t>(B) * H * S);
    const AttnIO fio{qkv->data, ld, qkv->data + qw, ld, qkv->data + qw + kw, ld, nullptr, 0, nullptr, 0, nullptr, 0};
    ck(attention_fwd(ctx, fio, out->data, lse, B, S, H, Hkv, hd, true, tp.stream()));
    out->gemm_data = out->data;
    if (!llama) return out;  // the reference attaches no GradFn (trainer.go:335-337)
    Tape* t = &tp;
    out->grad_fn = [this, t, out, qkv, lse, B, S, H, Hkv, T, ld, qw, kw]() {
      if (!out->grad_live) return;
      if (t->prepare_grad(qkv)) throw StepError{GLC_ERR_UNSUPPORTED};  // q/k/v have no other consumers
      float* D = t->alloc(static_cast<int64_t>(B) * H * S);
      const size_t np = attention_bwd_partial_floats(B, S, H, Hkv, hd);
      float* partial = np ? t->alloc(static_cast<int64_t>(np)) : nullptr;
      float* g = qkv->grad;
      const AttnIO io{qkv->data, ld, qkv->data + qw, ld, qkv->data + qw + kw, ld, g, ld, g + qw, ld, g + qw + kw, ld};
      // the backward RoPE rotation of dq and dk happens in the kernels that write them
      ck(attention_bwd(ctx, io, out->data, lse, out->grad, D, partial, B, S, H, Hkv, hd, true, t->stream(), cos_t,
                       sin_t));
      qkv->grad_round = qkv->grad;
    };
    return out;
  }

  // SiLUGrad (grad.go:417-449) and the product node (trainer.go:400-422) as
  // one node over the fused projection output gu = [gate | up] ([T, 2F]).
  // out: a node whose data the gate/up GEMM already filled with h (fused
  // epilogue), or nullptr to compute h here.
  Node* swiglu(Tape& tp, Node* gu, Node* out = nullptr) {
    const int64_t T = gu->rows, F = gu->cols / 2;
    const bool fused = out != nullptr;
    if (!out) out = tp.make(T, F);
    out->require_grad = true;
    out->parents = {gu};
    if (!fused)
      ck(swiglu_fwd(ctx, gu->data, gu->data + F, static_cast<size_t>(2 * F), out->data, static_cast<size_t>(F),
                    static_cast<size_t>(T), static_cast<size_t>(F), true, tp.stream(), llama));
    out->gemm_data = out->data;
    Tape* t = &tp;
    out->grad_fn = [this, t, out, gu, T, F]() {
      if (!out->grad_live) return;
      const bool acc = t->prepare_grad(gu);
      ck(swiglu_bwd(ctx, gu->data, gu->data + F, static_cast<size_t>(2 * F), out->grad, static_cast<size_t>(F),
                    gu->grad, gu->grad + F, static_cast<size_t>(2 * F), static_cast<size_t>(T), static_cast<size_t>(F),
                    acc, true, t->stream(), llama));
      gu->grad_round = gu->grad;
    };
    return out;
  }

  struct EmbedSegs {
    int* dev = nullptr;  // [seg_tok | seg_start | order]
    int nseg = 0;
  };

  // Embedding lookup (trainer.go:275-291); Llama semantics attach the
  // gradient scatter into TokenEmbed.
  Node* embedding(Tape& tp, const int64_t* tok_dev, int B, int S) {
    const int T = B * S, d = cfg.hidden_size;
    Node* out = tp.make(T, d);
    out->require_grad = true;
    Node* E = P(0);
    out->parents = llama ? std::vector<Node*>{E} : std::vector<Node*>{E, P(1)};
    ck(embed_fwd(ctx, tok_dev, E->data, llama ? nullptr : P(1)->data, out->data, T, S, d, cfg.vocab_size, tp.stream()));
    if (!llama) return out;  // no GradFn in the reference (trainer.go:290-291)
    // the scatter's segments (positions sorted by id) are built on the device
    // from the resident ids: no host copy and no synchronisation
    const EmbedSegLayout L(T);
    int* dev = reinterpret_cast<int*>(tp.alloc(L.total));
    ck(embed_segments_device(ctx, tok_dev, T, cfg.vocab_size, dev, tp.stream()));
    Tape* t = &tp;
    out->grad_fn = [this, t, out, E, dev, L, T, d]() {
      if (!out->grad_live) return;
      const bool acc = t->prepare_grad(E);
      if (!acc) ck(cudaMemsetAsync(E->grad, 0, sizeof(float) * E->numel(), t->stream()) == cudaSuccess ? 0 : GLC_ERR_CUDA);
      ck(embed_bwd(ctx, dev + L.seg_tok, dev + L.seg_start, dev + L.order, T, out->grad, E->grad, d, t->stream(),
                   dev + L.nseg));
    };
    return out;
  }

  // TrainableModel.Forward (trainer.go:271-305) -> logits node.
  Node* forward(Tape& tp, const int64_t* tok_dev, int B, int S) {
    Node* x = embedding(tp, tok_dev, B, S);
    for (int l = 0; l < cfg.num_layers; ++l) {
      // forwardLayer (trainer.go:308-320)
      Node* n1 = rmsnorm(tp, x, P(lp(l, P_ATTN_NORM)));
      // the q, k and v projections (trainer.go:325-327) as one GEMM over WQ|WK|WV
      Node* qkv = matmul(tp, n1, &qkv_view[l], nullptr, true);
      Node* att = attention(tp, qkv, B, S);
      Node* x1 = matmul(tp, att, P(lp(l, P_WO)), x, false, true);
      Node* n2 = rmsnorm(tp, x1, P(lp(l, P_FFN_NORM)));
      // forwardFFN (trainer.go:392-426): gate and up projections as one GEMM over
      // WGate|WUp.  On request (Llama semantics) its epilogue also writes
      // h = silu(g)*u; by default the SwiGLU kernel runs after the GEMM, which
      // is faster: the epilogue warps become the GEMM's bottleneck.
      Node* h = nullptr;
      if (llama && ctx->fuse_swiglu) {
        Node* hn = tp.make(n2->rows, cfg.intermediate_size);
        Node* gu = matmul(tp, n2, &gu_view[l], nullptr, false, false, hn->data);
        h = swiglu(tp, gu, hn);
      } else {
        Node* gu = matmul(tp, n2, &gu_view[l], nullptr);
        h = swiglu(tp, gu);
      }
      x = matmul(tp, h, P(lp(l, P_WDOWN)), x1);
    }
    Node* hf = rmsnorm(tp, x, P(out_norm()));
    return matmul(tp, hf, P(0), nullptr);  // tied LM head (trainer.go:252,302)
  }
};

bool Tape::prepare_grad(Node* n) {
  if (!n->group.empty()) {
    const bool acc = model_->grad_live[n->group[0]] != 0;
    for (int p : n->group) {
      if ((model_->grad_live[p] != 0) != acc) throw StepError{GLC_ERR_UNSUPPORTED};
      model_->grad_allocated[p] = 1;
      model_->grad_live[p] = 1;
      model_->param_nodes[p].grad_live = true;
    }
    n->grad_live = true;
    return acc;
  }
  if (n->param >= 0) {
    model_->grad_allocated[n->param] = 1;
    const bool acc = model_->grad_live[n->param] != 0;
    model_->grad_live[n->param] = 1;
    n->grad_live = true;
    return acc;
  }
  if (!n->grad) n->grad = alloc(n->numel());
  const bool acc = n->grad_live;
  n->grad_live = true;
  n->grad_round = nullptr;  // about to change
  return acc;
}

namespace {

uint64_t splitmix(uint64_t& s) {
  uint64_t z = (s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void init_normal_kernel(float* p, int64_t n, uint64_t seed, float std) {
  GLC_PDL_ENTRY();
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    uint64_t s = seed ^ (static_cast<uint64_t>(i) * 0xD1B54A32D192ED03ull);
    auto next = [&]() {
      uint64_t z = (s += 0x9E3779B97F4A7C15ull);
      z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
      z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
      return z ^ (z >> 31);
    };
    const double u1 = 1.0 - static_cast<double>(next() >> 11) * (1.0 / 9007199254740992.0);
    const double u2 = static_cast<double>(next() >> 11) * (1.0 / 9007199254740992.0);
    p[i] = static_cast<float>(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2) * std);
  }
}

}  // namespace

// Parameter layout in Params() order (host only; no device work).
bool Model::layout(const glc_train_config& conf) {
  cfg = conf;
  llama = cfg.semantics == GLC_SEMANTICS_LLAMA;
  if (cfg.num_kv_heads <= 0 || !llama) cfg.num_kv_heads = cfg.num_heads;
  if (cfg.num_heads <= 0 || cfg.hidden_size % cfg.num_heads || cfg.num_heads % cfg.num_kv_heads || cfg.vocab_size <= 0 ||
      cfg.num_layers < 0 || cfg.intermediate_size <= 0 || cfg.max_seq_len <= 0 || (cfg.hidden_size & 3) ||
      (cfg.intermediate_size & 3) || (cfg.vocab_size & 3))
    return false;
  hd = cfg.hidden_size / cfg.num_heads;
  kvh = cfg.num_kv_heads;
  const int64_t d = cfg.hidden_size, F = cfg.intermediate_size, kvd = static_cast<int64_t>(kvh) * hd;
  auto add = [&](int64_t r, int64_t cc) {
    offset.push_back(total);
    rows.push_back(r);
    cols.push_back(cc);
    total += r * cc;
  };
  add(cfg.vocab_size, d);
  if (!llama) add(cfg.max_seq_len, d);
  for (int l = 0; l < cfg.num_layers; ++l) {
    add(1, d);
    add(d, d);
    add(kvd, d);
    add(kvd, d);
    add(d, d);
    add(1, d);
    add(F, d);
    add(F, d);
    add(d, F);
  }
  add(1, d);
  plan_buckets();
  return true;
}

int Model::init(Context* c, const glc_train_config& conf) {
  ctx = c;
  if (!layout(conf))
    return c->fail(GLC_ERR_INVALID,
                  "model: inconsistent configuration (heads must divide hidden, kv heads must divide heads; hidden, "
                  "intermediate and vocab sizes must be multiples of 4)");
  const size_t bytes = sizeof(float) * static_cast<size_t>(total);
  for (float** p : {&params, &grads, &m, &v, &shadow}) {
    if (cudaMalloc(p, bytes) != cudaSuccess) return c->fail(GLC_ERR_NOMEM, "model: cannot allocate parameter arenas");
  }
  if (cudaMalloc(&pending_scale, sizeof(float)) != cudaSuccess) return c->fail(GLC_ERR_NOMEM, "model: clip scale");
  if (cudaMemsetAsync(grads, 0, bytes, c->stream) != cudaSuccess || cudaMemsetAsync(m, 0, bytes, c->stream) != cudaSuccess ||
      cudaMemsetAsync(v, 0, bytes, c->stream) != cudaSuccess)
    return c->fail(GLC_ERR_CUDA, "model: memset");
  grad_allocated.assign(num_params(), 0);
  grad_live.assign(num_params(), 0);
  // NewTrainableModel: matrices from a seeded normal, RMSNorm weights 1
  uint64_t s = cfg.seed;
  for (int i = 0; i < num_params(); ++i) {
    const int64_t n = rows[i] * cols[i];
    const uint64_t ps = splitmix(s);
    if (rows[i] == 1) {
      int rc = fill(c, params + offset[i], 1.0f, static_cast<size_t>(n), c->stream);
      if (rc) return rc;
    } else {
      glc::launch_pdl(c, init_normal_kernel, grid_for(static_cast<size_t>(n), 256, c->num_sms), 256, 0, c->stream,
                      params + offset[i], n, ps, cfg.init_std);
      GLC_LAUNCH_CHECK(c, "model init");
    }
  }
  int rc = round_copy(c, params, shadow, static_cast<size_t>(total), c->stream);
  if (rc) return rc;
  if (llama) {
    std::vector<float> ct(static_cast<size_t>(cfg.max_seq_len) * (hd / 2)), st(ct.size());
    rope_table_host(hd, cfg.max_seq_len, cfg.rope_theta, ct.data(), st.data());
    if (cudaMalloc(&cos_t, ct.size() * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&sin_t, st.size() * sizeof(float)) != cudaSuccess)
      return c->fail(GLC_ERR_NOMEM, "model: rope tables");
    cudaMemcpy(cos_t, ct.data(), ct.size() * sizeof(float), cudaMemcpyHostToDevice);
    cudaMemcpy(sin_t, st.data(), st.size() * sizeof(float), cudaMemcpyHostToDevice);
  }
  bind_param_nodes();
  bind_views();
  cudaError_t e = cudaStreamSynchronize(c->stream);
  return e == cudaSuccess ? 0 : c->fail_cuda(e, "model init");
}

// ---------------------------------------------------------------- trainer
// Floats per block of the clip-norm pass over the gradients no GEMM epilogue
// measured (a multiple of 4: segment starts and lengths are).
constexpr int64_t kNormChunk = 65536;

struct Trainer {
  Model* model = nullptr;
  Context* ctx = nullptr;
  std::unique_ptr<Tape> tape;
  // AdamW state (optimizer.go:10-21) and LRScheduler (optimizer.go:141-145)
  int adam_step = 0;
  int step = 0;
  float lr = 0.f;
  double last_norm = 0.0;
  uint64_t last_launches = 0;
  // device scalars: [loss f32][clip scale f32][norm f64]
  void* scalars = nullptr;
  float* loss_host = nullptr;
  int64_t* tok_dev = nullptr;
  int tok_cap = 0;
  float* row_logp = nullptr;
  int row_cap = 0;
  int64_t* segs_dev = nullptr;
  int nseg = 0;
  int64_t seg_elems = 0;
  std::vector<char> segs_for;
  // segments of the allocated gradients no GEMM epilogue measured (clip norm
  // from the epilogues), for the set they were built for
  int64_t* rest_segs_dev = nullptr;
  int nrest = 0;
  double rest_elems = 0;
  std::vector<char> rest_for;
  // data-parallel gradient buckets (Model::plan_buckets): per-step state
  std::vector<cudaEvent_t> bucket_ev;
  cudaEvent_t comm_done = nullptr;
  std::vector<int> consumers, bucket_pending;
  std::vector<char> bucket_launched;
  // Data parallelism: the clip norm's sums of squares are taken per bucket on
  // the communication stream right after the bucket's sum over the ranks
  // (chunks of at most kNormChunk floats of the allocated gradients, bucket
  // b's at [dp_chunk_off[b], dp_chunk_off[b + 1])), so no pass over all the
  // gradients follows the backward.  The tables are built for the set of
  // allocated gradients at the start of a step; a step that allocates new
  // ones (the first) takes the full pass instead.
  int64_t* dp_chunks_dev = nullptr;
  std::vector<int> dp_chunk_off;
  std::vector<char> dp_chunks_for;
  double* dp_slots = nullptr;  // [chunks] then the finishing sum's first level
  long long dp_nchunks = 0, dp_slots_cap = 0;
  double dp_chunk_elems = 0;

  ~Trainer() {
    for (cudaEvent_t e : bucket_ev) cudaEventDestroy(e);
    if (comm_done) cudaEventDestroy(comm_done);
    cudaFree(dp_chunks_dev);
    cudaFree(dp_slots);
    cudaFree(scalars);
    cudaFreeHost(loss_host);
    cudaFree(tok_dev);
    cudaFree(row_logp);
    cudaFree(segs_dev);
    cudaFree(rest_segs_dev);
  }

  float get_lr(int s) const {  // LRScheduler.GetLR (optimizer.go:157-166)
    const auto& c = model->cfg;
    if (s < c.warmup_steps) return c.learning_rate * static_cast<float>(s) / static_cast<float>(c.warmup_steps);
    const double progress = static_cast<double>(s - c.warmup_steps) / static_cast<double>(c.max_steps - c.warmup_steps);
    return c.learning_rate * static_cast<float>(0.5 * (1 + std::cos(M_PI * progress)));
  }

  // Segments {start, len} of the parameters that have a gradient, merged when adjacent.
  void refresh_segments() {
    if (segs_for == model->grad_allocated && segs_dev) return;
    std::vector<int64_t> s;
    for (int i = 0; i < model->num_params(); ++i) {
      if (!model->grad_allocated[i]) continue;
      const int64_t st = model->offset[i], len = model->rows[i] * model->cols[i];
      if (!s.empty() && s[s.size() - 2] + s[s.size() - 1] == st)
        s[s.size() - 1] += len;
      else {
        s.push_back(st);
        s.push_back(len);
      }
    }
    cudaFree(segs_dev);
    segs_dev = nullptr;
    nseg = static_cast<int>(s.size() / 2);
    seg_elems = 0;
    for (size_t i = 1; i < s.size(); i += 2) seg_elems += s[i];
    if (nseg) {
      if (cudaMalloc(&segs_dev, s.size() * sizeof(int64_t)) != cudaSuccess) throw StepError{GLC_ERR_NOMEM};
      if (cudaMemcpy(segs_dev, s.data(), s.size() * sizeof(int64_t), cudaMemcpyHostToDevice) != cudaSuccess)
        throw StepError{GLC_ERR_CUDA};
    }
    segs_for = model->grad_allocated;
  }

  void refresh_dp_chunks() {
    if (dp_chunks_for == model->grad_allocated && !dp_chunk_off.empty()) return;
    const int nb = static_cast<int>(model->bucket_begin.size());
    std::vector<int64_t> s;
    dp_chunk_off.assign(nb + 1, 0);
    dp_chunk_elems = 0;
    for (int b = 0; b < nb; ++b) {
      dp_chunk_off[b] = static_cast<int>(s.size() / 2);
      for (int i = 0; i < model->num_params(); ++i) {
        if (model->bucket_of[i] != b || !model->grad_allocated[i]) continue;
        const int64_t st = model->offset[i], len = model->rows[i] * model->cols[i];
        for (int64_t o = 0; o < len; o += kNormChunk) {
          s.push_back(st + o);
          s.push_back(std::min<int64_t>(kNormChunk, len - o));
        }
        dp_chunk_elems += static_cast<double>(len);
      }
    }
    dp_chunk_off[nb] = static_cast<int>(s.size() / 2);
    dp_nchunks = dp_chunk_off[nb];
    cudaFree(dp_chunks_dev);
    dp_chunks_dev = nullptr;
    if (!s.empty()) {
      if (cudaMalloc(&dp_chunks_dev, s.size() * sizeof(int64_t)) != cudaSuccess) throw StepError{GLC_ERR_NOMEM};
      if (cudaMemcpy(dp_chunks_dev, s.data(), s.size() * sizeof(int64_t), cudaMemcpyHostToDevice) != cudaSuccess)
        throw StepError{GLC_ERR_CUDA};
    }
    const long long need = dp_nchunks + dp_nchunks / 1024 + 2;
    if (need > dp_slots_cap) {
      cudaFree(dp_slots);
      dp_slots = nullptr;
      if (cudaMalloc(&dp_slots, sizeof(double) * static_cast<size_t>(need)) != cudaSuccess) throw StepError{GLC_ERR_NOMEM};
      dp_slots_cap = need;
    }
    dp_chunks_for = model->grad_allocated;
  }

  void refresh_rest_segments() {
    const int np = model->num_params();
    std::vector<char> key(np);
    for (int i = 0; i < np; ++i) key[i] = model->grad_allocated[i] ? (model->norm_covered[i] ? 2 : 1) : 0;
    if (key == rest_for && (rest_segs_dev || nrest == 0) && !rest_for.empty()) return;
    // adjacent gradients merged, then cut into chunks of at most kNormChunk
    // floats, one block each (the tied embedding is 65.5M floats, an RMSNorm
    // weight a few thousand)
    std::vector<int64_t> m;
    rest_elems = 0;
    for (int i = 0; i < np; ++i) {
      if (key[i] != 1) continue;
      const int64_t st = model->offset[i], len = model->rows[i] * model->cols[i];
      rest_elems += static_cast<double>(len);
      if (!m.empty() && m[m.size() - 2] + m[m.size() - 1] == st) {
        m[m.size() - 1] += len;
      } else {
        m.push_back(st);
        m.push_back(len);
      }
    }
    std::vector<int64_t> s;
    for (size_t k = 0; k < m.size(); k += 2)
      for (int64_t o = 0; o < m[k + 1]; o += kNormChunk) {
        s.push_back(m[k] + o);
        s.push_back(std::min<int64_t>(kNormChunk, m[k + 1] - o));
      }
    cudaFree(rest_segs_dev);
    rest_segs_dev = nullptr;
    nrest = static_cast<int>(s.size() / 2);
    if (nrest) {
      if (cudaMalloc(&rest_segs_dev, s.size() * sizeof(int64_t)) != cudaSuccess) throw StepError{GLC_ERR_NOMEM};
      if (cudaMemcpy(rest_segs_dev, s.data(), s.size() * sizeof(int64_t), cudaMemcpyHostToDevice) != cudaSuccess)
        throw StepError{GLC_ERR_CUDA};
    }
    rest_for = key;
  }

  int train_step(const int64_t* in_dev, const int64_t* tg_dev, int B, int S, float* loss_out);
};

int Trainer::train_step(const int64_t* in_dev, const int64_t* tg_dev, int B, int S,
                        float* loss_out) {
  const auto& c = model->cfg;
  if (B <= 0 || S <= 0) return ctx->fail(GLC_ERR_INVALID, "train_step: empty batch");
  if (S > c.max_seq_len) return ctx->fail(GLC_ERR_INVALID, "train_step: sequence longer than max_seq_len");
  const int T = B * S;
  const uint64_t l0 = ctx->launches;
  try {
    // TrainStep (trainer.go:462-505); every gradient is rewritten below
    model->scale_pending = false;
    ++step;
    lr = get_lr(step);
    // ZeroGrad (optimizer.go:79-83): existing gradients become zero; the
    // first GradFn that writes one overwrites instead of adding.
    std::fill(model->grad_live.begin(), model->grad_live.end(), 0);
    for (auto& n : model->param_nodes) {
      n.grad_live = false;
      n.grad_round = nullptr;
    }
    tape->reset();
    TraceRange trace_step(ctx, "glc train_step");
    Node* logits = nullptr;
    {
      TraceRange trace(ctx, "forward");
      logits = model->forward(*tape, in_dev, B, S);
    }
    if (row_cap < T) {
      cudaFree(row_logp);
      if (cudaMalloc(&row_logp, sizeof(float) * T) != cudaSuccess) throw StepError{GLC_ERR_NOMEM};
      row_cap = T;
    }
    float* d_loss = static_cast<float*>(scalars);
    float* d_scale = d_loss + 1;
    double* d_norm = reinterpret_cast<double*>(static_cast<char*>(scalars) + 8);
    const int W = c.world_size > 0 ? c.world_size : 1;
    // Gradient hooks.  Before the GradFns run, count each parameter's
    // consumers in the run order (the tied embedding has two; the fused
    // q/k/v and gate/up views count for each member) and zero the allocated
    // gradients nothing will write.  With W > 1, each GradFn's completion
    // lowers its parameters' counts; a bucket whose parameters are all final
    // is summed over the ranks on the communication stream while the
    // backward continues on the compute stream.
    const bool dp = W > 1;
    const int np = model->num_params(), nb = static_cast<int>(model->bucket_begin.size());
    // one GPU: the clip norm's squares come from the dW GEMM epilogues (with
    // data parallelism the norm is of the summed gradient: one pass after it)
    if (!dp && !model->norm_slots) {
      long long cap = 0;
      for (int i = 0; i < np; ++i)
        if (model->rows[i] > 1) cap += gemm_sumsq_slots(model->rows[i], model->cols[i]);
      const long long rest = model->total / kNormChunk + 2LL * np + 64;  // chunks of the remaining pass
      const long long lvl = (cap + rest) / 1024 + 1;
      if (cudaMalloc(&model->norm_slots, sizeof(double) * static_cast<size_t>(cap + rest + lvl)) == cudaSuccess) {
        model->norm_slot_cap = cap;
        model->norm_lvl = model->norm_slots + cap + rest;
        model->norm_lvl_cap = lvl;
      } else {
        model->norm_slots = nullptr;
        cudaGetLastError();
      }
    }
    model->norm_fused = !dp && model->norm_slots != nullptr;
    model->norm_slot_used = 0;
    if (dp && static_cast<int>(bucket_ev.size()) != nb) {
      for (int b = static_cast<int>(bucket_ev.size()); b < nb; ++b) {
        cudaEvent_t e;
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) throw StepError{GLC_ERR_CUDA};
        bucket_ev.push_back(e);
      }
      if (!comm_done && cudaEventCreateWithFlags(&comm_done, cudaEventDisableTiming) != cudaSuccess)
        throw StepError{GLC_ERR_CUDA};
    }
    auto for_params = [](Node* p, const std::function<void(int)>& f) {
      if (p->param >= 0) f(p->param);
      for (int i : p->group) f(i);
    };
    // per-bucket clip-norm tables for the gradients allocated so far
    if (dp) refresh_dp_chunks();
    const std::vector<char> alloc_at_start = dp ? model->grad_allocated : std::vector<char>();
    auto launch_bucket = [&](int b) {
      if (bucket_launched[b]) return;
      bucket_launched[b] = 1;
      if (cudaEventRecord(bucket_ev[b], ctx->stream) != cudaSuccess ||
          cudaStreamWaitEvent(ctx->comm_stream, bucket_ev[b], 0) != cudaSuccess)
        throw StepError{GLC_ERR_CUDA};
      ck(dp_allreduce_on(ctx, model->grads + model->bucket_begin[b],
                         static_cast<size_t>(model->bucket_end[b] - model->bucket_begin[b]), ctx->comm_stream));
      // the bucket's summed gradients are final: their squares, 32 blocks
      // beside the backward
      const int c0 = dp_chunk_off[b], c1 = dp_chunk_off[b + 1];
      if (c1 > c0)
        ck(grad_sumsq_chunks(ctx, model->grads, dp_chunks_dev + 2 * static_cast<int64_t>(c0), c1 - c0, 32,
                             dp_slots + c0, 0.0, ctx->comm_stream));
    };
    const Tape::OrderHook before = [&](const std::vector<Node*>& run) {
      consumers.assign(np, 0);
      for (Node* n : run)
        for (Node* p : n->parents) for_params(p, [&](int i) { ++consumers[i]; });
      if (model->norm_fused) {
        model->last_consumer.assign(np, nullptr);
        for (Node* n : run)
          for (Node* p : n->parents) for_params(p, [&](int i) { model->last_consumer[i] = n; });
        model->norm_covered.assign(np, 0);
        if (cudaMemsetAsync(model->norm_slots, 0, sizeof(double) * static_cast<size_t>(model->norm_slot_cap),
                            ctx->stream) != cudaSuccess)
          throw StepError{GLC_ERR_CUDA};
      }
      for (int i = 0; i < np; ++i)
        if (consumers[i] == 0 && model->grad_allocated[i] && !model->grad_live[i]) {
          if (cudaMemsetAsync(model->grads + model->offset[i], 0, sizeof(float) * model->rows[i] * model->cols[i],
                              ctx->stream) != cudaSuccess)
            throw StepError{GLC_ERR_CUDA};
          model->grad_live[i] = 1;
        }
      if (dp) {
        bucket_pending.assign(nb, 0);
        bucket_launched.assign(nb, 0);
        for (int i = 0; i < np; ++i)
          if (consumers[i] > 0) ++bucket_pending[model->bucket_of[i]];
      }
    };
    const Tape::NodeHook after = [&](Node* n) {
      if (!dp) return;
      for (Node* p : n->parents)
        for_params(p, [&](int i) {
          if (--consumers[i] != 0) return;
          // final: an allocated gradient no GradFn wrote this step is zero
          // before its bucket is summed over the ranks
          if (model->grad_allocated[i] && !model->grad_live[i]) {
            if (cudaMemsetAsync(model->grads + model->offset[i], 0,
                                sizeof(float) * model->rows[i] * model->cols[i], ctx->stream) != cudaSuccess)
              throw StepError{GLC_ERR_CUDA};
            model->grad_live[i] = 1;
          }
          if (--bucket_pending[model->bucket_of[i]] == 0) launch_bucket(model->bucket_of[i]);
        });
    };
    std::optional<TraceRange> trace_bwd;
    trace_bwd.emplace(ctx, "loss + backward");
    if (model->llama) {
      // loss node with the CE GradFn; the kernel writes (p - onehot)/N over
      // the logits, which nothing reads afterwards.  With W data-parallel
      // ranks the mean is over the global batch: scale 1/(W*T).
      const float scale = 1.0f / static_cast<float>(static_cast<int64_t>(W) * T);
      ck(softmax_ce(ctx, logits->data, tg_dev, T, c.vocab_size, scale, row_logp, d_loss, true, true, ctx->stream,
                    /*fast_exp=*/true));
      Node* lossn = tape->make(1, 1);
      lossn->require_grad = true;
      lossn->parents = {logits};
      lossn->grad_fn = [logits]() {
        logits->grad = logits->data;
        logits->grad_live = true;
        logits->grad_round = logits->data;
      };
      tape->backward(lossn, false, before, after);
    } else {
      ck(softmax_ce(ctx, logits->data, tg_dev, T, c.vocab_size, 1.0f, row_logp, d_loss, false, false, ctx->stream));
      // logits.Backward(): Grad is nil, so it is seeded with ones (grad.go:45-50)
      tape->backward(logits, true, before, after);
    }
    // a parameter whose gradient exists but received nothing this step is zero
    for (int i = 0; i < model->num_params(); ++i)
      if (model->grad_allocated[i] && !model->grad_live[i]) {
        if (cudaMemsetAsync(model->grads + model->offset[i], 0, sizeof(float) * model->rows[i] * model->cols[i],
                            ctx->stream) != cudaSuccess)
          throw StepError{GLC_ERR_CUDA};
        model->grad_live[i] = 1;
      }
    refresh_segments();
    trace_bwd.reset();
    if (dp) {
      TraceRange trace(ctx, "gradient sums (remaining buckets)");
      // buckets no GradFn completed (no consumer this step), then clipping
      // waits for every sum
      for (int b = 0; b < nb; ++b) launch_bucket(b);
      if (cudaEventRecord(comm_done, ctx->comm_stream) != cudaSuccess ||
          cudaStreamWaitEvent(ctx->stream, comm_done, 0) != cudaSuccess)
        throw StepError{GLC_ERR_CUDA};
    }
    if (nseg > 0) {
      TraceRange trace(ctx, "clip + AdamW");
      // GradientClipping (optimizer.go:169-196) then AdamW.Step (:37-76)
      if (model->norm_fused) {
        // the GEMM epilogues' slots, then the gradients they did not reach
        refresh_rest_segments();
        const int bx = 1;  // one block per chunk
        if (nrest > 0)
          ck(grad_sumsq(ctx, model->grads, rest_segs_dev, nrest, bx, model->norm_slots + model->norm_slot_used,
                        rest_elems, ctx->stream));
        ck(grad_norm_finish(ctx, model->norm_slots, model->norm_slot_used + static_cast<long long>(bx) * nrest,
                            c.grad_clip_norm, d_norm, d_scale, ctx->stream, model->norm_lvl, model->norm_lvl_cap));
      } else if (dp && model->grad_allocated == alloc_at_start && dp_nchunks > 0) {
        // the per-bucket sums taken after each allreduce (this step allocated
        // no new gradient, so the tables cover every one)
        ck(grad_norm_finish(ctx, dp_slots, dp_nchunks, c.grad_clip_norm, d_norm, d_scale, ctx->stream,
                            dp_slots + dp_nchunks, dp_slots_cap - dp_nchunks));
      } else {
        ck(grad_norm(ctx, model->grads, segs_dev, nseg, c.grad_clip_norm, d_norm, d_scale, nullptr, 0,
                     static_cast<double>(seg_elems), ctx->stream));
      }
      ++adam_step;
      ck(adamw(ctx, model->params, model->grads, model->m, model->v, model->shadow, segs_dev, nseg, d_scale, lr,
               c.beta1, c.beta2, c.epsilon, c.weight_decay, adam_step, static_cast<double>(seg_elems), ctx->stream,
               /*write_grad=*/false));
      if (cudaMemcpyAsync(model->pending_scale, d_scale, sizeof(float), cudaMemcpyDeviceToDevice, ctx->stream) !=
          cudaSuccess)
        throw StepError{GLC_ERR_CUDA};
      model->scale_pending = true;
    }
    TraceRange trace_sync(ctx, "loss readback (waits for the step)");
    if (cudaMemcpyAsync(loss_host, scalars, 16, cudaMemcpyDeviceToHost, ctx->stream) != cudaSuccess)
      throw StepError{GLC_ERR_CUDA};
    if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) throw StepError{GLC_ERR_CUDA};
    int err = 0;
    cudaMemcpy(&err, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost);
    if (err) {
      cudaMemset(ctx->d_err, 0, sizeof(int));
      return ctx->fail(GLC_ERR_DEVICE, "train_step: a kernel's bounded wait ran out (device error " + std::to_string(err) + ")");
    }
    std::memcpy(&last_norm, reinterpret_cast<char*>(loss_host) + 8, sizeof(double));
    if (loss_out) *loss_out = loss_host[0];
    last_launches = ctx->launches - l0;
    return 0;
  } catch (const StepError& e) {
    cudaError_t ce = cudaGetLastError();
    if (ctx->last_error.empty() || e.code == GLC_ERR_CUDA)
      ctx->last_error = std::string("train_step failed") + (ce != cudaSuccess ? std::string(": ") + cudaGetErrorString(ce) : "");
    return e.code;
  }
}

}  // namespace glc

// ---------------------------------------------------------------- C ABI
struct glc_model {
  glc::Model impl;
};
struct glc_trainer {
  glc::Trainer impl;
};

using glc::Context;

namespace glc {
bool param_sizes(const glc_train_config& cfg, std::vector<int64_t>* sizes) {
  Model model;  // layout only: no device memory
  if (!model.layout(cfg)) return false;
  sizes->clear();
  for (int i = 0; i < model.num_params(); ++i) sizes->push_back(model.rows[i] * model.cols[i]);
  return true;
}
}  // namespace glc

extern "C" {

int glc_default_train_config(glc_train_config* c) {
  if (!c) return GLC_ERR_INVALID;
  std::memset(c, 0, sizeof(*c));
  // DefaultTrainConfig (pkg/train/trainer.go:43-69)
  c->vocab_size = 32000;
  c->hidden_size = 512;
  c->num_layers = 8;
  c->num_heads = 8;
  c->intermediate_size = 1408;
  c->max_seq_len = 512;
  c->batch_size = 4;
  c->block_size = 256;
  c->learning_rate = 3e-4f;
  c->weight_decay = 0.01f;
  c->warmup_steps = 100;
  c->max_steps = 10000;
  c->grad_clip_norm = 1.0f;
  // NewAdamW (optimizer.go:24-34)
  c->beta1 = 0.9f;
  c->beta2 = 0.999f;
  c->epsilon = 1e-8f;
  c->num_kv_heads = 0;
  c->semantics = GLC_SEMANTICS_REFERENCE;
  c->norm_eps = 1e-5f;
  c->rope_theta = 10000.0f;
  c->init_std = 0.02f;
  c->seed = 42;
  c->world_size = 1;
  return GLC_OK;
}

int glc_model_create(glc_ctx* ctx, const glc_train_config* cfg, glc_model** out) {
  if (!ctx || !cfg || !out) return GLC_ERR_INVALID;
  *out = nullptr;
  auto* m = new glc_model();
  int rc = m->impl.init(reinterpret_cast<Context*>(ctx), *cfg);
  if (rc) {
    delete m;
    return rc;
  }
  *out = m;
  return GLC_OK;
}

int glc_model_destroy(glc_model* m) {
  if (!m) return GLC_ERR_INVALID;
  cudaStreamSynchronize(m->impl.ctx->stream);
  delete m;
  return GLC_OK;
}

int glc_model_num_params(glc_model* m, int* n, int64_t* total) {
  if (!m) return GLC_ERR_INVALID;
  if (n) *n = m->impl.num_params();
  if (total) *total = m->impl.total;
  return GLC_OK;
}

int glc_dp_bucket_plan(const glc_train_config* cfg, int64_t* begin, int64_t* end, int capacity, int* count) {
  if (!cfg || !count || capacity < 0 || (capacity > 0 && (!begin || !end))) return GLC_ERR_INVALID;
  glc::Model model;  // layout only: no device memory
  if (!model.layout(*cfg)) return GLC_ERR_INVALID;
  const int n = static_cast<int>(model.bucket_begin.size());
  *count = n;
  for (int i = 0; i < n && i < capacity; ++i) {
    begin[i] = model.bucket_begin[i];
    end[i] = model.bucket_end[i];
  }
  return GLC_OK;
}

int glc_model_param_info(glc_model* m, int idx, int64_t* offset, int64_t* rows, int64_t* cols, int* has_grad) {
  if (!m || idx < 0 || idx >= m->impl.num_params()) return GLC_ERR_INVALID;
  if (offset) *offset = m->impl.offset[idx];
  if (rows) *rows = m->impl.rows[idx];
  if (cols) *cols = m->impl.cols[idx];
  if (has_grad) *has_grad = m->impl.grad_allocated[idx];
  return GLC_OK;
}

static int arena_copy(glc_model* m, float* dev, float* host, const float* chost, int64_t n, bool to_dev) {
  if (!m || n != m->impl.total || (!host && !chost)) return GLC_ERR_INVALID;
  Context* c = m->impl.ctx;
  cudaError_t e = to_dev ? cudaMemcpyAsync(dev, chost, sizeof(float) * n, cudaMemcpyHostToDevice, c->stream)
                         : cudaMemcpyAsync(host, dev, sizeof(float) * n, cudaMemcpyDeviceToHost, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  return e == cudaSuccess ? GLC_OK : c->fail_cuda(e, "model arena copy");
}

int glc_model_set_params(glc_model* m, const float* host, int64_t n) {
  int rc = arena_copy(m, m ? m->impl.params : nullptr, nullptr, host, n, true);
  if (rc) return rc;
  Context* c = m->impl.ctx;
  rc = glc::round_copy(c, m->impl.params, m->impl.shadow, static_cast<size_t>(n), c->stream);
  if (rc) return rc;
  return cudaStreamSynchronize(c->stream) == cudaSuccess ? GLC_OK : GLC_ERR_CUDA;
}
int glc_model_get_params(glc_model* m, float* host, int64_t n) {
  return arena_copy(m, m ? m->impl.params : nullptr, host, nullptr, n, false);
}
int glc_model_get_grads(glc_model* m, float* host, int64_t n) {
  if (m && n == m->impl.total && m->impl.scale_pending) {
    // the gradients as GradientClipping left them (optimizer.go:169-196)
    glc::Model& md = m->impl;
    int rc = glc::scale_in_place(md.ctx, md.grads, static_cast<size_t>(md.total), md.pending_scale, md.ctx->stream);
    if (rc) return rc;
    md.scale_pending = false;
  }
  return arena_copy(m, m ? m->impl.grads : nullptr, host, nullptr, n, false);
}
int glc_model_get_moments(glc_model* m, float* mh, float* vh, int64_t n) {
  int rc = arena_copy(m, m ? m->impl.m : nullptr, mh, nullptr, n, false);
  if (rc) return rc;
  return arena_copy(m, m->impl.v, vh, nullptr, n, false);
}

int glc_trainer_create(glc_model* m, glc_trainer** out) {
  if (!m || !out) return GLC_ERR_INVALID;
  auto* t = new glc_trainer();
  glc::Trainer& tr = t->impl;
  tr.model = &m->impl;
  tr.ctx = m->impl.ctx;
  tr.tape.reset(new glc::Tape(tr.ctx, tr.model));
  if (cudaMalloc(&tr.scalars, 64) != cudaSuccess || cudaMallocHost(&tr.loss_host, 64) != cudaSuccess) {
    delete t;
    return GLC_ERR_NOMEM;
  }
  cudaMemset(tr.scalars, 0, 64);
  *out = t;
  return GLC_OK;
}

int glc_trainer_destroy(glc_trainer* t) {
  if (!t) return GLC_ERR_INVALID;
  cudaStreamSynchronize(t->impl.ctx->stream);
  delete t;
  return GLC_OK;
}

int glc_train_step(glc_trainer* t, const int64_t* inputs, const int64_t* targets, int B, int S, float* loss) {
  if (!t || !inputs || !targets || B <= 0 || S <= 0) return GLC_ERR_INVALID;
  glc::Trainer& tr = t->impl;
  const int T = B * S;
  if (tr.tok_cap < T) {
    cudaFree(tr.tok_dev);
    if (cudaMalloc(&tr.tok_dev, sizeof(int64_t) * 2 * T) != cudaSuccess) return GLC_ERR_NOMEM;
    tr.tok_cap = T;
  }
  cudaError_t e = cudaMemcpyAsync(tr.tok_dev, inputs, sizeof(int64_t) * T, cudaMemcpyHostToDevice, tr.ctx->stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(tr.tok_dev + T, targets, sizeof(int64_t) * T, cudaMemcpyHostToDevice, tr.ctx->stream);
  if (e != cudaSuccess) return tr.ctx->fail_cuda(e, "train_step: token upload");
  return tr.train_step(tr.tok_dev, tr.tok_dev + T, B, S, loss);
}

int glc_train_step_device(glc_trainer* t, const int64_t* in_dev, const int64_t* tg_dev, int B, int S, float* loss) {
  if (!t || !in_dev || !tg_dev || B <= 0 || S <= 0) return GLC_ERR_INVALID;
  return t->impl.train_step(in_dev, tg_dev, B, S, loss);
}

int glc_trainer_last_stats(glc_trainer* t, double* grad_norm, float* lr, int* step) {
  if (!t) return GLC_ERR_INVALID;
  if (grad_norm) *grad_norm = t->impl.last_norm;
  if (lr) *lr = t->impl.lr;
  if (step) *step = t->impl.step;
  return GLC_OK;
}

int glc_trainer_last_launches(glc_trainer* t, uint64_t* n) {
  if (!t || !n) return GLC_ERR_INVALID;
  *n = t->impl.last_launches;
  return GLC_OK;
}

// ---------------------------------------------------------------- checkpoints
// The files are written and read on the host in chunks (checkpoint.cpp); these
// move each chunk between a device arena and host memory on the context's
// stream, one synchronous copy at a time.
static bool chunk_d2h(Context* c, const float* dev, int64_t off, int64_t n, float* dst) {
  return cudaMemcpyAsync(dst, dev + off, sizeof(float) * n, cudaMemcpyDeviceToHost, c->stream) == cudaSuccess &&
         cudaStreamSynchronize(c->stream) == cudaSuccess;
}
static bool chunk_h2d(Context* c, float* dev, int64_t off, int64_t n, const float* src) {
  return cudaMemcpyAsync(dev + off, src, sizeof(float) * n, cudaMemcpyHostToDevice, c->stream) == cudaSuccess &&
         cudaStreamSynchronize(c->stream) == cudaSuccess;
}
static int ckpt_status(Context* c, int rc) {
  if (rc) c->last_error = glc::host_error();
  return rc;
}

int glc_trainer_save_checkpoint(glc_trainer* t, const char* dir, char* path_out, size_t path_cap) {
  if (!t || !dir) return GLC_ERR_INVALID;
  glc::Trainer& tr = t->impl;
  glc::Model& md = *tr.model;
  Context* c = tr.ctx;
  // fmt.Sprintf("%s/checkpoint_%d.bin", SavePath, step) (trainer.go:555)
  const std::string path = std::string(dir) + "/checkpoint_" + std::to_string(tr.step) + ".bin";
  if (path_out) {
    if (path_cap <= path.size()) return c->fail(GLC_ERR_INVALID, "save_checkpoint: path buffer too small");
    std::memcpy(path_out, path.c_str(), path.size() + 1);
  }
  if (cudaStreamSynchronize(c->stream) != cudaSuccess) return c->fail(GLC_ERR_CUDA, "save_checkpoint: sync");
  std::vector<int64_t> sizes;
  for (int i = 0; i < md.num_params(); ++i) sizes.push_back(md.rows[i] * md.cols[i]);
  return ckpt_status(c, glc::ckpt_text_write(path.c_str(), tr.step, md.cfg, sizes,
                                             [&](int64_t off, int64_t n, float* dst) {
                                               return chunk_d2h(c, md.params, off, n, dst);
                                             }));
}

int glc_trainer_save_state(glc_trainer* t, const char* path) {
  if (!t || !path) return GLC_ERR_INVALID;
  glc::Trainer& tr = t->impl;
  glc::Model& md = *tr.model;
  Context* c = tr.ctx;
  if (cudaStreamSynchronize(c->stream) != cudaSuccess) return c->fail(GLC_ERR_CUDA, "save_state: sync");
  const float* arenas[3] = {md.params, md.m, md.v};
  return ckpt_status(c, glc::state_write(path, glc::StateInfo{tr.step, tr.adam_step}, md.cfg, md.total,
                                         [&](int a, int64_t off, int64_t n, float* dst) {
                                           return chunk_d2h(c, arenas[a], off, n, dst);
                                         }));
}

int glc_trainer_load_state(glc_trainer* t, const char* path) {
  if (!t || !path) return GLC_ERR_INVALID;
  glc::Trainer& tr = t->impl;
  glc::Model& md = *tr.model;
  Context* c = tr.ctx;
  if (cudaStreamSynchronize(c->stream) != cudaSuccess) return c->fail(GLC_ERR_CUDA, "load_state: sync");
  float* arenas[3] = {md.params, md.m, md.v};
  glc::StateInfo info{};
  int rc = ckpt_status(c, glc::state_read(path, md.cfg, md.total, &info,
                                          [&](int a, int64_t off, int64_t n, const float* src) {
                                            return chunk_h2d(c, arenas[a], off, n, src);
                                          }));
  if (rc) return rc;
  // the GEMM operand copy of the weights follows the parameters
  rc = glc::round_copy(c, md.params, md.shadow, static_cast<size_t>(md.total), c->stream);
  if (rc) return rc;
  if (cudaStreamSynchronize(c->stream) != cudaSuccess) return c->fail(GLC_ERR_CUDA, "load_state: sync");
  tr.step = info.step;
  tr.adam_step = info.adam_step;
  tr.lr = info.step > 0 ? tr.get_lr(info.step) : 0.f;
  md.scale_pending = false;
  return GLC_OK;
}

}  // extern "C"
