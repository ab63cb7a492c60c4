// C ABI of the individual ops: what a GradFn of the reference tape
// (pkg/tensor/grad.go, pkg/train/trainer.go) calls through the cgo package.
#include <algorithm>
#include <vector>

#include "glc_internal.h"

using glc::Context;

static inline Context* C_(glc_ctx* c) { return reinterpret_cast<Context*>(c); }

extern "C" {

int glc_rmsnorm_fwd(glc_ctx* ctx, const float* x, const float* w, float* y, float* rms, int rows, int cols, float eps,
                    int round_out) {
  if (!ctx) return GLC_ERR_INVALID;
  return glc::rmsnorm_fwd(C_(ctx), x, w, y, rms, rows, cols, eps, round_out != 0, C_(ctx)->stream);
}

int glc_rmsnorm_bwd(glc_ctx* ctx, const float* x, const float* w, const float* rms, const float* dy, float* dx,
                    float* dx_round, float* dw, int rows, int cols, int full, int dx_accumulate, int dw_accumulate) {
  if (!ctx) return GLC_ERR_INVALID;
  return glc::rmsnorm_bwd(C_(ctx), x, w, rms, dy, dx, dx_round, dw, rows, cols, full != 0, dx_accumulate != 0,
                          dw_accumulate != 0, nullptr, 0, C_(ctx)->stream);
}

int glc_swiglu_fwd(glc_ctx* ctx, const float* gate, const float* up, float* h, size_t n, int round_out) {
  if (!ctx) return GLC_ERR_INVALID;
  return glc::swiglu_fwd(C_(ctx), gate, up, n, h, n, 1, n, round_out != 0, C_(ctx)->stream);
}

int glc_swiglu_bwd(glc_ctx* ctx, const float* gate, const float* up, const float* dh, float* dgate, float* dup,
                   size_t n, int accumulate, int round_out) {
  if (!ctx) return GLC_ERR_INVALID;
  return glc::swiglu_bwd(C_(ctx), gate, up, n, dh, n, dgate, dup, n, 1, n, accumulate != 0, round_out != 0,
                         C_(ctx)->stream);
}

int glc_rope(glc_ctx* ctx, float* x, int T, int S, int nh, int hd, const float* cos_t, const float* sin_t, int inverse,
             int round_out) {
  if (!ctx) return GLC_ERR_INVALID;
  return glc::rope(C_(ctx), x, nh * hd, T, S, nh, hd, cos_t, sin_t, inverse != 0, round_out != 0, C_(ctx)->stream);
}

int glc_rope_table(int hd, int max_seq, float theta, float* cos_host, float* sin_host) {
  if (hd <= 0 || (hd & 1) || max_seq <= 0 || !cos_host || !sin_host) return GLC_ERR_INVALID;
  glc::rope_table_host(hd, max_seq, theta, cos_host, sin_host);
  return GLC_OK;
}

int glc_attention_fwd(glc_ctx* ctx, const float* q, const float* k, const float* v, float* o, float* lse, int B,
                      int S, int H, int Hkv, int hd, int round_out) {
  if (!ctx) return GLC_ERR_INVALID;
  const glc::AttnIO io{q, H * hd, k, Hkv * hd, v, Hkv * hd, nullptr, 0, nullptr, 0, nullptr, 0};
  return glc::attention_fwd(C_(ctx), io, o, lse, B, S, H, Hkv, hd, round_out != 0, C_(ctx)->stream);
}

int glc_attention_bwd(glc_ctx* ctx, const float* q, const float* k, const float* v, const float* o, const float* lse,
                      const float* dO, float* dq, float* dk, float* dv, int B, int S, int H, int Hkv, int hd,
                      int round_dv) {
  if (!ctx || B <= 0 || S <= 0 || H <= 0 || Hkv <= 0) return GLC_ERR_INVALID;
  const size_t nd = static_cast<size_t>(B) * H * S, np = glc::attention_bwd_partial_floats(B, S, H, Hkv, hd);
  void* ws = nullptr;
  int rc = C_(ctx)->workspace(sizeof(float) * (((nd + 63) & ~size_t(63)) + np), &ws);
  if (rc) return rc;
  float* D = static_cast<float*>(ws);
  float* partial = np ? D + ((nd + 63) & ~size_t(63)) : nullptr;
  const glc::AttnIO io{q, H * hd, k, Hkv * hd, v, Hkv * hd, dq, H * hd, dk, Hkv * hd, dv, Hkv * hd};
  return glc::attention_bwd(C_(ctx), io, o, lse, dO, D, partial, B, S, H, Hkv, hd, round_dv != 0, C_(ctx)->stream);
}

int glc_softmax_ce(glc_ctx* ctx, float* logits, const int64_t* targets, int rows, int V, float scale, float* row_logp,
                   float* loss, int write_grad, int round_out) {
  if (!ctx) return GLC_ERR_INVALID;
  return glc::softmax_ce(C_(ctx), logits, targets, rows, V, scale, row_logp, loss, write_grad != 0, round_out != 0,
                         C_(ctx)->stream);
}

int glc_softmax_ce_llama(glc_ctx* ctx, float* logits, const int64_t* targets, int rows, int V, float scale,
                         float* row_logp, float* loss, int write_grad, int round_out) {
  if (!ctx) return GLC_ERR_INVALID;
  return glc::softmax_ce(C_(ctx), logits, targets, rows, V, scale, row_logp, loss, write_grad != 0, round_out != 0,
                         C_(ctx)->stream, /*fast_exp=*/true);
}

int glc_embed_fwd(glc_ctx* ctx, const int64_t* tokens, const float* E, const float* P, float* out, int T, int S, int d,
                  int V) {
  if (!ctx) return GLC_ERR_INVALID;
  return glc::embed_fwd(C_(ctx), tokens, E, P, out, T, S, d, V, C_(ctx)->stream);
}

int glc_embed_bwd(glc_ctx* ctx, const int64_t* tokens_host, int T, const float* dh, float* dE, int d, int V) {
  if (!ctx || T < 0 || (T && !tokens_host)) return GLC_ERR_INVALID;
  if (T == 0) return GLC_OK;
  Context* c = C_(ctx);
  std::vector<int> seg_tok, seg_start, order;
  glc::embed_segments_host(tokens_host, T, V, seg_tok, seg_start, order);
  const int nseg = static_cast<int>(seg_tok.size());
  std::vector<int> packed(seg_tok);
  packed.insert(packed.end(), seg_start.begin(), seg_start.end());
  packed.insert(packed.end(), order.begin(), order.end());
  void* ws = nullptr;
  int rc = c->workspace(packed.size() * sizeof(int), &ws);
  if (rc) return rc;
  int* dev = static_cast<int*>(ws);
  cudaError_t e = cudaMemcpyAsync(dev, packed.data(), packed.size() * sizeof(int), cudaMemcpyHostToDevice, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) return c->fail_cuda(e, "embed_bwd: segment upload");
  return glc::embed_bwd(c, dev, dev + nseg, dev + 2 * nseg + 1, nseg, dh, dE, d, c->stream);
}

int glc_embed_bwd_device(glc_ctx* ctx, const int64_t* tokens_dev, int T, const float* dh, float* dE, int d, int V) {
  if (!ctx || T < 0 || (T && !tokens_dev)) return GLC_ERR_INVALID;
  if (T == 0) return GLC_OK;
  Context* c = C_(ctx);
  const glc::EmbedSegLayout L(T);
  void* ws = nullptr;
  int rc = c->workspace(static_cast<size_t>(L.total) * sizeof(int), &ws);
  if (rc) return rc;
  int* dev = static_cast<int*>(ws);
  rc = glc::embed_segments_device(c, tokens_dev, T, V, dev, c->stream);
  if (rc) return rc;
  return glc::embed_bwd(c, dev + L.seg_tok, dev + L.seg_start, dev + L.order, T, dh, dE, d, c->stream, dev + L.nseg);
}

// Uploads a host segment table to the workspace (after `offset` bytes).
static int upload_segs(Context* c, const int64_t* segs, int nseg, size_t offset, int64_t** out, double* elems) {
  if (nseg <= 0 || !segs) return c->fail(GLC_ERR_INVALID, "segment table is empty");
  *elems = 0;
  for (int i = 0; i < nseg; ++i) {
    if (segs[2 * i] < 0 || segs[2 * i + 1] < 0 || (segs[2 * i] & 3) || (segs[2 * i + 1] & 3))
      return c->fail(GLC_ERR_INVALID, "segments must start and end on multiples of 4 floats");
    *elems += static_cast<double>(segs[2 * i + 1]);
  }
  void* ws = nullptr;
  const size_t bytes = sizeof(int64_t) * 2 * nseg;
  int rc = c->workspace(offset + bytes, &ws);
  if (rc) return rc;
  int64_t* dev = reinterpret_cast<int64_t*>(static_cast<char*>(ws) + offset);
  cudaError_t e = cudaMemcpyAsync(dev, segs, bytes, cudaMemcpyHostToDevice, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) return c->fail_cuda(e, "segment upload");
  *out = dev;
  return 0;
}

int glc_grad_clip_norm(glc_ctx* ctx, const float* grads, const int64_t* segs_host, int nseg, float max_norm,
                       double* norm_dev, float* scale_dev) {
  if (!ctx || !norm_dev || !scale_dev) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  const int bx_cap = 8 * c->num_sms;
  const size_t partial_bytes = sizeof(double) * static_cast<size_t>(nseg > 0 ? nseg : 1) * (bx_cap + 4);
  int64_t* segs = nullptr;
  double elems = 0;
  int rc = upload_segs(c, segs_host, nseg, partial_bytes, &segs, &elems);
  if (rc) return rc;
  void* ws = nullptr;
  c->workspace(partial_bytes, &ws);
  return glc::grad_norm(c, grads, segs, nseg, max_norm, norm_dev, scale_dev, static_cast<double*>(ws),
                        static_cast<int>(partial_bytes / sizeof(double)), elems, c->stream);
}

int glc_adamw_step(glc_ctx* ctx, float* params, float* grads, float* m, float* v, float* shadow,
                   const int64_t* segs_host, int nseg, const float* clip_scale_dev, float lr, float beta1, float beta2,
                   float eps, float weight_decay, int step) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  int64_t* segs = nullptr;
  double elems = 0;
  int rc = upload_segs(c, segs_host, nseg, 0, &segs, &elems);
  if (rc) return rc;
  return glc::adamw(c, params, grads, m, v, shadow, segs, nseg, clip_scale_dev, lr, beta1, beta2, eps, weight_decay,
                    step, elems, c->stream);
}

int glc_fill(glc_ctx* ctx, float* p, float value, size_t n) {
  if (!ctx) return GLC_ERR_INVALID;
  return glc::fill(C_(ctx), p, value, n, C_(ctx)->stream);
}

int glc_round_tf32(glc_ctx* ctx, const float* src, float* dst, size_t n) {
  if (!ctx) return GLC_ERR_INVALID;
  return glc::round_copy(C_(ctx), src, dst, n, C_(ctx)->stream);
}

int glc_exp32(glc_ctx* ctx, const float* x, float* y, size_t n) {
  if (!ctx) return GLC_ERR_INVALID;
  return glc::exp32(C_(ctx), x, y, n, C_(ctx)->stream);
}

int glc_add_inplace(glc_ctx* ctx, float* dst, const float* src, size_t n) {
  if (!ctx) return GLC_ERR_INVALID;
  return glc::add_inplace(C_(ctx), dst, src, n, C_(ctx)->stream);
}

int glc_gemm_tile_lists(int tiles0, int kb0, int tiles1, int kb1, int clusters, int* out, int capacity, int* used) {
  if (!used || tiles0 < 0 || tiles1 < 0 || kb0 < 0 || kb1 < 0 || clusters <= 0 || tiles0 + tiles1 <= 0)
    return GLC_ERR_INVALID;
  std::vector<int> h;
  *used = 0;
  if (!glc::gemm_tile_lists(tiles0, kb0, tiles1, kb1, clusters, &h)) return GLC_OK;
  if (!out || capacity < static_cast<int>(h.size())) return GLC_ERR_INVALID;
  std::copy(h.begin(), h.end(), out);
  *used = 1;
  return GLC_OK;
}

}  // extern "C"
