/*
 * oracle.h — CPU restatement of gollama's training hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This code is the checker for libgollama_cuda: the
 * parity tests, the smoke check and bench.py's CPU-baseline leg call it; the
 * product path never does.
 *
 * Parity status: UNPINNED.  The reference (pure Go, github.com/timastras9/
 * gollama) ships no tests, fixtures or golden vectors, and no Go toolchain is
 * available to run it, so this restatement is checked only by known-answer
 * tests derived from the Go source, closed forms and finite differences.
 *
 * One source, two builds: prefix orc_ computes in float32 exactly as the Go
 * code does (same loop order, float32 accumulators, the same float64 casts,
 * no fused multiply-add); prefix orcd_ is the same code in float64, used for
 * finite-difference checks of the backward.
 *
 * Two semantics (orc_config.mode):
 *   ORC_MODE_REFERENCE — pkg/train exactly, quirks included: learned position
 *     embedding, multi-head attention without a backward, simplified RMSNorm
 *     backward, backward seeded with ones on the logits.
 *   ORC_MODE_LLAMA — the Llama-style decoder: RoPE (consecutive pairs,
 *     pkg/model/rope.go), grouped-query attention (pkg/model/attention.go),
 *     causal attention backward, full RMSNorm backward, embedding-gradient
 *     scatter, backward seeded by the softmax-cross-entropy gradient.
 */
#ifndef GOLLAMA_ORACLE_H
#define GOLLAMA_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_MODE_REFERENCE 0
#define ORC_MODE_LLAMA 1

typedef struct {
  int vocab;      /* TrainConfig.VocabSize */
  int hidden;     /* TrainConfig.HiddenSize */
  int layers;     /* TrainConfig.NumLayers */
  int heads;      /* TrainConfig.NumHeads */
  int kv_heads;   /* Llama mode only; reference mode uses heads */
  int inter;      /* TrainConfig.IntermediateSize */
  int max_seq;    /* TrainConfig.MaxSeqLen (position-embedding rows, RoPE table) */
  float norm_eps; /* RMSNormTrainable.Eps = 1e-5 (pkg/train/trainer.go:136) */
  float rope_theta;
  int mode;
} orc_config;

typedef struct {
  /* AdamW (pkg/train/optimizer.go:10-21) */
  float lr, beta1, beta2, eps, weight_decay;
  int adam_step;
  /* LRScheduler (pkg/train/optimizer.go:141-145) */
  float initial_lr;
  int warmup_steps, total_steps;
  /* TrainConfig.GradClipNorm and Trainer.step (pkg/train/trainer.go:31,440) */
  float grad_clip;
  int trainer_step;
} orc_optim_state;

#define ORC_DECLARE(P, real)                                                                                  \
  int P##num_params(const orc_config* c);                                                                     \
  int64_t P##param_total(const orc_config* c);                                                                \
  void P##param_info(const orc_config* c, int idx, int64_t* offset, int64_t* rows, int64_t* cols);             \
  void P##set_threads(int nthreads, int literal);                                                             \
  /* single ops */                                                                                            \
  void P##matmul_transpose_b(const real* a, const real* b, real* out, int M, int K, int N);                   \
  void P##matmul_grad_da(const real* dc, const real* b, real* da, int M, int K, int N);                       \
  void P##matmul_grad_db(const real* dc, const real* a, real* db, int M, int K, int N);                       \
  void P##rmsnorm_fwd(const real* x, const real* w, real* out, real* rms, int rows, int cols, float eps);      \
  void P##rmsnorm_bwd(const real* x, const real* w, const real* rms, const real* dout, real* dx, real* dw,     \
                      int rows, int cols, int full);                                                          \
  float P##exp32(float x);                                                                                    \
  float P##fp16_to_fp32(uint16_t h);                                                                          \
  int P##dequantize(const uint8_t* data, real* out, int64_t n, int type);                                     \
  int P##linear_bwd_dx_q(const real* dy, const uint8_t* wq, int type, real* dx, int M, int K, int N);          \
  void P##exp32_array(const float* x, float* y, int64_t n);                                                   \
  float P##log32(float x);                                                                                    \
  double P##go_exp(double x);                                                                                 \
  double P##go_log(double x);                                                                                 \
  void P##silu_fwd(const real* x, real* out, real* sig, int64_t n);                                           \
  void P##silu_bwd(const real* x, const real* sig, const real* dout, real* dx, int64_t n);                    \
  real P##softmax_ce(const real* logits, const int64_t* targets, int rows, int V, real* probs);               \
  void P##softmax_ce_grad(const real* probs, const int64_t* targets, int rows, int V, real* dlogits);         \
  void P##rope_table(int dim, int max_seq, float theta, real* cos_t, real* sin_t);                            \
  void P##rope_apply(real* x, int T, int S, int nh, int hd, const real* cos_t, const real* sin_t, int inverse); \
  void P##attention_fwd(const real* q, const real* k, const real* v, real* out, int T, int S, int H, int Hkv,  \
                        int hd);                                                                              \
  void P##attention_bwd(const real* q, const real* k, const real* v, const real* dout, real* dq, real* dk,    \
                        real* dv, int T, int S, int H, int Hkv, int hd);                                      \
  double P##grad_clip(real* grads, const uint8_t* has_grad, const orc_config* c, float max_norm);            \
  void P##adamw_step(real* params, const real* grads, const uint8_t* has_grad, real* m, real* v,             \
                     const orc_config* c, orc_optim_state* st);                                               \
  float P##get_lr(const orc_optim_state* st, int step);                                                       \
  /* whole model */                                                                                           \
  real P##forward_backward(const orc_config* c, const real* params, real* grads, uint8_t* has_grad,          \
                           const int64_t* inputs, const int64_t* targets, int B, int S, int backward);        \
  real P##train_step(const orc_config* c, real* params, real* grads, uint8_t* has_grad, real* m, real* v,     \
                     orc_optim_state* st, const int64_t* inputs, const int64_t* targets, int B, int S,        \
                     double* grad_norm);

ORC_DECLARE(orc_, float)
ORC_DECLARE(orcd_, double)

#ifdef __cplusplus
}
#endif
#endif
