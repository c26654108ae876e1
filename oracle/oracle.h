/* oracle.h — CPU restatement of AutoANE's MeZO-LoRA-split projection path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the CUDA library is compared
 * against; it is never linked into, called by, or shipped with libb2p.so.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it.
 *
 * Every function restates a reference function (file:line in the AutoANE tree)
 * in plain C. Layouts follow the reference: channel-first activations [C, S]
 * row-major fp32, weights [out, in] row-major fp32. Matrix products go through
 * cblas_sgemm (OpenBLAS), as the reference's --cpu-only path does through
 * Accelerate's cblas_sgemm.
 */
#ifndef B2P_ORACLE_H
#define B2P_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- xoshiro256+ / splitmix64 (training/train_mezo.m:97-119) ---- */
typedef struct { uint64_t s[4]; } or_xo;
void or_xo_seed(or_xo* st, uint64_t seed);
uint64_t or_xo_next(or_xo* st);

/* perturb_buffer (training/train_mezo.m:122-136): buf[i] += bit ? scale : -scale,
 * 4 sign bits per draw (bits 0..3), a tail of n%4 elements one draw each (bit 0). */
void or_perturb_buffer(or_xo* st, float* buf, size_t n, float scale);

/* Sign bits of the perturbation stream for a sequence of buffers of the given
 * sizes, drawn as perturb_buffer draws them: bit i of `mask` (32-bit words,
 * little-endian bit order) is 1 when parameter i gets +scale. */
void or_sign_mask(uint64_t seed, const int64_t* sizes, int nbuf, uint32_t* mask);

/* ---- LoRA-split trainable-parameter layout (training/train_mezo.m:560-588) ----
 * theta = per layer [Aq r*D | Bq Q*r | Ak r*D | Bk KV*r | Av r*D | Bv KV*r |
 *                    Ao r*Q | Bo D*r | (--lora-ffn: A1 r*D | B1 H*r | A2 r*H | B2 D*r |
 *                    A3 r*D | B3 H*r) | rms_att D | rms_ffn D], then rms_final D. */
typedef struct {
  int64_t Aq, Bq, Ak, Bk, Av, Bv, Ao, Bo, rms_att, rms_ffn; /* offsets inside a layer */
  int64_t layer_size;
  int64_t rms_final; /* offset of rms_final */
  int64_t total;
  int64_t A1, B1, A2, B2, A3, B3; /* FFN adapters (-1 without --lora-ffn) */
} or_layout;
or_layout or_lora_layout(int nlayers, int dim, int q_dim, int kv_dim, int rank);
or_layout or_lora_layout_ffn(int nlayers, int dim, int q_dim, int kv_dim, int hidden, int rank, int ffn);
/* Buffer sizes in perturbation order (11 per layer... 10 per layer + 1). Returns count. */
int or_lora_buffer_sizes(int nlayers, int dim, int q_dim, int kv_dim, int rank, int64_t* sizes_out);
/* The same with the FFN adapters of --lora-ffn after Bo (train_mezo.m:575-582); 16 per layer + 1. */
int or_lora_buffer_sizes_ffn(int nlayers, int dim, int q_dim, int kv_dim, int hidden, int rank, int ffn,
                             int64_t* sizes_out);
/* perturb_lora_weights (train_mezo.m:560-588) over the flat theta. */
void or_perturb_lora(float* theta, int nlayers, int dim, int q_dim, int kv_dim, int rank, uint64_t seed,
                     float scale);
void or_perturb_lora_ffn(float* theta, int nlayers, int dim, int q_dim, int kv_dim, int hidden, int rank, int ffn,
                         uint64_t seed, float scale);

/* ---- model ---- */
typedef struct {
  int dim, hidden, heads, kv_heads, hd, seq, nlayers, vocab, cv, rank;
  float rope_theta, res_alpha;
  /* base weights per layer, fp32 row-major [out, in] */
  const float* const* Wq;
  const float* const* Wk;
  const float* const* Wv;
  const float* const* Wo;
  const float* const* W1;
  const float* const* W2;
  const float* const* W3;
  const float* embed;  /* [vocab, dim] */
  const float* cembed; /* [cv, dim] compact tied embedding (vocab_compact_embed, cpu_ops.h:171) */
  int lora_ffn;        /* --lora-ffn: adapters on W1, W2, W3 as well */
} or_model;

/* ---- ops (training/cpu_ops.h) ---- */
void or_rmsnorm(float* out, const float* x, const float* w, int d, int S);                   /* :7-22 */
void or_rope_forward(float* x, int seq, int dim, int hd, float theta);                       /* :299-315 */
void or_rope_tables(float* cos_out, float* sin_out, int seq, int hd, float theta);           /* same expressions */
void or_sdpa_forward(const float* Q, const float* Kt, const float* Vt, float* out, int heads, int hd,
                     int seq);                                                               /* :321-360 */
float or_cross_entropy(const float* logits, const uint16_t* targets, int V, int S);          /* :108-133 */
void or_lora_addmm(float* out, const float* A, const float* B, const float* x, float* tmp, int out_dim, int rank,
                   int in_dim, int seq);                                                     /* train_mezo.m:694-703 */
void or_sgemm_nn(int M, int N, int K, const float* A, const float* B, float* C, float beta); /* C = A·B + beta C */

/* Row statistics of the classifier for a forward (filled when non-NULL). */
typedef struct {
  float* x_final;   /* [dim, seq] residual stream after the last layer */
  float* xn_final;  /* [dim, seq] after the final RMSNorm */
  float* logits;    /* [seq, cv] */
  float* layer_x;   /* [nlayers+1][dim, seq] residual stream at each layer input (+ final) */
} or_taps;

/* DO_FORWARD_PASS, --cpu-only --lora-split branch (train_mezo.m:1528-1699) with the
 * trainable parameters read from `theta` (or_lora_layout order). Returns the mean CE. */
float or_forward_loss(const or_model* m, const float* theta, const uint16_t* tokens, const uint16_t* ctargets,
                      or_taps* taps);

/* One MeZO-LoRA-split step (train_mezo.m:2938-3012): +eps, forward, -2eps, forward,
 * +eps, g = (L+ - L-)/(2 eps), update with -lr*g; theta updated in place. */
void or_mezo_step(const or_model* m, float* theta, const uint16_t* tokens, const uint16_t* ctargets, uint64_t seed,
                  float eps, float lr, float* loss_plus, float* loss_minus, float* proj_grad);

/* BLAS thread count control (OpenBLAS); returns the count in effect. */
int or_set_threads(int n);

/* ---- backprop-LoRA (P16): train_mezo.m:1982-2117, backprop_lora.h:147-288 ---- */
void or_rmsnorm_bwd(float* dx, float* dw, const float* dy, const float* x, const float* w, int d, int S); /* :24-60 */
void or_rope_backward(float* dx, int seq, int dim, int hd, float theta);                               /* :377-393 */
void or_sdpa_backward(const float* Q, const float* Kt, const float* Vt, const float* da, float* dq, float* dk,
                      float* dv, int heads, int hd, int seq);                                         /* :213-290 */
/* Loss and gradient (theta layout, overwritten) of one sequence: forward on frozen
 * base weights + split LoRA (conv-fused P16), backward through W + B·A. */
float or_p16_grad(const or_model* m, const float* theta, const uint16_t* tokens, const uint16_t* ctargets,
                  float* grad);
/* Full backprop (train.m:686-1192): the P16 gradient plus dW of every projection
 * (dw: per layer Wq, Wk, Wv, Wo, W1, W2, W3, each [out, in]) and the embedding
 * gradient gembed [vocab, dim] (c2f: compact -> full id, NULL = identity). */
float or_full_grad(const or_model* m, const float* theta, const uint16_t* tokens, const uint16_t* ctargets,
                   float* grad, float* dw, float* gembed, const int32_t* c2f);
/* adam_update (cpu_ops.h:62-104) over n elements, step t >= 1 */
void or_adam(float* w, const float* g, float* m, float* v, size_t n, int t, float lr, float b1, float b2, float eps,
             float wd);

#ifdef __cplusplus
}
#endif
#endif
