/* b2p.h — C ABI of the B200 projection library (libb2p.so).
 *
 * This library takes the place of AutoANE's Neural-Engine device boundary:
 *   - the in-loop Kern API of training/io.h (compile_conv1x1_kern :165,
 *     compile_qkv_fused_conv1x1_kern :182, compile_ffn_fused_conv1x1_kern :209,
 *     io_write_conv_acts :102, io_write_ffn_fused_conv_input :232,
 *     io_read_dyn :109, ane_eval :242, free_kern :152), and
 *   - the ctypes-facing bridge of bridge/ane_bridge.h (ane_bridge_init :20,
 *     ane_bridge_compile :33, ane_bridge_eval :52, ane_bridge_write_input :55,
 *     ane_bridge_read_output :59, ane_bridge_free :63,
 *     ane_bridge_get_compile_count :66, ane_bridge_reset_compile_count :69).
 *
 * Conventions (same as the reference boundary): host tensors are fp32,
 * channel-first [C, S] row-major; the device side computes in fp16 or bf16
 * with fp32 accumulation. Unlike ane_eval (io.h:242, which ignores errors),
 * every call returns a status: 0 on success, a negative B2P_ERR_* otherwise,
 * with a message available from b2p_last_error(). Nothing here falls back to
 * the CPU: without a B200 the calls fail with B2P_ERR_CUDA / B2P_ERR_UNSUPPORTED.
 *
 * Threading: calls on one handle must not overlap; different handles may be
 * used from different threads. All device work is issued on the stream given
 * to the call (or the handle's stream), so host code can overlap its own work.
 */
#ifndef B2P_H
#define B2P_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define B2P_OK 0
#define B2P_ERR_ARG (-1)
#define B2P_ERR_CUDA (-2)
#define B2P_ERR_DEVICE (-3)
#define B2P_ERR_STATE (-4)
#define B2P_ERR_UNSUPPORTED (-5)
#define B2P_ERR_IO (-6)

/* ---- compute dtypes ---- */
#define B2P_F16 0
#define B2P_BF16 1

/* Initialise the library on `device` (makes it current for this thread).
 * Replaces ane_bridge_init (bridge/ane_bridge.h:20) / ane_init (training/config.h:131).
 * Returns 0, or a negative status (e.g. the device is not an sm_100 part). */
int b2p_init(int device);

/* Message for the last failed call on this thread (never NULL). */
const char* b2p_last_error(void);

/* Library version string. */
const char* b2p_version(void);

/* Read and clear the device status word written by bounded in-kernel waits.
 * Synchronises `stream`. Returns 0 or B2P_ERR_DEVICE. */
int b2p_device_status(void* stream);

/* Raw projection GEMM on device pointers (the tile engine itself):
 *   Y[M, N] = X[M, K] · W[N, K]^T
 * X and W are row-major 16-bit (dtype B2P_F16 / B2P_BF16), K a multiple of 8,
 * 16-byte aligned. Y is fp32 (out_f32 = 1) or the input dtype (out_f32 = 0),
 * row pitch ldy elements. This is the device-resident form of the reference's
 * cblas_sgemm projection call sites (training/train_mezo.m:1533-1538) in the
 * transposed, token-major layout: X holds tokens as rows, W output channels.
 * Up to 1024 rows, when the 128 x 64 output tiles fit one wave, one CTA per
 * tile spreads its K loop over four MMA issuers (b2p_gemm_mi), or, for a long
 * K (>= 2048) that a cluster of CTAs can split, the K loop of each tile is
 * split over the cluster; partial sums are added in a fixed order either way,
 * so results repeat bit for bit. Otherwise the CTA-pair engine (M >= 256) or
 * the persistent single-CTA engine runs it.
 * Asynchronous on `stream` (NULL = default stream). */
int b2p_gemm(const void* X, const void* W, void* Y, int M, int N, int K, int ldy, int dtype, int out_f32,
             void* stream);

/* Same contract as b2p_gemm on the CTA-pair engine: 256 x 256 output tiles
 * computed by clusters of two CTAs (tcgen05 cta_group::2), each CTA loading its
 * 128 rows of X and half of the W tile. Requires M >= 256. */
int b2p_gemm_pair(const void* X, const void* W, void* Y, int M, int N, int K, int ldy, int dtype, int out_f32,
                  void* stream);
/* b2p_gemm_pair with operands read in either layout, as the backward passes
 * hold them: X is [M][K] rows (x_mn 0) or [K][M] rows (x_mn 1), pitch ldx;
 * W is [N][K] rows (w_mn 0) or [K][N] rows (w_mn 1), pitch ldw. Y[M][N] =
 * X·W^T with X, W read where they lie (MN-major tcgen05 operands, no transposed
 * copies). Layouts: (0, 1) with fp32 or 16-bit output, (1, 1) with fp32
 * output, (0, 0) as b2p_gemm_pair. M >= 256; pitches multiples of 8 elements. */
int b2p_gemm_pair_mn(const void* X, int ldx, int x_mn, const void* W, int ldw, int w_mn, void* Y, int M, int N, int K,
                     int ldy, int dtype, int out_f32, void* stream);
/* Same contract as b2p_gemm on 128 x 64 output tiles, one CTA per tile, each
 * tile's K-blocks spread over four tcgen05 MMA issuer warps with an accumulator
 * each, added in a fixed order (results repeat bit for bit). For GEMMs of few
 * token rows, where a single issuer's K loop is the critical path. */
int b2p_gemm_mi(const void* X, const void* W, void* Y, int M, int N, int K, int ldy, int dtype, int out_f32,
                void* stream);

/* Causal GQA attention on device buffers (cpu_sdpa_forward,
 * training/cpu_ops.h:321-360, with K/V tiled over the query heads by
 * gqa_tile_kv, training/io.h:439-446), for n_seq independent sequences of
 * `seq` tokens stored as token-major 16-bit rows:
 *   qkv [n_seq*seq][ld_qkv]: post-RoPE Q in columns [0, 64*heads), K in the
 *       next 64*kv_heads columns, V after it (head_dim 64; query head h reads
 *       KV head h / (heads / kv_heads));
 *   out [n_seq*seq][ld_out]: softmax(Q·Kᵀ/8 + causal mask)·V per head, 64*heads columns;
 *   lse (may be NULL) fp32 [n_seq*seq][heads]: each row's softmax normaliser
 *       in the log2 domain, max·log2(e)/8 + log2(sum), the input b2p_attention_backward needs.
 * seq a multiple of 64 (the tcgen05 kernel takes 128 and 256, the mma.sync
 * kernel other lengths); row pitches multiples of 8 elements, 16-byte aligned
 * pointers. Asynchronous on `stream`; allocates its 8-byte work counter with
 * cudaMallocAsync on that stream. */
int b2p_attention(const void* qkv, int ld_qkv, void* out, int ld_out, float* lse, int n_seq, int seq, int heads,
                  int kv_heads, int dtype, void* stream);

/* Attention backward as bp_lora_backward runs it (training/backprop_lora.h:241-252):
 * cpu_sdpa_backward (cpu_ops.h:213-290) on post-RoPE Q, K, V and the output
 * gradient dout [n_seq*seq][ld_o], then dK and dV summed over each KV head's
 * query heads (gqa_reduce_kv, io.h:448-459) and the inverse RoPE of theta
 * rope_theta applied to dQ and dK (rope_backward_inplace, cpu_ops.h:364).
 * `out` and `lse` are b2p_attention's outputs for the same qkv. Writes dQ | dK | dV
 * into dqkv [n_seq*seq][ld_d] at qkv's column offsets. Same shape rules as
 * b2p_attention. Asynchronous on `stream` (its scratch comes from cudaMallocAsync). */
int b2p_attention_backward(const void* qkv, int ld_qkv, const void* out, const void* dout, int ld_o,
                           const float* lse, void* dqkv, int ld_d, int n_seq, int seq, int heads, int kv_heads,
                           float rope_theta, int dtype, void* stream);

/* ======================================================================
 * Device-resident model: the MeZO-LoRA-split hot path on the GPU.
 *
 * Replaces the per-layer compile/stage/eval/read round trips of
 * DO_FORWARD_PASS (training/train_mezo.m:1528-1699; conv-fused kernels
 * compiled at train_mezo.m:1296-1327) and the host-side in-place perturbation
 * of perturb_lora_weights (train_mezo.m:560-588). Base projection weights are
 * uploaded once and stay frozen (16-bit); the trainable LoRA A/B + RMS weights
 * live on the device as an fp32 master copy in the reference's perturbation
 * order; the ±εz perturbation is applied inside the kernels' operand loads.
 * ====================================================================== */
typedef struct b2p_model b2p_model;

typedef struct {
  int dim, hidden, heads, kv_heads, head_dim, seq, nlayers, vocab; /* sizes of the model header (training/models) */
  int rank;          /* LoRA rank (4 or 8), adapters on Wq/Wk/Wv/Wo */
  float rope_theta;  /* ROPE_THETA (cpu_ops.h:296) */
  float res_alpha;   /* residual scale (train_mezo.m:1262): 1 for fine-tuning */
  int dtype;         /* B2P_F16 or B2P_BF16 compute type, fp32 accumulation */
  int max_groups;    /* max (variant x sequence) forwards evaluated in one call */
  int lora_ffn;      /* --lora-ffn (train_mezo.m:866, 898): adapters on W1, W2, W3 too; the
                        trainable set then holds A1, B1, A2, B2, A3, B3 after Bo in every layer
                        (perturb_lora_weights order, train_mezo.m:575-582). MeZO only; needs
                        seq % 256 == 0 and hidden in {1152, 1408, 2560}. */
} b2p_model_config;

/* One evaluation point of the trainable parameters θ:
 *   mode 0: θ;  mode 1: θ + s1·z;  mode 2: (θ + s1·z) + s2·z   (fp32 adds, z = ±1)
 * with z the Rademacher signs of `seed` (xo_seed/perturb_buffer, train_mezo.m:110-136).
 * The reference's +ε pass is {seed, 1, ε, 0}; its -ε pass is {seed, 2, ε, -2ε}. */
typedef struct {
  uint64_t seed;
  int mode;
  float s1, s2;
} b2p_variant;

/* Allocate a model on the current device (after b2p_init). NULL on error. */
b2p_model* b2p_model_create(const b2p_model_config* cfg);
void b2p_model_free(b2p_model* m);
/* Number of trainable parameters (LoRA A/B + RMS weights; 1,700,800 for SmolLM2-360M r8). */
long long b2p_model_trainable_count(const b2p_model* m);
/* The model's CUDA stream (cudaStream_t), for callers that order their own work after it. */
void* b2p_model_stream(b2p_model* m);
/* Frozen base weights of one layer, fp32 row-major [out, in] as in LayerWeights
 * (training/config.h:48-52); converted to the compute dtype on upload.
 * Replaces compile_qkv_fused_conv1x1_kern / compile_ffn_fused_conv1x1_kern /
 * compile_conv1x1_kern weight baking (training/io.h:165-230). */
int b2p_model_set_layer(b2p_model* m, int layer, const float* Wq, const float* Wk, const float* Wv, const float* Wo,
                        const float* W1, const float* W2, const float* W3);
/* Full embedding [vocab, dim] (used for the token lookup, cpu_ops.h:190) and the
 * compact-vocabulary map; the tied lm-head uses the compact rows
 * (vocab_compact_embed, cpu_ops.h:171). */
int b2p_model_set_embedding(b2p_model* m, const float* embed, const int32_t* compact_to_full, int cv);
/* Trainable parameters in perturbation order (per layer Aq,Bq,Ak,Bk,Av,Bv,Ao,Bo,
 * rms_att,rms_ffn; then rms_final). Host or device pointer. */
int b2p_model_set_trainable(b2p_model* m, const float* theta, long long n);
int b2p_model_get_trainable(b2p_model* m, float* theta, long long n);

/* Forward + mean cross-entropy of n_seq sequences (tokens [n_seq][seq] uint16,
 * compact targets [n_seq][seq]) under each of n_var variants, in one batched
 * pass. losses[v] = mean over the sequences of the per-token mean CE
 * (cross_entropy_loss, cpu_ops.h:108-133). Host buffers; synchronous. */
int b2p_model_eval(b2p_model* m, const uint16_t* tokens, const uint16_t* ctargets, int n_seq,
                   const b2p_variant* vars, int n_var, float* losses);

/* Per-group losses of the model's last forward (any eval, MeZO or backprop-LoRA
 * call): out[g] = per-token mean CE of group g = v*n_seq + q, i.e. sequence q
 * under variant v (the single-sequence loss the reference's DO_FORWARD_PASS
 * returns, train_mezo.m:1695-1698). n <= the last forward's group count; host
 * or device `out`; synchronises the model stream. */
int b2p_model_group_losses(b2p_model* m, float* out, int n);

/* One MeZO-LoRA-split step exactly as train_mezo.m:2938-3012: evaluate θ+εz and
 * θ-εz (batched), then θ ← ((θ+εz)-2εz)+εz and θ ← θ - lr·g·z with
 * g = (L+ - L-)/(2ε) computed on the device. Outputs may be NULL. */
int b2p_mezo_step(b2p_model* m, const uint16_t* tokens, const uint16_t* ctargets, uint64_t seed, float eps,
                  float lr, float* loss_plus, float* loss_minus, float* proj_grad);

/* Data-parallel MeZO, evaluation half: for each of n_seeds seeds, L+ and L- over
 * the n_seq sequences. loss_pairs[2s] = L+, [2s+1] = L- (host or device pointer). */
int b2p_mezo_eval(b2p_model* m, const uint16_t* tokens, const uint16_t* ctargets, int n_seq, const uint64_t* seeds,
                  int n_seeds, float eps, float* loss_pairs);
/* Same as b2p_mezo_eval with the inputs already resident on the device: d_tokens
 * and d_targets are int32 [n_seq][seq] device arrays (out-of-range ids are
 * reported by b2p_model_sync as B2P_ERR_DEVICE). Fully asynchronous when
 * loss_pairs is device memory, so a collective can follow on the model stream. */
int b2p_mezo_eval_device(b2p_model* m, const int32_t* d_tokens, const int32_t* d_targets, int n_seq,
                         const uint64_t* seeds, int n_seeds, float eps, float* loss_pairs);
/* Data-parallel MeZO, update half: θ ← θ + c_s·z_s applied in seed order with
 * c_s = (-lr·(L+_s - L-_s)/(2ε)) / n_seeds (the K-direction averaged update of
 * train_mezo.m:2751-2768). Every replica given the same arguments ends bit-identical. */
int b2p_mezo_update(b2p_model* m, const uint64_t* seeds, const float* loss_pairs, int n_seeds, float eps, float lr);
/* θ ← fl(θ + (z ? c : -c)) for each (seeds[i], scales[i]) in order (perturb_lora_weights). */
int b2p_model_perturb(b2p_model* m, const uint64_t* seeds, const float* scales, int n);
/* Sign masks of the perturbation stream: out_words[i][w], bit b of word w = sign of
 * parameter 32w+b for seeds[i] (1 = +). ceil(P/32) words per seed. */
int b2p_sign_masks(b2p_model* m, const uint64_t* seeds, int n, uint32_t* out_words);

/* Allocation-free form of b2p_sign_masks, for callers that cannot allocate device
 * memory (all device memory owned by another allocator, or a fixed budget).
 * No counterpart in the reference (it draws signs on the host).
 * Writes the sign masks of the perturbation stream over an arbitrary buffer
 * layout into out_words, caller-owned device memory [nseeds][ceil(P/32)]
 * (P = sum of buffer_sizes). Bit b of word w is the sign of parameter 32w+b
 * (1 = +), drawn as perturb_buffer draws it (training/train_mezo.m:122-136).
 * Host inputs: buffer_sizes[nbufs], seeds[nseeds]. Limits: nbufs <= 1024,
 * nseeds <= 64, at most 524,288 draws per seed; larger inputs are rejected with
 * B2P_ERR_ARG. out_words must be on the current device (another device's
 * buffer is refused with B2P_ERR_ARG). Scratch is a fixed 281 KiB __device__
 * array that every GPU loading the library keeps until exit. The first call on
 * a device loads the library's device code there if CUDA has not yet done so
 * (lazy module loading brings the array in at that moment) and fills the array
 * with a copy it waits for; make that first call during set-up, before any
 * stream capture. All calls on a device share the array, so calls that overlap
 * on the GPU race. Asynchronous on `stream` otherwise. Calls no
 * cudaMalloc/cudaFree. */
int b2p_sign_masks_noalloc(const int64_t* buffer_sizes, int nbufs, const uint64_t* seeds, int nseeds,
                           uint32_t* out_words, void* stream);

/* Wait for the model stream and report any device-side status (bounded-wait
 * expiry, out-of-range token). b2p_mezo_update / b2p_model_perturb and the
 * device-pointer forms of the eval calls are asynchronous; this is their fence. */
int b2p_model_sync(b2p_model* m);
/* Time every projection-GEMM launch of subsequent forwards with CUDA events on the
 * model stream (enable = 1), or stop (0). Enabling clears the record. */
int b2p_model_profile(b2p_model* m, int enable);
/* Sum of the recorded GEMM launch durations (ms), their algorithmic FLOPs
 * (2·M·N·K each) and the launch count since profiling was enabled. */
int b2p_model_profile_read(b2p_model* m, double* gemm_ms, double* gemm_flops, long long* gemm_launches);
/* Number of kernels this library has launched in this process. */
long long b2p_launch_count(void);

/* Model options. B2P_OPT_PAIR_GEMM (default 1): run the projection GEMMs on the
 * CTA-pair engine (256 x 256 tiles over two SMs, tcgen05 cta_group::2) where it
 * applies; 0 forces the single-CTA engine (128-row tiles). Same results either
 * way up to fp32 summation order. */
#define B2P_OPT_PAIR_GEMM 1
/* B2P_OPT_GRAD_SCALE_LOG2 (default 0): the backprop-LoRA backward stores
 * dlogits as 2^value * (softmax - onehot) in the 16-bit compute type; raise it
 * if gradients underflow, lower it if they overflow (a non-finite gradient
 * makes the optimizer step a no-op and the call return B2P_ERR_DEVICE). */
#define B2P_OPT_GRAD_SCALE_LOG2 2
/* B2P_OPT_GRAPHS (default 1): the backprop-LoRA gradient pass is recorded once
 * into a CUDA graph per (token buffer, batch size, buffers) and replayed; 0 issues
 * every kernel from the host instead. */
#define B2P_OPT_GRAPHS 3
/* B2P_OPT_TC_ATTENTION (default 1): causal attention on the tcgen05 kernel
 * (sequences of 128 or 256 tokens); 0 uses the mma.sync kernel (64 x 64 tiles).
 * Same results up to fp32 summation order. */
#define B2P_OPT_TC_ATTENTION 4
/* B2P_OPT_TC_ATTENTION_BWD (default 1): the backprop-LoRA attention backward on
 * the tcgen05 kernels (dK|dV then dQ, sequences of 128 or 256 tokens, 64-wide
 * heads); 0 uses the mma.sync kernels. Same results up to fp32 summation order. */
#define B2P_OPT_TC_ATTENTION_BWD 5
/* B2P_OPT_PDL (default 1): the hot kernels (projection GEMMs, attention, RMSNorm /
 * LoRA-down, backward elementwise kernels) launch with programmatic dependent
 * launch, so each one's launch and prologue overlap the previous kernel's tail;
 * 0 launches them with plain stream order. Process-wide (all models and devices);
 * results are identical either way. */
#define B2P_OPT_PDL 6
int b2p_model_set_option(b2p_model* m, int option, int value);

/* ======================================================================
 * Backprop-LoRA training (the reference's P16 mode, train_mezo.m:1961-2136):
 * forward with activation saves, backward through the whole network
 * (bp_lora_backward, training/backprop_lora.h:147-288) with gradients for the
 * LoRA A/B and RMSNorm weights only, then Adam (cpu_ops.h:62-104).
 *
 * The adapters are applied split on frozen base weights, as the conv-fused
 * P16 forward does; the backward propagates through W + B·A. The loss of
 * n_seq sequences is the mean of their per-token mean cross-entropies; the
 * gradient is d(loss)/d(theta) in the layout of b2p_model_set_trainable.
 * ====================================================================== */

/* Forward + backward of n_seq sequences (host tokens / compact targets,
 * [n_seq][seq] uint16). `loss` (1 float) and `grad` (trainable-count floats,
 * host or device) may be NULL. Synchronous. */
int b2p_p16_grad(b2p_model* m, const uint16_t* tokens, const uint16_t* ctargets, int n_seq, float* loss,
                 float* grad);

/* Same on device int32 tokens/targets, asynchronous on the model stream; the
 * loss goes to the device float d_loss (may be NULL). */
int b2p_p16_grad_device(b2p_model* m, const int32_t* d_tokens, const int32_t* d_targets, int n_seq, float* d_loss);

/* Device pointer of the gradient buffer the last b2p_p16_grad* call wrote
 * (fp32, trainable-count elements), NULL before the first call. Data-parallel
 * callers all-reduce it in place (then divide by the rank count) before
 * b2p_adam_step. */
void* b2p_model_grad(b2p_model* m);

/* One Adam step on the trainable parameters with the gradient buffer
 * (adam_update, cpu_ops.h:62-104; per-element operation order of the
 * reference; the step counter t starts at 1). Asynchronous on the model
 * stream; a non-finite gradient skips the step and sets the device status. */
int b2p_adam_step(b2p_model* m, float lr, float b1, float b2, float eps, float wd);

/* Read (set = 0) or write (set = 1) the Adam step count and moment vectors
 * (trainable-count floats each, host or device; NULL skips a vector). */
int b2p_adam_state(b2p_model* m, int set, int* t, float* mom, float* vel);

/* One full step as train_mezo.m:1982-2117: b2p_p16_grad, then Adam with
 * b1 0.9, b2 0.95, eps 1e-8, no weight decay at learning rate lr. */
int b2p_p16_step(b2p_model* m, const uint16_t* tokens, const uint16_t* ctargets, int n_seq, float lr, float* loss);

/* ======================================================================
 * Full backprop (training/train.m:686-1520): every projection weight, the RMS
 * weights and the tied embedding are trained. The first call switches the
 * model to full mode: fp32 master copies of the projection weights are made
 * from the current 16-bit weights and kept on the device. The LoRA adapters
 * are left alone (keep their B at zero so they do not change the forward).
 * ====================================================================== */

/* Forward + backward of n_seq sequences: dX through every layer and dW of
 * Wq/Wk/Wv/Wo/W1/W2/W3, the RMS weights and the embedding (the classifier rows
 * scattered into it, vocab_scatter_grads, cpu_ops.h:176). Synchronous. */
int b2p_full_grad(b2p_model* m, const uint16_t* tokens, const uint16_t* ctargets, int n_seq, float* loss);

/* Global-norm clipping to `clip` (0: off) and AdamW (b1 0.9, b2 0.95, eps 1e-8;
 * weight decay wd on projection weights and embedding, none on RMS weights),
 * train.m:1309-1517; then the 16-bit weights the forward uses are refreshed.
 * grad_norm (may be NULL) receives the pre-clip norm. */
int b2p_full_update(b2p_model* m, float lr, float wd, float clip, float* grad_norm);

/* b2p_full_grad followed by b2p_full_update. */
int b2p_full_step(b2p_model* m, const uint16_t* tokens, const uint16_t* ctargets, int n_seq, float lr, float wd,
                  float clip, float* loss, float* grad_norm);

/* Number of fp32 projection-weight masters (switches the model to full mode). */
long long b2p_full_weight_count(b2p_model* m);

/* Copy a full-mode quantity to `out` (host or device, n floats):
 *   B2P_FULL_WEIGHTS / B2P_FULL_WEIGHT_GRADS: b2p_full_weight_count floats, laid out as
 *     [every layer's stacked Wq;Wk;Wv] [every Wo] [every W1/W3, interleaved in 128-row
 *     blocks] [every W2], each matrix row-major [out, in];
 *   B2P_FULL_EMBED / B2P_FULL_EMBED_GRAD: [vocab, dim];
 *   B2P_FULL_TRAINABLE_GRAD: trainable-count floats, RMS entries meaningful. */
#define B2P_FULL_WEIGHTS 0
#define B2P_FULL_WEIGHT_GRADS 1
#define B2P_FULL_EMBED 2
#define B2P_FULL_EMBED_GRAD 3
#define B2P_FULL_TRAINABLE_GRAD 4
int b2p_full_read(b2p_model* m, int what, float* out, long long n);

/* ======================================================================
 * Checkpoints: the reference's BLZT v4 file (CkptHdr, training/config.h:99-108;
 * writers mezo_save_checkpoint, train_mezo.m:706-744, and save_checkpoint,
 * train.m:176-208) and the LORA adapter sidecar (lora_save_checkpoint,
 * train_mezo.m:791-815). Little-endian fp32 in the reference's order, so the
 * reference's readers (generate.py, tools/export_to_gguf.py) take these files.
 * ====================================================================== */
typedef struct {
  int magic, version, step, total_steps;
  int n_layers, vocab_size, dim, hidden_dim, n_heads, seq_len;
  float lr, loss;
  double cum_compile, cum_train, cum_wall;
  int cum_steps, cum_batches, adam_t;
  int kv_heads, head_dim, q_dim;
} b2p_ckpt_header; /* 96 bytes */
#define B2P_CKPT_MAGIC 0x424C5A54 /* "BLZT" */
#define B2P_CKPT_VERSION 4
#define B2P_LORA_MAGIC 0x4C4F5241 /* "LORA" */

/* Read a BLZT file's header and check magic, version and that step and adam_t
 * lie in [0, 1e7] (train.m:217-229). Host only. */
int b2p_ckpt_read_header(const char* path, b2p_ckpt_header* hdr);

/* Write the model as BLZT v4. The structural fields come from the model; step,
 * total_steps, lr, loss, cum_* come from `hdr` (may be NULL: zeros).
 *   - full-backprop models write the fp32 masters, the AdamW moments and t
 *     (save_checkpoint, train.m:176-208);
 *   - other models write their frozen projections (the 16-bit values the forward
 *     uses, widened to fp32) with zero Adam slots and adam_t 0
 *     (mezo_save_checkpoint, train_mezo.m:706-744).
 * RMS vectors come from the trainable set, the embedding from the model.
 * With `lora_path` non-NULL the adapters also go to that sidecar (its adam_t is
 * the backprop-LoRA Adam step count) and the BLZT Wq/Wk/Wv/Wo are the merged
 * W + B·A (lora_merge_weight, config.h:278-283), as the backprop-LoRA run leaves
 * them in its checkpoint (train_mezo.m:2107-2110, 3180-3191). */
int b2p_ckpt_save(b2p_model* m, const char* path, const char* lora_path, const b2p_ckpt_header* hdr);

/* Load a BLZT v4 file written for this model's shapes (every structural header
 * field must match; load_checkpoint, train.m:211-258, mezo_load_checkpoint,
 * train_mezo.m:746-789): frozen projections, RMS vectors (into the trainable
 * set), rms_final and the embedding (compact rows rebuilt from
 * `compact_to_full`/`cv`, or from the model's current map when NULL).
 * Full-backprop models, or any model when `full` is 1, also take the fp32
 * masters, the AdamW moments and t. With `lora_path` non-NULL the sidecar's
 * adapters go into the trainable set, the backprop-LoRA Adam state restarts at
 * the sidecar's step count with zero moments, and the projections are
 * un-merged (W - B·A in fp32, train_mezo.m:1134-1151) before the upload. A
 * missing sidecar is an error (the reference falls back to fresh adapters;
 * here the caller chooses by passing NULL). hdr (may be NULL) receives the
 * file's header. Reads are length-checked; a short file is B2P_ERR_IO. */
int b2p_ckpt_load(b2p_model* m, const char* path, const char* lora_path, const int32_t* compact_to_full, int cv,
                  int full, b2p_ckpt_header* hdr);

/* ======================================================================
 * Kern-level boundary: one compiled operator with baked weights and
 * channel-first fp32 host I/O, the verbs of training/io.h and
 * bridge/ane_bridge.h without MIL text.
 *
 * Op kinds (weights[] in the order listed, each fp32 row-major [out, in]):
 *   B2P_OP_CONV1X1    {W[oc,ic]}          in0 x[ic,S]            out0 y[oc,S] = W·x
 *                     (compile_conv1x1_kern, training/io.h:165; gen_conv1x1_mil,
 *                     training/mil_dynamic.h:17)
 *   B2P_OP_QKV_FUSED  {Wq,Wk,Wv}          in0 xn[ic,S]           out0 [q+2kv,S] = concat(Wq·xn, Wk·xn, Wv·xn)
 *                     (compile_qkv_fused_conv1x1_kern, io.h:182; mil_dynamic.h:43)
 *   B2P_OP_FFN_FUSED  {W1,W3,W2}          in0 xn[ic,S], in1 x[ic,S]
 *                                         out0 x + alpha·W2·(silu(W1·xn) ⊙ W3·xn)  [ic,S]
 *                     (compile_ffn_fused_conv1x1_kern, io.h:209; mil_dynamic.h:82; the
 *                     reference's single [ic, 2S] input surface is in0|in1, see
 *                     io_write_ffn_fused_conv_input, io.h:232)
 *   B2P_OP_DYN_MATMUL (none)              in0 act[ic,S], in1 W[ic,oc]
 *                                         out0 y[oc,S], y[o,s] = sum_d act[d,s]·W[d,o]
 *                     (gen_dyn_matmul_mil, mil_dynamic.h:157; the weights travel with the
 *                     input as in io_write_dyn, io.h:79)
 *   B2P_OP_LM_HEAD_CE {E[oc,ic]}          in0 xn[ic,S], in1 int32 targets[S] in [0, oc)
 *                                         out0 loss[1] = mean_s CE(E·xn[:,s], target_s)
 *                     (classifier + cross_entropy_loss, training/train_mezo.m:1695-1698,
 *                     training/cpu_ops.h:108-133)
 *   B2P_OP_DX         {W_0..W_{n-1}}      in_i dy_i[part_oc[i],S]
 *                                         out0 dx[ic,S] = sum_i W_i^T·dy_i
 *                     (the backward data GEMMs: ffnBwdW2t / ffnBwdW13t / wotBwd /
 *                     qBwd / kvBwd, training/mil_dynamic.h:414-500, and
 *                     bp_lora_backward's dX, training/backprop_lora.h:147-288)
 *
 * Shape rules: ic and every output width are multiples of 8 (16-byte rows on
 * the device); S >= 1. Device compute is fp16/bf16 with fp32 accumulation; the
 * host sees fp32 on both sides.
 * ====================================================================== */
#define B2P_OP_CONV1X1 0
#define B2P_OP_QKV_FUSED 1
#define B2P_OP_FFN_FUSED 2
#define B2P_OP_DYN_MATMUL 3
#define B2P_OP_LM_HEAD_CE 4
#define B2P_OP_DX 5

typedef struct b2p_op_desc {
  int kind;          /* B2P_OP_* */
  int ic;            /* input channels (dim for the fused ops) */
  int oc;            /* output channels: conv1x1 / dyn_matmul; vocabulary for lm_head_ce */
  int seq;           /* spatial width S (tokens) */
  int q_dim, kv_dim; /* qkv_fused */
  int hidden;        /* ffn_fused */
  float res_alpha;   /* ffn_fused residual scale (the conv program uses 1) */
  int dtype;         /* B2P_F16 or B2P_BF16 */
  int n_parts;       /* dx: number of (W_i, dy_i) pairs, 1..3 */
  int part_oc[3];    /* dx: output channels of W_i */
} b2p_op_desc;

typedef struct b2p_kernel b2p_kernel;

/* Compile an operator: validates the descriptor, uploads the weights as 16-bit
 * device tensors (the copy is baked: later changes to `weights` have no
 * effect, as with the reference's BLOBFILE constants) and allocates the I/O
 * buffers. Returns NULL on failure with the reason in b2p_last_error().
 * Replaces compile_kern_mil_w (io.h:116) / ane_bridge_compile (ane_bridge.h:33). */
b2p_kernel* b2p_compile(const b2p_op_desc* desc, const float* const* weights);

/* Byte size of input / output `idx` (0 when idx is out of range). */
size_t b2p_input_bytes(const b2p_kernel* k, int idx);
size_t b2p_output_bytes(const b2p_kernel* k, int idx);

/* Copy host input `idx` (fp32 [C, S], or int32 targets for lm_head_ce in1) to
 * the device. `bytes` must equal b2p_input_bytes(k, idx).
 * Replaces io_write_conv_acts (io.h:102) / ane_bridge_write_input (ane_bridge.h:55). */
int b2p_write_input(b2p_kernel* k, int idx, const void* data, size_t bytes);

/* Write channels [ch_off, ch_off + channels) of fp32 input `idx`
 * (io_write_fp16_at, io.h:72). */
int b2p_write_input_channels(b2p_kernel* k, int idx, int ch_off, int channels, const float* data);

/* Run the operator; returns when the results are ready (ane_eval, io.h:242, which
 * discards errors; this returns B2P_ERR_DEVICE / B2P_ERR_CUDA instead). */
int b2p_eval(b2p_kernel* k);

/* Enqueue the operator on the handle's stream and return; b2p_read_output
 * (or b2p_device_status on the stream) reports errors. */
int b2p_eval_async(b2p_kernel* k);

/* Copy output `idx` to the host (waits for the handle's stream).
 * Replaces io_read_dyn (io.h:109) / ane_bridge_read_output (ane_bridge.h:59). */
int b2p_read_output(b2p_kernel* k, int idx, float* data, size_t bytes);

/* Read channels [ch_off, ch_off + channels) of output `idx` (io_read_fp16, io.h:58). */
int b2p_read_output_channels(b2p_kernel* k, int idx, int ch_off, int channels, float* data);

/* Release the operator (free_kern, io.h:152 / ane_bridge_free, ane_bridge.h:63). */
void b2p_free(b2p_kernel* k);

/* The CUDA stream the handle issues on (cudaStream_t). */
void* b2p_kernel_stream(const b2p_kernel* k);

/* Device-resident LoRA on conv1x1 (part 0) and qkv_fused (parts 0/1/2 = q/k/v):
 * out_part += B·(A·x) with A fp32 [rank, ic], B fp32 [part_out, rank], rank 4
 * or 8 (the host-side lora_addmm after the conv read, train_mezo.m:1558-1560,
 * 1609, moved into the GEMM). Requires ic in {512, 960, 1024, 2048} and S a
 * multiple of 128. Passing A = B = NULL removes the part's adapter. */
int b2p_set_lora(b2p_kernel* k, int part, const float* A, const float* B, int rank);

/* Evaluate with the adapters perturbed on the fly: theta' = theta + scale·z,
 * z the reference's Rademacher stream of `seed` (perturb_buffer,
 * train_mezo.m:122-136) drawn over the handle's adapters in the order A_0, B_0,
 * A_1, B_1, ... The stored adapters are not modified. scale 0 turns it off. */
int b2p_set_perturb(b2p_kernel* k, uint64_t seed, float scale);

/* Operators compiled by this process (ane_bridge_get_compile_count,
 * ane_bridge.h:66 / g_compile_count, io.h:138), and its reset (ane_bridge.h:69). */
int b2p_compile_count(void);
void b2p_reset_compile_count(void);

#ifdef __cplusplus
}
#endif
#endif /* B2P_H */
