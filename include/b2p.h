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
 * Asynchronous on `stream` (NULL = default stream). */
int b2p_gemm(const void* X, const void* W, void* Y, int M, int N, int K, int ldy, int dtype, int out_f32,
             void* stream);

/* Same contract as b2p_gemm on the CTA-pair engine: 256 x 256 output tiles
 * computed by clusters of two CTAs (tcgen05 cta_group::2), each CTA loading its
 * 128 rows of X and half of the W tile. Requires M >= 256. */
int b2p_gemm_pair(const void* X, const void* W, void* Y, int M, int N, int K, int ldy, int dtype, int out_f32,
                  void* stream);

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
  int dim, hidden, heads, kv_heads, head_dim, seq, nlayers, vocab; /* models/*.h sizes */
  int rank;          /* LoRA rank (4 or 8), adapters on Wq/Wk/Wv/Wo */
  float rope_theta;  /* ROPE_THETA (cpu_ops.h:296) */
  float res_alpha;   /* residual scale (train_mezo.m:1262): 1 for fine-tuning */
  int dtype;         /* B2P_F16 or B2P_BF16 compute type, fp32 accumulation */
  int max_groups;    /* max (variant x sequence) forwards evaluated in one call */
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
 * B2P_ERR_ARG. Scratch is a fixed 281 KiB __device__ array that every GPU
 * loading the library keeps until exit. The first call on a device fills it
 * (synchronous copy); make that call before any stream capture. All calls on a
 * device share the array, so calls that overlap on the GPU race. Asynchronous
 * on `stream` otherwise. Calls no cudaMalloc/cudaFree. */
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
int b2p_model_set_option(b2p_model* m, int option, int value);

#ifdef __cplusplus
}
#endif
#endif /* B2P_H */
