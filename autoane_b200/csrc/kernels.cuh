// kernels.cuh — glue kernels around the projection engine (token-major layout).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "gemm.cuh"

namespace b2p {

// Perturbation context shared by the fused kernels: which variant (θ, θ+εz,
// θ+εz-2εz) each group of `group_rows` token rows evaluates.
struct PerturbCtx {
  const float* theta;
  const uint32_t* masks;
  long long mask_words;
  const VariantInfo* variants;
  const int* group_variant;
  int group_rows;
};

// x[row, :] = embed[token(row), :]  (reference embed_lookup, training/cpu_ops.h:190-197)
// token(row) = tokens[group_seq[row / seq] * seq + row % seq]
int launch_embed(const float* embed, int vocab, int dim, const int32_t* tokens, const int* group_seq, int seq,
                 int rows, float* x, uint32_t* status, cudaStream_t st);

// Per token row: optional RMSNorm with the perturbed weight at theta[w_off]
// (training/cpu_ops.h:7-22) written as 16-bit xn, then U[row, u_col + 16*i + j] =
// A_i(perturbed)[j, :] · v for the n_a LoRA-down matrices at theta[a_off[i]]
// (first half of lora_addmm, training/train_mezo.m:698), v = normalised row in fp32
// (norm) or the 16-bit input row (no norm). U is 16-bit [rows, 64]; columns
// j >= rank of each 16-column group stay zero (they pad the tensor-core K step).
struct NormLoraArgs {
  const void* in;       // fp32 [rows, dim] (norm) or 16-bit [rows, dim]
  void* xn;             // 16-bit [rows, dim] (norm only)
  int rows, dim;
  int norm;             // 1: RMSNorm with weight, 0: LoRA-down of the raw 16-bit input
  long long w_off;      // rms weight offset in theta
  int n_a;              // number of LoRA-down matrices (0..3)
  long long a_off[3];
  int rank;
  void* U;
  int u_col;
  PerturbCtx pc;
  // Prepared operands (launch_lora_prep): when a_prep is set, the variant's perturbed
  // A rows are read from a_prep + variant * a_prep_vstride (16-bit, n_a*rank rows of
  // a_prep_ld elements) and the perturbed rms weight from w_prep + variant * w_prep_vstride.
  const void* a_prep;
  long long a_prep_vstride;
  int a_prep_ld;
  const float* w_prep;
  long long w_prep_vstride;
};
int launch_norm_lora(const NormLoraArgs& a, bool bf16, cudaStream_t st);

// Per-variant perturbed LoRA-down operands of every layer, made once per forward:
//   a_out[l][v][segs*r][ld]: rows 0..3r-1 = A_q, A_k, A_v (dim columns), rows 3r..4r-1 = A_o
//     (q_dim columns), with --lora-ffn rows 4r..6r-1 = A_1, A_3 (dim columns); 16-bit
//   a2_out[l][v][r][hidden]: A_2 (--lora-ffn), 16-bit
//   w_out[l][v][2][dim]: rms_att, rms_ffn (fp32); w_final[v][dim]: rms_final
// each parameter as perturb_value(theta, sign bit of the variant's seed).
struct LoraPrepArgs {
  const float* theta;
  const uint32_t* masks;
  long long mask_words;
  const VariantInfo* variants;
  int n_var, nlayers, dim, q_dim, rank, ld, segs, hidden;
  long long layer_size, oAq, oAk, oAv, oAo, oA1, oA3, oA2, oRa, oRf, oRfinal;
  void* a_out;
  void* a2_out;
  float* w_out;
  float* w_final;
};
int launch_lora_prep(const LoraPrepArgs& a, bool bf16, cudaStream_t st);

// Causal GQA attention over token-major Q|K|V rows (reference cpu_sdpa_forward,
// training/cpu_ops.h:321-360, with gqa_tile_kv, training/io.h:439-446):
// out[row, h*hd + d] for every group of `seq` rows. hd = 64.
struct AttnArgs {
  const void* qkv;
  int ld_qkv, q_off, k_off, v_off;
  void* out;
  int ld_out;
  int seq, heads, kv_heads, ngroups;
  float* lse;  // optional [rows, heads]: each row's log2-domain softmax normaliser (for the backward)
  int* sched = nullptr;  // 2 zeroed ints owned by the caller: enables the tcgen05 kernel (seq 128 / 256)
};
// Causal GQA attention: the tcgen05 kernel (attn_tc.cu) where it applies, else
// the mma.sync kernel (64 x 64 tiles).
int launch_attention(const AttnArgs& a, bool bf16, cudaStream_t st);
bool attention_tc_supported(const AttnArgs& a);
int launch_attention_tc(const AttnArgs& a, bool bf16, cudaStream_t st);

// Causal GQA attention backward operands (cpu_sdpa_backward, training/cpu_ops.h:213-290).
struct AttnBwdArgs {
  const void* qkv;  // [rows][ld] post-RoPE Q|K|V
  int ld, q_off, k_off, v_off;
  const void* o;    // [rows][ld_o] attention output
  const void* dout; // [rows][ld_o] dO
  int ld_o;
  const float* lse; // [rows][heads] forward row normaliser, log2 domain
  float* dvec;      // [rows][heads] D = sum_d dO O
  void* dqkv;       // [rows][ld_d] dQ | dK | dV, same column offsets as qkv
  int ld_d;
  const float* rope_cos;
  const float* rope_sin;  // [seq][32]
  int seq, heads, kv_heads, ngroups;
  float scale_log2, scale;
  int* sched = nullptr;   // 2 zeroed ints: enables the tcgen05 kernels (seq 128 / 256)
};
// D = rowsum(dO·O) into dvec, then dK|dV and dQ: the tcgen05 kernels where they apply
// and use_tc is set, else the mma.sync kernels (64 x 64 tiles). dQ and dK leave with the
// inverse RoPE applied (rope_backward_inplace, training/cpu_ops.h:364), dK and dV summed
// over each KV head's query heads (gqa_reduce_kv, training/io.h:448-459).
int launch_attention_backward(const AttnBwdArgs& a, bool bf16, bool use_tc, cudaStream_t st);
// dK|dV and dQ on the tcgen05 tensor cores (attn_bwd_tc.cu), D already in dvec.
bool attention_backward_tc_supported(const AttnBwdArgs& a);
int launch_attention_backward_tc(const AttnBwdArgs& a, bool bf16, cudaStream_t st);

// Row losses from the lm-head partials: loss_row = -(logit_tgt - M) + log(Σ s_i e^{m_i - M})
// (training/cpu_ops.h:108-133); group_loss[g] = mean over the group's rows.
int launch_ce_reduce(const float2* part, int ntiles, const float* tgt_logit, int rows, int seq, float* row_loss,
                     float* group_loss, cudaStream_t st, float* row_lse = nullptr);
// var_loss[v] = mean of group_loss over the n_seq groups of variant v (groups v*n_seq + q).
int launch_variant_loss(const float* group_loss, int n_var, int n_seq, float* var_loss, cudaStream_t st);

// In-place Rademacher steps on the trainable parameters (perturb_buffer,
// training/train_mezo.m:122-136), applied in order: θ_i ← fl(θ_i + (z_i ? c : -c)).
// The scale c of an op is either fixed, or computed on the device from a loss
// pair as the MeZO update -lr·(L+ - L-)/(2ε) / div (train_mezo.m:2997-3012).
struct PerturbOp {
  int slot;          // mask row
  int from_loss;     // 0: fixed `scale`; 1: from losses[2*loss_idx], losses[2*loss_idx+1]
  int loss_idx;
  float scale;
  float eps, lr, div;
};
constexpr int kMaxPerturbOps = 64;
struct PerturbOps {
  int n;
  PerturbOp op[kMaxPerturbOps];
};
int launch_perturb(float* theta, long long n, const uint32_t* masks, long long mask_words, const PerturbOps& ops,
                   const float* losses, cudaStream_t st);

// gate[r, c] = silu(h1) * h3 from the interleaved W1|W3 output h13 [rows, 2H]
// (h1 of column c at 256*(c/128) + c%128, h3 128 columns later; train_mezo.m:1664-1667).
int launch_swiglu_gate(const void* h13, int rows, int H, void* gate, bool bf16, cudaStream_t st);

// Layout conversion for the Kern-style boundary: host channel-first fp32 [C, S]
// <-> device token-major 16-bit / fp32 [S, C].
int launch_cf_to_tm16(const float* src, int C, int S, void* dst, int ld_dst, bool bf16, cudaStream_t st);
int launch_cf_to_tm32(const float* src, int C, int S, float* dst, int ld_dst, cudaStream_t st);
int launch_tm_to_cf32(const void* src, int ld_src, bool src_f32, bool bf16, int C, int S, float* dst,
                      cudaStream_t st);
int launch_f32_to_16(const float* src, void* dst, long long n, bool bf16, cudaStream_t st);

}  // namespace b2p
