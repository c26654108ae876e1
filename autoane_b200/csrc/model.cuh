// model.cuh — the device-resident model shared by the MeZO path (model.cu)
// and the backprop-LoRA path (p16.cu): frozen 16-bit base weights, fp32
// trainable parameters in the reference's perturbation order, activations.
#pragma once
#include <cstdint>
#include <vector>
#include "../../include/b2p.h"
#include "engine.cuh"
#include "kernels.cuh"
#include "rng.cuh"

namespace b2p {

// Activations the backprop-LoRA forward keeps for the backward (one slab per
// layer, token-major rows), the transposed frozen weights of the backward
// GEMMs, gradients and Adam state. Defined in p16.cu.
struct P16State;
void p16_release(P16State* s);

}  // namespace b2p

struct Stager {
  char* base = nullptr;
  size_t slot_bytes = 0;
  int nslots = 0, next = 0;
  std::vector<cudaEvent_t> ev;
  std::vector<char> armed;
};

struct b2p_model {
  b2p_model_config cfg{};
  int device = 0;
  bool bf16 = false;
  cudaStream_t st = nullptr;
  int q_dim = 0, kv_dim = 0, qkv_dim = 0, ffn2 = 0;
  // trainable layout (offsets inside a layer block, then rms_final)
  long long oAq, oBq, oAk, oBk, oAv, oBv, oAo, oBo, oRa, oRf, layer_size, oRfinal, P;
  bool ffn = false;  // --lora-ffn: FFN adapters after Bo in every layer (-1 offsets otherwise)
  long long oA1 = -1, oB1 = -1, oA2 = -1, oB2 = -1, oA3 = -1, oB3 = -1;
  // frozen weights (16-bit), per-layer contiguous
  void *wqkv = nullptr, *wo = nullptr, *w13 = nullptr, *w2 = nullptr, *cembed = nullptr;
  float* embed = nullptr;
  int cv = 0;
  std::vector<char> layer_set;
  bool embed_set = false;
  // trainable params + sign masks
  float* theta = nullptr;
  uint32_t* masks = nullptr;
  int max_slots = 0;
  long long mask_words = 0;
  b2p::SignBuffer* d_bufs = nullptr;
  int nbufs = 0;
  uint64_t* d_polys = nullptr;
  long long nchunks = 0;
  std::vector<uint64_t> slot_seed;  // seeds whose masks the slots currently hold (in slot order)
  long long total_draws = 0;
  uint64_t* d_seeds = nullptr;
  // activations
  int max_groups = 0, max_rows = 0, n_vt = 0;
  float* x = nullptr;
  void* xn = nullptr;
  void* U = nullptr;             // [max_rows][kUCols] 16-bit LoRA-down results (zero padded)
  void* qkv = nullptr;
  void* attn = nullptr;
  void* hbuf = nullptr;
  float2* ce_part = nullptr;
  float* ce_tgt = nullptr;
  float* row_loss = nullptr;
  float* group_loss = nullptr;
  float* var_loss = nullptr;
  float* pairs = nullptr;        // [2 * kMaxPerturbOps] loss pairs for updates
  int qkv_bn = 160;
  int cur_groups = 0, cur_vars = 0;  // group/variant table sizes of the forward being issued
  bool use_pair = true;               // CTA-pair GEMMs where they apply (b2p_model_set_option)
  int32_t* d_tok = nullptr;      // [max_seq_in][seq] tokens then targets
  int32_t* d_row_tgt = nullptr;  // [max_rows]
  int* d_meta = nullptr;         // group_seq[max_groups] | group_var[max_groups]
  b2p::VariantInfo* d_var = nullptr;
  void* prep_a = nullptr;         // [L][max_groups][prep_segs*r][prep_ld] perturbed A rows per variant (16-bit):
                                  // Aq, Ak, Av, Ao (+ A1, A3 with --lora-ffn)
  int prep_segs = 4;
  void* prep_a2 = nullptr;        // [L][max_groups][r][hidden] perturbed A2 rows per variant (--lora-ffn)
  float* prep_w = nullptr;        // [L][max_groups][2][dim] perturbed rms_att / rms_ffn per variant
  float* prep_wf = nullptr;       // [max_groups][dim] perturbed rms_final per variant
  int prep_ld = 0;
  int32_t* d_c2f = nullptr;       // [cv] compact -> full vocabulary id (device copy)
  std::vector<int32_t> h_c2f;     // host copy of the same map (checkpoint loads rebuild the compact rows)
  float* rope_cos = nullptr;
  float* rope_sin = nullptr;
  Stager stg;
  // optional CUDA-event timing of every projection-GEMM launch
  bool prof = false;
  std::vector<cudaEvent_t> ev_pool;
  size_t ev_used = 0;
  std::vector<double> prof_flops;
  // backprop-LoRA (P16) state, allocated on first use
  b2p::P16State* p16 = nullptr;
  int grad_scale_log2 = 0;  // B2P_OPT_GRAD_SCALE_LOG2
  int weights_version = 0;  // bumped by every frozen-weight upload
  int prof_epoch = 0;       // bumped by every b2p_model_profile call
  bool graphs = true;       // B2P_OPT_GRAPHS
  bool tc_attn = true;      // B2P_OPT_TC_ATTENTION
  bool tc_attn_bwd = true;  // B2P_OPT_TC_ATTENTION_BWD
  int* attn_sched = nullptr;  // [2] unit counter of the tcgen05 attention kernel (self-resetting)
};


namespace b2p {

// Helpers of model.cu used by p16.cu.
size_t model_esz(const b2p_model* m);
int model_ready(const b2p_model* m);
int model_stage_tokens(b2p_model* m, const uint16_t* tokens, const uint16_t* ctargets, int n_seq);
int model_stage_groups(b2p_model* m, int n_seq, const std::vector<VariantInfo>& vars, const int32_t* d_targets);
PerturbCtx model_pctx(const b2p_model* m);
LoraEpi model_lora_epi(const b2p_model* m);
int model_gemm(b2p_model* m, int bn, int kind, const void* X, int ldx, const void* W, int ldw, int M, int N, int K,
               void* out, int ldo, const void* u16, const EpiParams& ep);
// model_gemm with MN-major operands on the CTA-pair engine (opm as launch_gemm_pair_mn); returns
// B2P_ERR_UNSUPPORTED without launching when the pair engine does not take it.
int model_gemm_mn(b2p_model* m, int kind, int opm, const void* X, int ldx, const void* W, int ldw, int M, int N, int K,
                  void* out, int ldo, const EpiParams& ep);

// Where the forward writes the activations the backward reads (all null: the
// plain MeZO forward, which reuses one buffer per activation).
struct ForwardSaves {
  float* x_in = nullptr;     // [L][R][D] input of each layer
  float* x_mid = nullptr;    // [L][R][D] residual after attention
  void* xn = nullptr;        // [L][R][D] normalised attention input (16-bit)
  void* U = nullptr;         // [L][R][64] LoRA-down results
  void* qkv = nullptr;       // [L][R][q+2kv] post-LoRA, post-RoPE Q|K|V
  void* attn = nullptr;      // [L][R][q] attention output
  float* lse = nullptr;      // [L][R][heads] attention row normalisers (log2 domain)
  void* h13 = nullptr;       // [L][R][2H] W1|W3 outputs, interleaved in 128-column blocks
  void* xn2 = nullptr;       // [L][R][D] normalised FFN input (16-bit; kept for the W1/W3 weight gradients)
  float* x_final = nullptr;  // [R][D] input of the final norm
  void* xn_final = nullptr;  // [R][D]
  float* row_lse = nullptr;  // [R] lm-head log-sum-exp per row
};
int model_run_forward(b2p_model* m, int G, const int32_t* tok, const ForwardSaves* sv);

// Device buffers of the backprop state that checkpoints read and write (p16.cu).
// The full-mode fields are null unless the model is (or, with make_full, is made)
// a full-backprop model.
struct TrainView {
  float *adam_m = nullptr, *adam_v = nullptr;  // trainable-set Adam moments
  int* adam_t = nullptr;
  bool full = false;
  float *mw = nullptr, *am_w = nullptr, *av_w = nullptr;  // projection masters + AdamW moments
  float *am_e = nullptr, *av_e = nullptr;                 // embedding AdamW moments
  long long o_qkv = 0, o_o = 0, o_13 = 0, o_2 = 0;
  int* full_t = nullptr;
};
int p16_view(b2p_model* m, bool make_full, TrainView* v);

}  // namespace b2p
