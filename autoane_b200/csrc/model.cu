// model.cu — device-resident SmolLM2/Llama-style model for the MeZO-LoRA-split
// path: frozen 16-bit base weights, fp32 master copy of the trainable LoRA/RMS
// parameters (reference order, train_mezo.m:560-588), device sign masks, and a
// batched forward over groups of (variant, sequence).
//
// One forward evaluates G = n_var * n_seq groups of `seq` token rows at once
// (group g = v * n_seq + q evaluates sequence q under variant v), so the base
// projection weights are read once per layer for all ±ε evaluations.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>
#include "model.cuh"

using namespace b2p;

namespace {


size_t esz(const b2p_model*) { return 2; }

int model_alloc(b2p_model* m) {
  const auto& c = m->cfg;
  const size_t e = esz(m);
  const size_t L = c.nlayers;
  B2P_CHECK_CUDA(cudaMalloc(&m->wqkv, L * m->qkv_dim * c.dim * e));
  B2P_CHECK_CUDA(cudaMalloc(&m->wo, L * c.dim * m->q_dim * e));
  B2P_CHECK_CUDA(cudaMalloc(&m->w13, L * 2 * c.hidden * c.dim * e));
  B2P_CHECK_CUDA(cudaMalloc(&m->w2, L * c.dim * c.hidden * e));
  B2P_CHECK_CUDA(cudaMalloc(&m->embed, (size_t)c.vocab * c.dim * 4));
  B2P_CHECK_CUDA(cudaMalloc(&m->theta, m->P * 4));
  B2P_CHECK_CUDA(cudaMemset(m->theta, 0, m->P * 4));
  B2P_CHECK_CUDA(cudaMalloc(&m->masks, (size_t)m->max_slots * m->mask_words * 4));
  B2P_CHECK_CUDA(cudaMemset(m->masks, 0, (size_t)m->max_slots * m->mask_words * 4));
  B2P_CHECK_CUDA(cudaMalloc(&m->d_seeds, m->max_slots * 8));
  const size_t R = m->max_rows;
  B2P_CHECK_CUDA(cudaMalloc(&m->x, R * c.dim * 4));
  B2P_CHECK_CUDA(cudaMalloc(&m->xn, R * std::max(c.dim, m->q_dim) * e));
  B2P_CHECK_CUDA(cudaMalloc(&m->U, R * kUCols * e));
  B2P_CHECK_CUDA(cudaMemset(m->U, 0, R * kUCols * e));
  B2P_CHECK_CUDA(cudaMalloc(&m->qkv, R * m->qkv_dim * e));
  B2P_CHECK_CUDA(cudaMalloc(&m->attn, R * m->q_dim * e));
  B2P_CHECK_CUDA(cudaMalloc(&m->hbuf, R * c.hidden * e));
  const int ntiles = (c.vocab + 255) / 256;  // enough for any compact vocabulary
  B2P_CHECK_CUDA(cudaMalloc(&m->ce_part, R * 2 * ntiles * sizeof(float2)));
  B2P_CHECK_CUDA(cudaMalloc(&m->ce_tgt, R * 4));
  B2P_CHECK_CUDA(cudaMalloc(&m->row_loss, R * 4));
  B2P_CHECK_CUDA(cudaMalloc(&m->group_loss, m->max_groups * 4));
  B2P_CHECK_CUDA(cudaMalloc(&m->var_loss, m->max_groups * 4));
  B2P_CHECK_CUDA(cudaMalloc(&m->pairs, 2 * kMaxPerturbOps * 4));
  B2P_CHECK_CUDA(cudaMalloc(&m->d_tok, (size_t)2 * m->max_groups * c.seq * 4));
  B2P_CHECK_CUDA(cudaMalloc(&m->d_row_tgt, R * 4));
  B2P_CHECK_CUDA(cudaMalloc(&m->d_meta, 2 * m->max_groups * sizeof(int)));
  B2P_CHECK_CUDA(cudaMalloc(&m->d_var, m->max_groups * sizeof(VariantInfo)));
  B2P_CHECK_CUDA(cudaMalloc(&m->attn_sched, 2 * sizeof(int)));
  B2P_CHECK_CUDA(cudaMemset(m->attn_sched, 0, 2 * sizeof(int)));
  m->prep_ld = (std::max(c.dim, m->q_dim) + 7) / 8 * 8;
  B2P_CHECK_CUDA(
      cudaMalloc(&m->prep_a, (size_t)c.nlayers * m->max_groups * m->prep_segs * c.rank * m->prep_ld * e));
  if (m->ffn)
    B2P_CHECK_CUDA(cudaMalloc(&m->prep_a2, (size_t)c.nlayers * m->max_groups * c.rank * c.hidden * e));
  B2P_CHECK_CUDA(cudaMalloc(&m->prep_w, (size_t)c.nlayers * m->max_groups * 2 * c.dim * 4));
  B2P_CHECK_CUDA(cudaMalloc(&m->prep_wf, (size_t)m->max_groups * c.dim * 4));
  B2P_CHECK_CUDA(cudaMalloc(&m->rope_cos, (size_t)c.seq * (c.head_dim / 2) * 4));
  B2P_CHECK_CUDA(cudaMalloc(&m->rope_sin, (size_t)c.seq * (c.head_dim / 2) * 4));
  {
    Stager& sg = m->stg;
    size_t need = std::max<size_t>((size_t)2 * m->max_groups * c.seq * 4, (size_t)2 * m->max_groups * sizeof(int));
    need = std::max<size_t>(need, (size_t)m->max_groups * sizeof(VariantInfo));
    need = std::max<size_t>(need, (size_t)m->max_slots * 8);
    sg.slot_bytes = (need + 255) & ~size_t(255);
    sg.nslots = 8;
    B2P_CHECK_CUDA(cudaMallocHost(&sg.base, sg.slot_bytes * sg.nslots));
    sg.ev.resize(sg.nslots);
    sg.armed.assign(sg.nslots, 0);
    for (auto& e : sg.ev) B2P_CHECK_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  }
  // RoPE tables with the reference's expressions (training/cpu_ops.h:303-307)
  const int half = c.head_dim / 2;
  std::vector<float> cs((size_t)c.seq * half), sn((size_t)c.seq * half);
  for (int i = 0; i < half; i++) {
    const float freq = 1.0f / powf(c.rope_theta, 2.0f * i / (float)c.head_dim);
    for (int p = 0; p < c.seq; p++) {
      const float ang = p * freq;
      cs[(size_t)p * half + i] = cosf(ang);
      sn[(size_t)p * half + i] = sinf(ang);
    }
  }
  B2P_CHECK_CUDA(cudaMemcpy(m->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
  B2P_CHECK_CUDA(cudaMemcpy(m->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
  return B2P_OK;
}

void model_release(b2p_model* m) {
  void* dev[] = {m->wqkv, m->wo, m->w13, m->w2, m->cembed, m->embed, m->theta, m->masks, m->d_bufs,
                 m->d_polys, m->d_seeds, m->x, m->xn, m->U, m->qkv, m->attn, m->hbuf, m->ce_part,
                 m->ce_tgt, m->row_loss, m->group_loss, m->var_loss, m->pairs, m->d_tok, m->d_row_tgt, m->d_meta,
                 m->d_var, m->rope_cos, m->rope_sin, m->prep_a, m->prep_w, m->prep_wf, m->d_c2f, m->attn_sched,
                 m->prep_a2};
  for (void* p : dev)
    if (p) cudaFree(p);
  if (m->stg.base) cudaFreeHost(m->stg.base);
  for (auto e : m->stg.ev)
    if (e) cudaEventDestroy(e);
  for (auto e : m->ev_pool)
    if (e) cudaEventDestroy(e);
  if (m->p16) p16_release(m->p16);
  m->p16 = nullptr;
  if (m->st) cudaStreamDestroy(m->st);
}

// Convert an fp32 host matrix to 16-bit device storage at dst (row-major, same shape).
int upload16(b2p_model* m, void* dst, const float* src, size_t n) {
  float* tmp = nullptr;
  B2P_CHECK_CUDA(cudaMallocAsync(&tmp, n * 4, m->st));
  B2P_CHECK_CUDA(cudaMemcpyAsync(tmp, src, n * 4, cudaMemcpyHostToDevice, m->st));
  int rc = launch_f32_to_16(tmp, dst, (long long)n, m->bf16, m->st);
  B2P_CHECK_CUDA(cudaFreeAsync(tmp, m->st));
  if (rc) return rc;
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  return B2P_OK;
}

PerturbCtx pctx(const b2p_model* m) {
  PerturbCtx pc;
  pc.theta = m->theta;
  pc.masks = m->masks;
  pc.mask_words = m->mask_words;
  pc.variants = m->d_var;
  pc.group_variant = m->d_meta + m->max_groups;
  pc.group_rows = m->cfg.seq;
  return pc;
}

LoraEpi lora_epi(const b2p_model* m) {
  LoraEpi le;
  std::memset(&le, 0, sizeof(le));
  le.theta = m->theta;
  le.masks = m->masks;
  le.mask_words = m->mask_words;
  le.variants = m->d_var;
  le.group_variant = m->d_meta + m->max_groups;
  le.group_rows = m->cfg.seq;
  le.n_groups = m->cur_groups;
  le.n_variants = m->cur_vars;
  le.rank = m->cfg.rank;
  return le;
}

// launch_gemm, bracketed by CUDA events on the model stream when profiling is on.
int gemm_launch(b2p_model* m, int bn, int kind, const void* X, int ldx, const void* W, int ldw, int M, int N, int K,
                void* out, int ldo, const void* u16, const EpiParams& ep) {
  if (m->use_pair && pair_supported(kind, M, N, ep))
    return launch_gemm_pair(kind, m->bf16, X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, m->st);
  return launch_gemm(bn, kind, m->bf16, X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, m->st);
}

int gemm(b2p_model* m, int bn, int kind, const void* X, int ldx, const void* W, int ldw, int M, int N, int K,
         void* out, int ldo, const EpiParams& ep, const void* u16 = nullptr) {
  if (!u16) u16 = m->U;
  if (!m->prof) return gemm_launch(m, bn, kind, X, ldx, W, ldw, M, N, K, out, ldo, u16, ep);
  while (m->ev_pool.size() < m->ev_used + 2) {
    cudaEvent_t e;
    B2P_CHECK_CUDA(cudaEventCreate(&e));
    m->ev_pool.push_back(e);
  }
  // inside a stream capture the records must become event-record nodes of the graph
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  B2P_CHECK_CUDA(cudaStreamIsCapturing(m->st, &cap));
  const unsigned flags = cap == cudaStreamCaptureStatusActive ? cudaEventRecordExternal : 0u;
  B2P_CHECK_CUDA(cudaEventRecordWithFlags(m->ev_pool[m->ev_used], m->st, flags));
  int rc = gemm_launch(m, bn, kind, X, ldx, W, ldw, M, N, K, out, ldo, u16, ep);
  B2P_CHECK_CUDA(cudaEventRecordWithFlags(m->ev_pool[m->ev_used + 1], m->st, flags));
  m->ev_used += 2;
  m->prof_flops.push_back(2.0 * M * (double)N * K);
  return rc;
}

// gemm() for the MN-major CTA-pair launches of the backward (operands read in the layout they are
// stored in). Returns B2P_ERR_UNSUPPORTED, launching nothing, when the pair engine does not take the
// launch (B2P_OPT_PAIR_GEMM 0, fewer than 256 rows, unaligned operands): the caller then uses K-major
// copies on the engine chosen by gemm().
int gemm_mn(b2p_model* m, int kind, int opm, const void* X, int ldx, const void* W, int ldw, int M, int N, int K,
            void* out, int ldo, const EpiParams& ep) {
  if (!m->use_pair || ep.has_lora || !pair_mn_supported(kind, opm, M, N, K, X, ldx, W, ldw)) return B2P_ERR_UNSUPPORTED;
  if (!m->prof) return launch_gemm_pair_mn(kind, opm, m->bf16, X, ldx, W, ldw, M, N, K, out, ldo, ep, m->st);
  while (m->ev_pool.size() < m->ev_used + 2) {
    cudaEvent_t e;
    B2P_CHECK_CUDA(cudaEventCreate(&e));
    m->ev_pool.push_back(e);
  }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  B2P_CHECK_CUDA(cudaStreamIsCapturing(m->st, &cap));
  const unsigned flags = cap == cudaStreamCaptureStatusActive ? cudaEventRecordExternal : 0u;
  B2P_CHECK_CUDA(cudaEventRecordWithFlags(m->ev_pool[m->ev_used], m->st, flags));
  int rc = launch_gemm_pair_mn(kind, opm, m->bf16, X, ldx, W, ldw, M, N, K, out, ldo, ep, m->st);
  B2P_CHECK_CUDA(cudaEventRecordWithFlags(m->ev_pool[m->ev_used + 1], m->st, flags));
  m->ev_used += 2;
  m->prof_flops.push_back(2.0 * M * (double)N * K);
  return rc;
}

// The batched forward over G groups whose inputs are already staged on the device.
// With `sv`, every activation the backprop-LoRA backward reads is written to its
// per-layer slab instead of the shared scratch buffers, and the W1/W3 outputs are
// kept (16-bit GEMM output + a separate gate kernel instead of the fused SwiGLU
// epilogue).
int run_forward(b2p_model* m, int G, const int32_t* tok, const ForwardSaves* sv = nullptr) {
  const auto& c = m->cfg;
  const int R = G * c.seq;
  const int D = c.dim, H = c.hidden, QD = m->q_dim, KVD = m->kv_dim, QKV = m->qkv_dim;
  const size_t e = esz(m);
  DeviceCtx* ctx = nullptr;
  int rc = ctx_get(&ctx);
  if (rc) return rc;
  const int* group_seq = m->d_meta;
  rc = launch_embed(m->embed, c.vocab, D, tok, group_seq, c.seq, R, m->x, ctx->status, m->st);
  if (rc) return rc;
  const PerturbCtx pc = pctx(m);
  // every variant's perturbed LoRA-down operands and rms weights, once for all layers
  const int nv = m->cur_vars;
  LoraPrepArgs lp;
  lp.theta = m->theta;
  lp.masks = m->masks;
  lp.mask_words = m->mask_words;
  lp.variants = m->d_var;
  lp.n_var = nv;
  lp.nlayers = c.nlayers;
  lp.dim = D;
  lp.q_dim = QD;
  lp.rank = c.rank;
  lp.ld = m->prep_ld;
  lp.segs = m->prep_segs;
  lp.hidden = H;
  lp.layer_size = m->layer_size;
  lp.oAq = m->oAq; lp.oAk = m->oAk; lp.oAv = m->oAv; lp.oAo = m->oAo;
  lp.oA1 = m->oA1; lp.oA3 = m->oA3; lp.oA2 = m->oA2;
  lp.oRa = m->oRa; lp.oRf = m->oRf; lp.oRfinal = m->oRfinal;
  lp.a_out = m->prep_a;
  lp.a2_out = m->ffn ? m->prep_a2 : nullptr;
  lp.w_out = m->prep_w;
  lp.w_final = m->prep_wf;
  if ((rc = launch_lora_prep(lp, m->bf16, m->st))) return rc;
  const long long a_vstride = (long long)m->prep_segs * c.rank * m->prep_ld;
  const long long a2_vstride = (long long)c.rank * H;
  auto prep_a = [&](int l, int row) -> const void* {
    return static_cast<const char*>(m->prep_a) + ((size_t)l * nv * a_vstride + (size_t)row * m->prep_ld) * e;
  };
  auto slab = [R](void* base, int l, size_t row_bytes) -> void* {
    return static_cast<char*>(base) + (size_t)l * R * row_bytes;
  };
  for (int l = 0; l < c.nlayers; ++l) {
    const long long lb = (long long)l * m->layer_size;
    void* xn = sv ? slab(sv->xn, l, D * e) : m->xn;
    void* U = sv ? slab(sv->U, l, kUCols * e) : m->U;
    void* qkv = sv ? slab(sv->qkv, l, QKV * e) : m->qkv;
    void* attn = sv ? slab(sv->attn, l, QD * e) : m->attn;
    if (sv) B2P_CHECK_CUDA(cudaMemcpyAsync(slab(sv->x_in, l, D * 4), m->x, (size_t)R * D * 4,
                                           cudaMemcpyDeviceToDevice, m->st));
    // RMSNorm(rms_att) + LoRA-down for q, k, v
    NormLoraArgs na;
    std::memset(&na, 0, sizeof(na));
    na.in = m->x;
    na.xn = xn;
    na.rows = R;
    na.dim = D;
    na.norm = 1;
    na.w_off = lb + m->oRa;
    na.n_a = 3;
    na.a_off[0] = lb + m->oAq;
    na.a_off[1] = lb + m->oAk;
    na.a_off[2] = lb + m->oAv;
    na.rank = c.rank;
    na.U = U;
    na.u_col = 0;  // q, k, v at U16 columns 0, 16, 32
    na.pc = pc;
    na.a_prep = prep_a(l, 0);
    na.a_prep_vstride = a_vstride;
    na.a_prep_ld = m->prep_ld;
    na.w_prep = m->prep_w + (size_t)l * nv * 2 * D;
    na.w_prep_vstride = 2LL * D;
    if ((rc = launch_norm_lora(na, m->bf16, m->st))) return rc;
    // Q|K|V = xn · Wqkv^T + B·U (perturbed B), RoPE on Q and K
    EpiParams ep;
    std::memset(&ep, 0, sizeof(ep));
    ep.M = R;
    ep.N = QKV;
    ep.has_lora = 1;
    ep.lora = lora_epi(m);
    ep.lora.nseg = 3;
    ep.lora.seg_start[0] = 0;
    ep.lora.seg_start[1] = QD;
    ep.lora.seg_start[2] = QD + KVD;
    ep.lora.seg_start[3] = QKV;
    ep.lora.seg_boff[0] = lb + m->oBq;
    ep.lora.seg_boff[1] = lb + m->oBk;
    ep.lora.seg_boff[2] = lb + m->oBv;
    ep.lora.seg_ucol[0] = 0;
    ep.lora.seg_ucol[1] = 16;
    ep.lora.seg_ucol[2] = 32;
    ep.rope_cos = m->rope_cos;
    ep.rope_sin = m->rope_sin;
    ep.rope_cols = QD + KVD;
    ep.head_dim = c.head_dim;
    ep.seq_len = c.seq;
    const char* wqkv = static_cast<const char*>(m->wqkv) + (size_t)l * QKV * D * e;
    if ((rc = gemm(m, m->qkv_bn, EPI_QKV_ROPE, xn, D, wqkv, D, R, QKV, D, qkv, QKV, ep, U))) return rc;
    // attention
    AttnArgs aa;
    std::memset(&aa, 0, sizeof(aa));
    aa.qkv = qkv;
    aa.ld_qkv = QKV;
    aa.q_off = 0;
    aa.k_off = QD;
    aa.v_off = QD + KVD;
    aa.out = attn;
    aa.ld_out = QD;
    aa.seq = c.seq;
    aa.heads = c.heads;
    aa.kv_heads = c.kv_heads;
    aa.ngroups = G;
    aa.lse = sv ? sv->lse + (size_t)l * R * c.heads : nullptr;
    aa.sched = m->tc_attn ? m->attn_sched : nullptr;
    if ((rc = launch_attention(aa, m->bf16, m->st))) return rc;
    // LoRA-down of the attention output for Wo
    NormLoraArgs nb;
    std::memset(&nb, 0, sizeof(nb));
    nb.in = attn;
    nb.rows = R;
    nb.dim = QD;
    nb.norm = 0;
    nb.n_a = 1;
    nb.a_off[0] = lb + m->oAo;
    nb.rank = c.rank;
    nb.U = U;
    nb.u_col = 48;  // o at U16 column 48
    nb.pc = pc;
    nb.a_prep = prep_a(l, 3 * c.rank);
    nb.a_prep_vstride = a_vstride;
    nb.a_prep_ld = m->prep_ld;
    if ((rc = launch_norm_lora(nb, m->bf16, m->st))) return rc;
    // x += alpha * (attn · Wo^T + Bo·Uo)
    EpiParams eo;
    std::memset(&eo, 0, sizeof(eo));
    eo.M = R;
    eo.N = D;
    eo.alpha = c.res_alpha;
    eo.has_lora = 1;
    eo.lora = lora_epi(m);
    eo.lora.nseg = 1;
    eo.lora.seg_start[0] = 0;
    eo.lora.seg_start[1] = D;
    eo.lora.seg_boff[0] = lb + m->oBo;
    eo.lora.seg_ucol[0] = 48;
    const char* wo = static_cast<const char*>(m->wo) + (size_t)l * D * QD * e;
    if ((rc = gemm(m, pick_bn(D, EPI_RESID), EPI_RESID, attn, QD, wo, QD, R, D, QD, m->x, D, eo, U))) return rc;
    if (sv) B2P_CHECK_CUDA(cudaMemcpyAsync(slab(sv->x_mid, l, D * 4), m->x, (size_t)R * D * 4,
                                           cudaMemcpyDeviceToDevice, m->st));
    // RMSNorm(rms_ffn)
    NormLoraArgs nf;
    std::memset(&nf, 0, sizeof(nf));
    nf.in = m->x;
    void* xn2 = (sv && sv->xn2) ? slab(sv->xn2, l, D * e) : m->xn;
    nf.xn = xn2;
    nf.rows = R;
    nf.dim = D;
    nf.norm = 1;
    nf.w_off = lb + m->oRf;
    nf.n_a = 0;
    nf.pc = pc;
    if (m->ffn) {  // LoRA-down for W1 and W3 (U16 columns 0 and 16; q/k/v/o are consumed by now)
      nf.n_a = 2;
      nf.a_off[0] = lb + m->oA1;
      nf.a_off[1] = lb + m->oA3;
      nf.rank = c.rank;
      nf.U = U;
      nf.u_col = 0;
      nf.a_prep = prep_a(l, 4 * c.rank);
      nf.a_prep_vstride = a_vstride;
      nf.a_prep_ld = m->prep_ld;
    }
    nf.w_prep = m->prep_w + (size_t)l * nv * 2 * D + D;
    nf.w_prep_vstride = 2LL * D;
    if ((rc = launch_norm_lora(nf, m->bf16, m->st))) return rc;
    // h = silu(xn·W1^T) * (xn·W3^T)  (W1/W3 rows interleaved in 128-row blocks)
    EpiParams es;
    std::memset(&es, 0, sizeof(es));
    es.M = R;
    es.N = 2 * H;
    if (m->ffn) {  // h1 += B1·u1, h3 += B3·u3 (train_mezo.m:1634-1638)
      es.has_lora = 1;
      es.lora = lora_epi(m);
      es.lora.nseg = 2;
      es.lora.inter128 = 1;
      es.lora.seg_start[0] = 0;
      es.lora.seg_start[1] = H;
      es.lora.seg_start[2] = 2 * H;
      es.lora.seg_boff[0] = lb + m->oB1;
      es.lora.seg_boff[1] = lb + m->oB3;
      es.lora.seg_ucol[0] = 0;
      es.lora.seg_ucol[1] = 16;
    }
    const char* w13 = static_cast<const char*>(m->w13) + (size_t)l * 2 * H * D * e;
    if (sv) {
      void* h13 = slab(sv->h13, l, (size_t)2 * H * e);
      if ((rc = gemm(m, 256, EPI_H16, xn2, D, w13, D, R, 2 * H, D, h13, 2 * H, es))) return rc;
      if ((rc = launch_swiglu_gate(h13, R, H, m->hbuf, m->bf16, m->st))) return rc;
    } else {
      if ((rc = gemm(m, 256, EPI_SWIGLU, m->xn, D, w13, D, R, 2 * H, D, m->hbuf, H, es, m->ffn ? U : nullptr)))
        return rc;
    }
    if (m->ffn) {  // LoRA-down of the gated activation for W2 (U16 column 32)
      NormLoraArgs ng;
      std::memset(&ng, 0, sizeof(ng));
      ng.in = m->hbuf;
      ng.rows = R;
      ng.dim = H;
      ng.norm = 0;
      ng.n_a = 1;
      ng.a_off[0] = lb + m->oA2;
      ng.rank = c.rank;
      ng.U = U;
      ng.u_col = 32;
      ng.pc = pc;
      ng.a_prep = static_cast<const char*>(m->prep_a2) + (size_t)l * nv * a2_vstride * e;
      ng.a_prep_vstride = a2_vstride;
      ng.a_prep_ld = H;
      if ((rc = launch_norm_lora(ng, m->bf16, m->st))) return rc;
    }
    // x += alpha * (h · W2^T)
    EpiParams e2;
    std::memset(&e2, 0, sizeof(e2));
    e2.M = R;
    e2.N = D;
    e2.alpha = c.res_alpha;
    if (m->ffn) {  // o += B2·u2 (train_mezo.m:1658-1661)
      e2.has_lora = 1;
      e2.lora = lora_epi(m);
      e2.lora.nseg = 1;
      e2.lora.seg_start[0] = 0;
      e2.lora.seg_start[1] = D;
      e2.lora.seg_boff[0] = lb + m->oB2;
      e2.lora.seg_ucol[0] = 32;
    }
    const char* w2 = static_cast<const char*>(m->w2) + (size_t)l * D * H * e;
    if ((rc = gemm(m, pick_bn(D, EPI_RESID), EPI_RESID, m->hbuf, H, w2, H, R, D, H, m->x, D, e2,
                   m->ffn ? U : nullptr)))
      return rc;
  }
  // final RMSNorm + lm-head with fused cross-entropy partials
  if (sv) B2P_CHECK_CUDA(cudaMemcpyAsync(sv->x_final, m->x, (size_t)R * D * 4, cudaMemcpyDeviceToDevice, m->st));
  void* xnf = sv ? sv->xn_final : m->xn;
  NormLoraArgs nl;
  std::memset(&nl, 0, sizeof(nl));
  nl.in = m->x;
  nl.xn = xnf;
  nl.rows = R;
  nl.dim = D;
  nl.norm = 1;
  nl.w_off = m->oRfinal;
  nl.pc = pc;
  nl.w_prep = m->prep_wf;
  nl.w_prep_vstride = D;
  if ((rc = launch_norm_lora(nl, m->bf16, m->st))) return rc;
  const int ntiles = (m->cv + 255) / 256;
  EpiParams ec;
  std::memset(&ec, 0, sizeof(ec));
  ec.M = R;
  ec.N = m->cv;
  ec.targets = m->d_row_tgt;
  ec.ce_part = m->ce_part;
  ec.ce_tgt = m->ce_tgt;
  ec.n_tiles_n = ntiles;
  if ((rc = gemm(m, 256, EPI_CE, xnf, D, m->cembed, D, R, m->cv, D, nullptr, 0, ec))) return rc;
  return launch_ce_reduce(m->ce_part, 2 * ntiles, m->ce_tgt, R, c.seq, m->row_loss, m->group_loss, m->st,
                          sv ? sv->row_lse : nullptr);
}

__global__ void expand_targets_kernel(const int32_t* seq_tgt, const int* group_seq, int seq, int rows, int cv,
                                      int32_t* row_tgt, uint32_t* status) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const int g = row / seq, t = row - g * seq;
  int tg = seq_tgt[(long long)group_seq[g] * seq + t];
  if (tg < 0 || tg >= cv) {
    atomicCAS(status, 0u, (uint32_t)DEV_BAD_ARGS);
    tg = -1;
  }
  row_tgt[row] = tg;
}

// Copy a small host buffer to the device through a pinned ring slot. A slot is
// reused only after the copy that last read it has executed (event fence), so
// asynchronous calls never see their staging overwritten.
int stage_copy(b2p_model* m, void* dst, const void* src, size_t bytes) {
  Stager& s = m->stg;
  B2P_REQUIRE(bytes <= s.slot_bytes, "staging copy of %zu bytes exceeds slot size %zu", bytes, s.slot_bytes);
  const int k = s.next;
  s.next = (s.next + 1) % s.nslots;
  if (s.armed[k]) B2P_CHECK_CUDA(cudaEventSynchronize(s.ev[k]));
  char* p = s.base + (size_t)k * s.slot_bytes;
  std::memcpy(p, src, bytes);
  B2P_CHECK_CUDA(cudaMemcpyAsync(dst, p, bytes, cudaMemcpyHostToDevice, m->st));
  B2P_CHECK_CUDA(cudaEventRecord(s.ev[k], m->st));
  s.armed[k] = 1;
  return B2P_OK;
}

// Validate host tokens/targets of n_seq sequences and upload them (int32) to d_tok.
int stage_tokens(b2p_model* m, const uint16_t* tokens, const uint16_t* ctargets, int n_seq) {
  const auto& c = m->cfg;
  B2P_REQUIRE(tokens && ctargets, "null token/target buffer");
  B2P_REQUIRE(n_seq >= 1 && n_seq <= m->max_groups, "sequence count %d out of range", n_seq);
  const size_t nt = (size_t)n_seq * c.seq;
  std::vector<int32_t> h(2 * nt);
  for (size_t i = 0; i < nt; ++i) {
    B2P_REQUIRE(tokens[i] < c.vocab, "token[%zu]=%d out of range (vocab %d)", i, (int)tokens[i], c.vocab);
    B2P_REQUIRE(ctargets[i] < m->cv, "target[%zu]=%d out of range (compact vocab %d)", i, (int)ctargets[i], m->cv);
    h[i] = tokens[i];
    h[nt + i] = ctargets[i];
  }
  return stage_copy(m, m->d_tok, h.data(), h.size() * 4);
}

// Group tables for n_var variants x n_seq sequences, per-row targets, variant table.
int stage_groups(b2p_model* m, int n_seq, const std::vector<VariantInfo>& vars, const int32_t* d_targets) {
  const auto& c = m->cfg;
  const int n_var = (int)vars.size();
  const int G = n_seq * n_var;
  B2P_REQUIRE(n_seq >= 1 && n_var >= 1 && G <= m->max_groups, "groups %d x %d exceed max_groups %d", n_var, n_seq,
              m->max_groups);
  std::vector<int> meta(2 * m->max_groups, 0);
  for (int v = 0; v < n_var; ++v)
    for (int q = 0; q < n_seq; ++q) {
      meta[v * n_seq + q] = q;                  // group -> sequence
      meta[m->max_groups + v * n_seq + q] = v;  // group -> variant
    }
  m->cur_groups = G;
  m->cur_vars = n_var;
  int rc = stage_copy(m, m->d_meta, meta.data(), meta.size() * sizeof(int));
  if (rc) return rc;
  if ((rc = stage_copy(m, m->d_var, vars.data(), vars.size() * sizeof(VariantInfo)))) return rc;
  DeviceCtx* ctx = nullptr;
  if ((rc = ctx_get(&ctx))) return rc;
  expand_targets_kernel<<<(G * c.seq + 255) / 256, 256, 0, m->st>>>(d_targets, m->d_meta, c.seq, G * c.seq, m->cv,
                                                                     m->d_row_tgt, ctx->status);
  B2P_POST_LAUNCH();
  return B2P_OK;
}

int gen_masks(b2p_model* m, const uint64_t* seeds, int n) {
  B2P_REQUIRE(n >= 1 && n <= m->max_slots, "seed count %d exceeds mask slots %d", n, m->max_slots);
  // the slots already hold these seeds' masks (e.g. the update after the evaluation of the same seeds)
  if ((int)m->slot_seed.size() >= n && std::equal(seeds, seeds + n, m->slot_seed.begin())) return B2P_OK;
  int rc = stage_copy(m, m->d_seeds, seeds, (size_t)n * 8);
  if (rc) return rc;
  m->slot_seed.assign(seeds, seeds + n);
  rc = launch_sign_masks(m->d_bufs, m->nbufs, m->d_polys, m->nchunks, m->total_draws, m->mask_words, m->d_seeds, n,
                         m->masks, m->st);
  if (rc) m->slot_seed.clear();
  return rc;
}

int ready(const b2p_model* m) {
  if (!m) {
    set_error("null model");
    return B2P_ERR_ARG;
  }
  for (int l = 0; l < m->cfg.nlayers; ++l)
    if (!m->layer_set[l]) {
      set_error("layer %d weights not set", l);
      return B2P_ERR_STATE;
    }
  if (!m->embed_set) {
    set_error("embedding not set");
    return B2P_ERR_STATE;
  }
  return B2P_OK;
}

// Forward over n_seq sequences (device int32 tokens/targets) x variants; per-variant
// losses land in m->var_loss. Asynchronous on the model stream.
int eval_variants(b2p_model* m, const int32_t* d_tokens, const int32_t* d_targets, int n_seq,
                  const std::vector<VariantInfo>& vars) {
  int rc = stage_groups(m, n_seq, vars, d_targets);
  if (rc) return rc;
  if ((rc = run_forward(m, n_seq * (int)vars.size(), d_tokens))) return rc;
  return launch_variant_loss(m->group_loss, (int)vars.size(), n_seq, m->var_loss, m->st);
}

// ±ε variants of each seed: index 2s = θ+εz_s, 2s+1 = (θ+εz_s)-2εz_s.
int eval_pairs(b2p_model* m, const int32_t* d_tokens, const int32_t* d_targets, int n_seq, const uint64_t* seeds,
               int n_seeds, float eps) {
  B2P_REQUIRE(seeds && n_seeds >= 1, "no seeds");
  B2P_REQUIRE(2 * n_seeds * n_seq <= m->max_groups, "2 x %d seeds x %d sequences exceed max_groups %d", n_seeds,
              n_seq, m->max_groups);
  int rc = gen_masks(m, seeds, n_seeds);
  if (rc) return rc;
  const float m2e = -2.0f * eps;
  std::vector<VariantInfo> vars(2 * n_seeds);
  for (int s = 0; s < n_seeds; ++s) {
    vars[2 * s] = VariantInfo{s, 1, eps, 0.f};
    vars[2 * s + 1] = VariantInfo{s, 2, eps, m2e};
  }
  return eval_variants(m, d_tokens, d_targets, n_seq, vars);
}

bool is_device_ptr(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// Copy n floats of var_loss to out; synchronise (and check device status) only
// when out is host memory.
int copy_losses(b2p_model* m, float* out, int n) {
  B2P_CHECK_CUDA(cudaMemcpyAsync(out, m->var_loss, (size_t)n * 4, cudaMemcpyDefault, m->st));
  if (is_device_ptr(out)) return B2P_OK;
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  return check_device_status(m->st);
}

}  // namespace

namespace b2p {

size_t model_esz(const b2p_model* m) { return esz(m); }
int model_ready(const b2p_model* m) { return ready(m); }
int model_stage_tokens(b2p_model* m, const uint16_t* tokens, const uint16_t* ctargets, int n_seq) {
  return stage_tokens(m, tokens, ctargets, n_seq);
}
int model_stage_groups(b2p_model* m, int n_seq, const std::vector<VariantInfo>& vars, const int32_t* d_targets) {
  return stage_groups(m, n_seq, vars, d_targets);
}
PerturbCtx model_pctx(const b2p_model* m) { return pctx(m); }
LoraEpi model_lora_epi(const b2p_model* m) { return lora_epi(m); }
int model_gemm(b2p_model* m, int bn, int kind, const void* X, int ldx, const void* W, int ldw, int M, int N, int K,
               void* out, int ldo, const void* u16, const EpiParams& ep) {
  return gemm(m, bn, kind, X, ldx, W, ldw, M, N, K, out, ldo, ep, u16);
}
int model_gemm_mn(b2p_model* m, int kind, int opm, const void* X, int ldx, const void* W, int ldw, int M, int N, int K,
                  void* out, int ldo, const EpiParams& ep) {
  return gemm_mn(m, kind, opm, X, ldx, W, ldw, M, N, K, out, ldo, ep);
}
int model_run_forward(b2p_model* m, int G, const int32_t* tok, const ForwardSaves* sv) {
  return run_forward(m, G, tok, sv);
}

}  // namespace b2p

extern "C" {

b2p_model* b2p_model_create(const b2p_model_config* cfg) {
  if (!cfg) {
    set_error("null config");
    return nullptr;
  }
  const auto& c = *cfg;
  auto bad = [](const char* msg) -> b2p_model* {
    set_error("%s", msg);
    return nullptr;
  };
  if (c.dim <= 0 || c.dim % 64 || c.hidden <= 0 || c.hidden % 128 || c.head_dim != 64 || c.heads <= 0 ||
      c.kv_heads <= 0 || c.heads % c.kv_heads || c.seq <= 0 || c.seq % 128 || c.nlayers <= 0 || c.vocab <= 0)
    return bad("unsupported shape: need dim %% 64 == 0, hidden %% 128 == 0, head_dim 64, seq %% 128 == 0");
  if (c.rank != 4 && c.rank != 8) return bad("LoRA rank must be 4 or 8");
  if (c.dtype != B2P_F16 && c.dtype != B2P_BF16) return bad("dtype must be B2P_F16 or B2P_BF16");
  if (c.max_groups < 1 || c.max_groups > 256) return bad("max_groups must be in [1, 256]");
  if (c.lora_ffn != 0 && c.lora_ffn != 1) return bad("lora_ffn must be 0 or 1");
  if (c.lora_ffn && c.seq % 256) return bad("--lora-ffn needs seq %% 256 == 0 (two-segment SwiGLU LoRA tiles)");
  if (c.lora_ffn && c.hidden != 1152 && c.hidden != 1408 && c.hidden != 2560)
    return bad("--lora-ffn needs hidden in {1152, 1408, 2560} (LoRA-down width of the gated activation)");
  const int qd = c.heads * c.head_dim, kvd = c.kv_heads * c.head_dim;
  if (qd % 128 && qd % 160) return bad("q_dim must be a multiple of 128 or 160");
  const int qkv_bn = (qd % 160 == 0 && kvd % 160 == 0) ? 160 : ((qd % 128 == 0 && kvd % 128 == 0) ? 128 : 0);
  if (!qkv_bn) return bad("q_dim and kv_dim need a common Q|K|V tile width (128 or 160)");
  b2p_model* m = new b2p_model();
  m->qkv_bn = qkv_bn;
  m->cfg = c;
  m->bf16 = c.dtype == B2P_BF16;
  m->q_dim = qd;
  m->kv_dim = kvd;
  m->qkv_dim = qd + 2 * kvd;
  const long long r = c.rank, D = c.dim, Q = qd, KV = kvd;
  long long o = 0;
  m->oAq = o; o += r * D;
  m->oBq = o; o += Q * r;
  m->oAk = o; o += r * D;
  m->oBk = o; o += KV * r;
  m->oAv = o; o += r * D;
  m->oBv = o; o += KV * r;
  m->oAo = o; o += r * Q;
  m->oBo = o; o += D * r;
  if (c.lora_ffn) {  // train_mezo.m:575-582
    const long long H = c.hidden;
    m->ffn = true;
    m->prep_segs = 6;
    m->oA1 = o; o += r * D;
    m->oB1 = o; o += H * r;
    m->oA2 = o; o += r * H;
    m->oB2 = o; o += D * r;
    m->oA3 = o; o += r * D;
    m->oB3 = o; o += H * r;
  }
  m->oRa = o; o += D;
  m->oRf = o; o += D;
  m->layer_size = o;
  m->oRfinal = (long long)c.nlayers * o;
  m->P = m->oRfinal + D;
  m->mask_words = (m->P + 31) / 32;
  m->max_groups = c.max_groups;
  m->max_rows = c.max_groups * c.seq;
  m->max_slots = kMaxPerturbOps;  // sign-mask rows (64 seeds per call)
  m->layer_set.assign(c.nlayers, 0);
  int rc = cudaGetDevice(&m->device) == cudaSuccess ? B2P_OK : B2P_ERR_CUDA;
  DeviceCtx* ctx = nullptr;
  if (!rc) rc = ctx_get(&ctx);
  if (!rc && cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) != cudaSuccess) {
    set_error("cudaStreamCreate failed");
    rc = B2P_ERR_CUDA;
  }
  if (!rc) rc = model_alloc(m);
  if (!rc) {
    std::vector<long long> sizes;
    const long long H = c.hidden;
    for (int l = 0; l < c.nlayers; ++l) {
      const long long s[8] = {r * D, Q * r, r * D, KV * r, r * D, KV * r, r * Q, D * r};
      sizes.insert(sizes.end(), s, s + 8);
      if (m->ffn) {
        const long long f[6] = {r * D, H * r, r * H, D * r, r * D, H * r};
        sizes.insert(sizes.end(), f, f + 6);
      }
      sizes.push_back(D);
      sizes.push_back(D);
    }
    sizes.push_back(D);
    SignPlan plan = make_sign_plan(sizes);
    m->nbufs = (int)plan.bufs.size();
    m->nchunks = plan.nchunks;
    m->total_draws = plan.total_draws;
    if (!plan.valid) {
      set_error("xoshiro jump polynomial could not be established (Berlekamp-Massey / stepping check failed)");
      rc = B2P_ERR_STATE;
    } else if (cudaMalloc(&m->d_bufs, plan.bufs.size() * sizeof(SignBuffer)) != cudaSuccess ||
        cudaMalloc(&m->d_polys, plan.polys.size() * 8) != cudaSuccess ||
        cudaMemcpy(m->d_bufs, plan.bufs.data(), plan.bufs.size() * sizeof(SignBuffer), cudaMemcpyHostToDevice) !=
            cudaSuccess ||
        cudaMemcpy(m->d_polys, plan.polys.data(), plan.polys.size() * 8, cudaMemcpyHostToDevice) != cudaSuccess) {
      set_error("sign-plan upload failed");
      rc = B2P_ERR_CUDA;
    }
  }
  if (rc) {
    model_release(m);
    delete m;
    return nullptr;
  }
  return m;
}

void b2p_model_free(b2p_model* m) {
  if (!m) return;
  cudaStreamSynchronize(m->st);
  model_release(m);
  delete m;
}

long long b2p_model_trainable_count(const b2p_model* m) { return m ? m->P : -1; }

void* b2p_model_stream(b2p_model* m) { return m ? (void*)m->st : nullptr; }

int b2p_model_set_layer(b2p_model* m, int layer, const float* Wq, const float* Wk, const float* Wv, const float* Wo,
                        const float* W1, const float* W2, const float* W3) {
  B2P_REQUIRE(m && layer >= 0 && layer < m->cfg.nlayers, "bad model/layer");
  B2P_REQUIRE(Wq && Wk && Wv && Wo && W1 && W2 && W3, "null weight pointer");
  const auto& c = m->cfg;
  const int D = c.dim, H = c.hidden, QD = m->q_dim, KVD = m->kv_dim;
  const size_t e = esz(m);
  // stacked [Wq; Wk; Wv] rows (the qkv-fused kernel of training/io.h:182-206)
  std::vector<float> qkv((size_t)m->qkv_dim * D);
  std::memcpy(qkv.data(), Wq, (size_t)QD * D * 4);
  std::memcpy(qkv.data() + (size_t)QD * D, Wk, (size_t)KVD * D * 4);
  std::memcpy(qkv.data() + (size_t)(QD + KVD) * D, Wv, (size_t)KVD * D * 4);
  int rc = upload16(m, static_cast<char*>(m->wqkv) + (size_t)layer * m->qkv_dim * D * e, qkv.data(), qkv.size());
  if (rc) return rc;
  rc = upload16(m, static_cast<char*>(m->wo) + (size_t)layer * D * QD * e, Wo, (size_t)D * QD);
  if (rc) return rc;
  // W1/W3 interleaved in blocks of 128 rows: [W1 b | W3 b] per 256-row tile (SwiGLU epilogue pairs)
  std::vector<float> w13((size_t)2 * H * D);
  for (int b = 0; b < H / 128; ++b) {
    std::memcpy(w13.data() + (size_t)(2 * b) * 128 * D, W1 + (size_t)b * 128 * D, (size_t)128 * D * 4);
    std::memcpy(w13.data() + (size_t)(2 * b + 1) * 128 * D, W3 + (size_t)b * 128 * D, (size_t)128 * D * 4);
  }
  rc = upload16(m, static_cast<char*>(m->w13) + (size_t)layer * 2 * H * D * e, w13.data(), w13.size());
  if (rc) return rc;
  rc = upload16(m, static_cast<char*>(m->w2) + (size_t)layer * D * H * e, W2, (size_t)D * H);
  if (rc) return rc;
  m->layer_set[layer] = 1;
  m->weights_version++;
  return B2P_OK;
}

int b2p_model_set_embedding(b2p_model* m, const float* embed, const int32_t* compact_to_full, int cv) {
  B2P_REQUIRE(m && embed && compact_to_full, "null argument");
  B2P_REQUIRE(cv >= 1 && cv <= m->cfg.vocab, "compact vocab %d out of range", cv);
  const auto& c = m->cfg;
  for (int i = 0; i < cv; ++i)
    B2P_REQUIRE(compact_to_full[i] >= 0 && compact_to_full[i] < c.vocab, "compact_to_full[%d] out of range", i);
  B2P_CHECK_CUDA(cudaMemcpyAsync(m->embed, embed, (size_t)c.vocab * c.dim * 4, cudaMemcpyHostToDevice, m->st));
  // compact tied embedding (vocab_compact_embed, training/cpu_ops.h:171-176)
  std::vector<float> ce((size_t)cv * c.dim);
  for (int i = 0; i < cv; ++i)
    std::memcpy(ce.data() + (size_t)i * c.dim, embed + (size_t)compact_to_full[i] * c.dim, (size_t)c.dim * 4);
  if (m->cembed) cudaFree(m->cembed);
  m->cembed = nullptr;
  B2P_CHECK_CUDA(cudaMalloc(&m->cembed, (size_t)cv * c.dim * esz(m)));
  m->cv = cv;
  if (m->d_c2f) cudaFree(m->d_c2f);
  m->d_c2f = nullptr;
  B2P_CHECK_CUDA(cudaMalloc(&m->d_c2f, (size_t)cv * sizeof(int32_t)));
  B2P_CHECK_CUDA(cudaMemcpy(m->d_c2f, compact_to_full, (size_t)cv * sizeof(int32_t), cudaMemcpyHostToDevice));
  m->h_c2f.assign(compact_to_full, compact_to_full + cv);
  int rc = upload16(m, m->cembed, ce.data(), ce.size());
  if (rc) return rc;
  m->embed_set = true;
  m->weights_version++;
  return B2P_OK;
}

int b2p_model_set_trainable(b2p_model* m, const float* theta, long long n) {
  B2P_REQUIRE(m && theta, "null argument");
  B2P_REQUIRE(n == m->P, "trainable count %lld != %lld", n, m->P);
  B2P_CHECK_CUDA(cudaMemcpyAsync(m->theta, theta, n * 4, cudaMemcpyDefault, m->st));
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  return B2P_OK;
}

int b2p_model_get_trainable(b2p_model* m, float* theta, long long n) {
  B2P_REQUIRE(m && theta, "null argument");
  B2P_REQUIRE(n == m->P, "trainable count %lld != %lld", n, m->P);
  B2P_CHECK_CUDA(cudaMemcpyAsync(theta, m->theta, n * 4, cudaMemcpyDefault, m->st));
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  return B2P_OK;
}

int b2p_model_eval(b2p_model* m, const uint16_t* tokens, const uint16_t* ctargets, int n_seq,
                   const b2p_variant* vars, int n_var, float* losses) {
  int rc = ready(m);
  if (rc) return rc;
  B2P_REQUIRE(vars && losses && n_var >= 1, "null variants/losses");
  if ((rc = stage_tokens(m, tokens, ctargets, n_seq))) return rc;
  std::vector<uint64_t> seeds;
  std::vector<VariantInfo> vi(n_var);
  for (int v = 0; v < n_var; ++v) {
    B2P_REQUIRE(vars[v].mode >= 0 && vars[v].mode <= 2, "variant mode must be 0, 1 or 2");
    int slot = 0;
    if (vars[v].mode) {
      slot = -1;
      for (size_t i = 0; i < seeds.size(); ++i)
        if (seeds[i] == vars[v].seed) slot = (int)i;
      if (slot < 0) {
        slot = (int)seeds.size();
        seeds.push_back(vars[v].seed);
      }
    }
    vi[v] = VariantInfo{slot, vars[v].mode, vars[v].s1, vars[v].s2};
  }
  if (!seeds.empty() && (rc = gen_masks(m, seeds.data(), (int)seeds.size()))) return rc;
  const size_t nt = (size_t)n_seq * m->cfg.seq;
  if ((rc = eval_variants(m, m->d_tok, m->d_tok + nt, n_seq, vi))) return rc;
  return copy_losses(m, losses, n_var);
}

int b2p_model_group_losses(b2p_model* m, float* out, int n) {
  B2P_REQUIRE(m && out, "null argument");
  B2P_REQUIRE(m->cur_groups >= 1, "no forward has run on this model");
  B2P_REQUIRE(n >= 1 && n <= m->cur_groups, "%d group losses requested, the last forward had %d groups", n,
              m->cur_groups);
  B2P_CHECK_CUDA(cudaMemcpyAsync(out, m->group_loss, (size_t)n * 4, cudaMemcpyDefault, m->st));
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  return check_device_status(m->st);
}

int b2p_mezo_step(b2p_model* m, const uint16_t* tokens, const uint16_t* ctargets, uint64_t seed, float eps,
                  float lr, float* loss_plus, float* loss_minus, float* proj_grad) {
  int rc = ready(m);
  if (rc) return rc;
  if ((rc = stage_tokens(m, tokens, ctargets, 1))) return rc;
  const size_t nt = (size_t)m->cfg.seq;
  if ((rc = eval_pairs(m, m->d_tok, m->d_tok + nt, 1, &seed, 1, eps))) return rc;
  // +ε, -2ε, +ε (restore), then -lr·g with g from the two losses on the device
  const float m2e = -2.0f * eps;
  PerturbOps ops;
  std::memset(&ops, 0, sizeof(ops));
  ops.n = 4;
  ops.op[0] = PerturbOp{0, 0, 0, eps, 0.f, 0.f, 1.f};
  ops.op[1] = PerturbOp{0, 0, 0, m2e, 0.f, 0.f, 1.f};
  ops.op[2] = PerturbOp{0, 0, 0, eps, 0.f, 0.f, 1.f};
  ops.op[3] = PerturbOp{0, 1, 0, 0.f, eps, lr, 1.f};
  if ((rc = launch_perturb(m->theta, m->P, m->masks, m->mask_words, ops, m->var_loss, m->st))) return rc;
  float l2[2];
  if ((rc = copy_losses(m, l2, 2))) return rc;
  if (loss_plus) *loss_plus = l2[0];
  if (loss_minus) *loss_minus = l2[1];
  if (proj_grad) *proj_grad = (l2[0] - l2[1]) / (2.0f * eps);
  return B2P_OK;
}

int b2p_mezo_eval(b2p_model* m, const uint16_t* tokens, const uint16_t* ctargets, int n_seq, const uint64_t* seeds,
                  int n_seeds, float eps, float* loss_pairs) {
  int rc = ready(m);
  if (rc) return rc;
  B2P_REQUIRE(loss_pairs, "null loss buffer");
  if ((rc = stage_tokens(m, tokens, ctargets, n_seq))) return rc;
  const size_t nt = (size_t)n_seq * m->cfg.seq;
  if ((rc = eval_pairs(m, m->d_tok, m->d_tok + nt, n_seq, seeds, n_seeds, eps))) return rc;
  return copy_losses(m, loss_pairs, 2 * n_seeds);
}

int b2p_mezo_eval_device(b2p_model* m, const int32_t* d_tokens, const int32_t* d_targets, int n_seq,
                         const uint64_t* seeds, int n_seeds, float eps, float* loss_pairs) {
  int rc = ready(m);
  if (rc) return rc;
  B2P_REQUIRE(d_tokens && d_targets && loss_pairs, "null argument");
  if ((rc = eval_pairs(m, d_tokens, d_targets, n_seq, seeds, n_seeds, eps))) return rc;
  return copy_losses(m, loss_pairs, 2 * n_seeds);
}

int b2p_mezo_update(b2p_model* m, const uint64_t* seeds, const float* loss_pairs, int n_seeds, float eps, float lr) {
  B2P_REQUIRE(m && seeds && loss_pairs, "null argument");
  B2P_REQUIRE(n_seeds >= 1 && n_seeds <= kMaxPerturbOps && n_seeds <= m->max_slots, "seed count %d out of range",
              n_seeds);
  int rc = gen_masks(m, seeds, n_seeds);
  if (rc) return rc;
  if (is_device_ptr(loss_pairs)) {
    B2P_CHECK_CUDA(cudaMemcpyAsync(m->pairs, loss_pairs, (size_t)2 * n_seeds * 4, cudaMemcpyDeviceToDevice, m->st));
  } else if ((rc = stage_copy(m, m->pairs, loss_pairs, (size_t)2 * n_seeds * 4))) {
    return rc;
  }
  PerturbOps ops;
  std::memset(&ops, 0, sizeof(ops));
  ops.n = n_seeds;
  for (int s = 0; s < n_seeds; ++s) ops.op[s] = PerturbOp{s, 1, s, 0.f, eps, lr, (float)n_seeds};
  return launch_perturb(m->theta, m->P, m->masks, m->mask_words, ops, m->pairs, m->st);
}

int b2p_model_perturb(b2p_model* m, const uint64_t* seeds, const float* scales, int n) {
  B2P_REQUIRE(m && seeds && scales, "null argument");
  B2P_REQUIRE(n >= 1 && n <= kMaxPerturbOps && n <= m->max_slots, "op count %d out of range", n);
  int rc = gen_masks(m, seeds, n);
  if (rc) return rc;
  PerturbOps ops;
  std::memset(&ops, 0, sizeof(ops));
  ops.n = n;
  for (int s = 0; s < n; ++s) ops.op[s] = PerturbOp{s, 0, 0, scales[s], 0.f, 0.f, 1.f};
  return launch_perturb(m->theta, m->P, m->masks, m->mask_words, ops, nullptr, m->st);
}

int b2p_sign_masks(b2p_model* m, const uint64_t* seeds, int n, uint32_t* out_words) {
  B2P_REQUIRE(m && seeds && out_words, "null argument");
  int rc = gen_masks(m, seeds, n);
  if (rc) return rc;
  B2P_CHECK_CUDA(cudaMemcpyAsync(out_words, m->masks, (size_t)n * m->mask_words * 4, cudaMemcpyDefault, m->st));
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  return check_device_status(m->st);
}

int b2p_model_sync(b2p_model* m) {
  B2P_REQUIRE(m, "null model");
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  return check_device_status(m->st);
}

int b2p_model_profile(b2p_model* m, int enable) {
  B2P_REQUIRE(m, "null model");
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  m->prof = enable != 0;
  m->ev_used = 0;
  m->prof_flops.clear();
  m->prof_epoch++;
  return B2P_OK;
}

int b2p_model_profile_read(b2p_model* m, double* gemm_ms, double* gemm_flops, long long* gemm_launches) {
  B2P_REQUIRE(m, "null model");
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  double ms = 0, fl = 0;
  for (size_t i = 0; i + 1 < m->ev_used; i += 2) {
    float t = 0;
    B2P_CHECK_CUDA(cudaEventElapsedTime(&t, m->ev_pool[i], m->ev_pool[i + 1]));
    ms += t;
  }
  for (double f : m->prof_flops) fl += f;
  if (gemm_ms) *gemm_ms = ms;
  if (gemm_flops) *gemm_flops = fl;
  if (gemm_launches) *gemm_launches = (long long)(m->ev_used / 2);
  return B2P_OK;
}

long long b2p_launch_count(void) { return launch_count(); }

int b2p_model_set_option(b2p_model* m, int option, int value) {
  B2P_REQUIRE(m, "null model");
  switch (option) {
    case B2P_OPT_PAIR_GEMM:
      m->use_pair = value != 0;
      return B2P_OK;
    case B2P_OPT_GRAPHS:
      m->graphs = value != 0;
      return B2P_OK;
    case B2P_OPT_TC_ATTENTION:
      m->tc_attn = value != 0;
      return B2P_OK;
    case B2P_OPT_TC_ATTENTION_BWD:
      m->tc_attn_bwd = value != 0;
      return B2P_OK;
    case B2P_OPT_PDL:
      set_pdl(value != 0);
      return B2P_OK;
    case B2P_OPT_GRAD_SCALE_LOG2:
      B2P_REQUIRE(value >= -30 && value <= 30, "gradient scale exponent %d out of range [-30, 30]", value);
      m->grad_scale_log2 = value;
      return B2P_OK;
    default:
      set_error("unknown model option %d", option);
      return B2P_ERR_ARG;
  }
}

}  // extern "C"
