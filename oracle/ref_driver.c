/* ref_driver.c — exports the reference's own CPU code, compiled in place from
 * the AutoANE tree (training/cpu_ops.h, training/backprop_lora.h) against the
 * shim in oracle/shim, so tests can pin the oracle restatement to it.
 * TEST INFRASTRUCTURE ONLY; built into oracle/_ref/ by oracle/build.py and
 * never linked into the product.
 *
 * Model sizes are compile-time, as in the reference: the build passes
 * -include training/models/<model>.h (training/Makefile:15-23).
 */
#include "backprop_lora.h" /* reference header: pulls cpu_ops.h (reference) + shim config.h/io.h */

int ref_dims(float* out) {
  out[0] = DIM; out[1] = HIDDEN; out[2] = HEADS; out[3] = KV_HEADS; out[4] = HD;
  out[5] = SEQ; out[6] = NLAYERS; out[7] = VOCAB; out[8] = ROPE_THETA;
  return 9;
}

void ref_rmsnorm(float* out, const float* x, const float* w, int d, int S) { rmsnorm(out, x, w, d, S); }
void ref_rmsnorm_bwd(float* dx, float* dw, const float* dy, const float* x, const float* w, int d, int S) {
  rmsnorm_bwd(dx, dw, dy, x, w, d, S);
}
void ref_rope_forward(float* x, int seq, int dim, int hd) { rope_forward_inplace(x, seq, dim, hd); }
void ref_rope_backward(float* dx, int seq, int dim, int hd) { rope_backward_inplace(dx, seq, dim, hd); }
void ref_sdpa_forward(const float* Q, const float* K, const float* V, float* out, int heads, int hd, int seq) {
  cpu_sdpa_forward(Q, K, V, out, heads, hd, seq);
}
void ref_sdpa_backward(const float* Q, const float* K, const float* V, const float* da, float* dq, float* dk,
                       float* dv, int heads, int hd, int seq) {
  cpu_sdpa_backward(Q, K, V, da, dq, dk, dv, heads, hd, seq);
}
float ref_cross_entropy(float* dlogits, const float* logits, const uint16_t* targets, int V, int S) {
  return cross_entropy_loss(dlogits, logits, targets, V, S);
}
void ref_adam(float* w, const float* g, float* m, float* v, size_t n, int t, float lr, float b1, float b2, float eps,
              float wd) {
  AdamState s = {m, v, n};
  adam_update(w, g, &s, t, lr, b1, b2, eps, wd);
}
void ref_embed_lookup(float* x, const float* embed, const uint16_t* tokens, int dim, int seq, int vocab) {
  embed_lookup(x, embed, tokens, dim, seq, vocab);
}

/* lora_addmm as written in training/train_mezo.m:694-703 (that file is
 * Objective-C and cannot be compiled here; the two calls are transcribed). */
static void ref_lora_addmm(float* out, const float* A, const float* B, const float* x, float* tmp, int out_dim,
                           int rank, int in_dim) {
  cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, rank, SEQ, in_dim, 1.0f, A, in_dim, x, SEQ, 0.0f, tmp,
              SEQ);
  cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, out_dim, SEQ, rank, 1.0f, B, rank, tmp, SEQ, 1.0f, out,
              SEQ);
}

/* DO_FORWARD_PASS, cpu_only + lora_split branch (training/train_mezo.m:1528-1699),
 * transcribed over the reference's compiled cpu_ops.h functions.
 * lora[l*8 + {0..7}] = Aq,Bq,Ak,Bk,Av,Bv,Ao,Bo of layer l; rms[l*2 + {0,1}] =
 * rms_att, rms_ffn. */
float ref_forward_loss_ffn(const float* const* Wq, const float* const* Wk, const float* const* Wv,
                           const float* const* Wo, const float* const* W1, const float* const* W2,
                           const float* const* W3, const float* const* lora, const float* const* rms,
                           const float* rms_final, const float* embed, const float* cembed, int CV, int rank,
                           float res_alpha, const uint16_t* input_toks, const uint16_t* ctargets,
                           const float* const* ffn);

float ref_forward_loss(const float* const* Wq, const float* const* Wk, const float* const* Wv,
                       const float* const* Wo, const float* const* W1, const float* const* W2,
                       const float* const* W3, const float* const* lora, const float* const* rms,
                       const float* rms_final, const float* embed, const float* cembed, int CV, int rank,
                       float res_alpha, const uint16_t* input_toks, const uint16_t* ctargets) {
  return ref_forward_loss_ffn(Wq, Wk, Wv, Wo, W1, W2, W3, lora, rms, rms_final, embed, cembed, CV, rank, res_alpha,
                              input_toks, ctargets, NULL);
}

/* The same forward with --lora-ffn (train_mezo.m:1634-1661) when ffn != NULL:
 * ffn[l*6 + {0..5}] = A1, B1, A2, B2, A3, B3 of layer l. */
float ref_forward_loss_ffn(const float* const* Wq, const float* const* Wk, const float* const* Wv,
                           const float* const* Wo, const float* const* W1, const float* const* W2,
                           const float* const* W3, const float* const* lora, const float* const* rms,
                           const float* rms_final, const float* embed, const float* cembed, int CV, int rank,
                           float res_alpha, const uint16_t* input_toks, const uint16_t* ctargets,
                           const float* const* ffn) {
  float* x_cur = (float*)safe_malloc((size_t)SEQ * DIM * 4);
  float* xnorm_buf = (float*)safe_malloc((size_t)SEQ * DIM * 4);
  float* Q = (float*)safe_malloc((size_t)SEQ * Q_DIM * 4);
  float* K = (float*)safe_malloc((size_t)SEQ * KV_DIM * 4);
  float* V = (float*)safe_malloc((size_t)SEQ * KV_DIM * 4);
  float* attn_out = (float*)safe_malloc((size_t)SEQ * Q_DIM * 4);
  float* o_out = (float*)safe_malloc((size_t)SEQ * DIM * 4);
  float* h1 = (float*)safe_malloc((size_t)SEQ * HIDDEN * 4);
  float* h3 = (float*)safe_malloc((size_t)SEQ * HIDDEN * 4);
  float* silu_out = (float*)safe_malloc((size_t)SEQ * HIDDEN * 4);
  float* k_tiled = (float*)safe_malloc((size_t)SEQ * Q_DIM * 4);
  float* v_tiled = (float*)safe_malloc((size_t)SEQ * Q_DIM * 4);
  float* logits = (float*)safe_malloc((size_t)SEQ * CV * 4);
  float* dlogits = (float*)safe_malloc((size_t)SEQ * CV * 4);
  float* lora_tmp = (float*)safe_malloc((size_t)rank * SEQ * 4);
  float loss;
  embed_lookup(x_cur, embed, input_toks, DIM, SEQ, VOCAB);
  for (int L = 0; L < NLAYERS; L++) {
    const float* const* ll = lora + (size_t)L * 8;
    rmsnorm(xnorm_buf, x_cur, rms[2 * L], DIM, SEQ);
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, Q_DIM, SEQ, DIM, 1.0f, Wq[L], DIM, xnorm_buf, SEQ, 0.0f,
                Q, SEQ);
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, KV_DIM, SEQ, DIM, 1.0f, Wk[L], DIM, xnorm_buf, SEQ,
                0.0f, K, SEQ);
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, KV_DIM, SEQ, DIM, 1.0f, Wv[L], DIM, xnorm_buf, SEQ,
                0.0f, V, SEQ);
    ref_lora_addmm(Q, ll[0], ll[1], xnorm_buf, lora_tmp, Q_DIM, rank, DIM);
    ref_lora_addmm(K, ll[2], ll[3], xnorm_buf, lora_tmp, KV_DIM, rank, DIM);
    ref_lora_addmm(V, ll[4], ll[5], xnorm_buf, lora_tmp, KV_DIM, rank, DIM);
    rope_forward_inplace(Q, SEQ, Q_DIM, HD);
    rope_forward_inplace(K, SEQ, KV_DIM, HD);
    gqa_tile_kv(k_tiled, K, SEQ);
    gqa_tile_kv(v_tiled, V, SEQ);
    cpu_sdpa_forward(Q, k_tiled, v_tiled, attn_out, HEADS, HD, SEQ);
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, DIM, SEQ, Q_DIM, 1.0f, Wo[L], Q_DIM, attn_out, SEQ, 0.0f,
                o_out, SEQ);
    ref_lora_addmm(o_out, ll[6], ll[7], attn_out, lora_tmp, DIM, rank, Q_DIM);
    vDSP_vsma(o_out, 1, &res_alpha, x_cur, 1, x_cur, 1, (vDSP_Length)(SEQ * DIM));
    rmsnorm(xnorm_buf, x_cur, rms[2 * L + 1], DIM, SEQ);
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, HIDDEN, SEQ, DIM, 1.0f, W1[L], DIM, xnorm_buf, SEQ,
                0.0f, h1, SEQ);
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, HIDDEN, SEQ, DIM, 1.0f, W3[L], DIM, xnorm_buf, SEQ,
                0.0f, h3, SEQ);
    const float* const* lf = ffn ? ffn + (size_t)L * 6 : NULL;
    if (lf) {
      ref_lora_addmm(h1, lf[0], lf[1], xnorm_buf, lora_tmp, HIDDEN, rank, DIM);
      ref_lora_addmm(h3, lf[4], lf[5], xnorm_buf, lora_tmp, HIDDEN, rank, DIM);
    }
    for (int i = 0; i < HIDDEN * SEQ; i++) {
      float s = h1[i] / (1.0f + expf(-h1[i]));
      silu_out[i] = s * h3[i];
    }
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, DIM, SEQ, HIDDEN, 1.0f, W2[L], HIDDEN, silu_out, SEQ,
                0.0f, o_out, SEQ);
    if (lf) ref_lora_addmm(o_out, lf[2], lf[3], silu_out, lora_tmp, DIM, rank, HIDDEN);
    vDSP_vsma(o_out, 1, &res_alpha, x_cur, 1, x_cur, 1, (vDSP_Length)(SEQ * DIM));
  }
  rmsnorm(xnorm_buf, x_cur, rms_final, DIM, SEQ);
  cblas_sgemm(CblasRowMajor, CblasTrans, CblasTrans, SEQ, CV, DIM, 1.0f, xnorm_buf, SEQ, cembed, DIM, 0.0f, logits,
              CV);
  loss = cross_entropy_loss(dlogits, logits, ctargets, CV, SEQ);
  free(x_cur); free(xnorm_buf); free(Q); free(K); free(V); free(attn_out); free(o_out);
  free(h1); free(h3); free(silu_out); free(k_tiled); free(v_tiled); free(logits); free(dlogits); free(lora_tmp);
  return loss;
}

/* P16 step without the optimizer, as training/train_mezo.m:1982-2087 runs it in
 * conv-fused mode (frozen base projections + split LoRA in the forward, saves
 * in BP_LayerActs), with the reference's own bp_lora_backward
 * (training/backprop_lora.h:147-288) over weights merged as lora_merge_weight
 * does (training/config.h:278-283, transcribed: it lives in the Objective-C
 * config.h). Gradient outputs: glora[l*8 + {0..7}] = dAq,dBq,dAk,dBk,dAv,dBv,dAo,dBo;
 * grms[l*2 + {0,1}] = rms_att, rms_ffn; grms_final. All are zeroed first. */
float ref_p16_grad(const float* const* Wq, const float* const* Wk, const float* const* Wv, const float* const* Wo,
                   const float* const* W1, const float* const* W2, const float* const* W3,
                   const float* const* lora, const float* const* rms, const float* rms_final, const float* embed,
                   const float* cembed, int CV, int rank, float res_alpha, const uint16_t* input_toks,
                   const uint16_t* ctargets, float* const* glora, float* const* grms, float* grms_final) {
  static BP_LayerActs acts[NLAYERS];
  for (int L = 0; L < NLAYERS; L++) acts[L] = bp_layer_acts_alloc();
  float* x_cur = (float*)safe_malloc((size_t)SEQ * DIM * 4);
  float* xnorm_buf = (float*)safe_malloc((size_t)SEQ * DIM * 4);
  float* Q = (float*)safe_malloc((size_t)SEQ * Q_DIM * 4);
  float* K = (float*)safe_malloc((size_t)SEQ * KV_DIM * 4);
  float* V = (float*)safe_malloc((size_t)SEQ * KV_DIM * 4);
  float* attn_out = (float*)safe_malloc((size_t)SEQ * Q_DIM * 4);
  float* o_out = (float*)safe_malloc((size_t)SEQ * DIM * 4);
  float* k_tiled = (float*)safe_malloc((size_t)SEQ * Q_DIM * 4);
  float* v_tiled = (float*)safe_malloc((size_t)SEQ * Q_DIM * 4);
  float* logits = (float*)safe_malloc((size_t)SEQ * CV * 4);
  float* dlogits = (float*)safe_malloc((size_t)SEQ * CV * 4);
  float* lora_tmp = (float*)safe_malloc((size_t)rank * SEQ * 4);
  float* x_pre_final = (float*)safe_malloc((size_t)SEQ * DIM * 4);
  embed_lookup(x_cur, embed, input_toks, DIM, SEQ, VOCAB);
  for (int L = 0; L < NLAYERS; L++) {
    BP_LayerActs* ac = &acts[L];
    const float* const* ll = lora + (size_t)L * 8;
    memcpy(ac->x_pre, x_cur, (size_t)DIM * SEQ * 4);
    rmsnorm(xnorm_buf, x_cur, rms[2 * L], DIM, SEQ);
    memcpy(ac->xnorm, xnorm_buf, (size_t)DIM * SEQ * 4);
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, Q_DIM, SEQ, DIM, 1.0f, Wq[L], DIM, xnorm_buf, SEQ, 0.0f,
                Q, SEQ);
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, KV_DIM, SEQ, DIM, 1.0f, Wk[L], DIM, xnorm_buf, SEQ,
                0.0f, K, SEQ);
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, KV_DIM, SEQ, DIM, 1.0f, Wv[L], DIM, xnorm_buf, SEQ,
                0.0f, V, SEQ);
    ref_lora_addmm(Q, ll[0], ll[1], xnorm_buf, lora_tmp, Q_DIM, rank, DIM);
    ref_lora_addmm(K, ll[2], ll[3], xnorm_buf, lora_tmp, KV_DIM, rank, DIM);
    ref_lora_addmm(V, ll[4], ll[5], xnorm_buf, lora_tmp, KV_DIM, rank, DIM);
    memcpy(ac->Q, Q, (size_t)Q_DIM * SEQ * 4);
    memcpy(ac->K, K, (size_t)KV_DIM * SEQ * 4);
    memcpy(ac->V, V, (size_t)KV_DIM * SEQ * 4);
    rope_forward_inplace(Q, SEQ, Q_DIM, HD);
    rope_forward_inplace(K, SEQ, KV_DIM, HD);
    gqa_tile_kv(k_tiled, K, SEQ);
    gqa_tile_kv(v_tiled, V, SEQ);
    cpu_sdpa_forward(Q, k_tiled, v_tiled, attn_out, HEADS, HD, SEQ);
    memcpy(ac->attn_out, attn_out, (size_t)Q_DIM * SEQ * 4);
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, DIM, SEQ, Q_DIM, 1.0f, Wo[L], Q_DIM, attn_out, SEQ, 0.0f,
                o_out, SEQ);
    ref_lora_addmm(o_out, ll[6], ll[7], attn_out, lora_tmp, DIM, rank, Q_DIM);
    vDSP_vsma(o_out, 1, &res_alpha, x_cur, 1, x_cur, 1, (vDSP_Length)(SEQ * DIM));
    memcpy(ac->x2, x_cur, (size_t)DIM * SEQ * 4);
    rmsnorm(xnorm_buf, x_cur, rms[2 * L + 1], DIM, SEQ);
    memcpy(ac->x2norm, xnorm_buf, (size_t)DIM * SEQ * 4);
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, HIDDEN, SEQ, DIM, 1.0f, W1[L], DIM, xnorm_buf, SEQ, 0.0f,
                ac->h1, SEQ);
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, HIDDEN, SEQ, DIM, 1.0f, W3[L], DIM, xnorm_buf, SEQ, 0.0f,
                ac->h3, SEQ);
    for (int i = 0; i < HIDDEN * SEQ; i++) {
      float s = ac->h1[i] / (1.0f + expf(-ac->h1[i]));
      ac->silu_out[i] = s * ac->h3[i];
    }
    cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, DIM, SEQ, HIDDEN, 1.0f, W2[L], HIDDEN, ac->silu_out, SEQ,
                0.0f, o_out, SEQ);
    vDSP_vsma(o_out, 1, &res_alpha, x_cur, 1, x_cur, 1, (vDSP_Length)(SEQ * DIM));
  }
  memcpy(x_pre_final, x_cur, (size_t)DIM * SEQ * 4);
  rmsnorm(xnorm_buf, x_cur, rms_final, DIM, SEQ);
  cblas_sgemm(CblasRowMajor, CblasTrans, CblasTrans, SEQ, CV, DIM, 1.0f, xnorm_buf, SEQ, cembed, DIM, 0.0f, logits,
              CV);
  const float loss = cross_entropy_loss(dlogits, logits, ctargets, CV, SEQ);

  LayerWeights lw[NLAYERS];
  LoRALayer ll[NLAYERS];
  LoRAGrads lg[NLAYERS];
  float* ga[NLAYERS];
  float* gf[NLAYERS];
  for (int L = 0; L < NLAYERS; L++) {
    const float* const* lr = lora + (size_t)L * 8;
    float* merged[4];
    const float* base[4] = {Wq[L], Wk[L], Wv[L], Wo[L]};
    const int od[4] = {Q_DIM, KV_DIM, KV_DIM, DIM}, id[4] = {DIM, DIM, DIM, Q_DIM};
    for (int p = 0; p < 4; p++) {
      merged[p] = (float*)safe_malloc((size_t)od[p] * id[p] * 4);
      memcpy(merged[p], base[p], (size_t)od[p] * id[p] * 4);
      cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasNoTrans, od[p], id[p], rank, 1.0f, lr[2 * p + 1], rank,
                  lr[2 * p], id[p], 1.0f, merged[p], id[p]);
    }
    lw[L].Wq = merged[0]; lw[L].Wk = merged[1]; lw[L].Wv = merged[2]; lw[L].Wo = merged[3];
    lw[L].W1 = (float*)W1[L]; lw[L].W2 = (float*)W2[L]; lw[L].W3 = (float*)W3[L];
    lw[L].rms_att = (float*)rms[2 * L]; lw[L].rms_ffn = (float*)rms[2 * L + 1];
    memset(&ll[L], 0, sizeof(ll[L]));
    ll[L].rank = rank;
    ll[L].Aq = (float*)lr[0]; ll[L].Bq = (float*)lr[1]; ll[L].Ak = (float*)lr[2]; ll[L].Bk = (float*)lr[3];
    ll[L].Av = (float*)lr[4]; ll[L].Bv = (float*)lr[5]; ll[L].Ao = (float*)lr[6]; ll[L].Bo = (float*)lr[7];
    float* const* g = glora + (size_t)L * 8;
    const size_t gsz[8] = {(size_t)rank * DIM, (size_t)Q_DIM * rank, (size_t)rank * DIM, (size_t)KV_DIM * rank,
                           (size_t)rank * DIM, (size_t)KV_DIM * rank, (size_t)rank * Q_DIM, (size_t)DIM * rank};
    for (int k = 0; k < 8; k++) memset(g[k], 0, gsz[k] * 4);
    lg[L].Aq = g[0]; lg[L].Bq = g[1]; lg[L].Ak = g[2]; lg[L].Bk = g[3];
    lg[L].Av = g[4]; lg[L].Bv = g[5]; lg[L].Ao = g[6]; lg[L].Bo = g[7];
    ga[L] = grms[2 * L];
    gf[L] = grms[2 * L + 1];
    memset(ga[L], 0, (size_t)DIM * 4);
    memset(gf[L], 0, (size_t)DIM * 4);
  }
  memset(grms_final, 0, (size_t)DIM * 4);
  BP_WorkBufs work = bp_work_alloc();
  bp_lora_backward(dlogits, x_pre_final, cembed, (float*)rms_final, lw, acts, ll, lg, ga, gf, grms_final, res_alpha,
                   &work, rank, CV);
  bp_work_free(&work);
  for (int L = 0; L < NLAYERS; L++) {
    free(lw[L].Wq); free(lw[L].Wk); free(lw[L].Wv); free(lw[L].Wo);
    bp_layer_acts_free(&acts[L]);
  }
  free(x_cur); free(xnorm_buf); free(Q); free(K); free(V); free(attn_out); free(o_out); free(k_tiled);
  free(v_tiled); free(logits); free(dlogits); free(lora_tmp); free(x_pre_final);
  return loss;
}

/* ref_p16_grad that also returns the projection weight gradients the reference
 * materialises before projecting them onto the adapters (work->dW_Wo, dW_q and
 * dW_kv, training/backprop_lora.h:223-270): dw receives, for L = NLAYERS-1 down
 * to 0, dW_o [DIM, Q_DIM], dW_q [Q_DIM, DIM], dW_k [KV_DIM, DIM], dW_v [KV_DIM, DIM]. */
float ref_p16_grad_dw(const float* const* Wq, const float* const* Wk, const float* const* Wv, const float* const* Wo,
                      const float* const* W1, const float* const* W2, const float* const* W3,
                      const float* const* lora, const float* const* rms, const float* rms_final, const float* embed,
                      const float* cembed, int CV, int rank, float res_alpha, const uint16_t* input_toks,
                      const uint16_t* ctargets, float* const* glora, float* const* grms, float* grms_final,
                      float* dw) {
  ref_dw_sink = dw;
  ref_dw_pos = 0;
  const float loss = ref_p16_grad(Wq, Wk, Wv, Wo, W1, W2, W3, lora, rms, rms_final, embed, cembed, CV, rank,
                                  res_alpha, input_toks, ctargets, glora, grms, grms_final);
  ref_dw_sink = 0;
  return loss;
}
