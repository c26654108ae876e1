/* train_mezo.c — AutoANE's MeZO training loop (training/train_mezo.m) as plain C
 * on Linux, with every forward, perturbation and optimizer step issued through
 * libb2p (include/b2p.h) on a B200.
 *
 * Modes (same flags as the reference, train_mezo.m:883-915):
 *   --lora-split [--lora-rank r] [--lora-ffn]   MeZO-LoRA-split: +eps, forward, -2eps,
 *                                               forward, +eps, update (:2938-3012)
 *   --backprop-lora                             P16: forward + backward + Adam (:1961-2136)
 * with --scratch (drand48 init, :1032-1049) or --resume <BLZT file> (:1018-1031),
 * --steps, --time, --lr, --epsilon, --seed, --data, --val-every. The host does
 * what the reference's host does: data sampling (srand48(seed + step*7919),
 * :1946-1953), vocabulary compaction (cpu_ops.h:142-166), LoRA init
 * (srand48(seed + 12345), :1056-1103), the cosine learning-rate schedules
 * (:3133-3135, :2134-2135), validation and best-checkpoint saving (:3150-3194)
 * and the final report (:3197-3226). The model runs on the device: the
 * perturbation is applied inside the kernels, so nothing is re-staged per step.
 *
 * Model sizes are chosen at run time (--model, the reference's training/models
 * headers), not at compile time; head_dim must be 64.
 * Additions for checking and scripting: --layers N (fewer layers of the chosen
 * model), --ckpt PATH, --device N, --trace (per-step scalars in C99 hex),
 * --dump-theta PATH (trainable parameters after the run, fp32),
 * --positions N (print the first N training positions and exit; no GPU).
 *
 * Build: see INTEGRATION.md (gcc -std=c11 ... -lb2p -lm).
 */
#define _GNU_SOURCE
#include <fcntl.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include "b2p.h"

/* ---- model headers (training/models/<name>.h) ---- */
typedef struct {
  const char *name, *title, *ckpt, *data;
  int dim, hidden, heads, kv_heads, hd, seq, nlayers, vocab;
  float rope_theta;
} ModelDef;

static const ModelDef MODELS[] = {
    {"smollm2_360m", "SmolLM2-360M", "ane_smollm2_360m_ckpt.bin", "../tinystories_smollm2_data00.bin", 960, 2560,
     15, 5, 64, 256, 32, 49152, 100000.0f},
    {"smollm2_135m", "SmolLM2-135M", "ane_smollm2_135m_ckpt.bin", "../tinystories_data00.bin", 576, 1536, 9, 3, 64,
     256, 30, 49152, 100000.0f},
    {"autoresearch", "autoresearch-4L-512d", "ane_autoresearch_ckpt.bin", "../tinystories_smollm2_data00.bin", 512,
     1408, 8, 2, 64, 128, 4, 49152, 10000.0f},
    {"autoresearch_1536", "autoresearch-4L-1536d", "ane_autoresearch_1536_ckpt.bin",
     "../tinystories_smollm2_data00.bin", 1536, 4224, 24, 6, 64, 256, 4, 49152, 10000.0f},
    {"autoresearch_2048", "autoresearch-4L-2048d", "ane_autoresearch_2048_ckpt.bin",
     "../tinystories_smollm2_data00.bin", 2048, 5632, 32, 8, 64, 256, 4, 49152, 10000.0f},
    {"stories110m", "Stories110M", "ane_stories110M_dyn_ckpt.bin", "../tinystories_data00.bin", 768, 2048, 12, 12,
     64, 256, 12, 32000, 10000.0f},
};

static double now_ms(void) {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return ts.tv_sec * 1e3 + ts.tv_nsec / 1e6;
}

#define CHECK(call)                                                                  \
  do {                                                                               \
    int rc_ = (call);                                                                \
    if (rc_ != B2P_OK) {                                                             \
      fprintf(stderr, "FATAL: %s failed (%d): %s\n", #call, rc_, b2p_last_error()); \
      exit(1);                                                                       \
    }                                                                                \
  } while (0)

static void* xmalloc(size_t n) {
  void* p = malloc(n ? n : 1);
  if (!p) {
    fprintf(stderr, "FATAL: out of host memory (%zu bytes)\n", n);
    exit(1);
  }
  return p;
}

/* vocab_map_build (training/cpu_ops.h:142-166): active ids in ascending order. */
typedef struct {
  int cv;
  int *full_to_compact, *compact_to_full;
} VocabMap;

static VocabMap vocab_map_build(const uint16_t* data, size_t n, int vocab) {
  VocabMap vm;
  vm.full_to_compact = (int*)xmalloc((size_t)vocab * sizeof(int));
  for (int v = 0; v < vocab; v++) vm.full_to_compact[v] = -1;
  for (size_t i = 0; i < n; i++) vm.full_to_compact[data[i]] = 0;
  int cid = 0;
  for (int v = 0; v < vocab; v++)
    if (vm.full_to_compact[v] == 0) vm.full_to_compact[v] = cid++;
  vm.cv = cid;
  vm.compact_to_full = (int*)xmalloc((size_t)(cid ? cid : 1) * sizeof(int));
  for (int v = 0; v < vocab; v++)
    if (vm.full_to_compact[v] >= 0) vm.compact_to_full[vm.full_to_compact[v]] = v;
  return vm;
}

/* Trainable layout in perturb_lora_weights order (train_mezo.m:560-588). */
typedef struct {
  long long Aq, Bq, Ak, Bk, Av, Bv, Ao, Bo, A1, B1, A2, B2, A3, B3, rms_att, rms_ffn, layer, rms_final, total;
} Layout;

static Layout make_layout(const ModelDef* md, int nlayers, int r, int ffn) {
  const long long D = md->dim, H = md->hidden, QD = (long long)md->heads * md->hd, KVD = (long long)md->kv_heads * md->hd;
  Layout l;
  memset(&l, 0, sizeof(l));
  long long o = 0;
  l.Aq = o; o += r * D;
  l.Bq = o; o += QD * r;
  l.Ak = o; o += r * D;
  l.Bk = o; o += KVD * r;
  l.Av = o; o += r * D;
  l.Bv = o; o += KVD * r;
  l.Ao = o; o += r * QD;
  l.Bo = o; o += D * r;
  if (ffn) {
    l.A1 = o; o += r * D;
    l.B1 = o; o += H * r;
    l.A2 = o; o += r * H;
    l.B2 = o; o += D * r;
    l.A3 = o; o += r * D;
    l.B3 = o; o += H * r;
  }
  l.rms_att = o; o += D;
  l.rms_ffn = o; o += D;
  l.layer = o;
  l.rms_final = nlayers * o;
  l.total = l.rms_final + D;
  return l;
}

static int file_exists(const char* p) { return access(p, R_OK) == 0; }

int main(int argc, char** argv) {
  setbuf(stdout, NULL);
  /* ---- flags (train_mezo.m:883-915) ---- */
  int from_scratch = 0, use_lora = 0, lora_split = 0, lora_ffn = 0, backprop_lora = 0, lora_rank = 8;
  float lr = 1e-5f, base_lr = 1e-5f, epsilon = 1e-3f; /* reference defaults (train_mezo.m:851-853) */
  int lr_from_cli = 0, total_steps = 999999, val_every = 500, device = 0, layers_override = 0, trace = 0;
  long positions_only = -1;
  double time_budget_sec = 0;
  long init_seed = 42;
  const char *data_path = NULL, *ckpt_load_path = NULL, *ckpt_path = NULL, *model_name = "smollm2_360m";
  const char* dump_theta = NULL;
  for (int i = 1; i < argc; i++) {
    const char* a = argv[i];
    const int more = i + 1 < argc;
    if (!strcmp(a, "--scratch")) from_scratch = 1;
    else if (!strcmp(a, "--cpu-only") || !strcmp(a, "--ane-matmul-only") || !strcmp(a, "--conv-hybrid") ||
             !strcmp(a, "--conv-fused")) {
      /* the reference's device variants; here every mode runs on the B200 */
    } else if (!strcmp(a, "--lr") && more) { lr = (float)atof(argv[++i]); base_lr = lr; lr_from_cli = 1; }
    else if (!strcmp(a, "--epsilon") && more) epsilon = (float)atof(argv[++i]);
    else if (!strcmp(a, "--steps") && more) total_steps = atoi(argv[++i]);
    else if (!strcmp(a, "--time") && more) time_budget_sec = atof(argv[++i]);
    else if (!strcmp(a, "--seed") && more) init_seed = atol(argv[++i]);
    else if (!strcmp(a, "--data") && more) data_path = argv[++i];
    else if (!strcmp(a, "--val-every") && more) val_every = atoi(argv[++i]);
    else if (!strcmp(a, "--resume") && more) ckpt_load_path = argv[++i];
    else if (!strcmp(a, "--lora")) use_lora = 1;
    else if (!strcmp(a, "--lora-split")) { use_lora = 1; lora_split = 1; }
    else if (!strcmp(a, "--lora-rank") && more) lora_rank = atoi(argv[++i]);
    else if (!strcmp(a, "--lora-ffn")) { lora_ffn = 1; if (!use_lora) { use_lora = 1; lora_split = 1; } }
    else if (!strcmp(a, "--backprop-lora")) backprop_lora = 1;
    else if (!strcmp(a, "--model") && more) model_name = argv[++i];
    else if (!strcmp(a, "--layers") && more) layers_override = atoi(argv[++i]);
    else if (!strcmp(a, "--ckpt") && more) ckpt_path = argv[++i];
    else if (!strcmp(a, "--device") && more) device = atoi(argv[++i]);
    else if (!strcmp(a, "--trace")) trace = 1;
    else if (!strcmp(a, "--dump-theta") && more) dump_theta = argv[++i];
    else if (!strcmp(a, "--positions") && more) positions_only = atol(argv[++i]);
    else if (!strcmp(a, "--fzoo") || !strcmp(a, "--pgap") || !strcmp(a, "--ff-lora") || !strcmp(a, "--dszo") ||
             !strcmp(a, "--sparse-ratio") || !strcmp(a, "--hessian-alpha") || !strcmp(a, "--probe-gradient")) {
      fprintf(stderr, "ERROR: %s is not part of this build (MeZO-LoRA-split and backprop-LoRA only)\n", a);
      return 1;
    } else {
      fprintf(stderr, "ERROR: unknown argument %s\n", a);
      return 1;
    }
  }
  const ModelDef* md = NULL;
  for (size_t k = 0; k < sizeof(MODELS) / sizeof(MODELS[0]); k++)
    if (!strcmp(MODELS[k].name, model_name)) md = &MODELS[k];
  if (!md) {
    fprintf(stderr, "ERROR: unknown --model %s\n", model_name);
    return 1;
  }
  const int NL = layers_override > 0 ? layers_override : md->nlayers;
  const int DIM = md->dim, HIDDEN = md->hidden, SEQ = md->seq, VOCAB = md->vocab;
  const int Q_DIM = md->heads * md->hd, KV_DIM = md->kv_heads * md->hd;
  if (!data_path) data_path = md->data;
  if (!ckpt_path) ckpt_path = md->ckpt;
  /* backprop-lora implies lora-split (train_mezo.m:935-939) */
  if (backprop_lora && !lora_split) { use_lora = 1; lora_split = 1; }
  if (use_lora && !lora_split) {
    /* --lora merges W + B·A on the host after every perturbation; the device applies the
       adapters split, which is the same function of the parameters */
    printf("note: --lora runs split (adapters applied beside the frozen weights)\n");
    lora_split = 1;
  }
  if (!use_lora && positions_only < 0) {
    fprintf(stderr, "ERROR: full-parameter MeZO is not part of this build; use --lora-split or --backprop-lora\n");
    return 1;
  }
  if (backprop_lora && lora_ffn) {
    fprintf(stderr, "ERROR: --backprop-lora has no FFN-adapter gradients (backprop_lora.h); drop --lora-ffn\n");
    return 1;
  }
  if (lora_rank != 4 && lora_rank != 8) {
    fprintf(stderr, "ERROR: --lora-rank must be 4 or 8\n");
    return 1;
  }

  /* ---- token data (train_mezo.m:1227-1250) ---- */
  int data_fd = open(data_path, O_RDONLY);
  if (data_fd < 0) { fprintf(stderr, "Cannot open %s\n", data_path); return 1; }
  struct stat st;
  fstat(data_fd, &st);
  size_t data_len = (size_t)st.st_size;
  if (data_len == 0 || data_len % 2 != 0) { fprintf(stderr, "FATAL: invalid data file\n"); close(data_fd); return 1; }
  uint16_t* token_data = (uint16_t*)mmap(NULL, data_len, PROT_READ, MAP_PRIVATE, data_fd, 0);
  if (token_data == MAP_FAILED) { fprintf(stderr, "mmap failed\n"); close(data_fd); return 1; }
  const size_t n_tokens = data_len / 2;
  for (size_t i = 0; i < n_tokens; i++)
    if (token_data[i] >= VOCAB) {
      fprintf(stderr, "FATAL: token[%zu]=%d >= VOCAB=%d\n", i, token_data[i], VOCAB);
      return 1;
    }
  const size_t val_start = (size_t)(n_tokens * 0.9);
  const size_t train_tokens = val_start, val_tokens = n_tokens - val_start;
  if (train_tokens < (size_t)SEQ + 2) {
    fprintf(stderr, "FATAL: training split too small (%zu tokens < SEQ+2=%d)\n", train_tokens, SEQ + 2);
    return 1;
  }
  const size_t max_pos = train_tokens - SEQ - 1;
  if (positions_only >= 0) { /* the sampling stream alone (train_mezo.m:1946-1949), no device work */
    for (long step = 0; step < positions_only; step++) {
      srand48(init_seed + step * 7919LL);
      printf("%ld %zu\n", step, (size_t)(drand48() * max_pos));
    }
    return 0;
  }

  printf("=== MeZO (Zeroth-Order) Training: %s (%d layers, GQA %d/%d) on B200 ===\n", md->title, NL, md->heads,
         md->kv_heads);
  printf("dim=%d q_dim=%d kv_dim=%d hd=%d hidden=%d seq=%d vocab=%d\n", DIM, Q_DIM, KV_DIM, md->hd, HIDDEN, SEQ,
         VOCAB);
  printf("Tokens: %zu (train: %zu, val: %zu)\n", n_tokens, train_tokens, val_tokens);
  VocabMap vm = vocab_map_build(token_data, n_tokens, VOCAB);
  printf("Vocab compaction: %d -> %d active\n", VOCAB, vm.cv);

  CHECK(b2p_init(device));
  const float res_alpha = from_scratch ? 1.0f / sqrtf(2.0f * NL) : 1.0f; /* train_mezo.m:1262 */
  b2p_model_config cfg = {DIM, HIDDEN, md->heads, md->kv_heads, md->hd, SEQ, NL, VOCAB, lora_rank, md->rope_theta,
                          res_alpha, B2P_F16, backprop_lora ? 1 : 2, lora_ffn};
  b2p_model* m = b2p_model_create(&cfg);
  if (!m) { fprintf(stderr, "FATAL: b2p_model_create: %s\n", b2p_last_error()); return 1; }
  const Layout lay = make_layout(md, NL, lora_rank, lora_ffn);
  if (b2p_model_trainable_count(m) != lay.total) {
    fprintf(stderr, "FATAL: trainable layout %lld != library's %lld\n", lay.total, b2p_model_trainable_count(m));
    return 1;
  }
  float* theta = (float*)xmalloc((size_t)lay.total * 4);
  memset(theta, 0, (size_t)lay.total * 4);

  int start_step = 0;
  int adapters_loaded = 0;
  if (ckpt_load_path) { /* mezo_load_checkpoint (train_mezo.m:746-789), via the library's BLZT reader */
    char lora_path[512];
    snprintf(lora_path, sizeof(lora_path), "%s", ckpt_path);
    char* dot = strrchr(lora_path, '.');
    if (dot) snprintf(dot, sizeof(lora_path) - (size_t)(dot - lora_path), "_lora.bin");
    adapters_loaded = backprop_lora && file_exists(lora_path);
    b2p_ckpt_header hdr;
    CHECK(b2p_ckpt_load(m, ckpt_load_path, adapters_loaded ? lora_path : NULL, vm.compact_to_full, vm.cv, 0, &hdr));
    start_step = hdr.step;
    if (lr_from_cli) printf("  (using CLI lr=%g instead of checkpoint lr)\n", lr);
    else { lr = hdr.lr; base_lr = lr; }
    printf("[RESUMED from step %d, loss=%.4f]\n", start_step, hdr.loss);
    CHECK(b2p_model_get_trainable(m, theta, lay.total));
  } else if (from_scratch) { /* train_mezo.m:1032-1049: one drand48 stream over every weight */
    printf("Initializing from scratch (seed=%ld)\n", init_seed);
    srand48(init_seed);
    const float scale_d = 1.0f / sqrtf(DIM), scale_qd = 1.0f / sqrtf(Q_DIM), scale_h = 1.0f / sqrtf(HIDDEN);
    const float res_scale = 1.0f / sqrtf(2.0f * NL);
    const size_t szq = (size_t)Q_DIM * DIM, szkv = (size_t)KV_DIM * DIM, szo = (size_t)DIM * Q_DIM,
                 sz1 = (size_t)HIDDEN * DIM, sz2 = (size_t)DIM * HIDDEN;
    float *wq = xmalloc(szq * 4), *wk = xmalloc(szkv * 4), *wv = xmalloc(szkv * 4), *wo = xmalloc(szo * 4),
          *w1 = xmalloc(sz1 * 4), *w2 = xmalloc(sz2 * 4), *w3 = xmalloc(sz1 * 4);
    for (int L = 0; L < NL; L++) {
      for (size_t i = 0; i < szq; i++) wq[i] = scale_d * (2 * drand48() - 1);
      for (size_t i = 0; i < szkv; i++) wk[i] = scale_d * (2 * drand48() - 1);
      for (size_t i = 0; i < szkv; i++) wv[i] = scale_d * (2 * drand48() - 1);
      for (size_t i = 0; i < szo; i++) wo[i] = scale_qd * res_scale * (2 * drand48() - 1);
      for (size_t i = 0; i < sz1; i++) w1[i] = scale_h * (2 * drand48() - 1);
      for (size_t i = 0; i < sz2; i++) w2[i] = scale_d * res_scale * (2 * drand48() - 1);
      for (size_t i = 0; i < sz1; i++) w3[i] = scale_h * (2 * drand48() - 1);
      CHECK(b2p_model_set_layer(m, L, wq, wk, wv, wo, w1, w2, w3));
    }
    free(wq); free(wk); free(wv); free(wo); free(w1); free(w2); free(w3);
    float* embed = xmalloc((size_t)VOCAB * DIM * 4);
    for (size_t i = 0; i < (size_t)VOCAB * DIM; i++) embed[i] = 0.02f * (2 * drand48() - 1);
    CHECK(b2p_model_set_embedding(m, embed, vm.compact_to_full, vm.cv));
    free(embed);
    for (int L = 0; L < NL; L++)
      for (int i = 0; i < 2 * DIM; i++) theta[L * lay.layer + lay.rms_att + i] = 1.0f;
    for (int i = 0; i < DIM; i++) theta[lay.rms_final + i] = 1.0f;
  } else {
    fprintf(stderr, "Must specify --scratch or --resume <path>\n");
    return 1;
  }

  /* ---- LoRA initialization (train_mezo.m:1056-1103): A ~ U(±1/sqrt(r)), B = 0 ---- */
  if (!adapters_loaded) {
    const int r = lora_rank;
    const float a_scale = 1.0f / sqrtf((float)r);
    srand48(init_seed + 12345);
    for (int L = 0; L < NL; L++) {
      float* t = theta + L * lay.layer;
      const long long blocks[4][2] = {{lay.Aq, (long long)r * DIM}, {lay.Ak, (long long)r * DIM},
                                      {lay.Av, (long long)r * DIM}, {lay.Ao, (long long)r * Q_DIM}};
      for (int b = 0; b < 4; b++)
        for (long long i = 0; i < blocks[b][1]; i++) t[blocks[b][0] + i] = a_scale * (2 * drand48() - 1);
      memset(t + lay.Bq, 0, (size_t)(lay.Ak - lay.Bq) * 4);
      memset(t + lay.Bk, 0, (size_t)(lay.Av - lay.Bk) * 4);
      memset(t + lay.Bv, 0, (size_t)(lay.Ao - lay.Bv) * 4);
      memset(t + lay.Bo, 0, (size_t)DIM * r * 4);
      if (lora_ffn) {
        const float a2_scale = 1.0f / sqrtf((float)r);
        for (long long i = 0; i < (long long)r * DIM; i++) t[lay.A1 + i] = a_scale * (2 * drand48() - 1);
        for (long long i = 0; i < (long long)r * DIM; i++) t[lay.A3 + i] = a_scale * (2 * drand48() - 1);
        for (long long i = 0; i < (long long)r * HIDDEN; i++) t[lay.A2 + i] = a2_scale * (2 * drand48() - 1);
      }
    }
    CHECK(b2p_model_set_trainable(m, theta, lay.total));
  }
  printf("LoRA: rank=%d, trainable parameters %lld (adapters on Wq, Wk, Wv, Wo%s)\n", lora_rank, lay.total,
         lora_ffn ? ", W1, W2, W3" : "");
  if (backprop_lora) printf("P16: lr=%g seed=%ld val_every=%d rank=%d\n", lr, init_seed, val_every, lora_rank);
  else printf("MeZO+LoRA: lr=%g epsilon=%g seed=%ld val_every=%d rank=%d\n", lr, epsilon, init_seed, val_every,
              lora_rank);

  /* ---- training loop (train_mezo.m:1931-3194) ---- */
  uint16_t* ctargets = (uint16_t*)xmalloc((size_t)SEQ * 2);
  uint16_t* vtok = (uint16_t*)xmalloc((size_t)10 * SEQ * 2);
  uint16_t* vtgt = (uint16_t*)xmalloc((size_t)10 * SEQ * 2);
  float best_loss = 1e30f, last_loss_plus = 0, last_loss_minus = 0;
  double total_train_ms = 0;
  int total_steps_done = 0;
  const double t_wall_start = now_ms();
  printf("\nStarting %s training...\n\n", backprop_lora ? "P16 backprop-LoRA" : "MeZO");
  for (int step = start_step; step < total_steps; step++) {
    if (time_budget_sec > 0 && step > start_step + 2) {
      const double elapsed = (now_ms() - t_wall_start) / 1000.0;
      if (elapsed >= time_budget_sec) {
        printf("Time budget %.0fs reached at step %d (%.1fs elapsed)\n", time_budget_sec, step, elapsed);
        total_steps = step;
        break;
      }
    }
    const double t_step = now_ms();
    srand48(init_seed + step * 7919LL); /* deterministic data sampling per step */
    const size_t pos = (size_t)(drand48() * max_pos);
    const uint16_t* input_tokens = token_data + pos;
    const uint16_t* target_raw = token_data + pos + 1;
    for (int t = 0; t < SEQ; t++) ctargets[t] = (uint16_t)vm.full_to_compact[target_raw[t]];
    const uint64_t mezo_seed = (uint64_t)step * 1000003ULL + (uint64_t)init_seed;
    const float lr_used = lr;
    if (backprop_lora) {
      float loss = 0;
      CHECK(b2p_p16_step(m, input_tokens, ctargets, 1, lr, &loss)); /* Adam b1 .9, b2 .95, eps 1e-8, wd 0 */
      const double step_ms = now_ms() - t_step;
      total_train_ms += step_ms;
      total_steps_done++;
      last_loss_plus = last_loss_minus = loss;
      if (step % 10 == 0 || step == start_step)
        printf("step %d  loss=%.4f  lr=%.2e  %.1fms/step\n", step, loss, lr, step_ms);
      if (trace) printf("trace step=%d pos=%zu lr=%a loss=%a\n", step, pos, lr_used, loss);
      const float progress = (float)(step - start_step) / (float)(total_steps - start_step);
      lr = base_lr * 0.5f * (1.0f + cosf(3.14159f * progress)); /* train_mezo.m:2134-2135 */
    } else {
      float lp = 0, lm = 0, g = 0;
      CHECK(b2p_mezo_step(m, input_tokens, ctargets, mezo_seed, epsilon, lr, &lp, &lm, &g));
      const float min_lr = base_lr * 0.1f; /* cosine decay, no warmup (train_mezo.m:3133-3135) */
      const float decay = (float)(step - start_step) / (float)(total_steps - start_step);
      lr = min_lr + 0.5f * (1.0f + cosf(M_PI * decay)) * (base_lr - min_lr);
      const double step_ms = now_ms() - t_step;
      total_train_ms += step_ms;
      total_steps_done++;
      last_loss_plus = lp;
      last_loss_minus = lm;
      if (step % 100 == 0 || step == start_step)
        printf("step %d  loss_plus=%.4f  loss_minus=%.4f  proj_grad=%.6f  lr=%.2e  step_ms=%.1f\n", step, lp, lm, g,
               lr, step_ms);
      if (trace)
        printf("trace step=%d pos=%zu seed=%llu lr=%a lp=%a lm=%a g=%a\n", step, pos, (unsigned long long)mezo_seed,
               lr_used, lp, lm, g);
    }
    /* validation on 10 fixed held-out windows (train_mezo.m:3150-3167), unperturbed */
    if (val_every > 0 && (step + 1) % val_every == 0 && val_tokens > (size_t)SEQ + 1) {
      srand48(999);
      for (int vb = 0; vb < 10; vb++) {
        const size_t vpos = val_start + (size_t)(drand48() * (val_tokens - SEQ - 1));
        memcpy(vtok + (size_t)vb * SEQ, token_data + vpos, (size_t)SEQ * 2);
        for (int t = 0; t < SEQ; t++) vtgt[(size_t)vb * SEQ + t] = (uint16_t)vm.full_to_compact[token_data[vpos + 1 + t]];
      }
      float gl[10], val_loss = 0;
      b2p_variant v0 = {0, 0, 0.f, 0.f};
      for (int vb = 0; vb < 10; vb++) { /* one forward per window, as DO_FORWARD_PASS per batch */
        float l = 0;
        CHECK(b2p_model_eval(m, vtok + (size_t)vb * SEQ, vtgt + (size_t)vb * SEQ, 1, &v0, 1, &l));
        gl[vb] = l;
      }
      for (int vb = 0; vb < 10; vb++) val_loss += gl[vb];
      val_loss /= 10;
      printf("  [val_loss=%.4f at step %d]\n", val_loss, step + 1);
      if (val_loss < best_loss) {
        best_loss = val_loss;
        b2p_ckpt_header h;
        memset(&h, 0, sizeof(h));
        h.step = step + 1;
        h.total_steps = total_steps;
        h.lr = lr;
        h.loss = val_loss;
        h.cum_train = total_train_ms;
        h.cum_wall = now_ms() - t_wall_start;
        h.cum_steps = total_steps_done;
        char lora_path[512];
        snprintf(lora_path, sizeof(lora_path), "%s", ckpt_path);
        char* dot = strrchr(lora_path, '.');
        if (dot) snprintf(dot, sizeof(lora_path) - (size_t)(dot - lora_path), "_lora.bin");
        else strncat(lora_path, "_lora.bin", sizeof(lora_path) - strlen(lora_path) - 1);
        CHECK(b2p_ckpt_save(m, ckpt_path, backprop_lora ? lora_path : NULL, &h));
        printf("  [ckpt saved, best_val=%.4f]\n", best_loss);
      }
    }
  }

  /* ---- final report (train_mezo.m:3197-3226) ---- */
  const double wall = now_ms() - t_wall_start;
  printf("\n=== %s Efficiency Report ===\n", backprop_lora ? "P16 Backprop-LoRA" : "MeZO");
  printf("Total steps:         %d\n", total_steps_done);
  printf("Train time:          %.0fms (%.1fms/step)\n", total_train_ms, total_train_ms / fmax(1, total_steps_done));
  printf("Wall time:           %.1fs\n", wall / 1000.0);
  printf("\n---\n");
  printf("final_loss:          %.6f\n", last_loss_plus);
  if (!backprop_lora) printf("final_loss_minus:    %.6f\n", last_loss_minus);
  printf("final_val_loss:      %.6f\n", best_loss);
  printf("training_seconds:    %.1f\n", total_train_ms / 1000.0);
  printf("total_seconds:       %.1f\n", wall / 1000.0);
  printf("avg_ms_per_step:     %.1f\n", total_train_ms / fmax(1, total_steps_done));
  printf("num_steps:           %d\n", total_steps_done);
  printf("num_params_M:        %.1f\n",
         ((double)NL * ((double)Q_DIM * DIM * 2 + 2.0 * KV_DIM * DIM + 3.0 * HIDDEN * DIM + 2.0 * DIM) + DIM +
          (double)VOCAB * DIM) / 1e6);
  printf("mode:                %s-b200-lora-split\n", backprop_lora ? "backprop-lora" : "mezo");
  if (!backprop_lora) printf("epsilon:             %g\n", epsilon);
  printf("lr:                  %g\n", lr);
  printf("lora_rank:           %d\n", lora_rank);
  if (backprop_lora) printf("backprop_lora:       true\n");
  if (dump_theta) {
    CHECK(b2p_model_get_trainable(m, theta, lay.total));
    FILE* f = fopen(dump_theta, "wb");
    if (!f || fwrite(theta, 4, (size_t)lay.total, f) != (size_t)lay.total) {
      fprintf(stderr, "FATAL: cannot write %s\n", dump_theta);
      return 1;
    }
    fclose(f);
  }
  b2p_model_free(m);
  munmap(token_data, data_len);
  close(data_fd);
  free(theta); free(ctargets); free(vtok); free(vtgt);
  free(vm.full_to_compact); free(vm.compact_to_full);
  return 0;
}
