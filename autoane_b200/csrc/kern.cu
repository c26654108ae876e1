// kern.cu — the Kern-level operator boundary (b2p_compile / b2p_write_input /
// b2p_eval / b2p_read_output / b2p_free).
//
// A b2p_kernel is one compiled operator of the reference's device boundary
// (training/io.h:116-260, bridge/ane_bridge.h:20-94): weights are converted to
// 16-bit and baked on the device at compile time; host I/O stays fp32
// channel-first [C, S]. On the device every operand is token-major ([S, C],
// tokens as rows), the layout of the tile engine, so a write transposes and
// narrows the host tensor in one kernel and eval ends with the transpose back.
//
// Per kind, eval issues:
//   conv1x1 / qkv_fused : [LoRA-down U = x·A^T] -> GEMM y = x·W^T (+ U·B^T) -> transpose
//   ffn_fused           : GEMM h = silu(xn·W1^T) * (xn·W3^T) -> copy x -> GEMM x += alpha·h·W2^T -> transpose
//   dyn_matmul          : GEMM y = act·W (W arrives as input 1, transposed on write) -> transpose
//   lm_head_ce          : GEMM with fused cross-entropy partials -> row reduction -> mean loss
//   dx                  : GEMM dx = [dy_0|dy_1|..]·[W_0|W_1|..] (K-concatenated) -> transpose
#include <algorithm>
#include <atomic>
#include <cstring>
#include <vector>
#include "../../include/b2p.h"
#include "engine.cuh"
#include "kernels.cuh"
#include "rng.cuh"

using namespace b2p;

namespace {

std::atomic<int> g_compile_count{0};

enum IoType : int { IO_F32 = 0, IO_I32 = 1 };

struct IoSpec {
  int C = 0, S = 0, type = IO_F32;
  size_t bytes() const { return (size_t)C * S * 4; }
};

struct LoraPart {
  bool set = false;
  int out = 0;                   // rows of B (output channels of the part)
  std::vector<float> A, B;       // host copies, [rank, ic] and [out, rank]
};

}  // namespace

struct b2p_kernel {
  b2p_op_desc d{};
  bool bf16 = false;
  int device = 0;
  cudaStream_t st = nullptr;
  int n_in = 0, n_out = 0;
  IoSpec in[3], out[1];
  int N = 0, K = 0;              // main GEMM: output columns, reduction length
  int in_col[3] = {0, 0, 0};     // column of the token-major GEMM input each host input lands in
  void* w = nullptr;             // 16-bit main weight, [N, K] K-major
  void* w2 = nullptr;            // ffn_fused: W2 [ic, hidden]
  void* x16 = nullptr;           // token-major 16-bit GEMM input
  float* xres = nullptr;         // ffn_fused: token-major fp32 residual input [S, ic]
  void* h16 = nullptr;           // ffn_fused: gate [S, hidden]
  float* y32 = nullptr;          // token-major fp32 result [S, N]
  float* stage = nullptr;        // fp32 device staging of one host input
  float* outcf = nullptr;        // channel-first fp32 result, what b2p_read_output copies
  // lm_head_ce
  int32_t* tgt = nullptr;
  float2* ce_part = nullptr;
  float* ce_tgt = nullptr;
  float* row_loss = nullptr;
  int ce_tiles = 0;
  // LoRA (conv1x1 / qkv_fused)
  int rank = 0;
  LoraPart part[3];
  int n_parts = 0;               // parts the operator has (1 or 3)
  float* theta = nullptr;        // A_0, B_0, A_1, B_1, ... (reference perturbation order)
  long long a_off[3] = {0, 0, 0}, b_off[3] = {0, 0, 0};
  long long P = 0;
  void* U = nullptr;             // [S, 64] 16-bit LoRA-down results
  uint32_t* masks = nullptr;
  long long mask_words = 0;
  SignBuffer* d_bufs = nullptr;
  int nbufs = 0;
  uint64_t* d_polys = nullptr;
  long long nchunks = 0, total_draws = 0;
  uint64_t* d_seed = nullptr;
  VariantInfo* d_var = nullptr;
  int* d_gv = nullptr;
  uint64_t seed = 0;
  float scale = 0.f;
  bool masks_valid = false;
  bool lora_dirty = false;
};

namespace {

size_t esz() { return 2; }

void release(b2p_kernel* k) {
  void* dev[] = {k->w, k->w2, k->x16, k->xres, k->h16, k->y32, k->stage, k->outcf, k->tgt, k->ce_part,
                 k->ce_tgt, k->row_loss, k->theta, k->U, k->masks, k->d_bufs, k->d_polys, k->d_seed, k->d_var,
                 k->d_gv};
  for (void* p : dev)
    if (p) cudaFree(p);
  if (k->st) cudaStreamDestroy(k->st);
}

// Uploads go through the one staging buffer; the copies and conversions are
// ordered on the handle's stream, so a later upload never overwrites staging
// that an earlier conversion still reads.

// fp32 host matrix [C, S] -> 16-bit token-major [S, C] at dst (row pitch ld), via the staging buffer.
int upload_transposed(b2p_kernel* k, const float* src, int C, int S, void* dst, int ld) {
  B2P_CHECK_CUDA(cudaMemcpyAsync(k->stage, src, (size_t)C * S * 4, cudaMemcpyHostToDevice, k->st));
  return launch_cf_to_tm16(k->stage, C, S, dst, ld, k->bf16, k->st);
}

// fp32 host matrix [rows, cols] -> 16-bit device copy of the same shape.
int upload_plain(b2p_kernel* k, const float* src, size_t n, void* dst) {
  B2P_CHECK_CUDA(cudaMemcpyAsync(k->stage, src, n * 4, cudaMemcpyHostToDevice, k->st));
  return launch_f32_to_16(k->stage, dst, (long long)n, k->bf16, k->st);
}

bool mult8(int v) { return v > 0 && v % 8 == 0; }

int validate(const b2p_op_desc& d) {
  B2P_REQUIRE(d.dtype == B2P_F16 || d.dtype == B2P_BF16, "dtype must be B2P_F16 or B2P_BF16");
  B2P_REQUIRE(d.seq >= 1, "seq must be positive (got %d)", d.seq);
  B2P_REQUIRE(mult8(d.ic), "ic must be a positive multiple of 8 (got %d)", d.ic);
  switch (d.kind) {
    case B2P_OP_CONV1X1:
    case B2P_OP_DYN_MATMUL:
      B2P_REQUIRE(mult8(d.oc), "oc must be a positive multiple of 8 (got %d)", d.oc);
      return B2P_OK;
    case B2P_OP_QKV_FUSED:
      B2P_REQUIRE(mult8(d.q_dim) && mult8(d.kv_dim), "q_dim / kv_dim must be positive multiples of 8");
      return B2P_OK;
    case B2P_OP_FFN_FUSED:
      B2P_REQUIRE(d.hidden > 0 && d.hidden % 128 == 0, "hidden must be a positive multiple of 128 (got %d)",
                  d.hidden);
      return B2P_OK;
    case B2P_OP_LM_HEAD_CE:
      B2P_REQUIRE(d.oc >= 1, "vocabulary size must be positive");
      return B2P_OK;
    case B2P_OP_DX:
      B2P_REQUIRE(d.n_parts >= 1 && d.n_parts <= 3, "dx needs 1..3 weight parts (got %d)", d.n_parts);
      for (int i = 0; i < d.n_parts; ++i)
        B2P_REQUIRE(mult8(d.part_oc[i]), "part_oc[%d] must be a positive multiple of 8", i);
      return B2P_OK;
  }
  set_error("unknown op kind %d", d.kind);
  return B2P_ERR_ARG;
}

// Weight tensors b2p_compile reads for an op kind.
int n_weights(const b2p_op_desc& d) {
  switch (d.kind) {
    case B2P_OP_QKV_FUSED:
    case B2P_OP_FFN_FUSED: return 3;
    case B2P_OP_DYN_MATMUL: return 0;
    case B2P_OP_DX: return d.n_parts;
    default: return 1;
  }
}

size_t max_io_bytes(const b2p_kernel* k) {
  size_t m = 0;
  for (int i = 0; i < k->n_in; ++i) m = std::max(m, k->in[i].bytes());
  m = std::max(m, k->out[0].bytes());
  return m;
}

int build(b2p_kernel* k, const float* const* wts) {
  const b2p_op_desc& d = k->d;
  const int S = d.seq, IC = d.ic;
  const size_t e = esz();
  k->out[0].S = S;
  switch (d.kind) {
    case B2P_OP_CONV1X1:
      k->N = d.oc; k->K = IC; k->n_in = 1; k->n_parts = 1;
      k->in[0] = {IC, S, IO_F32};
      k->out[0].C = d.oc;
      k->part[0].out = d.oc;
      break;
    case B2P_OP_QKV_FUSED:
      k->N = d.q_dim + 2 * d.kv_dim; k->K = IC; k->n_in = 1; k->n_parts = 3;
      k->in[0] = {IC, S, IO_F32};
      k->out[0].C = k->N;
      k->part[0].out = d.q_dim;
      k->part[1].out = d.kv_dim;
      k->part[2].out = d.kv_dim;
      break;
    case B2P_OP_FFN_FUSED:
      k->N = 2 * d.hidden; k->K = IC; k->n_in = 2;
      k->in[0] = {IC, S, IO_F32};
      k->in[1] = {IC, S, IO_F32};
      k->out[0].C = IC;
      break;
    case B2P_OP_DYN_MATMUL:
      k->N = d.oc; k->K = IC; k->n_in = 2;
      k->in[0] = {IC, S, IO_F32};
      k->in[1] = {IC, d.oc, IO_F32};
      k->out[0].C = d.oc;
      break;
    case B2P_OP_LM_HEAD_CE:
      k->N = d.oc; k->K = IC; k->n_in = 2;
      k->in[0] = {IC, S, IO_F32};
      k->in[1] = {1, S, IO_I32};
      k->out[0].C = 1;
      k->out[0].S = 1;
      break;
    case B2P_OP_DX: {
      int koc = 0;
      for (int i = 0; i < d.n_parts; ++i) {
        k->in[i] = {d.part_oc[i], S, IO_F32};
        k->in_col[i] = koc;
        koc += d.part_oc[i];
      }
      k->N = IC; k->K = koc; k->n_in = d.n_parts;
      k->out[0].C = IC;
      break;
    }
  }
  k->n_out = 1;
  const int nw = n_weights(d);
  for (int i = 0; i < nw; ++i) B2P_REQUIRE(wts && wts[i], "weight %d of %d is NULL", i, nw);
  // device buffers
  size_t wbytes = (size_t)k->N * k->K * e;
  if (d.kind == B2P_OP_DYN_MATMUL) wbytes = 0;  // the weight is part of x16
  if (wbytes) B2P_CHECK_CUDA(cudaMalloc(&k->w, wbytes));
  const size_t xrows = d.kind == B2P_OP_DYN_MATMUL ? (size_t)S + d.oc : (size_t)S;
  B2P_CHECK_CUDA(cudaMalloc(&k->x16, xrows * k->K * e));
  B2P_CHECK_CUDA(cudaMemset(k->x16, 0, xrows * k->K * e));
  // staging holds one host tensor in fp32: an input, or the largest single weight upload
  size_t stage = max_io_bytes(k);
  if (d.kind == B2P_OP_FFN_FUSED) stage = std::max(stage, (size_t)d.hidden * IC * 4);
  else stage = std::max(stage, wbytes * 2);
  B2P_CHECK_CUDA(cudaMalloc(&k->stage, stage));
  B2P_CHECK_CUDA(cudaMalloc(&k->outcf, k->out[0].bytes()));
  B2P_CHECK_CUDA(cudaMemset(k->outcf, 0, k->out[0].bytes()));
  if (d.kind != B2P_OP_LM_HEAD_CE) B2P_CHECK_CUDA(cudaMalloc(&k->y32, (size_t)S * k->N * 4));
  int rc = B2P_OK;
  switch (d.kind) {
    case B2P_OP_CONV1X1:
      rc = upload_plain(k, wts[0], (size_t)d.oc * IC, k->w);
      break;
    case B2P_OP_QKV_FUSED: {
      // stacked [Wq; Wk; Wv] rows: one GEMM, outputs channel-stacked like the reference's concat
      char* w = static_cast<char*>(k->w);
      if (!(rc = upload_plain(k, wts[0], (size_t)d.q_dim * IC, w)))
        if (!(rc = upload_plain(k, wts[1], (size_t)d.kv_dim * IC, w + (size_t)d.q_dim * IC * e)))
          rc = upload_plain(k, wts[2], (size_t)d.kv_dim * IC, w + (size_t)(d.q_dim + d.kv_dim) * IC * e);
      break;
    }
    case B2P_OP_FFN_FUSED: {
      // W1/W3 interleaved in 128-row blocks (the SwiGLU epilogue pairs h1 and h3 columns of a 256-wide tile)
      const int H = d.hidden;
      B2P_CHECK_CUDA(cudaMalloc(&k->w2, (size_t)IC * H * e));
      B2P_CHECK_CUDA(cudaMalloc(&k->xres, (size_t)S * IC * 4));
      B2P_CHECK_CUDA(cudaMalloc(&k->h16, (size_t)S * H * e));
      char* w = static_cast<char*>(k->w);
      for (int b = 0; b < H / 128 && !rc; ++b) {
        rc = upload_plain(k, wts[0] + (size_t)b * 128 * IC, (size_t)128 * IC, w + (size_t)(2 * b) * 128 * IC * e);
        if (!rc)
          rc = upload_plain(k, wts[1] + (size_t)b * 128 * IC, (size_t)128 * IC,
                            w + (size_t)(2 * b + 1) * 128 * IC * e);
      }
      if (!rc) rc = upload_plain(k, wts[2], (size_t)IC * H, k->w2);
      break;
    }
    case B2P_OP_DYN_MATMUL:
      break;
    case B2P_OP_LM_HEAD_CE: {
      rc = upload_plain(k, wts[0], (size_t)d.oc * IC, k->w);
      k->ce_tiles = (d.oc + 255) / 256;
      B2P_CHECK_CUDA(cudaMalloc(&k->tgt, (size_t)S * 4));
      B2P_CHECK_CUDA(cudaMemset(k->tgt, 0xff, (size_t)S * 4));  // -1: no target until written
      B2P_CHECK_CUDA(cudaMalloc(&k->ce_part, (size_t)S * 2 * k->ce_tiles * sizeof(float2)));
      B2P_CHECK_CUDA(cudaMalloc(&k->ce_tgt, (size_t)S * 4));
      B2P_CHECK_CUDA(cudaMalloc(&k->row_loss, (size_t)S * 4));
      break;
    }
    case B2P_OP_DX:
      // W_i [oc_i, ic] -> columns [in_col[i], in_col[i] + oc_i) of W^T [ic, K]
      for (int i = 0; i < d.n_parts && !rc; ++i) {
        rc = upload_transposed(k, wts[i], d.part_oc[i], IC, static_cast<char*>(k->w) + (size_t)k->in_col[i] * e,
                               k->K);
      }
      break;
  }
  if (rc) return rc;
  B2P_CHECK_CUDA(cudaStreamSynchronize(k->st));
  return B2P_OK;
}

// Rebuild the trainable adapter copy and the sign plan after b2p_set_lora.
int rebuild_lora(b2p_kernel* k) {
  for (void** p : {(void**)&k->theta, (void**)&k->masks, (void**)&k->d_bufs, (void**)&k->d_polys})
    if (*p) {
      B2P_CHECK_CUDA(cudaFree(*p));
      *p = nullptr;
    }
  k->P = 0;
  k->masks_valid = false;
  k->lora_dirty = false;
  int active = 0;
  for (int i = 0; i < k->n_parts; ++i) active += k->part[i].set;
  if (!active) return B2P_OK;
  std::vector<float> th;
  std::vector<long long> sizes;
  for (int i = 0; i < k->n_parts; ++i) {
    const LoraPart& p = k->part[i];
    if (!p.set) continue;
    k->a_off[i] = (long long)th.size();
    th.insert(th.end(), p.A.begin(), p.A.end());
    k->b_off[i] = (long long)th.size();
    th.insert(th.end(), p.B.begin(), p.B.end());
    sizes.push_back((long long)p.A.size());
    sizes.push_back((long long)p.B.size());
  }
  k->P = (long long)th.size();
  B2P_CHECK_CUDA(cudaMalloc(&k->theta, th.size() * 4));
  B2P_CHECK_CUDA(cudaMemcpy(k->theta, th.data(), th.size() * 4, cudaMemcpyHostToDevice));
  SignPlan plan = make_sign_plan(sizes);
  if (!plan.valid) {
    set_error("xoshiro jump polynomial could not be established");
    return B2P_ERR_STATE;
  }
  k->nbufs = (int)plan.bufs.size();
  k->nchunks = plan.nchunks;
  k->total_draws = plan.total_draws;
  k->mask_words = (k->P + 31) / 32;
  B2P_CHECK_CUDA(cudaMalloc(&k->masks, (size_t)k->mask_words * 4));
  B2P_CHECK_CUDA(cudaMalloc(&k->d_bufs, plan.bufs.size() * sizeof(SignBuffer)));
  B2P_CHECK_CUDA(cudaMalloc(&k->d_polys, plan.polys.size() * 8));
  B2P_CHECK_CUDA(cudaMemcpy(k->d_bufs, plan.bufs.data(), plan.bufs.size() * sizeof(SignBuffer),
                            cudaMemcpyHostToDevice));
  B2P_CHECK_CUDA(cudaMemcpy(k->d_polys, plan.polys.data(), plan.polys.size() * 8, cudaMemcpyHostToDevice));
  return B2P_OK;
}

int lora_active(const b2p_kernel* k) {
  int n = 0;
  for (int i = 0; i < k->n_parts; ++i) n += k->part[i].set;
  return n;
}

// y32 = x16 · W^T (+ LoRA), the conv1x1 / qkv_fused / dyn_matmul / dx GEMM.
int run_projection(b2p_kernel* k, const void* W) {
  const int S = k->d.seq;
  EpiParams ep;
  std::memset(&ep, 0, sizeof(ep));
  ep.M = S;
  ep.N = k->N;
  const int active = lora_active(k);
  if (!active) {
    DeviceCtx* c = nullptr;
    int rc = ctx_get(&c);
    if (rc) return rc;
    if (const int route = small_gemm_route(EPI_F32, S, k->N, k->K, c->num_sms))
      return launch_gemm_small(route, EPI_F32, k->bf16, k->x16, k->K, W, k->K, S, k->N, k->K, k->y32, k->N, k->st);
    if (S >= 2 * kBM && pair_supported(EPI_F32, S, k->N, ep))
      return launch_gemm_pair(EPI_F32, k->bf16, k->x16, k->K, W, k->K, S, k->N, k->K, k->y32, k->N, nullptr, ep,
                              k->st);
    return launch_gemm(pick_bn(k->N, EPI_F32), EPI_F32, k->bf16, k->x16, k->K, W, k->K, S, k->N, k->K, k->y32, k->N,
                       nullptr, ep, k->st);
  }
  if (active != k->n_parts) {
    set_error("LoRA is set on %d of the operator's %d parts; set all or none", active, k->n_parts);
    return B2P_ERR_STATE;
  }
  int rc;
  if (k->lora_dirty && (rc = rebuild_lora(k))) return rc;
  VariantInfo vi;
  vi.mask_slot = 0;
  vi.mode = k->scale != 0.f ? 1 : 0;
  vi.s1 = k->scale;
  vi.s2 = 0.f;
  if (vi.mode && !k->masks_valid) {
    B2P_CHECK_CUDA(cudaMemcpyAsync(k->d_seed, &k->seed, 8, cudaMemcpyHostToDevice, k->st));
    if ((rc = launch_sign_masks(k->d_bufs, k->nbufs, k->d_polys, k->nchunks, k->total_draws, k->mask_words,
                                k->d_seed, 1, k->masks, k->st)))
      return rc;
    k->masks_valid = true;
  }
  B2P_CHECK_CUDA(cudaMemcpyAsync(k->d_var, &vi, sizeof(vi), cudaMemcpyHostToDevice, k->st));
  PerturbCtx pc;
  pc.theta = k->theta;
  pc.masks = k->masks;
  pc.mask_words = k->mask_words;
  pc.variants = k->d_var;
  pc.group_variant = k->d_gv;
  pc.group_rows = S;
  NormLoraArgs na;
  std::memset(&na, 0, sizeof(na));
  na.in = k->x16;
  na.rows = S;
  na.dim = k->d.ic;
  na.norm = 0;
  na.n_a = k->n_parts;
  for (int i = 0; i < k->n_parts; ++i) na.a_off[i] = k->a_off[i];
  na.rank = k->rank;
  na.U = k->U;
  na.u_col = 0;
  na.pc = pc;
  if ((rc = launch_norm_lora(na, k->bf16, k->st))) return rc;
  ep.has_lora = 1;
  LoraEpi& le = ep.lora;
  le.theta = k->theta;
  le.masks = k->masks;
  le.mask_words = k->mask_words;
  le.variants = k->d_var;
  le.group_variant = k->d_gv;
  le.group_rows = S;
  le.n_groups = 1;
  le.n_variants = 1;
  le.rank = k->rank;
  le.nseg = k->n_parts;
  int col = 0;
  for (int i = 0; i < k->n_parts; ++i) {
    le.seg_start[i] = col;
    le.seg_boff[i] = k->b_off[i];
    le.seg_ucol[i] = 16 * i;
    col += k->part[i].out;
  }
  le.seg_start[k->n_parts] = col;
  int bn = pick_bn(k->N, EPI_F32);
  if (k->n_parts > 1) {
    // every segment boundary must fall on a tile edge
    bn = 0;
    for (int cand : {256, 192, 160, 128})
      if (!bn && k->part[0].out % cand == 0 && (k->part[0].out + k->part[1].out) % cand == 0) bn = cand;
    if (!bn) {
      set_error("q_dim %d / kv_dim %d have no common LoRA tile width (128, 160, 192 or 256)", k->part[0].out,
                k->part[1].out);
      return B2P_ERR_UNSUPPORTED;
    }
  }
  return launch_gemm(bn, EPI_F32, k->bf16, k->x16, k->K, W, k->K, S, k->N, k->K, k->y32, k->N, k->U, ep, k->st);
}

int eval_async(b2p_kernel* k) {
  const b2p_op_desc& d = k->d;
  const int S = d.seq, IC = d.ic;
  int rc = B2P_OK;
  switch (d.kind) {
    case B2P_OP_CONV1X1:
    case B2P_OP_QKV_FUSED:
    case B2P_OP_DX:
      if ((rc = run_projection(k, k->w))) return rc;
      return launch_tm_to_cf32(k->y32, k->N, true, k->bf16, k->N, S, k->outcf, k->st);
    case B2P_OP_DYN_MATMUL:
      if ((rc = run_projection(k, static_cast<const char*>(k->x16) + (size_t)S * IC * esz()))) return rc;
      return launch_tm_to_cf32(k->y32, k->N, true, k->bf16, k->N, S, k->outcf, k->st);
    case B2P_OP_FFN_FUSED: {
      const int H = d.hidden;
      EpiParams es;
      std::memset(&es, 0, sizeof(es));
      es.M = S;
      es.N = 2 * H;
      if (S >= 2 * kBM && pair_supported(EPI_SWIGLU, S, 2 * H, es))
        rc = launch_gemm_pair(EPI_SWIGLU, k->bf16, k->x16, IC, k->w, IC, S, 2 * H, IC, k->h16, H, nullptr, es, k->st);
      else
        rc = launch_gemm(256, EPI_SWIGLU, k->bf16, k->x16, IC, k->w, IC, S, 2 * H, IC, k->h16, H, nullptr, es, k->st);
      if (rc) return rc;
      // x_next = x + alpha · W2·h, accumulated into a copy so repeated evals see the same input
      B2P_CHECK_CUDA(cudaMemcpyAsync(k->y32, k->xres, (size_t)S * IC * 4, cudaMemcpyDeviceToDevice, k->st));
      EpiParams e2;
      std::memset(&e2, 0, sizeof(e2));
      e2.M = S;
      e2.N = IC;
      e2.alpha = d.res_alpha;
      if (S >= 2 * kBM && pair_supported(EPI_RESID, S, IC, e2))
        rc = launch_gemm_pair(EPI_RESID, k->bf16, k->h16, H, k->w2, H, S, IC, H, k->y32, IC, nullptr, e2, k->st);
      else
        rc = launch_gemm(pick_bn(IC, EPI_RESID), EPI_RESID, k->bf16, k->h16, H, k->w2, H, S, IC, H, k->y32, IC,
                         nullptr, e2, k->st);
      if (rc) return rc;
      return launch_tm_to_cf32(k->y32, IC, true, k->bf16, IC, S, k->outcf, k->st);
    }
    case B2P_OP_LM_HEAD_CE: {
      EpiParams ec;
      std::memset(&ec, 0, sizeof(ec));
      ec.M = S;
      ec.N = d.oc;
      ec.targets = k->tgt;
      ec.ce_part = k->ce_part;
      ec.ce_tgt = k->ce_tgt;
      ec.n_tiles_n = k->ce_tiles;
      if (S >= 2 * kBM && pair_supported(EPI_CE, S, d.oc, ec))
        rc = launch_gemm_pair(EPI_CE, k->bf16, k->x16, IC, k->w, IC, S, d.oc, IC, nullptr, 0, nullptr, ec, k->st);
      else
        rc = launch_gemm(256, EPI_CE, k->bf16, k->x16, IC, k->w, IC, S, d.oc, IC, nullptr, 0, nullptr, ec, k->st);
      if (rc) return rc;
      return launch_ce_reduce(k->ce_part, 2 * k->ce_tiles, k->ce_tgt, S, S, k->row_loss, k->outcf, k->st);
    }
  }
  set_error("unknown op kind");
  return B2P_ERR_ARG;
}

int check_kernel(const b2p_kernel* k) {
  B2P_REQUIRE(k != nullptr, "null kernel handle");
  int dev = -1;
  B2P_CHECK_CUDA(cudaGetDevice(&dev));
  B2P_REQUIRE(dev == k->device, "kernel was compiled on device %d but device %d is current", k->device, dev);
  return B2P_OK;
}

}  // namespace

extern "C" {

b2p_kernel* b2p_compile(const b2p_op_desc* desc, const float* const* weights) {
  if (!desc) {
    set_error("null descriptor");
    return nullptr;
  }
  if (validate(*desc)) return nullptr;
  DeviceCtx* ctx = nullptr;
  if (ctx_get(&ctx)) return nullptr;
  b2p_kernel* k = new b2p_kernel();
  k->d = *desc;
  k->bf16 = desc->dtype == B2P_BF16;
  k->device = ctx->device;
  int rc = B2P_OK;
  if (cudaStreamCreateWithFlags(&k->st, cudaStreamNonBlocking) != cudaSuccess) {
    set_error("cudaStreamCreate failed");
    rc = B2P_ERR_CUDA;
  }
  if (!rc) rc = build(k, weights);
  if (!rc && (desc->kind == B2P_OP_CONV1X1 || desc->kind == B2P_OP_QKV_FUSED)) {
    const size_t S = desc->seq;
    if (cudaMalloc(&k->U, S * kUCols * esz()) != cudaSuccess || cudaMemset(k->U, 0, S * kUCols * esz()) ||
        cudaMalloc(&k->d_seed, 8) || cudaMalloc(&k->d_var, sizeof(VariantInfo)) || cudaMalloc(&k->d_gv, 4) ||
        cudaMemset(k->d_gv, 0, 4)) {
      set_error("LoRA buffer allocation failed");
      rc = B2P_ERR_CUDA;
    }
  }
  if (rc) {
    cudaStreamSynchronize(k->st);
    release(k);
    delete k;
    return nullptr;
  }
  g_compile_count.fetch_add(1);
  return k;
}

size_t b2p_input_bytes(const b2p_kernel* k, int idx) {
  return (k && idx >= 0 && idx < k->n_in) ? k->in[idx].bytes() : 0;
}

size_t b2p_output_bytes(const b2p_kernel* k, int idx) {
  return (k && idx >= 0 && idx < k->n_out) ? k->out[idx].bytes() : 0;
}

int b2p_write_input(b2p_kernel* k, int idx, const void* data, size_t bytes) {
  int rc = check_kernel(k);
  if (rc) return rc;
  B2P_REQUIRE(idx >= 0 && idx < k->n_in, "input index %d out of range (%d inputs)", idx, k->n_in);
  B2P_REQUIRE(data != nullptr, "null input data");
  const IoSpec& io = k->in[idx];
  B2P_REQUIRE(bytes == io.bytes(), "input %d is %zu bytes, got %zu", idx, io.bytes(), bytes);
  if (io.type == IO_I32) {
    const int32_t* t = static_cast<const int32_t*>(data);
    for (int i = 0; i < io.S; ++i)
      B2P_REQUIRE(t[i] >= 0 && t[i] < k->d.oc, "target %d = %d outside [0, %d)", i, t[i], k->d.oc);
    B2P_CHECK_CUDA(cudaMemcpyAsync(k->tgt, data, bytes, cudaMemcpyHostToDevice, k->st));
    return B2P_OK;
  }
  return b2p_write_input_channels(k, idx, 0, io.C, static_cast<const float*>(data));
}

int b2p_write_input_channels(b2p_kernel* k, int idx, int ch_off, int channels, const float* data) {
  int rc = check_kernel(k);
  if (rc) return rc;
  B2P_REQUIRE(idx >= 0 && idx < k->n_in, "input index %d out of range (%d inputs)", idx, k->n_in);
  const IoSpec& io = k->in[idx];
  B2P_REQUIRE(io.type == IO_F32, "input %d is not an fp32 tensor", idx);
  B2P_REQUIRE(data != nullptr && channels >= 1 && ch_off >= 0 && ch_off + channels <= io.C,
              "channels [%d, %d) outside input %d's %d channels", ch_off, ch_off + channels, idx, io.C);
  const b2p_op_desc& d = k->d;
  const size_t e = esz();
  B2P_CHECK_CUDA(cudaMemcpyAsync(k->stage, data, (size_t)channels * io.S * 4, cudaMemcpyHostToDevice, k->st));
  if (d.kind == B2P_OP_FFN_FUSED && idx == 1)
    return launch_cf_to_tm32(k->stage, channels, io.S, k->xres + ch_off, d.ic, k->st);
  char* base = static_cast<char*>(k->x16);
  if (d.kind == B2P_OP_DYN_MATMUL && idx == 1) base += (size_t)d.seq * d.ic * e;  // weight rows after the tokens
  base += (size_t)(k->in_col[idx] + ch_off) * e;
  return launch_cf_to_tm16(k->stage, channels, io.S, base, k->K, k->bf16, k->st);
}

int b2p_eval_async(b2p_kernel* k) {
  int rc = check_kernel(k);
  if (rc) return rc;
  return eval_async(k);
}

int b2p_eval(b2p_kernel* k) {
  int rc = b2p_eval_async(k);
  if (rc) return rc;
  B2P_CHECK_CUDA(cudaStreamSynchronize(k->st));
  return check_device_status(k->st);
}

int b2p_read_output(b2p_kernel* k, int idx, float* data, size_t bytes) {
  int rc = check_kernel(k);
  if (rc) return rc;
  B2P_REQUIRE(idx >= 0 && idx < k->n_out, "output index %d out of range (%d outputs)", idx, k->n_out);
  B2P_REQUIRE(bytes == k->out[idx].bytes(), "output %d is %zu bytes, got %zu", idx, k->out[idx].bytes(), bytes);
  return b2p_read_output_channels(k, idx, 0, k->out[idx].C, data);
}

int b2p_read_output_channels(b2p_kernel* k, int idx, int ch_off, int channels, float* data) {
  int rc = check_kernel(k);
  if (rc) return rc;
  B2P_REQUIRE(idx >= 0 && idx < k->n_out, "output index %d out of range (%d outputs)", idx, k->n_out);
  const IoSpec& io = k->out[idx];
  B2P_REQUIRE(data != nullptr && channels >= 1 && ch_off >= 0 && ch_off + channels <= io.C,
              "channels [%d, %d) outside output %d's %d channels", ch_off, ch_off + channels, idx, io.C);
  B2P_CHECK_CUDA(cudaStreamSynchronize(k->st));
  if ((rc = check_device_status(k->st))) return rc;
  B2P_CHECK_CUDA(cudaMemcpy(data, k->outcf + (size_t)ch_off * io.S, (size_t)channels * io.S * 4,
                            cudaMemcpyDeviceToHost));
  return B2P_OK;
}

void b2p_free(b2p_kernel* k) {
  if (!k) return;
  cudaStreamSynchronize(k->st);
  release(k);
  delete k;
}

void* b2p_kernel_stream(const b2p_kernel* k) { return k ? (void*)k->st : nullptr; }

int b2p_set_lora(b2p_kernel* k, int part, const float* A, const float* B, int rank) {
  int rc = check_kernel(k);
  if (rc) return rc;
  B2P_REQUIRE(k->d.kind == B2P_OP_CONV1X1 || k->d.kind == B2P_OP_QKV_FUSED,
              "LoRA applies to conv1x1 and qkv_fused operators only");
  B2P_REQUIRE(part >= 0 && part < k->n_parts, "part %d out of range (%d parts)", part, k->n_parts);
  LoraPart& p = k->part[part];
  if (!A && !B) {
    p.set = false;
    p.A.clear();
    p.B.clear();
    k->lora_dirty = true;
    return B2P_OK;
  }
  B2P_REQUIRE(A && B, "A and B must both be given (or both NULL)");
  B2P_REQUIRE(rank == 4 || rank == 8, "LoRA rank must be 4 or 8 (got %d)", rank);
  const int ic = k->d.ic;
  B2P_REQUIRE(ic == 512 || ic == 960 || ic == 1024 || ic == 2048, "LoRA needs ic in {512, 960, 1024, 2048} (got %d)",
              ic);
  B2P_REQUIRE(k->d.seq % kBM == 0, "LoRA needs seq %% %d == 0 (got %d)", kBM, k->d.seq);
  for (int i = 0; i < k->n_parts; ++i)
    B2P_REQUIRE(i == part || !k->part[i].set || rank == k->rank, "all parts must share one rank (%d set, got %d)",
                k->rank, rank);
  k->rank = rank;
  p.A.assign(A, A + (size_t)rank * ic);
  p.B.assign(B, B + (size_t)p.out * rank);
  p.set = true;
  k->lora_dirty = true;
  return B2P_OK;
}

int b2p_set_perturb(b2p_kernel* k, uint64_t seed, float scale) {
  int rc = check_kernel(k);
  if (rc) return rc;
  B2P_REQUIRE(k->d.kind == B2P_OP_CONV1X1 || k->d.kind == B2P_OP_QKV_FUSED,
              "perturbation applies to the LoRA adapters of conv1x1 / qkv_fused operators");
  if (seed != k->seed) k->masks_valid = false;
  k->seed = seed;
  k->scale = scale;
  return B2P_OK;
}

int b2p_compile_count(void) { return g_compile_count.load(); }

void b2p_reset_compile_count(void) { g_compile_count.store(0); }

}  // extern "C"
