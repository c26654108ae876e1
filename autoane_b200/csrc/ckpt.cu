// ckpt.cu — the reference's checkpoint files on the host side of the library:
// BLZT v4 (CkptHdr, training/config.h:99-108) and the LORA adapter sidecar
// (train_mezo.m:791-844).
//
// BLZT v4 body, little-endian fp32 (train.m:189-208, train_mezo.m:718-742):
//   per layer: Wq Wk Wv Wo W1 W2 W3 rms_att rms_ffn, then the Adam m,v pairs in the
//   same order (Wq.m Wq.v Wk.m Wk.v ... rms_ffn.m rms_ffn.v);
//   then rms_final, its m, v; then embed [vocab, dim], its m, v.
// LORA sidecar: int magic, rank, nlayers, adam_t; per layer Aq Bq Ak Bk Av Bv Ao Bo.
//
// Files are streamed one layer at a time through host buffers; device tensors
// move with plain cudaMemcpy on the model's stream. Every read is length-checked
// (the reference's fread return values are not).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdio>
#include <cstring>
#include <memory>
#include <vector>

#include "model.cuh"

namespace b2p {
namespace {

constexpr int kMaxStep = 10000000;  // train.m:227, train_mezo.m:762

struct File {
  FILE* f = nullptr;
  ~File() {
    if (f) std::fclose(f);
  }
};

int io_fail(const char* what, const char* path) {
  set_error("%s %s", what, path);
  return B2P_ERR_IO;
}

int put(FILE* f, const void* p, size_t bytes, const char* path) {
  if (bytes && std::fwrite(p, 1, bytes, f) != bytes) return io_fail("short write to", path);
  return B2P_OK;
}

int get(FILE* f, void* p, size_t bytes, const char* path) {
  if (bytes && std::fread(p, 1, bytes, f) != bytes) return io_fail("truncated file", path);
  return B2P_OK;
}

int put_zeros(FILE* f, size_t n, const char* path) {
  static const float z[4096] = {};
  while (n) {
    const size_t k = n < 4096 ? n : 4096;
    int rc = put(f, z, k * 4, path);
    if (rc) return rc;
    n -= k;
  }
  return B2P_OK;
}

// Per-layer tensor sizes in file order.
struct Shapes {
  size_t wq, wk, wv, wo, w1, w2, w3, d;
  size_t layer_w() const { return wq + wk + wv + wo + w1 + w2 + w3 + 2 * d; }
};

Shapes shapes(const b2p_model* m) {
  const size_t D = m->cfg.dim, H = m->cfg.hidden, QD = m->q_dim, KVD = m->kv_dim;
  return Shapes{QD * D, KVD * D, KVD * D, D * QD, H * D, D * H, H * D, D};
}

size_t body_bytes(const b2p_model* m) {
  const Shapes s = shapes(m);
  const size_t D = m->cfg.dim, V = m->cfg.vocab;
  return ((size_t)m->cfg.nlayers * 3 * s.layer_w() + 3 * D + 3 * V * D) * 4;
}

float to_f32(uint16_t h, bool bf16) {
  if (bf16) {
    __nv_bfloat16_raw r;
    r.x = h;
    return __bfloat162float(__nv_bfloat16(r));
  }
  __half_raw r;
  r.x = h;
  return __half2float(__half(r));
}

// One layer of frozen weights in the reference's separate matrices (fp32).
struct LayerW {
  std::vector<float> q, k, v, o, w1, w2, w3;
  explicit LayerW(const Shapes& s) : q(s.wq), k(s.wk), v(s.wv), o(s.wo), w1(s.w1), w2(s.w2), w3(s.w3) {}
};

// Split the device layout ([Wq;Wk;Wv] stacked, W1/W3 interleaved in 128-row blocks) into
// the reference's matrices; `src` yields `n` fp32 values starting at a device-layout index.
template <typename Src>
void split_layout(const b2p_model* m, LayerW& w, Src src) {
  const size_t D = m->cfg.dim, H = m->cfg.hidden, QD = m->q_dim, KVD = m->kv_dim;
  std::vector<float> qkv((QD + 2 * KVD) * D), w13(2 * H * D);
  src(0, qkv.data(), qkv.size());
  std::memcpy(w.q.data(), qkv.data(), QD * D * 4);
  std::memcpy(w.k.data(), qkv.data() + QD * D, KVD * D * 4);
  std::memcpy(w.v.data(), qkv.data() + (QD + KVD) * D, KVD * D * 4);
  src(1, w.o.data(), w.o.size());
  src(2, w13.data(), w13.size());
  for (size_t b = 0; b < H / 128; ++b) {
    std::memcpy(w.w1.data() + b * 128 * D, w13.data() + (2 * b) * 128 * D, 128 * D * 4);
    std::memcpy(w.w3.data() + b * 128 * D, w13.data() + (2 * b + 1) * 128 * D, 128 * D * 4);
  }
  src(3, w.w2.data(), w.w2.size());
}

// The inverse: the reference's matrices into the device layout, part by part.
template <typename Dst>
void join_layout(const b2p_model* m, const LayerW& w, Dst dst) {
  const size_t D = m->cfg.dim, H = m->cfg.hidden, QD = m->q_dim, KVD = m->kv_dim;
  std::vector<float> qkv((QD + 2 * KVD) * D), w13(2 * H * D);
  std::memcpy(qkv.data(), w.q.data(), QD * D * 4);
  std::memcpy(qkv.data() + QD * D, w.k.data(), KVD * D * 4);
  std::memcpy(qkv.data() + (QD + KVD) * D, w.v.data(), KVD * D * 4);
  dst(0, qkv.data(), qkv.size());
  dst(1, w.o.data(), w.o.size());
  for (size_t b = 0; b < H / 128; ++b) {
    std::memcpy(w13.data() + (2 * b) * 128 * D, w.w1.data() + b * 128 * D, 128 * D * 4);
    std::memcpy(w13.data() + (2 * b + 1) * 128 * D, w.w3.data() + b * 128 * D, 128 * D * 4);
  }
  dst(2, w13.data(), w13.size());
  dst(3, w.w2.data(), w.w2.size());
}

// Element offset of layer `l`'s part `p` (0 qkv, 1 o, 2 w13, 3 w2) inside the per-part
// arrays that hold every layer back to back (16-bit copies and the fp32 masters alike).
size_t part_offset(const b2p_model* m, int p, int l) {
  const size_t D = m->cfg.dim, H = m->cfg.hidden, QD = m->q_dim;
  const size_t per[4] = {(size_t)m->qkv_dim * D, D * QD, 2 * H * D, D * H};
  return (size_t)l * per[p];
}

// W += sign · B·A for one [out, in] matrix: B [out, r], A [r, in] row-major. The
// product is summed over k in ascending order in fp32 and then added to W, the
// order of lora_merge_weight's sgemm with beta = 1 (training/config.h:278-283).
// No fused multiply-add: the x86-64 host build has none to contract to.
void add_ba(float* W, const float* B, const float* A, int out, int r, int in, float sign) {
  std::vector<float> acc((size_t)in);
  for (int i = 0; i < out; ++i) {
    std::fill(acc.begin(), acc.end(), 0.0f);
    for (int k = 0; k < r; ++k) {
      const float b = B[(size_t)i * r + k];
      const float* a = A + (size_t)k * in;
      for (int j = 0; j < in; ++j) {
        const float p = b * a[j];
        acc[j] = acc[j] + p;
      }
    }
    float* w = W + (size_t)i * in;
    if (sign > 0)
      for (int j = 0; j < in; ++j) w[j] = w[j] + acc[j];
    else
      for (int j = 0; j < in; ++j) w[j] = w[j] - acc[j];
  }
}

// W{q,k,v,o} ± B·A of layer l with the adapters in θ (host copy).
void merge_layer(const b2p_model* m, LayerW& w, const float* theta, int l, float sign) {
  const int D = m->cfg.dim, QD = m->q_dim, KVD = m->kv_dim, r = m->cfg.rank;
  const float* t = theta + (size_t)l * m->layer_size;
  add_ba(w.q.data(), t + m->oBq, t + m->oAq, QD, r, D, sign);
  add_ba(w.k.data(), t + m->oBk, t + m->oAk, KVD, r, D, sign);
  add_ba(w.v.data(), t + m->oBv, t + m->oAv, KVD, r, D, sign);
  add_ba(w.o.data(), t + m->oBo, t + m->oAo, D, r, QD, sign);
}

int check_header(const b2p_model* m, const b2p_ckpt_header& h, const char* path) {
  if (h.magic != B2P_CKPT_MAGIC || h.version != B2P_CKPT_VERSION) {
    set_error("%s is not a BLZT v4 checkpoint (magic 0x%08X, version %d)", path, (unsigned)h.magic, h.version);
    return B2P_ERR_ARG;
  }
  if (h.step < 0 || h.step > kMaxStep || h.adam_t < 0 || h.adam_t > kMaxStep) {
    set_error("%s has an invalid step (%d) or adam_t (%d)", path, h.step, h.adam_t);
    return B2P_ERR_ARG;
  }
  if (!m) return B2P_OK;
  const auto& c = m->cfg;
  if (h.n_layers != c.nlayers || h.dim != c.dim || h.vocab_size != c.vocab || h.hidden_dim != c.hidden ||
      h.seq_len != c.seq || h.n_heads != c.heads || h.kv_heads != c.kv_heads || h.head_dim != c.head_dim ||
      h.q_dim != m->q_dim) {
    set_error("%s was written for %dL/%dd/%dv/%dh/%dseq/%dq/%dkv/%dhd/%dqd, the model is "
              "%dL/%dd/%dv/%dh/%dseq/%dq/%dkv/%dhd/%dqd",
              path, h.n_layers, h.dim, h.vocab_size, h.hidden_dim, h.seq_len, h.n_heads, h.kv_heads, h.head_dim,
              h.q_dim, c.nlayers, c.dim, c.vocab, c.hidden, c.seq, c.heads, c.kv_heads, c.head_dim, m->q_dim);
    return B2P_ERR_ARG;
  }
  return B2P_OK;
}

int read_header(const char* path, b2p_ckpt_header* h, File* keep) {
  B2P_REQUIRE(path && h, "null argument");
  static_assert(sizeof(b2p_ckpt_header) == 96, "CkptHdr is 96 bytes");
  File local;
  File* fp = keep ? keep : &local;
  fp->f = std::fopen(path, "rb");
  if (!fp->f) return io_fail("cannot open", path);
  return get(fp->f, h, sizeof(*h), path);
}

long long file_size(FILE* f) {
  const long pos = std::ftell(f);
  std::fseek(f, 0, SEEK_END);
  const long long n = std::ftell(f);
  std::fseek(f, pos, SEEK_SET);
  return n;
}

int d2h(b2p_model* m, void* dst, const void* src, size_t bytes) {
  B2P_CHECK_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, m->st));
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  return B2P_OK;
}

int h2d(b2p_model* m, void* dst, const void* src, size_t bytes) {
  B2P_CHECK_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, m->st));
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  return B2P_OK;
}

void* part16(const b2p_model* m, int p) {
  void* base[4] = {m->wqkv, m->wo, m->w13, m->w2};
  return base[p];
}

// The LORA sidecar: adapters of θ (host copy) and the Adam step count.
int write_sidecar(const b2p_model* m, const char* path, const float* theta, int adam_t) {
  File f;
  f.f = std::fopen(path, "wb");
  if (!f.f) return io_fail("cannot write", path);
  const int head[4] = {B2P_LORA_MAGIC, m->cfg.rank, m->cfg.nlayers, adam_t};
  int rc = put(f.f, head, sizeof(head), path);
  // Aq..Bo are the first eight blocks of each layer's trainable block, in file order (the
  // sidecar holds the attention adapters only, as lora_save_checkpoint writes it)
  const size_t n = (size_t)(m->oBo + (long long)m->cfg.dim * m->cfg.rank);
  for (int l = 0; l < m->cfg.nlayers && !rc; ++l) rc = put(f.f, theta + (size_t)l * m->layer_size, n * 4, path);
  if (!rc && std::fflush(f.f) != 0) rc = io_fail("cannot flush", path);
  return rc;
}

int read_sidecar(const b2p_model* m, const char* path, float* theta, int* adam_t) {
  File f;
  f.f = std::fopen(path, "rb");
  if (!f.f) return io_fail("cannot open LoRA sidecar", path);
  int head[4];
  int rc = get(f.f, head, sizeof(head), path);
  if (rc) return rc;
  if (head[0] != B2P_LORA_MAGIC) {
    set_error("%s is not a LORA sidecar (magic 0x%08X)", path, (unsigned)head[0]);
    return B2P_ERR_ARG;
  }
  if (head[1] != m->cfg.rank || head[2] != m->cfg.nlayers) {
    set_error("LoRA sidecar %s has rank %d / %d layers, the model rank %d / %d layers", path, head[1], head[2],
              m->cfg.rank, m->cfg.nlayers);
    return B2P_ERR_ARG;
  }
  if (head[3] < 0 || head[3] > kMaxStep) {
    set_error("LoRA sidecar %s has an invalid adam_t %d", path, head[3]);
    return B2P_ERR_ARG;
  }
  const size_t n = (size_t)(m->oBo + (long long)m->cfg.dim * m->cfg.rank);
  if (file_size(f.f) != (long long)(16 + (size_t)m->cfg.nlayers * n * 4))
    return io_fail("wrong size for a LoRA sidecar of this model:", path);
  for (int l = 0; l < m->cfg.nlayers && !rc; ++l) rc = get(f.f, theta + (size_t)l * m->layer_size, n * 4, path);
  *adam_t = head[3];
  return rc;
}

int save(b2p_model* m, const char* path, const char* lora_path, const b2p_ckpt_header* hin) {
  B2P_REQUIRE(m && path, "null argument");
  int rc = model_ready(m);
  if (rc) return rc;
  TrainView tv;
  if ((rc = p16_view(m, false, &tv))) return rc;
  const auto& c = m->cfg;
  const Shapes sh = shapes(m);
  const size_t D = c.dim, V = c.vocab;
  std::vector<float> theta((size_t)m->P);
  if ((rc = d2h(m, theta.data(), m->theta, theta.size() * 4))) return rc;

  b2p_ckpt_header h;
  std::memset(&h, 0, sizeof(h));
  if (hin) h = *hin;
  h.magic = B2P_CKPT_MAGIC;
  h.version = B2P_CKPT_VERSION;
  h.n_layers = c.nlayers;
  h.vocab_size = c.vocab;
  h.dim = c.dim;
  h.hidden_dim = c.hidden;
  h.n_heads = c.heads;
  h.seq_len = c.seq;
  h.kv_heads = c.kv_heads;
  h.head_dim = c.head_dim;
  h.q_dim = m->q_dim;
  h.adam_t = tv.full ? *tv.full_t : 0;  // the MeZO writer stores zero Adam slots and t 0
  if (lora_path && (rc = write_sidecar(m, lora_path, theta.data(), tv.adam_t ? *tv.adam_t : 0))) return rc;

  File f;
  f.f = std::fopen(path, "wb");
  if (!f.f) return io_fail("cannot write", path);
  if ((rc = put(f.f, &h, sizeof(h), path))) return rc;
  const size_t e = model_esz(m);
  LayerW w(sh), am(sh), av(sh);
  std::vector<uint16_t> h16;
  std::vector<float> rms_m(2 * D), rms_v(2 * D);
  for (int l = 0; l < c.nlayers; ++l) {
    int err = B2P_OK;
    if (tv.full) {
      const float* parts[4] = {tv.mw + tv.o_qkv, tv.mw + tv.o_o, tv.mw + tv.o_13, tv.mw + tv.o_2};
      auto from = [&](const float* const* base, LayerW& dst) {
        split_layout(m, dst, [&](int p, float* out, size_t n) {
          if (!err) err = d2h(m, out, base[p] + part_offset(m, p, l), n * 4);
        });
      };
      from(parts, w);
      const float* pm[4] = {tv.am_w + tv.o_qkv, tv.am_w + tv.o_o, tv.am_w + tv.o_13, tv.am_w + tv.o_2};
      const float* pv[4] = {tv.av_w + tv.o_qkv, tv.av_w + tv.o_o, tv.av_w + tv.o_13, tv.av_w + tv.o_2};
      from(pm, am);
      from(pv, av);
      const size_t ro = (size_t)l * m->layer_size + m->oRa;  // rms_att, rms_ffn adjacent
      if (!err) err = d2h(m, rms_m.data(), tv.adam_m + ro, 2 * D * 4);
      if (!err) err = d2h(m, rms_v.data(), tv.adam_v + ro, 2 * D * 4);
    } else {
      split_layout(m, w, [&](int p, float* out, size_t n) {
        if (err) return;
        h16.resize(n);
        err = d2h(m, h16.data(), static_cast<const char*>(part16(m, p)) + part_offset(m, p, l) * e, n * e);
        for (size_t i = 0; i < n && !err; ++i) out[i] = to_f32(h16[i], m->bf16);
      });
      if (lora_path) merge_layer(m, w, theta.data(), l, +1.0f);
    }
    if (err) return err;
    const float* rms = theta.data() + (size_t)l * m->layer_size + m->oRa;
    const std::vector<float>* mats[7] = {&w.q, &w.k, &w.v, &w.o, &w.w1, &w.w2, &w.w3};
    for (auto* t : mats)
      if ((rc = put(f.f, t->data(), t->size() * 4, path))) return rc;
    if ((rc = put(f.f, rms, 2 * D * 4, path))) return rc;
    if (tv.full) {
      const std::vector<float>* mm[7] = {&am.q, &am.k, &am.v, &am.o, &am.w1, &am.w2, &am.w3};
      const std::vector<float>* vv[7] = {&av.q, &av.k, &av.v, &av.o, &av.w1, &av.w2, &av.w3};
      for (int i = 0; i < 7; ++i) {
        if ((rc = put(f.f, mm[i]->data(), mm[i]->size() * 4, path))) return rc;
        if ((rc = put(f.f, vv[i]->data(), vv[i]->size() * 4, path))) return rc;
      }
      for (int i = 0; i < 2; ++i) {
        if ((rc = put(f.f, rms_m.data() + i * D, D * 4, path))) return rc;
        if ((rc = put(f.f, rms_v.data() + i * D, D * 4, path))) return rc;
      }
    } else if ((rc = put_zeros(f.f, 2 * sh.layer_w(), path))) {
      return rc;
    }
  }
  if ((rc = put(f.f, theta.data() + m->oRfinal, D * 4, path))) return rc;
  std::vector<float> buf(V * D);
  if (tv.full) {
    if ((rc = d2h(m, rms_m.data(), tv.adam_m + m->oRfinal, D * 4))) return rc;
    if ((rc = d2h(m, rms_v.data(), tv.adam_v + m->oRfinal, D * 4))) return rc;
    if ((rc = put(f.f, rms_m.data(), D * 4, path)) || (rc = put(f.f, rms_v.data(), D * 4, path))) return rc;
  } else if ((rc = put_zeros(f.f, 2 * D, path))) {
    return rc;
  }
  if ((rc = d2h(m, buf.data(), m->embed, V * D * 4))) return rc;
  if ((rc = put(f.f, buf.data(), V * D * 4, path))) return rc;
  if (tv.full) {
    if ((rc = d2h(m, buf.data(), tv.am_e, V * D * 4)) || (rc = put(f.f, buf.data(), V * D * 4, path))) return rc;
    if ((rc = d2h(m, buf.data(), tv.av_e, V * D * 4)) || (rc = put(f.f, buf.data(), V * D * 4, path))) return rc;
  } else if ((rc = put_zeros(f.f, 2 * V * D, path))) {
    return rc;
  }
  if (std::fflush(f.f) != 0) return io_fail("cannot flush", path);
  return B2P_OK;
}

int load(b2p_model* m, const char* path, const char* lora_path, const int32_t* c2f, int cv, int full,
         b2p_ckpt_header* hout) {
  B2P_REQUIRE(m && path, "null argument");
  const auto& c = m->cfg;
  B2P_REQUIRE(c2f || !m->h_c2f.empty(), "no compact vocabulary map: pass compact_to_full or set the embedding first");
  if (c2f) {
    B2P_REQUIRE(cv >= 1 && cv <= c.vocab, "compact vocab %d out of range", cv);
  }
  File f;
  b2p_ckpt_header h;
  int rc = read_header(path, &h, &f);
  if (rc) return rc;
  if ((rc = check_header(m, h, path))) return rc;
  if (file_size(f.f) < (long long)(sizeof(h) + body_bytes(m)))
    return io_fail("file too short for this model's shapes:", path);
  TrainView tv;
  if ((rc = p16_view(m, full != 0, &tv))) return rc;
  const Shapes sh = shapes(m);
  const size_t D = c.dim, V = c.vocab;
  std::vector<float> theta((size_t)m->P);
  if ((rc = d2h(m, theta.data(), m->theta, theta.size() * 4))) return rc;
  int sidecar_t = 0;
  if (lora_path && (rc = read_sidecar(m, lora_path, theta.data(), &sidecar_t))) return rc;

  LayerW w(sh), am(sh), av(sh);
  std::vector<float> skip;
  for (int l = 0; l < c.nlayers; ++l) {
    std::vector<float>* mats[7] = {&w.q, &w.k, &w.v, &w.o, &w.w1, &w.w2, &w.w3};
    for (auto* t : mats)
      if ((rc = get(f.f, t->data(), t->size() * 4, path))) return rc;
    float* rms = theta.data() + (size_t)l * m->layer_size + m->oRa;
    if ((rc = get(f.f, rms, 2 * D * 4, path))) return rc;
    std::vector<float> rms_m(2 * D), rms_v(2 * D);
    std::vector<float>* mm[7] = {&am.q, &am.k, &am.v, &am.o, &am.w1, &am.w2, &am.w3};
    std::vector<float>* vv[7] = {&av.q, &av.k, &av.v, &av.o, &av.w1, &av.w2, &av.w3};
    for (int i = 0; i < 7; ++i) {
      if ((rc = get(f.f, mm[i]->data(), mm[i]->size() * 4, path))) return rc;
      if ((rc = get(f.f, vv[i]->data(), vv[i]->size() * 4, path))) return rc;
    }
    for (int i = 0; i < 2; ++i) {
      if ((rc = get(f.f, rms_m.data() + i * D, D * 4, path))) return rc;
      if ((rc = get(f.f, rms_v.data() + i * D, D * 4, path))) return rc;
    }
    if (lora_path) merge_layer(m, w, theta.data(), l, -1.0f);
    if ((rc = b2p_model_set_layer(m, l, w.q.data(), w.k.data(), w.v.data(), w.o.data(), w.w1.data(), w.w2.data(),
                                  w.w3.data())))
      return rc;
    if (tv.full) {
      int err = B2P_OK;
      auto to = [&](float* base, const LayerW& src) {
        float* parts[4] = {base + tv.o_qkv, base + tv.o_o, base + tv.o_13, base + tv.o_2};
        join_layout(m, src, [&](int p, const float* in, size_t n) {
          if (!err) err = h2d(m, parts[p] + part_offset(m, p, l), in, n * 4);
        });
      };
      to(tv.mw, w);
      to(tv.am_w, am);
      to(tv.av_w, av);
      const size_t ro = (size_t)l * m->layer_size + m->oRa;
      if (!err) err = h2d(m, tv.adam_m + ro, rms_m.data(), 2 * D * 4);
      if (!err) err = h2d(m, tv.adam_v + ro, rms_v.data(), 2 * D * 4);
      if (err) return err;
    }
  }
  std::vector<float> fm(D), fv(D), buf(V * D);
  if ((rc = get(f.f, theta.data() + m->oRfinal, D * 4, path))) return rc;
  if ((rc = get(f.f, fm.data(), D * 4, path)) || (rc = get(f.f, fv.data(), D * 4, path))) return rc;
  if ((rc = get(f.f, buf.data(), V * D * 4, path))) return rc;
  if (c2f) {
    rc = b2p_model_set_embedding(m, buf.data(), c2f, cv);
  } else {
    const std::vector<int32_t> cur = m->h_c2f;
    rc = b2p_model_set_embedding(m, buf.data(), cur.data(), (int)cur.size());
  }
  if (rc) return rc;
  if ((rc = h2d(m, m->theta, theta.data(), theta.size() * 4))) return rc;
  if (tv.full) {
    if ((rc = h2d(m, tv.adam_m + m->oRfinal, fm.data(), D * 4))) return rc;
    if ((rc = h2d(m, tv.adam_v + m->oRfinal, fv.data(), D * 4))) return rc;
    if ((rc = get(f.f, buf.data(), V * D * 4, path)) || (rc = h2d(m, tv.am_e, buf.data(), V * D * 4))) return rc;
    if ((rc = get(f.f, buf.data(), V * D * 4, path)) || (rc = h2d(m, tv.av_e, buf.data(), V * D * 4))) return rc;
    *tv.full_t = h.adam_t;
  }
  if (lora_path && tv.adam_m) {
    // train_mezo.m:1134-1137: the adapters resume at the sidecar's step count with fresh moments
    B2P_CHECK_CUDA(cudaMemsetAsync(tv.adam_m, 0, (size_t)m->P * 4, m->st));
    B2P_CHECK_CUDA(cudaMemsetAsync(tv.adam_v, 0, (size_t)m->P * 4, m->st));
    *tv.adam_t = sidecar_t;
  }
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  if (hout) *hout = h;
  return B2P_OK;
}

}  // namespace
}  // namespace b2p

extern "C" {

int b2p_ckpt_read_header(const char* path, b2p_ckpt_header* hdr) {
  b2p_ckpt_header h;
  int rc = b2p::read_header(path, &h, nullptr);
  if (rc) return rc;
  if ((rc = b2p::check_header(nullptr, h, path))) return rc;
  *hdr = h;
  return B2P_OK;
}

int b2p_ckpt_save(b2p_model* m, const char* path, const char* lora_path, const b2p_ckpt_header* hdr) {
  return b2p::save(m, path, lora_path, hdr);
}

int b2p_ckpt_load(b2p_model* m, const char* path, const char* lora_path, const int32_t* compact_to_full, int cv,
                  int full, b2p_ckpt_header* hdr) {
  return b2p::load(m, path, lora_path, compact_to_full, cv, full, hdr);
}

}  // extern "C"
