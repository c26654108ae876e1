// attn_api.cu — C-ABI entry points for causal GQA attention on device buffers:
// the forward (cpu_sdpa_forward, training/cpu_ops.h:321-360, over K/V tiled by
// gqa_tile_kv, training/io.h:439-446) and the backward as bp_lora_backward runs
// it (cpu_sdpa_backward, cpu_ops.h:213-290; gqa_reduce_kv, io.h:448-459;
// rope_backward_inplace, cpu_ops.h:364; training/backprop_lora.h:241-252).
// They drive the same kernels as the model's forward and backprop-LoRA
// backward, on token-major 16-bit rows of n_seq independent sequences.
#include <cmath>
#include <cstdint>
#include <vector>
#include "engine.cuh"
#include "kernels.cuh"

using namespace b2p;

namespace {

constexpr int kHeadDim = 64;

int check_common(const void* qkv, int ld_qkv, int n_seq, int seq, int heads, int kv_heads, int dtype) {
  B2P_REQUIRE(qkv, "null qkv");
  B2P_REQUIRE(dtype == B2P_F16 || dtype == B2P_BF16, "dtype must be B2P_F16 or B2P_BF16");
  B2P_REQUIRE(n_seq >= 1, "n_seq must be >= 1");
  B2P_REQUIRE(seq >= 64 && seq % 64 == 0, "seq must be a positive multiple of 64 (got %d)", seq);
  B2P_REQUIRE(heads >= 1 && kv_heads >= 1 && heads % kv_heads == 0, "heads (%d) must be a multiple of kv_heads (%d)",
              heads, kv_heads);
  B2P_REQUIRE(ld_qkv >= (heads + 2 * kv_heads) * kHeadDim && ld_qkv % 8 == 0,
              "ld_qkv must hold Q|K|V (%d columns) and keep 16-byte rows", (heads + 2 * kv_heads) * kHeadDim);
  B2P_REQUIRE((reinterpret_cast<uintptr_t>(qkv) & 15u) == 0, "qkv must be 16-byte aligned");
  return B2P_OK;
}

}  // namespace

extern "C" {

int b2p_attention(const void* qkv, int ld_qkv, void* out, int ld_out, float* lse, int n_seq, int seq, int heads,
                  int kv_heads, int dtype, void* stream) {
  int rc = check_common(qkv, ld_qkv, n_seq, seq, heads, kv_heads, dtype);
  if (rc) return rc;
  B2P_REQUIRE(out, "null out");
  B2P_REQUIRE(ld_out >= heads * kHeadDim && ld_out % 8 == 0, "ld_out must hold %d columns and keep 16-byte rows",
              heads * kHeadDim);
  B2P_REQUIRE((reinterpret_cast<uintptr_t>(out) & 15u) == 0, "out must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* sched = nullptr;
  B2P_CHECK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&sched), 2 * sizeof(int), st));
  B2P_CHECK_CUDA(cudaMemsetAsync(sched, 0, 2 * sizeof(int), st));
  AttnArgs a;
  a.qkv = qkv;
  a.ld_qkv = ld_qkv;
  a.q_off = 0;
  a.k_off = heads * kHeadDim;
  a.v_off = (heads + kv_heads) * kHeadDim;
  a.out = out;
  a.ld_out = ld_out;
  a.seq = seq;
  a.heads = heads;
  a.kv_heads = kv_heads;
  a.ngroups = n_seq;
  a.lse = lse;
  a.sched = sched;
  rc = launch_attention(a, dtype == B2P_BF16, st);
  B2P_CHECK_CUDA(cudaFreeAsync(sched, st));
  return rc;
}

int b2p_attention_backward(const void* qkv, int ld_qkv, const void* out, const void* dout, int ld_o,
                           const float* lse, void* dqkv, int ld_d, int n_seq, int seq, int heads, int kv_heads,
                           float rope_theta, int dtype, void* stream) {
  int rc = check_common(qkv, ld_qkv, n_seq, seq, heads, kv_heads, dtype);
  if (rc) return rc;
  B2P_REQUIRE(out && dout && lse && dqkv, "null operand");
  B2P_REQUIRE(ld_o >= heads * kHeadDim && ld_o % 8 == 0, "ld_o must hold %d columns and keep 16-byte rows",
              heads * kHeadDim);
  B2P_REQUIRE(ld_d >= (heads + 2 * kv_heads) * kHeadDim && ld_d % 8 == 0,
              "ld_d must hold dQ|dK|dV and keep 16-byte rows");
  B2P_REQUIRE(rope_theta > 0.f, "rope_theta must be positive");
  for (const void* p : {out, dout, static_cast<const void*>(dqkv)})
    B2P_REQUIRE((reinterpret_cast<uintptr_t>(p) & 15u) == 0, "operands must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // RoPE tables with the reference's expressions (training/cpu_ops.h:303-307)
  const int half = kHeadDim / 2;
  std::vector<float> tab(2 * (size_t)seq * half);
  for (int i = 0; i < half; i++) {
    const float freq = 1.0f / powf(rope_theta, 2.0f * i / (float)kHeadDim);
    for (int p = 0; p < seq; p++) {
      tab[(size_t)p * half + i] = cosf(p * freq);
      tab[(size_t)seq * half + (size_t)p * half + i] = sinf(p * freq);
    }
  }
  const long long rows = (long long)n_seq * seq;
  float* d_tab = nullptr;
  float* dvec = nullptr;
  int* sched = nullptr;
  B2P_CHECK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&d_tab), tab.size() * 4, st));
  B2P_CHECK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&dvec), (size_t)rows * heads * 4, st));
  B2P_CHECK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&sched), 2 * sizeof(int), st));
  B2P_CHECK_CUDA(cudaMemsetAsync(sched, 0, 2 * sizeof(int), st));
  // pageable source: the copy is staged before cudaMemcpyAsync returns, so `tab` may go
  B2P_CHECK_CUDA(cudaMemcpyAsync(d_tab, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice, st));
  AttnBwdArgs a;
  a.qkv = qkv;
  a.ld = ld_qkv;
  a.q_off = 0;
  a.k_off = heads * kHeadDim;
  a.v_off = (heads + kv_heads) * kHeadDim;
  a.o = out;
  a.dout = dout;
  a.ld_o = ld_o;
  a.lse = lse;
  a.dvec = dvec;
  a.dqkv = dqkv;
  a.ld_d = ld_d;
  a.rope_cos = d_tab;
  a.rope_sin = d_tab + (size_t)seq * half;
  a.seq = seq;
  a.heads = heads;
  a.kv_heads = kv_heads;
  a.ngroups = n_seq;
  a.scale_log2 = a.scale = 0.f;  // set by the launcher
  a.sched = sched;
  rc = launch_attention_backward(a, dtype == B2P_BF16, true, st);
  B2P_CHECK_CUDA(cudaFreeAsync(sched, st));
  B2P_CHECK_CUDA(cudaFreeAsync(dvec, st));
  B2P_CHECK_CUDA(cudaFreeAsync(d_tab, st));
  return rc;
}

}  // extern "C"
