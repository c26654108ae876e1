// gemm.cuh — the projection tile engine: a persistent, warp-specialised
// tcgen05 GEMM for sm_100a.
//
//   D[M, N] = X[M, K] · W[N, K]^T          (token-major activations X, weights W)
//
// X rows are tokens (the MMA "M" side, 128-row tiles), W rows are output
// channels (the "N" side, BN-column tiles). Both operands are K-major 16-bit
// (fp16 or bf16) and are brought into shared memory by TMA with 128-byte
// swizzle; the fp32 accumulator lives in TMEM (two BN-column buffers so the
// epilogue of tile i overlaps the MMAs of tile i+1).
//
// Warp roles (192 threads):
//   warp 0      TMA producer (one lane)
//   warp 1      TMEM allocator + UMMA issuer (one lane)
//   warps 2..5  epilogue: TMEM -> registers -> fused epilogue -> HBM
//
// This is the channel-first projection Y[out,T] = W[out,in]·X[in,T] of the
// reference (training/train_mezo.m:1533-1538, 1598, 1630-1633, 1669, 1696)
// stored transposed: the device keeps activations token-major so that every
// fused epilogue (LoRA-up, RoPE pairs, SiLU·gate pairs, residual, CE row
// statistics) sees one token row per thread.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include "ptx.cuh"

namespace b2p {

constexpr int kBM = 128;          // token rows per tile (UMMA M)
constexpr int kBK = 64;           // K elements per pipeline stage (128 B of 16-bit)
constexpr int kUmmaK = 16;        // K per tcgen05.mma for kind::f16
constexpr int kGemmThreads = 192;
constexpr int kMaxRank = 16;

enum EpiKind : int {
  EPI_F32 = 0,       // out fp32 [M, ldo] = acc (+ LoRA)
  EPI_H16 = 1,       // out 16-bit [M, ldo] = acc (+ LoRA)
  EPI_QKV_ROPE = 2,  // out 16-bit: acc + LoRA(seg), RoPE on columns < rope_cols
  EPI_RESID = 3,     // out fp32 x [M, ldo] += alpha * (acc + LoRA)
  EPI_SWIGLU = 4,    // tile = [gate half | up half]; out 16-bit [M, ldo] = silu(gate) * up
  EPI_CE = 5,        // per-row (max, sum exp) partials over the tile's valid columns + target logit
};

// One perturbed evaluation of the trainable parameters: θ, θ+s1·z or
// (θ+s1·z)+s2·z with z the Rademacher signs of `mask_slot`.
struct VariantInfo {
  int mask_slot;   // row of the sign-mask array (ignored when mode == 0)
  int mode;        // 0: θ; 1: θ + s1 z; 2: (θ + s1 z) + s2 z
  float s1, s2;
};

__device__ __forceinline__ float perturb_value(float th, uint32_t bit, const VariantInfo& v) {
  if (v.mode == 0) return th;
  float p = __fadd_rn(th, bit ? v.s1 : -v.s1);
  if (v.mode == 2) p = __fadd_rn(p, bit ? v.s2 : -v.s2);
  return p;
}
__device__ __forceinline__ uint32_t mask_bit(const uint32_t* mask, long long idx) {
  return (__ldg(mask + (idx >> 5)) >> (idx & 31)) & 1u;
}

// LoRA-up epilogue operands: Y += B_v · U  where U = A_v · x was produced per
// token by the LoRA-down stage and B_v is the perturbed LoRA B for the tile's
// variant (reference lora_addmm, training/train_mezo.m:694-703).
struct LoraEpi {
  const float* theta;          // flat trainable parameters (fp32 master copy)
  const uint32_t* masks;       // [slots][mask_words] sign bits, bit i <-> parameter i
  long long mask_words;
  const VariantInfo* variants;
  const int* group_variant;    // variant id of each group of `group_rows` token rows
  int group_rows;
  const float* U;              // [M, ldu] fp32
  int ldu;
  int rank;
  int nseg;                    // column segments sharing one epilogue (1, or 3 for Q|K|V)
  int seg_start[4];            // seg_start[nseg] == N; every boundary a multiple of BN
  long long seg_boff[3];       // offset of segment's B [rows, rank] inside theta
  int seg_ucol[3];             // first U column of the segment
};

struct EpiParams {
  int M, N;
  void* out;
  int ldo;
  float alpha;
  int has_lora;
  LoraEpi lora;
  // RoPE (interleaved pairs, reference training/cpu_ops.h:299-315)
  const float* rope_cos;       // [seq_len, head_dim/2]
  const float* rope_sin;
  int rope_cols;
  int head_dim;
  int seq_len;
  // cross-entropy partials
  const int* targets;          // [M] compact target id per token row (-1: none)
  float2* ce_part;             // [M, n_tiles_n]
  float* ce_tgt;               // [M]
  int n_tiles_n;
  uint32_t* status;            // device error word
};

template <int BN>
struct GemmSmem {
  static constexpr int kAStage = kBM * kBK * 2;  // 16 KB
  static constexpr int kBStage = BN * kBK * 2;
  static constexpr int kStageBytes = kAStage + kBStage;
  static constexpr int kEpiBytes = BN * kMaxRank * 4;  // perturbed LoRA B tile
  static constexpr int kBudget = 224 * 1024;
  static constexpr int kStages = ((kBudget - kEpiBytes - 1024) / kStageBytes) > 8
                                     ? 8
                                     : ((kBudget - kEpiBytes - 1024) / kStageBytes);
  static constexpr int kBarOff = kStages * kStageBytes + kEpiBytes;
  static constexpr int kTotal = kBarOff + 256 + 1024;  // + barriers + alignment slack
  static constexpr int kAccStride = BN <= 128 ? 128 : 256;  // TMEM columns per accumulator buffer
  static constexpr int kTmemCols = 2 * kAccStride;
  static_assert(kTotal <= 227 * 1024, "shared memory over the 227 KB per-CTA limit");
  static_assert(kStages >= 2, "pipeline needs at least two stages");
};

__device__ __forceinline__ float silu_f(float h) { return h / (1.0f + expf(-h)); }

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Store 32 consecutive values of one row as 16-bit, vectorised when the whole
// chunk is in range.
template <typename T>
__device__ __forceinline__ void store_row16(T* dst, const float* v, int nvalid) {
  if (nvalid >= 32) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 w;
      w.x = pack2<T>(v[8 * q + 0], v[8 * q + 1]);
      w.y = pack2<T>(v[8 * q + 2], v[8 * q + 3]);
      w.z = pack2<T>(v[8 * q + 4], v[8 * q + 5]);
      w.w = pack2<T>(v[8 * q + 6], v[8 * q + 7]);
      d4[q] = w;
    }
  } else {
#pragma unroll
    for (int c = 0; c < 32; ++c)
      if (c < nvalid) dst[c] = static_cast<T>(v[c]);
  }
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
template <int BN, int KIND, typename OutT, bool BF16>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, int M, int N,
                   int K, EpiParams ep) {
  using S = GemmSmem<BN>;
  constexpr int STAGES = S::kStages;
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN must be a multiple of 32 in [32, 256]");
  static_assert(KIND != EPI_SWIGLU || BN % 64 == 0, "SwiGLU tiles hold two halves of 32-column chunks");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::kAStage;
  float* sLoraB = reinterpret_cast<float*>(smem + STAGES * S::kStageBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBarOff);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* tfull_bar = bars + 2 * STAGES;
  uint64_t* tempty_bar = bars + 2 * STAGES + 2;
  uint64_t* drain_bar = bars + 2 * STAGES + 4;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile uint32_t* abort_flag = tmem_holder + 1;
  volatile uint32_t* epi_abort = tmem_holder + 2;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 4);  // one arrive per epilogue warp
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  const int num_m = (M + kBM - 1) / kBM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int kblocks = (K + kBK - 1) / kBK;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int mt = tile / num_n, nt = tile % num_n;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, ep.status, DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], S::kStageBytes);
          tma_load_2d(sA + stage * S::kAStage, &tmX, &full_bar[stage], kb * kBK, mt * kBM);
          tma_load_2d(sB + stage * S::kBStage, &tmW, &full_bar[stage], kb * kBK, nt * BN);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Drain: let every issued copy land before the CTA can exit.
        int pending = issued < STAGES ? issued : STAGES;
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < pending; ++i) {
          if (--s < 0) {
            s = STAGES - 1;
            ph ^= 1u;
          }
          mbar_wait_drain(&full_bar[s], ph);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- UMMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(BF16, kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued_any = false;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, ep.status, DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * S::kAccStride;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, ep.status, DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = sw128_kmajor_desc(smem_u32(sA + stage * S::kAStage));
          const uint64_t bdesc = sw128_kmajor_desc(smem_u32(sB + stage * S::kBStage));
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            // +32 bytes per K step == +2 in the encoded start address.
            umma_f16_ss(d_tmem, adesc + 2ull * k, bdesc + 2ull * k, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          issued_any = true;
          umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && issued_any) {
        // Let the MMAs in flight finish before TMEM is released.
        umma_commit(drain_bar);
        mbar_wait_drain(drain_bar, 0);
      }
    }
  } else {
    // ---------------- Epilogue (warps 2..5) ----------------
    const int lg = warp & 3;               // TMEM lane quarter this warp may access
    const int row_in_tile = lg * 32 + lane;
    const int et = threadIdx.x - 64;       // 0..127 within the epilogue group
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int mt = tile / num_n, nt = tile % num_n;
      const int m0 = mt * kBM, n0 = nt * BN;
      const int row = m0 + row_in_tile;
      const bool row_ok = row < M;

      // ---- stage the perturbed LoRA B tile for this tile's variant ----
      int seg = 0;
      float u[kMaxRank];
      const int rank = ep.has_lora ? ep.lora.rank : 0;
      if (ep.has_lora) {
        while (seg + 1 < ep.lora.nseg && n0 >= ep.lora.seg_start[seg + 1]) ++seg;
        const int grp = m0 / ep.lora.group_rows;
        const VariantInfo vi = ep.lora.variants[ep.lora.group_variant[grp]];
        const uint32_t* mask = ep.lora.masks + (long long)(vi.mode ? vi.mask_slot : 0) * ep.lora.mask_words;
        named_bar_sync(1, 128);  // previous tile done reading sLoraB
        const int cs = n0 - ep.lora.seg_start[seg];
        const int seg_rows = ep.lora.seg_start[seg + 1] - ep.lora.seg_start[seg];
        for (int i = et; i < BN * rank; i += 128) {
          const int c = i / rank, j = i - c * rank;
          float b = 0.f;
          if (cs + c < seg_rows) {
            const long long pidx = ep.lora.seg_boff[seg] + (long long)(cs + c) * rank + j;
            const float th = __ldg(ep.lora.theta + pidx);
            b = vi.mode ? perturb_value(th, mask_bit(mask, pidx), vi) : th;
          }
          sLoraB[c * kMaxRank + j] = b;
        }
        named_bar_sync(1, 128);
#pragma unroll
        for (int j = 0; j < kMaxRank; ++j)
          u[j] = (j < rank && row_ok) ? __ldg(ep.lora.U + (long long)row * ep.lora.ldu + ep.lora.seg_ucol[seg] + j)
                                      : 0.f;
      }

      mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, ep.status, DEV_TIMEOUT_EPILOGUE);
      // All four epilogue warps take the same continue/abort decision, so no
      // warp is ever left waiting at a named barrier that the others skip.
      named_bar_sync(2, 128);
      if (et == 0) *epi_abort = *abort_flag;
      named_bar_sync(2, 128);
      if (*epi_abort) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + acc * S::kAccStride + ((uint32_t)(lg * 32) << 16);

      float ce_m = -INFINITY, ce_s = 0.f;
      int tgt = -1;
      if (KIND == EPI_CE && row_ok) tgt = ep.targets[row];

      if (KIND == EPI_SWIGLU) {
        constexpr int HALF = BN / 2;
#pragma unroll 1
        for (int c0 = 0; c0 < HALF; c0 += 32) {
          uint32_t g[32], up[32];
          __syncwarp();
          tmem_ld32(t_row + c0, g);
          tmem_ld32(t_row + HALF + c0, up);
          tmem_ld_wait();
          float* v = reinterpret_cast<float*>(g);
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] = silu_f(__uint_as_float(g[c])) * __uint_as_float(up[c]);
          const int ocol = nt * HALF + c0;
          if (row_ok && ocol < ep.N / 2)
            store_row16<OutT>(reinterpret_cast<OutT*>(ep.out) + (long long)row * ep.ldo + ocol, v,
                              min(32, ep.N / 2 - ocol));
        }
      } else {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t r[32];
          __syncwarp();
          tmem_ld32(t_row + c0, r);
          tmem_ld_wait();
          float v[32];
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] = __uint_as_float(r[c]);
          if (ep.has_lora) {
#pragma unroll
            for (int c = 0; c < 32; ++c) {
              const float4* bl = reinterpret_cast<const float4*>(sLoraB + (c0 + c) * kMaxRank);
              float a = v[c];
#pragma unroll
              for (int q = 0; q < kMaxRank / 4; ++q) {
                if (4 * q < rank) {
                  const float4 b4 = bl[q];
                  a = fmaf(b4.x, u[4 * q + 0], a);
                  a = fmaf(b4.y, u[4 * q + 1], a);
                  a = fmaf(b4.z, u[4 * q + 2], a);
                  a = fmaf(b4.w, u[4 * q + 3], a);
                }
              }
              v[c] = a;
            }
          }
          const int col = n0 + c0;
          const int nvalid = min(32, N - col);
          if (KIND == EPI_CE) {
            if (row_ok && nvalid > 0) {
              float cm = -INFINITY;
#pragma unroll
              for (int c = 0; c < 32; ++c)
                if (c < nvalid) cm = fmaxf(cm, v[c]);
              if (cm > ce_m) {
                ce_s *= expf(ce_m - cm);
                ce_m = cm;
              }
#pragma unroll
              for (int c = 0; c < 32; ++c)
                if (c < nvalid) ce_s += expf(v[c] - ce_m);
              if (tgt >= col && tgt < col + nvalid) {
#pragma unroll
                for (int c = 0; c < 32; ++c)
                  if (col + c == tgt) ep.ce_tgt[row] = v[c];
              }
            }
          } else if (row_ok && nvalid > 0) {
          if (KIND == EPI_QKV_ROPE && col < ep.rope_cols) {
            const int pos = row % ep.seq_len;
            const int half = ep.head_dim >> 1;
            const float* cs_row = ep.rope_cos + (long long)pos * half;
            const float* sn_row = ep.rope_sin + (long long)pos * half;
#pragma unroll
            for (int c = 0; c < 32; c += 2) {
              const int i = ((col + c) % ep.head_dim) >> 1;
              const float cs = __ldg(cs_row + i), sn = __ldg(sn_row + i);
              const float v0 = v[c], v1 = v[c + 1];
              v[c] = v0 * cs - v1 * sn;
              v[c + 1] = v0 * sn + v1 * cs;
            }
          }
          if (KIND == EPI_F32) {
            float* dst = reinterpret_cast<float*>(ep.out) + (long long)row * ep.ldo + col;
            if (nvalid >= 32) {
#pragma unroll
              for (int q = 0; q < 8; ++q)
                reinterpret_cast<float4*>(dst)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            } else {
#pragma unroll
              for (int c = 0; c < 32; ++c)
                if (c < nvalid) dst[c] = v[c];
            }
          } else if (KIND == EPI_RESID) {
            float* dst = reinterpret_cast<float*>(ep.out) + (long long)row * ep.ldo + col;
            if (nvalid >= 32) {
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                float4 x = reinterpret_cast<float4*>(dst)[q];
                x.x = fmaf(ep.alpha, v[4 * q + 0], x.x);
                x.y = fmaf(ep.alpha, v[4 * q + 1], x.y);
                x.z = fmaf(ep.alpha, v[4 * q + 2], x.z);
                x.w = fmaf(ep.alpha, v[4 * q + 3], x.w);
                reinterpret_cast<float4*>(dst)[q] = x;
              }
            } else {
#pragma unroll
              for (int c = 0; c < 32; ++c)
                if (c < nvalid) dst[c] = fmaf(ep.alpha, v[c], dst[c]);
            }
          } else {  // EPI_H16, EPI_QKV_ROPE
            store_row16<OutT>(reinterpret_cast<OutT*>(ep.out) + (long long)row * ep.ldo + col, v, nvalid);
          }
          }  // row_ok && nvalid > 0
        }
      }
      if (KIND == EPI_CE && row_ok) ep.ce_part[(long long)row * ep.n_tiles_n + nt] = make_float2(ce_m, ce_s);

      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

}  // namespace b2p
