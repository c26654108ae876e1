// gemm.cuh — the projection tile engine: a persistent, warp-specialised
// tcgen05 GEMM for sm_100a.
//
//   D[M, N] = X[M, K] · W[N, K]^T  (+ U[M, 16] · Bv[N, 16]^T  with LoRA)
//
// X rows are tokens (the MMA "M" side, 128-row tiles), W rows are output
// channels (the "N" side, BN-column tiles). Both operands are K-major 16-bit
// (fp16 or bf16) and are brought into shared memory by TMA with 128-byte
// swizzle; the fp32 accumulator lives in TMEM (two buffers so the epilogue of
// tile i overlaps the MMAs of tile i+1).
//
// The LoRA-split correction out += B·(A·x) (reference lora_addmm,
// training/train_mezo.m:694-703) runs on the tensor cores as one extra K=16
// MMA per tile: U = A·x (per token, 16-bit, zero-padded to 16 columns) is
// loaded by TMA, and the perturbed B rows of the tile's variant,
// fl(fl(B + s1·z) + s2·z), are computed on the fly from the fp32 master copy
// and the sign mask straight into shared memory (never stored to HBM).
//
// Warp roles (352 threads):
//   warp 0       TMA producer (one lane)
//   warp 1       TMEM allocator + UMMA issuer (one lane)
//   warp 2       LoRA operand warp (perturbed B tile + U tile TMA), LoRA kernels only
//   warps 3..10  epilogue: TMEM -> registers -> fused epilogue -> swizzled smem
//                -> TMA store / TMA reduce-add. Warps w and w+4 share TMEM lane
//                quarter w%4 and split the tile's 32-column chunks.
//
// This is the channel-first projection Y[out,T] = W[out,in]·X[in,T] of the
// reference (training/train_mezo.m:1533-1538, 1598, 1630-1633, 1669, 1696)
// stored transposed: the device keeps activations token-major so that every
// fused epilogue (RoPE pairs, SiLU·gate pairs, residual, CE row statistics)
// sees one token row per thread.
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
constexpr int kEpiWarps = 8;
constexpr int kFirstEpiWarp = 3;
constexpr int kGemmThreads = 32 * (kFirstEpiWarp + kEpiWarps);  // 352
constexpr int kMaxRank = 16;      // LoRA rank padded to one UMMA K step
constexpr int kUCols = 64;        // U16 row: 4 projections x 16 columns
constexpr int kMaxGroups = 256;   // variant groups / variants a LoRA launch may reference

enum EpiKind : int {
  EPI_F32 = 0,       // out fp32 [M, ldo] = acc (+ LoRA)
  EPI_H16 = 1,       // out 16-bit [M, ldo] = acc (+ LoRA)
  EPI_QKV_ROPE = 2,  // out 16-bit: acc + LoRA(seg), RoPE on columns < rope_cols
  EPI_RESID = 3,     // out fp32 x [M, ldo] += alpha * (acc + LoRA)   (TMA reduce-add)
  EPI_SWIGLU = 4,    // tile = [gate half | up half]; out 16-bit [M, ldo] = silu(gate) * up
  EPI_CE = 5,        // per-row (max, sum exp) partials over the tile's valid columns + target logit
  EPI_CE_GRAD = 6,   // out 16-bit = alpha * (exp(acc - row_lse[row]) - [col == target[row]])  (dlogits)
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

// LoRA operands of a GEMM: U16 tile via TMA, perturbed B from theta.
struct LoraEpi {
  const float* theta;          // flat trainable parameters (fp32 master copy)
  const uint32_t* masks;       // [slots][mask_words] sign bits, bit i <-> parameter i
  long long mask_words;
  const VariantInfo* variants;
  const int* group_variant;    // variant id of each group of `group_rows` token rows
  int group_rows;
  int n_groups;                // entries of group_variant (<= kMaxGroups)
  int n_variants;              // entries of variants (<= kMaxGroups)
  int rank;                    // 4 or 8 (<= 16)
  int nseg;                    // column segments (1, or 3 for Q|K|V)
  int seg_start[4];            // seg_start[nseg] == N; every boundary a multiple of BN
  long long seg_boff[3];       // offset of segment's B [rows, rank] inside theta (multiple of rank)
  int seg_ucol[3];             // first U16 column of the segment (multiple of 16)
  int inter128;                // 1: two segments interleaved in 128-column blocks (the W1|W3 tiles of the
                               // SwiGLU GEMM): column c is row ((c/256)*128 + c%128) of segment (c/128)%2
};

struct EpiParams {
  int M, N;
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
  float2* ce_part;             // [M, 2 * n_tiles_n] (one partial per epilogue column half)
  float* ce_tgt;               // [M]
  int n_tiles_n;
  const float* row_lse;        // EPI_CE_GRAD: [M] log-sum-exp of each row's logits
  uint32_t* status;            // device error word
};

template <int BN, int KIND>
struct GemmSmem {
  static constexpr bool kOutF32 = (KIND == EPI_F32 || KIND == EPI_RESID);
  static constexpr bool kStores = (KIND != EPI_CE);
  static constexpr int kAStage = kBM * kBK * 2;  // 16 KB
  static constexpr int kBStage = BN * kBK * 2;
  static constexpr int kStageBytes = kAStage + kBStage;
  // per epilogue warp: one 32 x 32 staging box (fp32 128 B rows / 16-bit 64 B rows)
  static constexpr int kStageOutBytes = kStores ? (kOutF32 ? 4096 : 2048) : 0;
  static constexpr int kOutBytes = kStageOutBytes * kEpiWarps;
  static constexpr int kLoraU = kBM * kMaxRank * 2;   // 4 KB
  static constexpr int kLoraB = BN * kMaxRank * 2;    // BN x 32 B
  static constexpr int kLoraBytes = 2 * (kLoraU + kLoraB);
  static constexpr int kBudget = 224 * 1024;
  static constexpr int kFree = kBudget - kOutBytes - kLoraBytes - kMaxGroups * 20 - 1024 - 256;
  static constexpr int kStages = (kFree / kStageBytes) > 8 ? 8 : (kFree / kStageBytes);
  static constexpr int kOutOff = kStages * kStageBytes;
  static constexpr int kLoraOff = kOutOff + kOutBytes;
  static constexpr int kVarOff = kLoraOff + kLoraBytes;          // group -> variant table, variant infos
  static constexpr int kVarBytes = kMaxGroups * 4 + kMaxGroups * 16;
  static constexpr int kBarOff = kVarOff + kVarBytes;
  static constexpr int kTotal = kBarOff + 256 + 1024;  // + barriers + alignment slack
  static constexpr int kAccStride = BN <= 128 ? 128 : 256;  // TMEM columns per accumulator buffer
  static constexpr int kTmemCols = 2 * kAccStride;
  static_assert(kTotal <= 227 * 1024, "shared memory over the 227 KB per-CTA limit");
  static_assert(kStages >= 2, "pipeline needs at least two stages");
  static_assert(kLoraOff % 1024 == 0 && kOutOff % 1024 == 0, "1 KB alignment of swizzled buffers");
};

__device__ __forceinline__ float silu_f(float h) { return __fdividef(h, 1.0f + __expf(-h)); }

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

// Write one 32-value row of a 32 x 32 staging box in the TMA swizzle layout:
// fp32 rows are 128 B (SWIZZLE_128B: chunk c of row r at c ^ (r & 7)),
// 16-bit rows are 64 B (SWIZZLE_64B: chunk c of row r at c ^ ((r >> 1) & 3)).
template <bool F32, typename OutT>
__device__ __forceinline__ void stage_row(uint8_t* box, int r, const float* v) {
  if (F32) {
    uint8_t* row = box + r * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<float4*>(row + ((c ^ (r & 7)) << 4)) =
          make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
  } else {
    uint8_t* row = box + r * 64;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint4 w;
      w.x = pack2<OutT>(v[8 * c + 0], v[8 * c + 1]);
      w.y = pack2<OutT>(v[8 * c + 2], v[8 * c + 3]);
      w.z = pack2<OutT>(v[8 * c + 4], v[8 * c + 5]);
      w.w = pack2<OutT>(v[8 * c + 6], v[8 * c + 7]);
      *reinterpret_cast<uint4*>(row + ((c ^ ((r >> 1) & 3)) << 4)) = w;
    }
  }
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
template <int BN, int KIND, typename OutT, bool BF16, bool LORA>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                   const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmU, int M, int N,
                   int K, EpiParams ep) {
  using S = GemmSmem<BN, KIND>;
  constexpr int STAGES = S::kStages;
  constexpr int NCHUNK = (KIND == EPI_SWIGLU) ? BN / 64 : BN / 32;  // 32-column output chunks per tile
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN must be a multiple of 32 in [32, 256]");
  static_assert(KIND != EPI_SWIGLU || BN % 64 == 0, "SwiGLU tiles hold two halves of 32-column chunks");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::kAStage;
  uint8_t* sOut = smem + S::kOutOff;
  uint8_t* sLU = smem + S::kLoraOff;                 // 2 x U tile   [128][16] 16-bit, SW32
  uint8_t* sLB = sLU + 2 * S::kLoraU;                // 2 x Bv tile  [BN][16]  16-bit, SW32
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBarOff);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + STAGES;
  uint64_t* tfull_bar = bars + 2 * STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* lfull_bar = tfull_bar + 4;
  uint64_t* lempty_bar = tfull_bar + 6;
  uint64_t* drain_bar = tfull_bar + 8;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tfull_bar + 9);
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
      mbar_init(&tempty_bar[a], kEpiWarps);  // one arrive per epilogue warp
      mbar_init(&lfull_bar[a], 1);
      mbar_init(&lempty_bar[a], 1);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
    if (S::kStores) tma_prefetch_desc(&tmOut);
    if (LORA) tma_prefetch_desc(&tmU);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_enter();  // the previous kernel's outputs are complete from here on

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
      int lb = 0;
      uint32_t lphase = 0;
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
        if (LORA) {
          // += U[128 x 16] · Bv[BN x 16]^T, one K=16 step
          if (!mbar_wait(&lfull_bar[lb], lphase, abort_flag, ep.status, DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          umma_f16_ss(d_tmem, sw32_kmajor_desc(smem_u32(sLU + lb * S::kLoraU)),
                      sw32_kmajor_desc(smem_u32(sLB + lb * S::kLoraB)), idesc, 1u);
          umma_commit(&lempty_bar[lb]);
          if (++lb == 2) {
            lb = 0;
            lphase ^= 1u;
          }
        }
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
  } else if (warp == 2) {
    // ---------------- LoRA operand warp ----------------
    if (LORA) {
      int* s_gvar = reinterpret_cast<int*>(smem + S::kVarOff);
      VariantInfo* s_var = reinterpret_cast<VariantInfo*>(smem + S::kVarOff + kMaxGroups * 4);
      for (int i = lane; i < ep.lora.n_groups; i += 32) s_gvar[i] = ep.lora.group_variant[i];
      for (int i = lane; i < ep.lora.n_variants; i += 32) s_var[i] = ep.lora.variants[i];
      __syncwarp();
      constexpr int RPL = (BN + 31) / 32;  // B rows per lane
      int lb = 0;
      uint32_t lphase = 0;
      const int rank = ep.lora.rank;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        const int mt = tile / num_n, nt = tile % num_n;
        const int m0 = mt * kBM, n0 = nt * BN;
        int seg = 0;
        while (seg + 1 < ep.lora.nseg && n0 >= ep.lora.seg_start[seg + 1]) ++seg;
        const VariantInfo vi = s_var[s_gvar[m0 / ep.lora.group_rows]];
        const uint32_t* mask = ep.lora.masks + (long long)(vi.mode ? vi.mask_slot : 0) * ep.lora.mask_words;
        const int cs = n0 - ep.lora.seg_start[seg];
        const int seg_rows = ep.lora.seg_start[seg + 1] - ep.lora.seg_start[seg];
        // issue every load of this tile's B rows before using any (rank divides 32 and each
        // row starts at a multiple of rank, so a row's signs share one mask word)
        float4 th[RPL][2];
        uint32_t mw[RPL];
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
          const int n = lane + 32 * i;
          const bool ok = n < BN && cs + n < seg_rows;
          const long long p0 = ep.lora.seg_boff[seg] + (long long)(cs + n) * rank;
          th[i][0] = ok ? __ldg(reinterpret_cast<const float4*>(ep.lora.theta + p0)) : make_float4(0.f, 0.f, 0.f, 0.f);
          th[i][1] = (ok && rank > 4) ? __ldg(reinterpret_cast<const float4*>(ep.lora.theta + p0 + 4))
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
          mw[i] = (ok && vi.mode) ? (__ldg(mask + (p0 >> 5)) >> (p0 & 31)) : 0u;
        }
        int ok = 1;
        if (lane == 0) ok = mbar_wait(&lempty_bar[lb], lphase ^ 1u, abort_flag, ep.status, DEV_TIMEOUT_PRODUCER);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        uint8_t* bt = sLB + lb * S::kLoraB;
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
          const int n = lane + 32 * i;
          if (n < BN) {
            float b[8] = {th[i][0].x, th[i][0].y, th[i][0].z, th[i][0].w,
                          th[i][1].x, th[i][1].y, th[i][1].z, th[i][1].w};
            if (vi.mode) {
#pragma unroll
              for (int j = 0; j < 8; ++j)
                if (j < rank) b[j] = perturb_value(b[j], (mw[i] >> j) & 1u, vi);
            }
            // SWIZZLE_32B K-major: 32-byte rows, 16-byte chunk c of row n at c ^ ((n >> 2) & 1);
            // K columns 8..15 are the zero padding of the rank
            uint8_t* rowp = bt + n * 32;
            uint4 w0, w1;
            w0.x = pack2<OutT>(b[0], b[1]);
            w0.y = pack2<OutT>(b[2], b[3]);
            w0.z = pack2<OutT>(b[4], b[5]);
            w0.w = pack2<OutT>(b[6], b[7]);
            w1 = make_uint4(0u, 0u, 0u, 0u);
            const int sw = (n >> 2) & 1;
            *reinterpret_cast<uint4*>(rowp + ((0 ^ sw) << 4)) = w0;
            *reinterpret_cast<uint4*>(rowp + ((1 ^ sw) << 4)) = w1;
          }
        }
        fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
        __syncwarp();
        if (lane == 0) {
          mbar_arrive_expect_tx(&lfull_bar[lb], S::kLoraU);
          tma_load_2d(sLU + lb * S::kLoraU, &tmU, &lfull_bar[lb], ep.lora.seg_ucol[seg], m0);
        }
        if (++lb == 2) {
          lb = 0;
          lphase ^= 1u;
        }
      }
    }
  } else {
    // ---------------- Epilogue (warps 3..10) ----------------
    const int ew = warp - kFirstEpiWarp;   // 0..7
    const int lg = warp & 3;               // TMEM lane quarter this warp may access
    const int half = ew >> 2;              // which interleaved half of the tile's chunks
    const int row_in_tile = lg * 32 + lane;
    const int et = threadIdx.x - kFirstEpiWarp * 32;  // 0..255 within the epilogue group
    uint8_t* box = sOut + ew * S::kStageOutBytes;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int mt = tile / num_n, nt = tile % num_n;
      const int m0 = mt * kBM, n0 = nt * BN;
      const int row = m0 + row_in_tile;
      const bool row_ok = row < M;

      // RoPE factors of this row for the tile, loaded while the tile's MMAs run: with head_dim
      // 64 every chunk of this warp (chunks half, half + 2, ...) covers the same half of the 32
      // frequencies, ((n0 / 32) + half) % 2 (the tables hold 64 KB, more than the L1 left beside
      // the pipeline's shared memory, so per-chunk loads would each go to L2)
      float rcs[16], rsn[16];
      if (KIND == EPI_QKV_ROPE) {
        const int pos = (m0 % ep.seq_len) + row_in_tile;
        const int fh = ((n0 >> 5) + half) & 1;
        const float4* cs4 = reinterpret_cast<const float4*>(ep.rope_cos + (long long)pos * 32 + 16 * fh);
        const float4* sn4 = reinterpret_cast<const float4*>(ep.rope_sin + (long long)pos * 32 + 16 * fh);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 c4 = __ldg(cs4 + q), s4 = __ldg(sn4 + q);
          rcs[4 * q] = c4.x; rcs[4 * q + 1] = c4.y; rcs[4 * q + 2] = c4.z; rcs[4 * q + 3] = c4.w;
          rsn[4 * q] = s4.x; rsn[4 * q + 1] = s4.y; rsn[4 * q + 2] = s4.z; rsn[4 * q + 3] = s4.w;
        }
      }

      mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, ep.status, DEV_TIMEOUT_EPILOGUE);
      // All epilogue warps take the same continue/abort decision.
      named_bar_sync(2, 32 * kEpiWarps);
      if (et == 0) *epi_abort = *abort_flag;
      named_bar_sync(2, 32 * kEpiWarps);
      if (*epi_abort) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + acc * S::kAccStride + ((uint32_t)(lg * 32) << 16);

      float ce_m = -INFINITY, ce_s = 0.f;
      int tgt = -1;
      if ((KIND == EPI_CE || KIND == EPI_CE_GRAD) && row_ok) tgt = ep.targets[row];
      const float lse = (KIND == EPI_CE_GRAD && row_ok) ? ep.row_lse[row] : 0.f;

#pragma unroll 1
      for (int ch = half; ch < NCHUNK; ch += 2) {
        float v[32];
        int col;
        __syncwarp();
        if (KIND == EPI_SWIGLU) {
          uint32_t g[32], up[32];
          tmem_ld32(t_row + ch * 32, g);
          tmem_ld32(t_row + BN / 2 + ch * 32, up);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] = silu_f(__uint_as_float(g[c])) * __uint_as_float(up[c]);
          col = nt * (BN / 2) + ch * 32;
        } else {
          uint32_t r[32];
          tmem_ld32(t_row + ch * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] = __uint_as_float(r[c]);
          col = n0 + ch * 32;
        }
        if (KIND == EPI_CE) {
          const int nvalid = min(32, N - col);
          if (row_ok && nvalid > 0) {
            float cm = -INFINITY;
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (c < nvalid) cm = fmaxf(cm, v[c]);
            if (cm > ce_m) {
              ce_s *= __expf(ce_m - cm);
              ce_m = cm;
            }
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (c < nvalid) ce_s += __expf(v[c] - ce_m);
            if (tgt >= col && tgt < col + nvalid) {
#pragma unroll
              for (int c = 0; c < 32; ++c)
                if (col + c == tgt) ep.ce_tgt[row] = v[c];
            }
          }
          continue;
        }
        if (KIND == EPI_QKV_ROPE && col < ep.rope_cols) {
          // head_dim 64: the chunk covers frequency indices 16·fh .. 16·fh + 15 of one head
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float v0 = v[2 * i], v1 = v[2 * i + 1];
            v[2 * i] = v0 * rcs[i] - v1 * rsn[i];
            v[2 * i + 1] = v0 * rsn[i] + v1 * rcs[i];
          }
        }
        if (KIND == EPI_RESID) {
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] *= ep.alpha;
        }
        if (KIND == EPI_CE_GRAD) {
          // softmax - one-hot (cross_entropy_loss, training/cpu_ops.h:118-130), times the gradient scale
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float p = __expf(v[c] - lse);
            v[c] = ep.alpha * (col + c == tgt ? p - 1.0f : p);
          }
        }
        // stage the 32 x 32 box (the previous store must have finished reading it)
        if (lane == 0) bulk_wait_read0();
        __syncwarp();
        stage_row<S::kOutF32, OutT>(box, lane, v);
        fence_proxy_async_smem();
        __syncwarp();
        // boxes that start inside the tensor are clipped by TMA; boxes wholly outside are skipped
        if (lane == 0 && m0 + lg * 32 < M && col < (KIND == EPI_SWIGLU ? N / 2 : N)) {
          if (KIND == EPI_RESID)
            tma_reduce_add_2d(&tmOut, box, col, m0 + lg * 32);
          else
            tma_store_2d(&tmOut, box, col, m0 + lg * 32);
          bulk_commit();
        }
      }
      if (KIND == EPI_CE && row_ok)
        ep.ce_part[(long long)row * (2 * ep.n_tiles_n) + 2 * nt + half] = make_float2(ce_m, ce_s);

      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (S::kStores && lane == 0) bulk_wait0();  // every store of this warp has completed
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

}  // namespace b2p
