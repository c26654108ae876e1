// gemm2.cuh — the CTA-pair (tcgen05 cta_group::2) form of the projection tile
// engine: one 256 x BN output tile per cluster of two CTAs on a TPC.
//
// Each CTA loads, per K step, its own 128 rows of X and its half (BN/2 rows) of
// W, so an SM moves (128 + BN/2) x 128 B per 256 x BN x 64 MMA step: half the
// W bytes of the single-CTA engine, which is bounded by per-SM L2->SMEM ingress
// at 128 x BN tiles. The leader CTA (rank 0) issues the M=256 MMAs; their
// accumulators land in both CTAs' TMEM (rows 0-127 in the leader, 128-255 in
// the peer) and each CTA runs the same epilogues as the single-CTA engine on its
// own 128 rows.
//
// Synchronisation (every TMA load lands in its own CTA; commits name each CTA):
//   full[s]   leader only. The leader's producer arrives with the bytes of both
//             CTAs; both producers' TMA loads complete on it.
//   empty[s]  both CTAs; the leader's MMA thread commits to each in turn.
//   tfull[a]  both CTAs; committed by the leader's MMA thread to each.
//   tempty[a] leader only; 8 local + 8 remote epilogue-warp arrivals.
//   lfull[b]  leader only; LoRA operand warps of both CTAs (one local arrive
//             with both U tiles' bytes + one remote arrive).
//   lempty[b] both CTAs; committed by the leader's MMA thread.
//
// Operand layouts (OPM): bit 0 set, X is given MN-major, as [K][M] rows (the A
// tile of a K step is two 64-row atoms of 64 K rows each, one TMA box apiece);
// bit 1 set, W is given MN-major, as [K][N] rows (BN/128 atoms per CTA). The
// data-gradient GEMMs of the backward multiply by W itself (dX = dY·W, W stored
// [out][in]) and the weight gradients by dY^T and X (stored [tokens][features]):
// MN-major operands read them where they lie instead of from transposed copies.
//
// LoRA: the correction Σ_s U_s · Bv_s^T runs as one K=16 MMA per segment s
// (Q, K, V of the fused QKV projection are three segments; Wo is one). A tile
// may span segments: rows of Bv_s outside segment s are zero.
#pragma once
#include "gemm.cuh"

namespace b2p {

constexpr int kPairThreads = kGemmThreads;  // same warp roles as the single-CTA engine

template <int BN, int KIND, int NSEG>
struct PairSmem {
  static constexpr bool kOutF32 = (KIND == EPI_F32 || KIND == EPI_RESID);
  static constexpr bool kStores = (KIND != EPI_CE);
  static constexpr int kAStage = kBM * kBK * 2;         // 16 KB: this CTA's 128 rows
  static constexpr int kBStage = (BN / 2) * kBK * 2;    // this CTA's BN/2 rows of W
  static constexpr int kStageBytes = kAStage + kBStage;
  static constexpr int kStageOutBytes = kStores ? (kOutF32 ? 4096 : 2048) : 0;
  static constexpr int kOutBytes = kStageOutBytes * kEpiWarps;
  static constexpr int kLoraU = kBM * kMaxRank * 2;           // 4 KB per segment
  static constexpr int kLoraB = (BN / 2) * kMaxRank * 2;      // BN/2 x 32 B per segment
  static constexpr int kLoraBuf = NSEG * (kLoraU + kLoraB);
  // Two or more segments: one operand buffer, so the shared memory goes to a deeper K pipeline
  // (the LoRA warp fills it for the next tile during that tile's whole main loop).
  static constexpr int kLoraBufs = NSEG >= 2 ? 1 : 2;
  static constexpr int kLoraBytes = kLoraBufs * kLoraBuf;
  static constexpr int kVarBytes = NSEG ? kMaxGroups * 20 : 0;
  static constexpr int kBudget = 227 * 1024;  // the opt-in per-CTA limit (232448 B)
  static constexpr int kFree = kBudget - kOutBytes - kLoraBytes - kVarBytes - 1024 - 256;
  static constexpr int kStages = (kFree / kStageBytes) > 8 ? 8 : (kFree / kStageBytes);
  static constexpr int kOutOff = kStages * kStageBytes;
  static constexpr int kLoraOff = kOutOff + kOutBytes;
  static constexpr int kVarOff = kLoraOff + kLoraBytes;
  static constexpr int kBarOff = kVarOff + kVarBytes;
  static constexpr int kTotal = kBarOff + 256 + 1024;
  static constexpr int kAccStride = BN <= 128 ? 128 : 256;
  static constexpr int kTmemCols = 2 * kAccStride;
  static_assert(kTotal <= 227 * 1024, "shared memory over the 227 KB per-CTA limit");
  static_assert(kStages >= 2, "pipeline needs at least two stages");
  static_assert(kBStage % 1024 == 0 && kLoraOff % 1024 == 0 && kOutOff % 1024 == 0, "swizzle alignment");
};

// Output tiles of a pair launch: num_m row tiles of 256 rows times nfull column tiles of BN columns, then
// (when N is not a multiple of BN and the epilogue allows it) one column tile per row tile of nw_last
// columns, issued as narrower MMAs instead of BN-wide ones over zero-filled W rows. Tile i < num_m * nfull
// is (row i / nfull, column i % nfull); the narrow tiles follow in row order. In round r cluster c takes
// tile r * ncl + (r odd ? ncl - 1 - c : c), so the cheap narrow tiles at the end of the order go first to
// the clusters that received one full tile fewer.
struct PairTiles {
  int num_m, nfull, nw_last, total;
};

template <int BN>
__device__ __forceinline__ PairTiles pair_tiles(int M, int N, bool narrow) {
  PairTiles t;
  t.num_m = (M + 2 * kBM - 1) / (2 * kBM);
  if (narrow) {
    t.nfull = N / BN;
    const int rem = N - t.nfull * BN;
    t.nw_last = (rem + 31) & ~31;  // a multiple of 32 columns: 16 W rows per CTA at least
  } else {
    t.nfull = (N + BN - 1) / BN;
    t.nw_last = 0;
  }
  t.total = t.num_m * (t.nfull + (t.nw_last > 0 ? 1 : 0));
  return t;
}

__device__ __forceinline__ int pair_tile_at(int r, int cid, int ncl) {
  return r * ncl + ((r & 1) ? ncl - 1 - cid : cid);
}

// tile i -> row tile mt, column tile nt, first column n0, width nw
template <int BN>
__device__ __forceinline__ void pair_tile(const PairTiles& t, int i, int& mt, int& nt, int& n0, int& nw) {
  const int nf = t.num_m * t.nfull;
  if (i < nf) {
    mt = i / t.nfull;
    nt = i - mt * t.nfull;
    nw = BN;
  } else {
    mt = i - nf;
    nt = t.nfull;
    nw = t.nw_last;
  }
  n0 = nt * BN;
}

template <int BN, int KIND, typename OutT, bool BF16, int NSEG, int OPM = 0>
__global__ void __launch_bounds__(kPairThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                     const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmU, int M, int N,
                     int K, EpiParams ep) {
  using S = PairSmem<BN, KIND, NSEG>;
  constexpr int STAGES = S::kStages;
  constexpr bool LORA = NSEG > 0;
  constexpr int NCHUNK = (KIND == EPI_SWIGLU) ? BN / 64 : BN / 32;
  constexpr int HB = BN / 2;  // W rows per CTA
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "BN must be a multiple of 32 in [64, 256]");
  static_assert(KIND != EPI_SWIGLU || BN % 64 == 0, "SwiGLU tiles hold two halves of 32-column chunks");
  static_assert(OPM == 0 || (NSEG == 0 && BN % 128 == 0), "MN-major operands: plain tiles of 128 or 256 columns");
  constexpr bool A_MN = (OPM & 1) != 0, B_MN = (OPM & 2) != 0;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::kAStage;
  uint8_t* sOut = smem + S::kOutOff;
  uint8_t* sL = smem + S::kLoraOff;  // buffer b: [NSEG x U tile][NSEG x Bv tile]
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
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const uint32_t peer = rank ^ 1u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * kEpiWarps);
      mbar_init(&lfull_bar[a], 2);
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
    tmem_alloc_pair(tmem_holder, S::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_enter();  // the previous kernel's outputs are complete from here on

  // SwiGLU tiles interleave gate and up halves and the cross-entropy partials are indexed per BN tile:
  // those two keep BN-wide tiles throughout
  const PairTiles tl = pair_tiles<BN>(M, N, KIND != EPI_SWIGLU && KIND != EPI_CE);
  const int kblocks = (K + kBK - 1) / kBK;
  const int cid = (int)cluster_id_x(), ncl = (int)nclusters_x();

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int r = 0; ok; ++r) {
        const int tile = pair_tile_at(r, cid, ncl);
        if (tile >= tl.total) break;
        int mt, nt, n0, nw;
        pair_tile<BN>(tl, tile, mt, nt, n0, nw);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, ep.status, DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          const uint32_t fb = mapa_shared(smem_u32(&full_bar[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * S::kStageBytes);
          if (A_MN) {
#pragma unroll
            for (int at = 0; at < kBM / 64; ++at)
              tma_load_2d_pair(sA + stage * S::kAStage + at * 8192, &tmX, fb, mt * 2 * kBM + (int)rank * kBM + at * 64,
                               kb * kBK);
          } else {
            tma_load_2d_pair(sA + stage * S::kAStage, &tmX, fb, kb * kBK, mt * 2 * kBM + (int)rank * kBM);
          }
          if (B_MN) {
#pragma unroll
            for (int at = 0; at < HB / 64; ++at)
              tma_load_2d_pair(sB + stage * S::kBStage + at * 8192, &tmW, fb, n0 + (int)rank * (nw / 2) + at * 64,
                               kb * kBK);
          } else {
            tma_load_2d_pair(sB + stage * S::kBStage, &tmW, fb, kb * kBK, n0 + (int)rank * (nw / 2));
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && leader) {
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
    // ---------------- UMMA issuer (leader only) ----------------
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      int lb = 0;
      uint32_t lphase = 0;
      bool ok = true;
      bool issued_any = false;
      for (int r = 0; ok; ++r) {
        const int tile = pair_tile_at(r, cid, ncl);
        if (tile >= tl.total) break;
        int mt, nt, n0, nw;
        pair_tile<BN>(tl, tile, mt, nt, n0, nw);
        const uint32_t idesc_l = umma_idesc_f16(BF16, 2 * kBM, nw);  // K-major (LoRA step)
        const uint32_t idesc = idesc_l | (A_MN ? (1u << 15) : 0u) | (B_MN ? (1u << 16) : 0u);
        if (!mbar_wait_cluster(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, ep.status, DEV_TIMEOUT_MMA)) {
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
          // K-major: +32 B per K = 16 step inside the swizzle atom; MN-major: +16 K rows (2048 B)
          const uint64_t adesc = A_MN ? sw128_mn_desc(smem_u32(sA + stage * S::kAStage), 8192)
                                      : sw128_kmajor_desc(smem_u32(sA + stage * S::kAStage));
          const uint64_t bdesc = B_MN ? sw128_mn_desc(smem_u32(sB + stage * S::kBStage), 8192)
                                      : sw128_kmajor_desc(smem_u32(sB + stage * S::kBStage));
          constexpr uint64_t a_step = A_MN ? (2048u >> 4) : 2u, b_step = B_MN ? (2048u >> 4) : 2u;
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k)
            umma_f16_ss_pair(d_tmem, adesc + a_step * k, bdesc + b_step * k, idesc, (kb | k) != 0 ? 1u : 0u);
          issued_any = true;
          const uint32_t eb = smem_u32(&empty_bar[stage]);
          umma_commit_pair(eb);
          umma_commit_pair(mapa_shared(eb, peer));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (LORA) {
          if (!mbar_wait_cluster(&lfull_bar[lb], lphase, abort_flag, ep.status, DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* buf = sL + lb * S::kLoraBuf;
#pragma unroll
          for (int s = 0; s < NSEG; ++s)
            umma_f16_ss_pair(d_tmem, sw32_kmajor_desc(smem_u32(buf + s * S::kLoraU)),
                             sw32_kmajor_desc(smem_u32(buf + NSEG * S::kLoraU + s * S::kLoraB)), idesc_l, 1u);
          const uint32_t le = smem_u32(&lempty_bar[lb]);
          umma_commit_pair(le);
          umma_commit_pair(mapa_shared(le, peer));
          if (++lb == S::kLoraBufs) {
            lb = 0;
            lphase ^= 1u;
          }
        }
        const uint32_t tf = smem_u32(&tfull_bar[acc]);
        umma_commit_pair(tf);
        umma_commit_pair(mapa_shared(tf, peer));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && issued_any) {
        umma_commit_pair(smem_u32(drain_bar));
        mbar_wait_drain(drain_bar, 0);
      }
    }
  } else if (warp == 2) {
    // ---------------- LoRA operand warp (both CTAs) ----------------
    if (LORA) {
      int* s_gvar = reinterpret_cast<int*>(smem + S::kVarOff);
      VariantInfo* s_var = reinterpret_cast<VariantInfo*>(smem + S::kVarOff + kMaxGroups * 4);
      for (int i = lane; i < ep.lora.n_groups; i += 32) s_gvar[i] = ep.lora.group_variant[i];
      for (int i = lane; i < ep.lora.n_variants; i += 32) s_var[i] = ep.lora.variants[i];
      __syncwarp();
      constexpr int RPL = (HB + 31) / 32;
      int lb = 0;
      uint32_t lphase = 0;
      const int rank_r = ep.lora.rank;
      for (int r = 0;; ++r) {
        const int tile = pair_tile_at(r, cid, ncl);
        if (tile >= tl.total) break;
        int mt, nt, n0, nw;
        pair_tile<BN>(tl, tile, mt, nt, n0, nw);
        const int hw = nw / 2;                               // W rows of this CTA in this tile
        const int m0 = mt * 2 * kBM + (int)rank * kBM;      // this CTA's first row
        const int c0 = n0 + (int)rank * hw;                  // this CTA's first W row / output column
        const VariantInfo vi = s_var[s_gvar[(mt * 2 * kBM) / ep.lora.group_rows]];
        const uint32_t* mask = ep.lora.masks + (long long)(vi.mode ? vi.mask_slot : 0) * ep.lora.mask_words;
        float4 th[RPL][2];
        uint32_t mw[RPL];
        int sg[RPL];
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
          const int col = c0 + lane + 32 * i;
          int seg = 0, rel;
          if (NSEG == 2 && ep.lora.inter128) {
            seg = (col >> 7) & 1;
            rel = ((col >> 8) << 7) + (col & 127);
          } else {
#pragma unroll
            for (int s = 1; s < NSEG; ++s)
              if (col >= ep.lora.seg_start[s]) seg = s;
            rel = col - ep.lora.seg_start[seg];
          }
          const bool ok = lane + 32 * i < hw && col < N;
          sg[i] = ok ? seg : -1;
          const long long p0 = ep.lora.seg_boff[seg] + (long long)rel * rank_r;
          th[i][0] = ok ? __ldg(reinterpret_cast<const float4*>(ep.lora.theta + p0)) : make_float4(0.f, 0.f, 0.f, 0.f);
          th[i][1] = (ok && rank_r > 4) ? __ldg(reinterpret_cast<const float4*>(ep.lora.theta + p0 + 4))
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
          mw[i] = (ok && vi.mode) ? (__ldg(mask + (p0 >> 5)) >> (p0 & 31)) : 0u;
        }
        int okw = 1;
        if (lane == 0) okw = mbar_wait(&lempty_bar[lb], lphase ^ 1u, abort_flag, ep.status, DEV_TIMEOUT_PRODUCER);
        okw = __shfl_sync(0xffffffffu, okw, 0);
        if (!okw) break;
        uint8_t* buf = sL + lb * S::kLoraBuf;
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
          const int n = lane + 32 * i;
          if (n < HB) {
            float b[8] = {th[i][0].x, th[i][0].y, th[i][0].z, th[i][0].w,
                          th[i][1].x, th[i][1].y, th[i][1].z, th[i][1].w};
            if (vi.mode) {
#pragma unroll
              for (int j = 0; j < 8; ++j)
                if (j < rank_r) b[j] = perturb_value(b[j], (mw[i] >> j) & 1u, vi);
            }
            uint4 w0;
            w0.x = pack2<OutT>(b[0], b[1]);
            w0.y = pack2<OutT>(b[2], b[3]);
            w0.z = pack2<OutT>(b[4], b[5]);
            w0.w = pack2<OutT>(b[6], b[7]);
            const uint4 z = make_uint4(0u, 0u, 0u, 0u);
            const int sw = (n >> 2) & 1;  // SWIZZLE_32B: chunk c of row n at c ^ ((n >> 2) & 1)
#pragma unroll
            for (int s = 0; s < NSEG; ++s) {
              uint8_t* rowp = buf + NSEG * S::kLoraU + s * S::kLoraB + n * 32;
              *reinterpret_cast<uint4*>(rowp + ((0 ^ sw) << 4)) = (sg[i] == s) ? w0 : z;
              *reinterpret_cast<uint4*>(rowp + ((1 ^ sw) << 4)) = z;
            }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const uint32_t lf = mapa_shared(smem_u32(&lfull_bar[lb]), 0);
          if (leader) mbar_arrive_expect_tx(&lfull_bar[lb], 2 * NSEG * S::kLoraU);
#pragma unroll
          for (int s = 0; s < NSEG; ++s) tma_load_2d_pair(buf + s * S::kLoraU, &tmU, lf, ep.lora.seg_ucol[s], m0);
          if (!leader) mbar_arrive_cluster(lf);
        }
        if (++lb == S::kLoraBufs) {
          lb = 0;
          lphase ^= 1u;
        }
      }
    }
  } else {
    // ---------------- Epilogue (warps 3..10, both CTAs, own 128 rows) ----------------
    const int ew = warp - kFirstEpiWarp;
    const int lg = warp & 3;
    const int half = ew >> 2;
    const int row_in_tile = lg * 32 + lane;
    const int et = threadIdx.x - kFirstEpiWarp * 32;
    uint8_t* box = sOut + ew * S::kStageOutBytes;
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty_bar[0]), 0);
    const uint32_t tempty_leader1 = mapa_shared(smem_u32(&tempty_bar[1]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int r = 0;; ++r) {
      const int tile = pair_tile_at(r, cid, ncl);
      if (tile >= tl.total) break;
      int mt, nt, n0, nw;
      pair_tile<BN>(tl, tile, mt, nt, n0, nw);
      const int m0 = mt * 2 * kBM + (int)rank * kBM;
      const int nch = (KIND == EPI_SWIGLU) ? NCHUNK : nw / 32;
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
      named_bar_sync(2, 32 * kEpiWarps);
      if (et == 0) *epi_abort = *abort_flag;
      named_bar_sync(2, 32 * kEpiWarps);
      if (*epi_abort) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + acc * S::kAccStride + ((uint32_t)(lg * 32) << 16);

      float ce_m = -INFINITY, ce_s = 0.f;
      int tgt = -1;
      if (KIND == EPI_CE && row_ok) tgt = ep.targets[row];

#pragma unroll 1
      for (int ch = half; ch < nch; ch += 2) {
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
        if (lane == 0) bulk_wait_read0();
        __syncwarp();
        stage_row<S::kOutF32, OutT>(box, lane, v);
        fence_proxy_async_smem();
        __syncwarp();
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
      if (lane == 0) {
        if (leader)
          mbar_arrive(&tempty_bar[acc]);
        else
          mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (S::kStores && lane == 0) bulk_wait0();
  }

  tc_fence_before();
  cluster_sync();  // neither CTA leaves while its peer may still touch its barriers or TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, S::kTmemCols);
  }
}

}  // namespace b2p
