// attn_bwd_tc.cu — causal GQA attention backward on the tcgen05 tensor cores, for
// sequences of 128 or 256 tokens (cpu_sdpa_backward, training/cpu_ops.h:213-290,
// with gqa_tile_kv / gqa_reduce_kv, training/io.h:439-459, and the inverse RoPE of
// rope_backward_inplace, cpu_ops.h:377-393).
//
// P is recomputed from the forward's row normaliser (log2 domain), D_i = sum_d dO_i,d O_i,d
// (computed beforehand) stands for the reference's sum_j dP_ij P_ij, dS = P (dP - D) / sqrt(hd).
// Two deterministic passes, each a persistent kernel with the unit scheduling, TMA
// producer, polling MMA issuer and two alternating softmax warpgroups of the forward,
// plus an epilogue warpgroup that writes a finished unit's accumulators (staged in shared
// memory, stored by TMA) while the softmax groups go on with the next unit:
//
//   DKDV: unit = (sequence, KV head, 128-key block); the block's K and V stay in shared
//         memory while 64-query chunks (Q, dO) of its query heads stream through:
//           S^T = K Q^T, dP^T = V dO^T            (tcgen05, M = 128 keys, N = 64 queries)
//           P^T, dS^T written back into TMEM as 16-bit over the consumed S^T, dP^T columns
//           dV += P^T dO, dK += dS^T Q             (A = P^T / dS^T from TMEM, B = dO / Q MN-major)
//         dK (inverse RoPE) and dV leave summed over the GQA group.
//   DQ:   unit = (sequence, query head, 128-query block); Q and dO stay, 64-key chunks (K, V)
//         stream: S = Q K^T, dP = dO V^T, dS into TMEM, dQ += dS K; dQ leaves with inverse RoPE.
//
// The same shared-memory tile serves as a K-major operand (S, dP) and as an MN-major
// operand (dV, dK, dQ): both are 64-element, 128-byte-swizzled rows. The row normalisers
// and D values a chunk (DKDV) or unit (DQ) needs arrive by cp.async on the same barrier
// as its tiles. dS is kept unscaled in 16 bit; the 1/sqrt(hd) factor (a power of two for
// hd = 64) is applied to dK and dQ in fp32 in the epilogue.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "engine.cuh"
#include "kernels.cuh"
#include "mma.cuh"
#include "ptx.cuh"

namespace b2p {
namespace {

constexpr int kBR = 128;   // stationary rows per unit (UMMA M)
constexpr int kBC = 64;    // moving rows per chunk (UMMA N of S, dP; K of the accumulating MMAs)
constexpr int kHD = 64;
// warp 0 TMA producer + TMEM owner, 1 MMA issuer, 2-5 and 6-9 softmax groups, 10-13 epilogue
constexpr int kBwThreads = 448;
constexpr int kBwRing = 4;
constexpr int kMvStages = 4;  // moving chunks in flight (their TMA loads run ahead of the MMAs)

struct BwSmem {
  static constexpr int kStat = kBR * kHD * 2;            // 16 KB: one 128-row stationary tile
  static constexpr int kMove = kBC * kHD * 2;            // 8 KB: one 64-row moving tile
  static constexpr int kSlab = 32 * kHD * 2;             // 4 KB: one epilogue warp's 32 output rows
  static constexpr int kStatOff = 0;                     // [2 stages][2 tiles]
  static constexpr int kMoveOff = kStatOff + 4 * kStat;  // [kMvStages][2 tiles]
  static constexpr int kOutOff = kMoveOff + 2 * kMvStages * kMove;  // [4 warps][2 slabs] (DQ uses one)
  static constexpr int kMvVecOff = kOutOff + 8 * kSlab;            // [kMvStages][64] (lse, D) of the moving queries
  static constexpr int kStVecOff = kMvVecOff + kMvStages * kBC * 8;  // [2 stages][128] (lse, D) of the stationary queries
  static constexpr int kBarOff = kStVecOff + 2 * kBR * 8;
  static constexpr int kNumBars = 12 + 2 * kMvStages + 2 * kBwRing + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kTotal = kMiscOff + 64 + 1024;
  static_assert(kOutOff % 1024 == 0, "128-byte-swizzled staging needs 1024-byte alignment");
};

__device__ __forceinline__ uint64_t bw_mn_desc(uint32_t saddr) {  // MN-major, 128B swizzle, one N atom
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

__device__ __forceinline__ void bw_umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void bw_tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

__device__ __forceinline__ void bw_tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// tcgen05.wait::ld with the loaded registers as operands, so no use of them moves above it
__device__ __forceinline__ void bw_ld_wait2(uint32_t (&r)[16], uint32_t (&q)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(q[0]), "+r"(q[1]), "+r"(q[2]), "+r"(q[3]), "+r"(q[4]), "+r"(q[5]), "+r"(q[6]),
                 "+r"(q[7]), "+r"(q[8]), "+r"(q[9]), "+r"(q[10]), "+r"(q[11]), "+r"(q[12]), "+r"(q[13]),
                 "+r"(q[14]), "+r"(q[15])
               :
               : "memory");
}

__device__ __forceinline__ void bw_ld_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

__device__ __forceinline__ float bw_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 4-byte global -> shared copy whose completion a later cp_async_arrive_noinc reports
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
// one of the barrier's expected arrivals, made once this thread's cp.async copies have landed
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Unit u -> (sequence g, head index hh (KV head for DKDV, query head for DQ), block blk),
// heaviest blocks first. Chunk count: DKDV gq * (seq/64 - 2 blk), DQ 2 blk + 2.
template <bool DKDV>
struct BwUnit {
  int g, hh, blk, nch;
};

template <bool DKDV>
__device__ __forceinline__ BwUnit<DKDV> bw_unit(int u, const AttnBwdArgs& a) {
  const int nheads = DKDV ? a.kv_heads : a.heads;
  const int per = a.ngroups * nheads;
  const int nblk = a.seq / kBR;
  BwUnit<DKDV> r;
  r.blk = DKDV ? u / per : nblk - 1 - u / per;
  const int rem = u % per;
  r.g = rem / nheads;
  r.hh = rem % nheads;
  const int gq = a.heads / a.kv_heads;
  r.nch = DKDV ? gq * (a.seq / kBC - 2 * r.blk) : 2 * r.blk + 2;
  return r;
}

// Rows of the moving chunk c of a unit: (head, first row within the sequence).
template <bool DKDV>
__device__ __forceinline__ void bw_chunk(const BwUnit<DKDV>& un, int c, const AttnBwdArgs& a, int& head, int& row0) {
  if (DKDV) {
    const int gq = a.heads / a.kv_heads;
    const int per = a.seq / kBC - 2 * un.blk;
    head = un.hh * gq + c / per;           // query head
    row0 = (2 * un.blk + c % per) * kBC;  // first query
  } else {
    head = un.hh / (a.heads / a.kv_heads);  // KV head
    row0 = c * kBC;                         // first key
  }
}

// P and unscaled dS of 16 moving columns of this lane's stationary row. DKDV: the moving
// rows are queries with (lse, D) pairs in lsed; DQ: one (lse, D) for the lane's query.
// MASK: the chunk crosses the diagonal (key > query is masked).
template <bool DKDV, bool MASK, typename T>
__device__ __forceinline__ void bw_math(const uint32_t (&sv)[16], const uint32_t (&dv)[16], const float4* lsed,
                                        float lse_r, float d_r, float scale_log2, int spos, int mpos0,
                                        uint32_t (&pk)[8], uint32_t (&dk)[8]) {
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    float l0, d0, l1, d1;
    if (DKDV) {
      const float4 v = lsed[i >> 1];
      l0 = v.x;
      d0 = v.y;
      l1 = v.z;
      d1 = v.w;
    } else {
      l0 = l1 = lse_r;
      d0 = d1 = d_r;
    }
    float p0 = bw_exp2(fmaf(__uint_as_float(sv[i]), scale_log2, -l0));
    float p1 = bw_exp2(fmaf(__uint_as_float(sv[i + 1]), scale_log2, -l1));
    if (MASK) {
      const int m = mpos0 + i;
      if (DKDV ? (spos > m) : (m > spos)) p0 = 0.f;
      if (DKDV ? (spos > m + 1) : (m + 1 > spos)) p1 = 0.f;
    }
    pk[i >> 1] = pack_h2<T>(p0, p1);
    dk[i >> 1] = pack_h2<T>(p0 * (__uint_as_float(dv[i]) - d0), p1 * (__uint_as_float(dv[i + 1]) - d1));
  }
}

// 32 fp32 accumulator columns (half h of a 64-column row) -> 16-bit chunks 4h..4h+3 of the row
// in a 128-byte-swizzled staging slab (chunk c of row r at c ^ (r & 7)), times `mul`, with the
// inverse RoPE when cs/sn (the row's cos/sin tables) are given: pairs (2i, 2i+1) of position
// pos (rope_backward_inplace, cpu_ops.h:377-393).
template <typename T>
__device__ __forceinline__ void bw_stage_half(uint8_t* slab, int r, int h, const uint32_t (&v)[32], float mul,
                                              const float* cs, const float* sn) {
  const uint32_t row_addr = smem_u32(slab) + r * 128;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int c = 4 * h + q;
    float x[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = __uint_as_float(v[q * 8 + e]) * mul;
    if (cs != nullptr) {
      const float4 c4 = __ldg(reinterpret_cast<const float4*>(cs) + c);
      const float4 s4 = __ldg(reinterpret_cast<const float4*>(sn) + c);
      const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float x0 = x[2 * e], x1 = x[2 * e + 1];
        x[2 * e] = x0 * cc[e] + x1 * ss[e];
        x[2 * e + 1] = -x0 * ss[e] + x1 * cc[e];
      }
    }
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(row_addr + ((c ^ (r & 7)) << 4)),
                 "r"(pack_h2<T>(x[0], x[1])), "r"(pack_h2<T>(x[2], x[3])), "r"(pack_h2<T>(x[4], x[5])),
                 "r"(pack_h2<T>(x[6], x[7]))
                 : "memory");
  }
}

template <typename T, bool DKDV>
__global__ void __launch_bounds__(kBwThreads, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_dq, AttnBwdArgs a, int total_units, uint32_t* status) {
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* s_stat = smem + BwSmem::kStatOff;
  uint8_t* s_move = smem + BwSmem::kMoveOff;
  uint8_t* s_out = smem + BwSmem::kOutOff;
  float2* s_mvvec = reinterpret_cast<float2*>(smem + BwSmem::kMvVecOff);
  float2* s_stvec = reinterpret_cast<float2*>(smem + BwSmem::kStVecOff);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BwSmem::kBarOff);
  uint64_t* st_full = bars;        // [2] stationary tiles of a unit (DQ: + its (lse, D))
  uint64_t* st_empty = bars + 2;
  uint64_t* s_full = bars + 4;     // [2] S, dP of a chunk in TMEM
  uint64_t* p_full = bars + 6;     // [2] P, dS written back
  uint64_t* acc_full = bars + 8;   // [2] a unit's accumulators complete
  uint64_t* acc_empty = bars + 10;
  uint64_t* mv_full = bars + 12;   // [kMvStages] moving chunk (DKDV: + its (lse, D))
  uint64_t* mv_empty = mv_full + kMvStages;
  uint64_t* u_full = mv_empty + kMvStages;
  uint64_t* u_empty = u_full + kBwRing;
  uint64_t* drain_bar = u_empty + kBwRing;
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + BwSmem::kMiscOff);
  uint32_t* tmem_holder = misc;
  volatile uint32_t* abort_flag = misc + 1;
  volatile uint32_t* wg_abort = misc + 2;  // [2]
  volatile int* ring = reinterpret_cast<volatile int*>(misc + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kMvStages; ++i) {
      mbar_init(&mv_full[i], DKDV ? 1 + 32 : 1);  // + the producer lanes' cp.async arrivals
      mbar_init(&mv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&st_full[i], DKDV ? 1 : 1 + 32);
      mbar_init(&st_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);     // the chunk's softmax warps
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);  // the epilogue warps
    }
    for (int i = 0; i < kBwRing; ++i) {
      mbar_init(&u_full[i], 1);
      mbar_init(&u_empty[i], 1 + 8 + 4);  // issuer, softmax warps, epilogue warps
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    wg_abort[0] = wg_abort[1] = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_qkv);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_dq);
  }
  if (warp == 0) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_enter();  // the previous kernel's outputs are complete from here on

  if (warp == 0) {
    // ---------------- TMA producer (lane 0) + (lse, D) copies (all lanes) ----------------
    int k = 0, t = 0;
    bool ok = true;
    for (;; ++k) {
      const int slot = k % kBwRing;
      int u = 0;
      if (lane == 0) {
        ok = mbar_wait(&u_empty[slot], ((uint32_t)(k / kBwRing) & 1u) ^ 1u, abort_flag, status, DEV_TIMEOUT_PRODUCER);
        if (ok) {
          u = atomicAdd(a.sched, 1);
          ring[slot] = u;
          mbar_arrive(&u_full[slot]);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      u = __shfl_sync(0xffffffffu, u, 0);
      if (!ok || u >= total_units) break;
      const BwUnit<DKDV> un = bw_unit<DKDV>(u, a);
      const int ss = k & 1;
      if (lane == 0)
        ok = mbar_wait(&st_empty[ss], ((uint32_t)(k >> 1) & 1u) ^ 1u, abort_flag, status, DEV_TIMEOUT_PRODUCER);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      // stationary: DKDV K, V of the key block; DQ Q, dO of the query block (two 64-row boxes each)
      const int srow = un.g * a.seq + un.blk * kBR;
      if (lane == 0) {
        mbar_arrive_expect_tx(&st_full[ss], 2u * BwSmem::kStat);
        uint8_t* s0 = s_stat + (2 * ss) * BwSmem::kStat;
        uint8_t* s1 = s0 + BwSmem::kStat;
        for (int hb = 0; hb < 2; ++hb) {
          if (DKDV) {
            tma_load_2d(s0 + hb * BwSmem::kMove, &tm_qkv, &st_full[ss], a.k_off + un.hh * kHD, srow + hb * kBC);
            tma_load_2d(s1 + hb * BwSmem::kMove, &tm_qkv, &st_full[ss], a.v_off + un.hh * kHD, srow + hb * kBC);
          } else {
            tma_load_2d(s0 + hb * BwSmem::kMove, &tm_qkv, &st_full[ss], a.q_off + un.hh * kHD, srow + hb * kBC);
            tma_load_2d(s1 + hb * BwSmem::kMove, &tm_do, &st_full[ss], un.hh * kHD, srow + hb * kBC);
          }
        }
      }
      if (!DKDV) {  // (lse, D) of the block's 128 queries, head hh
        const uint32_t dst = smem_u32(s_stvec + ss * kBR);
        for (int q = lane; q < kBR; q += 32) {
          const long long i = (long long)(srow + q) * a.heads + un.hh;
          cp_async4(dst + q * 8, a.lse + i);
          cp_async4(dst + q * 8 + 4, a.dvec + i);
        }
        cp_async_arrive_noinc(&st_full[ss]);
      }
      for (int c = 0; c < un.nch && ok; ++c, ++t) {
        const int mb = t % kMvStages;
        if (lane == 0)
          ok = mbar_wait(&mv_empty[mb], ((uint32_t)(t / kMvStages) & 1u) ^ 1u, abort_flag, status,
                         DEV_TIMEOUT_PRODUCER);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        int head, row0;
        bw_chunk<DKDV>(un, c, a, head, row0);
        const int mrow = un.g * a.seq + row0;
        if (lane == 0) {
          uint8_t* m0 = s_move + (2 * mb) * BwSmem::kMove;
          mbar_arrive_expect_tx(&mv_full[mb], 2u * BwSmem::kMove);
          if (DKDV) {  // Q, dO of 64 queries of query head `head`
            tma_load_2d(m0, &tm_qkv, &mv_full[mb], a.q_off + head * kHD, mrow);
            tma_load_2d(m0 + BwSmem::kMove, &tm_do, &mv_full[mb], head * kHD, mrow);
          } else {     // K, V of 64 keys of KV head `head`
            tma_load_2d(m0, &tm_qkv, &mv_full[mb], a.k_off + head * kHD, mrow);
            tma_load_2d(m0 + BwSmem::kMove, &tm_qkv, &mv_full[mb], a.v_off + head * kHD, mrow);
          }
        }
        if (DKDV) {  // (lse, D) of the chunk's 64 queries
          const uint32_t dst = smem_u32(s_mvvec + mb * kBC);
          for (int q = lane; q < kBC; q += 32) {
            const long long i = (long long)(mrow + q) * a.heads + head;
            cp_async4(dst + q * 8, a.lse + i);
            cp_async4(dst + q * 8 + 4, a.dvec + i);
          }
          cp_async_arrive_noinc(&mv_full[mb]);
        }
      }
      if (!ok) break;
    }
    if (!ok && lane == 0) {
      for (int i = 1; i <= kMvStages && t - i >= 0; ++i)
        mbar_wait_drain(&mv_full[(t - i) % kMvStages], ((uint32_t)((t - i) / kMvStages)) & 1u);
      for (int i = 1; i <= 2 && k - i >= 0; ++i) mbar_wait_drain(&st_full[(k - i) & 1], ((uint32_t)((k - i) >> 1)) & 1u);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == 1) {
    // ---------------- MMA issuer (polls: S/dP of the next chunk, or the accumulating MMAs of the oldest) ----------------
    if (lane == 0) {
      const uint32_t idesc_s = umma_idesc_f16(BF16, kBR, kBC);
      const uint32_t idesc_acc = umma_idesc_f16(BF16, kBR, kHD) | (1u << 16);  // B MN-major
      int t_s = 0, t_p = 0, k = 0, c = 0, k_p = 0, c_p = 0;
      bool need_unit = true, need_stat = false, done_s = false, issued_any = false, ok = true;
      BwUnit<DKDV> un{};
      int nch_p[4] = {0, 0, 0, 0};  // chunk count of units k_p .. (ring of 4, indexed by unit)
      uint64_t t_idle = 0;
      for (uint32_t it = 0;; ++it) {
        bool did = false;
        // accumulating MMAs of chunk t_p (unit k_p, chunk c_p) once its P / dS are in TMEM
        if (t_p < t_s && mbar_test_wait(&p_full[t_p & 1], (uint32_t)(t_p >> 1) & 1u) &&
            (c_p != 0 || mbar_test_wait(&acc_empty[k_p & 1], ((uint32_t)(k_p >> 1) & 1u) ^ 1u))) {
          tc_fence_after();
          const int b = t_p & 1, ab = k_p & 1, mb = t_p % kMvStages;
          const uint32_t s_tm = tmem_base + b * 128, dp_tm = s_tm + 64;
          const uint32_t acc_tm = tmem_base + 256 + ab * 128;
          const uint32_t m0 = smem_u32(s_move + (2 * mb) * BwSmem::kMove);
          for (int kk = 0; kk < kBC / 16; ++kk) {
            const uint32_t acc = (c_p > 0 || kk > 0) ? 1u : 0u;
            if (DKDV) {
              // dV += P^T dO (acc cols 64..127), dK += dS^T Q (acc cols 0..63)
              bw_umma_ts(acc_tm + 64, s_tm + kk * 8, bw_mn_desc(m0 + BwSmem::kMove + kk * 2048), idesc_acc, acc);
              bw_umma_ts(acc_tm, dp_tm + kk * 8, bw_mn_desc(m0 + kk * 2048), idesc_acc, acc);
            } else {
              // dQ += dS K
              bw_umma_ts(acc_tm, dp_tm + kk * 8, bw_mn_desc(m0 + kk * 2048), idesc_acc, acc);
            }
          }
          umma_commit(&mv_empty[mb]);
          if (c_p + 1 == nch_p[k_p & 3]) {
            umma_commit(&acc_full[ab]);
            umma_commit(&st_empty[k_p & 1]);
            ++k_p;
            c_p = 0;
          } else {
            ++c_p;
          }
          ++t_p;
          did = true;
        }
        if (!done_s && t_s < t_p + 2) {
          if (need_unit) {
            const int slot = k % kBwRing;
            if (mbar_test_wait(&u_full[slot], (uint32_t)(k / kBwRing) & 1u)) {
              const int u = ring[slot];
              mbar_arrive(&u_empty[slot]);
              if (u >= total_units) {
                done_s = true;
              } else {
                un = bw_unit<DKDV>(u, a);
                nch_p[k & 3] = un.nch;
                need_unit = false;
                need_stat = true;
                c = 0;
              }
              did = true;
            }
          } else if (need_stat) {
            if (mbar_test_wait(&st_full[k & 1], (uint32_t)(k >> 1) & 1u)) {
              need_stat = false;
              did = true;
            }
          } else if (mbar_test_wait(&mv_full[t_s % kMvStages], (uint32_t)(t_s / kMvStages) & 1u)) {
            tc_fence_after();
            const int b = t_s & 1;
            const uint32_t s_tm = tmem_base + b * 128;
            const uint32_t st0 = smem_u32(s_stat + (2 * (k & 1)) * BwSmem::kStat);
            const uint32_t m0 = smem_u32(s_move + (2 * (t_s % kMvStages)) * BwSmem::kMove);
            for (int kk = 0; kk < kHD / 16; ++kk) {
              umma_f16_ss(s_tm, sw128_kmajor_desc(st0 + kk * 32), sw128_kmajor_desc(m0 + kk * 32), idesc_s,
                          kk > 0 ? 1u : 0u);
              umma_f16_ss(s_tm + 64, sw128_kmajor_desc(st0 + BwSmem::kStat + kk * 32),
                          sw128_kmajor_desc(m0 + BwSmem::kMove + kk * 32), idesc_s, kk > 0 ? 1u : 0u);
            }
            umma_commit(&s_full[b]);
            issued_any = true;
            ++t_s;
            if (++c == un.nch) {
              ++k;
              need_unit = true;
            }
            did = true;
          }
        }
        if (done_s && t_p == t_s) break;
        if (did) {
          t_idle = 0;
        } else if ((it & 255u) == 0u) {
          if (*abort_flag) {
            ok = false;
            break;
          }
          const uint64_t now = sm_cycles();
          if (t_idle == 0) {
            t_idle = now;
          } else if (now - t_idle > kWaitBudgetCycles) {
            *abort_flag = 1;
            atomicCAS(status, 0u, (uint32_t)DEV_TIMEOUT_MMA);
            ok = false;
            break;
          }
        }
      }
      if (!ok && issued_any) {  // let the MMAs in flight finish before TMEM is released
        umma_commit(drain_bar);
        mbar_wait_drain(drain_bar, 0);
      }
    }
  } else if (warp < 10) {
    // ---------------- softmax warpgroups: chunk t goes to group t & 1 ----------------
    const int wg = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;     // stationary row in the tile
    const int wt = threadIdx.x - 64 - wg * 128;
    const uint32_t bar_id = 1 + wg;
    auto agree = [&](bool ok_wait) -> bool {
      named_bar_sync(bar_id, 128);
      if (wt == 0) wg_abort[wg] = (*abort_flag || !ok_wait) ? 1u : 0u;
      named_bar_sync(bar_id, 128);
      return wg_abort[wg] == 0;
    };
    int t = 0;
    bool stop = false;
    for (int k = 0; !stop; ++k) {
      const int slot = k % kBwRing;
      const bool okw = mbar_wait(&u_full[slot], (uint32_t)(k / kBwRing) & 1u, abort_flag, status, DEV_TIMEOUT_EPILOGUE);
      if (!agree(okw)) break;
      const int u = ring[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&u_empty[slot]);
      if (u >= total_units) break;
      const BwUnit<DKDV> un = bw_unit<DKDV>(u, a);
      const int spos = un.blk * kBR + r;  // this lane's stationary position (key for DKDV, query for DQ)
      float lse_r = 0.f, d_r = 0.f;       // DQ: this query row's lse and D (per query head)
      bool have_vec = DKDV;
      for (int c = 0; c < un.nch; ++c, ++t) {
        if ((t & 1) != wg) continue;
        const int b = t & 1;
        int head, row0;
        bw_chunk<DKDV>(un, c, a, head, row0);
        if (!agree(mbar_wait(&s_full[b], (uint32_t)(t >> 1) & 1u, abort_flag, status, DEV_TIMEOUT_EPILOGUE))) {
          stop = true;
          break;
        }
        tc_fence_after();
        // the (lse, D) copies completed with the barrier whose tiles S / dP were computed from
        const int mb = t % kMvStages;
        if (DKDV) {
          if (!mbar_wait(&mv_full[mb], (uint32_t)(t / kMvStages) & 1u, abort_flag, status, DEV_TIMEOUT_EPILOGUE)) {
            stop = true;
            break;
          }
        } else if (!have_vec) {
          if (!mbar_wait(&st_full[k & 1], (uint32_t)(k >> 1) & 1u, abort_flag, status, DEV_TIMEOUT_EPILOGUE)) {
            stop = true;
            break;
          }
          const float2 v = s_stvec[(k & 1) * kBR + r];
          lse_r = v.x;
          d_r = v.y;
          have_vec = true;
        }
        const bool diag = DKDV ? (row0 < un.blk * kBR + kBR - 1) : (row0 + kBC - 1 > un.blk * kBR);
        const uint32_t t_row = tmem_base + b * 128 + ((uint32_t)(quarter * 32) << 16);
#pragma unroll 1
        for (int qt = 0; qt < 4; ++qt) {  // 16 moving rows at a time
          uint32_t sv[16], dv[16];
          bw_tmem_ld16(t_row + qt * 16, sv);
          bw_tmem_ld16(t_row + 64 + qt * 16, dv);
          bw_ld_wait2(sv, dv);
          uint32_t pk[8], dk[8];
          const float4* lsed = reinterpret_cast<const float4*>(s_mvvec + mb * kBC + qt * 16);
          if (diag)
            bw_math<DKDV, true, T>(sv, dv, lsed, lse_r, d_r, a.scale_log2, spos, row0 + qt * 16, pk, dk);
          else
            bw_math<DKDV, false, T>(sv, dv, lsed, lse_r, d_r, a.scale_log2, spos, row0 + qt * 16, pk, dk);
          // P (DKDV only) over the S columns, dS over the dP columns, both already read
          if (DKDV) bw_tmem_st8(t_row + qt * 8, pk);
          bw_tmem_st8(t_row + 64 + qt * 8, dk);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[b]);
      }
    }
  } else {
    // ---------------- epilogue warpgroup: a unit's accumulators -> dK (inverse RoPE) and dV, or dQ ----------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    uint8_t* slab0 = s_out + quarter * 2 * BwSmem::kSlab;
    uint8_t* slab1 = slab0 + BwSmem::kSlab;
    for (int k = 0;; ++k) {
      const int slot = k % kBwRing;
      if (!mbar_wait(&u_full[slot], (uint32_t)(k / kBwRing) & 1u, abort_flag, status, DEV_TIMEOUT_EPILOGUE)) break;
      const int u = ring[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&u_empty[slot]);
      if (u >= total_units) break;
      const BwUnit<DKDV> un = bw_unit<DKDV>(u, a);
      const int ab = k & 1;
      if (!mbar_wait(&acc_full[ab], (uint32_t)(k >> 1) & 1u, abort_flag, status, DEV_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const uint32_t acc_row = tmem_base + 256 + ab * 128 + ((uint32_t)(quarter * 32) << 16);
      if (lane == 0) bulk_wait_read0();  // the previous unit's stores have read the staging slabs
      __syncwarp();
      const int pos = un.blk * kBR + r;
      // dK (DKDV) or dQ: 1/sqrt(hd) and the inverse RoPE; then dV (DKDV) as accumulated
      const int nout = DKDV ? 2 : 1;
      for (int o = 0; o < nout; ++o) {
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          uint32_t v[32];
          tmem_ld32(acc_row + o * 64 + h * 32, v);
          bw_ld_wait(v);
          if (o == nout - 1 && h == 1) {  // every accumulator column of this warp's rows read
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[ab]);
          }
          if (o == 0)
            bw_stage_half<T>(slab0, lane, h, v, a.scale, a.rope_cos + pos * 32, a.rope_sin + pos * 32);
          else
            bw_stage_half<T>(slab1, lane, h, v, 1.f, nullptr, nullptr);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int row = un.g * a.seq + un.blk * kBR + quarter * 32;
        if (DKDV) {
          tma_store_2d(&tm_dq, slab0, a.k_off + un.hh * kHD, row);
          tma_store_2d(&tm_dq, slab1, a.v_off + un.hh * kHD, row);
        } else {
          tma_store_2d(&tm_dq, slab0, a.q_off + un.hh * kHD, row);
        }
        bulk_commit();
      }
    }
    if (lane == 0) bulk_wait0();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.sched + 1, 1) == (int)gridDim.x - 1) {
      a.sched[0] = 0;
      a.sched[1] = 0;
      __threadfence();
    }
  }
}

template <typename T, bool DKDV>
int launch_bw(const AttnBwdArgs& a, cudaStream_t st) {
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  DeviceCtx* c = nullptr;
  int rc = ctx_get(&c);
  if (rc) return rc;
  const long long rows = (long long)a.ngroups * a.seq;
  CUtensorMap tq, td;
  if ((rc = make_tmap_2d(&tq, a.qkv, BF16 ? TM_BF16 : TM_F16, (uint64_t)a.ld, (uint64_t)rows, (uint64_t)a.ld, kHD,
                         kBC, 128)))
    return rc;
  if ((rc = make_tmap_2d(&td, a.dout, BF16 ? TM_BF16 : TM_F16, (uint64_t)a.ld_o, (uint64_t)rows, (uint64_t)a.ld_o,
                         kHD, kBC, 128)))
    return rc;
  CUtensorMap tdq;  // output: 64 columns x 32 rows per epilogue warp
  if ((rc = make_tmap_2d(&tdq, a.dqkv, BF16 ? TM_BF16 : TM_F16, (uint64_t)a.ld_d, (uint64_t)rows, (uint64_t)a.ld_d,
                         kHD, 32, 128)))
    return rc;
  const int total = a.ngroups * (DKDV ? a.kv_heads : a.heads) * (a.seq / kBR);
  const int grid = total < c->num_sms ? total : c->num_sms;
  static thread_local uint64_t attr_mask = 0;  // one per instantiation
  if (!(attr_mask & (1ull << (c->device & 63)))) {
    B2P_CHECK_CUDA(
        cudaFuncSetAttribute(attn_bwd_tc_kernel<T, DKDV>, cudaFuncAttributeMaxDynamicSharedMemorySize, BwSmem::kTotal));
    attr_mask |= 1ull << (c->device & 63);
  }
  B2P_CHECK_CUDA(launch_pdl(attn_bwd_tc_kernel<T, DKDV>, dim3(grid), dim3(kBwThreads), BwSmem::kTotal, st, tq, td,
                            tdq, a, total, c->status));
  B2P_POST_LAUNCH();
  return B2P_OK;
}

}  // namespace

bool attention_backward_tc_supported(const AttnBwdArgs& a) {
  return a.sched != nullptr && (a.seq == 128 || a.seq == 256) && a.ld % 8 == 0 && a.ld_o % 8 == 0 &&
         a.ld_d % 8 == 0 && a.q_off % 8 == 0 && a.k_off % 8 == 0 && a.v_off % 8 == 0 && a.kv_heads > 0 &&
         a.heads % a.kv_heads == 0;
}

int launch_attention_backward_tc(const AttnBwdArgs& a, bool bf16, cudaStream_t st) {
  B2P_REQUIRE(attention_backward_tc_supported(a), "tcgen05 attention backward needs seq 128 or 256, 16-byte "
                                                  "aligned operands and a unit counter");
  int rc = bf16 ? launch_bw<__nv_bfloat16, true>(a, st) : launch_bw<__half, true>(a, st);
  if (rc) return rc;
  return bf16 ? launch_bw<__nv_bfloat16, false>(a, st) : launch_bw<__half, false>(a, st);
}

}  // namespace b2p
