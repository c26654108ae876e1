// attn_tc.cu — causal GQA attention forward on the tcgen05 tensor cores, for
// sequences of 128 or 256 tokens (causal SDPA with the GQA tile of
// training/io.h:439-446 and training/cpu_ops.h:321-360; softmax with the
// 1/sqrt(64) scale, exact row maximum, fp32 sums).
//
// Work unit: (sequence g, KV head, 128-row query block qb). Its K and V rows
// [0, 128·(qb+1)) are loaded once by TMA and serve the unit's heads/kv_heads
// query heads. Persistent CTAs (one per SM) take units from a device counter,
// heaviest query blocks first; the counter resets itself when the last CTA
// finishes.
//
// Per query head (one 128 x 64 Q tile):
//   MMA warp:   S = Q·Kᵀ  (tcgen05.mma, M 128, N = keys, K 64) into TMEM
//   softmax:    two warpgroups share the head, one per half of its keys (A: the
//               first nkeys/2, B: the rest). Each reads its half of the S rows
//               (one TMEM lane per thread), takes the row maximum over its causal
//               keys; the two partial maxima meet in shared memory; each writes
//               P = exp2((s - max)·scale·log2e) as 16-bit pairs into its own part
//               of the consumed S columns (A at columns [0, nkeys/4), B at
//               [nkeys/2, 3·nkeys/4)), and the partial row sums meet the same way
//   MMA warp:   O = P·V   (A = P from TMEM, B = V in shared memory, MN-major),
//               O at columns [192, 256) of the buffer
//   softmax:    A writes output columns 0-31 of O / l, B columns 32-63, both in
//               16 bit with 64-byte row stores; A saves the row log2-sum-exp for
//               the backward.
// Two TMEM buffers of 256 columns and two warpgroup pairs alternate over the
// heads, so the softmax of one head overlaps the MMAs of the next; splitting a
// head's keys halves the serial softmax path of its rows.
//
// Warps: 0 TMEM owner and TMA producer, 1 and 18 the MMA issuers of buffers 0
// and 1, 2-9 the pair of buffer 0 (2-5 side A, 6-9 side B), 10-17 the pair of
// buffer 1 (warp % 4 selects the warp's 32-lane TMEM quarter). Head t's S is
// issued once head t-1 has its row maxima, so at most one pair is in its exp
// pass at a time.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "engine.cuh"
#include "kernels.cuh"
#include "mma.cuh"
#include "ptx.cuh"

namespace b2p {
namespace {

constexpr int kAtRows = 128;   // query rows per tile (UMMA M)
constexpr int kAtHD = 64;      // head dim
constexpr int kAtMaxKeys = 256;
constexpr int kAtThreads = 608;   // 3 + 16 warps
constexpr int kAtSoftWarps = 8;    // per buffer: 4 on each half of the keys
constexpr int kAtOCol = 192;       // O = P·V columns inside a 256-column buffer
constexpr int kAtRing = 4;     // unit-id ring between the producer and the consumers
constexpr int kAtBatch = 1;    // 32-key chunks per TMEM round trip in the softmax passes
constexpr uint32_t kAtTmemCols = 512;

struct AtSmem {
  static constexpr int kQ = kAtRows * kAtHD * 2;         // 16 KB Q tile
  static constexpr int kKV = kAtMaxKeys * kAtHD * 2;     // 32 KB K or V tile
  static constexpr int kQOff = 0;                        // 2 Q tiles (head double buffer)
  static constexpr int kKOff = kQOff + 2 * kQ;           // 2 K tiles (unit double buffer)
  static constexpr int kVOff = kKOff + 2 * kKV;          // 2 V tiles
  static constexpr int kBarOff = kVOff + 2 * kKV;
  static constexpr int kNumBars = 18 + 2 * kAtRing + 2;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kRedOff = kMiscOff + 64;           // [buffer][side][128] partial max, then sum
  static constexpr int kTotal = kRedOff + 2 * 2 * 128 * 4 + 1024;  // + 1024-byte alignment slack
};

// MN-major operand tile written by TMA with 128-byte swizzle: each 128-byte row
// holds 64 consecutive N elements at one K index; groups of 8 K rows sit 1024 B
// apart (SBO). The tile is one 64-element atom wide in N, so LBO is not used.
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;             // LBO (single atom in N)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;     // SBO: 8 K rows x 128 B
  d |= static_cast<uint64_t>(1u) << 46;             // descriptor version for sm_100
  d |= static_cast<uint64_t>(2u) << 61;             // SWIZZLE_128B
  return d;
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16 (A read from tensor memory).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 TMEM lanes x 32 bit, 16 consecutive columns <- 16 registers per thread.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Wait for this thread's outstanding tcgen05.ld; the destination registers pass
// through the wait so no use of them is scheduled above it.
__device__ __forceinline__ void tmem_ld_wait_regs(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// The SFU base-2 exponential (ex2.approx.ftz.f32; the inputs here are <= 0 and
// results below 2^-126 flush to zero, far below what a 16-bit P can hold).
__device__ __forceinline__ float sfu_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Max over a 32-key chunk; keys above `lim` (the query position) are masked when MASK.
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
template <bool MASK>
__device__ __forceinline__ float chunk_max(const uint32_t (&v)[32], float mx, int key0, int lim) {
  if (MASK) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (key0 + i <= lim) mx = fmaxf(mx, __uint_as_float(v[i]));
    return mx;
  }
  float m0 = mx, m1 = __uint_as_float(v[0]);
#pragma unroll
  for (int i = 1; i < 31; i += 4) {
    m0 = max3(m0, __uint_as_float(v[i]), __uint_as_float(v[i + 1]));
    m1 = max3(m1, __uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
  }
  return max3(m0, m1, __uint_as_float(v[31]));
}

// P = exp2(s·scale - ms) of a 32-key chunk as 16 packed 16-bit pairs; adds the
// fp32 values to l. Keys above `lim` (the query position) get P = 0 when MASK.
template <typename T, bool MASK>
__device__ __forceinline__ void chunk_exp(const uint32_t (&v)[32], uint32_t (&pk)[16], float& l, float scale,
                                          float ms, int key0, int lim) {
  float la = 0.f, lb = 0.f;
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    float p0 = sfu_exp2(fmaf(__uint_as_float(v[i]), scale, -ms));
    float p1 = sfu_exp2(fmaf(__uint_as_float(v[i + 1]), scale, -ms));
    if (MASK) {
      p0 = key0 + i <= lim ? p0 : 0.f;
      p1 = key0 + i + 1 <= lim ? p1 : 0.f;
    }
    la += p0;
    lb += p1;
    pk[i >> 1] = pack_h2<T>(p0, p1);
  }
  l += la + lb;
}

struct Unit {
  int g, kvh, qb, nkeys;
};

__device__ __forceinline__ Unit decode_unit(int u, const AttnArgs& a) {
  const int per_qb = a.ngroups * a.kv_heads;
  const int nqb = a.seq / kAtRows;
  Unit r;
  r.qb = nqb - 1 - u / per_qb;  // longest query blocks first
  const int rem = u % per_qb;
  r.g = rem / a.kv_heads;
  r.kvh = rem % a.kv_heads;
  r.nkeys = (r.qb + 1) * kAtRows;
  return r;
}

template <typename T>
__global__ void __launch_bounds__(kAtThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm, AttnArgs a, float scale_log2, int total_units,
                   uint32_t* status) {
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + AtSmem::kQOff;
  uint8_t* sK = smem + AtSmem::kKOff;
  uint8_t* sV = smem + AtSmem::kVOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + AtSmem::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 2;
  uint64_t* kv_full = bars + 4;
  uint64_t* kv_empty = bars + 6;
  uint64_t* s_full = bars + 8;
  uint64_t* p_full = bars + 10;
  uint64_t* o_full = bars + 12;
  uint64_t* t_empty = bars + 14;
  uint64_t* m_full = bars + 16;
  uint64_t* u_full = bars + 18;
  uint64_t* u_empty = u_full + kAtRing;
  uint64_t* drain_bar = u_empty + kAtRing;  // [2], one per MMA issuer
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + AtSmem::kMiscOff);
  uint32_t* tmem_holder = misc;
  volatile uint32_t* abort_flag = misc + 1;
  volatile uint32_t* wg_abort = misc + 2;  // [2]
  volatile int* ring = reinterpret_cast<volatile int*>(misc + 4);  // [kAtRing]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int gq = a.heads / a.kv_heads;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 2);            // both MMA issuers (each commits after its last use)
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kAtSoftWarps);   // one arrive per softmax warp of the buffer
      mbar_init(&o_full[i], 1);
      mbar_init(&t_empty[i], kAtSoftWarps);
      mbar_init(&m_full[i], kAtSoftWarps);   // the buffer's head has its row maxima
    }
    for (int i = 0; i < kAtRing; ++i) {
      mbar_init(&u_full[i], 1);
      mbar_init(&u_empty[i], 2 + 2 * kAtSoftWarps);  // both MMA threads + one arrive per softmax warp
    }
    mbar_init(&drain_bar[0], 1);
    mbar_init(&drain_bar[1], 1);
    *abort_flag = 0;
    wg_abort[0] = wg_abort[1] = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm);
  }
  if (warp == 0) {
    tmem_alloc(tmem_holder, kAtTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_enter();  // the previous kernel's outputs are complete from here on

  if (warp == 0) {
    // ---------------- TMA producer: unit ids, K/V per unit, Q per head ----------------
    if (lane == 0) {
      int t = 0, k = 0;
      bool ok = true;
      for (;; ++k) {
        const int slot = k % kAtRing;
        const uint32_t ph = (uint32_t)(k / kAtRing) & 1u;
        if (!mbar_wait(&u_empty[slot], ph ^ 1u, abort_flag, status, DEV_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        // the first unit of each CTA is its block index (no counter round trip at start-up); the
        // rest come from the counter, offset by the grid size
        const int u = k == 0 ? (int)blockIdx.x : (int)gridDim.x + atomicAdd(a.sched, 1);
        ring[slot] = u;
        mbar_arrive(&u_full[slot]);
        if (u >= total_units) break;
        const Unit un = decode_unit(u, a);
        const int kvs = k & 1;
        if (!mbar_wait(&kv_empty[kvs], ((uint32_t)(k >> 1) & 1u) ^ 1u, abort_flag, status, DEV_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&kv_full[kvs], (uint32_t)(2 * un.nkeys * kAtHD * 2));
        const int row0 = un.g * a.seq;
        for (int kb = 0; kb <= un.qb; ++kb) {
          tma_load_2d(sK + kvs * AtSmem::kKV + kb * AtSmem::kQ, &tm, &kv_full[kvs], a.k_off + un.kvh * kAtHD,
                      row0 + kb * kAtRows);
          tma_load_2d(sV + kvs * AtSmem::kKV + kb * AtSmem::kQ, &tm, &kv_full[kvs], a.v_off + un.kvh * kAtHD,
                      row0 + kb * kAtRows);
        }
        for (int j = 0; j < gq && ok; ++j, ++t) {
          const int qs = t & 1;
          if (!mbar_wait(&q_empty[qs], ((uint32_t)(t >> 1) & 1u) ^ 1u, abort_flag, status, DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&q_full[qs], (uint32_t)AtSmem::kQ);
          tma_load_2d(sQ + qs * AtSmem::kQ, &tm, &q_full[qs], a.q_off + (un.kvh * gq + j) * kAtHD,
                      row0 + un.qb * kAtRows);
        }
        if (!ok) break;
      }
      if (!ok) {
        // Let the copies in flight land before the CTA can exit (bounded waits).
        for (int i = 1; i <= 2 && t - i >= 0; ++i) mbar_wait_drain(&q_full[(t - i) & 1], ((uint32_t)((t - i) >> 1)) & 1u);
        for (int i = 1; i <= 2 && k - i >= 0; ++i)
          mbar_wait_drain(&kv_full[(k - i) & 1], ((uint32_t)((k - i) >> 1)) & 1u);
        // (the abort flag is set: every consumer's bounded wait returns)
      }
    }
  } else if (warp == 1 || warp == kAtThreads / 32 - 1) {
    // ---------------- MMA issuers: warp 1 for TMEM buffer 0 (even heads), the last warp for buffer 1 ----------------
    // A tcgen05.mma holds its issuing thread for about as long as an N = 256 step takes, whatever its
    // N (measured: ~105-150 cycles for N = 64 with one issuer), while two issuers' N = 64 streams
    // overlap on the tensor core. So each buffer has its own issuer: one head's P·V no longer delays
    // the other buffer's S. Head t's S issues once head t-1 (other buffer) has its row maxima (m_full):
    // its max pass then overlaps that head's exp pass, and the two pairs' exp passes, which share the
    // MUFU of each SM sub-partition, follow one another instead of running together.
    if (lane == 0) {
      const int b = warp == 1 ? 0 : 1;
      const uint32_t idesc_s128 = umma_idesc_f16(BF16, kAtRows, 128);
      const uint32_t idesc_s256 = umma_idesc_f16(BF16, kAtRows, 256);
      const uint32_t idesc_o = umma_idesc_f16(BF16, kAtRows, kAtHD) | (1u << 16);  // B = V, MN-major
      bool ok = true, issued_any = false;
      int t0 = 0;  // global index of the unit's first head
      for (int k = 0; ok; ++k, t0 += gq) {
        const int slot = k % kAtRing;
        if (!mbar_wait(&u_full[slot], (uint32_t)(k / kAtRing) & 1u, abort_flag, status, DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        const int u = ring[slot];
        mbar_arrive(&u_empty[slot]);
        if (u >= total_units) break;
        const Unit un = decode_unit(u, a);
        const int kvs = k & 1;
        // this issuer's heads of the unit: t0 + j with (t0 + j) % 2 == b
        const int j_first = ((t0 & 1) == b) ? 0 : 1;
        int j_last = -1;
        for (int j = j_first; j < gq; j += 2) j_last = j;
        // (also without heads here: an arrival on kv_empty before this unit's K/V has landed could be
        // counted towards the stage's previous unit, whose other issuer may still be reading it)
        if (!mbar_wait(&kv_full[kvs], (uint32_t)(k >> 1) & 1u, abort_flag, status, DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        if (j_last < 0) {  // none of this unit's heads: release its K/V stage for this issuer
          mbar_arrive(&kv_empty[kvs]);
          continue;
        }
        const uint32_t k_base = smem_u32(sK + kvs * AtSmem::kKV);
        const uint32_t v_base = smem_u32(sV + kvs * AtSmem::kKV);
        const uint32_t idesc_s = un.nkeys == 256 ? idesc_s256 : idesc_s128;
        for (int j = j_first; j < gq; j += 2) {
          const int t = t0 + j;
          const uint32_t n = (uint32_t)(t >> 1) & 1u;  // phase of buffer b's barriers for head t
          const int tp = t - 1;                          // previous head, on the other buffer
          if ((tp >= 0 && !mbar_wait(&m_full[b ^ 1], (uint32_t)(tp >> 1) & 1u, abort_flag, status, DEV_TIMEOUT_MMA)) ||
              !mbar_wait(&q_full[b], n, abort_flag, status, DEV_TIMEOUT_MMA) ||
              !mbar_wait(&t_empty[b], n ^ 1u, abort_flag, status, DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t q_base = smem_u32(sQ + b * AtSmem::kQ);
          for (int kk = 0; kk < kAtHD / 16; ++kk)
            umma_f16_ss(tmem_base + b * 256, sw128_kmajor_desc(q_base + kk * 32), sw128_kmajor_desc(k_base + kk * 32),
                        idesc_s, kk > 0 ? 1u : 0u);
          umma_commit(&s_full[b]);
          umma_commit(&q_empty[b]);
          issued_any = true;
          if (!mbar_wait(&p_full[b], n, abort_flag, status, DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t o_tmem = tmem_base + b * 256 + kAtOCol;
          const uint32_t p_tmem = tmem_base + b * 256;
          const int nch = un.nkeys / 32;  // 16-key steps ks < nch hold side A's P, the rest side B's
          for (int ks = 0; ks < un.nkeys / 16; ++ks)
            umma_f16_ts(o_tmem, p_tmem + ks * 8 + (ks >= nch ? nch * 8 : 0), sw128_mnmajor_desc(v_base + ks * 2048),
                        idesc_o, ks > 0 ? 1u : 0u);
          umma_commit(&o_full[b]);
          if (j == j_last) umma_commit(&kv_empty[kvs]);
        }
      }
      if (!ok && issued_any) {
        umma_commit(&drain_bar[b]);
        mbar_wait_drain(&drain_bar[b], 0);
      }
    }
  } else {
    // ---------------- softmax / output warpgroup pairs (warps 2-9, 10-17) ----------------
    const int wg = (warp - 2) >> 3;          // buffer this pair owns
    const int side = ((warp - 2) >> 2) & 1;  // 0: first half of the keys, 1: second half
    const int quarter = warp & 3;            // TMEM lane quarter
    const int r = quarter * 32 + lane;       // row inside the query tile
    const int wt = threadIdx.x - 64 - wg * 256;  // 0..255 within the pair
    const uint32_t bar_id = 1 + wg;
    float* red = reinterpret_cast<float*>(smem + AtSmem::kRedOff) + wg * 256;  // [side][128]
    auto agree = [&](bool ok_wait) -> bool {
      // every thread of the pair takes the same continue/abort decision
      named_bar_sync(bar_id, 256);
      if (wt == 0) wg_abort[wg] = (*abort_flag || !ok_wait) ? 1u : 0u;
      named_bar_sync(bar_id, 256);
      return wg_abort[wg] == 0;
    };
    int t = 0;
    for (int k = 0;; ++k) {
      const int slot = k % kAtRing;
      const bool okw = mbar_wait(&u_full[slot], (uint32_t)(k / kAtRing) & 1u, abort_flag, status, DEV_TIMEOUT_EPILOGUE);
      if (!agree(okw)) break;
      const int u = ring[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&u_empty[slot]);
      if (u >= total_units) break;
      const Unit un = decode_unit(u, a);
      const int qpos = un.qb * kAtRows + r;
      const int diag = un.qb * 4 + quarter;  // 32-key chunk holding this warp's diagonal
      const int nch = un.nkeys / 32;
      const int c_lo = side ? nch / 2 : 0, c_hi = side ? nch : nch / 2;  // this side's chunks
      const int c_last = min(c_hi - 1, diag);                           // last causal chunk of the side
      const int p_off = side ? nch * 8 : 0;  // P of chunk c at column 16c + p_off
      bool stop = false;
      for (int j = 0; j < gq; ++j, ++t) {
        if ((t & 1) != wg) continue;
        const uint32_t n = (uint32_t)(t >> 1) & 1u;
        const int h = un.kvh * gq + j;
        if (!agree(mbar_wait(&s_full[wg], n, abort_flag, status, DEV_TIMEOUT_EPILOGUE))) {
          stop = true;
          break;
        }
        tc_fence_after();
        const uint32_t t_row = tmem_base + wg * 256 + ((uint32_t)(quarter * 32) << 16);
        // pass 1: row maximum over this side's causal keys (only the diagonal chunk is
        // masked); the two sides' maxima meet in shared memory
        float mx = -INFINITY;
        for (int c = c_lo; c <= c_last; ++c) {
          uint32_t v[32];
          tmem_ld32(t_row + c * 32, v);
          tmem_ld_wait_regs(v);
          mx = c < diag ? chunk_max<false>(v, mx, 0, 0) : chunk_max<true>(v, mx, c * 32, qpos);
        }
        red[side * 128 + r] = mx;
        named_bar_sync(bar_id, 256);
        __syncwarp();
        if (lane == 0) mbar_arrive(&m_full[wg]);  // the next head's S may issue now
        mx = fmaxf(mx, red[(side ^ 1) * 128 + r]);
        // pass 2: P = exp2((s - max)·scale) as 16-bit pairs, chunk c at columns
        // [16c + p_off, +16) (this side's own S columns, read before they are written),
        // zeros past the diagonal
        const float ms = mx * scale_log2;
        float l = 0.f;
        for (int c = c_lo; c <= c_last; ++c) {
          uint32_t v[32];
          uint32_t pk[16];
          tmem_ld32(t_row + c * 32, v);
          tmem_ld_wait_regs(v);
          if (c < diag)
            chunk_exp<T, false>(v, pk, l, scale_log2, ms, 0, 0);
          else
            chunk_exp<T, true>(v, pk, l, scale_log2, ms, c * 32, qpos);
          tmem_st16(t_row + c * 16 + p_off, pk);
        }
        {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) pk[i] = 0u;
          for (int c = max(c_lo, diag + 1); c < c_hi; ++c) tmem_st16(t_row + c * 16 + p_off, pk);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[wg]);
        // the partial sums meet (both sides read the maxima before this barrier)
        named_bar_sync(bar_id, 256);
        red[side * 128 + r] = l;
        named_bar_sync(bar_id, 256);
        l += red[(side ^ 1) * 128 + r];
        const long long row = (long long)un.g * a.seq + qpos;
        // output: this side's 32 columns of O / l
        if (!agree(mbar_wait(&o_full[wg], n, abort_flag, status, DEV_TIMEOUT_EPILOGUE))) {
          stop = true;
          break;
        }
        tc_fence_after();
        if (a.lse && side == 0) a.lse[row * a.heads + h] = ms + log2f(l);
        const float inv = 1.0f / l;
        T* out = static_cast<T*>(a.out) + row * a.ld_out + h * kAtHD + side * 32;
        uint32_t o[32];
        tmem_ld32(t_row + kAtOCol + side * 32, o);
        tmem_ld_wait_regs(o);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&t_empty[wg]);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w[e] = pack_h2<T>(__uint_as_float(o[c * 8 + 2 * e]) * inv, __uint_as_float(o[c * 8 + 2 * e + 1]) * inv);
          *reinterpret_cast<uint4*>(out + c * 8) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      if (stop) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kAtTmemCols);
  }
  if (threadIdx.x == 0) {
    // the last CTA to finish resets the unit counter for the next launch
    __threadfence();
    if (atomicAdd(a.sched + 1, 1) == (int)gridDim.x - 1) {
      a.sched[0] = 0;
      a.sched[1] = 0;
      __threadfence();
    }
  }
}

}  // namespace

bool attention_tc_supported(const AttnArgs& a) {
  return a.sched != nullptr && (a.seq == 128 || a.seq == 256) && a.ld_out % 8 == 0 && a.ld_qkv % 8 == 0 &&
         a.q_off % 8 == 0 && a.k_off % 8 == 0 && a.v_off % 8 == 0 && a.kv_heads > 0 && a.heads % a.kv_heads == 0;
}

template <typename T>
int launch_tc_t(const AttnArgs& a, cudaStream_t st) {
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  DeviceCtx* c = nullptr;
  int rc = ctx_get(&c);
  if (rc) return rc;
  const long long rows = (long long)a.ngroups * a.seq;
  CUtensorMap tm;
  if ((rc = make_tmap_2d(&tm, a.qkv, BF16 ? TM_BF16 : TM_F16, (uint64_t)a.ld_qkv, (uint64_t)rows,
                         (uint64_t)a.ld_qkv, kAtHD, kAtRows, 128)))
    return rc;
  const int total = a.ngroups * a.kv_heads * (a.seq / kAtRows);
  const int grid = total < c->num_sms ? total : c->num_sms;
  const float scale_log2 = (1.0f / sqrtf((float)kAtHD)) * 1.4426950408889634f;
  static thread_local uint64_t attr_mask = 0;  // one per instantiation (per dtype)
  if (!(attr_mask & (1ull << (c->device & 63)))) {
    B2P_CHECK_CUDA(cudaFuncSetAttribute(attn_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, AtSmem::kTotal));
    attr_mask |= 1ull << (c->device & 63);
  }
  B2P_CHECK_CUDA(launch_pdl(attn_tc_kernel<T>, dim3(grid), dim3(kAtThreads), AtSmem::kTotal, st, tm, a, scale_log2,
                            total, c->status));
  B2P_POST_LAUNCH();
  return B2P_OK;
}

int launch_attention_tc(const AttnArgs& a, bool bf16, cudaStream_t st) {
  B2P_REQUIRE(attention_tc_supported(a), "tcgen05 attention needs seq 128 or 256, 16-byte aligned operands and a "
                                         "unit counter");
  return bf16 ? launch_tc_t<__nv_bfloat16>(a, st) : launch_tc_t<__half>(a, st);
}

}  // namespace b2p
