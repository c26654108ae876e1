// gemm_sk.cu — projection GEMMs of few token rows.
//
//   Y[M, N] = X[M, K] · W[N, K]^T,  M <= 1024 (the per-call sizes of the
//   Kern-level operators: one 128-1024-token sequence per call,
//   training/train_mezo.m:1545-1627)
//
// At these sizes a tile per CTA leaves most SMs idle and each CTA runs a long,
// latency-fed K loop. Output tiles are 128 x 64. A tcgen05.mma of N = 64 holds
// its issuing thread about as long as one of N = 256, so each CTA spreads its
// K-blocks over four MMA issuer warps with a TMEM accumulator each (summed in
// issuer order). Where a long K loop (K >= 2048) can be split over a cluster of
// 2 or 4 CTAs, each CTA takes a slice of K and the partial tiles meet in CTA 0
// by bulk copies over distributed shared memory, added in rank order. Results
// never depend on timing.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "engine.cuh"
#include "ptx.cuh"

namespace b2p {
namespace {

constexpr int kSkBN = 64;       // output columns per tile (UMMA N)
constexpr int kSkMaxSplit = 4;  // CTA 0 holds a 32 KB slot for each other CTA of the cluster
constexpr int kSkMaxRows = 1024;
constexpr int kSkAStage = kBM * kBK * 2;     // 16 KB
constexpr int kSkBStage = kSkBN * kBK * 2;   // 8 KB
constexpr int kSkSlot = kBM * kSkBN * 4;     // one fp32 partial tile, 32 KB

// Byte offset of 16-byte chunk c of row r inside a partial slot: rows of 256 B, chunks XOR-swizzled
// with the row so that eight consecutive rows writing the same chunk hit eight different bank groups.
__device__ __forceinline__ uint32_t slot_off(int r, int c) { return (uint32_t)(r * 256 + ((c ^ (r & 15)) << 4)); }

__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack_pair<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack_pair<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ---------------------------------------------------------------------------
// Several MMA issuers per tile. A tcgen05.mma of N = 64 holds its issuing thread about as long as
// one of N = 256 (~105-150 cycles per K = 16 step), so a 128 x 64 tile fed by one issuer runs its
// K loop at about a quarter of the tensor core's rate; issuers on different warps overlap. Here
// kMiIssuers warps take the tile's K-blocks in turn (block j to issuer j % kMiIssuers), each into
// its own 64-column TMEM accumulator, and the epilogue adds the accumulators in issuer order (the
// result does not depend on timing). One CTA per tile, no cluster and no reduction traffic.
//
// Warps: 0 TMA producer, 1-3 and 8 MMA issuers, 4-7 epilogue (warp % 4 = TMEM lane quarter);
// warp 1 owns the TMEM allocation.
constexpr int kMiIssuers = 4;
constexpr int kMiStages = 8;   // a multiple of kMiIssuers: issuer i consumes stages i, i + 4
constexpr int kMiThreads = 9 * 32;
constexpr int kMiBarOff = kMiStages * (kSkAStage + kSkBStage);
constexpr int kMiSmem = kMiBarOff + 256 + 1024;
static_assert(kMiStages % kMiIssuers == 0, "stage ownership");
static_assert(kMiSmem <= 227 * 1024, "shared memory over the per-CTA limit");

__device__ __forceinline__ int mi_issuer_of_warp(int warp) { return warp >= 1 && warp <= 3 ? warp - 1 : (warp == 8 ? 3 : -1); }

template <typename T, bool OUT_F32>
__global__ void __launch_bounds__(kMiThreads, 1)
    gemm_mi_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, void* out,
                   int ldo, int M, int N, int K, uint32_t* status) {
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kMiStages * kSkAStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kMiBarOff);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + kMiStages;
  uint64_t* tfull_bar = bars + 2 * kMiStages;
  uint64_t* drain_bar = tfull_bar + 1;  // [kMiIssuers]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + kMiIssuers);
  volatile uint32_t* abort_flag = tmem_holder + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nt = blockIdx.x, mt = blockIdx.y;
  const int kblocks = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kMiStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tfull_bar, kMiIssuers);
    for (int i = 0; i < kMiIssuers; ++i) mbar_init(&drain_bar[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kMiIssuers * kSkBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_enter();  // the previous kernel's outputs are complete from here on

  const int issuer = mi_issuer_of_warp(warp);
  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb) {
        const int stage = kb % kMiStages;
        const uint32_t phase = (uint32_t)(kb / kMiStages) & 1u;
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, status, DEV_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full_bar[stage], kSkAStage + kSkBStage);
        tma_load_2d(sA + stage * kSkAStage, &tmX, &full_bar[stage], kb * kBK, mt * kBM);
        tma_load_2d(sB + stage * kSkBStage, &tmW, &full_bar[stage], kb * kBK, nt * kSkBN);
        ++issued;
      }
      if (!ok) {  // let every issued copy land before the CTA can go on
        for (int kb = issued - 1; kb >= 0 && kb >= issued - kMiStages; --kb)
          mbar_wait_drain(&full_bar[kb % kMiStages], (uint32_t)(kb / kMiStages) & 1u);
      }
    }
  } else if (issuer >= 0) {
    // ---------------- MMA issuers: K-blocks issuer, issuer + 4, ... into accumulator `issuer` ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(BF16, kBM, kSkBN);
      const uint32_t d_tmem = tmem_base + issuer * kSkBN;
      bool ok = true, issued_any = false;
      for (int kb = issuer; kb < kblocks; kb += kMiIssuers) {
        const int stage = kb % kMiStages;
        if (!mbar_wait(&full_bar[stage], (uint32_t)(kb / kMiStages) & 1u, abort_flag, status, DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t adesc = sw128_kmajor_desc(smem_u32(sA + stage * kSkAStage));
        const uint64_t bdesc = sw128_kmajor_desc(smem_u32(sB + stage * kSkBStage));
#pragma unroll
        for (int k = 0; k < kBK / kUmmaK; ++k)
          umma_f16_ss(d_tmem, adesc + 2ull * k, bdesc + 2ull * k, idesc, (kb > issuer || k) ? 1u : 0u);
        issued_any = true;
        umma_commit(&empty_bar[stage]);
      }
      if (!ok && issued_any) {  // nothing of this issuer may still run when the CTA leaves
        umma_commit(&drain_bar[issuer]);
        mbar_wait_drain(&drain_bar[issuer], 0);
      }
      if (issued_any)
        umma_commit(tfull_bar);
      else
        mbar_arrive(tfull_bar);
    }
  } else {
    // ---------------- epilogue (warps 4-7): sum the accumulators in issuer order, store ----------------
    const int quarter = warp & 3;
    const bool ok = mbar_wait(tfull_bar, 0, abort_flag, status, DEV_TIMEOUT_EPILOGUE);
    tc_fence_after();
    if (ok && !*abort_flag) {
      float v[kSkBN];
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16);
      const int nacc = kblocks < kMiIssuers ? kblocks : kMiIssuers;
      for (int i = 0; i < nacc; ++i) {
        uint32_t r0[32], r1[32];
        tmem_ld32(taddr + i * kSkBN, r0);
        tmem_ld32(taddr + i * kSkBN + 32, r1);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (i == 0) {
            v[j] = __uint_as_float(r0[j]);
            v[32 + j] = __uint_as_float(r1[j]);
          } else {
            v[j] += __uint_as_float(r0[j]);
            v[32 + j] += __uint_as_float(r1[j]);
          }
        }
      }
      const int row = mt * kBM + quarter * 32 + lane;
      const int col0 = nt * kSkBN;
      if (row < M) {
        if (OUT_F32) {
          float* y = static_cast<float*>(out) + (long long)row * ldo + col0;
          if (col0 + kSkBN <= N) {
#pragma unroll
            for (int c = 0; c < kSkBN / 4; ++c)
              reinterpret_cast<float4*>(y)[c] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < kSkBN; ++j)
              if (col0 + j < N) y[j] = v[j];
          }
        } else {
          T* y = static_cast<T*>(out) + (long long)row * ldo + col0;
          if (col0 + kSkBN <= N) {
#pragma unroll
            for (int c = 0; c < kSkBN / 8; ++c) {
              uint4 w;
              w.x = pack_pair<T>(v[8 * c], v[8 * c + 1]);
              w.y = pack_pair<T>(v[8 * c + 2], v[8 * c + 3]);
              w.z = pack_pair<T>(v[8 * c + 4], v[8 * c + 5]);
              w.w = pack_pair<T>(v[8 * c + 6], v[8 * c + 7]);
              reinterpret_cast<uint4*>(y)[c] = w;
            }
          } else {
#pragma unroll
            for (int j = 0; j < kSkBN; ++j)
              if (col0 + j < N) y[j] = static_cast<T>(v[j]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kMiIssuers * kSkBN);
  }
}

// The same with each tile's K loop split over a cluster of S CTAs (S = 2 or 4): CTA s takes K-blocks
// [s·kps, (s+1)·kps) with four issuers of its own, so each SM loads only its slice of the operands.
// CTAs 1..S-1 write their summed partial tile into their own (idle) pipeline shared memory and move
// it with one bulk copy into their slot of CTA 0's shared memory, completing on an mbarrier of CTA 0
// that expects all S-1 tiles' bytes; CTA 0 adds the slots in rank order (the sum does not depend on
// timing) and writes the tile. (Per-thread remote stores into CTA 0 and a cluster barrier cost ~3.5 us
// in an earlier form of this kernel.)
constexpr int kMsStages = 4;  // one stage per issuer: each CTA has few K-blocks
constexpr int kMsSlotOff = kMsStages * (kSkAStage + kSkBStage);
constexpr int kMsBarOff = kMsSlotOff + (kSkMaxSplit - 1) * kSkSlot;
constexpr int kMsSmem = kMsBarOff + 256 + 1024;
static_assert(kMsStages == kMiIssuers, "issuer i owns stage i");
static_assert(kMsSmem <= 227 * 1024, "shared memory over the per-CTA limit");

__device__ __forceinline__ void bulk_copy_to_cluster(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes,
                                                     uint32_t mbar_cluster) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst_cluster),
               "r"(src_cta), "r"(bytes), "r"(mbar_cluster)
               : "memory");
}

template <typename T, bool OUT_F32>
__global__ void __launch_bounds__(kMiThreads, 1)
    gemm_mis_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, void* out,
                    int ldo, int M, int N, int K, int kps, uint32_t* status) {
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kMsStages * kSkAStage;
  uint8_t* slots = smem + kMsSlotOff;  // CTA 0: the partials of CTAs 1..S-1
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kMsBarOff);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + kMsStages;
  uint64_t* tfull_bar = bars + 2 * kMsStages;
  uint64_t* drain_bar = tfull_bar + 1;  // [kMiIssuers]
  uint64_t* red_bar = drain_bar + kMiIssuers;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(red_bar + 1);
  volatile uint32_t* abort_flag = tmem_holder + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t nsplit = cluster_nctarank();
  const int nt = blockIdx.x, mt = blockIdx.y;
  const int kblocks = (K + kBK - 1) / kBK;
  const int kb0 = (int)rank * kps;
  const int nk = min(kblocks, kb0 + kps) - kb0;  // the host guarantees nk >= 1

  if (threadIdx.x == 0) {
    for (int s = 0; s < kMsStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tfull_bar, kMiIssuers);
    for (int i = 0; i < kMiIssuers; ++i) mbar_init(&drain_bar[i], 1);
    mbar_init(red_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    if (rank == 0) mbar_arrive_expect_tx(red_bar, (nsplit - 1) * (uint32_t)kSkSlot);
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kMiIssuers * kSkBN);
    tmem_relinquish();
  }
  tc_fence_before();
  cluster_sync();  // CTA 0's reduction barrier is initialised before any remote copy completes on it
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_enter();  // the previous kernel's outputs are complete from here on

  const int issuer = mi_issuer_of_warp(warp);
  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < nk; ++j) {
        const int stage = j % kMsStages;
        if (!mbar_wait(&empty_bar[stage], ((uint32_t)(j / kMsStages) & 1u) ^ 1u, abort_flag, status,
                       DEV_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full_bar[stage], kSkAStage + kSkBStage);
        tma_load_2d(sA + stage * kSkAStage, &tmX, &full_bar[stage], (kb0 + j) * kBK, mt * kBM);
        tma_load_2d(sB + stage * kSkBStage, &tmW, &full_bar[stage], (kb0 + j) * kBK, nt * kSkBN);
        ++issued;
      }
      if (!ok) {
        for (int j = issued - 1; j >= 0 && j >= issued - kMsStages; --j)
          mbar_wait_drain(&full_bar[j % kMsStages], (uint32_t)(j / kMsStages) & 1u);
      }
    }
  } else if (issuer >= 0) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(BF16, kBM, kSkBN);
      const uint32_t d_tmem = tmem_base + issuer * kSkBN;
      bool ok = true, issued_any = false;
      for (int j = issuer; j < nk; j += kMiIssuers) {
        const int stage = j % kMsStages;
        if (!mbar_wait(&full_bar[stage], (uint32_t)(j / kMsStages) & 1u, abort_flag, status, DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t adesc = sw128_kmajor_desc(smem_u32(sA + stage * kSkAStage));
        const uint64_t bdesc = sw128_kmajor_desc(smem_u32(sB + stage * kSkBStage));
#pragma unroll
        for (int k = 0; k < kBK / kUmmaK; ++k)
          umma_f16_ss(d_tmem, adesc + 2ull * k, bdesc + 2ull * k, idesc, (j > issuer || k) ? 1u : 0u);
        issued_any = true;
        umma_commit(&empty_bar[stage]);
      }
      if (!ok && issued_any) {
        umma_commit(&drain_bar[issuer]);
        mbar_wait_drain(&drain_bar[issuer], 0);
      }
      if (issued_any)
        umma_commit(tfull_bar);
      else
        mbar_arrive(tfull_bar);
    }
  } else {
    // ---------------- epilogue (warps 4-7) ----------------
    const int quarter = warp & 3;
    const int row_in = quarter * 32 + lane;
    const bool ok = mbar_wait(tfull_bar, 0, abort_flag, status, DEV_TIMEOUT_EPILOGUE);
    tc_fence_after();
    float v[kSkBN];
#pragma unroll
    for (int j = 0; j < kSkBN; ++j) v[j] = 0.f;
    if (ok && !*abort_flag) {
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16);
      const int nacc = nk < kMiIssuers ? nk : kMiIssuers;
      for (int i = 0; i < nacc; ++i) {
        uint32_t r0[32], r1[32];
        tmem_ld32(taddr + i * kSkBN, r0);
        tmem_ld32(taddr + i * kSkBN + 32, r1);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          v[j] += __uint_as_float(r0[j]);
          v[32 + j] += __uint_as_float(r1[j]);
        }
      }
    }
    if (rank != 0) {
      // this CTA's partial into its own (now idle) pipeline memory, then one bulk copy to CTA 0
      uint8_t* stg = smem;
#pragma unroll
      for (int c = 0; c < kSkBN / 4; ++c)
        *reinterpret_cast<float4*>(stg + slot_off(row_in, c)) = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2],
                                                                             v[4 * c + 3]);
      fence_proxy_async_smem();
      named_bar_sync(1, 128);
      if (warp == 4 && lane == 0)
        bulk_copy_to_cluster(mapa_shared(smem_u32(slots + (rank - 1) * kSkSlot), 0), smem_u32(stg), kSkSlot,
                             mapa_shared(smem_u32(red_bar), 0));
    } else {
      bool red_ok = true;
      if (nsplit > 1) red_ok = mbar_wait(red_bar, 0, abort_flag, status, DEV_TIMEOUT_EPILOGUE);
      if (red_ok && !*abort_flag) {
        for (uint32_t p = 1; p < nsplit; ++p) {  // rank order: the sum does not depend on timing
          const uint8_t* slot = slots + (p - 1) * kSkSlot;
#pragma unroll
          for (int c = 0; c < kSkBN / 4; ++c) {
            const float4 q = *reinterpret_cast<const float4*>(slot + slot_off(row_in, c));
            v[4 * c] += q.x;
            v[4 * c + 1] += q.y;
            v[4 * c + 2] += q.z;
            v[4 * c + 3] += q.w;
          }
        }
        const int row = mt * kBM + row_in;
        const int col0 = nt * kSkBN;
        if (row < M) {
          if (OUT_F32) {
            float* y = static_cast<float*>(out) + (long long)row * ldo + col0;
            if (col0 + kSkBN <= N) {
#pragma unroll
              for (int c = 0; c < kSkBN / 4; ++c)
                reinterpret_cast<float4*>(y)[c] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
            } else {
#pragma unroll
              for (int j = 0; j < kSkBN; ++j)
                if (col0 + j < N) y[j] = v[j];
            }
          } else {
            T* y = static_cast<T*>(out) + (long long)row * ldo + col0;
            if (col0 + kSkBN <= N) {
#pragma unroll
              for (int c = 0; c < kSkBN / 8; ++c) {
                uint4 w;
                w.x = pack_pair<T>(v[8 * c], v[8 * c + 1]);
                w.y = pack_pair<T>(v[8 * c + 2], v[8 * c + 3]);
                w.z = pack_pair<T>(v[8 * c + 4], v[8 * c + 5]);
                w.w = pack_pair<T>(v[8 * c + 6], v[8 * c + 7]);
                reinterpret_cast<uint4*>(y)[c] = w;
              }
            } else {
#pragma unroll
              for (int j = 0; j < kSkBN; ++j)
                if (col0 + j < N) y[j] = static_cast<T>(v[j]);
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kMiIssuers * kSkBN);
  }
  // CTA 0 has taken every partial before any CTA of the cluster leaves (the copies read the senders'
  // shared memory until they complete on CTA 0's barrier)
  cluster_sync();
}

template <typename T, bool OUT_F32>
int launch_mis_t(const void* X, int ldx, const void* W, int ldw, int M, int N, int K, void* out, int ldo, int nsplit,
                 int kps, cudaStream_t st) {
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  DeviceCtx* c = nullptr;
  int rc = ctx_get(&c);
  if (rc) return rc;
  CUtensorMap tx, tw;
  const TmapType in_t = BF16 ? TM_BF16 : TM_F16;
  if ((rc = make_tmap_2d(&tx, X, in_t, (uint64_t)K, (uint64_t)M, (uint64_t)ldx, kBK, kBM, 128))) return rc;
  if ((rc = make_tmap_2d(&tw, W, in_t, (uint64_t)K, (uint64_t)N, (uint64_t)ldw, kBK, kSkBN, 128))) return rc;
  auto kern = gemm_mis_kernel<T, OUT_F32>;
  static thread_local uint64_t attr_mask = 0;
  if (!(attr_mask & (1ull << (c->device & 63)))) {
    B2P_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMsSmem));
    attr_mask |= 1ull << (c->device & 63);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((N + kSkBN - 1) / kSkBN), (unsigned)((M + kBM - 1) / kBM), (unsigned)nsplit);
  cfg.blockDim = dim3(kMiThreads, 1, 1);
  cfg.dynamicSmemBytes = kMsSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)nsplit;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // the kernel calls pdl_enter()
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  B2P_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, tx, tw, out, ldo, M, N, K, kps, c->status));
  B2P_POST_LAUNCH();
  return B2P_OK;
}

template <typename T, bool OUT_F32>
int launch_mi_t(const void* X, int ldx, const void* W, int ldw, int M, int N, int K, void* out, int ldo,
                cudaStream_t st) {
  constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
  DeviceCtx* c = nullptr;
  int rc = ctx_get(&c);
  if (rc) return rc;
  CUtensorMap tx, tw;
  const TmapType in_t = BF16 ? TM_BF16 : TM_F16;
  if ((rc = make_tmap_2d(&tx, X, in_t, (uint64_t)K, (uint64_t)M, (uint64_t)ldx, kBK, kBM, 128))) return rc;
  if ((rc = make_tmap_2d(&tw, W, in_t, (uint64_t)K, (uint64_t)N, (uint64_t)ldw, kBK, kSkBN, 128))) return rc;
  auto kern = gemm_mi_kernel<T, OUT_F32>;
  static thread_local uint64_t attr_mask = 0;
  if (!(attr_mask & (1ull << (c->device & 63)))) {
    B2P_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMiSmem));
    attr_mask |= 1ull << (c->device & 63);
  }
  B2P_CHECK_CUDA(launch_pdl(kern, dim3((unsigned)((N + kSkBN - 1) / kSkBN), (unsigned)((M + kBM - 1) / kBM)),
                            dim3(kMiThreads), kMiSmem, st, tx, tw, out, ldo, M, N, K, c->status));
  B2P_POST_LAUNCH();
  return B2P_OK;
}

}  // namespace

bool splitk_applies(int kind, int M, int N, int num_sms) {
  const long long tiles = (long long)((M + kBM - 1) / kBM) * ((N + kSkBN - 1) / kSkBN);
  return (kind == EPI_F32 || kind == EPI_H16) && M >= 1 && M <= kSkMaxRows && tiles <= num_sms;
}

int splitk_factor(int M, int N, int K, int num_sms, int* kps_out);


int splitk_factor(int M, int N, int K, int num_sms, int* kps_out) {
  const int tiles = ((M + kBM - 1) / kBM) * ((N + kSkBN - 1) / kSkBN);
  const int kblocks = (K + kBK - 1) / kBK;
  int s = 1;
  while (2 * s <= kSkMaxSplit && tiles * 2 * s <= num_sms && kblocks >= 4 * s) s *= 2;
  int kps = (kblocks + s - 1) / s;
  while (s > 1 && (s - 1) * kps >= kblocks) {  // every CTA of the cluster gets at least one K-block
    s /= 2;
    kps = (kblocks + s - 1) / s;
  }
  *kps_out = kps;
  return s;
}

int launch_gemm_splitk(int kind, bool bf16, const void* X, int ldx, const void* W, int ldw, int M, int N, int K,
                       void* out, int ldo, cudaStream_t st) {
  DeviceCtx* c = nullptr;
  int rc = ctx_get(&c);
  if (rc) return rc;
  B2P_REQUIRE(splitk_applies(kind, M, N, c->num_sms),
              "split-K GEMM takes plain outputs, at most %d rows and one wave of 128 x 64 tiles", kSkMaxRows);
  B2P_REQUIRE(N > 0 && K > 0 && out, "empty split-K GEMM");
  B2P_REQUIRE(kind == EPI_F32 ? ldo % 4 == 0 : ldo % 8 == 0, "output rows must stay 16-byte aligned");
  int kps = 1;
  const int s = splitk_factor(M, N, K, c->num_sms, &kps);
  const bool f32 = kind == EPI_F32;
  if (s < 2) return launch_gemm_mi(kind, bf16, X, ldx, W, ldw, M, N, K, out, ldo, st);
  if (bf16)
    return f32 ? launch_mis_t<__nv_bfloat16, true>(X, ldx, W, ldw, M, N, K, out, ldo, s, kps, st)
               : launch_mis_t<__nv_bfloat16, false>(X, ldx, W, ldw, M, N, K, out, ldo, s, kps, st);
  return f32 ? launch_mis_t<__half, true>(X, ldx, W, ldw, M, N, K, out, ldo, s, kps, st)
             : launch_mis_t<__half, false>(X, ldx, W, ldw, M, N, K, out, ldo, s, kps, st);
}

int small_gemm_route(int kind, int M, int N, int K, int num_sms) {
  if (!splitk_applies(kind, M, N, num_sms)) return SMALL_GEMM_NONE;
  // Measured per shape at 128-1024 rows (graph-timed, HBM-fresh operands): the cluster split pays for
  // its reduction only over a long K loop (W2, K = 2560, at 128 / 256 rows: 9.5 / 9.5 us against
  // 11.5 / 11.6 unsplit); at K = 960 one CTA per tile with four MMA issuers is fastest (Wq at 128 / 256
  // rows 6.6 us unsplit against 7.3 / 7.5 split four ways, and 8.8 on the persistent engines).
  int kps = 0;
  const int s = splitk_factor(M, N, K, num_sms, &kps);
  return (s >= 2 && K >= 2048) ? SMALL_GEMM_SPLITK : SMALL_GEMM_MULTI_ISSUER;
}

int launch_gemm_small(int route, int kind, bool bf16, const void* X, int ldx, const void* W, int ldw, int M, int N,
                      int K, void* out, int ldo, cudaStream_t st) {
  if (route == SMALL_GEMM_SPLITK) return launch_gemm_splitk(kind, bf16, X, ldx, W, ldw, M, N, K, out, ldo, st);
  return launch_gemm_mi(kind, bf16, X, ldx, W, ldw, M, N, K, out, ldo, st);
}

int launch_gemm_mi(int kind, bool bf16, const void* X, int ldx, const void* W, int ldw, int M, int N, int K,
                   void* out, int ldo, cudaStream_t st) {
  B2P_REQUIRE(kind == EPI_F32 || kind == EPI_H16, "multi-issuer GEMM takes plain fp32 / 16-bit outputs");
  B2P_REQUIRE(M > 0 && N > 0 && K > 0 && out, "empty multi-issuer GEMM");
  B2P_REQUIRE(kind == EPI_F32 ? ldo % 4 == 0 : ldo % 8 == 0, "output rows must stay 16-byte aligned");
  const bool f32 = kind == EPI_F32;
  if (bf16)
    return f32 ? launch_mi_t<__nv_bfloat16, true>(X, ldx, W, ldw, M, N, K, out, ldo, st)
               : launch_mi_t<__nv_bfloat16, false>(X, ldx, W, ldw, M, N, K, out, ldo, st);
  return f32 ? launch_mi_t<__half, true>(X, ldx, W, ldw, M, N, K, out, ldo, st)
             : launch_mi_t<__half, false>(X, ldx, W, ldw, M, N, K, out, ldo, st);
}

}  // namespace b2p
