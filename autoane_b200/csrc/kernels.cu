// kernels.cu — glue kernels (embedding, RMSNorm + LoRA-down, attention,
// cross-entropy reduction, perturbation steps, layout conversion).
#include <algorithm>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include "engine.cuh"
#include "kernels.cuh"
#include "mma.cuh"

namespace b2p {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// embedding gather
// ---------------------------------------------------------------------------
__global__ void embed_kernel(const float* __restrict__ embed, int vocab, int dim, const int32_t* __restrict__ tokens,
                             const int* __restrict__ group_seq, int seq, int rows, float* __restrict__ x,
                             uint32_t* status) {
  const int row = blockIdx.x;
  if (row >= rows) return;
  const int g = row / seq, t = row - g * seq;
  const int tok = tokens[(long long)group_seq[g] * seq + t];
  if (tok < 0 || tok >= vocab) {
    if (threadIdx.x == 0) atomicCAS(status, 0u, (uint32_t)DEV_BAD_ARGS);
    return;
  }
  const float4* src = reinterpret_cast<const float4*>(embed + (long long)tok * dim);
  float4* dst = reinterpret_cast<float4*>(x + (long long)row * dim);
  for (int i = threadIdx.x; i < dim / 4; i += blockDim.x) dst[i] = __ldg(src + i);
}

int launch_embed(const float* embed, int vocab, int dim, const int32_t* tokens, const int* group_seq, int seq,
                 int rows, float* x, uint32_t* status, cudaStream_t st) {
  B2P_REQUIRE(dim % 4 == 0, "dim must be a multiple of 4");
  embed_kernel<<<rows, 128, 0, st>>>(embed, vocab, dim, tokens, group_seq, seq, rows, x, status);
  B2P_POST_LAUNCH();
  return B2P_OK;
}

// ---------------------------------------------------------------------------
// RMSNorm (perturbed weight) + LoRA-down (perturbed A), one warp per token row
// ---------------------------------------------------------------------------
constexpr int kNormRowsPerBlock = 64;
constexpr int kNormThreads = 256;

// Sum v[k] over the 32 lanes for k < NV (NV a power of two <= 32); on return
// lane l holds the total of value (l & (NV - 1)) in v[0]. Lanes exchange
// halves of their vectors (31 shuffles for NV = 32) instead of reducing each
// value separately.
template <int NV>
__device__ __forceinline__ void transpose_reduce(float (&v)[32], int lane) {
#pragma unroll
  for (int off = 16; off >= NV; off >>= 1)
#pragma unroll
    for (int k = 0; k < NV; ++k) v[k] += __shfl_xor_sync(0xffffffffu, v[k], off);
#pragma unroll
  for (int h = NV / 2; h >= 1; h >>= 1) {
    const bool up = (lane & h) != 0;
#pragma unroll
    for (int k = 0; k < h; ++k) {
      const float mine = up ? v[k + h] : v[k];
      const float other = up ? v[k] : v[k + h];
      v[k] = mine + __shfl_xor_sync(0xffffffffu, other, h);
    }
  }
}

template <int NA>
struct PadPow2 {
  static constexpr int v = NA <= 1 ? 1 : NA <= 2 ? 2 : NA <= 4 ? 4 : NA <= 8 ? 8 : NA <= 16 ? 16 : 32;
};

template <int NP, typename T, bool NORM, int NA>
__global__ void __launch_bounds__(kNormThreads) norm_lora_kernel(NormLoraArgs a) {
  extern __shared__ float sm[];
  pdl_enter();
  float* s_w = sm;                  // [dim]   perturbed rms weight
  float* s_a = sm + a.dim;          // [NA][dim] perturbed LoRA A rows
  using HV = typename H2<T>::V;
  constexpr int dim = NP * 64;
  const int row0 = blockIdx.x * kNormRowsPerBlock;
  const int grp = row0 / a.pc.group_rows;
  const VariantInfo vi = a.pc.variants[a.pc.group_variant[grp]];
  const uint32_t* mask = a.pc.masks + (long long)(vi.mode ? vi.mask_slot : 0) * a.pc.mask_words;

  // stage perturbed operands: θ (+ s1 z) (+ s2 z), exactly as perturb_buffer adds them.
  // 4 parameters per load (offsets and widths are multiples of 4, so their signs share
  // a mask word); 8 loads in flight per thread.
  constexpr int kUnits = (NORM ? dim / 4 : 0) + NA * dim / 4;
  const bool prepped = NA == 0 && a.w_prep != nullptr;  // rms weight already perturbed for this variant
  if (prepped) {
    const float4* wp = reinterpret_cast<const float4*>(a.w_prep + (long long)a.pc.group_variant[grp] * a.w_prep_vstride);
    for (int i = threadIdx.x; i < dim / 4; i += kNormThreads) reinterpret_cast<float4*>(s_w)[i] = __ldg(wp + i);
  }
  for (int u0 = threadIdx.x; !prepped && u0 < kUnits; u0 += 8 * kNormThreads) {
    float4 th[8];
    uint32_t mw[8];
    long long pidx[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int u = u0 + q * kNormThreads;
      long long p = 0;
      if (u < kUnits) {
        if (NORM && u < dim / 4) {
          p = a.w_off + 4LL * u;
        } else {
          const int i = 4 * (u - (NORM ? dim / 4 : 0));
          const int ja = i / dim, c = i - ja * dim;
          const int m = ja / a.rank, j = ja - m * a.rank;
          p = a.a_off[m] + (long long)j * dim + c;
        }
        th[q] = __ldg(reinterpret_cast<const float4*>(a.pc.theta + p));
        mw[q] = vi.mode ? (__ldg(mask + (p >> 5)) >> (p & 31)) : 0u;
      }
      pidx[q] = p;
    }
    (void)pidx;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int u = u0 + q * kNormThreads;
      if (u >= kUnits) break;
      float4 t = th[q];
      if (vi.mode) {
        t.x = perturb_value(t.x, mw[q] & 1u, vi);
        t.y = perturb_value(t.y, (mw[q] >> 1) & 1u, vi);
        t.z = perturb_value(t.z, (mw[q] >> 2) & 1u, vi);
        t.w = perturb_value(t.w, (mw[q] >> 3) & 1u, vi);
      }
      float* dst = (NORM && u < dim / 4) ? s_w + 4 * u : s_a + 4 * (u - (NORM ? dim / 4 : 0));
      *reinterpret_cast<float4*>(dst) = t;
    }
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kWarps = kNormThreads / 32;
  for (int r = warp; r < kNormRowsPerBlock; r += kWarps) {
    const int row = row0 + r;
    if (row >= a.rows) break;
    float2 v[NP];
    if (NORM) {
      const float2* src = reinterpret_cast<const float2*>(static_cast<const float*>(a.in) + (long long)row * dim);
#pragma unroll
      for (int k = 0; k < NP; ++k) v[k] = src[lane + 32 * k];
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < NP; ++k) ss += v[k].x * v[k].x + v[k].y * v[k].y;
      ss = warp_sum(ss);
      const float m = __fmul_rn(ss, 1.0f / (float)dim);
      const float rstd = 1.0f / sqrtf(__fadd_rn(m, 1e-5f));
      HV* dst = reinterpret_cast<HV*>(static_cast<T*>(a.xn) + (long long)row * dim);
#pragma unroll
      for (int k = 0; k < NP; ++k) {
        const int c = 2 * (lane + 32 * k);
        v[k].x = __fmul_rn(__fmul_rn(v[k].x, rstd), s_w[c]);
        v[k].y = __fmul_rn(__fmul_rn(v[k].y, rstd), s_w[c + 1]);
        dst[lane + 32 * k] = H2<T>::from_f2(v[k].x, v[k].y);
      }
    } else {
      const HV* src = reinterpret_cast<const HV*>(static_cast<const T*>(a.in) + (long long)row * dim);
#pragma unroll
      for (int k = 0; k < NP; ++k) v[k] = H2<T>::to_f2(src[lane + 32 * k]);
    }
    if (NA > 0) {
      constexpr int NV = PadPow2<NA>::v;
      float acc[32];
#pragma unroll
      for (int ja = 0; ja < 32; ++ja) acc[ja] = 0.f;
#pragma unroll
      for (int ja = 0; ja < NA; ++ja) {
        const float2* arow = reinterpret_cast<const float2*>(s_a + ja * dim);
        float p = 0.f;
#pragma unroll
        for (int k = 0; k < NP; ++k) {
          const float2 w = arow[lane + 32 * k];
          p = fmaf(v[k].x, w.x, p);
          p = fmaf(v[k].y, w.y, p);
        }
        acc[ja] = p;
      }
      transpose_reduce<NV>(acc, lane);
      if (lane < NA) {
        const int m = lane / a.rank, j = lane - m * a.rank;
        static_cast<T*>(a.U)[(long long)row * kUCols + a.u_col + 16 * m + j] = static_cast<T>(acc[0]);
      }
    }
  }
}

// RMSNorm (optional) + LoRA-down on the tensor cores: a 64-row tile of the
// (normalised) input is kept in shared memory as 16-bit, the perturbed A rows
// of the tile's variant are staged next to it, and U = X · A^T is computed with
// mma.sync m16n8k16 (fp32 accumulation), then rounded to 16 bit like the U
// operand of the LoRA-up tensor-core step that consumes it.
constexpr int kLdRows = 32;

template <int NP, typename T, bool NORM, int NA>
__global__ void __launch_bounds__(256, 2) norm_lora_mma_kernel(NormLoraArgs a) {
  constexpr int dim = NP * 64;
  constexpr int XS = dim + 8;                 // padded row stride (elements): conflict-free ldmatrix
  constexpr int NT = (NA + 7) / 8;            // 8-column n-tiles of U
  extern __shared__ __align__(16) uint8_t smx[];
  float* s_w = reinterpret_cast<float*>(smx);                                 // [dim] fp32
  T* s_a = reinterpret_cast<T*>(smx + dim * 4);                               // [NT*8][XS]
  T* s_x = reinterpret_cast<T*>(smx + dim * 4 + NT * 8 * XS * 2);             // [kLdRows][XS]
  using HV = typename H2<T>::V;
  const int row0 = blockIdx.x * kLdRows;
  const int grp = row0 / a.pc.group_rows;
  const int var = a.pc.group_variant[grp];
  const VariantInfo vi = a.pc.variants[var];
  const uint32_t* mask = a.pc.masks + (long long)(vi.mode ? vi.mask_slot : 0) * a.pc.mask_words;

  if (a.a_prep) {
    // ---- prepared operands: 16-bit A rows and fp32 rms weight of this variant, by cp.async ----
    const T* ap = static_cast<const T*>(a.a_prep) + (long long)var * a.a_prep_vstride;
    const uint32_t sab = smem_u32(s_a);
    for (int i = threadIdx.x; i < NT * 8 * (dim / 8); i += 256) {
      const int r = i / (dim / 8), c8 = i - r * (dim / 8);
      if (r < NA)
        cp_async16(sab + (uint32_t)((r * XS + c8 * 8) * 2), ap + (long long)r * a.a_prep_ld + c8 * 8);
      else
        *reinterpret_cast<uint4*>(s_a + r * XS + c8 * 8) = make_uint4(0u, 0u, 0u, 0u);
    }
    if (NORM) {
      const float* wp = a.w_prep + (long long)var * a.w_prep_vstride;
      const uint32_t swb = smem_u32(s_w);
      for (int i = threadIdx.x; i < dim / 4; i += 256) cp_async16(swb + 16u * i, wp + 4 * i);
    }
    cp_async_commit();
  }
  // ---- otherwise stage perturbed rms weight (fp32) and A rows (16-bit; rows >= NA zero) from theta ----
  constexpr int kWU = NORM ? dim / 4 : 0;
  constexpr int kUnits = kWU + NT * 8 * dim / 4;
  for (int u0 = threadIdx.x; !a.a_prep && u0 < kUnits; u0 += 8 * 256) {
    float4 th[8];
    uint32_t mw[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int u = u0 + q * 256;
      th[q] = make_float4(0.f, 0.f, 0.f, 0.f);
      mw[q] = 0u;
      if (u >= kUnits) continue;
      long long p;
      if (u < kWU) {
        p = a.w_off + 4LL * u;
      } else {
        const int i = 4 * (u - kWU);
        const int ja = i / dim, c = i - ja * dim;
        if (ja >= NA) continue;
        const int m = ja / a.rank, j = ja - m * a.rank;
        p = a.a_off[m] + (long long)j * dim + c;
      }
      th[q] = __ldg(reinterpret_cast<const float4*>(a.pc.theta + p));
      mw[q] = vi.mode ? (__ldg(mask + (p >> 5)) >> (p & 31)) : 0u;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int u = u0 + q * 256;
      if (u >= kUnits) break;
      float4 t = th[q];
      if (vi.mode) {
        t.x = perturb_value(t.x, mw[q] & 1u, vi);
        t.y = perturb_value(t.y, (mw[q] >> 1) & 1u, vi);
        t.z = perturb_value(t.z, (mw[q] >> 2) & 1u, vi);
        t.w = perturb_value(t.w, (mw[q] >> 3) & 1u, vi);
      }
      if (u < kWU) {
        *reinterpret_cast<float4*>(s_w + 4 * u) = t;
      } else {
        const int i = 4 * (u - kWU);
        const int ja = i / dim, c = i - ja * dim;
        HV* d = reinterpret_cast<HV*>(s_a + ja * XS + c);
        d[0] = H2<T>::from_f2(t.x, t.y);
        d[1] = H2<T>::from_f2(t.z, t.w);
      }
    }
  }
  if (a.a_prep) cp_async_wait<0>();
  __syncthreads();

  // ---- input tile: RMSNorm to HBM + smem, or a copy of the 16-bit rows ----
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (NORM) {
    // each warp normalises rows warp, warp+8, ...; the next row's loads are in
    // flight while the current row is reduced and written
    float2 cur[NP], nxt[NP];
    auto load_row = [&](float2 (&v)[NP], int r) {
      const int row = row0 + r;
      if (row < a.rows) {
        const float2* src = reinterpret_cast<const float2*>(static_cast<const float*>(a.in) + (long long)row * dim);
#pragma unroll
        for (int k = 0; k < NP; ++k) v[k] = src[lane + 32 * k];
      } else {
#pragma unroll
        for (int k = 0; k < NP; ++k) v[k] = make_float2(0.f, 0.f);
      }
    };
    load_row(cur, warp);
#pragma unroll 1
    for (int r = warp; r < kLdRows; r += 8) {
      if (r + 8 < kLdRows) load_row(nxt, r + 8);
      const int row = row0 + r;
      HV* sx = reinterpret_cast<HV*>(s_x + r * XS);
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < NP; ++k) ss += cur[k].x * cur[k].x + cur[k].y * cur[k].y;
      ss = warp_sum(ss);
      const float m = __fmul_rn(ss, 1.0f / (float)dim);
      const float rstd = 1.0f / sqrtf(__fadd_rn(m, 1e-5f));
      HV* dst = reinterpret_cast<HV*>(static_cast<T*>(a.xn) + (long long)row * dim);
#pragma unroll
      for (int k = 0; k < NP; ++k) {
        const int c = 2 * (lane + 32 * k);
        const HV h = H2<T>::from_f2(__fmul_rn(__fmul_rn(cur[k].x, rstd), s_w[c]),
                                    __fmul_rn(__fmul_rn(cur[k].y, rstd), s_w[c + 1]));
        if (row < a.rows) dst[lane + 32 * k] = h;
        sx[lane + 32 * k] = h;
      }
#pragma unroll
      for (int k = 0; k < NP; ++k) cur[k] = nxt[k];
    }
  } else {
    // whole tile in flight at once: 16-byte cp.async per (row, chunk)
    const uint32_t sxb0 = smem_u32(s_x);
    for (int i = threadIdx.x; i < kLdRows * (dim / 8); i += 256) {
      const int r = i / (dim / 8), c8 = i - r * (dim / 8);
      const int row = row0 + r;
      const uint32_t dsts = sxb0 + (uint32_t)((r * XS + c8 * 8) * 2);
      if (row < a.rows) {
        cp_async16(dsts, static_cast<const T*>(a.in) + (long long)row * dim + c8 * 8);
      } else {
        *reinterpret_cast<uint4*>(s_x + r * XS + c8 * 8) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    cp_async_commit();
    cp_async_wait<0>();
  }
  __syncthreads();

  // ---- U[rows x 8NT] = X[rows x dim] · A[8NT x dim]^T  (mma.sync m16n8k16), one (m16, n8) task per warp ----
  constexpr int MT = kLdRows / 16;
  const int lm = lane >> 3, lr = lane & 7;
  const uint32_t sxb = smem_u32(s_x), sab = smem_u32(s_a);
  for (int task = warp; task < MT * NT; task += 8) {
    const int mt = task % MT, nt = task / MT;
    float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int kk = 0; kk < dim / 16; ++kk) {
      uint32_t af[4], b0, b1, b2, b3;
      ldsm_x4(sxb + (uint32_t)(((mt * 16 + (lm & 1) * 8 + lr) * XS + kk * 16 + (lm >> 1) * 8) * 2), af[0], af[1],
              af[2], af[3]);
      // x4 over the 8 A rows of the n-tile: k 0-7, k 8-15 (b0, b1); the second pair repeats them
      ldsm_x4(sab + (uint32_t)(((nt * 8 + lr) * XS + kk * 16 + (lm & 1) * 8) * 2), b0, b1, b2, b3);
      mma16816<T>(c, af, b0, b1);
    }
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int rr = mt * 16 + g + ((e >> 1) << 3);
      const int n = nt * 8 + 2 * t + (e & 1);
      const int row = row0 + rr;
      if (n < NA && row < a.rows) {
        const int m = n / a.rank, j = n - m * a.rank;
        static_cast<T*>(a.U)[(long long)row * kUCols + a.u_col + 16 * m + j] = static_cast<T>(c[e]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Persistent LoRA-down kernels with prepared operands. Each CTA takes a
// contiguous range of 16-row tiles; loader warps fill a ring of 16-bit tiles in
// shared memory (full/empty mbarriers with bounded waits) and LoRA warps take
// whole tiles from it in turn, U = X · A^T over the full K with mma.sync
// m16n8k16 (fp32 accumulation), rounded to 16 bit like the U operand of the
// LoRA-up tensor-core step that consumes it. No CTA-wide barrier inside the loop.
//
// Variant operands: the range meets groups g0 .. g0 + k_last (group = row /
// group_rows); group g0 + k uses operand slot k % VS. Slots 0 .. VS-1 are staged
// at the start; at the first tile of a group k >= VS the role that reads a slot
// meets on its own named barrier (all of its tiles before that group are done,
// so nobody still reads group k - VS), restages the slot and meets again.
// ---------------------------------------------------------------------------

// One warp's 16 x (8 NT) product over K = 16 KS: X rows at sxb, A rows at sab (16-bit,
// row pitch XS elements, conflict-free ldmatrix). K-step kk accumulates into chain
// kk % 4 (four independent mma dependency chains); the chains are added at the end
// as (c0 + c1) + (c2 + c3).
template <typename T, int NT, int KS, int XS>
__device__ __forceinline__ void warp_tile_down(uint32_t sxb, uint32_t sab, int lane, float (&c)[NT][4]) {
  static_assert(KS % 4 == 0, "K must be a multiple of 64");
  float acc[4][NT][4];
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[q][nt][e] = 0.f;
  const int lm = lane >> 3, lr = lane & 7;
  // A fragment: matrices (rows 0-7 | 8-15) x (k 0-7 | 8-15); B: one x4 load gives
  // k-steps kk and kk + 1, low and high k halves, of an 8-row n-tile of A
  const uint32_t a_off = (uint32_t)((((lm & 1) * 8 + lr) * XS + (lm >> 1) * 8) * 2);
  const uint32_t b_off = (uint32_t)((lr * XS + (lm >> 1) * 16 + (lm & 1) * 8) * 2);
#pragma unroll 1
  for (int kk = 0; kk < KS; kk += 4) {
    uint32_t af[4][4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      ldsm_x4(sxb + a_off + (uint32_t)((kk + q) * 32), af[q][0], af[q][1], af[q][2], af[q][3]);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sab + b_off + (uint32_t)(nt * 8 * XS * 2 + (kk + 2 * h) * 32), b0, b1, b2, b3);
        mma16816<T>(acc[2 * h][nt], af[2 * h], b0, b1);
        mma16816<T>(acc[2 * h + 1][nt], af[2 * h + 1], b2, b3);
      }
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) c[nt][e] = (acc[0][nt][e] + acc[1][nt][e]) + (acc[2][nt][e] + acc[3][nt][e]);
}

// U[row0 + r, u_col + 16 m + j] for the accumulator fragment of warp_tile_down
// (column n = m * rank + j < NA), rows past a.rows skipped.
template <typename T, int NT, int NA>
__device__ __forceinline__ void store_u_tile(const NormLoraArgs& a, int row0, int lane, const float (&c)[NT][4]) {
  const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int n = nt * 8 + 2 * t4 + (e & 1), row = row0 + g + ((e >> 1) << 3);
      if (n < NA && row < a.rows) {
        const int m = n / a.rank, j = n - m * a.rank;
        static_cast<T*>(a.U)[(long long)row * kUCols + a.u_col + 16 * m + j] = static_cast<T>(c[nt][e]);
      }
    }
}

// Stage the prepared A rows of `var` (NA rows of dim 16-bit values) into a slot
// of pitch XS, by `nthr` threads (index tid); waits for its own copies.
template <typename T, int NA, int dim, int XS>
__device__ __forceinline__ void stage_a_rows(const NormLoraArgs& a, int var, T* slot, int tid, int nthr) {
  const T* ap = static_cast<const T*>(a.a_prep) + (long long)var * a.a_prep_vstride;
  const uint32_t dst = smem_u32(slot);
  for (int i = tid; i < NA * (dim / 8); i += nthr) {
    const int r = i / (dim / 8), c8 = i - r * (dim / 8);
    cp_async16(dst + (uint32_t)((r * XS + c8 * 8) * 2), ap + (long long)r * a.a_prep_ld + c8 * 8);
  }
  cp_async_commit();
  cp_async_wait<0>();
}

// Zero the rows NA .. 8 NT - 1 of every A slot (the n-tile padding; never restaged).
template <typename T, int NA, int NT, int XS, int VS>
__device__ __forceinline__ void zero_a_padding(T* s_a, int tid, int nthr) {
  if constexpr (NA < NT * 8) {
    constexpr int kPer = (NT * 8 - NA) * (XS / 8);  // 16-byte chunks per slot
    for (int i = tid; i < VS * kPer; i += nthr) {
      const int sl = i / kPer, rem = i - sl * kPer;
      const int r = NA + rem / (XS / 8), c8 = rem % (XS / 8);
      *reinterpret_cast<uint4*>(s_a + (sl * NT * 8 + r) * XS + c8 * 8) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

// LoRA-down of a 16-bit input (no norm): one loader warp moves each tile's rows
// with 1-D bulk copies (one per row, into rows of pitch XS) completing on the
// tile's full barrier; CW LoRA warps take tiles in turn. Tile i uses slot i % NS
// with NS a multiple of CW, so each LoRA warp has slots of its own and waits for
// their phases in order (a warp never waits on a slot whose previous phase, a tile
// of another warp, may still be pending: bulk copies complete in any order).
template <int NP, int NA>
struct LdSmem {
  static constexpr int RT = 16, CW = NP <= 16 ? 4 : 2, THREADS = 32 * (CW + 1);
  static constexpr int dim = NP * 64, XS = dim + 8, NT = (NA + 7) / 8, KS = dim / 16;
  static constexpr int kX = RT * XS * 2;      // one 16-bit tile
  static constexpr int kA = NT * 8 * XS * 2;  // one variant's A rows (zero padded to whole n-tiles)
  static constexpr int kBudget = 227 * 1024 - 128;
  static constexpr int VS = 2 * kA + 3 * kX <= kBudget ? 2 : 1;
  static constexpr int kFit = (kBudget - VS * kA) / kX;
  static constexpr int NS = (kFit >= 6 ? 6 : kFit) / CW * CW;
  static constexpr int kAOff = NS * kX, kBarOff = kAOff + VS * kA;
  static constexpr int kTotal = kBarOff + (2 * NS + 2) * 8;
};

template <int NP, typename T, int NA>
__global__ void __launch_bounds__(LdSmem<NP, NA>::THREADS, 1) lora_down_kernel(NormLoraArgs a, uint32_t* status) {
  using S = LdSmem<NP, NA>;
  constexpr int RT = S::RT, CW = S::CW, dim = S::dim, XS = S::XS, NT = S::NT, VS = S::VS, NS = S::NS;
  extern __shared__ __align__(16) uint8_t smx[];
  T* s_x = reinterpret_cast<T*>(smx);                 // [NS][RT][XS]
  T* s_a = reinterpret_cast<T*>(smx + S::kAOff);      // [VS][NT*8][XS]
  uint64_t* full = reinterpret_cast<uint64_t*>(smx + S::kBarOff);
  uint64_t* empty = full + NS;
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(empty + NS);
  pdl_enter();
  const int ntiles = (a.rows + RT - 1) / RT;
  const int t_begin = (int)((long long)blockIdx.x * ntiles / gridDim.x);
  const int t_end = (int)((long long)(blockIdx.x + 1) * ntiles / gridDim.x);
  if (t_begin >= t_end) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 32);
    }
    *abort_flag = 0u;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == CW) {
    // ---- loader ----
    const T* in = static_cast<const T*>(a.in);
    int issued = 0;
    for (int tile = t_begin; tile < t_end; ++tile, ++issued) {
      const int i = tile - t_begin, slot = i % NS;
      if (!mbar_wait(&empty[slot], ((i / NS) & 1) ^ 1, abort_flag, status, DEV_TIMEOUT_PRODUCER)) break;
      const int row0 = tile * RT;
      const int nr = a.rows - row0 < RT ? a.rows - row0 : RT;
      if (lane == 0) mbar_arrive_expect_tx(&full[slot], (uint32_t)(nr * dim * 2));
      __syncwarp();
      if (lane < nr)
        bulk_load(s_x + (slot * RT + lane) * XS, in + (long long)(row0 + lane) * dim, dim * 2, &full[slot]);
    }
    // copies still in flight when the consumers gave up (abort path) land before the CTA exits
    for (int i = issued - 1; i >= 0 && i >= issued - NS; --i) mbar_wait_drain(&full[i % NS], (i / NS) & 1);
    return;
  }

  // ---- LoRA warps ----
  const int g0 = (t_begin * RT) / a.pc.group_rows;
  const int k_last = ((t_end - 1) * RT) / a.pc.group_rows - g0;
  const int tid = threadIdx.x;  // 0 .. 32 CW - 1
  zero_a_padding<T, NA, NT, XS, VS>(s_a, tid, 32 * CW);
  for (int k = 0; k < VS && k <= k_last; ++k)
    stage_a_rows<T, NA, dim, XS>(a, a.pc.group_variant[g0 + k], s_a + k * NT * 8 * XS, tid, 32 * CW);
  named_bar_sync(1, 32 * CW);
  int kdone = VS - 1;
  auto advance = [&](int k) {
    while (kdone < k) {
      ++kdone;
      named_bar_sync(1, 32 * CW);
      stage_a_rows<T, NA, dim, XS>(a, a.pc.group_variant[g0 + kdone], s_a + (kdone % VS) * NT * 8 * XS, tid,
                                   32 * CW);
      named_bar_sync(1, 32 * CW);
    }
  };
  for (int tile = t_begin + warp; tile < t_end; tile += CW) {
    const int k = (tile * RT) / a.pc.group_rows - g0;
    advance(k);
    const int i = tile - t_begin, slot = i % NS;
    if (mbar_wait(&full[slot], (i / NS) & 1, abort_flag, status, DEV_TIMEOUT_MMA)) {
      float c[NT][4];
      warp_tile_down<T, NT, S::KS, XS>(smem_u32(s_x + slot * RT * XS), smem_u32(s_a + (k % VS) * NT * 8 * XS), lane,
                                       c);
      store_u_tile<T, NT, NA>(a, tile * RT, lane, c);
    }
    mbar_arrive(&empty[slot]);
  }
  advance(k_last);
}

// RMSNorm (perturbed weight) + LoRA-down: NW norm warps take the rows of the range in
// turn (row j to warp j % NW), keep their next two rows in flight in registers while
// they normalise the current one (the same arithmetic and per-lane order as
// norm_lora_mma_kernel) and write it to HBM (xn) and, as 16 bit, into the tile ring;
// LW LoRA warps take tiles in turn. 16 warps in all, so that a thread may hold 128
// registers. The norm warps restage the rms weight slots, the LoRA warps the A slots.
template <int NP, int NA>
struct NdSmem {
  static constexpr int RT = 16, NW = 14, LW = 2, THREADS = 32 * (NW + LW);
  static constexpr int dim = NP * 64, XS = dim + 8, NT = (NA + 7) / 8, KS = dim / 16, VS = 2;
  static constexpr int kX = RT * XS * 2, kA = NT * 8 * XS * 2, kW = dim * 4;
  static constexpr int kFit = (227 * 1024 - 128 - VS * (kA + kW)) / kX;
  static constexpr int NS = (kFit >= 4 ? 4 : kFit) / LW * LW;  // a multiple of LW, as in LdSmem
  static_assert(NW <= RT, "every norm warp has a row in every tile");
  static constexpr int kAOff = NS * kX, kWOff = kAOff + VS * kA, kBarOff = kWOff + VS * kW;
  static constexpr int kTotal = kBarOff + (2 * NS + 2) * 8;
};

template <int NP, typename T, int NA>
__global__ void __launch_bounds__(NdSmem<NP, NA>::THREADS, 1) norm_down_kernel(NormLoraArgs a, uint32_t* status) {
  using S = NdSmem<NP, NA>;
  constexpr int RT = S::RT, NW = S::NW, LW = S::LW, dim = S::dim, XS = S::XS, NT = S::NT, VS = S::VS,
                NS = S::NS;
  using HV = typename H2<T>::V;
  extern __shared__ __align__(16) uint8_t smx[];
  T* s_x = reinterpret_cast<T*>(smx);                      // [NS][RT][XS]
  T* s_a = reinterpret_cast<T*>(smx + S::kAOff);           // [VS][NT*8][XS]
  float* s_w = reinterpret_cast<float*>(smx + S::kWOff);   // [VS][dim]
  uint64_t* full = reinterpret_cast<uint64_t*>(smx + S::kBarOff);
  uint64_t* empty = full + NS;
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(empty + NS);
  pdl_enter();
  const int ntiles = (a.rows + RT - 1) / RT;
  const int t_begin = (int)((long long)blockIdx.x * ntiles / gridDim.x);
  const int t_end = (int)((long long)(blockIdx.x + 1) * ntiles / gridDim.x);
  if (t_begin >= t_end) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 32 * RT);  // every lane of every row of the tile
      mbar_init(&empty[s], 32);
    }
    *abort_flag = 0u;
    fence_mbar_init();
  }
  __syncthreads();
  const int g0 = (t_begin * RT) / a.pc.group_rows;
  const int k_last = ((t_end - 1) * RT) / a.pc.group_rows - g0;

  if (warp < NW) {
    // ---- norm warps ----
    const float2* in = static_cast<const float2*>(a.in);
    const int r_begin = t_begin * RT, nrows = (t_end - t_begin) * RT;  // rows past a.rows normalise zeros
    auto load_row = [&](int q, float2 (&v)[NP]) {
      const int j = warp + NW * q, row = r_begin + j;
      if (j < nrows && row < a.rows) {
        const float2* src = in + (long long)row * (dim / 2);
#pragma unroll
        for (int k = 0; k < NP; ++k) v[k] = __ldg(src + lane + 32 * k);
      } else {
#pragma unroll
        for (int k = 0; k < NP; ++k) v[k] = make_float2(0.f, 0.f);
      }
    };
    auto stage_w = [&](int k) {
      const float* wp = a.w_prep + (long long)a.pc.group_variant[g0 + k] * a.w_prep_vstride;
      const uint32_t dst = smem_u32(s_w + (k % VS) * dim);
      for (int i = threadIdx.x; i < dim / 4; i += 32 * NW) cp_async16(dst + 16u * i, wp + 4 * i);
      cp_async_commit();
      cp_async_wait<0>();
    };
    float2 xa[NP], xb[NP], xc[NP];
    load_row(0, xa);
    load_row(1, xb);
    for (int k = 0; k < VS && k <= k_last; ++k) stage_w(k);
    named_bar_sync(1, 32 * NW);
    int kdone = VS - 1;
    auto advance = [&](int k) {
      while (kdone < k) {  // every norm warp is past the rows of group kdone + 1 - VS
        ++kdone;
        named_bar_sync(1, 32 * NW);
        stage_w(kdone);
        named_bar_sync(1, 32 * NW);
      }
    };
    // normalise range row j = warp + NW q (j < nrows)
    auto norm_row = [&](int q, const float2 (&v)[NP]) {
      const int j = warp + NW * q, row = r_begin + j;
      const int k = (r_begin + (j / RT) * RT) / a.pc.group_rows - g0;  // the tile's group (rows past a.rows too)
      advance(k);
      const int i = j / RT, slot = i % NS;
      mbar_wait(&empty[slot], ((i / NS) & 1) ^ 1, abort_flag, status, DEV_TIMEOUT_PRODUCER);
      const float* w = s_w + (k % VS) * dim;
      float ss = 0.f;
#pragma unroll
      for (int p = 0; p < NP; ++p) ss += v[p].x * v[p].x + v[p].y * v[p].y;
      ss = warp_sum(ss);
      const float m = __fmul_rn(ss, 1.0f / (float)dim);
      const float rstd = 1.0f / sqrtf(__fadd_rn(m, 1e-5f));
      HV* sx = reinterpret_cast<HV*>(s_x + (slot * RT + j % RT) * XS);
      HV* dst = reinterpret_cast<HV*>(static_cast<T*>(a.xn) + (long long)row * dim);
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        const int c = 2 * (lane + 32 * p);
        const HV h = H2<T>::from_f2(__fmul_rn(__fmul_rn(v[p].x, rstd), w[c]),
                                    __fmul_rn(__fmul_rn(v[p].y, rstd), w[c + 1]));
        if (row < a.rows) dst[lane + 32 * p] = h;
        sx[lane + 32 * p] = h;
      }
      mbar_arrive(&full[slot]);
    };
    const int nq = (nrows - warp + NW - 1) / NW;  // rows of this warp
    for (int q = 0; q < nq; q += 3) {
      load_row(q + 2, xc);
      norm_row(q, xa);
      if (q + 1 >= nq) break;
      load_row(q + 3, xa);
      norm_row(q + 1, xb);
      if (q + 2 >= nq) break;
      load_row(q + 4, xb);
      norm_row(q + 2, xc);
    }
    advance(k_last);
    return;
  }

  // ---- LoRA warps ----
  const int lw = warp - NW, tid = threadIdx.x - 32 * NW;
  zero_a_padding<T, NA, NT, XS, VS>(s_a, tid, 32 * LW);
  for (int k = 0; k < VS && k <= k_last; ++k)
    stage_a_rows<T, NA, dim, XS>(a, a.pc.group_variant[g0 + k], s_a + k * NT * 8 * XS, tid, 32 * LW);
  named_bar_sync(2, 32 * LW);
  int kdone = VS - 1;
  auto advance = [&](int k) {
    while (kdone < k) {
      ++kdone;
      named_bar_sync(2, 32 * LW);
      stage_a_rows<T, NA, dim, XS>(a, a.pc.group_variant[g0 + kdone], s_a + (kdone % VS) * NT * 8 * XS, tid,
                                   32 * LW);
      named_bar_sync(2, 32 * LW);
    }
  };
  for (int tile = t_begin + lw; tile < t_end; tile += LW) {
    const int k = (tile * RT) / a.pc.group_rows - g0;
    advance(k);
    const int i = tile - t_begin, slot = i % NS;
    if (mbar_wait(&full[slot], (i / NS) & 1, abort_flag, status, DEV_TIMEOUT_MMA)) {
      float c[NT][4];
      warp_tile_down<T, NT, S::KS, XS>(smem_u32(s_x + slot * RT * XS), smem_u32(s_a + (k % VS) * NT * 8 * XS), lane,
                                       c);
      store_u_tile<T, NT, NA>(a, tile * RT, lane, c);
    }
    mbar_arrive(&empty[slot]);
  }
  advance(k_last);
}

template <typename S, auto K>  // one instantiation (and shared-memory attribute) per kernel
static int launch_down(const NormLoraArgs& a, cudaStream_t st) {
  constexpr auto k = K;
  static_assert(S::kTotal <= 227 * 1024, "LoRA-down tiles exceed shared memory");
  static_assert(S::NS >= 2, "LoRA-down needs at least two ring slots");
  B2P_REQUIRE(a.pc.group_rows % S::RT == 0, "variant groups must be multiples of %d rows", S::RT);
  DeviceCtx* c = nullptr;
  int rc = ctx_get(&c);
  if (rc) return rc;
  static thread_local uint64_t attr_mask = 0;  // one per instantiation
  if (!(attr_mask & (1ull << (c->device & 63)))) {
    B2P_CHECK_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal));
    attr_mask |= 1ull << (c->device & 63);
  }
  const int ntiles = (a.rows + S::RT - 1) / S::RT;
  const int grid = ntiles < c->num_sms ? ntiles : c->num_sms;
  B2P_CHECK_CUDA(launch_pdl(k, dim3(grid), dim3(S::THREADS), S::kTotal, st, a, c->status));
  B2P_POST_LAUNCH();
  return B2P_OK;
}

template <int NP, typename T, int NA>
static int launch_norm_down(const NormLoraArgs& a, cudaStream_t st) {
  return launch_down<NdSmem<NP, NA>, norm_down_kernel<NP, T, NA>>(a, st);
}

template <int NP, typename T, int NA>
static int launch_lora_down(const NormLoraArgs& a, cudaStream_t st) {
  B2P_REQUIRE(((uintptr_t)a.in & 15) == 0, "LoRA-down input must be 16-byte aligned");
  return launch_down<LdSmem<NP, NA>, lora_down_kernel<NP, T, NA>>(a, st);
}

template <int NP, typename T, bool NORM, int NA>
static int launch_nl_mma(const NormLoraArgs& a, cudaStream_t st) {
  constexpr int dim = NP * 64, XS = dim + 8, NT = (NA + 7) / 8;
  const size_t smem = (size_t)dim * 4 + (size_t)NT * 8 * XS * 2 + (size_t)kLdRows * XS * 2;
  auto k = norm_lora_mma_kernel<NP, T, NORM, NA>;
  B2P_CHECK_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  k<<<(a.rows + kLdRows - 1) / kLdRows, 256, smem, st>>>(a);
  B2P_POST_LAUNCH();
  return B2P_OK;
}

template <int NP, typename T, bool NORM, int NA>
static int launch_nl(const NormLoraArgs& a, size_t smem, int blocks, cudaStream_t st) {
  auto k = norm_lora_kernel<NP, T, NORM, NA>;
  B2P_CHECK_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  B2P_CHECK_CUDA(launch_pdl(k, dim3(blocks), dim3(kNormThreads), smem, st, a));
  B2P_POST_LAUNCH();
  return B2P_OK;
}

template <int NP, typename T, bool NORM>
static int launch_nl_na(const NormLoraArgs& a, size_t smem, int blocks, cudaStream_t st) {
  if (!NORM && a.a_prep) {
    switch (a.n_a * a.rank) {
      case 4: return launch_lora_down<NP, T, 4>(a, st);
      case 8: return launch_lora_down<NP, T, 8>(a, st);
      default: break;
    }
  }
  if constexpr (NORM && NP <= 16) {  // the norm warps' register ring fits up to dim 1024
    if (a.a_prep && a.w_prep) {
      switch (a.n_a * a.rank) {
        case 8: return launch_norm_down<NP, T, 8>(a, st);
        case 12: return launch_norm_down<NP, T, 12>(a, st);
        case 16: return launch_norm_down<NP, T, 16>(a, st);
        case 24: return launch_norm_down<NP, T, 24>(a, st);
        default: break;
      }
    }
  }
  switch (a.n_a * a.rank) {
    case 0: return launch_nl<NP, T, NORM, 0>(a, smem, blocks, st);
    case 4: return launch_nl_mma<NP, T, NORM, 4>(a, st);
    case 8: return launch_nl_mma<NP, T, NORM, 8>(a, st);
    case 12: return launch_nl_mma<NP, T, NORM, 12>(a, st);
    case 16: return launch_nl_mma<NP, T, NORM, 16>(a, st);
    case 24: return launch_nl_mma<NP, T, NORM, 24>(a, st);
    default:
      set_error("norm/LoRA-down: unsupported LoRA-down row count %d", a.n_a * a.rank);
      return B2P_ERR_UNSUPPORTED;
  }
}

template <typename T, bool NORM>
static int launch_norm_lora_t(const NormLoraArgs& a, cudaStream_t st) {
  const int np = a.dim / 64;
  const size_t smem = sizeof(float) * ((size_t)a.dim + (size_t)a.n_a * a.rank * a.dim);
  const int blocks = (a.rows + kNormRowsPerBlock - 1) / kNormRowsPerBlock;
  switch (np) {
    case 8: return launch_nl_na<8, T, NORM>(a, smem, blocks, st);
    case 15: return launch_nl_na<15, T, NORM>(a, smem, blocks, st);
    case 16: return launch_nl_na<16, T, NORM>(a, smem, blocks, st);
    case 32: return launch_nl_na<32, T, NORM>(a, smem, blocks, st);
    default:
      break;
  }
  // LoRA-down of a gated FFN activation (--lora-ffn A2, no norm): the hidden widths
  if (!NORM && a.a_prep && (a.n_a * a.rank == 4 || a.n_a * a.rank == 8)) {
    const bool r8 = a.n_a * a.rank == 8;
    switch (np) {
      case 18: return r8 ? launch_lora_down<18, T, 8>(a, st) : launch_lora_down<18, T, 4>(a, st);
      case 22: return r8 ? launch_lora_down<22, T, 8>(a, st) : launch_lora_down<22, T, 4>(a, st);
      case 40: return r8 ? launch_lora_down<40, T, 8>(a, st) : launch_lora_down<40, T, 4>(a, st);
      default: break;
    }
  }
  switch (np) {
    default:
      set_error("norm/LoRA-down: unsupported width %d (need dim in {512, 960, 1024, 2048})", a.dim);
      return B2P_ERR_UNSUPPORTED;
  }
}

int launch_norm_lora(const NormLoraArgs& a, bool bf16, cudaStream_t st) {
  B2P_REQUIRE(a.dim % 64 == 0, "dim %d must be a multiple of 64", a.dim);
  B2P_REQUIRE(a.n_a >= 0 && a.n_a <= 3 && (a.n_a == 0 || (a.rank > 0 && a.rank <= 16)), "bad LoRA-down count");
  B2P_REQUIRE(a.u_col % 16 == 0 && a.u_col + 16 * a.n_a <= kUCols, "LoRA-down columns out of range");
  B2P_REQUIRE(a.w_off % 4 == 0 && a.a_off[0] % 4 == 0 && a.a_off[1] % 4 == 0 && a.a_off[2] % 4 == 0,
              "parameter offsets must be multiples of 4");
  B2P_REQUIRE(a.pc.group_rows % kNormRowsPerBlock == 0, "variant groups must be multiples of %d rows",
              kNormRowsPerBlock);
  const size_t smem = sizeof(float) * ((size_t)a.dim + (size_t)a.n_a * a.rank * a.dim);
  B2P_REQUIRE(smem <= 227 * 1024, "LoRA-down operands (%zu bytes) exceed shared memory", smem);
  if (a.norm) return bf16 ? launch_norm_lora_t<__nv_bfloat16, true>(a, st) : launch_norm_lora_t<__half, true>(a, st);
  return bf16 ? launch_norm_lora_t<__nv_bfloat16, false>(a, st) : launch_norm_lora_t<__half, false>(a, st);
}

// ---------------------------------------------------------------------------
// causal GQA attention, head_dim 64, 64-query x 64-key tiles, mma.sync m16n8k16
// ---------------------------------------------------------------------------
constexpr int kAttnTile = 64;
constexpr int kHD = 64;

// Loads a [64 rows][64 cols] 16-bit tile (row pitch ld elements) into swizzled smem.
template <typename T>
__device__ __forceinline__ void load_tile_async(uint32_t s_base, const T* g, long long ld) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = threadIdx.x + i * 128;  // 512 chunks of 16 B
    const int r = idx >> 3, c = idx & 7;
    cp_async16(s_base + swz(r, c), g + r * ld + c * 8);
  }
}

template <typename T>
__global__ void __launch_bounds__(128) attn_fwd_kernel(AttnArgs a, float scale_log2) {
  __shared__ __align__(128) uint8_t s_q[kAttnTile * kHD * 2];
  __shared__ __align__(128) uint8_t s_k[2][kAttnTile * kHD * 2];
  __shared__ __align__(128) uint8_t s_v[2][kAttnTile * kHD * 2];
  const int nqb = a.seq / kAttnTile;
  const int qb = nqb - 1 - blockIdx.x;  // longest rows first
  const int h = blockIdx.y, g = blockIdx.z;
  const int kvh = h / (a.heads / a.kv_heads);
  const T* base = static_cast<const T*>(a.qkv) + (long long)g * a.seq * a.ld_qkv;
  const T* gq = base + (long long)qb * kAttnTile * a.ld_qkv + a.q_off + h * kHD;
  const T* gk = base + a.k_off + kvh * kHD;
  const T* gv = base + a.v_off + kvh * kHD;
  const uint32_t sq = smem_u32(s_q), sk0 = smem_u32(s_k[0]), sv0 = smem_u32(s_v[0]);
  constexpr uint32_t kTileBytes = kAttnTile * kHD * 2;

  load_tile_async<T>(sq, gq, a.ld_qkv);
  load_tile_async<T>(sk0, gk, a.ld_qkv);
  load_tile_async<T>(sv0, gv, a.ld_qkv);
  cp_async_commit();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lg = lane >> 2, lt = lane & 3;
  const int lm = lane >> 3, lr = lane & 7;

  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  uint32_t qf[4][4];

  for (int kb = 0; kb <= qb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 <= qb) {
      load_tile_async<T>(sk0 + (buf ^ 1) * kTileBytes, gk + (long long)(kb + 1) * kAttnTile * a.ld_qkv, a.ld_qkv);
      load_tile_async<T>(sv0 + (buf ^ 1) * kTileBytes, gv + (long long)(kb + 1) * kAttnTile * a.ld_qkv, a.ld_qkv);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        ldsm_x4(sq + swz(warp * 16 + (lm & 1) * 8 + lr, kk * 2 + (lm >> 1)), qf[kk][0], qf[kk][1], qf[kk][2],
                qf[kk][3]);
    }
    const uint32_t skb = sk0 + buf * kTileBytes, svb = sv0 + buf * kTileBytes;
    // S = Q K^T  (16 query rows x 64 keys per warp)
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(skb + swz(nt * 16 + (lm >> 1) * 8 + lr, kk * 2 + (lm & 1)), b0, b1, b2, b3);
        mma16816<T>(s[2 * nt], qf[kk], b0, b1);
        mma16816<T>(s[2 * nt + 1], qf[kk], b2, b3);
      }
    }
    // scale (log2 domain), causal mask on the diagonal tile, online softmax
    const int q_row0 = warp * 16 + lg;  // within the tile; second row is +8
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = s[nt][e] * scale_log2;
        if (kb == qb) {
          const int key = nt * 8 + 2 * lt + (e & 1);
          const int qr = q_row0 + ((e >> 1) << 3);
          if (key > qr) v = -INFINITY;
        }
        s[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
    }
    float corr[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float m_new = fmaxf(m_run[i], mx[i]);
      corr[i] = exp2f(m_run[i] - m_new);
      m_run[i] = m_new;
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p = exp2f(s[nt][e] - m_run[e >> 1]);
        s[nt][e] = p;
        rs[e >> 1] += p;
      }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 1);
      rs[i] += __shfl_xor_sync(0xffffffffu, rs[i], 2);
      l_run[i] = l_run[i] * corr[i] + rs[i];
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      o[nt][0] *= corr[0];
      o[nt][1] *= corr[0];
      o[nt][2] *= corr[1];
      o[nt][3] *= corr[1];
    }
    // O += P V
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      uint32_t pa[4];
      pa[0] = pack_h2<T>(s[2 * kc][0], s[2 * kc][1]);
      pa[1] = pack_h2<T>(s[2 * kc][2], s[2 * kc][3]);
      pa[2] = pack_h2<T>(s[2 * kc + 1][0], s[2 * kc + 1][1]);
      pa[3] = pack_h2<T>(s[2 * kc + 1][2], s[2 * kc + 1][3]);
#pragma unroll
      for (int dt = 0; dt < 4; ++dt) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(svb + swz(kc * 16 + (lm & 1) * 8 + lr, dt * 2 + (lm >> 1)), b0, b1, b2, b3);
        mma16816<T>(o[2 * dt], pa, b0, b1);
        mma16816<T>(o[2 * dt + 1], pa, b2, b3);
      }
    }
    __syncthreads();  // buffer `buf` is refilled two iterations later
  }
  // normalise and store
  const float inv0 = 1.0f / l_run[0], inv1 = 1.0f / l_run[1];
  if (a.lse && lt == 0) {
    const long long r0 = (long long)g * a.seq + qb * kAttnTile + warp * 16 + lg;
    a.lse[r0 * a.heads + h] = m_run[0] + log2f(l_run[0]);
    a.lse[(r0 + 8) * a.heads + h] = m_run[1] + log2f(l_run[1]);
  }
  T* out = static_cast<T*>(a.out) + ((long long)g * a.seq + qb * kAttnTile + warp * 16 + lg) * a.ld_out + h * kHD;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    const int col = nt * 8 + 2 * lt;
    *reinterpret_cast<uint32_t*>(out + col) = pack_h2<T>(o[nt][0] * inv0, o[nt][1] * inv0);
    *reinterpret_cast<uint32_t*>(out + 8LL * a.ld_out + col) = pack_h2<T>(o[nt][2] * inv1, o[nt][3] * inv1);
  }
}

int launch_attention(const AttnArgs& a, bool bf16, cudaStream_t st) {
  if (attention_tc_supported(a)) return launch_attention_tc(a, bf16, st);
  B2P_REQUIRE(a.seq % kAttnTile == 0, "attention needs seq %% 64 == 0 (got %d)", a.seq);
  B2P_REQUIRE(a.kv_heads > 0 && a.heads % a.kv_heads == 0, "heads must be a multiple of kv_heads");
  B2P_REQUIRE(a.ld_qkv % 8 == 0 && a.q_off % 8 == 0 && a.k_off % 8 == 0 && a.v_off % 8 == 0 && a.ld_out % 2 == 0,
              "attention operands must be 16-byte aligned");
  dim3 grid(a.seq / kAttnTile, a.heads, a.ngroups);
  const float scale_log2 = (1.0f / sqrtf((float)kHD)) * 1.4426950408889634f;
  if (bf16)
    attn_fwd_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(a, scale_log2);
  else
    attn_fwd_kernel<__half><<<grid, 128, 0, st>>>(a, scale_log2);
  B2P_POST_LAUNCH();
  return B2P_OK;
}

// ---------------------------------------------------------------------------
// cross-entropy reduction
// ---------------------------------------------------------------------------
__global__ void ce_reduce_kernel(const float2* __restrict__ part, int ntiles, const float* __restrict__ tgt_logit,
                                 int seq, float* __restrict__ row_loss, float* __restrict__ group_loss,
                                 float* __restrict__ row_lse) {
  __shared__ float red[256];
  const int g = blockIdx.x;
  float acc = 0.f;
  for (int t = threadIdx.x; t < seq; t += blockDim.x) {
    const long long row = (long long)g * seq + t;
    const float2* p = part + row * ntiles;
    float M = -INFINITY;
    for (int i = 0; i < ntiles; ++i) M = fmaxf(M, p[i].x);
    float S = 0.f;
    for (int i = 0; i < ntiles; ++i) S += p[i].y * expf(p[i].x - M);
    const float l = -(tgt_logit[row] - M) + logf(S);
    row_loss[row] = l;
    if (row_lse) row_lse[row] = M + logf(S);
    acc += l;
  }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int s = blockDim.x / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0) group_loss[g] = red[0] / (float)seq;
}

int launch_ce_reduce(const float2* part, int ntiles, const float* tgt_logit, int rows, int seq, float* row_loss,
                     float* group_loss, cudaStream_t st, float* row_lse) {
  B2P_REQUIRE(rows % seq == 0, "rows must be whole sequences");
  ce_reduce_kernel<<<rows / seq, 256, 0, st>>>(part, ntiles, tgt_logit, seq, row_loss, group_loss, row_lse);
  B2P_POST_LAUNCH();
  return B2P_OK;
}

__global__ void variant_loss_kernel(const float* group_loss, int n_var, int n_seq, float* var_loss) {
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= n_var) return;
  float s = 0.f;
  for (int q = 0; q < n_seq; ++q) s += group_loss[v * n_seq + q];
  var_loss[v] = s / (float)n_seq;
}

int launch_variant_loss(const float* group_loss, int n_var, int n_seq, float* var_loss, cudaStream_t st) {
  variant_loss_kernel<<<(n_var + 63) / 64, 64, 0, st>>>(group_loss, n_var, n_seq, var_loss);
  B2P_POST_LAUNCH();
  return B2P_OK;
}

// ---------------------------------------------------------------------------
// in-place Rademacher steps
// ---------------------------------------------------------------------------
__global__ void perturb_kernel(float* __restrict__ theta, long long n, const uint32_t* __restrict__ masks,
                               long long mask_words, PerturbOps ops, const float* __restrict__ losses) {
  __shared__ float s_scale[kMaxPerturbOps];
  if (threadIdx.x < ops.n) {
    const PerturbOp& op = ops.op[threadIdx.x];
    float c = op.scale;
    if (op.from_loss) {
      const float lp = losses[2 * op.loss_idx], lm = losses[2 * op.loss_idx + 1];
      const float g = __fdiv_rn(__fsub_rn(lp, lm), __fmul_rn(2.0f, op.eps));  // (L+ - L-) / (2 eps)
      c = __fmul_rn(-op.lr, g);                                               // update_scale = -lr * g
      if (op.div != 1.0f) c = __fdiv_rn(c, op.div);
    }
    s_scale[threadIdx.x] = c;
  }
  __syncthreads();
  const long long w = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // one 32-parameter word per thread
  if (w >= mask_words) return;
  const long long p0 = w * 32;
  const int cnt = (int)min(32LL, n - p0);
  float v[32];
#pragma unroll
  for (int k = 0; k < 32; ++k) v[k] = k < cnt ? theta[p0 + k] : 0.f;
  for (int o = 0; o < ops.n; ++o) {
    const uint32_t bits = __ldg(masks + (long long)ops.op[o].slot * mask_words + w);
    const float c = s_scale[o];
#pragma unroll
    for (int k = 0; k < 32; ++k) v[k] = __fadd_rn(v[k], ((bits >> k) & 1u) ? c : -c);
  }
#pragma unroll
  for (int k = 0; k < 32; ++k)
    if (k < cnt) theta[p0 + k] = v[k];
}

int launch_perturb(float* theta, long long n, const uint32_t* masks, long long mask_words, const PerturbOps& ops,
                   const float* losses, cudaStream_t st) {
  B2P_REQUIRE(ops.n >= 0 && ops.n <= kMaxPerturbOps, "too many perturbation ops (%d)", ops.n);
  if (ops.n == 0) return B2P_OK;
  const int threads = 128;
  perturb_kernel<<<(unsigned)((mask_words + threads - 1) / threads), threads, 0, st>>>(theta, n, masks, mask_words,
                                                                                      ops, losses);
  B2P_POST_LAUNCH();
  return B2P_OK;
}

// ---------------------------------------------------------------------------
// layout conversion
// ---------------------------------------------------------------------------
template <typename T>
__global__ void cf_to_tm16_kernel(const float* __restrict__ src, int C, int S, T* __restrict__ dst, int ld) {
  __shared__ float tile[32][33];
  const int c0 = blockIdx.y * 32, s0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, s = s0 + threadIdx.x;
    tile[i][threadIdx.x] = (c < C && s < S) ? src[(long long)c * S + s] : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int s = s0 + i, c = c0 + threadIdx.x;
    if (s < S && c < C) dst[(long long)s * ld + c] = static_cast<T>(tile[threadIdx.x][i]);
  }
}

template <typename T, bool F32>
__global__ void tm_to_cf32_kernel(const void* __restrict__ srcv, int ld, int C, int S, float* __restrict__ dst) {
  __shared__ float tile[32][33];
  const int c0 = blockIdx.y * 32, s0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int s = s0 + i, c = c0 + threadIdx.x;
    float v = 0.f;
    if (s < S && c < C)
      v = F32 ? static_cast<const float*>(srcv)[(long long)s * ld + c]
              : static_cast<float>(static_cast<const T*>(srcv)[(long long)s * ld + c]);
    tile[i][threadIdx.x] = v;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, s = s0 + threadIdx.x;
    if (c < C && s < S) dst[(long long)c * S + s] = tile[threadIdx.x][i];
  }
}

int launch_cf_to_tm16(const float* src, int C, int S, void* dst, int ld_dst, bool bf16, cudaStream_t st) {
  dim3 grid((S + 31) / 32, (C + 31) / 32), block(32, 8);
  if (bf16)
    cf_to_tm16_kernel<__nv_bfloat16><<<grid, block, 0, st>>>(src, C, S, static_cast<__nv_bfloat16*>(dst), ld_dst);
  else
    cf_to_tm16_kernel<__half><<<grid, block, 0, st>>>(src, C, S, static_cast<__half*>(dst), ld_dst);
  B2P_POST_LAUNCH();
  return B2P_OK;
}

int launch_cf_to_tm32(const float* src, int C, int S, float* dst, int ld_dst, cudaStream_t st) {
  dim3 grid((S + 31) / 32, (C + 31) / 32), block(32, 8);
  cf_to_tm16_kernel<float><<<grid, block, 0, st>>>(src, C, S, dst, ld_dst);
  B2P_POST_LAUNCH();
  return B2P_OK;
}

int launch_tm_to_cf32(const void* src, int ld_src, bool src_f32, bool bf16, int C, int S, float* dst,
                      cudaStream_t st) {
  dim3 grid((S + 31) / 32, (C + 31) / 32), block(32, 8);
  if (src_f32)
    tm_to_cf32_kernel<float, true><<<grid, block, 0, st>>>(src, ld_src, C, S, dst);
  else if (bf16)
    tm_to_cf32_kernel<__nv_bfloat16, false><<<grid, block, 0, st>>>(src, ld_src, C, S, dst);
  else
    tm_to_cf32_kernel<__half, false><<<grid, block, 0, st>>>(src, ld_src, C, S, dst);
  B2P_POST_LAUNCH();
  return B2P_OK;
}

template <typename T>
__global__ void lora_prep_kernel(LoraPrepArgs a) {
  const int r = a.rank;
  const long long per_a = (long long)a.segs * r * a.ld;  // A elements per (layer, variant)
  const long long per_a2 = a.a2_out ? (long long)r * a.hidden : 0;
  const long long per_w = 2LL * a.dim;                // rms elements per (layer, variant)
  const long long n_a = (long long)a.nlayers * a.n_var * per_a;
  const long long n_a2 = (long long)a.nlayers * a.n_var * per_a2;
  const long long n_w = (long long)a.nlayers * a.n_var * per_w + (long long)a.n_var * a.dim;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n_a + n_a2 + n_w;
       i += (long long)gridDim.x * blockDim.x) {
    long long p;
    int v;
    bool valid = true;
    if (i < n_a + n_a2) {
      const bool a2 = i >= n_a;
      const long long ii = a2 ? i - n_a : i;
      const long long per = a2 ? per_a2 : per_a;
      const int ld = a2 ? a.hidden : a.ld;
      // 32-bit index arithmetic (the launcher checks that every count fits): 64-bit divisions cost
      // several times the rest of the element's work
      const uint32_t ii32 = (uint32_t)ii, per32 = (uint32_t)per;
      const uint32_t lv = ii32 / per32, e = ii32 - lv * per32;
      const int l = (int)(lv / (uint32_t)a.n_var);
      v = (int)(lv - (uint32_t)l * (uint32_t)a.n_var);
      const int row = (int)(e / (uint32_t)ld), c = (int)(e - (uint32_t)row * (uint32_t)ld);
      const int m = row / r, j = row - m * r;
      int width;
      long long off;
      if (a2) {
        width = a.hidden;
        off = a.oA2;
      } else {
        width = (m < 3 || m > 3) ? a.dim : a.q_dim;
        const long long offs[6] = {a.oAq, a.oAk, a.oAv, a.oAo, a.oA1, a.oA3};
        off = offs[m];
      }
      valid = c < width;
      p = (long long)l * a.layer_size + off + (long long)j * width + c;
      float val = 0.f;
      if (valid) {
        const VariantInfo vi = a.variants[v];
        const uint32_t* mask = a.masks + (long long)(vi.mode ? vi.mask_slot : 0) * a.mask_words;
        const uint32_t bit = vi.mode ? (__ldg(mask + (p >> 5)) >> (p & 31)) & 1u : 0u;
        val = perturb_value(__ldg(a.theta + p), bit, vi);
      }
      if (a2)
        static_cast<T*>(a.a2_out)[ii] = static_cast<T>(val);
      else
        static_cast<T*>(a.a_out)[ii] = static_cast<T>(val);
      continue;
    }
    const long long k = i - n_a - n_a2;
    float* dst;
    const long long nl = (long long)a.nlayers * a.n_var * per_w;
    if (k < nl) {
      const uint32_t k32 = (uint32_t)k, pw32 = (uint32_t)per_w;
      const uint32_t lv = k32 / pw32, e = k32 - lv * pw32;
      const int l = (int)(lv / (uint32_t)a.n_var);
      v = (int)(lv - (uint32_t)l * (uint32_t)a.n_var);
      const int which = (int)(e / (uint32_t)a.dim), c = (int)(e - (uint32_t)which * (uint32_t)a.dim);
      p = (long long)l * a.layer_size + (which ? a.oRf : a.oRa) + c;
      dst = a.w_out + k;
    } else {
      const uint32_t e = (uint32_t)(k - nl);
      v = (int)(e / (uint32_t)a.dim);
      p = a.oRfinal + (long long)(e - (uint32_t)v * (uint32_t)a.dim);
      dst = a.w_final + e;
    }
    const VariantInfo vi = a.variants[v];
    const uint32_t* mask = a.masks + (long long)(vi.mode ? vi.mask_slot : 0) * a.mask_words;
    const uint32_t bit = vi.mode ? (__ldg(mask + (p >> 5)) >> (p & 31)) & 1u : 0u;
    *dst = perturb_value(__ldg(a.theta + p), bit, vi);
  }
}

int launch_lora_prep(const LoraPrepArgs& a, bool bf16, cudaStream_t st) {
  B2P_REQUIRE(a.n_var >= 1 && a.rank >= 1 && a.rank <= 8 && a.ld >= a.dim && a.ld >= a.q_dim && a.ld % 8 == 0 &&
                  (a.segs == 4 || a.segs == 6) && (!a.a2_out || a.hidden % 8 == 0),
              "bad LoRA prep shape");
  {
    const long long per_a = (long long)a.segs * a.rank * a.ld, per_a2 = a.a2_out ? (long long)a.rank * a.hidden : 0;
    const long long n = (long long)a.nlayers * a.n_var * (per_a + per_a2 + 2LL * a.dim) + (long long)a.n_var * a.dim;
    B2P_REQUIRE(n < (1LL << 31), "LoRA prep of %lld elements exceeds the kernel's 32-bit indexing", n);
  }
  if (bf16)
    lora_prep_kernel<__nv_bfloat16><<<148 * 8, 256, 0, st>>>(a);
  else
    lora_prep_kernel<__half><<<148 * 8, 256, 0, st>>>(a);
  B2P_POST_LAUNCH();
  return B2P_OK;
}

template <typename T>
__global__ void swiglu_gate_kernel(const T* __restrict__ h13, int rows, int H, T* __restrict__ gate) {
  pdl_enter();
  const long long n8 = (long long)rows * H / 8;  // 8 gate columns per thread (never straddle a 128-block)
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const long long e = i * 8;
    const long long r = e / H;
    const int c = (int)(e - r * H);
    const T* src = h13 + r * 2 * H + (c >> 7) * 256 + (c & 127);
    const uint4 a = *reinterpret_cast<const uint4*>(src);
    const uint4 b = *reinterpret_cast<const uint4*>(src + 128);
    const uint32_t av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 h1 = H2<T>::to_f2(*reinterpret_cast<const typename H2<T>::V*>(&av[k]));
      const float2 h3 = H2<T>::to_f2(*reinterpret_cast<const typename H2<T>::V*>(&bv[k]));
      o[k] = pack_h2<T>(silu_f(h1.x) * h3.x, silu_f(h1.y) * h3.y);
    }
    *reinterpret_cast<uint4*>(gate + e) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

int launch_swiglu_gate(const void* h13, int rows, int H, void* gate, bool bf16, cudaStream_t st) {
  B2P_REQUIRE(H % 128 == 0, "hidden %d must be a multiple of 128", H);
  const long long n8 = (long long)rows * H / 8;
  const int blocks = (int)std::min<long long>((n8 + 255) / 256, 148 * 16);
  if (bf16)
    B2P_CHECK_CUDA(launch_pdl(swiglu_gate_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, st,
                              static_cast<const __nv_bfloat16*>(h13), rows, H, static_cast<__nv_bfloat16*>(gate)));
  else
    B2P_CHECK_CUDA(launch_pdl(swiglu_gate_kernel<__half>, dim3(blocks), dim3(256), 0, st,
                              static_cast<const __half*>(h13), rows, H, static_cast<__half*>(gate)));
  B2P_POST_LAUNCH();
  return B2P_OK;
}

template <typename T>
__global__ void f32_to_16_kernel(const float* __restrict__ src, T* __restrict__ dst, long long n) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    dst[i] = static_cast<T>(src[i]);
}

int launch_f32_to_16(const float* src, void* dst, long long n, bool bf16, cudaStream_t st) {
  const long long nb = (n + 255) / 256;
  const int blocks = (int)(nb < 148 * 16 ? nb : 148 * 16);
  if (bf16)
    f32_to_16_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(src, static_cast<__nv_bfloat16*>(dst), n);
  else
    f32_to_16_kernel<__half><<<blocks, 256, 0, st>>>(src, static_cast<__half*>(dst), n);
  B2P_POST_LAUNCH();
  return B2P_OK;
}

}  // namespace b2p
