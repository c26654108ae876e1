// rng.cu — GF(2) jump-ahead sign-mask generation (see rng.cuh).
#include <cuda_runtime.h>
#include "engine.cuh"
#include "rng.cuh"

namespace b2p {

void host_xo_seed(uint64_t s[4], uint64_t seed) {
  for (int i = 0; i < 4; i++) {
    seed += 0x9E3779B97F4A7C15ULL;
    uint64_t z = seed;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    s[i] = z ^ (z >> 31);
  }
}

static inline uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

uint64_t host_xo_next(uint64_t s[4]) {
  const uint64_t result = s[0] + s[3];
  const uint64_t t = s[1] << 17;
  s[2] ^= s[0];
  s[3] ^= s[1];
  s[1] ^= s[2];
  s[0] ^= s[3];
  s[2] ^= t;
  s[3] = rotl64(s[3], 45);
  return result;
}

namespace {
using Mat = std::vector<uint64_t>;  // 256 rows x 4 words; row i = coefficients of output bit i

inline bool bit_of(const uint64_t* v, int j) { return (v[j >> 6] >> (j & 63)) & 1u; }

// C = A * B over GF(2) (apply B first, then A).
Mat matmul(const Mat& A, const Mat& B) {
  Mat C(256 * 4, 0);
  for (int i = 0; i < 256; ++i) {
    uint64_t r[4] = {0, 0, 0, 0};
    for (int j = 0; j < 256; ++j)
      if (bit_of(&A[i * 4], j))
        for (int w = 0; w < 4; ++w) r[w] ^= B[j * 4 + w];
    for (int w = 0; w < 4; ++w) C[i * 4 + w] = r[w];
  }
  return C;
}

// Transition matrix of one xoshiro256 step (state bit b = word b/64, bit b%64).
Mat transition() {
  Mat T(256 * 4, 0);
  for (int j = 0; j < 256; ++j) {
    uint64_t s[4] = {0, 0, 0, 0};
    s[j >> 6] = 1ull << (j & 63);
    host_xo_next(s);
    for (int i = 0; i < 256; ++i)
      if (bit_of(s, i)) T[i * 4 + (j >> 6)] |= 1ull << (j & 63);
  }
  return T;
}
}  // namespace

SignPlan make_sign_plan(const std::vector<long long>& sizes) {
  SignPlan p;
  long long pp = 0, dd = 0;
  for (long long n : sizes) {
    p.bufs.push_back({pp, dd, n});
    pp += n;
    dd += n / 4 + n % 4;
  }
  p.total_params = pp;
  p.total_draws = dd;
  const long long nchunks = (dd + kChunkDraws - 1) / kChunkDraws;
  int nj = 1;
  while ((1ll << nj) < nchunks) ++nj;
  p.njump = nj;
  Mat J = transition();
  for (int k = 0; (1 << k) < kChunkDraws; ++k) J = matmul(J, J);  // T^kChunkDraws
  p.jumps.reserve((size_t)nj * 1024);
  for (int k = 0; k < nj; ++k) {
    p.jumps.insert(p.jumps.end(), J.begin(), J.end());
    J = matmul(J, J);
  }
  return p;
}

__device__ __forceinline__ uint64_t dev_rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

__device__ __forceinline__ void apply_jump(uint64_t s[4], const uint64_t* __restrict__ M) {
  uint64_t o[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    uint64_t acc = 0;
#pragma unroll 8
    for (int b = 0; b < 64; ++b) {
      const ulonglong2 r01 = __ldg(reinterpret_cast<const ulonglong2*>(M + (w * 64 + b) * 4));
      const ulonglong2 r23 = __ldg(reinterpret_cast<const ulonglong2*>(M + (w * 64 + b) * 4 + 2));
      const int par = __popcll(r01.x & s[0]) ^ __popcll(r01.y & s[1]) ^ __popcll(r23.x & s[2]) ^
                      __popcll(r23.y & s[3]);
      acc |= (uint64_t)(par & 1) << b;
    }
    o[w] = acc;
  }
#pragma unroll
  for (int w = 0; w < 4; ++w) s[w] = o[w];
}

__global__ void sign_mask_kernel(const SignBuffer* __restrict__ bufs, int nbufs, const uint64_t* __restrict__ jumps,
                                 int njump, long long total_draws, long long mask_words,
                                 const uint64_t* __restrict__ seeds, uint32_t* __restrict__ masks) {
  const long long chunk = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long d_begin = chunk * kChunkDraws;
  if (d_begin >= total_draws) return;
  uint32_t* mask = masks + (long long)blockIdx.y * mask_words;

  uint64_t s[4];
  uint64_t seed = seeds[blockIdx.y];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    seed += 0x9E3779B97F4A7C15ULL;
    uint64_t z = seed;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    s[i] = z ^ (z >> 31);
  }
  for (int k = 0; k < njump; ++k)
    if ((chunk >> k) & 1) apply_jump(s, jumps + (size_t)k * 1024);

  // first buffer whose draw range contains d_begin (largest d0 <= d_begin)
  int lo = 0, hi = nbufs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (bufs[mid].d0 <= d_begin) lo = mid; else hi = mid - 1;
  }
  int b = lo;
  long long cur_word = -1;
  uint32_t acc = 0;
  const long long d_end = min(d_begin + kChunkDraws, total_draws);
  for (long long d = d_begin; d < d_end; ++d) {
    while (b < nbufs - 1 && d >= bufs[b].d0 + bufs[b].n / 4 + bufs[b].n % 4) ++b;
    const uint64_t r = s[0] + s[3];
    {
      const uint64_t t = s[1] << 17;
      s[2] ^= s[0];
      s[3] ^= s[1];
      s[1] ^= s[2];
      s[0] ^= s[3];
      s[2] ^= t;
      s[3] = dev_rotl(s[3], 45);
    }
    const long long local = d - bufs[b].d0;
    const long long full = bufs[b].n / 4;
    long long p;
    int nbits;
    uint32_t bits;
    if (local < full) {
      p = bufs[b].p0 + 4 * local;
      nbits = 4;
      bits = (uint32_t)(r & 15u);
    } else {
      p = bufs[b].p0 + 4 * full + (local - full);
      nbits = 1;
      bits = (uint32_t)(r & 1u);
    }
    for (int k = 0; k < nbits; ++k) {
      const long long q = p + k;
      const long long w = q >> 5;
      if (w != cur_word) {
        if (cur_word >= 0 && acc) atomicOr(mask + cur_word, acc);
        cur_word = w;
        acc = 0;
      }
      acc |= ((bits >> k) & 1u) << (q & 31);
    }
  }
  if (cur_word >= 0 && acc) atomicOr(mask + cur_word, acc);
}

int launch_sign_masks(const SignBuffer* d_bufs, int nbufs, const uint64_t* d_jumps, int njump,
                      long long total_draws, long long mask_words, const uint64_t* d_seeds, int nseeds,
                      uint32_t* d_masks, void* stv) {
  cudaStream_t st = static_cast<cudaStream_t>(stv);
  B2P_REQUIRE(nseeds > 0 && nseeds <= 65535, "seed count %d out of range", nseeds);
  B2P_CHECK_CUDA(cudaMemsetAsync(d_masks, 0, (size_t)nseeds * mask_words * 4, st));
  const long long nchunks = (total_draws + kChunkDraws - 1) / kChunkDraws;
  const int threads = 64;
  dim3 grid((unsigned)((nchunks + threads - 1) / threads), (unsigned)nseeds);
  sign_mask_kernel<<<grid, threads, 0, st>>>(d_bufs, nbufs, d_jumps, njump, total_draws, mask_words, d_seeds,
                                             d_masks);
  B2P_POST_LAUNCH();
  return B2P_OK;
}

}  // namespace b2p
