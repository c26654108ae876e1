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
// Polynomials over GF(2) of degree < 256: bit i of word i/64 = coefficient of x^i.
struct Poly {
  uint64_t w[4] = {0, 0, 0, 0};
  bool bit(int i) const { return (w[i >> 6] >> (i & 63)) & 1u; }
};

// Berlekamp-Massey over GF(2): connection polynomial c (c[0] = 1) of the
// shortest LFSR generating s, i.e. s[i] = sum_{j=1..L} c[j] s[i-j].
std::vector<uint8_t> berlekamp_massey(const std::vector<uint8_t>& s) {
  const int n = (int)s.size();
  std::vector<uint8_t> C(n + 1, 0), B(n + 1, 0), T;
  C[0] = B[0] = 1;
  int L = 0, m = 1;
  for (int i = 0; i < n; ++i) {
    uint8_t d = s[i];
    for (int j = 1; j <= L; ++j) d ^= (uint8_t)(C[j] & s[i - j]);
    if (!d) {
      ++m;
    } else if (2 * L <= i) {
      T = C;
      for (int j = 0; j + m <= n; ++j) C[j + m] ^= B[j];
      L = i + 1 - L;
      B = T;
      m = 1;
    } else {
      for (int j = 0; j + m <= n; ++j) C[j + m] ^= B[j];
      ++m;
    }
  }
  C.resize(L + 1);
  return C;
}

// a·x mod P, where P = x^256 + low
inline void mulx(Poly& a, const Poly& low) {
  const bool carry = a.bit(255);
  for (int k = 3; k > 0; --k) a.w[k] = (a.w[k] << 1) | (a.w[k - 1] >> 63);
  a.w[0] <<= 1;
  if (carry)
    for (int k = 0; k < 4; ++k) a.w[k] ^= low.w[k];
}

// a·b mod P (Horner over the bits of b)
Poly mulmod(const Poly& a, const Poly& b, const Poly& low) {
  Poly r;
  for (int i = 255; i >= 0; --i) {
    mulx(r, low);
    if (b.bit(i))
      for (int k = 0; k < 4; ++k) r.w[k] ^= a.w[k];
  }
  return r;
}

// T^n s0 = p_n(T) s0
void host_jump(const Poly& p, uint64_t s[4]) {
  uint64_t acc[4] = {0, 0, 0, 0};
  for (int i = 0; i < 256; ++i) {
    if (p.bit(i))
      for (int k = 0; k < 4; ++k) acc[k] ^= s[k];
    host_xo_next(s);
  }
  for (int k = 0; k < 4; ++k) s[k] = acc[k];
}
}  // namespace

bool jump_polys(long long nchunks, std::vector<uint64_t>& polys) {
  // characteristic polynomial from 512 output bits of a nonzero state
  uint64_t s[4];
  host_xo_seed(s, 0x5DEECE66DULL);
  std::vector<uint8_t> bits(512);
  for (int i = 0; i < 512; ++i) {
    bits[i] = (uint8_t)(s[0] & 1u);
    host_xo_next(s);
  }
  const std::vector<uint8_t> C = berlekamp_massey(bits);
  const int L = (int)C.size() - 1;
  if (L != 256) return false;
  // P(x) = x^256 + sum_{j=1..256} c_j x^(256-j): low part holds the c_j
  Poly low;
  for (int j = 1; j <= 256; ++j)
    if (C[j]) low.w[(256 - j) >> 6] |= 1ull << ((256 - j) & 63);

  Poly xc;  // x^kChunkDraws mod P
  xc.w[0] = 1;
  for (int i = 0; i < kChunkDraws; ++i) mulx(xc, low);
  polys.assign((size_t)nchunks * 4, 0);
  Poly cur;
  cur.w[0] = 1;  // x^0
  for (long long c = 0; c < nchunks; ++c) {
    for (int k = 0; k < 4; ++k) polys[(size_t)c * 4 + k] = cur.w[k];
    cur = mulmod(cur, xc, low);
  }
  // check the jump against sequential stepping at a few chunk starts
  const long long checks[4] = {1, 3, nchunks / 2, nchunks - 1};
  for (long long c : checks) {
    if (c <= 0 || c >= nchunks) continue;
    uint64_t a[4], b[4];
    host_xo_seed(a, 42 + (uint64_t)c);
    for (int k = 0; k < 4; ++k) b[k] = a[k];
    Poly pc;
    for (int k = 0; k < 4; ++k) pc.w[k] = polys[(size_t)c * 4 + k];
    host_jump(pc, a);
    for (long long i = 0; i < c * kChunkDraws; ++i) host_xo_next(b);
    for (int k = 0; k < 4; ++k)
      if (a[k] != b[k]) return false;
  }
  return true;
}

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
  p.nchunks = (dd + kChunkDraws - 1) / kChunkDraws;
  if (p.nchunks == 0) p.nchunks = 1;

  p.valid = jump_polys(p.nchunks, p.polys);
  return p;
}

__device__ __forceinline__ uint64_t dev_rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

__device__ __forceinline__ void dev_step(uint64_t s[4]) {
  const uint64_t t = s[1] << 17;
  s[2] ^= s[0];
  s[3] ^= s[1];
  s[1] ^= s[2];
  s[0] ^= s[3];
  s[2] ^= t;
  s[3] = dev_rotl(s[3], 45);
}

__global__ void sign_mask_kernel(const SignBuffer* __restrict__ bufs, int nbufs, const uint64_t* __restrict__ polys,
                                 long long nchunks, long long total_draws, long long mask_words,
                                 const uint64_t* __restrict__ seeds, uint32_t* __restrict__ masks) {
  const long long chunk = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (chunk >= nchunks) return;
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
  if (chunk > 0) {  // s <- T^(chunk * kChunkDraws) s = sum_i p_i T^i s
    uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll 1
    for (int w = 0; w < 4; ++w) {
      uint64_t pw = __ldg(polys + chunk * 4 + w);
#pragma unroll 4
      for (int b = 0; b < 64; ++b) {
        const uint64_t sel = 0ull - (pw & 1ull);
        acc[0] ^= s[0] & sel;
        acc[1] ^= s[1] & sel;
        acc[2] ^= s[2] & sel;
        acc[3] ^= s[3] & sel;
        pw >>= 1;
        dev_step(s);
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) s[k] = acc[k];
  }

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
    dev_step(s);
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

int launch_sign_masks(const SignBuffer* d_bufs, int nbufs, const uint64_t* d_polys, long long nchunks,
                      long long total_draws, long long mask_words, const uint64_t* d_seeds, int nseeds,
                      uint32_t* d_masks, void* stv) {
  cudaStream_t st = static_cast<cudaStream_t>(stv);
  B2P_REQUIRE(nseeds > 0 && nseeds <= 65535, "seed count %d out of range", nseeds);
  B2P_CHECK_CUDA(cudaMemsetAsync(d_masks, 0, (size_t)nseeds * mask_words * 4, st));
  const int threads = 128;
  dim3 grid((unsigned)((nchunks + threads - 1) / threads), (unsigned)nseeds);
  sign_mask_kernel<<<grid, threads, 0, st>>>(d_bufs, nbufs, d_polys, nchunks, total_draws, mask_words, d_seeds,
                                             d_masks);
  B2P_POST_LAUNCH();
  return B2P_OK;
}

}  // namespace b2p
