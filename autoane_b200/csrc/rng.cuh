// rng.cuh — device generation of the MeZO Rademacher sign stream.
//
// The reference draws signs sequentially with xoshiro256+ seeded by splitmix64
// (training/train_mezo.m:97-136): for each buffer in perturbation order, one
// 64-bit draw yields the signs of four consecutive parameters (bits 0..3), and a
// buffer's n%4 tail elements take one draw each (bit 0). perturb_lora_weights
// (train_mezo.m:560-588) walks the LoRA/RMS buffers in a fixed order, so the
// sign of parameter i is a pure function of (seed, i).
//
// The xoshiro256 state transition T is linear over GF(2) with a primitive
// characteristic polynomial P of degree 256, so T^n = p_n(T) with
// p_n(x) = x^n mod P (the jump-polynomial method published with xoshiro,
// Blackman & Vigna, "Scrambled linear pseudorandom number generators"). P is
// recovered once on the host with Berlekamp-Massey from the generator's own
// output and checked against sequential stepping; p_n is precomputed for the
// start draw n = c * kChunkDraws of every chunk c. Thread c then reaches its
// chunk with 256 steps: state = sum_{i : p_i = 1} T^i s0, and draws its chunk
// sequentially. Output: a bit mask per seed, bit i = 1 when parameter i gets
// +scale, written with 32-bit word ORs.
#pragma once
#include <cstdint>
#include <vector>

namespace b2p {

constexpr int kChunkDraws = 64;

// One perturbation buffer: `n` parameters starting at parameter `p0`, whose
// draws start at draw `d0` of the stream.
struct SignBuffer {
  long long p0, d0, n;
};

struct SignPlan {
  std::vector<SignBuffer> bufs;
  long long total_params = 0;
  long long total_draws = 0;
  long long nchunks = 0;
  std::vector<uint64_t> polys;   // [nchunks][4]: coefficients of x^(c*kChunkDraws) mod P
  bool valid = false;            // P recovered and the jump checked against stepping
};

// Build the buffer table for the given buffer sizes (perturbation order) and
// the per-chunk jump polynomials covering its draw count.
SignPlan make_sign_plan(const std::vector<long long>& sizes);

// Jump polynomials x^(c*kChunkDraws) mod P for chunks c < nchunks ([nchunks][4]
// words); false if P could not be recovered or the jump disagrees with stepping.
bool jump_polys(long long nchunks, std::vector<uint64_t>& polys);

// Host xoshiro256+ (for tests of the plan itself).
void host_xo_seed(uint64_t s[4], uint64_t seed);
uint64_t host_xo_next(uint64_t s[4]);

// Launch: masks[slot][words] = sign bits of seeds[slot] for slot < nseeds.
// d_bufs / d_polys are the device copies of plan.bufs / plan.polys. The mask
// rows are zeroed first (inside, on `st`).
int launch_sign_masks(const SignBuffer* d_bufs, int nbufs, const uint64_t* d_polys, long long nchunks,
                      long long total_draws, long long mask_words, const uint64_t* d_seeds, int nseeds,
                      uint32_t* d_masks, void* st);

}  // namespace b2p
