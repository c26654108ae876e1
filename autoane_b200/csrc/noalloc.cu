// noalloc.cu — sign-mask generation that allocates no device memory.
//
// b2p_sign_masks builds its scratch (jump-polynomial table, buffer table,
// seeds) inside a b2p_model, which allocates with cudaMalloc. Some callers
// cannot allocate device memory at all: code that runs where every device byte
// belongs to another allocator (a host framework that hands out fixed pools,
// or a process with a hard memory budget), or code that must not add
// allocations between its own set-up and teardown. For them,
// b2p_sign_masks_noalloc writes the masks into the caller's output buffer and
// keeps its scratch in one fixed, file-scope __device__ array below. Every GPU
// that loads the library holds that array until the process exits.
#include <cstring>
#include <mutex>
#include <vector>
#include "../../include/b2p.h"
#include "engine.cuh"
#include "rng.cuh"

using namespace b2p;

namespace {

constexpr long long kNaMaxChunks = 8192;    // draws <= 8192 * 64 = 524,288 (about 2.1 M parameters)
constexpr int kNaMaxBufs = 1024;            // perturbation buffers per layout
constexpr int kNaMaxSeeds = 64;             // seeds per call
constexpr size_t kNaPolyBytes = (size_t)kNaMaxChunks * 4 * sizeof(uint64_t);  // 256 KiB
constexpr size_t kNaBufBytes = (size_t)kNaMaxBufs * sizeof(SignBuffer);         // 24 KiB
constexpr size_t kNaSeedBytes = (size_t)kNaMaxSeeds * sizeof(uint64_t);         // 512 B
constexpr size_t kNaScratchBytes = kNaPolyBytes + kNaBufBytes + kNaSeedBytes;

// Scratch shared by every call on a device: [jump polynomials | buffer table | seeds].
// In host code this name is only a host-side stand-in; kernels get the device
// address from cudaGetSymbolAddress (na_setup).
static __device__ __align__(256) unsigned char g_na_scratch[kNaScratchBytes];

std::mutex g_na_mu;
unsigned char* g_na_dev[64] = {};  // device address of g_na_scratch, per device ordinal

// Once per device, with that device current: look up the array's device address
// and fill the (seed- and layout-independent) jump-polynomial table.
int na_setup(unsigned char** out) {
  int dev = 0;
  B2P_CHECK_CUDA(cudaGetDevice(&dev));
  B2P_REQUIRE(dev >= 0 && dev < 64, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_na_mu);
  if (!g_na_dev[dev]) {
    void* p = nullptr;
    B2P_CHECK_CUDA(cudaGetSymbolAddress(&p, g_na_scratch));
    static std::vector<uint64_t> polys;  // host copy, shared by all devices
    if (polys.empty() && !jump_polys(kNaMaxChunks, polys)) {
      polys.clear();
      set_error("xoshiro jump polynomial could not be established");
      return B2P_ERR_STATE;
    }
    // A copy from pageable memory may return before it reaches the device, and a
    // kernel on a non-blocking stream is not ordered after the legacy stream: wait
    // for the copy itself before any call can launch on this device.
    B2P_CHECK_CUDA(cudaMemcpyAsync(p, polys.data(), kNaPolyBytes, cudaMemcpyHostToDevice, cudaStreamLegacy));
    B2P_CHECK_CUDA(cudaStreamSynchronize(cudaStreamLegacy));
    g_na_dev[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_na_dev[dev];
  return B2P_OK;
}

}  // namespace

extern "C" int b2p_sign_masks_noalloc(const int64_t* buffer_sizes, int nbufs, const uint64_t* seeds, int nseeds,
                                      uint32_t* out_words, void* stream) {
  B2P_REQUIRE(buffer_sizes && seeds && out_words, "null argument");
  B2P_REQUIRE(nbufs >= 1 && nbufs <= kNaMaxBufs, "buffer count %d outside [1, %d]", nbufs, kNaMaxBufs);
  B2P_REQUIRE(nseeds >= 1 && nseeds <= kNaMaxSeeds, "seed count %d outside [1, %d]", nseeds, kNaMaxSeeds);
  std::vector<SignBuffer> bufs((size_t)nbufs);
  long long params = 0, draws = 0;
  for (int b = 0; b < nbufs; ++b) {
    B2P_REQUIRE(buffer_sizes[b] >= 0, "buffer %d has a negative size", b);
    bufs[b] = SignBuffer{params, draws, buffer_sizes[b]};
    params += buffer_sizes[b];
    draws += buffer_sizes[b] / 4 + buffer_sizes[b] % 4;
  }
  B2P_REQUIRE(params >= 1, "empty layout");
  const long long nchunks = (draws + kChunkDraws - 1) / kChunkDraws;
  B2P_REQUIRE(nchunks <= kNaMaxChunks,
              "layout needs %lld draws; b2p_sign_masks_noalloc supports at most %lld (use b2p_sign_masks)", draws,
              kNaMaxChunks * kChunkDraws);
  cudaPointerAttributes attr;
  B2P_CHECK_CUDA(cudaPointerGetAttributes(&attr, out_words));
  B2P_REQUIRE(attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged,
              "out_words must be device memory");
  int cur = 0;
  B2P_CHECK_CUDA(cudaGetDevice(&cur));
  // the scratch and the launch belong to the current device; another GPU's buffer
  // would be written over peer access or fault, so it is refused before any work
  B2P_REQUIRE(attr.type == cudaMemoryTypeManaged || attr.device == cur,
              "out_words lives on device %d but device %d is current", attr.device, cur);
  unsigned char* scratch = nullptr;
  int rc = na_setup(&scratch);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SignBuffer* d_bufs = reinterpret_cast<SignBuffer*>(scratch + kNaPolyBytes);
  uint64_t* d_seeds = reinterpret_cast<uint64_t*>(scratch + kNaPolyBytes + kNaBufBytes);
  const uint64_t* d_polys = reinterpret_cast<const uint64_t*>(scratch);
  B2P_CHECK_CUDA(cudaMemcpyAsync(d_bufs, bufs.data(), bufs.size() * sizeof(SignBuffer), cudaMemcpyHostToDevice, st));
  B2P_CHECK_CUDA(cudaMemcpyAsync(d_seeds, seeds, (size_t)nseeds * sizeof(uint64_t), cudaMemcpyHostToDevice, st));
  // launch_sign_masks zeroes the output rows itself before setting bits
  return launch_sign_masks(d_bufs, nbufs, d_polys, nchunks > 0 ? nchunks : 1, draws, (params + 31) / 32, d_seeds,
                           nseeds, out_words, st);
}
