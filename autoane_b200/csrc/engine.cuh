// engine.cuh — host-side plumbing shared by every translation unit of the
// library: error reporting, the per-device context (stream, status word,
// SM count), TMA tensor-map encoding and the GEMM launch dispatcher.
#pragma once
#include <cstdint>
#include <cstdio>
#include <string>
#include <cuda.h>
#include <cuda_runtime.h>
#include "gemm.cuh"
#include "../../include/b2p.h"

namespace b2p {

// Status codes (B2P_OK, B2P_ERR_*) are the macros of include/b2p.h.

void set_error(const char* fmt, ...);
const char* last_error();

#define B2P_CHECK_CUDA(expr)                                                            \
  do {                                                                                  \
    cudaError_t e_ = (expr);                                                            \
    if (e_ != cudaSuccess) {                                                            \
      ::b2p::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, \
                       __LINE__);                                                       \
      return B2P_ERR_CUDA;                                                       \
    }                                                                                   \
  } while (0)

#define B2P_REQUIRE(cond, ...)       \
  do {                               \
    if (!(cond)) {                   \
      ::b2p::set_error(__VA_ARGS__); \
      return B2P_ERR_ARG;     \
    }                                \
  } while (0)

// Count of kernels this library has launched (all devices, all threads).
void count_launch();
// Adjust the count by n (kernels recorded into a CUDA graph run once per replay).
void count_launches(long long n);
long long launch_count();

#define B2P_POST_LAUNCH()                         \
  do {                                            \
    ::b2p::count_launch();                        \
    B2P_CHECK_CUDA(cudaGetLastError());           \
  } while (0)

// Programmatic dependent launch on or off for the whole process (B2P_OPT_PDL).
bool pdl_enabled();
void set_pdl(bool on);

// Launch with programmatic stream serialization: the kernel may start (prologue: barrier
// init, TMEM allocation, descriptor prefetch) while the previous kernel in the stream is
// still finishing. Every kernel launched this way calls pdl_enter() before touching global
// memory: that waits until the preceding grid has completed and its writes are visible.
// With PDL off the attribute is left out and pdl_enter() returns at once.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

struct DeviceCtx {
  int device = -1;
  int num_sms = 0;
  uint32_t* status = nullptr;  // device word written by bounded waits
};

// Initialise (once per device) and return the context of the current device.
int ctx_get(DeviceCtx** out);

// Read and clear the device status word; returns B2P_ERR_DEVICE if non-zero.
int check_device_status(cudaStream_t st);

// Element type of a tensor map.
enum TmapType : int { TM_F16 = 0, TM_BF16 = 1, TM_F32 = 2 };

// 2-D tensor map over a row-major [rows, inner] matrix (row pitch ld elements),
// box = box_inner x box_rows elements, given swizzle (0 none, 32, 64, 128 bytes),
// zero fill out of bounds.
int make_tmap_2d(CUtensorMap* map, const void* base, TmapType type, uint64_t inner, uint64_t rows, uint64_t ld,
                 uint32_t box_inner, uint32_t box_rows, int swizzle_bytes);

// Launch D = X·W^T (+ U·Bv^T with LoRA) with the given epilogue. `bn` is the
// compiled tile width (128, 160, 192 or 256). `out`/`ldo` is the destination of
// the stored kinds (fp32 for EPI_F32/EPI_RESID, 16-bit otherwise); `u16` is the
// [M, 64] 16-bit LoRA-down buffer when ep.has_lora.
int launch_gemm(int bn, int kind, bool bf16, const void* X, int ldx, const void* W, int ldw, int M, int N, int K,
                void* out, int ldo, const void* u16, const EpiParams& ep, cudaStream_t st);

// The CTA-pair engine (gemm2.cuh): 256-row x 256-column tiles over clusters of
// two CTAs. pair_supported() tells whether a launch qualifies (M >= 256, LoRA
// variant groups of whole 256-row tiles, LoRA only on the fused QKV / residual
// epilogues); launch_gemm_pair() has the same contract as launch_gemm.
bool pair_supported(int kind, int M, int N, const EpiParams& ep);
// MN-major operands on the CTA-pair engine (plain tiles, no LoRA): opm bit 0 = X given as [K][M]
// rows of pitch ldx, bit 1 = W given as [K][N] rows of pitch ldw. Epilogues: EPI_F32 (opm 2, 3),
// EPI_H16 (opm 2), EPI_RESID (opm 3). pair_mn_supported() tells whether a launch qualifies.
bool pair_mn_supported(int kind, int opm, int M, int N, int K, const void* X, int ldx, const void* W, int ldw);
int launch_gemm_pair_mn(int kind, int opm, bool bf16, const void* X, int ldx, const void* W, int ldw, int M, int N,
                        int K, void* out, int ldo, const EpiParams& ep, cudaStream_t st);
// Plain fp32 / 16-bit output GEMM on 128 x 64 tiles, one CTA per tile, its K-blocks spread over
// four MMA issuer warps with one TMEM accumulator each (summed in issuer order in the epilogue).
int launch_gemm_mi(int kind, bool bf16, const void* X, int ldx, const void* W, int ldw, int M, int N, int K,
                   void* out, int ldo, cudaStream_t st);
// Route of a plain fp32 / 16-bit GEMM of at most 1024 rows whose 128 x 64 tiles fit one wave:
// SMALL_GEMM_NONE (the persistent engines), SMALL_GEMM_SPLITK or SMALL_GEMM_MULTI_ISSUER.
enum SmallGemmRoute { SMALL_GEMM_NONE = 0, SMALL_GEMM_SPLITK = 1, SMALL_GEMM_MULTI_ISSUER = 2 };
int small_gemm_route(int kind, int M, int N, int K, int num_sms);
int launch_gemm_small(int route, int kind, bool bf16, const void* X, int ldx, const void* W, int ldw, int M, int N,
                      int K, void* out, int ldo, cudaStream_t st);
int launch_gemm_pair(int kind, bool bf16, const void* X, int ldx, const void* W, int ldw, int M, int N, int K,
                     void* out, int ldo, const void* u16, const EpiParams& ep, cudaStream_t st);

// Plain fp32 / 16-bit output GEMMs of at most 1024 rows whose 128 x 64 tiles fit one wave
// (gemm_sk.cu): each tile's K loop is split over a cluster of up to 4 CTAs (four MMA issuers
// each), the partial tiles moved by bulk copies into CTA 0 and added in rank order.
// splitk_applies() tells whether a launch qualifies.
bool splitk_applies(int kind, int M, int N, int num_sms);
int launch_gemm_splitk(int kind, bool bf16, const void* X, int ldx, const void* W, int ldw, int M, int N, int K,
                       void* out, int ldo, cudaStream_t st);

// Pick the tile width for an N-column output (largest width whose padding
// waste is minimal; SwiGLU and CE need multiples of 64 / any).
int pick_bn(int N, int kind);
// Tile width for a plain fp32 / 16-bit output GEMM of M rows on `ctas` CTAs: pick_bn's width
// when its tiles fill every CTA once, else 128 or 64 columns so that more CTAs share the weight
// stream (small M: the T <= 1024 token counts of single calls).
int pick_bn_rows(int M, int N, int kind, int ctas);

}  // namespace b2p
