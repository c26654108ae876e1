// b2p_api.cu — C-ABI entry points: initialisation, errors and the raw GEMM.
#include <cstring>
#include "engine.cuh"
#include "../../include/b2p.h"

using namespace b2p;

extern "C" {

int b2p_init(int device) {
  int n = 0;
  B2P_CHECK_CUDA(cudaGetDeviceCount(&n));
  B2P_REQUIRE(device >= 0 && device < n, "device %d out of range (%d visible)", device, n);
  B2P_CHECK_CUDA(cudaSetDevice(device));
  DeviceCtx* c = nullptr;
  return ctx_get(&c);
}

const char* b2p_last_error(void) { return last_error(); }

const char* b2p_version(void) { return "b2p 0.1 (sm_100a tcgen05 projection engine)"; }

int b2p_device_status(void* stream) { return check_device_status(static_cast<cudaStream_t>(stream)); }

int b2p_gemm(const void* X, const void* W, void* Y, int M, int N, int K, int ldy, int dtype, int out_f32,
             void* stream) {
  B2P_REQUIRE(X && W && Y, "null operand");
  B2P_REQUIRE(dtype == B2P_F16 || dtype == B2P_BF16, "dtype must be B2P_F16 or B2P_BF16");
  B2P_REQUIRE(ldy >= N, "ldy (%d) < N (%d)", ldy, N);
  B2P_REQUIRE(out_f32 ? (ldy % 4 == 0) : (ldy % 8 == 0), "ldy must keep 16-byte row alignment");
  B2P_REQUIRE((reinterpret_cast<uintptr_t>(Y) & 15u) == 0, "Y must be 16-byte aligned");
  EpiParams ep;
  std::memset(&ep, 0, sizeof(ep));
  ep.M = M;
  ep.N = N;
  const int kind = out_f32 ? EPI_F32 : EPI_H16;
  DeviceCtx* c = nullptr;
  int rc = ctx_get(&c);
  if (rc) return rc;
  if (const int route = small_gemm_route(kind, M, N, K, c->num_sms))
    return launch_gemm_small(route, kind, dtype == B2P_BF16, X, K, W, K, M, N, K, Y, ldy,
                             static_cast<cudaStream_t>(stream));
  if (M >= 2 * kBM && pair_supported(kind, M, N, ep))
    return launch_gemm_pair(kind, dtype == B2P_BF16, X, K, W, K, M, N, K, Y, ldy, nullptr, ep,
                            static_cast<cudaStream_t>(stream));
  return launch_gemm(pick_bn_rows(M, N, kind, c->num_sms), kind, dtype == B2P_BF16, X, K, W, K, M, N, K, Y, ldy,
                     nullptr, ep, static_cast<cudaStream_t>(stream));
}

int b2p_gemm_pair(const void* X, const void* W, void* Y, int M, int N, int K, int ldy, int dtype, int out_f32,
                  void* stream) {
  B2P_REQUIRE(X && W && Y, "null operand");
  B2P_REQUIRE(dtype == B2P_F16 || dtype == B2P_BF16, "dtype must be B2P_F16 or B2P_BF16");
  B2P_REQUIRE(M >= 2 * kBM, "the CTA-pair engine needs M >= %d (got %d)", 2 * kBM, M);
  B2P_REQUIRE(ldy >= N, "ldy (%d) < N (%d)", ldy, N);
  B2P_REQUIRE(out_f32 ? (ldy % 4 == 0) : (ldy % 8 == 0), "ldy must keep 16-byte row alignment");
  B2P_REQUIRE((reinterpret_cast<uintptr_t>(Y) & 15u) == 0, "Y must be 16-byte aligned");
  EpiParams ep;
  std::memset(&ep, 0, sizeof(ep));
  ep.M = M;
  ep.N = N;
  return launch_gemm_pair(out_f32 ? EPI_F32 : EPI_H16, dtype == B2P_BF16, X, K, W, K, M, N, K, Y, ldy, nullptr, ep,
                          static_cast<cudaStream_t>(stream));
}

int b2p_gemm_pair_mn(const void* X, int ldx, int x_mn, const void* W, int ldw, int w_mn, void* Y, int M, int N, int K,
                     int ldy, int dtype, int out_f32, void* stream) {
  B2P_REQUIRE(X && W && Y, "null operand");
  B2P_REQUIRE(dtype == B2P_F16 || dtype == B2P_BF16, "dtype must be B2P_F16 or B2P_BF16");
  B2P_REQUIRE(M >= 2 * kBM, "the CTA-pair engine needs M >= %d (got %d)", 2 * kBM, M);
  B2P_REQUIRE((x_mn == 0 || x_mn == 1) && (w_mn == 0 || w_mn == 1), "x_mn / w_mn must be 0 or 1");
  B2P_REQUIRE(ldy >= N, "ldy (%d) < N (%d)", ldy, N);
  B2P_REQUIRE(out_f32 ? (ldy % 4 == 0) : (ldy % 8 == 0), "ldy must keep 16-byte row alignment");
  B2P_REQUIRE((reinterpret_cast<uintptr_t>(Y) & 15u) == 0, "Y must be 16-byte aligned");
  EpiParams ep;
  std::memset(&ep, 0, sizeof(ep));
  ep.M = M;
  ep.N = N;
  const int kind = out_f32 ? EPI_F32 : EPI_H16;
  if (!x_mn && !w_mn) {
    B2P_REQUIRE(ldx >= K && ldw >= K && ldx % 8 == 0 && ldw % 8 == 0, "row pitches must be >= K, multiples of 8");
    return launch_gemm_pair(kind, dtype == B2P_BF16, X, ldx, W, ldw, M, N, K, Y, ldy, nullptr, ep,
                            static_cast<cudaStream_t>(stream));
  }
  return launch_gemm_pair_mn(kind, (x_mn ? 1 : 0) | (w_mn ? 2 : 0), dtype == B2P_BF16, X, ldx, W, ldw, M, N, K, Y, ldy,
                             ep, static_cast<cudaStream_t>(stream));
}

int b2p_gemm_mi(const void* X, const void* W, void* Y, int M, int N, int K, int ldy, int dtype, int out_f32,
                void* stream) {
  B2P_REQUIRE(X && W && Y, "null operand");
  B2P_REQUIRE(dtype == B2P_F16 || dtype == B2P_BF16, "dtype must be B2P_F16 or B2P_BF16");
  B2P_REQUIRE(K % 8 == 0, "K must be a multiple of 8 (16-byte rows)");
  B2P_REQUIRE(ldy >= N, "ldy (%d) < N (%d)", ldy, N);
  B2P_REQUIRE((reinterpret_cast<uintptr_t>(Y) & 15u) == 0, "Y must be 16-byte aligned");
  return launch_gemm_mi(out_f32 ? EPI_F32 : EPI_H16, dtype == B2P_BF16, X, K, W, K, M, N, K, Y, ldy,
                        static_cast<cudaStream_t>(stream));
}

}  // extern "C"
