// engine.cu — error state, device context, tensor maps and the GEMM dispatcher.
#include <cstdarg>
#include <cstring>
#include <atomic>
#include <mutex>
#include <cudaTypedefs.h>
#include "engine.cuh"

namespace b2p {

namespace {
thread_local std::string g_last_error;
std::mutex g_ctx_mu;
DeviceCtx g_ctx[64];
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::atomic<long long> g_launches{0};
std::atomic<int> g_pdl{1};
}  // namespace

bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }
void set_pdl(bool on) { g_pdl.store(on ? 1 : 0, std::memory_order_relaxed); }

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
void count_launches(long long n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}
const char* last_error() { return g_last_error.c_str(); }

int ctx_get(DeviceCtx** out) {
  int dev = 0;
  B2P_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) {
    set_error("device ordinal %d out of range", dev);
    return B2P_ERR_ARG;
  }
  std::lock_guard<std::mutex> lk(g_ctx_mu);
  DeviceCtx& c = g_ctx[dev];
  if (c.device < 0) {
    int major = 0, minor = 0;
    B2P_CHECK_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    B2P_CHECK_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
    if (major != 10 || minor != 0) {
      set_error("device %d is sm_%d%d; this library is built for sm_100a (B200) only", dev, major, minor);
      return B2P_ERR_UNSUPPORTED;
    }
    B2P_CHECK_CUDA(cudaDeviceGetAttribute(&c.num_sms, cudaDevAttrMultiProcessorCount, dev));
    B2P_CHECK_CUDA(cudaMalloc(&c.status, sizeof(uint32_t)));
    B2P_CHECK_CUDA(cudaMemset(c.status, 0, sizeof(uint32_t)));
    if (!g_encode) {
      cudaDriverEntryPointQueryResult q;
      void* fn = nullptr;
      B2P_CHECK_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
      if (q != cudaDriverEntryPointSuccess || !fn) {
        set_error("cuTensorMapEncodeTiled not available from the driver");
        return B2P_ERR_CUDA;
      }
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    c.device = dev;
  }
  *out = &c;
  return B2P_OK;
}

int check_device_status(cudaStream_t st) {
  DeviceCtx* c = nullptr;
  int rc = ctx_get(&c);
  if (rc) return rc;
  uint32_t h = 0;
  B2P_CHECK_CUDA(cudaMemcpyAsync(&h, c->status, sizeof(h), cudaMemcpyDeviceToHost, st));
  B2P_CHECK_CUDA(cudaStreamSynchronize(st));
  if (h != 0) {
    B2P_CHECK_CUDA(cudaMemsetAsync(c->status, 0, sizeof(uint32_t), st));
    set_error("device status %u (1-4: a bounded wait inside a kernel expired: producer, mma, epilogue, drain; "
              "5: an index out of range; 6: a non-finite gradient, the optimizer step was skipped)", h);
    return B2P_ERR_DEVICE;
  }
  return B2P_OK;
}

int make_tmap_2d(CUtensorMap* map, const void* base, TmapType type, uint64_t inner, uint64_t rows, uint64_t ld,
                 uint32_t box_inner, uint32_t box_rows, int swizzle_bytes) {
  const uint64_t esz = type == TM_F32 ? 4 : 2;
  B2P_REQUIRE(base != nullptr, "tensor map over a null pointer");
  B2P_REQUIRE((reinterpret_cast<uintptr_t>(base) & 15u) == 0, "tensor base must be 16-byte aligned");
  B2P_REQUIRE(inner >= 1 && (ld * esz) % 16 == 0 && ld >= inner,
              "inner=%llu / ld=%llu: row pitch must be a multiple of 16 bytes", (unsigned long long)inner,
              (unsigned long long)ld);
  B2P_REQUIRE(rows >= 1 && box_rows >= 1 && box_rows <= 256 && box_inner >= 1 && box_inner <= 256, "bad box");
  CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE;
  if (swizzle_bytes == 32) sw = CU_TENSOR_MAP_SWIZZLE_32B;
  if (swizzle_bytes == 64) sw = CU_TENSOR_MAP_SWIZZLE_64B;
  if (swizzle_bytes == 128) sw = CU_TENSOR_MAP_SWIZZLE_128B;
  B2P_REQUIRE(swizzle_bytes == 0 || box_inner * esz == (uint64_t)swizzle_bytes,
              "box inner extent must equal the swizzle span");
  const CUtensorMapDataType dt = type == TM_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : type == TM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t gdim[2] = {inner, rows};
  cuuint64_t gstride[1] = {ld * esz};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = g_encode(map, dt, 2, const_cast<void*>(base), gdim, gstride, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return B2P_ERR_CUDA;
  }
  return B2P_OK;
}

int pick_bn_rows(int M, int N, int kind, int ctas) {
  const int bn = pick_bn(N, kind);
  if (kind != EPI_F32 && kind != EPI_H16) return bn;
  const long long mt = (M + kBM - 1) / kBM;
  if (mt * ((N + bn - 1) / bn) >= ctas) return bn;
  return mt * ((N + 127) / 128) >= ctas ? 128 : 64;
}

int pick_bn(int N, int kind) {
  if (kind == EPI_SWIGLU) return 256;
  if (kind == EPI_CE) return 256;
  const int cands[4] = {256, 192, 160, 128};
  int best = 256;
  long long best_pad = -1;
  for (int i = 0; i < 4; ++i) {
    const int bn = cands[i];
    const long long pad = (long long)((N + bn - 1) / bn) * bn - N;
    if (best_pad < 0 || pad < best_pad) {
      best_pad = pad;
      best = bn;
    }
  }
  return best;
}

template <int BN, int KIND, typename OutT, bool BF16, bool LORA>
static int launch_t(const void* X, int ldx, const void* W, int ldw, int M, int N, int K, void* out, int ldo,
                    const void* u16, const EpiParams& ep, cudaStream_t st) {
  DeviceCtx* c = nullptr;
  int rc = ctx_get(&c);
  if (rc) return rc;
  const TmapType in_t = BF16 ? TM_BF16 : TM_F16;
  CUtensorMap tx, tw, to, tu;
  if ((rc = make_tmap_2d(&tx, X, in_t, (uint64_t)K, (uint64_t)M, (uint64_t)ldx, 64, kBM, 128))) return rc;
  if ((rc = make_tmap_2d(&tw, W, in_t, (uint64_t)K, (uint64_t)N, (uint64_t)ldw, 64, BN, 128))) return rc;
  using S = GemmSmem<BN, KIND>;
  if (S::kStores) {
    const int ncols = KIND == EPI_SWIGLU ? N / 2 : N;
    if (S::kOutF32) {
      if ((rc = make_tmap_2d(&to, out, TM_F32, (uint64_t)ncols, (uint64_t)M, (uint64_t)ldo, 32, 32, 128))) return rc;
    } else {
      if ((rc = make_tmap_2d(&to, out, in_t, (uint64_t)ncols, (uint64_t)M, (uint64_t)ldo, 32, 32, 64))) return rc;
    }
  } else {
    to = tx;
  }
  if (LORA) {
    if ((rc = make_tmap_2d(&tu, u16, in_t, (uint64_t)kUCols, (uint64_t)M, (uint64_t)kUCols, 16, kBM, 32))) return rc;
  } else {
    tu = tx;
  }
  auto kern = gemm_tc_kernel<BN, KIND, OutT, BF16, LORA>;
  static thread_local uint64_t attr_dev_mask = 0;
  if (!(attr_dev_mask & (1ull << (c->device & 63)))) {
    B2P_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal));
    attr_dev_mask |= 1ull << (c->device & 63);
  }
  const long long tiles = (long long)((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
  const int grid = (int)(tiles < c->num_sms ? tiles : c->num_sms);
  EpiParams e = ep;
  e.status = c->status;
  B2P_CHECK_CUDA(launch_pdl(kern, dim3(grid), dim3(kGemmThreads), S::kTotal, st, tx, tw, to, tu, M, N, K, e));
  B2P_POST_LAUNCH();
  return B2P_OK;
}

template <int KIND, typename OutH, bool BF16, bool LORA>
static int dispatch_bn(int bn, const void* X, int ldx, const void* W, int ldw, int M, int N, int K, void* out,
                       int ldo, const void* u16, const EpiParams& ep, cudaStream_t st) {
  switch (bn) {
    case 64: return launch_t<64, KIND, OutH, BF16, LORA>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
    case 128: return launch_t<128, KIND, OutH, BF16, LORA>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
    case 160: return launch_t<160, KIND, OutH, BF16, LORA>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
    case 192: return launch_t<192, KIND, OutH, BF16, LORA>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
    case 256: return launch_t<256, KIND, OutH, BF16, LORA>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
    default: set_error("unsupported tile width %d", bn); return B2P_ERR_UNSUPPORTED;
  }
}

template <typename H, bool BF16>
static int dispatch_kind(int bn, int kind, const void* X, int ldx, const void* W, int ldw, int M, int N, int K,
                         void* out, int ldo, const void* u16, const EpiParams& ep, cudaStream_t st) {
  const bool lora = ep.has_lora != 0;
  switch (kind) {
    case EPI_F32:
      if (lora) return dispatch_bn<EPI_F32, H, BF16, true>(bn, X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
      return dispatch_bn<EPI_F32, H, BF16, false>(bn, X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
    case EPI_H16:
      if (lora) return dispatch_bn<EPI_H16, H, BF16, true>(bn, X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
      return dispatch_bn<EPI_H16, H, BF16, false>(bn, X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
    case EPI_QKV_ROPE:
      if (!lora) break;
      return bn == 128 ? launch_t<128, EPI_QKV_ROPE, H, BF16, true>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st)
                       : launch_t<160, EPI_QKV_ROPE, H, BF16, true>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
    case EPI_RESID:
      if (lora) return dispatch_bn<EPI_RESID, H, BF16, true>(bn, X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
      return dispatch_bn<EPI_RESID, H, BF16, false>(bn, X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
    case EPI_SWIGLU:
      return launch_t<256, EPI_SWIGLU, H, BF16, false>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
    case EPI_CE:
      return launch_t<256, EPI_CE, H, BF16, false>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
    case EPI_CE_GRAD:
      return launch_t<256, EPI_CE_GRAD, H, BF16, false>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
  }
  set_error("unsupported epilogue kind %d (LoRA %d)", kind, (int)lora);
  return B2P_ERR_UNSUPPORTED;
}

int launch_gemm(int bn, int kind, bool bf16, const void* X, int ldx, const void* W, int ldw, int M, int N, int K,
                void* out, int ldo, const void* u16, const EpiParams& ep, cudaStream_t st) {
  B2P_REQUIRE(M > 0 && N > 0 && K > 0, "empty GEMM (M=%d N=%d K=%d)", M, N, K);
  if (ep.has_lora) {
    B2P_REQUIRE(u16 != nullptr, "LoRA GEMM without a U buffer");
    B2P_REQUIRE(ep.lora.rank == 4 || ep.lora.rank == 8, "LoRA rank must be 4 or 8 (got %d)", ep.lora.rank);
    B2P_REQUIRE(ep.lora.n_groups >= (M + ep.lora.group_rows - 1) / ep.lora.group_rows &&
                    ep.lora.n_groups <= kMaxGroups && ep.lora.n_variants >= 1 && ep.lora.n_variants <= kMaxGroups,
                "LoRA group/variant tables out of range");
    B2P_REQUIRE(ep.lora.group_rows % kBM == 0, "LoRA variant groups must span whole 128-row tiles");
    for (int s = 0; s < ep.lora.nseg; ++s) {
      B2P_REQUIRE(ep.lora.seg_boff[s] % ep.lora.rank == 0, "LoRA B offset must be a multiple of the rank");
      B2P_REQUIRE(ep.lora.seg_ucol[s] % 16 == 0 && ep.lora.seg_ucol[s] + 16 <= kUCols, "bad U column");
    }
    for (int s = 1; s < ep.lora.nseg; ++s)
      B2P_REQUIRE(ep.lora.seg_start[s] % bn == 0, "segment boundary %d not a multiple of tile width %d",
                  ep.lora.seg_start[s], bn);
  }
  if (kind != EPI_CE) B2P_REQUIRE(out != nullptr, "GEMM without an output");
  if (kind == EPI_QKV_ROPE)
    B2P_REQUIRE(ep.head_dim == 64 && ep.seq_len % kBM == 0 && ep.rope_cols % 64 == 0,
                "RoPE epilogue needs head_dim 64, seq %% 128 == 0 and whole heads");
  if (kind == EPI_SWIGLU) B2P_REQUIRE(N % 256 == 0, "SwiGLU needs N %% 256 == 0");
  B2P_REQUIRE(!(kind == EPI_SWIGLU && ep.has_lora),
              "SwiGLU with LoRA runs on the CTA-pair engine only (M >= 256, variant groups of whole 256-row tiles)");
  if (kind == EPI_CE_GRAD) B2P_REQUIRE(ep.targets && ep.row_lse, "CE gradient needs targets and row LSE");
  if (bf16) return dispatch_kind<__nv_bfloat16, true>(bn, kind, X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
  return dispatch_kind<__half, false>(bn, kind, X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
}

}  // namespace b2p
