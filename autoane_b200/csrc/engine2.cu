// engine2.cu — host launcher of the CTA-pair projection engine (gemm2.cuh).
#include "engine.cuh"
#include "gemm2.cuh"

namespace b2p {

namespace {

template <int BN, int KIND, typename OutT, bool BF16, int NSEG, int OPM = 0>
int launch_pair_t(const void* X, int ldx, const void* W, int ldw, int M, int N, int K, void* out, int ldo,
                  const void* u16, const EpiParams& ep, cudaStream_t st) {
  DeviceCtx* c = nullptr;
  int rc = ctx_get(&c);
  if (rc) return rc;
  using S = PairSmem<BN, KIND, NSEG>;
  const TmapType in_t = BF16 ? TM_BF16 : TM_F16;
  CUtensorMap tx, tw, to, tu;
  // K-major: [M][K] / [N][K] rows, one box of 64 K x the tile's rows; MN-major: [K][M] / [K][N] rows,
  // boxes of 64 M (or N) x 64 K
  if (OPM & 1) {
    if ((rc = make_tmap_2d(&tx, X, in_t, (uint64_t)M, (uint64_t)K, (uint64_t)ldx, 64, 64, 128))) return rc;
  } else {
    if ((rc = make_tmap_2d(&tx, X, in_t, (uint64_t)K, (uint64_t)M, (uint64_t)ldx, 64, kBM, 128))) return rc;
  }
  if (OPM & 2) {
    if ((rc = make_tmap_2d(&tw, W, in_t, (uint64_t)N, (uint64_t)K, (uint64_t)ldw, 64, 64, 128))) return rc;
  } else {
    if ((rc = make_tmap_2d(&tw, W, in_t, (uint64_t)K, (uint64_t)N, (uint64_t)ldw, 64, BN / 2, 128))) return rc;
  }
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
  if (NSEG > 0) {
    if ((rc = make_tmap_2d(&tu, u16, in_t, (uint64_t)kUCols, (uint64_t)M, (uint64_t)kUCols, 16, kBM, 32))) return rc;
  } else {
    tu = tx;
  }
  auto kern = gemm_pair_kernel<BN, KIND, OutT, BF16, NSEG, OPM>;
  static thread_local uint64_t attr_dev_mask = 0;
  if (!(attr_dev_mask & (1ull << (c->device & 63)))) {
    B2P_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal));
    attr_dev_mask |= 1ull << (c->device & 63);
  }
  const long long tiles = (long long)((M + 2 * kBM - 1) / (2 * kBM)) * ((N + BN - 1) / BN);
  const int max_clusters = c->num_sms / 2;
  const int clusters = (int)(tiles < max_clusters ? tiles : max_clusters);
  EpiParams e = ep;
  e.status = c->status;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * clusters), 1, 1);
  cfg.blockDim = dim3(kPairThreads, 1, 1);
  cfg.dynamicSmemBytes = S::kTotal;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // the kernel calls pdl_enter()
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  B2P_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, tx, tw, to, tu, M, N, K, e));
  B2P_POST_LAUNCH();
  return B2P_OK;
}

template <typename H, bool BF16>
int dispatch_pair(int kind, const void* X, int ldx, const void* W, int ldw, int M, int N, int K, void* out, int ldo,
                  const void* u16, const EpiParams& ep, cudaStream_t st) {
  const int nseg = ep.has_lora ? ep.lora.nseg : 0;
  // plain outputs whose 256 x 256 tiles would keep fewer than a quarter of the clusters busy (small
  // M): 64-column tiles put four times as many clusters on the weight stream. (Measured: at a
  // quarter or more, and with 128-column tiles, the extra per-tile cost outweighs the parallelism.)
  int bn = 256;
  if ((kind == EPI_F32 || kind == EPI_H16) && nseg == 0) {
    DeviceCtx* c = nullptr;
    int rc = ctx_get(&c);
    if (rc) return rc;
    const long long mt = (M + 2 * kBM - 1) / (2 * kBM), clusters = c->num_sms / 2;
    if (4 * mt * ((N + 255) / 256) < clusters) bn = 64;
  }
  switch (kind) {
    case EPI_F32:
      if (nseg == 0 && bn == 64)
        return launch_pair_t<64, EPI_F32, H, BF16, 0>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
      if (nseg == 0) return launch_pair_t<256, EPI_F32, H, BF16, 0>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
      break;
    case EPI_H16:
      if (nseg == 0 && bn == 64)
        return launch_pair_t<64, EPI_H16, H, BF16, 0>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
      if (nseg == 0) return launch_pair_t<256, EPI_H16, H, BF16, 0>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
      break;
    case EPI_QKV_ROPE:
      if (nseg == 3)
        return launch_pair_t<256, EPI_QKV_ROPE, H, BF16, 3>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
      break;
    case EPI_RESID:
      if (nseg == 0) return launch_pair_t<256, EPI_RESID, H, BF16, 0>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
      if (nseg == 1) return launch_pair_t<256, EPI_RESID, H, BF16, 1>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
      break;
    case EPI_SWIGLU:
      if (nseg == 0) return launch_pair_t<256, EPI_SWIGLU, H, BF16, 0>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
      if (nseg == 2 && ep.lora.inter128)
        return launch_pair_t<256, EPI_SWIGLU, H, BF16, 2>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
      break;
    case EPI_CE:
      if (nseg == 0) return launch_pair_t<256, EPI_CE, H, BF16, 0>(X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
      break;
  }
  set_error("no CTA-pair kernel for epilogue %d with %d LoRA segments", kind, nseg);
  return B2P_ERR_UNSUPPORTED;
}

template <typename H, bool BF16>
int dispatch_pair_mn(int kind, int opm, const void* X, int ldx, const void* W, int ldw, int M, int N, int K, void* out,
                     int ldo, const EpiParams& ep, cudaStream_t st) {
  switch (kind) {
    case EPI_F32:
      if (opm == 2) return launch_pair_t<256, EPI_F32, H, BF16, 0, 2>(X, ldx, W, ldw, M, N, K, out, ldo, nullptr, ep, st);
      if (opm == 3) return launch_pair_t<256, EPI_F32, H, BF16, 0, 3>(X, ldx, W, ldw, M, N, K, out, ldo, nullptr, ep, st);
      break;
    case EPI_H16:
      if (opm == 2) return launch_pair_t<256, EPI_H16, H, BF16, 0, 2>(X, ldx, W, ldw, M, N, K, out, ldo, nullptr, ep, st);
      break;
    case EPI_RESID:
      if (opm == 3)
        return launch_pair_t<256, EPI_RESID, H, BF16, 0, 3>(X, ldx, W, ldw, M, N, K, out, ldo, nullptr, ep, st);
      break;
  }
  set_error("no MN-major CTA-pair kernel for epilogue %d with operand layout %d", kind, opm);
  return B2P_ERR_UNSUPPORTED;
}

}  // namespace

bool pair_mn_supported(int kind, int opm, int M, int N, int K, const void* X, int ldx, const void* W, int ldw) {
  // MN-major boxes start on 64-element boundaries of the contiguous dimension (16-byte TMA rule);
  // rows of 16-byte multiples
  if (M < 2 * kBM || N < 1 || K < 1 || ldx % 8 != 0 || ldw % 8 != 0) return false;
  if ((reinterpret_cast<uintptr_t>(X) & 15u) != 0 || (reinterpret_cast<uintptr_t>(W) & 15u) != 0) return false;
  return (kind == EPI_F32 && (opm == 2 || opm == 3)) || (kind == EPI_H16 && opm == 2) ||
         (kind == EPI_RESID && opm == 3);
}

int launch_gemm_pair_mn(int kind, int opm, bool bf16, const void* X, int ldx, const void* W, int ldw, int M, int N,
                        int K, void* out, int ldo, const EpiParams& ep, cudaStream_t st) {
  B2P_REQUIRE(M > 0 && N > 0 && K > 0, "empty GEMM (M=%d N=%d K=%d)", M, N, K);
  B2P_REQUIRE(!ep.has_lora, "MN-major CTA-pair GEMMs take no LoRA segments");
  B2P_REQUIRE(out != nullptr, "GEMM without an output");
  B2P_REQUIRE(pair_mn_supported(kind, opm, M, N, K, X, ldx, W, ldw),
              "MN-major CTA-pair GEMM: epilogue %d / layout %d unsupported, M < 256, or unaligned operands", kind, opm);
  B2P_REQUIRE((opm & 1 ? ldx >= M : ldx >= K) && (opm & 2 ? ldw >= N : ldw >= K), "operand row pitch too small");
  if (bf16) return dispatch_pair_mn<__nv_bfloat16, true>(kind, opm, X, ldx, W, ldw, M, N, K, out, ldo, ep, st);
  return dispatch_pair_mn<__half, false>(kind, opm, X, ldx, W, ldw, M, N, K, out, ldo, ep, st);
}

bool pair_supported(int kind, int M, int N, const EpiParams& ep) {
  (void)N;
  if (M < 2 * kBM) return false;
  if (kind == EPI_CE_GRAD) return false;  // single-CTA engine only
  if (ep.has_lora) {
    if (ep.lora.group_rows % (2 * kBM) != 0) return false;
    if (!(kind == EPI_QKV_ROPE && ep.lora.nseg == 3) && !(kind == EPI_RESID && ep.lora.nseg == 1) &&
        !(kind == EPI_SWIGLU && ep.lora.nseg == 2 && ep.lora.inter128))
      return false;
  }
  if (kind == EPI_QKV_ROPE && ep.seq_len % (2 * kBM) != 0 && ep.seq_len % kBM != 0) return false;
  return true;
}

int launch_gemm_pair(int kind, bool bf16, const void* X, int ldx, const void* W, int ldw, int M, int N, int K,
                     void* out, int ldo, const void* u16, const EpiParams& ep, cudaStream_t st) {
  B2P_REQUIRE(M > 0 && N > 0 && K > 0, "empty GEMM (M=%d N=%d K=%d)", M, N, K);
  if (ep.has_lora) {
    B2P_REQUIRE(u16 != nullptr, "LoRA GEMM without a U buffer");
    B2P_REQUIRE(ep.lora.rank == 4 || ep.lora.rank == 8, "LoRA rank must be 4 or 8 (got %d)", ep.lora.rank);
    B2P_REQUIRE(ep.lora.group_rows % (2 * kBM) == 0, "LoRA variant groups must span whole 256-row tiles");
    B2P_REQUIRE(ep.lora.n_groups >= (M + ep.lora.group_rows - 1) / ep.lora.group_rows &&
                    ep.lora.n_groups <= kMaxGroups && ep.lora.n_variants >= 1 && ep.lora.n_variants <= kMaxGroups,
                "LoRA group/variant tables out of range");
    for (int s = 0; s < ep.lora.nseg; ++s) {
      B2P_REQUIRE(ep.lora.seg_boff[s] % ep.lora.rank == 0, "LoRA B offset must be a multiple of the rank");
      B2P_REQUIRE(ep.lora.seg_ucol[s] % 16 == 0 && ep.lora.seg_ucol[s] + 16 <= kUCols, "bad U column");
    }
  }
  if (kind != EPI_CE) B2P_REQUIRE(out != nullptr, "GEMM without an output");
  if (kind == EPI_SWIGLU) B2P_REQUIRE(N % 256 == 0, "SwiGLU needs N %% 256 == 0");
  if (kind == EPI_QKV_ROPE)
    B2P_REQUIRE(ep.head_dim == 64 && ep.seq_len % kBM == 0 && ep.rope_cols % 64 == 0,
                "RoPE epilogue needs head_dim 64, seq %% 128 == 0 and whole heads");
  if (bf16) return dispatch_pair<__nv_bfloat16, true>(kind, X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
  return dispatch_pair<__half, false>(kind, X, ldx, W, ldw, M, N, K, out, ldo, u16, ep, st);
}

}  // namespace b2p
