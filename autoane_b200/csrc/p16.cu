// p16.cu — backprop-LoRA training step on the device (the reference's P16
// path: forward with activation saves, fp32 backward of the whole network
// with gradients only for the LoRA adapters and RMSNorm weights, Adam).
//
// Reference: training/train_mezo.m:1961-2136 (step), training/backprop_lora.h:147-288
// (bp_lora_backward), training/cpu_ops.h:24-104 (rmsnorm_bwd, adam_update),
// :108-133 (cross_entropy_loss), :213-290 (cpu_sdpa_backward), :377-393
// (rope_backward_inplace), training/config.h:286-292 (lora_grad_project).
//
// Semantics follow the reference's conv-fused P16 mode: the frozen base
// weights stay unmerged on the device, the adapters are applied split
// (W·x + B·(A·x)), and the backward propagates through W_eff = W + B·A exactly
// as bp_lora_backward does with the merged weights (dX = W^T·dY + A^T·(B^T·dY)).
// dW of a LoRA'd projection is never formed: dB = dY^T·(X·A^T) and
// dA = (dY·B)^T·X, the factored form of lora_grad_project.
//
// Layout: token-major rows (R = n_seq * seq), 16-bit GEMM operands, fp32
// residual-stream gradients. The backward GEMMs run on the tcgen05 engine
// against transposed copies of the frozen weights built once per upload.
// Gradients carry a scale lambda = 2^k * R (dlogits are stored as
// 2^k * (softmax - onehot), 16-bit); the weight gradients are multiplied by
// 1/lambda when they are written.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>
#include "model.cuh"
#include "mma.cuh"

namespace b2p {

// One factored LoRA weight-gradient: out = scale * sum_t X[t, c] * U[t, ucol + j]
// for c < ncols, j < rank, written [ncols][rank] (B layout) or [rank][ncols] (A layout).
// One factored weight gradient out_s[c][j] = sum_t X[t, c] · U[t, ucol + 16 s + j] for the
// nu segments s of U (16-column groups), stored in the A ([rank][ncols]) or B ([ncols][rank])
// layout of the trainable set.
struct WgradJob {
  const void* X;
  long long ldx;
  int ncols;
  int ucol;
  const void* U;  // [R][ldu]
  long long ldu;
  float* out[3];
  int nu;
  int a_layout;
};
constexpr int kMaxWgradJobs = 6;
constexpr int kWgradSplit = 8;  // row chunks per weight gradient (partials summed in chunk order)
constexpr int kRmsTeam = 128;   // threads per row of the RMSNorm backward
constexpr int kRmsTeams = 4;    // rows in flight per block
constexpr int kRmsBlocks = 296; // blocks (dw partial rows) per RMSNorm backward launch, 2 per SM

struct P16State {
  int rows = 0;
  int weights_version = -1;
  int cv_pad = 0;
  void *wqkvT = nullptr, *woT = nullptr, *w13T = nullptr, *w2T = nullptr, *cembedT = nullptr;
  int kmajor_version = -1;  // weights_version of w13T / w2T / cembedT (built only for the K-major path)
  int cembedT_pad = 0;
  bool use_mn = false;      // this step reads W1|W3, W2, the embedding (and dW's operands) MN-major
  ForwardSaves sv;
  void* dlogits = nullptr;  // (full mode also keeps sv.xn2)
  float *dy = nullptr, *dy2 = nullptr, *dxf = nullptr, *dsilu = nullptr;
  void *d16 = nullptr, *dh13 = nullptr, *da = nullptr, *dqkv = nullptr, *ub_o = nullptr;
  float* dvec = nullptr;
  float* rms_part = nullptr;
  float* wgrad_part = nullptr;
  float* a_oT = nullptr;
  void *bblk_qkv = nullptr, *bblk_o = nullptr;
  float* grad = nullptr;
  float *adam_m = nullptr, *adam_v = nullptr;
  int adam_t = 0;
  uint32_t* flag = nullptr;
  WgradJob* d_jobs = nullptr;
  int* d_rms_off = nullptr;
  int gen = 0;  // bumped whenever a buffer a captured graph points into is reallocated
  // full backprop (train.m): fp32 masters of every projection weight, laid out as the 16-bit
  // copies ([all layers' Wq|Wk|Wv] [all Wo] [all W1|W3 interleaved] [all W2]), their gradients,
  // Adam moments, embedding gradients and scratch
  bool full = false;
  float *mw = nullptr, *gw = nullptr, *am_w = nullptr, *av_w = nullptr;
  long long n_w = 0, o_qkv = 0, o_o = 0, o_13 = 0, o_2 = 0;
  float *g_embed = nullptr, *g_cembed = nullptr, *am_e = nullptr, *av_e = nullptr;
  void *tA = nullptr, *tB = nullptr, *gate = nullptr;
  int32_t* d_seg = nullptr;  // [1 + rows + 1 + rows]: segment count, starts, row order (rows grouped by token)
  long long* d_nseg = nullptr;  // norm / Adam segment tables: [3 + 2L+1] offsets then lengths
  float* norm_part = nullptr;  // [kNormBlocks]; then norm, clip scale
  int full_t = 0;
  // the captured forward + backward (CUDA graph), replayed while its key matches
  struct Graph {
    const void* tok = nullptr;
    int n_seq = 0, gen = -1, scale_log2 = 0, prof_epoch = -1;
    bool pair = true, tc_attn = true, tc_attn_bwd = true, pdl = true;
    cudaGraphExec_t exec = nullptr;
    long long launches = 0;
  } graph;
};

namespace {

void free_ptrs(std::initializer_list<void*> ps) {
  for (void* p : ps)
    if (p) cudaFree(p);
}

void release_rows(P16State* s) {
  const ForwardSaves& v = s->sv;
  free_ptrs({s->tA, s->tB, s->gate, s->d_seg, v.xn2});
  s->tA = s->tB = s->gate = nullptr;
  s->d_seg = nullptr;
  free_ptrs({v.x_in, v.x_mid, v.xn, v.U, v.qkv, v.attn, v.lse, v.h13, v.x_final, v.xn_final, v.row_lse, s->dlogits,
             s->dy, s->dy2, s->dxf, s->dsilu, s->d16, s->dh13, s->da, s->dqkv, s->ub_o, s->dvec,
             s->rms_part, s->wgrad_part});
  s->sv = ForwardSaves();
  s->dlogits = s->d16 = s->dh13 = s->da = s->dqkv = s->ub_o = nullptr;
  s->dy = s->dy2 = s->dxf = s->dsilu = s->dvec = s->rms_part = s->wgrad_part = nullptr;
  s->rows = 0;
}

// ---------------------------------------------------------------------------
// layout kernels
// ---------------------------------------------------------------------------
template <typename T>
__global__ void transpose16_kernel(const T* __restrict__ src, int rows, int cols, long long ld_src, T* __restrict__ dst,
                                   long long ld_dst) {
  __shared__ T tile[32][34];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = src[(long long)r * ld_src + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) dst[(long long)c * ld_dst + r] = tile[threadIdx.x][i];
  }
}

// dst[c][r] = src[r][c] for one [rows, cols] 16-bit matrix
int transpose16(const void* src, int rows, int cols, long long ld_src, void* dst, long long ld_dst, bool bf16,
                cudaStream_t st) {
  dim3 grid((cols + 31) / 32, (rows + 31) / 32), block(32, 8);
  if (bf16)
    transpose16_kernel<__nv_bfloat16><<<grid, block, 0, st>>>(static_cast<const __nv_bfloat16*>(src), rows, cols,
                                                              ld_src, static_cast<__nv_bfloat16*>(dst), ld_dst);
  else
    transpose16_kernel<__half><<<grid, block, 0, st>>>(static_cast<const __half*>(src), rows, cols, ld_src,
                                                       static_cast<__half*>(dst), ld_dst);
  B2P_POST_LAUNCH();
  return B2P_OK;
}

template <typename T>
__global__ void scale16_kernel(const float* __restrict__ src, long long n, float alpha, T* __restrict__ dst) {
  pdl_enter();
  for (long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4; i < n;
       i += (long long)gridDim.x * blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(src + i);
    uint2 o;
    o.x = pack_h2<T>(v.x * alpha, v.y * alpha);
    o.y = pack_h2<T>(v.z * alpha, v.w * alpha);
    *reinterpret_cast<uint2*>(dst + i) = o;
  }
}

int scale16(const float* src, long long n, float alpha, void* dst, bool bf16, cudaStream_t st) {
  const int blocks = (int)std::min<long long>((n / 4 + 255) / 256, 148 * 8);
  if (bf16)
    B2P_CHECK_CUDA(launch_pdl(scale16_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, st, src, n, alpha,
                              static_cast<__nv_bfloat16*>(dst)));
  else
    B2P_CHECK_CUDA(launch_pdl(scale16_kernel<__half>, dim3(blocks), dim3(256), 0, st, src, n, alpha,
                              static_cast<__half*>(dst)));
  B2P_POST_LAUNCH();
  return B2P_OK;
}

// ---------------------------------------------------------------------------
// SwiGLU backward (backprop_lora.h:171-191):
//   sig = 1/(1+e^-h1); dh3 = ds * h1 * sig; dh1 = ds * h3 * (sig + h1*sig*(1-sig))
// written back into the interleaved W1|W3 column order of h13.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void swiglu_bwd_kernel(const float* __restrict__ dsilu, const T* __restrict__ h13, int rows, int H,
                                  T* __restrict__ dh13) {
  pdl_enter();
  const long long n4 = (long long)rows * H / 4;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const long long e = i * 4;
    const long long r = e / H;
    const int c = (int)(e - r * H);
    const long long o1 = r * 2 * H + (c >> 7) * 256 + (c & 127), o3 = o1 + 128;
    const float4 ds = *reinterpret_cast<const float4*>(dsilu + e);
    const uint2 a = *reinterpret_cast<const uint2*>(h13 + o1);
    const uint2 b = *reinterpret_cast<const uint2*>(h13 + o3);
    const float2 h1a = H2<T>::to_f2(*reinterpret_cast<const typename H2<T>::V*>(&a.x));
    const float2 h1b = H2<T>::to_f2(*reinterpret_cast<const typename H2<T>::V*>(&a.y));
    const float2 h3a = H2<T>::to_f2(*reinterpret_cast<const typename H2<T>::V*>(&b.x));
    const float2 h3b = H2<T>::to_f2(*reinterpret_cast<const typename H2<T>::V*>(&b.y));
    const float h1[4] = {h1a.x, h1a.y, h1b.x, h1b.y}, h3[4] = {h3a.x, h3a.y, h3b.x, h3b.y};
    const float d[4] = {ds.x, ds.y, ds.z, ds.w};
    float g1[4], g3[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float sig = 1.0f / (1.0f + expf(-h1[k]));
      g3[k] = d[k] * (h1[k] * sig);
      g1[k] = d[k] * h3[k] * (sig * (1.0f + h1[k] * (1.0f - sig)));
    }
    *reinterpret_cast<uint2*>(dh13 + o1) = make_uint2(pack_h2<T>(g1[0], g1[1]), pack_h2<T>(g1[2], g1[3]));
    *reinterpret_cast<uint2*>(dh13 + o3) = make_uint2(pack_h2<T>(g3[0], g3[1]), pack_h2<T>(g3[2], g3[3]));
  }
}

int swiglu_bwd(const float* dsilu, const void* h13, int rows, int H, void* dh13, bool bf16, cudaStream_t st) {
  const long long n4 = (long long)rows * H / 4;
  const int blocks = (int)std::min<long long>((n4 + 255) / 256, 148 * 16);
  if (bf16)
    B2P_CHECK_CUDA(launch_pdl(swiglu_bwd_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, st, dsilu,
                              static_cast<const __nv_bfloat16*>(h13), rows, H, static_cast<__nv_bfloat16*>(dh13)));
  else
    B2P_CHECK_CUDA(launch_pdl(swiglu_bwd_kernel<__half>, dim3(blocks), dim3(256), 0, st, dsilu,
                              static_cast<const __half*>(h13), rows, H, static_cast<__half*>(dh13)));
  B2P_POST_LAUNCH();
  return B2P_OK;
}

// ---------------------------------------------------------------------------
// RMSNorm backward (rmsnorm_bwd, training/cpu_ops.h:24-60), one warp per row:
//   rrms = 1/sqrt(sum x^2 / d + 1e-5); dot = sum_i w_i g_i x_i * rrms^2 / d
//   dx_i = (w_i g_i - x_i dot) * rrms (+ resid_i);  dw_i += g_i x_i rrms
// The dw partials of a block go to part[block][d] and are summed in block order
// by rms_part_reduce_kernel.
// ---------------------------------------------------------------------------
struct RmsBwdArgs {
  const float* g;
  const float* x;
  const float* w;
  const float* resid;  // may be null
  float* out;
  void* out16;         // may be null: 16-bit copy of out * alpha16
  float alpha16;
  float* part;         // [blocks][D]
  int rows;
};

// A team of 128 threads owns one row at a time (float4 chunks c4 = tt + 128k);
// kRmsTeams teams per block walk the rows grid-stride, so each block's dw partial
// covers a fixed, deterministic row set.
template <typename T, int NCH>
__global__ void __launch_bounds__(kRmsTeam * kRmsTeams) rms_bwd_kernel(RmsBwdArgs a, int D) {
  pdl_enter();
  __shared__ float s_red[kRmsTeams][2][4][2];  // [team][row parity][warp][ss, dot]
  __shared__ float4 s_acc[kRmsTeams][kRmsTeam * NCH];
  const int team = threadIdx.x / kRmsTeam, tt = threadIdx.x % kRmsTeam;
  const int wit = tt >> 5, lane = tt & 31;
  const int nc4 = D / 4;
  const float4* w4 = reinterpret_cast<const float4*>(a.w);
  float4 wv[NCH], acc[NCH];
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    const int c4 = tt + kRmsTeam * k;
    wv[k] = c4 < nc4 ? __ldg(w4 + c4) : make_float4(0.f, 0.f, 0.f, 0.f);
    acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const float invd = 1.0f / (float)D;
  int parity = 0;
  for (int row = blockIdx.x * kRmsTeams + team; row < a.rows; row += gridDim.x * kRmsTeams) {
    const float4* g4 = reinterpret_cast<const float4*>(a.g + (long long)row * D);
    const float4* x4 = reinterpret_cast<const float4*>(a.x + (long long)row * D);
    float4 gv[NCH], xv[NCH];
    float ss = 0.f, dot = 0.f;
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      const int c4 = tt + kRmsTeam * k;
      gv[k] = c4 < nc4 ? g4[c4] : make_float4(0.f, 0.f, 0.f, 0.f);
      xv[k] = c4 < nc4 ? x4[c4] : make_float4(0.f, 0.f, 0.f, 0.f);
      ss += xv[k].x * xv[k].x + xv[k].y * xv[k].y + xv[k].z * xv[k].z + xv[k].w * xv[k].w;
      dot += (wv[k].x * gv[k].x) * xv[k].x + (wv[k].y * gv[k].y) * xv[k].y + (wv[k].z * gv[k].z) * xv[k].z +
             (wv[k].w * gv[k].w) * xv[k].w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ss += __shfl_xor_sync(0xffffffffu, ss, o);
      dot += __shfl_xor_sync(0xffffffffu, dot, o);
    }
    if (lane == 0) {
      s_red[team][parity][wit][0] = ss;
      s_red[team][parity][wit][1] = dot;
    }
    named_bar_sync(1 + team, kRmsTeam);
    ss = s_red[team][parity][0][0] + s_red[team][parity][1][0] + s_red[team][parity][2][0] + s_red[team][parity][3][0];
    dot = s_red[team][parity][0][1] + s_red[team][parity][1][1] + s_red[team][parity][2][1] + s_red[team][parity][3][1];
    parity ^= 1;
    const float rrms = 1.0f / sqrtf(ss * invd + 1e-5f);
    const float dots = dot * (rrms * rrms * invd);
    float4* o4 = reinterpret_cast<float4*>(a.out + (long long)row * D);
    const float4* r4 = a.resid ? reinterpret_cast<const float4*>(a.resid + (long long)row * D) : nullptr;
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      const int c4 = tt + kRmsTeam * k;
      if (c4 >= nc4) continue;
      float4 d;
      d.x = (wv[k].x * gv[k].x - xv[k].x * dots) * rrms;
      d.y = (wv[k].y * gv[k].y - xv[k].y * dots) * rrms;
      d.z = (wv[k].z * gv[k].z - xv[k].z * dots) * rrms;
      d.w = (wv[k].w * gv[k].w - xv[k].w * dots) * rrms;
      if (r4) {
        const float4 r = r4[c4];
        d.x += r.x; d.y += r.y; d.z += r.z; d.w += r.w;
      }
      o4[c4] = d;
      acc[k].x += (gv[k].x * xv[k].x) * rrms;
      acc[k].y += (gv[k].y * xv[k].y) * rrms;
      acc[k].z += (gv[k].z * xv[k].z) * rrms;
      acc[k].w += (gv[k].w * xv[k].w) * rrms;
      if (a.out16) {
        uint2 h;
        h.x = pack_h2<T>(d.x * a.alpha16, d.y * a.alpha16);
        h.y = pack_h2<T>(d.z * a.alpha16, d.w * a.alpha16);
        *reinterpret_cast<uint2*>(static_cast<T*>(a.out16) + (long long)row * D + 4 * c4) = h;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < NCH; ++k) s_acc[team][tt + kRmsTeam * k] = acc[k];
  __syncthreads();
  float4* p4 = reinterpret_cast<float4*>(a.part + (long long)blockIdx.x * D);
  for (int c4 = threadIdx.x; c4 < nc4; c4 += blockDim.x) {
    float4 t = s_acc[0][c4];
#pragma unroll
    for (int m = 1; m < kRmsTeams; ++m) {
      const float4 u = s_acc[m][c4];
      t.x += u.x; t.y += u.y; t.z += u.z; t.w += u.w;
    }
    p4[c4] = t;
  }
}

int rms_blocks(int rows) { return std::min(kRmsBlocks, (rows + kRmsTeams - 1) / kRmsTeams); }

template <typename T>
int rms_bwd_t(const RmsBwdArgs& a, int D, cudaStream_t st) {
  const int blocks = rms_blocks(a.rows);
  const int nch = (D / 4 + kRmsTeam - 1) / kRmsTeam;
  switch (nch) {
    case 1: B2P_CHECK_CUDA(launch_pdl(rms_bwd_kernel<T, 1>, dim3(blocks), dim3(kRmsTeam * kRmsTeams), 0, st, a, D)); break;
    case 2: B2P_CHECK_CUDA(launch_pdl(rms_bwd_kernel<T, 2>, dim3(blocks), dim3(kRmsTeam * kRmsTeams), 0, st, a, D)); break;
    case 3: B2P_CHECK_CUDA(launch_pdl(rms_bwd_kernel<T, 3>, dim3(blocks), dim3(kRmsTeam * kRmsTeams), 0, st, a, D)); break;
    case 4: B2P_CHECK_CUDA(launch_pdl(rms_bwd_kernel<T, 4>, dim3(blocks), dim3(kRmsTeam * kRmsTeams), 0, st, a, D)); break;
    default: set_error("RMSNorm backward: unsupported width %d", D); return B2P_ERR_UNSUPPORTED;
  }
  B2P_POST_LAUNCH();
  return B2P_OK;
}

int rms_bwd(const RmsBwdArgs& a, int D, bool bf16, cudaStream_t st) {
  B2P_REQUIRE(D % 4 == 0 && D <= 4 * kRmsTeam * 4, "RMSNorm backward: width %d must be a multiple of 4, <= 2048", D);
  return bf16 ? rms_bwd_t<__nv_bfloat16>(a, D, st) : rms_bwd_t<__half>(a, D, st);
}

// grad[off[v] + d] = scale * sum_b part[v][b][d]  (blocks summed in order)
__global__ void rms_part_reduce_kernel(const float* __restrict__ part, int nvec, int nblk, int D,
                                       const int* __restrict__ off, float scale, float* __restrict__ grad) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nvec * D) return;
  const int v = i / D, d = i - v * D;
  const float* p = part + (long long)v * nblk * D + d;
  float s = 0.f;
  for (int b = 0; b < nblk; ++b) s += p[(long long)b * D];
  grad[off[v] + d] = s * scale;
}

// ---------------------------------------------------------------------------
// factored LoRA weight gradients (lora_grad_project, training/config.h:286-292,
// without forming dW) on the tensor cores: Xᵀ·U as an [ncols x R]·[R x 8 nu] product.
// One block per (128-column tile, job, row chunk); 8 warps own 16 columns each and
// run mma.sync m16n8k16 (fp32 accumulation) over the chunk's rows, 64 rows per
// cp.async stage, two stages in flight. Xᵀ and U fragments come from ldmatrix.trans
// of the row-major tiles. Partials part[job][chunk][c][24] are summed over the chunks
// in order by a second kernel (deterministic), which scales and stores them.
// ---------------------------------------------------------------------------
constexpr int kWgRows = 64;    // rows per stage
constexpr int kWgCols = 128;   // columns per block
constexpr int kWgXs = kWgCols + 8;  // padded smem row (elements): conflict-free ldmatrix
constexpr int kWgUs = 40;           // up to three 8-column U segments; 80-byte rows: conflict-free ldmatrix
constexpr int kWgPartJ = 24;        // partial entries per column

template <typename T>
__global__ void __launch_bounds__(256) lora_wgrad_kernel(const WgradJob* __restrict__ jobs, int rows,
                                                        float* __restrict__ part, int max_cols) {
  pdl_enter();
  __shared__ __align__(128) T s_x[2][kWgRows][kWgXs];
  __shared__ __align__(128) T s_u[2][kWgRows][kWgUs];
  const WgradJob jb = jobs[blockIdx.y];
  const int c0 = blockIdx.x * kWgCols;
  if (c0 >= jb.ncols) return;
  const int chunk_rows = (rows + kWgradSplit - 1) / kWgradSplit;
  const int r_begin = blockIdx.z * chunk_rows, r_end = min(rows, r_begin + chunk_rows);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const T* X = static_cast<const T*>(jb.X);
  const T* U = static_cast<const T*>(jb.U);
  const int nu = jb.nu;
  const uint32_t sx0 = smem_u32(&s_x[0][0][0]), su0 = smem_u32(&s_u[0][0][0]);
  constexpr uint32_t kXStage = kWgRows * kWgXs * 2, kUStage = kWgRows * kWgUs * 2;

  auto load_stage = [&](int st, int t0) {
    // X: 64 rows x 128 columns = 1024 chunks of 16 B; columns past ncols and rows past
    // the chunk are zero-filled
    for (int i = tid; i < kWgRows * (kWgCols / 8); i += 256) {
      const int r = i >> 4, ch = i & 15;
      const uint32_t dst = sx0 + st * kXStage + (uint32_t)((r * kWgXs + ch * 8) * 2);
      if (t0 + r < r_end && c0 + ch * 8 < jb.ncols)
        cp_async16(dst, X + (long long)(t0 + r) * jb.ldx + c0 + ch * 8);
      else
        *reinterpret_cast<uint4*>(&s_x[st][r][ch * 8]) = make_uint4(0u, 0u, 0u, 0u);
    }
    // U: 64 rows x nu segments of 8 columns (16 B each)
    for (int i = tid; i < kWgRows * 3; i += 256) {
      const int r = i / 3, sg = i - r * 3;
      if (sg >= nu) continue;
      const uint32_t dst = su0 + st * kUStage + (uint32_t)((r * kWgUs + sg * 8) * 2);
      if (t0 + r < r_end)
        cp_async16(dst, U + (long long)(t0 + r) * jb.ldu + jb.ucol + 16 * sg);
      else
        *reinterpret_cast<uint4*>(&s_u[st][r][sg * 8]) = make_uint4(0u, 0u, 0u, 0u);
    }
    cp_async_commit();
  };

  float acc[3][4];
#pragma unroll
  for (int s3 = 0; s3 < 3; ++s3) acc[s3][0] = acc[s3][1] = acc[s3][2] = acc[s3][3] = 0.f;
  const int nst = (r_end - r_begin + kWgRows - 1) / kWgRows;
  if (nst > 0) load_stage(0, r_begin);
  const int q = lane >> 3, lr = lane & 7;
  for (int it = 0; it < nst; ++it) {
    const int st = it & 1;
    if (it + 1 < nst) {
      load_stage(st ^ 1, r_begin + (it + 1) * kWgRows);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kWgRows / 16; ++kk) {
      // A = Xᵀ (16 columns x 16 rows): matrices (m 0-7 | 8-15) x (k 0-7 | 8-15), transposed
      uint32_t a[4];
      const int k_row = kk * 16 + (q >> 1) * 8 + lr, m_col = warp * 16 + (q & 1) * 8;
      ldsm_x4_t(sx0 + st * kXStage + (uint32_t)((k_row * kWgXs + m_col) * 2), a[0], a[1], a[2], a[3]);
#pragma unroll
      for (int sg = 0; sg < 3; ++sg) {
        if (sg >= nu) break;
        // B = U (16 rows x 8 columns), transposed: (k 0-7) and (k 8-15)
        uint32_t b0, b1, b2, b3;
        const int u_row = kk * 16 + (q & 1) * 8 + lr;
        ldsm_x4_t(su0 + st * kUStage + (uint32_t)((u_row * kWgUs + sg * 8) * 2), b0, b1, b2, b3);
        mma16816<T>(acc[sg], a, b0, b1);
      }
    }
    __syncthreads();  // stage `st` is refilled by the next iteration's prefetch
  }
  // D fragment: rows = columns c (lane/4, +8), cols = j (2 (lane%4) + {0,1})
  float* p = part + (long long)(blockIdx.y * kWgradSplit + blockIdx.z) * max_cols * kWgPartJ;
  const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int sg = 0; sg < 3; ++sg) {
    if (sg >= nu) break;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int col = c0 + warp * 16 + g + ((e >> 1) << 3);
      const int jj = 2 * t4 + (e & 1);
      if (col < jb.ncols) p[(long long)col * kWgPartJ + sg * 8 + jj] = acc[sg][e];
    }
  }
}

__global__ void lora_wgrad_reduce_kernel(const WgradJob* __restrict__ jobs, int rank, const float* __restrict__ part,
                                         int max_cols, float scale) {
  pdl_enter();
  const WgradJob jb = jobs[blockIdx.y];
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // (segment, col, j)
  const int per = jb.ncols * rank;
  if (i >= jb.nu * per) return;
  const int sg = i / per, rem = i - sg * per;
  const int col = rem / rank, j = rem - col * rank;
  float s = 0.f;
  for (int z = 0; z < kWgradSplit; ++z)
    s += part[((long long)(blockIdx.y * kWgradSplit + z) * max_cols + col) * kWgPartJ + sg * 8 + j];
  if (jb.a_layout)
    jb.out[sg][(long long)j * jb.ncols + col] = s * scale;
  else
    jb.out[sg][(long long)col * rank + j] = s * scale;
}

int lora_wgrad(const WgradJob* d_jobs, int njobs, int max_cols, int rows, int rank, float scale, float* part,
               bool bf16, cudaStream_t st) {
  B2P_REQUIRE(rank == 4 || rank == 8, "LoRA rank must be 4 or 8");
  dim3 grid((max_cols + kWgCols - 1) / kWgCols, njobs, kWgradSplit);
  if (bf16)
    B2P_CHECK_CUDA(launch_pdl(lora_wgrad_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, d_jobs, rows, part, max_cols));
  else
    B2P_CHECK_CUDA(launch_pdl(lora_wgrad_kernel<__half>, grid, dim3(256), 0, st, d_jobs, rows, part, max_cols));
  B2P_POST_LAUNCH();
  dim3 g2((3 * max_cols * rank + 255) / 256, njobs);
  B2P_CHECK_CUDA(launch_pdl(lora_wgrad_reduce_kernel, g2, dim3(256), 0, st, d_jobs, rank, part, max_cols, scale));
  B2P_POST_LAUNCH();
  return B2P_OK;
}

// ---------------------------------------------------------------------------
// per-step transposed adapter operands for the backward GEMMs
//   bblk_qkv[l]: [64][q+2kv] 16-bit, row 16p+j = B_p[:, j]^T over part p's columns
//   bblk_o[l]:   [64][D],    row j = B_o[:, j]^T
//   a_oT[l]:     [q][rank] fp32, A_o^T (LoRA-up operand of the Wo data gradient)
// ---------------------------------------------------------------------------
struct LoraTArgs {
  const float* theta;
  long long layer_size, oBq, oBk, oBv, oBo, oAo, oAq, oAk, oAv;
  int L, D, QD, KVD, rank;
  void* bblk_qkv;
  void* bblk_o;
  float* a_oT;
  void* wqkvT;   // [L][D][ldw]: columns QKV + 16p + j receive A_p[j, :] (the LoRA K-extension)
  int ldw;
};

template <typename T>
__global__ void lora_t_kernel(LoraTArgs a) {
  const int QKV = a.QD + 2 * a.KVD;
  const long long per_layer = (long long)QKV * a.rank + (long long)a.D * a.rank + (long long)a.QD * a.rank +
                              3LL * a.rank * a.D;
  const long long n = per_layer * a.L;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int l = (int)(i / per_layer);
    long long k = i - (long long)l * per_layer;
    const float* th = a.theta + (long long)l * a.layer_size;
    if (k < (long long)QKV * a.rank) {
      const int col = (int)(k / a.rank), j = (int)(k % a.rank);
      float v;
      int seg;
      if (col < a.QD) { seg = 0; v = th[a.oBq + (long long)col * a.rank + j]; }
      else if (col < a.QD + a.KVD) { seg = 1; v = th[a.oBk + (long long)(col - a.QD) * a.rank + j]; }
      else { seg = 2; v = th[a.oBv + (long long)(col - a.QD - a.KVD) * a.rank + j]; }
      static_cast<T*>(a.bblk_qkv)[((long long)l * 64 + 16 * seg + j) * QKV + col] = static_cast<T>(v);
      continue;
    }
    k -= (long long)QKV * a.rank;
    if (k < (long long)a.D * a.rank) {
      const int col = (int)(k / a.rank), j = (int)(k % a.rank);
      static_cast<T*>(a.bblk_o)[((long long)l * 64 + j) * a.D + col] =
          static_cast<T>(th[a.oBo + (long long)col * a.rank + j]);
      continue;
    }
    k -= (long long)a.D * a.rank;
    if (k < (long long)a.QD * a.rank) {
      const int col = (int)(k / a.rank), j = (int)(k % a.rank);
      a.a_oT[((long long)l * a.QD + col) * a.rank + j] = th[a.oAo + (long long)j * a.QD + col];
      continue;
    }
    k -= (long long)a.QD * a.rank;
    // A_q, A_k, A_v rows as extra K columns of W_qkv^T: dX = dQKV·W_qkv + U'·A
    const int p = (int)(k / ((long long)a.rank * a.D));
    const long long rem = k - (long long)p * a.rank * a.D;
    const int j = (int)(rem / a.D), d = (int)(rem % a.D);
    const long long aoff = p == 0 ? a.oAq : (p == 1 ? a.oAk : a.oAv);
    static_cast<T*>(a.wqkvT)[((long long)l * a.D + d) * a.ldw + QKV + 16 * p + j] =
        static_cast<T>(th[aoff + (long long)j * a.D + d]);
  }
}

// ---------------------------------------------------------------------------
// Adam (adam_update, training/cpu_ops.h:62-104) with the reference's operation
// order, every step rounded once as the vectorised calls round:
//   m = fl(fl(g*(1-b1)) + fl(m*b1)); v = fl(fl(fl(g*g)*(1-b2)) + fl(v*b2))
//   u = fl(fl(m*ibc1) / fl(sqrt(fl(v*ibc2)) + eps)); [u = fl(fl(w*wd) + u)]
//   w = fl(fl(u*(-lr)) + w)
// The step is skipped (and the status word set) if any gradient is not finite.
// ---------------------------------------------------------------------------
__global__ void finite_check_kernel(const float* __restrict__ g, long long n, uint32_t* flag) {
  bool bad = false;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    bad |= !isfinite(g[i]);
  if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicOr(flag, 1u);
}

struct AdamArgs {
  float* w;
  const float* g;
  float* m;
  float* v;
  long long n;
  float b1, omb1, b2, omb2, ibc1, ibc2, eps, neg_lr, wd;
  const uint32_t* flag;
  uint32_t* status;
};

__global__ void adam_kernel(AdamArgs a) {
  if (*a.flag) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicCAS(a.status, 0u, (uint32_t)DEV_NONFINITE_GRAD);
    return;
  }
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += (long long)gridDim.x * blockDim.x) {
    const float g = a.g[i];
    const float m = __fadd_rn(__fmul_rn(g, a.omb1), __fmul_rn(a.m[i], a.b1));
    const float v = __fadd_rn(__fmul_rn(__fmul_rn(g, g), a.omb2), __fmul_rn(a.v[i], a.b2));
    a.m[i] = m;
    a.v[i] = v;
    const float mh = __fmul_rn(m, a.ibc1);
    const float vh = __fmul_rn(v, a.ibc2);
    float u = __fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), a.eps));
    if (a.wd > 0.f) u = __fadd_rn(__fmul_rn(a.w[i], a.wd), u);
    a.w[i] = __fadd_rn(__fmul_rn(u, a.neg_lr), a.w[i]);
  }
}

// ---------------------------------------------------------------------------
// causal GQA attention backward (cpu_sdpa_backward, training/cpu_ops.h:213-290,
// with gqa_tile_kv / gqa_reduce_kv, training/io.h:439-459, and
// rope_backward_inplace, cpu_ops.h:377-393), head_dim 64, 64 x 64 tiles on
// mma.sync m16n8k16. P is recomputed from the forward's row normaliser lse
// (log2 domain); D_i = sum_d dO_i,d O_i,d stands for the reference's
// sum_j dP_ij P_ij. dS = P (dP - D) / sqrt(hd).
//   dq kernel:   one CTA per (group, head, query block): dQ = dS K over key blocks <= it
//   dkdv kernel: one CTA per (group, kv head, key block): dV = P^T dO and dK = dS^T Q over
//                the kv head's query heads and the query blocks >= it (GQA reduction in registers)
// dQ and dK leave with the inverse RoPE rotation applied (gradients of the pre-RoPE Q, K).
// ---------------------------------------------------------------------------
constexpr int kAT = 64;   // tile rows (queries or keys)
constexpr int kAHD = 64;  // head_dim
constexpr int kDkdvSmem = 6 * kAT * kAHD * 2 + 4 * kAT * 4;


template <typename T>
__device__ __forceinline__ void ab_load_tile(uint32_t s_base, const T* g, long long ld) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = threadIdx.x + i * 128;  // 512 chunks of 16 B
    const int r = idx >> 3, c = idx & 7;
    cp_async16(s_base + swz(r, c), g + r * ld + c * 8);
  }
}

template <typename T>
__global__ void attn_bwd_prep_kernel(AttnBwdArgs a) {
  pdl_enter();
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long n = (long long)a.ngroups * a.seq * a.heads;
  if (i >= n) return;
  const long long row = i / a.heads;
  const int h = (int)(i - row * a.heads);
  const T* o = static_cast<const T*>(a.o) + row * a.ld_o + h * kAHD;
  const T* d = static_cast<const T*>(a.dout) + row * a.ld_o + h * kAHD;
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < kAHD; c += 8) {
    const uint4 ov = *reinterpret_cast<const uint4*>(o + c);
    const uint4 dv = *reinterpret_cast<const uint4*>(d + c);
    const uint32_t oo[4] = {ov.x, ov.y, ov.z, ov.w}, dd[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 of = H2<T>::to_f2(*reinterpret_cast<const typename H2<T>::V*>(&oo[k]));
      const float2 df = H2<T>::to_f2(*reinterpret_cast<const typename H2<T>::V*>(&dd[k]));
      s += of.x * df.x + of.y * df.y;
    }
  }
  a.dvec[i] = s;
}

// Inverse RoPE on one (2i, 2i+1) pair at position pos, frequency index fi.
__device__ __forceinline__ void rope_bwd_pair(const AttnBwdArgs& a, int pos, int fi, float& d0, float& d1) {
  const float c = __ldg(a.rope_cos + pos * 32 + fi), s = __ldg(a.rope_sin + pos * 32 + fi);
  const float x0 = d0, x1 = d1;
  d0 = x0 * c + x1 * s;
  d1 = -x0 * s + x1 * c;
}

template <typename T>
__global__ void __launch_bounds__(128) attn_bwd_dq_kernel(AttnBwdArgs a) {
  __shared__ __align__(128) uint8_t s_q[kAT * kAHD * 2];
  __shared__ __align__(128) uint8_t s_do[kAT * kAHD * 2];
  __shared__ __align__(128) uint8_t s_k[2][kAT * kAHD * 2];
  __shared__ __align__(128) uint8_t s_v[2][kAT * kAHD * 2];
  const int nqb = a.seq / kAT;
  const int qb = nqb - 1 - blockIdx.x;  // longest rows first
  const int h = blockIdx.y, g = blockIdx.z;
  const int kvh = h / (a.heads / a.kv_heads);
  const long long row_base = (long long)g * a.seq;
  const T* base = static_cast<const T*>(a.qkv) + row_base * a.ld;
  const T* gq = base + (long long)qb * kAT * a.ld + a.q_off + h * kAHD;
  const T* gk = base + a.k_off + kvh * kAHD;
  const T* gv = base + a.v_off + kvh * kAHD;
  const T* gdo = static_cast<const T*>(a.dout) + (row_base + (long long)qb * kAT) * a.ld_o + h * kAHD;
  const uint32_t sq = smem_u32(s_q), sdo = smem_u32(s_do), sk0 = smem_u32(s_k[0]), sv0 = smem_u32(s_v[0]);
  constexpr uint32_t kTileBytes = kAT * kAHD * 2;
  ab_load_tile<T>(sq, gq, a.ld);
  ab_load_tile<T>(sdo, gdo, a.ld_o);
  ab_load_tile<T>(sk0, gk, a.ld);
  ab_load_tile<T>(sv0, gv, a.ld);
  cp_async_commit();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lg = lane >> 2, lt = lane & 3;
  const int lm = lane >> 3, lr = lane & 7;
  const int q0 = warp * 16 + lg;  // query row in the tile (second row +8)
  float lse2[2], dvr[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const long long row = row_base + (long long)qb * kAT + q0 + 8 * i;
    lse2[i] = a.lse[row * a.heads + h];
    dvr[i] = a.dvec[row * a.heads + h];
  }
  float dq[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
  uint32_t qf[4][4], df[4][4];

  for (int kb = 0; kb <= qb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 <= qb) {
      ab_load_tile<T>(sk0 + (buf ^ 1) * kTileBytes, gk + (long long)(kb + 1) * kAT * a.ld, a.ld);
      ab_load_tile<T>(sv0 + (buf ^ 1) * kTileBytes, gv + (long long)(kb + 1) * kAT * a.ld, a.ld);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        ldsm_x4(sq + swz(warp * 16 + (lm & 1) * 8 + lr, kk * 2 + (lm >> 1)), qf[kk][0], qf[kk][1], qf[kk][2],
                qf[kk][3]);
        ldsm_x4(sdo + swz(warp * 16 + (lm & 1) * 8 + lr, kk * 2 + (lm >> 1)), df[kk][0], df[kk][1], df[kk][2],
                df[kk][3]);
      }
    }
    const uint32_t skb = sk0 + buf * kTileBytes, svb = sv0 + buf * kTileBytes;
    float s[8][4], dp[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
      dp[i][0] = dp[i][1] = dp[i][2] = dp[i][3] = 0.f;
    }
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(skb + swz(nt * 16 + (lm >> 1) * 8 + lr, kk * 2 + (lm & 1)), b0, b1, b2, b3);
        mma16816<T>(s[2 * nt], qf[kk], b0, b1);
        mma16816<T>(s[2 * nt + 1], qf[kk], b2, b3);
        ldsm_x4(svb + swz(nt * 16 + (lm >> 1) * 8 + lr, kk * 2 + (lm & 1)), b0, b1, b2, b3);
        mma16816<T>(dp[2 * nt], df[kk], b0, b1);
        mma16816<T>(dp[2 * nt + 1], df[kk], b2, b3);
      }
    }
    // P and dS = P (dP - D) * scale
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = nt * 8 + 2 * lt + (e & 1);
        const int qr = q0 + ((e >> 1) << 3);
        float p = exp2f(s[nt][e] * a.scale_log2 - lse2[e >> 1]);
        if (kb == qb && key > qr) p = 0.f;
        s[nt][e] = p * (dp[nt][e] - dvr[e >> 1]) * a.scale;
      }
    // dQ += dS K
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
        ldsm_x4_t(skb + swz(kc * 16 + (lm & 1) * 8 + lr, dt * 2 + (lm >> 1)), b0, b1, b2, b3);
        mma16816<T>(dq[2 * dt], pa, b0, b1);
        mma16816<T>(dq[2 * dt + 1], pa, b2, b3);
      }
    }
    __syncthreads();
  }
  // inverse RoPE on the (2i, 2i+1) pairs each thread holds, then store
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int pos = qb * kAT + q0 + 8 * half;
    T* out = static_cast<T*>(a.dqkv) + (row_base + pos) * a.ld_d + a.q_off + h * kAHD;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float d0 = dq[nt][2 * half], d1 = dq[nt][2 * half + 1];
      rope_bwd_pair(a, pos, nt * 4 + lt, d0, d1);
      *reinterpret_cast<uint32_t*>(out + nt * 8 + 2 * lt) = pack_h2<T>(d0, d1);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(128) attn_bwd_dkdv_kernel(AttnBwdArgs a) {
  // dynamic shared memory: K, V, Q[2], dO[2] tiles (8 KB each), then lse[2][64], D[2][64]
  extern __shared__ __align__(128) uint8_t ab_smem[];
  uint8_t* s_k = ab_smem;
  uint8_t* s_v = ab_smem + kAT * kAHD * 2;
  uint8_t(*s_q)[kAT * kAHD * 2] = reinterpret_cast<uint8_t(*)[kAT * kAHD * 2]>(ab_smem + 2 * kAT * kAHD * 2);
  uint8_t(*s_do)[kAT * kAHD * 2] = reinterpret_cast<uint8_t(*)[kAT * kAHD * 2]>(ab_smem + 4 * kAT * kAHD * 2);
  float(*s_lse)[kAT] = reinterpret_cast<float(*)[kAT]>(ab_smem + 6 * kAT * kAHD * 2);
  float(*s_dv)[kAT] = reinterpret_cast<float(*)[kAT]>(ab_smem + 6 * kAT * kAHD * 2 + 2 * kAT * 4);
  const int nqb = a.seq / kAT;
  const int kb = blockIdx.x;  // small kb = most query blocks: launched first
  const int kvh = blockIdx.y, g = blockIdx.z;
  const int ratio = a.heads / a.kv_heads;
  const long long row_base = (long long)g * a.seq;
  const T* base = static_cast<const T*>(a.qkv) + row_base * a.ld;
  const T* gk = base + (long long)kb * kAT * a.ld + a.k_off + kvh * kAHD;
  const T* gv = base + (long long)kb * kAT * a.ld + a.v_off + kvh * kAHD;
  const uint32_t sk = smem_u32(s_k), sv = smem_u32(s_v), sq0 = smem_u32(s_q[0]), sdo0 = smem_u32(s_do[0]);
  constexpr uint32_t kTileBytes = kAT * kAHD * 2;
  const int nq = nqb - kb;          // query blocks per head
  const int iters = ratio * nq;
  // iteration it: head kvh*ratio + it / nq, query block kb + it % nq
  auto issue = [&](int it, int buf) {
    const int h = kvh * ratio + it / nq, qb = kb + it % nq;
    ab_load_tile<T>(sq0 + buf * kTileBytes, base + (long long)qb * kAT * a.ld + a.q_off + h * kAHD, a.ld);
    ab_load_tile<T>(sdo0 + buf * kTileBytes,
                    static_cast<const T*>(a.dout) + (row_base + (long long)qb * kAT) * a.ld_o + h * kAHD, a.ld_o);
    if (threadIdx.x < kAT) {
      const long long row = row_base + (long long)qb * kAT + threadIdx.x;
      s_lse[buf][threadIdx.x] = a.lse[row * a.heads + h];
      s_dv[buf][threadIdx.x] = a.dvec[row * a.heads + h];
    }
  };
  ab_load_tile<T>(sk, gk, a.ld);
  ab_load_tile<T>(sv, gv, a.ld);
  issue(0, 0);
  cp_async_commit();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lg = lane >> 2, lt = lane & 3;
  const int lm = lane >> 3, lr = lane & 7;
  const int k0 = warp * 16 + lg;  // key row in the tile (second row +8)
  float dk[8][4], dv[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    dk[i][0] = dk[i][1] = dk[i][2] = dk[i][3] = 0.f;
    dv[i][0] = dv[i][1] = dv[i][2] = dv[i][3] = 0.f;
  }
  uint32_t kf[4][4], vf[4][4];

  for (int it = 0; it < iters; ++it) {
    const int buf = it & 1;
    if (it + 1 < iters) {
      issue(it + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (it == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        ldsm_x4(sk + swz(warp * 16 + (lm & 1) * 8 + lr, kk * 2 + (lm >> 1)), kf[kk][0], kf[kk][1], kf[kk][2],
                kf[kk][3]);
        ldsm_x4(sv + swz(warp * 16 + (lm & 1) * 8 + lr, kk * 2 + (lm >> 1)), vf[kk][0], vf[kk][1], vf[kk][2],
                vf[kk][3]);
      }
    }
    const bool diag = (it % nq) == 0;  // query block == key block
    const uint32_t sqb = sq0 + buf * kTileBytes, sdob = sdo0 + buf * kTileBytes;
    // S^T = K Q^T and dP^T = V dO^T (16 keys x 64 queries per warp)
    float st[8][4], dpt[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      st[i][0] = st[i][1] = st[i][2] = st[i][3] = 0.f;
      dpt[i][0] = dpt[i][1] = dpt[i][2] = dpt[i][3] = 0.f;
    }
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sqb + swz(nt * 16 + (lm >> 1) * 8 + lr, kk * 2 + (lm & 1)), b0, b1, b2, b3);
        mma16816<T>(st[2 * nt], kf[kk], b0, b1);
        mma16816<T>(st[2 * nt + 1], kf[kk], b2, b3);
        ldsm_x4(sdob + swz(nt * 16 + (lm >> 1) * 8 + lr, kk * 2 + (lm & 1)), b0, b1, b2, b3);
        mma16816<T>(dpt[2 * nt], vf[kk], b0, b1);
        mma16816<T>(dpt[2 * nt + 1], vf[kk], b2, b3);
      }
    }
    // P^T (causal on the diagonal block) and dS^T = P^T (dP^T - D) * scale
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int q = nt * 8 + 2 * lt + (e & 1);
        const int key = k0 + ((e >> 1) << 3);
        float p = exp2f(st[nt][e] * a.scale_log2 - s_lse[buf][q]);
        if (diag && key > q) p = 0.f;
        st[nt][e] = p;
        dpt[nt][e] = p * (dpt[nt][e] - s_dv[buf][q]) * a.scale;
      }
    // dV += P^T dO ; dK += dS^T Q
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      uint32_t pa[4], sa[4];
      pa[0] = pack_h2<T>(st[2 * kc][0], st[2 * kc][1]);
      pa[1] = pack_h2<T>(st[2 * kc][2], st[2 * kc][3]);
      pa[2] = pack_h2<T>(st[2 * kc + 1][0], st[2 * kc + 1][1]);
      pa[3] = pack_h2<T>(st[2 * kc + 1][2], st[2 * kc + 1][3]);
      sa[0] = pack_h2<T>(dpt[2 * kc][0], dpt[2 * kc][1]);
      sa[1] = pack_h2<T>(dpt[2 * kc][2], dpt[2 * kc][3]);
      sa[2] = pack_h2<T>(dpt[2 * kc + 1][0], dpt[2 * kc + 1][1]);
      sa[3] = pack_h2<T>(dpt[2 * kc + 1][2], dpt[2 * kc + 1][3]);
#pragma unroll
      for (int dt = 0; dt < 4; ++dt) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(sdob + swz(kc * 16 + (lm & 1) * 8 + lr, dt * 2 + (lm >> 1)), b0, b1, b2, b3);
        mma16816<T>(dv[2 * dt], pa, b0, b1);
        mma16816<T>(dv[2 * dt + 1], pa, b2, b3);
        ldsm_x4_t(sqb + swz(kc * 16 + (lm & 1) * 8 + lr, dt * 2 + (lm >> 1)), b0, b1, b2, b3);
        mma16816<T>(dk[2 * dt], sa, b0, b1);
        mma16816<T>(dk[2 * dt + 1], sa, b2, b3);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int pos = kb * kAT + k0 + 8 * half;
    T* ok = static_cast<T*>(a.dqkv) + (row_base + pos) * a.ld_d + a.k_off + kvh * kAHD;
    T* ov = static_cast<T*>(a.dqkv) + (row_base + pos) * a.ld_d + a.v_off + kvh * kAHD;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float d0 = dk[nt][2 * half], d1 = dk[nt][2 * half + 1];
      rope_bwd_pair(a, pos, nt * 4 + lt, d0, d1);
      *reinterpret_cast<uint32_t*>(ok + nt * 8 + 2 * lt) = pack_h2<T>(d0, d1);
      *reinterpret_cast<uint32_t*>(ov + nt * 8 + 2 * lt) = pack_h2<T>(dv[nt][2 * half], dv[nt][2 * half + 1]);
    }
  }
}

int attention_backward(const AttnBwdArgs& a0, bool bf16, bool use_tc, cudaStream_t st) {
  AttnBwdArgs a = a0;
  B2P_REQUIRE(a.seq % kAT == 0, "attention backward needs seq %% 64 == 0 (got %d)", a.seq);
  B2P_REQUIRE(a.kv_heads > 0 && a.heads % a.kv_heads == 0, "heads must be a multiple of kv_heads");
  B2P_REQUIRE(a.ld % 8 == 0 && a.ld_d % 2 == 0 && a.q_off % 8 == 0 && a.k_off % 8 == 0 && a.v_off % 8 == 0 &&
                  a.ld_o % 8 == 0,
              "attention operands must be 16-byte aligned");
  a.scale = 1.0f / sqrtf((float)kAHD);
  a.scale_log2 = a.scale * 1.4426950408889634f;
  const long long n = (long long)a.ngroups * a.seq * a.heads;
  const int pb = (int)((n + 255) / 256);
  dim3 gq(a.seq / kAT, a.heads, a.ngroups), gk(a.seq / kAT, a.kv_heads, a.ngroups);
  if (use_tc && attention_backward_tc_supported(a)) {  // D first, then dK|dV and dQ on tcgen05
    if (bf16)
      B2P_CHECK_CUDA(launch_pdl(attn_bwd_prep_kernel<__nv_bfloat16>, dim3(pb), dim3(256), 0, st, a));
    else
      B2P_CHECK_CUDA(launch_pdl(attn_bwd_prep_kernel<__half>, dim3(pb), dim3(256), 0, st, a));
    B2P_POST_LAUNCH();
    return launch_attention_backward_tc(a, bf16, st);
  }
  if (bf16) {
    B2P_CHECK_CUDA(cudaFuncSetAttribute(attn_bwd_dkdv_kernel<__nv_bfloat16>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, kDkdvSmem));
    attn_bwd_prep_kernel<__nv_bfloat16><<<pb, 256, 0, st>>>(a);
    B2P_POST_LAUNCH();
    attn_bwd_dkdv_kernel<__nv_bfloat16><<<gk, 128, kDkdvSmem, st>>>(a);
    B2P_POST_LAUNCH();
    attn_bwd_dq_kernel<__nv_bfloat16><<<gq, 128, 0, st>>>(a);
  } else {
    B2P_CHECK_CUDA(cudaFuncSetAttribute(attn_bwd_dkdv_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kDkdvSmem));
    attn_bwd_prep_kernel<__half><<<pb, 256, 0, st>>>(a);
    B2P_POST_LAUNCH();
    attn_bwd_dkdv_kernel<__half><<<gk, 128, kDkdvSmem, st>>>(a);
    B2P_POST_LAUNCH();
    attn_bwd_dq_kernel<__half><<<gq, 128, 0, st>>>(a);
  }
  B2P_POST_LAUNCH();
  return B2P_OK;
}

// ---------------------------------------------------------------------------
// state: transposed frozen weights (per upload), row buffers (per batch size),
// gradients and Adam moments (per model)
// ---------------------------------------------------------------------------
#define P16_ALLOC(ptr, bytes)                                                  \
  do {                                                                         \
    B2P_CHECK_CUDA(cudaMalloc(reinterpret_cast<void**>(&(ptr)), (bytes)));     \
  } while (0)

int ensure_model_state(b2p_model* m) {
  if (m->p16) return B2P_OK;
  // bp_lora_backward (backprop_lora.h:147-288) has no FFN-adapter gradients
  B2P_REQUIRE(!m->ffn, "backprop-LoRA and full backprop are not defined for --lora-ffn models");
  const auto& c = m->cfg;
  const size_t L = c.nlayers, D = c.dim, H = c.hidden, QD = m->q_dim, QKV = m->qkv_dim, r = c.rank;
  const size_t e = model_esz(m);
  P16State* s = new P16State();
  m->p16 = s;
  P16_ALLOC(s->wqkvT, L * D * (QKV + kUCols) * e);
  B2P_CHECK_CUDA(cudaMemset(s->wqkvT, 0, L * D * (QKV + kUCols) * e));
  P16_ALLOC(s->woT, L * QD * D * e);
  P16_ALLOC(s->a_oT, L * QD * r * 4);
  P16_ALLOC(s->bblk_qkv, L * 64 * QKV * e);
  P16_ALLOC(s->bblk_o, L * 64 * D * e);
  B2P_CHECK_CUDA(cudaMemset(s->bblk_qkv, 0, L * 64 * QKV * e));
  B2P_CHECK_CUDA(cudaMemset(s->bblk_o, 0, L * 64 * D * e));
  P16_ALLOC(s->grad, (size_t)m->P * 4);
  P16_ALLOC(s->adam_m, (size_t)m->P * 4);
  P16_ALLOC(s->adam_v, (size_t)m->P * 4);
  B2P_CHECK_CUDA(cudaMemset(s->grad, 0, (size_t)m->P * 4));
  B2P_CHECK_CUDA(cudaMemset(s->adam_m, 0, (size_t)m->P * 4));
  B2P_CHECK_CUDA(cudaMemset(s->adam_v, 0, (size_t)m->P * 4));
  P16_ALLOC(s->flag, 4);
  P16_ALLOC(s->d_jobs, L * kMaxWgradJobs * sizeof(WgradJob));
  std::vector<int> off(2 * L + 1);
  for (size_t l = 0; l < L; ++l) {
    off[2 * l] = (int)(l * m->layer_size + m->oRa);
    off[2 * l + 1] = (int)(l * m->layer_size + m->oRf);
  }
  off[2 * L] = (int)m->oRfinal;
  P16_ALLOC(s->d_rms_off, off.size() * sizeof(int));
  B2P_CHECK_CUDA(cudaMemcpy(s->d_rms_off, off.data(), off.size() * sizeof(int), cudaMemcpyHostToDevice));
  return B2P_OK;
}

// Transposed copies of the frozen weights for the data-gradient GEMMs that read them K-major: Wqkv
// (with the LoRA K-extension columns) and Wo, whose GEMMs carry LoRA terms. W1|W3, W2 and the compact
// embedding are read where they lie, MN-major, on the CTA-pair engine; their transposed copies are
// built only for steps that cannot use it (ensure_weights_kmajor).
int ensure_weights(b2p_model* m) {
  P16State* s = m->p16;
  if (s->weights_version == m->weights_version) return B2P_OK;
  const auto& c = m->cfg;
  const int L = c.nlayers, D = c.dim, QD = m->q_dim, QKV = m->qkv_dim;
  const size_t e = model_esz(m);
  const int cv_pad = (m->cv + 63) / 64 * 64;
  if (cv_pad != s->cv_pad) {
    s->cv_pad = cv_pad;
    s->gen++;
    release_rows(s);  // dlogits rows depend on the padded vocabulary
  }
  int rc;
  const bool bf = m->bf16;
  for (int l = 0; l < L; ++l) {
    const char* wqkv = static_cast<const char*>(m->wqkv) + (size_t)l * QKV * D * e;
    const char* wo = static_cast<const char*>(m->wo) + (size_t)l * D * QD * e;
    if ((rc = transpose16(wqkv, QKV, D, D, static_cast<char*>(s->wqkvT) + (size_t)l * D * (QKV + kUCols) * e,
                          QKV + kUCols, bf, m->st)))
      return rc;
    if ((rc = transpose16(wo, D, QD, QD, static_cast<char*>(s->woT) + (size_t)l * QD * D * e, D, bf, m->st)))
      return rc;
  }
  s->weights_version = m->weights_version;
  return B2P_OK;
}

// K-major (transposed) copies of W1|W3, W2 and the compact embedding, for steps on the single-CTA
// engine (fewer than 256 token rows, or B2P_OPT_PAIR_GEMM 0).
int ensure_weights_kmajor(b2p_model* m) {
  P16State* s = m->p16;
  if (s->kmajor_version == m->weights_version && s->cembedT_pad == s->cv_pad) return B2P_OK;
  const auto& c = m->cfg;
  const int L = c.nlayers, D = c.dim, H = c.hidden;
  const size_t e = model_esz(m);
  if (!s->w13T) P16_ALLOC(s->w13T, (size_t)L * D * 2 * H * e);
  if (!s->w2T) P16_ALLOC(s->w2T, (size_t)L * H * D * e);
  if (s->cembedT_pad != s->cv_pad) {
    if (s->cembedT) cudaFree(s->cembedT);
    s->cembedT = nullptr;
    P16_ALLOC(s->cembedT, (size_t)D * s->cv_pad * e);
    s->cembedT_pad = s->cv_pad;
  }
  B2P_CHECK_CUDA(cudaMemsetAsync(s->cembedT, 0, (size_t)D * s->cv_pad * e, m->st));
  int rc;
  const bool bf = m->bf16;
  for (int l = 0; l < L; ++l) {
    const char* w13 = static_cast<const char*>(m->w13) + (size_t)l * 2 * H * D * e;
    const char* w2 = static_cast<const char*>(m->w2) + (size_t)l * D * H * e;
    if ((rc = transpose16(w13, 2 * H, D, D, static_cast<char*>(s->w13T) + (size_t)l * D * 2 * H * e, 2 * H, bf,
                          m->st)))
      return rc;
    if ((rc = transpose16(w2, D, H, H, static_cast<char*>(s->w2T) + (size_t)l * H * D * e, D, bf, m->st)))
      return rc;
  }
  if ((rc = transpose16(m->cembed, m->cv, D, D, s->cembedT, s->cv_pad, bf, m->st))) return rc;
  s->kmajor_version = m->weights_version;
  return B2P_OK;
}

int ensure_rows(b2p_model* m, int R) {
  P16State* s = m->p16;
  if (s->rows == R) return B2P_OK;
  release_rows(s);
  s->gen++;
  const auto& c = m->cfg;
  const size_t L = c.nlayers, D = c.dim, H = c.hidden, QD = m->q_dim, KVD = m->kv_dim, QKV = m->qkv_dim;
  const size_t e = model_esz(m), Rz = R, heads = c.heads;
  ForwardSaves& v = s->sv;
  P16_ALLOC(v.x_in, L * Rz * D * 4);
  P16_ALLOC(v.x_mid, L * Rz * D * 4);
  P16_ALLOC(v.xn, L * Rz * D * e);
  P16_ALLOC(v.U, L * Rz * kUCols * e);
  B2P_CHECK_CUDA(cudaMemset(v.U, 0, L * Rz * kUCols * e));
  P16_ALLOC(v.qkv, L * Rz * QKV * e);
  P16_ALLOC(v.attn, L * Rz * QD * e);
  P16_ALLOC(v.lse, L * Rz * heads * 4);
  P16_ALLOC(v.h13, L * Rz * 2 * H * e);
  P16_ALLOC(v.x_final, Rz * D * 4);
  P16_ALLOC(v.xn_final, Rz * D * e);
  P16_ALLOC(v.row_lse, Rz * 4);
  P16_ALLOC(s->dlogits, Rz * s->cv_pad * e);
  B2P_CHECK_CUDA(cudaMemset(s->dlogits, 0, Rz * s->cv_pad * e));
  P16_ALLOC(s->dy, Rz * D * 4);
  P16_ALLOC(s->dy2, Rz * D * 4);
  P16_ALLOC(s->dxf, Rz * D * 4);
  P16_ALLOC(s->dsilu, Rz * H * 4);
  P16_ALLOC(s->d16, Rz * D * e);
  P16_ALLOC(s->dh13, Rz * 2 * H * e);
  P16_ALLOC(s->da, Rz * QD * e);
  P16_ALLOC(s->dqkv, Rz * (QKV + kUCols) * e);
  B2P_CHECK_CUDA(cudaMemset(s->dqkv, 0, Rz * (QKV + kUCols) * e));
  P16_ALLOC(s->ub_o, Rz * kUCols * e);
  B2P_CHECK_CUDA(cudaMemset(s->ub_o, 0, Rz * kUCols * e));
  P16_ALLOC(s->dvec, Rz * heads * 4);
  const size_t nblk = rms_blocks(R);
  P16_ALLOC(s->rms_part, (2 * L + 1) * nblk * D * 4);
  P16_ALLOC(s->wgrad_part, (size_t)kMaxWgradJobs * kWgradSplit * std::max(D, QD) * kWgPartJ * 4);
  if (s->full) {
    const size_t rows_t = std::max<size_t>(std::max<size_t>(QKV, 2 * H), (size_t)s->cv_pad);
    P16_ALLOC(s->tA, rows_t * Rz * e);
    P16_ALLOC(s->tB, std::max(std::max(D, H), QD) * Rz * e);
    P16_ALLOC(s->gate, Rz * H * e);
    P16_ALLOC(v.xn2, L * Rz * D * e);
    P16_ALLOC(s->d_seg, (2 * Rz + 2) * sizeof(int32_t));
  }
  s->rows = R;
  // weight-gradient jobs of every layer (fixed once the buffers are)
  std::vector<WgradJob> jobs(L * kMaxWgradJobs);
  auto at = [&](void* base, size_t l, size_t row_elems) -> const void* {
    return static_cast<const char*>(base) + l * Rz * row_elems * e;
  };
  for (size_t l = 0; l < L; ++l) {
    const long long lb = (long long)l * m->layer_size;
    float* g = s->grad + lb;
    const void* Ul = at(v.U, l, kUCols);
    const void* xnl = at(v.xn, l, D);
    const char* dq = static_cast<const char*>(s->dqkv);
    const long long ldq = QKV + kUCols;
    const void* up = dq + QKV * e;  // U'_{q,k,v} = dQKV · B, columns QKV.. of dqkv
    WgradJob* j = &jobs[l * kMaxWgradJobs];
    j[0] = {s->d16, (long long)D, (int)D, 48, Ul, kUCols, {g + m->oBo, nullptr, nullptr}, 1, 0};  // dB_o
    j[1] = {at(v.attn, l, QD), (long long)QD, (int)QD, 0, s->ub_o, kUCols, {g + m->oAo, nullptr, nullptr}, 1,
            1};                                                                                       // dA_o
    j[2] = {dq, ldq, (int)QD, 0, Ul, kUCols, {g + m->oBq, nullptr, nullptr}, 1, 0};                  // dB_q
    j[3] = {dq + QD * e, ldq, (int)KVD, 16, Ul, kUCols, {g + m->oBk, nullptr, nullptr}, 1, 0};       // dB_k
    j[4] = {dq + (QD + KVD) * e, ldq, (int)KVD, 32, Ul, kUCols, {g + m->oBv, nullptr, nullptr}, 1, 0};  // dB_v
    // dA_q, dA_k, dA_v share X = xn: one pass over it with the three U' segments
    j[5] = {xnl, (long long)D, (int)D, 0, up, ldq, {g + m->oAq, g + m->oAk, g + m->oAv}, 3, 1};
  }
  B2P_CHECK_CUDA(cudaMemcpy(s->d_jobs, jobs.data(), jobs.size() * sizeof(WgradJob), cudaMemcpyHostToDevice));
  return B2P_OK;
}

// Forward with saves + cross-entropy + backward; gradients (theta layout) in s->grad,
// the mean loss in m->var_loss[0]. Tokens/targets already staged at d_tok / d_tgt.
// ---------------------------------------------------------------------------
// full-backprop helpers (train.m)
// ---------------------------------------------------------------------------
// g_embed[tok, :] += scale * (sum of the dx rows of the token, in sequence order)
// (embed_backward, training/cpu_ops.h:199-207), one block per distinct token.
__global__ void embed_scatter_kernel(const float* __restrict__ dx, int D, const int32_t* __restrict__ seg, int rows,
                                     const int32_t* __restrict__ tokens, float* __restrict__ g_embed, float scale) {
  // seg[0] = number of segments, seg[1 .. rows + 1] their starts, seg[rows + 2 ..] the row order
  const int sgi = blockIdx.x;
  if (sgi >= seg[0]) return;
  const int32_t* order = seg + rows + 2;
  const int b = seg[1 + sgi], e = seg[2 + sgi];
  const int tok = tokens[order[b]];
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float acc = 0.f;
    for (int i = b; i < e; ++i) acc += dx[(long long)order[i] * D + c];
    g_embed[(long long)tok * D + c] += acc * scale;
  }
}

// g_embed[c2f[v], :] += g_cembed[v, :]  (vocab_scatter_grads, training/cpu_ops.h:176-182)
__global__ void cembed_scatter_kernel(const float* __restrict__ g_cembed, const int32_t* __restrict__ c2f, int cv,
                                      int D, float* __restrict__ g_embed) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)cv * D) return;
  const int v = (int)(i / D), c = (int)(i - (long long)v * D);
  g_embed[(long long)c2f[v] * D + c] += g_cembed[i];
}

// squared-norm partials over segments (offset, length) of one buffer
constexpr int kNormBlocks = 296;

__global__ void sqnorm_kernel(const float* __restrict__ base, const long long* seg_off, const long long* seg_len,
                              int nseg, float* __restrict__ part) {
  __shared__ float red[256];
  float acc = 0.f;
  for (int sg = 0; sg < nseg; ++sg)
    for (long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x; j < seg_len[sg];
         j += (long long)gridDim.x * blockDim.x) {
      const float g = base[seg_off[sg] + j];
      acc += g * g;
    }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int st = blockDim.x / 2; st > 0; st >>= 1) {
    if (threadIdx.x < st) red[threadIdx.x] += red[threadIdx.x + st];
    __syncthreads();
  }
  if (threadIdx.x == 0) part[blockIdx.x] = red[0];
}

// norm = sqrt(sum of partials in block order); scale = clip / norm if clip > 0 and norm > clip,
// else 1 (train.m:1344-1401); a non-finite norm sets *flag, which turns the optimizer step off
__global__ void clip_scale_kernel(float* part, int nblk, float clip, uint32_t* flag, uint32_t* status) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  float s = 0.f;
  for (int i = 0; i < nblk; ++i) s += part[i];
  const float norm = sqrtf(s);
  part[nblk] = norm;
  part[nblk + 1] = (clip > 0.f && norm > clip) ? clip / norm : 1.0f;
  if (!isfinite(norm)) {
    *flag = 1u;
    atomicCAS(status, 0u, (uint32_t)DEV_NONFINITE_GRAD);
  }
}

template <typename T>
__global__ void f16_to_f32_kernel(const T* __restrict__ src, float* __restrict__ dst, long long n) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    dst[i] = static_cast<float>(src[i]);
}

// Adam over segments (offset, length) of one parameter/gradient/moment layout, gradients first
// multiplied by *gscale (the clip factor; the reference scales the gradients in place first)
struct AdamSegArgs {
  float* w;
  const float* g;
  float* m;
  float* v;
  const long long* seg_off;
  const long long* seg_len;
  int nseg;
  const float* gscale;
  float b1, omb1, b2, omb2, ibc1, ibc2, eps, neg_lr, wd;
  const uint32_t* flag;
};

__global__ void adam_seg_kernel(AdamSegArgs a) {
  if (*a.flag) return;
  const float gs = a.gscale ? *a.gscale : 1.0f;
  for (int sg = 0; sg < a.nseg; ++sg) {
    const long long off = a.seg_off[sg], len = a.seg_len[sg];
    for (long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x; j < len; j += (long long)gridDim.x * blockDim.x) {
      const long long i = off + j;
      const float g = a.gscale ? __fmul_rn(a.g[i], gs) : a.g[i];
      const float m = __fadd_rn(__fmul_rn(g, a.omb1), __fmul_rn(a.m[i], a.b1));
      const float v = __fadd_rn(__fmul_rn(__fmul_rn(g, g), a.omb2), __fmul_rn(a.v[i], a.b2));
      a.m[i] = m;
      a.v[i] = v;
      const float mh = __fmul_rn(m, a.ibc1);
      const float vh = __fmul_rn(v, a.ibc2);
      float u = __fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), a.eps));
      if (a.wd > 0.f) u = __fadd_rn(__fmul_rn(a.w[i], a.wd), u);
      a.w[i] = __fadd_rn(__fmul_rn(u, a.neg_lr), a.w[i]);
    }
  }
}

// 16-bit compact tied embedding from the fp32 full embedding (vocab_compact_embed, cpu_ops.h:171-176)
template <typename T>
__global__ void cembed_refresh_kernel(const float* __restrict__ embed, const int32_t* __restrict__ c2f, int cv, int D,
                                      T* __restrict__ cembed) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)cv * D) return;
  const int v = (int)(i / D), c = (int)(i - (long long)v * D);
  cembed[i] = static_cast<T>(embed[(long long)c2f[v] * D + c]);
}

int p16_kernels(b2p_model* m, const int32_t* d_tok, int n_seq);

int p16_grad(b2p_model* m, const int32_t* d_tok, const int32_t* d_tgt, int n_seq) {
  int rc;
  if ((rc = model_ready(m))) return rc;
  const auto& c = m->cfg;
  const int R = n_seq * c.seq;
  B2P_REQUIRE(c.rank == 4 || c.rank == 8, "backprop-LoRA needs rank 4 or 8");
  if ((rc = ensure_model_state(m))) return rc;
  P16State* s = m->p16;
  if ((rc = ensure_weights(m))) return rc;
  if ((rc = ensure_rows(m, R))) return rc;
  s->use_mn = m->use_pair && R >= 2 * kBM;
  if (!s->use_mn && (rc = ensure_weights_kmajor(m))) return rc;
  // group/variant tables and per-row targets (host-staged, outside any graph)
  std::vector<VariantInfo> vars(1, VariantInfo{0, 0, 0.f, 0.f});
  if ((rc = model_stage_groups(m, n_seq, vars, d_tgt))) return rc;
  if (!m->graphs) return p16_kernels(m, d_tok, n_seq);
  // the graph reads tokens from the model's own buffer, so any caller buffer can feed a replay
  if (d_tok != m->d_tok) {
    B2P_CHECK_CUDA(cudaMemcpyAsync(m->d_tok, d_tok, (size_t)n_seq * c.seq * sizeof(int32_t),
                                   cudaMemcpyDeviceToDevice, m->st));
    d_tok = m->d_tok;
  }
  // With profiling on, the graph also holds the per-GEMM event records; a replay
  // re-records them, so b2p_model_profile_read reports the latest step.
  P16State::Graph& gr = s->graph;
  const bool hit = gr.exec && gr.tok == d_tok && gr.n_seq == n_seq && gr.gen == s->gen &&
                   gr.scale_log2 == m->grad_scale_log2 && gr.pair == m->use_pair && gr.tc_attn == m->tc_attn &&
                   gr.tc_attn_bwd == m->tc_attn_bwd && gr.pdl == pdl_enabled() &&
                   gr.prof_epoch == m->prof_epoch;
  if (!hit) {
    if (gr.exec) cudaGraphExecDestroy(gr.exec);
    gr.exec = nullptr;
    const long long n0 = launch_count();
    B2P_CHECK_CUDA(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeRelaxed));
    rc = p16_kernels(m, d_tok, n_seq);
    cudaGraph_t g = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(m->st, &g);
    const long long captured = launch_count() - n0;
    count_launches(-captured);  // recorded, not run: counted on every replay instead
    if (rc || ce != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      cudaGetLastError();
      if (!rc) set_error("graph capture of the backprop-LoRA step failed: %s", cudaGetErrorString(ce));
      return rc ? rc : B2P_ERR_CUDA;
    }
    const cudaError_t ie = cudaGraphInstantiate(&gr.exec, g, 0);
    cudaGraphDestroy(g);
    if (ie != cudaSuccess) {
      gr.exec = nullptr;
      set_error("cudaGraphInstantiate failed: %s", cudaGetErrorString(ie));
      return B2P_ERR_CUDA;
    }
    gr.tok = d_tok;
    gr.n_seq = n_seq;
    gr.gen = s->gen;
    gr.scale_log2 = m->grad_scale_log2;
    gr.pair = m->use_pair;
    gr.tc_attn = m->tc_attn;
    gr.tc_attn_bwd = m->tc_attn_bwd;
    gr.pdl = pdl_enabled();
    gr.prof_epoch = m->prof_epoch;
    gr.launches = captured;
  }
  B2P_CHECK_CUDA(cudaGraphLaunch(gr.exec, m->st));
  count_launches(gr.launches);
  return B2P_OK;
}

// Every device operation of the backprop-LoRA gradient after the host staging:
// forward with saves, loss, backward, gradient assembly (capturable).
int p16_kernels(b2p_model* m, const int32_t* d_tok, int n_seq) {
  int rc;
  const auto& c = m->cfg;
  const int L = c.nlayers, D = c.dim, H = c.hidden, QD = m->q_dim, KVD = m->kv_dim, QKV = m->qkv_dim;
  const int R = n_seq * c.seq, r = c.rank;
  const size_t e = model_esz(m);
  const bool bf = m->bf16;
  P16State* s = m->p16;
  const ForwardSaves& v = s->sv;
  if ((rc = model_run_forward(m, n_seq, d_tok, &v))) return rc;
  if ((rc = launch_variant_loss(m->group_loss, 1, n_seq, m->var_loss, m->st))) return rc;

  // transposed adapter operands from the current θ
  LoraTArgs lt;
  lt.theta = m->theta;
  lt.layer_size = m->layer_size;
  lt.oBq = m->oBq; lt.oBk = m->oBk; lt.oBv = m->oBv; lt.oBo = m->oBo; lt.oAo = m->oAo;
  lt.oAq = m->oAq; lt.oAk = m->oAk; lt.oAv = m->oAv;
  lt.L = L; lt.D = D; lt.QD = QD; lt.KVD = KVD; lt.rank = r;
  lt.bblk_qkv = s->bblk_qkv;
  lt.bblk_o = s->bblk_o;
  lt.a_oT = s->a_oT;
  lt.wqkvT = s->wqkvT;
  lt.ldw = QKV + kUCols;
  if (bf) lora_t_kernel<__nv_bfloat16><<<148 * 4, 256, 0, m->st>>>(lt);
  else lora_t_kernel<__half><<<148 * 4, 256, 0, m->st>>>(lt);
  B2P_POST_LAUNCH();

  const float gscale_store = ldexpf(1.0f, m->grad_scale_log2);    // dlogits = 2^k (softmax - onehot)
  const float inv_lambda = 1.0f / (gscale_store * (float)R);      // back to d(mean loss)
  const float alpha = c.res_alpha;
  // dlogits (16-bit, recomputed lm-head tile) and dy = dlogits · cembed
  EpiParams eg;
  std::memset(&eg, 0, sizeof(eg));
  eg.M = R;
  eg.N = m->cv;
  eg.alpha = gscale_store;
  eg.targets = m->d_row_tgt;
  eg.row_lse = v.row_lse;
  if ((rc = model_gemm(m, 256, EPI_CE_GRAD, v.xn_final, D, m->cembed, D, R, m->cv, D, s->dlogits, s->cv_pad, nullptr,
                       eg)))
    return rc;
  EpiParams ef;
  std::memset(&ef, 0, sizeof(ef));
  ef.M = R;
  ef.N = D;
  // dy = dlogits · E over the CV real vocabulary columns (E stored [CV][D]: MN-major operand)
  if (s->use_mn) {
    if ((rc = model_gemm_mn(m, EPI_F32, 2, s->dlogits, s->cv_pad, m->cembed, D, R, D, m->cv, s->dxf, D, ef)))
      return rc;
  } else if ((rc = model_gemm(m, pick_bn(D, EPI_F32), EPI_F32, s->dlogits, s->cv_pad, s->cembedT, s->cv_pad, R, D,
                              s->cv_pad, s->dxf, D, nullptr, ef))) {
    return rc;
  }
  // full backprop: dW[out, in] += (1/lambda) * dY^T X over the R token rows, as a GEMM of the
  // transposed 16-bit operands (K = R) accumulated into the fp32 gradient by the reduce-add epilogue
  auto wgrad_gemm = [&](const void* dY, int ld_dy, int n_out, const void* X, int ld_x, int n_in, float* out) -> int {
    int rc2;
    EpiParams ew;
    std::memset(&ew, 0, sizeof(ew));
    ew.M = n_out;
    ew.N = n_in;
    ew.alpha = inv_lambda;
    // dY and X as stored ([R][features]): both MN-major operands, K = R, no transposes
    if (s->use_mn && (rc2 = model_gemm_mn(m, EPI_RESID, 3, dY, ld_dy, X, ld_x, n_out, n_in, R, out, n_in, ew)) !=
                         B2P_ERR_UNSUPPORTED)
      return rc2;
    if ((rc2 = transpose16(dY, R, n_out, ld_dy, s->tA, R, bf, m->st))) return rc2;
    if ((rc2 = transpose16(X, R, n_in, ld_x, s->tB, R, bf, m->st))) return rc2;
    return model_gemm(m, pick_bn(n_in, EPI_RESID), EPI_RESID, s->tA, R, s->tB, R, n_out, n_in, R, out, n_in, nullptr,
                      ew);
  };
  if (s->full) {
    B2P_CHECK_CUDA(cudaMemsetAsync(s->gw, 0, (size_t)s->n_w * 4, m->st));
    B2P_CHECK_CUDA(cudaMemsetAsync(s->g_embed, 0, (size_t)c.vocab * D * 4, m->st));
    B2P_CHECK_CUDA(cudaMemsetAsync(s->g_cembed, 0, (size_t)m->cv * D * 4, m->st));
    // classifier: g_cembed[CV, D] = dlogits^T · xn_final  (train.m:938-941)
    if ((rc = wgrad_gemm(s->dlogits, s->cv_pad, m->cv, v.xn_final, D, D, s->g_cembed))) return rc;
  }
  const int nblk = rms_blocks(R);
  auto part = [&](int idx) { return s->rms_part + (size_t)idx * nblk * D; };
  RmsBwdArgs ra;
  std::memset(&ra, 0, sizeof(ra));
  ra.g = s->dxf;
  ra.x = v.x_final;
  ra.w = m->theta + m->oRfinal;
  ra.out = s->dy;
  ra.part = part(2 * L);
  ra.rows = R;
  if ((rc = rms_bwd(ra, D, bf, m->st))) return rc;
  float* cur = s->dy;
  float* oth = s->dy2;
  auto slab = [&](void* base, int l, size_t row_elems) -> void* {
    return static_cast<char*>(base) + (size_t)l * R * row_elems * e;
  };
  for (int l = L - 1; l >= 0; --l) {
    const long long lb = (long long)l * m->layer_size;
    // FFN: dffn = alpha dy; dsilu = dffn · W2; SwiGLU backward; dx_ffn = [dh1|dh3] · [W1;W3]
    if ((rc = scale16(cur, (long long)R * D, alpha, s->d16, bf, m->st))) return rc;
    EpiParams p0;
    std::memset(&p0, 0, sizeof(p0));
    p0.M = R;
    p0.N = H;
    // W2 stored [D][H]: MN-major operand of dsilu = dffn · W2
    if (s->use_mn) {
      if ((rc = model_gemm_mn(m, EPI_F32, 2, s->d16, D, static_cast<const char*>(m->w2) + (size_t)l * D * H * e, H, R,
                              H, D, s->dsilu, H, p0)))
        return rc;
    } else if ((rc = model_gemm(m, pick_bn(H, EPI_F32), EPI_F32, s->d16, D,
                                static_cast<char*>(s->w2T) + (size_t)l * H * D * e, D, R, H, D, s->dsilu, H, nullptr,
                                p0))) {
      return rc;
    }
    if ((rc = swiglu_bwd(s->dsilu, slab(v.h13, l, 2 * H), R, H, s->dh13, bf, m->st))) return rc;
    if (s->full) {
      // dW2 = dffn^T · silu_out and dW1|W3 = [dh1|dh3]^T · x2norm  (train.m:1027-1034)
      if ((rc = launch_swiglu_gate(slab(v.h13, l, 2 * H), R, H, s->gate, bf, m->st))) return rc;
      if ((rc = wgrad_gemm(s->d16, D, D, s->gate, H, H, s->gw + s->o_2 + (size_t)l * D * H))) return rc;
      if ((rc = wgrad_gemm(s->dh13, 2 * H, 2 * H, slab(v.xn2, l, D), D, D, s->gw + s->o_13 + (size_t)l * 2 * H * D)))
        return rc;
    }
    EpiParams p1;
    std::memset(&p1, 0, sizeof(p1));
    p1.M = R;
    p1.N = D;
    // W1|W3 stored [2H][D] (interleaved rows): MN-major operand of dx_ffn = [dh1|dh3] · [W1;W3]
    if (s->use_mn) {
      if ((rc = model_gemm_mn(m, EPI_F32, 2, s->dh13, 2 * H, static_cast<const char*>(m->w13) + (size_t)l * 2 * H * D * e,
                              D, R, D, 2 * H, s->dxf, D, p1)))
        return rc;
    } else if ((rc = model_gemm(m, pick_bn(D, EPI_F32), EPI_F32, s->dh13, 2 * H,
                                static_cast<char*>(s->w13T) + (size_t)l * D * 2 * H * e, 2 * H, R, D, 2 * H, s->dxf,
                                D, nullptr, p1))) {
      return rc;
    }
    // RMSNorm2 backward + skip: dx2 = rmsnorm_bwd(dx_ffn) + dy; d16 = alpha dx2
    std::memset(&ra, 0, sizeof(ra));
    ra.g = s->dxf;
    ra.x = static_cast<const float*>(static_cast<void*>(v.x_mid)) + (size_t)l * R * D;
    ra.w = m->theta + lb + m->oRf;
    ra.resid = cur;
    ra.out = oth;
    ra.out16 = s->d16;
    ra.alpha16 = alpha;
    ra.part = part(2 * l + 1);
    ra.rows = R;
    if ((rc = rms_bwd(ra, D, bf, m->st))) return rc;
    // dWo = (alpha dx2)^T · attn_out  (train.m:1067-1070)
    if (s->full && (rc = wgrad_gemm(s->d16, D, D, slab(v.attn, l, QD), QD, QD, s->gw + s->o_o + (size_t)l * D * QD)))
      return rc;
    // Wo: U'_o = dx2s · B_o; da = dx2s · Wo + U'_o · A_o
    EpiParams p2;
    std::memset(&p2, 0, sizeof(p2));
    p2.M = R;
    p2.N = kUCols;
    if ((rc = model_gemm(m, 128, EPI_H16, s->d16, D, static_cast<char*>(s->bblk_o) + (size_t)l * 64 * D * e, D, R,
                         kUCols, D, s->ub_o, kUCols, nullptr, p2)))
      return rc;
    EpiParams p3;
    std::memset(&p3, 0, sizeof(p3));
    p3.M = R;
    p3.N = QD;
    p3.has_lora = 1;
    p3.lora = model_lora_epi(m);
    p3.lora.theta = s->a_oT;
    p3.lora.nseg = 1;
    p3.lora.seg_start[0] = 0;
    p3.lora.seg_start[1] = QD;
    p3.lora.seg_boff[0] = (long long)l * QD * r;
    p3.lora.seg_ucol[0] = 0;
    if ((rc = model_gemm(m, pick_bn(QD, EPI_H16), EPI_H16, s->d16, D,
                         static_cast<char*>(s->woT) + (size_t)l * QD * D * e, D, R, QD, D, s->da, QD, s->ub_o, p3)))
      return rc;
    // attention backward -> dQ | dK | dV (pre-RoPE)
    AttnBwdArgs ab;
    std::memset(&ab, 0, sizeof(ab));
    ab.qkv = slab(v.qkv, l, QKV);
    ab.ld = QKV;
    ab.q_off = 0;
    ab.k_off = QD;
    ab.v_off = QD + KVD;
    ab.o = slab(v.attn, l, QD);
    ab.dout = s->da;
    ab.ld_o = QD;
    ab.lse = v.lse + (size_t)l * R * c.heads;
    ab.dvec = s->dvec;
    ab.dqkv = s->dqkv;
    ab.ld_d = QKV + kUCols;
    ab.rope_cos = m->rope_cos;
    ab.rope_sin = m->rope_sin;
    ab.seq = c.seq;
    ab.heads = c.heads;
    ab.kv_heads = c.kv_heads;
    ab.ngroups = n_seq;
    ab.sched = m->tc_attn_bwd ? m->attn_sched : nullptr;
    if ((rc = attention_backward(ab, bf, m->tc_attn_bwd, m->st))) return rc;
    // dWq|dWk|dWv = dQKV^T · xnorm  (train.m:1143-1151)
    if (s->full && (rc = wgrad_gemm(s->dqkv, QKV + kUCols, QKV, slab(v.xn, l, D), D, D,
                                    s->gw + s->o_qkv + (size_t)l * QKV * D)))
      return rc;
    // U'_{q,k,v} = d{q,k,v} · B_{q,k,v} into the 64 extra columns of dqkv; then
    // dx_attn = [dQKV | U'] · [W_qkv ; A_qkv]  (base data gradient + A^T (B^T dY) in one GEMM)
    const int QKVp = QKV + kUCols;
    EpiParams p4;
    std::memset(&p4, 0, sizeof(p4));
    p4.M = R;
    p4.N = kUCols;
    if ((rc = model_gemm(m, 128, EPI_H16, s->dqkv, QKVp, static_cast<char*>(s->bblk_qkv) + (size_t)l * 64 * QKV * e,
                         QKV, R, kUCols, QKV, static_cast<char*>(s->dqkv) + (size_t)QKV * e, QKVp, nullptr, p4)))
      return rc;
    EpiParams p5;
    std::memset(&p5, 0, sizeof(p5));
    p5.M = R;
    p5.N = D;
    if ((rc = model_gemm(m, pick_bn(D, EPI_F32), EPI_F32, s->dqkv, QKVp,
                         static_cast<char*>(s->wqkvT) + (size_t)l * D * QKVp * e, QKVp, R, D, QKVp, s->dxf, D, nullptr,
                         p5)))
      return rc;
    // RMSNorm1 backward + skip: dy = rmsnorm_bwd(dx_attn) + dx2
    std::memset(&ra, 0, sizeof(ra));
    ra.g = s->dxf;
    ra.x = v.x_in + (size_t)l * R * D;
    ra.w = m->theta + lb + m->oRa;
    ra.resid = oth;
    ra.out = cur;
    ra.part = part(2 * l);
    ra.rows = R;
    if ((rc = rms_bwd(ra, D, bf, m->st))) return rc;
    // factored LoRA weight gradients of the layer (the adapters are not trained in full mode)
    if (!s->full && (rc = lora_wgrad(s->d_jobs + (size_t)l * kMaxWgradJobs, kMaxWgradJobs, std::max(D, QD), R, r,
                                     inv_lambda, s->wgrad_part, bf, m->st)))
      return rc;
  }
  if (s->full) {
    // embedding: rows of dx grouped by token (embed_backward), then the classifier rows
    embed_scatter_kernel<<<R, 256, 0, m->st>>>(cur, D, s->d_seg, R, d_tok, s->g_embed, inv_lambda);
    B2P_POST_LAUNCH();
    cembed_scatter_kernel<<<(int)(((long long)m->cv * D + 255) / 256), 256, 0, m->st>>>(s->g_cembed, m->d_c2f, m->cv,
                                                                                      D, s->g_embed);
    B2P_POST_LAUNCH();
  }
  const int nvec = 2 * L + 1;
  rms_part_reduce_kernel<<<(nvec * D + 255) / 256, 256, 0, m->st>>>(s->rms_part, nvec, nblk, D, s->d_rms_off,
                                                                     inv_lambda, s->grad);
  B2P_POST_LAUNCH();
  return B2P_OK;
}

int adam_step(b2p_model* m, float lr, float b1, float b2, float eps, float wd) {
  B2P_REQUIRE(m && m->p16, "no gradient: run a backprop-LoRA step first");
  P16State* s = m->p16;
  DeviceCtx* ctx = nullptr;
  int rc = ctx_get(&ctx);
  if (rc) return rc;
  s->adam_t++;
  // bias corrections as the reference computes them on the host (cpu_ops.h:87-88)
  const float bc1 = 1.0f - powf(b1, (float)s->adam_t), bc2 = 1.0f - powf(b2, (float)s->adam_t);
  AdamArgs a;
  a.w = m->theta;
  a.g = s->grad;
  a.m = s->adam_m;
  a.v = s->adam_v;
  a.n = m->P;
  a.b1 = b1;
  a.omb1 = 1.0f - b1;
  a.b2 = b2;
  a.omb2 = 1.0f - b2;
  a.ibc1 = 1.0f / bc1;
  a.ibc2 = 1.0f / bc2;
  a.eps = eps;
  a.neg_lr = -lr;
  a.wd = wd;
  a.flag = s->flag;
  a.status = ctx->status;
  B2P_CHECK_CUDA(cudaMemsetAsync(s->flag, 0, 4, m->st));
  finite_check_kernel<<<148 * 2, 256, 0, m->st>>>(s->grad, m->P, s->flag);
  B2P_POST_LAUNCH();
  adam_kernel<<<148 * 4, 256, 0, m->st>>>(a);
  B2P_POST_LAUNCH();
  return B2P_OK;
}

// Switch the state to full backprop: fp32 masters up-converted from the current 16-bit
// weights (the masters start from what the forward computes with), gradients, moments.
int ensure_full(b2p_model* m) {
  P16State* s = m->p16;
  if (s->full && s->mw) return B2P_OK;
  const auto& c = m->cfg;
  const long long L = c.nlayers, D = c.dim, H = c.hidden, QD = m->q_dim, QKV = m->qkv_dim;
  const long long n_qkv = L * QKV * D, n_o = L * D * QD, n_13 = L * 2 * H * D, n_2 = L * D * H;
  s->o_qkv = 0;
  s->o_o = n_qkv;
  s->o_13 = s->o_o + n_o;
  s->o_2 = s->o_13 + n_13;
  s->n_w = s->o_2 + n_2;
  const size_t nw = (size_t)s->n_w, ne = (size_t)c.vocab * D;
  P16_ALLOC(s->mw, nw * 4);
  P16_ALLOC(s->gw, nw * 4);
  P16_ALLOC(s->am_w, nw * 4);
  P16_ALLOC(s->av_w, nw * 4);
  P16_ALLOC(s->g_embed, ne * 4);
  P16_ALLOC(s->g_cembed, ne * 4);
  P16_ALLOC(s->am_e, ne * 4);
  P16_ALLOC(s->av_e, ne * 4);
  P16_ALLOC(s->norm_part, (3 * kNormBlocks + 2) * 4);
  B2P_CHECK_CUDA(cudaMemset(s->am_w, 0, nw * 4));
  B2P_CHECK_CUDA(cudaMemset(s->av_w, 0, nw * 4));
  B2P_CHECK_CUDA(cudaMemset(s->am_e, 0, ne * 4));
  B2P_CHECK_CUDA(cudaMemset(s->av_e, 0, ne * 4));
  // segment table: [0] weights, [1] embedding, [2 ..] rms vectors (rms_att|rms_ffn per layer, rms_final)
  const int nrs = (int)L + 1;
  std::vector<long long> off(2 + nrs), len(2 + nrs);
  off[0] = 0; len[0] = s->n_w;
  off[1] = 0; len[1] = (long long)ne;
  for (int l = 0; l < (int)L; ++l) {
    off[2 + l] = (long long)l * m->layer_size + m->oRa;  // rms_att and rms_ffn are adjacent
    len[2 + l] = 2 * D;
  }
  off[2 + L] = m->oRfinal;
  len[2 + L] = D;
  P16_ALLOC(s->d_nseg, 2 * off.size() * sizeof(long long));
  B2P_CHECK_CUDA(cudaMemcpy(s->d_nseg, off.data(), off.size() * 8, cudaMemcpyHostToDevice));
  B2P_CHECK_CUDA(cudaMemcpy(s->d_nseg + off.size(), len.data(), len.size() * 8, cudaMemcpyHostToDevice));
  const bool bf = m->bf16;
  auto up = [&](const void* src, float* dst, long long n) -> int {
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148 * 16);
    if (bf)
      f16_to_f32_kernel<__nv_bfloat16><<<blocks, 256, 0, m->st>>>(static_cast<const __nv_bfloat16*>(src), dst, n);
    else
      f16_to_f32_kernel<__half><<<blocks, 256, 0, m->st>>>(static_cast<const __half*>(src), dst, n);
    B2P_POST_LAUNCH();
    return B2P_OK;
  };
  int rc;
  if ((rc = up(m->wqkv, s->mw + s->o_qkv, n_qkv)) || (rc = up(m->wo, s->mw + s->o_o, n_o)) ||
      (rc = up(m->w13, s->mw + s->o_13, n_13)) || (rc = up(m->w2, s->mw + s->o_2, n_2)))
    return rc;
  s->full = true;
  s->full_t = 0;
  release_rows(s);  // the row buffers gain the full-mode scratch
  s->gen++;
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  return B2P_OK;
}

// Host tokens -> staged tokens/targets, the per-token row segments, then the gradient pass.
int full_grad(b2p_model* m, const uint16_t* tokens, const uint16_t* ctargets, int n_seq) {
  int rc = model_ready(m);
  if (rc) return rc;
  if ((rc = ensure_model_state(m))) return rc;
  if ((rc = ensure_full(m))) return rc;
  if ((rc = ensure_weights(m))) return rc;
  const int R = n_seq * m->cfg.seq;
  if ((rc = ensure_rows(m, R))) return rc;
  m->p16->use_mn = m->use_pair && R >= 2 * kBM;
  if (!m->p16->use_mn && (rc = ensure_weights_kmajor(m))) return rc;
  if ((rc = model_stage_tokens(m, tokens, ctargets, n_seq))) return rc;
  // rows grouped by token, each group in sequence order (deterministic embedding scatter)
  std::vector<int32_t> idx(R);
  for (int i = 0; i < R; ++i) idx[i] = i;
  std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) { return tokens[a] < tokens[b]; });
  std::vector<int32_t> seg(2 * (size_t)R + 2, 0);
  int nseg = 0;
  for (int i = 0; i < R; ++i)
    if (i == 0 || tokens[idx[i]] != tokens[idx[i - 1]]) seg[1 + nseg++] = i;
  seg[1 + nseg] = R;
  seg[0] = nseg;
  std::copy(idx.begin(), idx.end(), seg.begin() + R + 2);
  B2P_CHECK_CUDA(cudaMemcpyAsync(m->p16->d_seg, seg.data(), seg.size() * 4, cudaMemcpyHostToDevice, m->st));
  return p16_grad(m, m->d_tok, m->d_tok + (size_t)n_seq * m->cfg.seq, n_seq);
}

// Global-norm clip and AdamW over weights (wd), embedding (wd) and rms weights (no wd),
// train.m:1309-1517; then the 16-bit weights, compact embedding and transposes follow.
int full_update(b2p_model* m, float lr, float wd, float clip) {
  B2P_REQUIRE(m && m->p16 && m->p16->full, "no full-backprop gradient: run b2p_full_grad first");
  P16State* s = m->p16;
  DeviceCtx* ctx = nullptr;
  int rc = ctx_get(&ctx);
  if (rc) return rc;
  const auto& c = m->cfg;
  const long long* soff = s->d_nseg;
  const long long* slen = s->d_nseg + (c.nlayers + 3);
  const int nrs = c.nlayers + 1;
  B2P_CHECK_CUDA(cudaMemsetAsync(s->flag, 0, 4, m->st));
  sqnorm_kernel<<<kNormBlocks, 256, 0, m->st>>>(s->gw, soff, slen, 1, s->norm_part);
  B2P_POST_LAUNCH();
  sqnorm_kernel<<<kNormBlocks, 256, 0, m->st>>>(s->g_embed, soff + 1, slen + 1, 1, s->norm_part + kNormBlocks);
  B2P_POST_LAUNCH();
  sqnorm_kernel<<<kNormBlocks, 256, 0, m->st>>>(s->grad, soff + 2, slen + 2, nrs, s->norm_part + 2 * kNormBlocks);
  B2P_POST_LAUNCH();
  clip_scale_kernel<<<1, 32, 0, m->st>>>(s->norm_part, 3 * kNormBlocks, clip, s->flag, ctx->status);
  B2P_POST_LAUNCH();
  s->full_t++;
  const float b1 = 0.9f, b2 = 0.95f, eps = 1e-8f;  // train.m:266
  const float bc1 = 1.0f - powf(b1, (float)s->full_t), bc2 = 1.0f - powf(b2, (float)s->full_t);
  AdamSegArgs a;
  a.gscale = s->norm_part + 3 * kNormBlocks + 1;
  a.b1 = b1;
  a.omb1 = 1.0f - b1;
  a.b2 = b2;
  a.omb2 = 1.0f - b2;
  a.ibc1 = 1.0f / bc1;
  a.ibc2 = 1.0f / bc2;
  a.eps = eps;
  a.neg_lr = -lr;
  a.flag = s->flag;
  auto run = [&](float* w, const float* g, float* mo, float* ve, const long long* o, const long long* n, int ns,
                 float wdv) -> int {
    a.w = w; a.g = g; a.m = mo; a.v = ve; a.seg_off = o; a.seg_len = n; a.nseg = ns; a.wd = wdv;
    adam_seg_kernel<<<148 * 8, 256, 0, m->st>>>(a);
    B2P_POST_LAUNCH();
    return B2P_OK;
  };
  if ((rc = run(s->mw, s->gw, s->am_w, s->av_w, soff, slen, 1, wd))) return rc;
  if ((rc = run(m->embed, s->g_embed, s->am_e, s->av_e, soff + 1, slen + 1, 1, wd))) return rc;
  if ((rc = run(m->theta, s->grad, s->adam_m, s->adam_v, soff + 2, slen + 2, nrs, 0.0f))) return rc;
  // refresh the compute copies
  const long long n_qkv = s->o_o - s->o_qkv, n_o = s->o_13 - s->o_o, n_13 = s->o_2 - s->o_13, n_2 = s->n_w - s->o_2;
  if ((rc = launch_f32_to_16(s->mw + s->o_qkv, m->wqkv, n_qkv, m->bf16, m->st)) ||
      (rc = launch_f32_to_16(s->mw + s->o_o, m->wo, n_o, m->bf16, m->st)) ||
      (rc = launch_f32_to_16(s->mw + s->o_13, m->w13, n_13, m->bf16, m->st)) ||
      (rc = launch_f32_to_16(s->mw + s->o_2, m->w2, n_2, m->bf16, m->st)))
    return rc;
  const long long ncv = (long long)m->cv * c.dim;
  if (m->bf16)
    cembed_refresh_kernel<__nv_bfloat16><<<(int)((ncv + 255) / 256), 256, 0, m->st>>>(
        m->embed, m->d_c2f, m->cv, c.dim, static_cast<__nv_bfloat16*>(m->cembed));
  else
    cembed_refresh_kernel<__half><<<(int)((ncv + 255) / 256), 256, 0, m->st>>>(m->embed, m->d_c2f, m->cv, c.dim,
                                                                              static_cast<__half*>(m->cembed));
  B2P_POST_LAUNCH();
  m->weights_version++;  // the transposed copies are rebuilt before the next backward
  return B2P_OK;
}

}  // namespace

int launch_attention_backward(const AttnBwdArgs& a, bool bf16, bool use_tc, cudaStream_t st) {
  return attention_backward(a, bf16, use_tc, st);
}

void p16_release(P16State* s) {
  if (!s) return;
  if (s->graph.exec) cudaGraphExecDestroy(s->graph.exec);
  release_rows(s);
  free_ptrs({s->wqkvT, s->woT, s->w13T, s->w2T, s->cembedT, s->a_oT, s->bblk_qkv, s->bblk_o, s->grad, s->adam_m,
             s->adam_v, s->flag, s->d_jobs, s->d_rms_off, s->mw, s->gw, s->am_w, s->av_w, s->g_embed, s->g_cembed,
             s->am_e, s->av_e, s->norm_part, s->d_nseg});
  delete s;
}

}  // namespace b2p

using namespace b2p;

extern "C" {

int b2p_p16_grad(b2p_model* m, const uint16_t* tokens, const uint16_t* ctargets, int n_seq, float* loss,
                 float* grad) {
  int rc = model_ready(m);
  if (rc) return rc;
  if ((rc = model_stage_tokens(m, tokens, ctargets, n_seq))) return rc;
  if ((rc = p16_grad(m, m->d_tok, m->d_tok + (size_t)n_seq * m->cfg.seq, n_seq))) return rc;
  if (loss) B2P_CHECK_CUDA(cudaMemcpyAsync(loss, m->var_loss, 4, cudaMemcpyDeviceToHost, m->st));
  if (grad) B2P_CHECK_CUDA(cudaMemcpyAsync(grad, m->p16->grad, (size_t)m->P * 4, cudaMemcpyDefault, m->st));
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  return check_device_status(m->st);
}

int b2p_p16_grad_device(b2p_model* m, const int32_t* d_tokens, const int32_t* d_targets, int n_seq, float* d_loss) {
  int rc = model_ready(m);
  if (rc) return rc;
  B2P_REQUIRE(d_tokens && d_targets, "null token/target buffer");
  B2P_REQUIRE(n_seq >= 1 && n_seq <= m->max_groups, "sequence count %d out of range", n_seq);
  if ((rc = p16_grad(m, d_tokens, d_targets, n_seq))) return rc;
  if (d_loss) B2P_CHECK_CUDA(cudaMemcpyAsync(d_loss, m->var_loss, 4, cudaMemcpyDeviceToDevice, m->st));
  return B2P_OK;
}

}  // extern "C"

namespace b2p {

int p16_view(b2p_model* m, bool make_full, TrainView* v) {
  *v = TrainView();
  if (m->ffn && !make_full) return B2P_OK;  // --lora-ffn models keep no backprop state
  int rc = ensure_model_state(m);
  if (rc) return rc;
  if (make_full && (rc = ensure_full(m))) return rc;
  P16State* s = m->p16;
  *v = TrainView();
  v->adam_m = s->adam_m;
  v->adam_v = s->adam_v;
  v->adam_t = &s->adam_t;
  if (s->full && s->mw) {
    v->full = true;
    v->mw = s->mw;
    v->am_w = s->am_w;
    v->av_w = s->av_w;
    v->am_e = s->am_e;
    v->av_e = s->av_e;
    v->o_qkv = s->o_qkv;
    v->o_o = s->o_o;
    v->o_13 = s->o_13;
    v->o_2 = s->o_2;
    v->full_t = &s->full_t;
  }
  return B2P_OK;
}

}  // namespace b2p

extern "C" {

void* b2p_model_grad(b2p_model* m) { return (m && m->p16) ? (void*)m->p16->grad : nullptr; }

int b2p_adam_step(b2p_model* m, float lr, float b1, float b2, float eps, float wd) {
  return adam_step(m, lr, b1, b2, eps, wd);
}

int b2p_adam_state(b2p_model* m, int set, int* t, float* mom, float* vel) {
  B2P_REQUIRE(m, "null model");
  int rc = ensure_model_state(m);
  if (rc) return rc;
  P16State* s = m->p16;
  if (set) {
    B2P_REQUIRE(t && *t >= 0, "step count must be given and non-negative");
    s->adam_t = *t;
    if (mom) B2P_CHECK_CUDA(cudaMemcpyAsync(s->adam_m, mom, (size_t)m->P * 4, cudaMemcpyDefault, m->st));
    if (vel) B2P_CHECK_CUDA(cudaMemcpyAsync(s->adam_v, vel, (size_t)m->P * 4, cudaMemcpyDefault, m->st));
  } else {
    if (t) *t = s->adam_t;
    if (mom) B2P_CHECK_CUDA(cudaMemcpyAsync(mom, s->adam_m, (size_t)m->P * 4, cudaMemcpyDefault, m->st));
    if (vel) B2P_CHECK_CUDA(cudaMemcpyAsync(vel, s->adam_v, (size_t)m->P * 4, cudaMemcpyDefault, m->st));
  }
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  return B2P_OK;
}

int b2p_p16_step(b2p_model* m, const uint16_t* tokens, const uint16_t* ctargets, int n_seq, float lr, float* loss) {
  int rc = model_ready(m);
  if (rc) return rc;
  if ((rc = model_stage_tokens(m, tokens, ctargets, n_seq))) return rc;
  if ((rc = p16_grad(m, m->d_tok, m->d_tok + (size_t)n_seq * m->cfg.seq, n_seq))) return rc;
  // train_mezo.m:2093-2117: b1 0.9, b2 0.95, eps 1e-8, no weight decay
  if ((rc = adam_step(m, lr, 0.9f, 0.95f, 1e-8f, 0.0f))) return rc;
  if (loss) B2P_CHECK_CUDA(cudaMemcpyAsync(loss, m->var_loss, 4, cudaMemcpyDeviceToHost, m->st));
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  return check_device_status(m->st);
}

}  // extern "C"

extern "C" {

int b2p_full_grad(b2p_model* m, const uint16_t* tokens, const uint16_t* ctargets, int n_seq, float* loss) {
  int rc = full_grad(m, tokens, ctargets, n_seq);
  if (rc) return rc;
  if (loss) B2P_CHECK_CUDA(cudaMemcpyAsync(loss, m->var_loss, 4, cudaMemcpyDeviceToHost, m->st));
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  return check_device_status(m->st);
}

int b2p_full_update(b2p_model* m, float lr, float wd, float clip, float* grad_norm) {
  int rc = full_update(m, lr, wd, clip);
  if (rc) return rc;
  if (grad_norm)
    B2P_CHECK_CUDA(cudaMemcpyAsync(grad_norm, m->p16->norm_part + 3 * kNormBlocks, 4, cudaMemcpyDeviceToHost, m->st));
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  return check_device_status(m->st);
}

int b2p_full_step(b2p_model* m, const uint16_t* tokens, const uint16_t* ctargets, int n_seq, float lr, float wd,
                  float clip, float* loss, float* grad_norm) {
  int rc = full_grad(m, tokens, ctargets, n_seq);
  if (rc) return rc;
  if ((rc = full_update(m, lr, wd, clip))) return rc;
  if (loss) B2P_CHECK_CUDA(cudaMemcpyAsync(loss, m->var_loss, 4, cudaMemcpyDeviceToHost, m->st));
  if (grad_norm)
    B2P_CHECK_CUDA(cudaMemcpyAsync(grad_norm, m->p16->norm_part + 3 * kNormBlocks, 4, cudaMemcpyDeviceToHost, m->st));
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  return check_device_status(m->st);
}

long long b2p_full_weight_count(b2p_model* m) {
  if (!m || ensure_model_state(m) || ensure_full(m)) return -1;
  return m->p16->n_w;
}

int b2p_full_read(b2p_model* m, int what, float* out, long long n) {
  B2P_REQUIRE(m && out, "null argument");
  int rc = ensure_model_state(m);
  if (rc) return rc;
  if ((rc = ensure_full(m))) return rc;
  P16State* s = m->p16;
  const long long ne = (long long)m->cfg.vocab * m->cfg.dim;
  const void* src = nullptr;
  long long cnt = 0;
  switch (what) {
    case B2P_FULL_WEIGHTS: src = s->mw; cnt = s->n_w; break;
    case B2P_FULL_WEIGHT_GRADS: src = s->gw; cnt = s->n_w; break;
    case B2P_FULL_EMBED: src = m->embed; cnt = ne; break;
    case B2P_FULL_EMBED_GRAD: src = s->g_embed; cnt = ne; break;
    case B2P_FULL_TRAINABLE_GRAD: src = s->grad; cnt = m->P; break;
    default: set_error("unknown quantity %d", what); return B2P_ERR_ARG;
  }
  B2P_REQUIRE(n == cnt, "quantity %d has %lld floats, got %lld", what, cnt, n);
  B2P_CHECK_CUDA(cudaMemcpyAsync(out, src, (size_t)cnt * 4, cudaMemcpyDefault, m->st));
  B2P_CHECK_CUDA(cudaStreamSynchronize(m->st));
  return B2P_OK;
}

}  // extern "C"
