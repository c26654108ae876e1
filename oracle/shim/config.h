/* shim/config.h — stands in for training/config.h when the reference's plain-C
 * headers (cpu_ops.h, backprop_lora.h) are compiled on Linux for the oracle.
 * TEST INFRASTRUCTURE ONLY.
 *
 * Provides what those headers use from config.h and Apple's Accelerate:
 *   - safe_malloc / safe_calloc (config.h:20-29 semantics: abort on failure);
 *   - the structs they touch (AdamState, LayerWeights, LoRALayer, LoRAGrads);
 *   - lora_grad_project (config.h:286-292 semantics);
 *   - the vDSP / vForce element-wise calls, written as plain C loops
 *     (Accelerate's own implementations are closed; argument order follows
 *     Apple's documented conventions, e.g. vDSP_vsub/vdiv take B first);
 *   - CBLAS prototypes for OpenBLAS (which ships no header in the wheel).
 * Model sizes (DIM, SEQ, ...) come from the reference's models/*.h, passed
 * with -include exactly as training/Makefile:15-23 does.
 */
#pragma once
#include <math.h>
#include <stdbool.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

static inline void* safe_malloc(size_t sz) {
  void* p = malloc(sz);
  if (!p && sz > 0) { fprintf(stderr, "FATAL: malloc(%zu) failed\n", sz); abort(); }
  return p;
}
static inline void* safe_calloc(size_t n, size_t sz) {
  void* p = calloc(n, sz);
  if (!p && n > 0 && sz > 0) { fprintf(stderr, "FATAL: calloc(%zu, %zu) failed\n", n, sz); abort(); }
  return p;
}

#define WQ_SZ (Q_DIM * DIM)
#define WK_SZ (KV_DIM * DIM)
#define WV_SZ (KV_DIM * DIM)
#define WO_SZ (DIM * Q_DIM)
#define W1_SZ (HIDDEN * DIM)
#define W2_SZ (DIM * HIDDEN)
#define W3_SZ (HIDDEN * DIM)

/* ---- CBLAS (OpenBLAS) ---- */
typedef enum { CblasRowMajor = 101, CblasColMajor = 102 } CBLAS_ORDER;
typedef enum { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 } CBLAS_TRANSPOSE;
void cblas_sgemm(CBLAS_ORDER o, CBLAS_TRANSPOSE ta, CBLAS_TRANSPOSE tb, int M, int N, int K, float alpha,
                 const float* A, int lda, const float* B, int ldb, float beta, float* C, int ldc);
void cblas_scopy(int n, const float* x, int incx, float* y, int incy);
void cblas_saxpy(int n, float a, const float* x, int incx, float* y, int incy);

/* ---- vDSP / vForce as plain C ---- */
typedef unsigned long vDSP_Length;
typedef long vDSP_Stride;
static inline void vDSP_vmul(const float* A, vDSP_Stride ia, const float* B, vDSP_Stride ib, float* C,
                             vDSP_Stride ic, vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; i++) C[i * ic] = A[i * ia] * B[i * ib];
}
static inline void vDSP_vadd(const float* A, vDSP_Stride ia, const float* B, vDSP_Stride ib, float* C,
                             vDSP_Stride ic, vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; i++) C[i * ic] = A[i * ia] + B[i * ib];
}
/* C = A - B (B is the first argument) */
static inline void vDSP_vsub(const float* B, vDSP_Stride ib, const float* A, vDSP_Stride ia, float* C,
                             vDSP_Stride ic, vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; i++) C[i * ic] = A[i * ia] - B[i * ib];
}
/* C = A / B (B is the first argument) */
static inline void vDSP_vdiv(const float* B, vDSP_Stride ib, const float* A, vDSP_Stride ia, float* C,
                             vDSP_Stride ic, vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; i++) C[i * ic] = A[i * ia] / B[i * ib];
}
static inline void vDSP_vsmul(const float* A, vDSP_Stride ia, const float* b, float* C, vDSP_Stride ic,
                              vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; i++) C[i * ic] = A[i * ia] * (*b);
}
static inline void vDSP_vsadd(const float* A, vDSP_Stride ia, const float* b, float* C, vDSP_Stride ic,
                              vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; i++) C[i * ic] = A[i * ia] + (*b);
}
/* D = A*b + c (scalars b, c) */
static inline void vDSP_vsmsa(const float* A, vDSP_Stride ia, const float* b, const float* c, float* D,
                              vDSP_Stride id, vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; i++) { const float p = A[i * ia] * (*b); D[i * id] = p + (*c); }
}
/* D = A*b + C (scalar b) */
static inline void vDSP_vsma(const float* A, vDSP_Stride ia, const float* b, const float* C, vDSP_Stride ic,
                             float* D, vDSP_Stride id, vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; i++) { const float p = A[i * ia] * (*b); D[i * id] = p + C[i * ic]; }
}
static inline void vDSP_vneg(const float* A, vDSP_Stride ia, float* C, vDSP_Stride ic, vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; i++) C[i * ic] = -A[i * ia];
}
static inline void vDSP_sve(const float* A, vDSP_Stride ia, float* c, vDSP_Length n) {
  float s = 0; for (vDSP_Length i = 0; i < n; i++) s += A[i * ia]; *c = s;
}
static inline void vDSP_maxv(const float* A, vDSP_Stride ia, float* c, vDSP_Length n) {
  float m = -INFINITY; for (vDSP_Length i = 0; i < n; i++) m = fmaxf(m, A[i * ia]); *c = m;
}
static inline void vvexpf(float* y, const float* x, const int* n) { for (int i = 0; i < *n; i++) y[i] = expf(x[i]); }
static inline void vvsqrtf(float* y, const float* x, const int* n) { for (int i = 0; i < *n; i++) y[i] = sqrtf(x[i]); }
static inline void vvrsqrtf(float* y, const float* x, const int* n) {
  for (int i = 0; i < *n; i++) y[i] = 1.0f / sqrtf(x[i]);
}
static inline void vvrecf(float* y, const float* x, const int* n) { for (int i = 0; i < *n; i++) y[i] = 1.0f / x[i]; }

/* ---- structs used by cpu_ops.h / backprop_lora.h ---- */
typedef struct { float *m, *v; size_t n; } AdamState;
typedef struct {
  float *Wq, *Wk, *Wv, *Wo;
  float *W1, *W2, *W3;
  float *rms_att, *rms_ffn;
} LayerWeights;
typedef struct {
  int rank;
  bool has_ffn;
  float *Aq, *Bq, *Ak, *Bk, *Av, *Bv, *Ao, *Bo;
  float *Wq_base, *Wk_base, *Wv_base, *Wo_base;
  float *A1, *B1, *A2, *B2, *A3, *B3;
  float *W1_base, *W2_base, *W3_base;
} LoRALayer;
typedef struct { float *Aq, *Bq, *Ak, *Bk, *Av, *Bv, *Ao, *Bo; } LoRAGrads;

/* Test hook: while ref_dw_sink is set, every dW that bp_lora_backward hands to
 * lora_grad_project is also copied there, back to back in call order (per layer
 * from the last: Wo, Wq, Wk, Wv; training/backprop_lora.h:223-270). */
static float* ref_dw_sink = 0;
static size_t ref_dw_pos = 0;

/* dB += dW·Aᵀ ; dA += Bᵀ·dW  (same contract as the reference's lora_grad_project) */
static void lora_grad_project(float* dA, float* dB, const float* dW, const float* A, const float* B, int out_dim,
                              int rank, int in_dim) {
  if (ref_dw_sink) {
    memcpy(ref_dw_sink + ref_dw_pos, dW, (size_t)out_dim * in_dim * sizeof(float));
    ref_dw_pos += (size_t)out_dim * in_dim;
  }
  cblas_sgemm(CblasRowMajor, CblasNoTrans, CblasTrans, out_dim, rank, in_dim, 1.0f, dW, in_dim, A, in_dim, 1.0f,
              dB, rank);
  cblas_sgemm(CblasRowMajor, CblasTrans, CblasNoTrans, rank, in_dim, out_dim, 1.0f, B, rank, dW, in_dim, 1.0f, dA,
              in_dim);
}
