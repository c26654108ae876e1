/* b2p_io.h — source-compatible stand-in for AutoANE's training/io.h device
 * boundary, on top of the Kern-level C ABI of b2p.h.
 *
 * A call site written against io.h (the conv-fused forward of
 * training/train_mezo.m:1545-1627, the P16 forward :1998-2053) compiles
 * unchanged with this header in place of io.h, after b2p_init(device) where
 * ane_init() was. It provides the same names and argument meaning:
 *
 *   Kern {model, ioIn, ioOut, request, tmpDir}          config.h:75
 *   make_surface, IOSurfaceLock/Unlock/GetBaseAddress    io.h:6 (IOSurface)
 *   cvt_f16_f32, cvt_f32_f16                             io.h:33-51
 *   io_write_fp16, io_read_fp16, io_write_fp16_at, io_copy   io.h:53-77
 *   io_write_dyn, io_write_dyn_acts                      io.h:79-101
 *   io_write_conv_acts, io_read_dyn                      io.h:102-114
 *   compile_kern_mil_w (dynamic-matmul programs)         io.h:116-150
 *   compile_conv1x1_kern, compile_qkv_fused_conv1x1_kern,
 *   compile_ffn_fused_conv1x1_kern                       io.h:165-229
 *   io_write_ffn_fused_conv_input                        io.h:232-240
 *   ane_eval, ane_eval_req, make_request, free_kern      io.h:152, 242-257
 *   gen_conv1x1_mil, gen_qkv_fused_conv1x1_mil,
 *   gen_ffn_fused_conv1x1_mil, gen_dyn_matmul_mil        mil_dynamic.h:17-173
 *
 * Objective-C literals at the call sites become C: the weights dictionary of
 * compile_kern_mil_w is NULL (its dynamic-matmul programs take no baked
 * weights, train.m:82-106 passes @{}), and requests are released with
 * CFRelease as surfaces are.
 *
 * A surface is a host fp16 buffer, as an IOSurface is: writes land in it, and
 * ane_eval uploads the input surface of a kernel (fp16 -> fp32 -> device)
 * before it runs and marks the output surface for refresh; reading an output
 * surface (io_read_*, or IOSurfaceLock followed by IOSurfaceGetBaseAddress)
 * fetches the result first. The MIL text has no meaning here: the gen_*_mil
 * functions return a tag and the compile call fixes the operator.
 *
 * Difference from io.h: ane_eval does not ignore errors. A failed call prints
 * b2p_last_error() and aborts, so results are never silently stale. Code that
 * wants to handle errors calls b2p_eval(k->model) itself.
 *
 * Needs a C compiler with _Float16 (gcc >= 12 on x86-64, clang) and libb2p.so.
 */
#ifndef B2P_IO_H
#define B2P_IO_H

#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "b2p.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef char NSString;   /* MIL text stand-in: the operator tag returned by gen_*_mil */
typedef void NSDictionary; /* compile_kern_mil_w weights: NULL (no baked weights) */

#define B2P_IO_SURFACE_TAG 0x53524643 /* first word of a surface */
#define B2P_IO_REQUEST_TAG 0x51455243 /* first word of a request */

typedef struct b2p_surface {
  int tag;
  size_t bytes;
  int channels, width; /* [channels, width] fp16 when bound to a kernel */
  int split;           /* two-input kernels: columns of input 0 in each row (0: one input) */
  _Float16* mem;       /* the surface contents (fp16, channel-first) */
  b2p_kernel* owner;   /* kernel this surface is bound to (NULL: free-standing) */
  int is_output;
  int dirty;           /* input written since the last upload */
  int stale;           /* output not yet fetched since the last eval */
  struct b2p_surface* uploaded; /* kernel input surfaces: which surface the device input holds */
} b2p_surface;
typedef b2p_surface* IOSurfaceRef;

typedef struct {
  int tag;
  void* kern;       /* Kern* the request evaluates */
  IOSurfaceRef in;  /* its input surface (make_request, io.h:250-257) */
} b2p_request;

typedef struct {
  void* model; /* b2p_kernel* */
  IOSurfaceRef ioIn, ioOut;
  void* request;
  void* tmpDir;
} Kern;

#define kIOSurfaceLockReadOnly 1u

static inline void b2p_io_fail(const char* what) {
  fprintf(stderr, "b2p_io: %s failed: %s\n", what, b2p_last_error());
  abort();
}

static inline IOSurfaceRef make_surface(size_t bytes) {
  b2p_surface* s = (b2p_surface*)calloc(1, sizeof(b2p_surface));
  if (!s || !(s->mem = (_Float16*)calloc(bytes ? bytes : 2, 1))) {
    fprintf(stderr, "b2p_io: out of host memory\n");
    abort();
  }
  s->tag = B2P_IO_SURFACE_TAG;
  s->bytes = bytes;
  return s;
}

static inline void b2p_io_free_surface(IOSurfaceRef s) {
  if (!s) return;
  free(s->mem);
  free(s);
}

/* ---- fp16 <-> fp32 ---- */
static inline void cvt_f16_f32(float* dst, const _Float16* src, int n) {
  for (int i = 0; i < n; i++) dst[i] = (float)src[i];
}
static inline void cvt_f32_f16(_Float16* dst, const float* src, int n) {
  for (int i = 0; i < n; i++) dst[i] = (_Float16)src[i];
}

/* Fetch a kernel's output into its surface if an eval ran since the last fetch. */
static inline void b2p_io_refresh(IOSurfaceRef s) {
  if (!s->owner || !s->is_output || !s->stale) return;
  const size_t n = s->bytes / 2;
  float* tmp = (float*)malloc(n * 4);
  if (!tmp) b2p_io_fail("output fetch (host memory)");
  if (b2p_read_output(s->owner, 0, tmp, n * 4) != 0) b2p_io_fail("b2p_read_output");
  cvt_f32_f16(s->mem, tmp, (int)n);
  free(tmp);
  s->stale = 0;
}

static inline int IOSurfaceLock(IOSurfaceRef s, unsigned flags, void* seed) {
  (void)flags;
  (void)seed;
  b2p_io_refresh(s);
  return 0;
}
static inline int IOSurfaceUnlock(IOSurfaceRef s, unsigned flags, void* seed) {
  (void)seed;
  if (!(flags & kIOSurfaceLockReadOnly) && !s->is_output) s->dirty = 1;
  return 0;
}
static inline void* IOSurfaceGetBaseAddress(IOSurfaceRef s) { return s->mem; }
/* Releases a surface (make_surface) or a request (make_request). */
static inline void CFRelease(const void* obj) {
  if (!obj) return;
  if (*(const int*)obj == B2P_IO_REQUEST_TAG) {
    free((void*)obj);
    return;
  }
  if (*(const int*)obj != B2P_IO_SURFACE_TAG) {
    fprintf(stderr, "b2p_io: CFRelease of an object this shim did not make\n");
    abort();
  }
  b2p_io_free_surface((IOSurfaceRef)obj);
}

/* ---- surface I/O, channel-first [C, S] (io.h:53-114) ---- */
static inline void io_write_fp16(IOSurfaceRef s, const float* data, int channels, int sp) {
  cvt_f32_f16(s->mem, data, channels * sp);
  s->dirty = 1;
}
static inline void io_read_fp16(IOSurfaceRef s, float* data, int ch_off, int channels, int sp) {
  b2p_io_refresh(s);
  cvt_f16_f32(data, s->mem + (size_t)ch_off * sp, channels * sp);
}
static inline void io_copy(IOSurfaceRef dst, int dst_ch, IOSurfaceRef src, int src_ch, int channels, int sp) {
  b2p_io_refresh(src);
  memcpy(dst->mem + (size_t)dst_ch * sp, src->mem + (size_t)src_ch * sp, (size_t)channels * sp * 2);
  dst->dirty = 1;
}
static inline void io_write_fp16_at(IOSurfaceRef s, int ch_off, const float* data, int channels, int sp) {
  cvt_f32_f16(s->mem + (size_t)ch_off * sp, data, channels * sp);
  s->dirty = 1;
}
/* Dynamic-matmul input surface [ic, seq + oc]: row d holds act[d, :] then W[d, :] (io.h:79-89). */
static inline void io_write_dyn(IOSurfaceRef s, const float* act, int ic, int seq, const float* W, int oc) {
  const int sp = seq + oc;
  for (int d = 0; d < ic; d++) {
    cvt_f32_f16(s->mem + (size_t)d * sp, act + (size_t)d * seq, seq);
    cvt_f32_f16(s->mem + (size_t)d * sp + seq, W + (size_t)d * oc, oc);
  }
  s->dirty = 1;
}
/* Activations only, the weights already staged in the surface (io.h:92-99). */
static inline void io_write_dyn_acts(IOSurfaceRef s, const float* act, int ic, int seq, int sp) {
  for (int d = 0; d < ic; d++) cvt_f32_f16(s->mem + (size_t)d * sp, act + (size_t)d * seq, seq);
  s->dirty = 1;
}
static inline void io_write_conv_acts(IOSurfaceRef s, const float* act, int ic, int seq) {
  io_write_fp16(s, act, ic, seq);
}
static inline void io_read_dyn(IOSurfaceRef s, float* out, int oc, int seq) { io_read_fp16(s, out, 0, oc, seq); }
static inline void io_write_ffn_fused_conv_input(IOSurfaceRef s, const float* xnorm, const float* x_cur, int dim,
                                                 int seq) {
  for (int d = 0; d < dim; d++) {
    cvt_f32_f16(s->mem + (size_t)d * 2 * seq, xnorm + (size_t)d * seq, seq);
    cvt_f32_f16(s->mem + (size_t)d * 2 * seq + seq, x_cur + (size_t)d * seq, seq);
  }
  s->dirty = 1;
}

/* ---- MIL tags (mil_dynamic.h:17, :43, :82) ---- */
static inline NSString* gen_conv1x1_mil(int ic, int oc, int seq) {
  (void)ic; (void)oc; (void)seq;
  return (NSString*)"conv1x1";
}
static inline NSString* gen_qkv_fused_conv1x1_mil(int dim, int q_dim, int kv_dim, int seq) {
  (void)dim; (void)q_dim; (void)kv_dim; (void)seq;
  return (NSString*)"qkv_fused_conv1x1";
}
static inline NSString* gen_ffn_fused_conv1x1_mil(int dim, int hidden, int seq) {
  (void)dim; (void)hidden; (void)seq;
  return (NSString*)"ffn_fused_conv1x1";
}
/* y[oc, seq] = W^T · act with W staged in the input surface (mil_dynamic.h:157-173).
 * The tag carries the sizes; it lives in a per-thread ring of 8 buffers. */
static inline NSString* gen_dyn_matmul_mil(int ic, int oc, int seq) {
  static _Thread_local char ring[8][64];
  static _Thread_local int next = 0;
  char* t = ring[next];
  next = (next + 1) % 8;
  snprintf(t, sizeof(ring[0]), "dyn_matmul:%d:%d:%d", ic, oc, seq);
  return (NSString*)t;
}

/* ---- compile / eval / free ---- */
static inline Kern* b2p_io_kern(const b2p_op_desc* d, const float* const* w, int in_ch, int in_w, int out_ch,
                                int split) {
  b2p_kernel* bk = b2p_compile(d, w);
  if (!bk) {
    printf("  [compile] FAIL: %s\n", b2p_last_error()); /* compile_kern_mil_w reports and returns NULL */
    return NULL;
  }
  Kern* k = (Kern*)calloc(1, sizeof(Kern));
  if (!k) b2p_io_fail("compile (host memory)");
  k->model = bk;
  k->ioIn = make_surface((size_t)in_ch * in_w * 2);
  k->ioOut = make_surface((size_t)out_ch * d->seq * 2);
  k->ioIn->channels = in_ch;
  k->ioIn->width = in_w;
  k->ioIn->split = split;
  k->ioOut->channels = out_ch;
  k->ioOut->width = d->seq;
  k->ioIn->owner = bk;
  k->ioOut->owner = bk;
  k->ioOut->is_output = 1;
  return k;
}

static inline b2p_op_desc b2p_io_desc(int kind, int ic, int seq) {
  b2p_op_desc d;
  memset(&d, 0, sizeof(d));
  d.kind = kind;
  d.ic = ic;
  d.seq = seq;
  d.res_alpha = 1.0f;
  d.dtype = B2P_F16;
  return d;
}

static inline Kern* compile_conv1x1_kern(NSString* mil, const float* W, int ic, int oc, int seq) {
  (void)mil;
  b2p_op_desc d = b2p_io_desc(B2P_OP_CONV1X1, ic, seq);
  d.oc = oc;
  const float* w[1] = {W};
  return b2p_io_kern(&d, w, ic, seq, oc, 0);
}

static inline Kern* compile_qkv_fused_conv1x1_kern(NSString* mil, const float* Wq, const float* Wk, const float* Wv,
                                                   int dim, int q_dim, int kv_dim, int seq) {
  (void)mil;
  b2p_op_desc d = b2p_io_desc(B2P_OP_QKV_FUSED, dim, seq);
  d.q_dim = q_dim;
  d.kv_dim = kv_dim;
  const float* w[3] = {Wq, Wk, Wv};
  return b2p_io_kern(&d, w, dim, seq, q_dim + 2 * kv_dim, 0);
}

static inline Kern* compile_ffn_fused_conv1x1_kern(NSString* mil, const float* W1, const float* W3, const float* W2,
                                                   int dim, int hidden, int seq) {
  (void)mil;
  b2p_op_desc d = b2p_io_desc(B2P_OP_FFN_FUSED, dim, seq);
  d.hidden = hidden;
  const float* w[3] = {W1, W3, W2};
  return b2p_io_kern(&d, w, dim, 2 * seq, dim, seq);
}

/* Upload input surface `s` (the kernel's own or a request's) with the kernel's input
 * layout: [C, S] for conv / qkv; two inputs side by side in each row for ffn
 * ([xnorm_d (S) | x_d (S)]) and dynamic matmul ([act_d (seq) | W_d (oc)]). */
static inline void b2p_io_upload(Kern* k, IOSurfaceRef s) {
  b2p_kernel* bk = (b2p_kernel*)k->model;
  const IOSurfaceRef g = k->ioIn; /* geometry */
  const size_t n = (size_t)g->channels * g->width;
  if (s->bytes < n * 2) b2p_io_fail("input upload (surface smaller than the kernel's input)");
  float* tmp = (float*)malloc(n * 4);
  if (!tmp) b2p_io_fail("input upload (host memory)");
  int rc;
  if (g->split == 0) {
    cvt_f16_f32(tmp, s->mem, (int)n);
    rc = b2p_write_input(bk, 0, tmp, n * 4);
  } else {
    const int a = g->split, b = g->width - g->split;
    float* t1 = tmp + (size_t)g->channels * a;
    for (int d = 0; d < g->channels; d++) {
      cvt_f16_f32(tmp + (size_t)d * a, s->mem + (size_t)d * g->width, a);
      cvt_f16_f32(t1 + (size_t)d * b, s->mem + (size_t)d * g->width + a, b);
    }
    rc = b2p_write_input(bk, 0, tmp, (size_t)g->channels * a * 4);
    if (rc == 0) rc = b2p_write_input(bk, 1, t1, (size_t)g->channels * b * 4);
  }
  free(tmp);
  if (rc != 0) b2p_io_fail("b2p_write_input");
  s->dirty = 0;
  g->uploaded = s;
}

static inline void b2p_io_eval_with(Kern* k, IOSurfaceRef in) {
  if (in->dirty || k->ioIn->uploaded != in) b2p_io_upload(k, in);
  if (b2p_eval((b2p_kernel*)k->model) != 0) b2p_io_fail("b2p_eval");
  k->ioOut->stale = 1;
}

static inline void ane_eval(Kern* k) { b2p_io_eval_with(k, k->ioIn); }

/* A request binds another input surface to a compiled kernel, whose output goes
 * to the kernel's ioOut (make_request, io.h:250-257). */
static inline void* make_request(Kern* k, IOSurfaceRef ioIn) {
  b2p_request* r = (b2p_request*)calloc(1, sizeof(b2p_request));
  if (!r) b2p_io_fail("make_request (host memory)");
  r->tag = B2P_IO_REQUEST_TAG;
  r->kern = k;
  r->in = ioIn;
  return r;
}

static inline void ane_eval_req(Kern* k, void* request) {
  b2p_request* r = (b2p_request*)request;
  if (!r || r->tag != B2P_IO_REQUEST_TAG || r->kern != (void*)k) b2p_io_fail("ane_eval_req (request of another kernel)");
  b2p_io_eval_with(k, r->in);
}

/* Compile a program from its MIL text (io.h:116-150). The tags of gen_dyn_matmul_mil
 * compile to B2P_OP_DYN_MATMUL; ic_bytes / oc_bytes size the surfaces as in the
 * reference and must match the program. Other programs, or a weights dictionary,
 * are reported and give NULL, as a failed compile does there. */
static inline Kern* compile_kern_mil_w(NSString* mil, NSDictionary* weights, int ic_bytes, int oc_bytes) {
  int ic = 0, oc = 0, seq = 0;
  if (!mil || weights || sscanf(mil, "dyn_matmul:%d:%d:%d", &ic, &oc, &seq) != 3) {
    printf("  [compile] FAIL: this shim compiles only gen_dyn_matmul_mil programs without weights (got %s)\n",
           mil ? mil : "NULL");
    return NULL;
  }
  if ((long long)ic_bytes != (long long)ic * (seq + oc) * 2 || (long long)oc_bytes != (long long)oc * seq * 2) {
    printf("  [compile] FAIL: surface sizes %d / %d do not match dyn_matmul %d x %d x %d\n", ic_bytes, oc_bytes, ic,
           oc, seq);
    return NULL;
  }
  b2p_op_desc d = b2p_io_desc(B2P_OP_DYN_MATMUL, ic, seq);
  d.oc = oc;
  return b2p_io_kern(&d, NULL, ic, seq + oc, oc, seq);
}

static inline void free_kern(Kern* k) {
  if (!k) return;
  b2p_free((b2p_kernel*)k->model);
  b2p_io_free_surface(k->ioIn);
  b2p_io_free_surface(k->ioOut);
  free(k);
}

#ifdef __cplusplus
}
#endif
#endif /* B2P_IO_H */
