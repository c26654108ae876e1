/* One transformer layer's projections driven through the io.h verbs, written the
 * way the conv-fused forward calls them (training/train_mezo.m:1545-1627):
 * QKV fused conv, Wo conv, FFN fused conv with the residual. Compiled against
 * include/b2p_io.h in place of io.h; the test loads it with ctypes. */
#include "b2p_io.h"

int site_layer(const float* Wq, const float* Wk, const float* Wv, const float* Wo, const float* W1,
               const float* W2, const float* W3, int DIM, int Q_DIM, int KV_DIM, int HIDDEN, int SEQ,
               const float* xnorm_buf, const float* attn_out, const float* x2norm, float* x_cur, float* Q, float* K,
               float* V, float* o_out) {
  if (b2p_init(0) != 0) return -1;
  NSString* mil_qkv = gen_qkv_fused_conv1x1_mil(DIM, Q_DIM, KV_DIM, SEQ);
  NSString* mil_wo_conv = gen_conv1x1_mil(Q_DIM, DIM, SEQ);
  NSString* mil_ffn = gen_ffn_fused_conv1x1_mil(DIM, HIDDEN, SEQ);
  Kern* qkvConv = compile_qkv_fused_conv1x1_kern(mil_qkv, Wq, Wk, Wv, DIM, Q_DIM, KV_DIM, SEQ);
  Kern* woConv = compile_conv1x1_kern(mil_wo_conv, Wo, Q_DIM, DIM, SEQ);
  Kern* ffnConv = compile_ffn_fused_conv1x1_kern(mil_ffn, W1, W3, W2, DIM, HIDDEN, SEQ);
  if (!qkvConv || !woConv || !ffnConv) return -2;

  io_write_conv_acts(qkvConv->ioIn, xnorm_buf, DIM, SEQ);
  ane_eval(qkvConv);
  {
    IOSurfaceLock(qkvConv->ioOut, kIOSurfaceLockReadOnly, NULL);
    _Float16* qkv_buf = (_Float16*)IOSurfaceGetBaseAddress(qkvConv->ioOut);
    cvt_f16_f32(Q, qkv_buf, Q_DIM * SEQ);
    cvt_f16_f32(K, qkv_buf + Q_DIM * SEQ, KV_DIM * SEQ);
    cvt_f16_f32(V, qkv_buf + (Q_DIM + KV_DIM) * SEQ, KV_DIM * SEQ);
    IOSurfaceUnlock(qkvConv->ioOut, kIOSurfaceLockReadOnly, NULL);
  }
  io_write_conv_acts(woConv->ioIn, attn_out, Q_DIM, SEQ);
  ane_eval(woConv);
  io_read_dyn(woConv->ioOut, o_out, DIM, SEQ);

  io_write_ffn_fused_conv_input(ffnConv->ioIn, x2norm, x_cur, DIM, SEQ);
  ane_eval(ffnConv);
  io_read_dyn(ffnConv->ioOut, x_cur, DIM, SEQ);

  free_kern(qkvConv);
  free_kern(woConv);
  free_kern(ffnConv);
  return 0;
}
