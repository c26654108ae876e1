/* Dynamic-matmul call sites as the ANE-matmul-only path writes them (training/train.m:
 * 82-106 compile, :518-556 requests): one compiled program evaluated on its own
 * surface and, through make_request, on a second per-layer surface whose weights
 * are staged once and whose activations are rewritten with io_write_dyn_acts.
 * Compiled against include/b2p_io.h in place of io.h; the test loads it with ctypes.
 * out holds four [oc, seq] results: own surface, request (W2, act2), request after
 * io_write_dyn_acts (W2, act3), own surface again (W1, act1). */
#include "b2p_io.h"

int site_dyn(const float* act1, const float* W1, const float* act2, const float* W2, const float* act3, int ic,
             int oc, int seq, float* out) {
  if (b2p_init(0) != 0) return -1;
  const int sp = seq + oc;
  Kern* k = compile_kern_mil_w(gen_dyn_matmul_mil(ic, oc, seq), NULL, ic * sp * 2, oc * seq * 2);
  if (!k) return -2;
  if (compile_kern_mil_w(gen_dyn_matmul_mil(ic, oc, seq), NULL, ic * sp * 2 + 2, oc * seq * 2)) return -3;
  io_write_dyn(k->ioIn, act1, ic, seq, W1, oc);
  ane_eval(k);
  io_read_dyn(k->ioOut, out, oc, seq);

  IOSurfaceRef layer_in = make_surface((size_t)ic * sp * 2);
  io_write_dyn(layer_in, act2, ic, seq, W2, oc);
  void* req = make_request(k, layer_in);
  ane_eval_req(k, req);
  io_read_dyn(k->ioOut, out + (size_t)oc * seq, oc, seq);
  io_write_dyn_acts(layer_in, act3, ic, seq, sp);
  ane_eval_req(k, req);
  io_read_dyn(k->ioOut, out + 2 * (size_t)oc * seq, oc, seq);
  ane_eval(k); /* back to the kernel's own surface, unchanged since its last write */
  io_read_dyn(k->ioOut, out + 3 * (size_t)oc * seq, oc, seq);

  CFRelease(req);
  CFRelease(layer_in);
  free_kern(k);
  return 0;
}
