/* b2p.h — C ABI of the B200 projection library (libb2p.so).
 *
 * This library takes the place of AutoANE's Neural-Engine device boundary:
 *   - the in-loop Kern API of training/io.h (compile_conv1x1_kern :165,
 *     compile_qkv_fused_conv1x1_kern :182, compile_ffn_fused_conv1x1_kern :209,
 *     io_write_conv_acts :102, io_write_ffn_fused_conv_input :232,
 *     io_read_dyn :109, ane_eval :242, free_kern :152), and
 *   - the ctypes-facing bridge of bridge/ane_bridge.h (ane_bridge_init :20,
 *     ane_bridge_compile :33, ane_bridge_eval :52, ane_bridge_write_input :55,
 *     ane_bridge_read_output :59, ane_bridge_free :63,
 *     ane_bridge_get_compile_count :66, ane_bridge_reset_compile_count :69).
 *
 * Conventions (same as the reference boundary): host tensors are fp32,
 * channel-first [C, S] row-major; the device side computes in fp16 or bf16
 * with fp32 accumulation. Unlike ane_eval (io.h:242, which ignores errors),
 * every call returns a status: 0 on success, a negative B2P_ERR_* otherwise,
 * with a message available from b2p_last_error(). Nothing here falls back to
 * the CPU: without a B200 the calls fail with B2P_ERR_CUDA / B2P_ERR_UNSUPPORTED.
 *
 * Threading: calls on one handle must not overlap; different handles may be
 * used from different threads. All device work is issued on the stream given
 * to the call (or the handle's stream), so host code can overlap its own work.
 */
#ifndef B2P_H
#define B2P_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define B2P_OK 0
#define B2P_ERR_ARG (-1)
#define B2P_ERR_CUDA (-2)
#define B2P_ERR_DEVICE (-3)
#define B2P_ERR_STATE (-4)
#define B2P_ERR_UNSUPPORTED (-5)

/* ---- compute dtypes ---- */
#define B2P_F16 0
#define B2P_BF16 1

/* Initialise the library on `device` (makes it current for this thread).
 * Replaces ane_bridge_init (bridge/ane_bridge.h:20) / ane_init (training/config.h:131).
 * Returns 0, or a negative status (e.g. the device is not an sm_100 part). */
int b2p_init(int device);

/* Message for the last failed call on this thread (never NULL). */
const char* b2p_last_error(void);

/* Library version string. */
const char* b2p_version(void);

/* Read and clear the device status word written by bounded in-kernel waits.
 * Synchronises `stream`. Returns 0 or B2P_ERR_DEVICE. */
int b2p_device_status(void* stream);

/* Raw projection GEMM on device pointers (the tile engine itself):
 *   Y[M, N] = X[M, K] · W[N, K]^T
 * X and W are row-major 16-bit (dtype B2P_F16 / B2P_BF16), K a multiple of 8,
 * 16-byte aligned. Y is fp32 (out_f32 = 1) or the input dtype (out_f32 = 0),
 * row pitch ldy elements. This is the device-resident form of the reference's
 * cblas_sgemm projection call sites (training/train_mezo.m:1533-1538) in the
 * transposed, token-major layout: X holds tokens as rows, W output channels.
 * Asynchronous on `stream` (NULL = default stream). */
int b2p_gemm(const void* X, const void* W, void* Y, int M, int N, int K, int ldy, int dtype, int out_f32,
             void* stream);

#ifdef __cplusplus
}
#endif
#endif /* B2P_H */
