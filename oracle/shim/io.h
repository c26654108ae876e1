/* shim/io.h — stands in for training/io.h (ANE/IOSurface code) when the
 * reference's backprop_lora.h is compiled for the oracle. Only the two plain-C
 * GQA helpers it calls are provided (same contract as io.h:439-459).
 * TEST INFRASTRUCTURE ONLY. */
#pragma once
#include "config.h"
static void gqa_tile_kv(float* out, const float* in, int seq) {
  for (int kv = 0; kv < KV_HEADS; kv++)
    for (int r = 0; r < GQA_RATIO; r++)
      memcpy(out + (size_t)(kv * GQA_RATIO + r) * HD * seq, in + (size_t)kv * HD * seq, (size_t)HD * seq * 4);
}
static void gqa_reduce_kv(float* out, const float* in, int seq) {
  memset(out, 0, (size_t)KV_DIM * seq * 4);
  for (int kv = 0; kv < KV_HEADS; kv++)
    for (int r = 0; r < GQA_RATIO; r++) {
      const float* src = in + (size_t)(kv * GQA_RATIO + r) * HD * seq;
      float* dst = out + (size_t)kv * HD * seq;
      for (size_t i = 0; i < (size_t)HD * seq; i++) dst[i] = src[i] + dst[i];
    }
}
