/* 36.4M-parameter "autoresearch" configuration with 8 query / 8 KV heads and
 * SwiGLU hidden 1152 (same projection-weight count per layer, 2,818,048, as the
 * 8/2-head, 1408-hidden variant of training/models/autoresearch.h). Sizes only;
 * used to build the oracle's reference library for that variant. */
#pragma once
#define MODEL_NAME "autoresearch-4L-512d-mha"
#define DIM 512
#define HIDDEN 1152
#define HEADS 8
#define KV_HEADS 8
#define HD 64
#define GQA_RATIO (HEADS / KV_HEADS)
#define Q_DIM (HEADS * HD)
#define KV_DIM (KV_HEADS * HD)
#define SEQ 128
#define NLAYERS 4
#define VOCAB 49152
