/*
 * spark_b200 persistent decode step: one launch runs a whole batch-1 decode
 * step of the synthetic 4B-class decoder (all layers, the lm_head and the
 * greedy argmax) as a single cooperative kernel with one CTA per SM.
 *
 * It replaces, for batch 1, the per-operator launch sequence of one decode
 * step that the reference builds from its operators - Attention.__call__
 * (spark_mlx_llm/model.py:172-207), TransformerBlock.__call__ (:249-262), the
 * compiled FFN (spark_mlx_llm/ops/ffn.py:83-105), the W8 per-channel / W4
 * affine projections (ops/linear.py:180-191,413-476), spark_qkv_rope
 * (src/spark_qkv_rope.cpp:14-104), int8_quantized_sdpa's decode
 * (spark_mlx_ext/int8_quantized_sdpa.py:156-287) and the greedy sampler of
 * the generation loop (spark_mlx_llm/generation.py:411-446) - with the same
 * arithmetic and bf16 rounding points as the per-operator entry points.
 *
 * Inside the kernel each SM's producer warp streams that SM's slice of every
 * weight matrix, in consumption order, through a ring of shared-memory slots
 * (1-D bulk async copies); it runs ahead across layer boundaries while the
 * consumer warps wait for activations, so HBM keeps streaming through the
 * dependency waits between operators.
 *
 * Weight streams ("tiles" in consumption order, built once at load time by
 * the host, see spark_b200/step.py, from the MLX affine / int8 / bf16
 * checkpoint tensors; rows in blocks of 16, a tile = one row block x one K
 * chunk, tiles ordered row-block-major; lane L = 4*g + c of a 32-lane warp,
 * rows g and g+8 of the block):
 *   W8 (per-channel int8, chunk of Kc values): per 32-column block j, 512 B:
 *       lane L's 16 bytes = row g bytes [32j+8c, +4), row g+8 same, row g
 *       bytes [32j+8c+4, +4), row g+8 same, each byte = int8 code XOR 0x80.
 *   W4 (MLX affine 4-bit, group 64, chunk of Gc groups, 1 or 2 matrices per
 *       tile - gate and up share a tile): per group, per matrix, 512 B: lane
 *       L's 16 bytes = packed words (8g+... see step.py) [row g word c, row
 *       g+8 word c, row g word c+4, row g+8 word c+4] of the group; then the
 *       group metadata: scales [round][matrix][16 rows][8] bf16, then biases
 *       likewise (rounds of 8 groups, zero padded).
 *   BF16 (lm_head, chunk of Kc values): per 16-column block j, 512 B: lane
 *       L's 16 bytes = row g cols 16j+4c+{0,1}, row g+8 same, row g cols
 *       16j+4c+{2,3}, row g+8 same.
 * Chunk sizes are fixed by the model shape, not by the GPU or the
 * tensor-parallel degree: every output row is the sum, in chunk order, of
 * per-chunk partial sums computed the same way everywhere, so results are
 * bit-identical across launches, GPUs and tensor-parallel degrees.
 *
 * Conventions as spark_b200.h: device pointers, caller-owned buffers, a status
 * code, no allocation, no synchronization. The workspace (sb_step_workspace_size
 * bytes) must be zero-filled before the first launch; launches leave it ready
 * for the next one (each launch zeroes only its first SB_STEP_STATUS_OFFSET
 * bytes). Status word (uint32 at byte SB_STEP_STATUS_OFFSET of the workspace,
 * sticky across launches until the caller clears it): bit 0 - a bounded
 * device-side wait gave up and the kernel returned early; bit 1 -
 * positions[0] was outside [0, capacity), so the step did nothing (no cache
 * row is ever written out of bounds).
 */
#ifndef SPARK_B200_STEP_H
#define SPARK_B200_STEP_H

#include <stddef.h>
#include <stdint.h>

#include "spark_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Per-layer device pointers (an array of these lives in device memory). */
typedef struct sb_step_layer {
  const void* qkv;        /* W8 stream of the QKV rows (RoPE pair order, see step.py) */
  const float* qkv_scale; /* per-row fp32 scales in stream row order */
  const void* o;          /* W8 stream of o_proj (this rank's K chunks) */
  const float* o_scale;   /* [hidden] fp32 */
  const void* gateup;     /* W4 stream, gate and up rows paired per tile */
  const void* down;       /* W4 stream of down_proj (this rank's K chunks) */
  const void* in_norm;    /* [hidden] bf16 */
  const void* post_norm;  /* [hidden] bf16 */
  int8_t* k_cache;        /* [kv_heads, capacity, 128] int8 (this rank's heads) */
  void* k_scale;          /* [kv_heads, capacity] fp16 */
  int8_t* v_cache;
  void* v_scale;
} sb_step_layer;

typedef struct sb_step_desc {
  const sb_step_layer* layers; /* device array [num_layers] */
  int num_layers;
  int hidden;     /* multiple of 512 */
  int num_heads;  /* this rank's query heads */
  int num_kv_heads; /* this rank's KV heads; num_heads / num_kv_heads in {1, 2, 4} */
  int head_dim;   /* 128 */
  int inter;      /* this rank's intermediate rows (multiple of 16) */
  int inter_total; /* all ranks' intermediate size (down K), multiple of 512 */
  int vocab;      /* this rank's vocabulary rows */
  int vocab_offset; /* first vocabulary row of this rank */
  int capacity;   /* KV cache capacity (tokens) */
  float rms_eps;
  float rope_theta;
  const void* embed;      /* [vocab_total, hidden] bf16 (full table) */
  int vocab_total;
  const void* head;       /* BF16 stream of this rank's lm_head rows (padded to 16) */
  const void* final_norm; /* [hidden] bf16 */
  const int32_t* tokens;     /* [1] current input token (device) */
  const int32_t* positions;  /* [1] its position (device) */
  void* x;     /* [hidden] bf16 residual stream (scratch) */
  void* q;     /* [num_heads * 128] bf16 (scratch) */
  void* kv_new;/* [2, num_kv_heads * 128] bf16 (scratch) */
  void* attn;  /* [num_heads * 128] bf16 (scratch) */
  void* act;   /* [inter] bf16 (scratch) */
  unsigned long long* argmax_key; /* [1] greedy key (zero before the launch) */
  void* workspace;
  size_t workspace_bytes;
  int world;   /* tensor-parallel degree (1 in this build) */
  int rank;
  /* Optional (NULL = off): per-CTA timing, [grid CTAs][sb_step_trace_slots][4]
   * uint64: for every operator boundary the arrival (this CTA's operator done)
   * and release (all CTAs arrived) as globaltimer ns; then, for the middle
   * layer, a per-warp list of (event code, SM clock) pairs. */
  unsigned long long* trace;
} sb_step_desc;

/* Byte offset of the status word in the workspace. */
#define SB_STEP_STATUS_OFFSET 1024
size_t sb_step_status_offset(void);

/* Trace slots per CTA in sb_step_desc.trace (the layers' operator marks, the
 * lm_head, the kernel start, the attention items' marks and a per-warp event
 * timeline of the middle layer). */
int sb_step_trace_slots(int num_layers);

/* Bytes of the workspace for `desc` (0 if the shape is unsupported). */
size_t sb_step_workspace_size(const sb_step_desc* desc);

/* Tile bytes of each weight stream: [0] QKV, [1] o, [2] gate/up, [3] down,
 * [4] lm_head (0 for an unsupported shape). */
int sb_step_tile_bytes(const sb_step_desc* desc, int64_t out[5]);

/* Enqueue one decode step on `stream`: reads tokens[0] at positions[0],
 * appends its K/V to every layer's cache at that position, and leaves the
 * greedy next token's key in argmax_key (sb_decode_advance turns it into the
 * next token and position). */
int sb_step_run(const sb_step_desc* desc, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPARK_B200_STEP_H */
