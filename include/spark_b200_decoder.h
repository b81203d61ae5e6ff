/*
 * spark_b200 decoder entry points: the fused steps of one decode step of the
 * synthetic 4B-class decoder (RMSNorm + QKV + RoPE, INT8 KV append, INT8-KV
 * attention with device-resident lengths, o_proj + residual, RMSNorm +
 * gate/up + SwiGLU, down + residual, RMSNorm + lm_head + greedy argmax).
 *
 * They replace, in fused form, the per-layer graph the reference model builds
 * from its operators: Attention.__call__ (spark_mlx_llm/model.py:172-207),
 * TransformerBlock.__call__ (:249-262), the compiled residual/RMSNorm/FFN graph
 * (spark_mlx_llm/ops/ffn.py:83-105) and the greedy sampler of the generation
 * loop (spark_mlx_llm/generation.py:411-446 via mlx_lm). Same conventions as
 * spark_b200.h: device pointers, caller-owned buffers, status codes, and
 * per-step values (positions, lengths, tokens) read from device memory so a
 * whole decode step can be captured once in a CUDA graph and replayed.
 */
#ifndef SPARK_B200_DECODER_H
#define SPARK_B200_DECODER_H

#include <stddef.h>
#include <stdint.h>

#include "spark_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Weight formats of sb_linear_ex. */
#define SB_WEIGHT_AFFINE4 0 /* MLX affine 4-bit: uint32 [N, K/8], scales/biases [N, K/G] */
#define SB_WEIGHT_AFFINE8 1 /* MLX affine 8-bit: uint32 [N, K/4], scales/biases [N, K/G] */
#define SB_WEIGHT_INT8_PC 2 /* int8 [N, K] with fp32 scales [N] (biases unused)        */
#define SB_WEIGHT_BF16 3    /* bf16 [N, K]                                             */

/* Epilogues of sb_linear_ex. */
#define SB_EPI_STORE 0  /* y[m, n] = T(acc)                                              */
#define SB_EPI_RESID 1  /* y[m, n] = T(residual[m, n] + T(acc))                          */
#define SB_EPI_SWIGLU 2 /* y[m, n] = T(act(T(gate)) * T(up)); weight = gate, weight2 = up;
                         act = SiLU or exact GELU (sb_linear_ex_desc.activation)      */
#define SB_EPI_ROPE 3   /* QKV rows -> q/k/v [B, heads, L, head_dim], RoPE on q and k    */
#define SB_EPI_ARGMAX 4 /* argmax_keys[m] = max over n of (fp32 logit, lowest index)     */

typedef struct sb_linear_ex_desc {
  const void* x; /* [M, ldx] activations */
  int x_dtype;   /* SB_DTYPE_BF16 or SB_DTYPE_F16 */
  int64_t ldx;   /* 0 = K */
  int64_t M, N, K;
  int weight_format;
  const void* weight; /* see SB_WEIGHT_* */
  const void* scales;
  const void* biases;
  const void* weight2; /* SB_EPI_SWIGLU: up projection (same format) */
  const void* scales2;
  const void* biases2;
  int group_size;          /* affine formats */
  const void* norm_weight; /* non-NULL: x is RMS-normalised first (fp32 stats) */
  float norm_eps;
  int epilogue;
  void* y; /* STORE/RESID/SWIGLU output [M, ldy] */
  int64_t ldy;
  const void* residual; /* RESID (may alias y) */
  int64_t ldr;
  /* ROPE */
  const int32_t* positions; /* [M] device */
  int num_heads, num_kv_heads, head_dim, seq_len;
  float rope_base;
  void* q_out;
  void* k_out;
  void* v_out;
  /* ARGMAX: [M] keys, zero before the launch; row indices are reported plus
   * argmax_offset (the first vocabulary row of this shard) */
  unsigned long long* argmax_keys;
  int argmax_offset;
  void* workspace;
  size_t workspace_bytes;
  /* 1: weights/scales are not written by any kernel still in flight on the
   * stream (model weights), so the kernel may start streaming them before the
   * previous kernel has finished; 0: wait for the previous kernel first. */
  int weights_constant;
  /* ROPE, optional fused cache append (head_dim 64 or 128): when kv_k_cache is
   * non-NULL the K and V heads are not stored to k_out/v_out; instead each
   * (token m, KV head) row is rounded to the activation dtype and quantized
   * like sb_kv_append_int8 into the INT8 cache [B, KH, kv_capacity, D] at
   * position positions[m] (fp16 scale [B, KH, kv_capacity]). */
  int8_t* kv_k_cache;
  void* kv_k_scale;
  int8_t* kv_v_cache;
  void* kv_v_scale;
  int64_t kv_capacity;
  /* RESID, optional fused tensor-parallel all-reduce (ar_world 2..8): y is
   * T(residual + T(sum over ranks of the fp32 partial products)). Each rank
   * stores its partial rows into every rank's exchange buffer over NVLink,
   * signals per CTA, waits (bounded) for the other ranks' same CTA and adds
   * the ranks' partials in a balanced binary tree (pairs (0,1) (2,3) ..., then
   * pairs of pairs; the order of k_chunks below) - this replaces all-reduce + residual-add after the row-split
   * o/down projections. ar_buffers[r] is rank r's exchange buffer as mapped in
   * this process (sb_peer_buffer_alloc / _open), sb_tp_exchange_bytes(ar_world,
   * N) bytes, zeroed at creation; consecutive exchanges alternate ar_channel
   * 0/1. Every rank must launch the same shapes in the same order. */
  int ar_world;
  int ar_rank;
  int ar_channel;
  void* ar_buffers[8];
  /* SB_EPI_SWIGLU activation of the gate: 0 SiLU (SwiGLU, the synthetic model),
   * 1 exact GELU 0.5 x (1 + erf(x / sqrt 2)) (the GELU-gated FFN of the
   * reference's Spark2_5 block, spark_mlx_llm/ops/ffn.py:98-103). */
  int activation;
  /* Summation order fixed across tensor-parallel degrees (greedy tokens that are
   * bit-identical at TP 1/2/4/8):
   * k_chunks 2..8 (STORE/RESID, no norm_weight): K is k_chunks equal chunks of
   *   whole groups (16-byte multiples of weight bytes). Each chunk's fp32 partial
   *   is computed exactly as a launch over that chunk's K alone computes it (the
   *   chunks are CTA groups of one thread-block cluster), and the partials are
   *   added in a balanced binary tree in chunk order before the epilogue. A
   *   row-split projection whose unsharded K has c chunks then rounds
   *   identically when rank r of a TP-n group holds chunks [r c/n, (r+1) c/n)
   *   with k_chunks = c/n, plan_k_chunks = c, and the fused all-reduce adds the
   *   ranks' partials.
   * plan_rows > 0: choose the K split as for plan_rows output rows (a
   *   column-split shard names the unsharded row count, so each of its rows sums
   *   exactly as in the whole matrix); plan_k_chunks > 0 likewise plans for that
   *   many K chunks resident at once (the unsharded chunk count). 0 = this
   *   launch's own shape. */
  int k_chunks;
  int64_t plan_rows;
  int plan_k_chunks;
  /* SB_EPI_STORE: 1 stores y as fp32 (the unrounded sum, e.g. a partial for an
   * external all-reduce), 0 in the activation dtype. */
  int y_fp32;
  /* Affine formats: scale/bias groups per weight row in scales/biases (and
   * scales2/biases2), >= K / group_size; 0 = K / group_size. Rows padded to a
   * multiple of 8 groups (16 bytes) let the tables stream by TMA. */
  int64_t scales_ld;
} sb_linear_ex_desc;

/* Fused weight-streaming linear (1 <= M <= 8). */
int sb_linear_ex(const sb_linear_ex_desc* desc, void* stream);
/* The launch plan sb_linear_ex would use for `desc`, without launching (needs
 * the device for its occupancy queries): plan[0..7] = CTAs per cluster,
 * clusters (row groups), threads per CTA, dynamic shared memory bytes, CTAs
 * per K chunk, K sub-parts per CTA, TMA ring depth per warp, 128-byte weight
 * stages per row (of one K chunk). For M > 4 with group 32 (two launches) the
 * first launch's plan. */
int sb_linear_ex_plan(const sb_linear_ex_desc* desc, int* plan);
size_t sb_linear_ex_workspace_size(const sb_linear_ex_desc* desc);

/*
 * Quantize new K/V rows ([B, KH, L, D] bf16) into the INT8 cache at positions
 * start[b] + l: symmetric per token per head, fp16 scale = absmax / 127
 * (1 for a zero row), code = clamp(rint(x / scale), -127, 127). Replaces the
 * cache update of Attention.__call__ (spark_mlx_llm/model.py:192-193).
 */
int sb_kv_append_int8(const void* k_new, const void* v_new, int8_t* k_cache, void* k_scale, int8_t* v_cache,
                      void* v_scale, int64_t batch, int num_kv_heads, int64_t seq_len, int head_dim,
                      int64_t capacity, const int32_t* start, void* stream);

/*
 * Batched-prompt split of a QKV projection: rows qkv[m, :] (stride ld,
 * [H + 2 KH heads x D] bf16, m = b * seq_len + l) -> query heads RoPE-rotated
 * (non-traditional: feature i < rope_dims/2 pairs with i + rope_dims/2, angle
 * positions[m] * rope_base^(-2i/rope_dims); features from rope_dims on are left
 * as they are - partial rotary) into q_out [B, seq_len, H, D];
 * key heads rotated and value heads as they are, quantized into the INT8 cache
 * at positions[m] (the arithmetic of sb_kv_append_int8). Replaces the split,
 * RoPE and cache update of Attention.__call__ (spark_mlx_llm/model.py:172-193,
 * ops/qkv.py:140-177) for a prompt chunk. Rows whose position is outside
 * [0, capacity) write nothing to the cache. D = 64, 128 or 256; rope_dims even,
 * 2..D. With seq_len = 1 it is the decode step's split + RoPE + cache append
 * for shapes the fused QKV epilogue does not take (partial rotary, D = 256).
 */
/*
 * sb_rope_kv_append into a rotating cache (the sliding-window layers'
 * RotatingKVCache, spark_mlx_llm/model.py:362-370, with keep = 0): position p
 * is written to slot p % ring of each [capacity]-row head (ring <= capacity;
 * RoPE still uses p; seq_len <= ring). Once p >= ring - 1 the slots [0, ring)
 * hold exactly the last `ring` positions, so a decode query attends to slots
 * [0, min(p + 1, ring)) - in slot order, which attention does not depend on
 * beyond its fp32 summation order.
 */
int sb_rope_kv_append_ring(const void* qkv, int64_t ld, const int32_t* positions, void* q_out, int8_t* k_cache,
                           void* k_scale, int8_t* v_cache, void* v_scale, int64_t batch, int64_t seq_len,
                           int num_heads, int num_kv_heads, int head_dim, int64_t capacity, int rope_dims,
                           float rope_base, int64_t ring, void* stream);

int sb_rope_kv_append(const void* qkv, int64_t ld, const int32_t* positions, void* q_out, int8_t* k_cache,
                      void* k_scale, int8_t* v_cache, void* v_scale, int64_t batch, int64_t seq_len,
                      int num_heads, int num_kv_heads, int head_dim, int64_t capacity, int rope_dims,
                      float rope_base, void* stream);

/* out = bf16(silu(gate) * up) elementwise over `count` bf16 values (the gated MLP
 * of spark_mlx_llm/ops/ffn.py:98-103 with SiLU); 16-byte aligned buffers. */
int sb_swiglu(const void* gate, const void* up, void* out, int64_t count, void* stream);

/* out = bf16(act(gate) * up): activation 0 SiLU, 1 exact GELU 0.5 x (1 + erf(x / sqrt 2))
 * (nn.gelu in the reference's Spark2_5 FFN, spark_mlx_llm/ops/ffn.py:98-103). */
int sb_gated_activation(const void* gate, const void* up, void* out, int64_t count, int activation,
                        void* stream);

/*
 * Attention-output head gate of the Spark2_5 block (spark_mlx_llm/ops/attention_output.py:91-95):
 * per row m and head h, d = bf16(x[m, :] . gate_weight[h, :]) (fp32 accumulation),
 * gate = bf16(sigmoid(d)) in fp32, out[m, h, :] = bf16(attn[m, h, :] * gate).
 *   x [rows, hidden] bf16 (hidden a multiple of 8), gate_weight [heads, hidden] bf16,
 *   attn / out [rows, heads, head_dim] bf16 (out may alias attn); x, gate_weight 16-byte aligned.
 */
int sb_head_gate(const void* x, const void* gate_weight, const void* attn, void* out, int64_t rows,
                 int64_t hidden, int num_heads, int head_dim, void* stream);

/* INT8-KV decode attention with per-batch lengths lengths[b] + length_offset read on
 * the device; max_length bounds them (it sizes the split-K workspace).
 * prefix_constant = 1 promises that `lengths` and every cache row except the
 * newest one (position lengths[b] + length_offset - 1) were written before the
 * kernel that precedes this launch in the stream; the kernel then streams those
 * rows while that kernel still runs (programmatic dependent launch). 0 waits
 * for the previous kernel before reading anything. plan_kv_heads > 0 splits
 * the tokens as a launch over that many KV heads would (a tensor-parallel shard
 * naming the unsharded KV head count computes its heads bit-identically to the
 * unsharded launch); the workspace must then hold that plan's splits
 * (sb_int8_sdpa_workspace_size with the unsharded head counts suffices). */
int sb_int8_sdpa_decode_dev(const void* q, const int8_t* k, const void* k_scale, const int8_t* v,
                            const void* v_scale, void* out, int64_t batch, int num_heads, int num_kv_heads,
                            const int32_t* lengths, int length_offset, int64_t max_length, int64_t capacity,
                            int head_dim, float scale, int prefix_constant, int plan_kv_heads, void* workspace,
                            size_t workspace_bytes, void* stream);

/* Exchange buffers of the fused tensor-parallel all-reduce (sb_linear_ex
 * ar_*): size for `world` ranks and N output rows; a zeroed device buffer
 * exported as a 64-byte CUDA IPC handle; mapping another rank's buffer into
 * this process (peer access over NVLink); unmapping; freeing. */
size_t sb_tp_exchange_bytes(int world, int64_t n);
int sb_peer_buffer_alloc(size_t bytes, void** ptr, void* handle64);
int sb_peer_buffer_open(const void* handle64, void** ptr);
int sb_peer_buffer_close(void* ptr);
int sb_peer_buffer_free(void* ptr);

/* out[r, :] = table[ids[r], :] (bf16 embedding rows). Replaces nn.Embedding
 * (spark_mlx_llm/model.py:296-305). */
/*
 * Rows of an MLX-affine quantized embedding table (nn.QuantizedEmbedding, the
 * reference's quantized checkpoints; tied to the lm_head): out[r, :] =
 * bf16(scale * q + bias) of table row ids[r] (ids clamped to [0, vocab)).
 *   weight uint32 [vocab, hidden * bits / 32], scales / biases bf16
 *   [vocab, hidden / group_size]; bits 4 or 8, group_size 32, 64 or 128,
 *   hidden a multiple of 8; out bf16 [rows, hidden].
 */
int sb_embed_rows_affine(const void* weight, const void* scales, const void* biases, const int32_t* ids, void* out,
                         int64_t rows, int64_t hidden, int64_t vocab, int group_size, int bits, void* stream);

int sb_embed_rows(const void* table, const int32_t* ids, void* out, int64_t rows, int64_t hidden, int64_t vocab,
                  void* stream);

/* x = T(x + y) elementwise over `count` bf16 values (the residual add after a
 * tensor-parallel all-reduce; replaces `x + attention_output`, ops/ffn.py:98). */
int sb_residual_add(void* x, const void* y, int64_t count, void* stream);

/* Greedy step bookkeeping: tokens[b] = index encoded in argmax_keys[b],
 * argmax_keys[b] = 0, positions[b] += advance. */
int sb_decode_advance(unsigned long long* argmax_keys, int32_t* tokens, int32_t* positions, int batch, int advance,
                      void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPARK_B200_DECODER_H */
