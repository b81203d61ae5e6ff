// Weight-streaming linear ("GEMV") family for M <= 8 activation rows.
//
// y[m, n] = sum_k x[m, k] * W[n, k] for the weight formats on the decode path:
//   W_AFF4 / W_AFF8 : MLX affine codes (uint32 little-endian words, element j
//                     at bits [j*b, j*b+b)), bf16 scale/bias per group of G
//                     along K: W = scale * q + bias
//                     (mx.quantized_matmul, spark_mlx_llm/ops/linear.py:180-191)
//   W_I8PC          : signed int8 [N, K] with an fp32 scale per row
//                     (w8a16_per_channel, src/spark_w8a16.cpp:80-110)
//   W_BF16          : plain bf16 [N, K] (the synthetic model's lm_head)
//
// Design (B200): the path is HBM-bound, so each weight byte is read once with
// coalesced 8/16-byte loads and dequantized in registers. The dot products
// run on the tensor cores through mma.sync m16n8k16 using the RAW codes as the
// A operand: a 4-bit code q becomes the exact bf16 value 128+q by OR-ing it
// into the mantissa of 128.0 (0x4300), an 8-bit code is split into two exact
// nibble planes, and fp16 activations use 1024+q (0x6400). Products are exact
// and accumulate in fp32; the per-group scale and bias are applied in fp32
// afterwards as  y += scale * sum(code*x) + bias * sum(x),  the same
// reassociation the reference kernels use (spark_mlx_ext/_w4a16_sources.py:
// 24-39). sum(x) per group comes from one extra MMA against a matrix of ones.
// The activation columns (M <= 8) fill the MMA's n=8 dimension, so M = 1..8
// costs the same instruction count. A warp owns 32 weight rows (two m16
// tiles) over a K range; K is split across warps when N alone cannot fill the
// 148 SMs, and the last warp to finish a row block reduces the partial sums
// in a fixed order (deterministic, single launch).
#pragma once

#include "sb_common.cuh"

namespace sb {

enum WeightFormat : int { W_AFF4 = 0, W_AFF8 = 1, W_I8PC = 2, W_BF16 = 3 };
enum Epilogue : int {
  EPI_STORE = 0,   // y = T(acc)
  EPI_RESID = 1,   // y = T(residual + T(acc))
  EPI_SWIGLU = 2,  // rows paired gate/up: y = T(silu(T(g)) * T(u))
  EPI_ROPE = 3,    // fused QKV head split + RoPE
  EPI_ARGMAX = 4,  // greedy token: argmax over rows of fp32 logits
};

constexpr int kGemvWarps = 4;   // warps per CTA (one work unit each)
constexpr int kGemvTiles = 2;   // m16 tiles per warp (32 weight rows)
constexpr int kMaxRopeHalf = 128;

struct GemvParams {
  // TMA descriptors of weight set 0 and 1 ([rows][K*bits/8] bytes, 16x128 B boxes)
  alignas(64) CUtensorMap tmap0;
  alignas(64) CUtensorMap tmap1;
  // activations [M][ldx] (bf16 or fp16)
  const void* x;
  int ldx;
  int M, N, K;
  // weight set 0 and (EPI_SWIGLU) set 1
  const void* w0;
  const void* s0;
  const void* b0;
  const void* w1;
  const void* s1;
  const void* b1;
  int group_size;  // affine group; 0 for per-channel / bf16
  // split-K
  int splits;
  int groups_total;  // number of K groups (affine: K/G; others: K/64)
  float* partial;    // [splits][rows_padded][8]
  unsigned* counters;  // [rowblocks], zero on entry, left zero on exit
  int rows_padded;
  // rms-norm prologue (optional)
  const void* norm_w;
  float eps;
  // outputs
  void* y;
  int ldy;
  const void* residual;
  int ldr;
  // rope epilogue
  const int* positions;  // [M]
  int heads_q, heads_kv, head_dim, seq_len;
  void* q_out;
  void* k_out;
  void* v_out;
  float inv_freq[kMaxRopeHalf];
  // argmax epilogue
  unsigned long long* argmax_keys;  // [M]
  int argmax_offset;                // added to row indices (vocab-parallel shards)
  int x_seg;                        // K values of x staged in shared memory at a time
  unsigned* status;                 // device status word (bounded-wait timeouts) or null
  // 1: the weights are constant across the stream (model weights), so the
  // kernel may start streaming them before the previous kernel finishes.
  int early_prefetch;
};

// Common request for every linear entry point.
struct LinearRequest {
  int wf;
  int x_dtype;
  const void* x;
  int ldx;
  int M, N, K;
  const void *w0, *s0, *b0, *w1, *s1, *b1;
  int group_size;
  int epi;
  bool norm;
  const void* norm_w;
  float eps;
  void* y;
  int ldy;
  const void* residual;
  int ldr;
  // rope
  const int* positions;
  int heads_q, heads_kv, head_dim, seq_len, rope_dims;
  float rope_base;
  void *q_out, *k_out, *v_out;
  unsigned long long* argmax_keys;
  int argmax_offset;
  void* workspace;
  size_t workspace_bytes;
  bool weights_constant;
};

int run_linear(const LinearRequest& r, cudaStream_t stream);
size_t linear_workspace_size(int epi, int N, int K, int group_k);

}  // namespace sb
