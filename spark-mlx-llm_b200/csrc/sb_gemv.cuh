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
// Design (B200): the path is HBM-bound, so each weight byte is read once,
// streamed by 2-D TMA (16 rows x 128 B boxes, 128-byte swizzle) into a
// per-warp ring of shared-memory stages, and dequantized in registers. The dot
// products run on the tensor cores (mma.sync m16n8k16) with the RAW codes as
// the A operand: OR-ing a code into the mantissa of a power of two gives an
// exact small integer (4-bit: low nibble bf16 128+q, high nibble fp16 64+q,
// one shift and four LOP3 per 8 codes; 8-bit: fp16 1024+u, one byte permute
// per 2 codes). The activations are staged once per CTA in the matching
// operand type, scaled by a power of two per K group (exact; the group's
// largest value lands in [2^14, 2^15) so fp16 cannot overflow), with the
// group's sums sum(offset_k * xs_k) and sum(x). Products are exact and
// accumulate in fp32; the group's scale and bias are applied afterwards as
//     y += scale * 2^-e * (acc - sum(offset_k * xs_k)) + bias * sum(x),
// the reassociation the reference kernels use (spark_mlx_ext/
// _w4a16_sources.py:24-39). The MMA's 8 columns carry (activation row, group
// slot) pairs, so at M = 1 one accumulator tile holds up to 8 groups and the
// scale epilogue runs once per stage. bf16 weights (lm_head) multiply bf16
// activations directly. A warp owns 32 weight rows (two m16 tiles); a CTA's 4
// warps share one K range and one staged activation segment. When N alone
// cannot fill the 148 SMs, K is split over the CTAs of a thread-block cluster,
// and the partial sums meet in distributed shared memory: each CTA reduces a
// slice of the rows from every rank in a fixed order (deterministic, one
// launch, no global workspace).
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

constexpr int kGemvWarps = 4;   // 32-row blocks per CTA (one warp each per K sub-part)
constexpr int kGemvMaxWarps = 8; // warps per CTA: 4 row blocks x 1 or 2 K sub-parts
constexpr int kGemvMaxRing = 8; // TMA stages in flight per warp (upper bound)
constexpr int kMaxRopeHalf = 128;

struct GemvParams {
  // TMA descriptors of weight set 0 and 1 ([rows][K*bits/8] bytes, 16x128 B boxes)
  alignas(64) CUtensorMap tmap0;
  alignas(64) CUtensorMap tmap1;
  // TMA descriptors of the scales and biases of sets 0 and 1 (affine, when
  // sc_tma): uint16 [N][K/G], boxes of 16 rows x sc_ld groups
  alignas(64) CUtensorMap smap0;
  alignas(64) CUtensorMap bmap0;
  alignas(64) CUtensorMap smap1;
  alignas(64) CUtensorMap bmap1;
  // activations [M][ldx] (bf16 or fp16); m0 = index of row 0 in the outputs
  // (and positions / argmax keys) when one request is split into launches
  const void* x;
  int ldx;
  int M, N, K;
  int m0;
  // weight set 0 and (EPI_SWIGLU) set 1
  const void* w0;
  const void* s0;
  const void* b0;
  const void* w1;
  const void* s1;
  const void* b1;
  int group_size;  // affine group; 0 for per-channel / bf16
  // K partition: stages (128 weight bytes per row) in total; gridDim.x CTAs of
  // a cluster split them; each warp keeps `ring` stages in flight
  int stages_total;
  int ring;
  int seg_stages;  // stages whose activations are staged in shared memory at a time
  int y_ld;        // bytes per activation row of the staged segment
  int meta_ld;     // groups per activation row of the staged segment
  int pair_scales; // 1 when two consecutive groups' scales are 4-byte aligned
  int sc_ld;       // staged scale/bias elements per weight row (affine formats)
  int sc_tma;      // 1: scales/biases are staged by TMA (rows 16-byte multiples, aligned)
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
  // fused INT8 cache append of the K/V heads (kv_k_cache != null)
  int8_t* kv_k_cache;
  __half* kv_k_scale;
  int8_t* kv_v_cache;
  __half* kv_v_scale;
  int kv_capacity;
  // fused tensor-parallel all-reduce of a RESID epilogue (ar_world > 1)
  int ar_world, ar_rank, ar_channel, ar_np;
  uint8_t* ar_buf[8];
  float inv_freq[kMaxRopeHalf];
  // argmax epilogue
  unsigned long long* argmax_keys;  // [M]
  int argmax_offset;                // added to row indices (vocab-parallel shards)
  unsigned* status;                 // device status word (bounded-wait timeouts) or null
  // 1: the weights are constant across the stream (model weights), so the
  // kernel may start streaming them before the previous kernel finishes.
  int early_prefetch;
  int act;  // EPI_SWIGLU: 0 SiLU, 1 exact GELU
  // K chunks (RESID/STORE): chunk z is K values [z*K, (z+1)*K) of rows that
  // hold chunk_wbytes * chunks weight bytes and sc_stride scale/bias groups.
  // The cluster's CTAs are chunk-major: CTA rank c = z * chunk_parts + q, and
  // the chunk's chunk_parts CTAs split its stages as a launch over that chunk
  // alone would. Each chunk's fp32 partial (its K parts added in rank order,
  // times the per-channel scale) is computed exactly as such a launch computes
  // it; the chunks' partials are then added in a balanced binary tree.
  int chunks;
  int chunk_parts;
  int chunk_wbytes;
  int sc_stride;  // scale/bias groups per weight row in the tables
  int y_f32;  // EPI_STORE: y is fp32 (the sum before any rounding)
  int* plan_out;  // host only: report the plan instead of launching
  // launch planning only: the K split is chosen as for plan_rows output rows in
  // plan_chunks chunks (the unsharded matrix), so that every tensor-parallel
  // shard sums its rows exactly as the whole matrix does
  int plan_rows, plan_chunks;
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
  int8_t* kv_k_cache;
  void* kv_k_scale;
  int8_t* kv_v_cache;
  void* kv_v_scale;
  int64_t kv_capacity;
  int ar_world, ar_rank, ar_channel;
  void* ar_buffers[8];
  int activation;  // EPI_SWIGLU: 0 SiLU, 1 exact GELU
  unsigned long long* argmax_keys;
  int argmax_offset;
  void* workspace;
  size_t workspace_bytes;
  bool weights_constant;
  int k_chunks;  // > 1: fixed K chunks summed in a balanced tree (GemvParams)
  int plan_rows, plan_chunks;
  bool y_f32;
  int* plan_out;  // non-null: report the launch plan (sb_linear_ex_plan) instead of launching
  int scales_ld;  // affine: scale/bias groups per weight row in the tables (0: K / group)
};

int run_linear(const LinearRequest& r, cudaStream_t stream);

// Exchange-buffer layout of the fused tensor-parallel all-reduce, per channel
// (2 channels): 8-byte slots [world][np][8] holding (fp32 partial, epoch), then
// one epoch counter per CTA [kArCtas]. np = N rounded up to 64.
constexpr int kArCtas = 2048;
inline size_t ar_np(int64_t n) { return static_cast<size_t>((n + 63) / 64 * 64); }
inline size_t ar_channel_bytes(int world, int64_t n) {
  return static_cast<size_t>(world) * ar_np(n) * 8 * 8 + static_cast<size_t>(kArCtas) * 4;
}
size_t linear_workspace_size(int epi, int N, int K, int group_k);
// Balanced binary tree over v[0..n) (n <= 8) in index order: pairs (0,1) (2,3)
// ..., then pairs of pairs: how the fused all-reduce adds the ranks' partials.
// The K chunks of one launch meet in the same tree (built incrementally there),
// so a sum split over 1, 2, 4 or 8 ranks rounds identically.
__device__ __forceinline__ float tree_sum8(float (&v)[8], int n) {
#pragma unroll
  for (int s = 1; s < 8; s <<= 1)
#pragma unroll
    for (int i = 0; i + s < 8; i += 2 * s)
      if (i + s < n) v[i] += v[i + s];
  return v[0];
}

}  // namespace sb
