// Tensor-core (tcgen05 + TMEM) linear for M >= 9 activation rows.
//
// y[m, n] = sum_k x[m, k] * W[n, k] with the weight streamed by TMA, tiles of
// 128 weight rows (the MMA's M, one TMEM lane per row) by up to 256 activation
// rows (the MMA's N, TMEM columns), fp32 (or int32) accumulation in TMEM.
//   TW_AFF4 / TW_AFF8 : MLX affine codes + bf16/fp16 scale/bias per group,
//                       dequantized into 128-byte-swizzled shared memory as the
//                       activation dtype, kind::f16 MMA
//                       (mx.quantized_matmul, spark_mlx_llm/ops/linear.py:180-191)
//   TW_I8             : signed int8 rows converted exactly to the activation
//                       dtype, kind::f16 MMA, fp32 scale per row in the epilogue
//                       (w8a16_per_channel, src/spark_w8a16.cpp:80-110)
//   TW_S8             : int8 x int8 kind::i8 MMA with exact int32 accumulators
//                       (int8_matmul_int32 / w8a8_linear, src/spark_w8a8.cpp:218-257)
#pragma once

#include "sb_common.cuh"

namespace sb {

enum TcWeight : int { TW_AFF4 = 0, TW_AFF8 = 1, TW_I8 = 2, TW_S8 = 3 };
enum TcEpilogue : int {
  TE_STORE = 0,    // y = T(acc)
  TE_CHSCALE = 1,  // y = T(acc * wscale[n])
  TE_I32 = 2,      // y = acc (int32)
  TE_W8A8 = 3,     // y = T(((float(acc) * ascale[m]) * wscale[n]) + bias[n])
  TE_ROPE = 4,     // QKV head split + RoPE (head_dim 128 = one weight tile)
};

struct TcRequest {
  int tw = TW_AFF4;
  int te = TE_STORE;
  int act_dtype = SB_DTYPE_BF16;  // 16-bit operand type of the kind::f16 MMA (TW_AFF*, TW_I8)
  const void* x = nullptr;        // [M][K] activations (int8 for TW_S8), row stride K
  int M = 0, N = 0, K = 0;
  const void* w = nullptr;        // weight rows
  const void* scales = nullptr;   // affine: [N][K/G] u16
  const void* biases = nullptr;
  int group_size = 0;
  void* y = nullptr;
  int ldy = 0;
  int y_dtype = SB_DTYPE_BF16;   // TE_W8A8: BF16/F16/F32
  const float* wscale = nullptr;
  const float* ascale = nullptr;
  const void* bias = nullptr;
  int bias_dtype = -1;
  // TE_ROPE
  const int* positions = nullptr;
  int heads_q = 0, heads_kv = 0, seq_len = 1;
  float rope_base = 0.f;
  void *q_out = nullptr, *k_out = nullptr, *v_out = nullptr;
};

// 1 when the request fits the tensor-core kernel (shapes, alignment), else 0
// (the caller then uses the weight-streaming kernel in blocks of 8 rows).
bool tc_linear_supported(const TcRequest& r);
// Workspace bytes of a W8A8 call with M > 8: the counter region, then the
// per-token INT8 activations [M][K] (256-byte aligned) and their fp32 scales [M].
inline size_t tc_w8a8_bytes(int64_t M, int64_t K) {
  return kCounterBytes + static_cast<size_t>((M * K + 255) / 256) * 256 + static_cast<size_t>(M) * 4;
}
int run_tc_linear(const TcRequest& r, cudaStream_t stream);

}  // namespace sb
