/*
 * spark_b200 - C ABI of the B200 (sm_100a) decode hot path of Spark-MLX-LLM.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as void*, NULL = legacy default stream), enqueues its kernels on
 * that stream and returns a status code; it never synchronizes, never
 * allocates device memory and never frees caller memory. Outputs are written
 * into caller-allocated buffers; inputs are never modified. Scratch memory,
 * where an entry point needs it, is a caller-provided `workspace` whose size
 * comes from the matching *_workspace_size function; it must be zero-filled
 * before its first use and is left zero-filled by every call that returns
 * SB_OK. Calls that share one workspace must be ordered (same stream).
 *
 * Element types use the SB_DTYPE_* codes. Activations are row-major.
 *
 * The interface each entry point replaces is cited as path:line inside the
 * reference project (XHToken/Spark-MLX-LLM).
 */
#ifndef SPARK_B200_H
#define SPARK_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define SB_OK 0
#define SB_EINVAL 1       /* bad shape, dtype, pointer alignment or argument */
#define SB_EUNSUPPORTED 2 /* valid request this build does not implement */
#define SB_ECUDA 3        /* CUDA launch/runtime error */
#define SB_ETIMEOUT 4     /* a bounded device-side wait gave up */

/* Element type codes. */
#define SB_DTYPE_BF16 0
#define SB_DTYPE_F16 1
#define SB_DTYPE_F32 2

/* Library version (major * 10000 + minor * 100 + patch). */
int sb_version(void);

/* Message of the last failing call on this host thread ("" if none). */
const char* sb_last_error_message(void);

/*
 * 1 if `device` is a compute-capability 10.x GPU this library was built for,
 * else 0. Replaces is_w8a8_available()
 * (extensions/spark-mlx-ext/src/spark_w8a8.cpp:204-216, _ext.pyi:5).
 */
int sb_device_supported(int device);

/*
 * MLX affine quantized linear, y[M,N] = x[M,K] @ W^T with
 * W[n,k] = scales[n,k/G] * q[n,k] + biases[n,k/G].
 * Replaces mx.quantized_matmul(x, w, scales, biases, transpose=True,
 * group_size, bits, mode="affine") as called by AffineParameters.native
 * (spark_mlx_llm/ops/linear.py:180-191) and w4a16_qmv / w4a16_multirow
 * (extensions/spark-mlx-ext/spark_mlx_ext/w4a16_qmv.py:37-98,
 *  w4a16_multirow.py:238-437).
 *   x        : [M, K] activations of x_dtype (BF16 or F16), row stride K
 *   w        : [N, K*bits/32] uint32 words, code j of a word at bits [j*bits, j*bits+bits)
 *   scales, biases : [N, K/G] of x_dtype
 *   y        : [M, N] of x_dtype
 *   bits 4 or 8; group_size 32, 64 or 128; M >= 1. M <= 8 runs the
 *   weight-streaming kernel (exact products of the codes); M > 8 runs the
 *   tensor-core kernel (tcgen05, dequantized weight tiles rounded to x_dtype,
 *   as MLX's multi-row path does) when K/group_size is a multiple of 8 and
 *   x, w, scales and biases are 16-byte aligned, else blocks of 8 rows.
 */
int sb_affine_linear(const void* x, int x_dtype, const uint32_t* w, const void* scales,
                     const void* biases, void* y, int64_t M, int64_t N, int64_t K,
                     int group_size, int bits, void* workspace, size_t workspace_bytes,
                     void* stream);
size_t sb_affine_linear_workspace_size(int64_t M, int64_t N, int64_t K, int group_size,
                                       int bits);

/*
 * Per-channel int8 weight linear, y = x(dtype) . ((sum_k x*w) * scales[n]).
 * Replaces w8a16_per_channel (extensions/spark-mlx-ext/src/spark_w8a16.cpp:80-110,
 * bindings.cpp:13-30) and w8a16_multirow (spark_mlx_ext/w8a16_multirow.py:44-129).
 *   x [M,K] BF16/F16, w [N,K] int8, scales [N] fp32, y [M,N] of x_dtype; M >= 1
 *   (M > 8: tensor-core kernel, int8 converted exactly to x_dtype).
 */
int sb_w8a16_per_channel(const void* x, int x_dtype, const int8_t* w, const float* scales,
                         void* y, int64_t M, int64_t N, int64_t K, void* workspace,
                         size_t workspace_bytes, void* stream);
size_t sb_w8a16_per_channel_workspace_size(int64_t M, int64_t N, int64_t K);

/*
 * Per-token symmetric INT8 activation quantization:
 * scale[m] = max|x[m,:]| / 127 (1 when the row is zero), q = clamp(rint(x/scale), -127, 127).
 * Replaces quantize_per_token_* (extensions/spark-mlx-ext/src/kernels/w8a8_quantize.metal:6-43).
 *   x [M,K] BF16/F16/F32, q [M,K] int8, scales [M] fp32.
 */
int sb_quantize_per_token(const void* x, int x_dtype, int8_t* q, float* scales, int64_t M,
                          int64_t K, void* stream);

/*
 * Exact int8 GEMM with int32 accumulation, out[M,N] = x[M,K] @ w[N,K]^T.
 * Replaces int8_matmul_int32 (extensions/spark-mlx-ext/src/spark_w8a8.cpp:218-228).
 *   K a multiple of 32 and <= 131040 (no int32 overflow). M > 8 runs the
 *   tcgen05 kind::i8 kernel (int32 accumulators in TMEM, exact).
 */
int sb_int8_matmul_int32(const int8_t* x, const int8_t* w, int32_t* out, int64_t M, int64_t N,
                         int64_t K, void* stream);

/*
 * W8A8 linear: per-token INT8 activations x INT8 weights, INT32 accumulation,
 * y = T(float(acc) * scale_a[m] * scales[n] + bias[n]).
 * Replaces w8a8_linear / W8A8Linear (extensions/spark-mlx-ext/src/spark_w8a8.cpp:230-257,
 * spark_mlx_ext/linear.py:9-55).
 *   x [M,K] BF16/F16/F32 (y has the same dtype), w [N,K] int8, scales [N] fp32,
 *   bias [N] of bias_dtype or NULL. K a multiple of 32 and <= 131040.
 *   M > 8 (with a workspace of sb_w8a8_linear_workspace_size bytes): per-token
 *   quantization into the workspace, then the tcgen05 kind::i8 kernel.
 */
int sb_w8a8_linear(const void* x, int x_dtype, const int8_t* w, const float* scales,
                   const void* bias, int bias_dtype, void* y, int64_t M, int64_t N, int64_t K,
                   void* workspace, size_t workspace_bytes, void* stream);
size_t sb_w8a8_linear_workspace_size(int64_t M, int64_t N, int64_t K);

/*
 * Fused QKV projection + head split + RoPE (non-traditional, scale 1).
 * Replaces spark_qkv_rope (extensions/spark-mlx-ext/src/spark_qkv_rope.cpp:14-104,
 * _ext.pyi:27-44) and the compiled QKV route of dispatch_qkv
 * (spark_mlx_llm/ops/qkv.py:18-87,140-177).
 *   x [B*L, hidden] of x_dtype; w/scales/biases: affine (bits 4/8) QKV weight with
 *   N = (num_heads + 2*num_kv_heads) * head_dim rows; positions [B*L] int32
 *   (absolute token positions; the reference's scalar `offset` is positions = offset + l).
 *   q_out [B, num_heads, L, head_dim], k_out/v_out [B, num_kv_heads, L, head_dim].
 *   B*L <= 8: weight-streaming kernel; B*L > 8: tensor-core kernel (head_dim
 *   128, hidden/group_size a multiple of 8, 16-byte aligned tensors).
 */
int sb_qkv_rope(const void* x, int x_dtype, const uint32_t* w, const void* scales,
                const void* biases, const int32_t* positions, void* q_out, void* k_out,
                void* v_out, int64_t batch, int64_t seq_len, int64_t hidden, int num_heads,
                int num_kv_heads, int head_dim, int rope_dims, float rope_base, int group_size,
                int bits, void* workspace, size_t workspace_bytes, void* stream);
size_t sb_qkv_rope_workspace_size(int64_t batch, int64_t seq_len, int64_t hidden, int num_heads,
                                  int num_kv_heads, int head_dim, int group_size, int bits);

/*
 * INT8-KV single-query decode attention (flash-decoding split-K).
 * Replaces int8_quantized_sdpa's decode path
 * (extensions/spark-mlx-ext/spark_mlx_ext/int8_quantized_sdpa.py:156-287 and the
 * kernels in _int8_sdpa_sources.py:8-181,363-376) for the symmetric per-token,
 * per-head INT8 KV format:
 *   q       [B, H, 1, D] BF16
 *   k, v    [B, KH, capacity, D] int8 (token t of head h at ((b*KH + h)*capacity + t)*D)
 *   k_scale, v_scale [B, KH, capacity] fp16; K[t] = k[t] * k_scale[t]
 *   out     [B, H, 1, D] BF16; attends to tokens 0..length-1 (the query is the last
 *   position, so the bottom-right causal mask keeps them all).
 *   D = 128 or 256 (the reference model's 256: int8_quantized_sdpa.py:226-230);
 *   H % KH == 0 with H/KH in {1, 2, 4, 8}; softmax in fp32.
 */
int sb_int8_sdpa_decode(const void* q, const int8_t* k, const void* k_scale, const int8_t* v,
                        const void* v_scale, void* out, int64_t batch, int num_heads,
                        int num_kv_heads, int64_t length, int64_t capacity, int head_dim,
                        float scale, void* workspace, size_t workspace_bytes, void* stream);
size_t sb_int8_sdpa_workspace_size(int64_t batch, int num_heads, int num_kv_heads,
                                   int64_t length, int head_dim);

/*
 * Same computation as sb_int8_sdpa_decode, for callers that cannot allocate
 * device memory and so cannot supply a workspace: code that only receives
 * input/output buffers from a host runtime or plugin host that owns all device
 * memory, and latency-bound services that allocate nothing after start-up
 * (cudaMalloc synchronizes the device). This entry point has no counterpart in
 * the reference.
 *   Scratch: a 4 MiB array inside the library (one per GPU that loads it, kept
 *   until the process exits). Shapes whose split-K scratch
 *   (sb_int8_sdpa_workspace_size) exceeds 4 MiB are rejected with SB_EINVAL.
 *   The first call on a device looks up the array's device address
 *   (cudaGetSymbolAddress) with that device current; make that first call
 *   before any stream capture. Each call clears the array's counters on
 *   `stream` before its kernel. All calls on a device share the one array:
 *   calls that overlap on the GPU (different streams, no ordering) race and
 *   must not be issued.
 *   Failure reporting: this call returns before its kernel runs, and the
 *   device status word that a timed-out bounded wait sets lives in the
 *   library array, which the next call clears - so on this entry point such
 *   a timeout is NOT reported (the output is then incomplete). Callers that
 *   must detect it use sb_int8_sdpa_decode with their own workspace and read
 *   its status word.
 *   Arguments and layouts are those of sb_int8_sdpa_decode.
 */
int sb_int8_sdpa_decode_static(const void* q, const int8_t* k, const void* k_scale, const int8_t* v,
                               const void* v_scale, void* out, int64_t batch, int num_heads,
                               int num_kv_heads, int64_t length, int64_t capacity, int head_dim,
                               float scale, void* stream);

/*
 * INT8-KV multi-query attention (prefill / chunked prompt), the BASELINE KV
 * format of sb_int8_sdpa_decode with L >= 1 queries per sequence. Replaces the
 * prefill route of int8_quantized_sdpa (spark_mlx_ext/int8_quantized_sdpa_prefill.py:44-57,
 * kernel _int8_prefill_sources.py:7-154) and its staged recipe
 * (int8_quantized_sdpa.py:122-153) for this format:
 *   q    [B, H, q_len, D] BF16 (layout 0) or [B, q_len, H, D] (layout 1)
 *   k, v [B, KH, capacity, D] int8; k_scale, v_scale [B, KH, capacity] fp16
 *   out  same layout as q, BF16
 * The queries are the last q_len of `length` positions; causal != 0 applies
 * the bottom-right mask (query l sees keys [0, length - q_len + l]), else every
 * query sees keys [0, length). Scores, softmax and accumulation in fp32; the
 * probabilities times the V scale are rounded to fp16 for P.V. D = 128 or 256
 * (the reference's fused path is D = 256; q 16-byte aligned at 256), H/KH
 * in {1, 2, 4, 8}, q_len <= length <= capacity, K/V caches 16-byte aligned.
 * No workspace.
 */
int sb_int8_sdpa_prefill(const void* q, const int8_t* k, const void* k_scale, const int8_t* v,
                         const void* v_scale, void* out, int64_t batch, int num_heads,
                         int num_kv_heads, int64_t q_len, int64_t length, int64_t capacity,
                         int head_dim, float scale, int causal, int layout, void* stream);

/*
 * sb_int8_sdpa_prefill with the bottom-right causal mask and a sliding window:
 * query l (position length - q_len + l) sees keys (position - window, position]
 * (window 0: no window). The chunked prompt of a sliding-window layer
 * (spark_mlx_llm/model.py:313-320, the mask of its RotatingKVCache chunk,
 * :362-370) over the INT8 cache; arguments and layouts as sb_int8_sdpa_prefill.
 * A query's keys start at row 0 of k / v, so a caller holding only a window of
 * the cache passes pointers offset to its first row (row stride `capacity`).
 */
int sb_int8_sdpa_prefill_window(const void* q, const int8_t* k, const void* k_scale, const int8_t* v,
                                const void* v_scale, void* out, int64_t batch, int num_heads,
                                int num_kv_heads, int64_t q_len, int64_t length, int64_t capacity,
                                int head_dim, float scale, int window, int layout, void* stream);

/*
 * BF16 multi-query attention (speculative verification, sliding-window layers).
 * Replaces bf16_sdpa_multiquery (spark_mlx_ext/bf16_sdpa_multiquery.py:155-189)
 * and the BF16 scaled_dot_product_attention it falls back to:
 *   q    [B, H, q_len, D] BF16 (layout 0) or [B, q_len, H, D] (layout 1)
 *   k, v [B, KH, capacity, D] BF16; out: the layout of q, BF16
 * The queries are the last q_len of `length` positions. Masks combine: causal
 * != 0 - bottom-right causal (query l sees keys [0, length - q_len + l]);
 * window > 0 (with causal) - also only the last `window` keys up to the query's
 * position; mask != NULL - bytes [q_len, mask_ld] (nonzero = visible, shared by
 * every batch row and head). Scores, softmax and accumulation in fp32; the
 * probabilities enter P.V as a bf16 hi + lo pair. A query with no visible key
 * gets zeros. D = 128 or 256, H/KH in {1, 2, 4, 8}, 16-byte aligned K/V. No workspace.
 */
int sb_bf16_sdpa_multiquery(const void* q, const void* k, const void* v, void* out, int64_t batch,
                            int num_heads, int num_kv_heads, int64_t q_len, int64_t length,
                            int64_t capacity, int head_dim, float scale, int causal, int window,
                            const uint8_t* mask, int64_t mask_ld, int layout, void* stream);

/*
 * Attention over MLX affine-quantized KV tuples: the int8_quantized_sdpa input
 * format (spark_mlx_ext/int8_quantized_sdpa.py:156-287, staged recipe
 * _fallback :122-153). Replaces int8_quantized_sdpa for its affine tuples.
 *   q        [B, H, L, dk] in `dtype` (SB_DTYPE_BF16 / F16 / F32)
 *   k_packed [B, KH, N, dk*bits/32] uint32, k_scales/k_biases [B, KH, N, dk/G]
 *   v_packed [B, KH, N, dv*bits/32] uint32, v_scales/v_biases [B, KH, N, dv/G]
 *   out      [B, H, L, dv] in `dtype`
 * K[n,d] = scale_k[n,d/G] * code + bias_k[n,d/G] (V likewise); scores
 * scale * q.K, softmax and P.V accumulate in fp32; causal != 0 applies the
 * bottom-right causal mask (query l of L sees keys [0, N-L+l]). bits 2/4/8,
 * group 32/64/128, dk/dv multiples of the group <= 256, H % KH == 0.
 * Single-query decode at dk = dv = 128 or 256 (4/8-bit, BF16/F16 q, H/KH in
 * {1, 2, 4, 8}, 16-byte aligned packed codes) runs on the tensor cores: K and
 * V enter the dot products as fp16 values of scale * code + bias (one
 * rounding, relative 2^-11; K/V magnitudes must lie within about 1e-4 ... 6.5e4),
 * with fp32 scores, softmax and accumulation.
 * Workspace: sb_affine_sdpa_workspace_size bytes (0 = single-split launch);
 * it must be 16-byte aligned for the decode kernels' split merge (else they
 * run one split).
 */
int sb_affine_sdpa(const void* q, int dtype, const void* k_packed, const void* k_scales,
                   const void* k_biases, const void* v_packed, const void* v_scales,
                   const void* v_biases, void* out, int64_t batch, int num_heads, int num_kv_heads,
                   int64_t length, int64_t n, int dk, int dv, int group_size, int bits, float scale,
                   int causal, void* workspace, size_t workspace_bytes, void* stream);
size_t sb_affine_sdpa_workspace_size(int64_t batch, int num_heads, int64_t length, int64_t n,
                                     int dv);

/*
 * RMSNorm, y = T(x * rsqrt(mean(x^2) + eps) * weight), fp32 statistics.
 * Replaces mx.fast.rms_norm as used by dispatch_ffn (spark_mlx_llm/ops/ffn.py:99)
 * and nn.RMSNorm (spark_mlx_llm/model.py:240-243).
 */
int sb_rms_norm(const void* x, const void* weight, void* y, int x_dtype, int64_t rows,
                int64_t dim, float eps, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPARK_B200_H */
