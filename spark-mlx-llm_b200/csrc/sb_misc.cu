// Small kernels of the decode step and the C-ABI wrappers of the linear family.
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>

#include "sb_common.cuh"
#include "sb_gemv.cuh"
#include "sb_tcgemm.cuh"
#include "spark_b200_decoder.h"

namespace sb {

// ------------------------------------------------------------ error state
namespace {
thread_local std::string g_last_error;
}

void set_error(const std::string& message) { g_last_error = message; }

int fail(int status, const std::string& message) {
  g_last_error = message;
  return status;
}

size_t sdpa_workspace_bytes(int64_t batch, int num_heads, int num_kv_heads, int64_t length, int D);

// ------------------------------------------------------------ TMA descriptors
namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}
}  // namespace

int make_tmap_rows(CUtensorMap* map, const void* base, uint64_t rows, uint64_t row_bytes, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(SB_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || row_bytes % 16)
    return fail(SB_EINVAL, "TMA source must be 16-byte aligned with rows a multiple of 16 bytes");
  const cuuint64_t dims[2] = {row_bytes, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {128, box_rows};
  const cuuint32_t elem[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SB_ECUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(r)) + ")");
  return SB_OK;
}

int make_tmap_u16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_cols,
                  uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(SB_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (cols * 2) % 16 || (box_cols * 2) % 16 || box_cols > 256)
    return fail(SB_EINVAL, "u16 TMA source must be 16-byte aligned with 16-byte rows and boxes");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t elem[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SB_ECUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(r)) + ")");
  return SB_OK;
}

int make_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t rows, uint64_t cols, uint64_t ld,
                 uint32_t box_cols, uint32_t box_rows, bool swizzle128) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(SB_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * elem_bytes) % 16 || (box_cols * elem_bytes) % 16 ||
      box_cols * elem_bytes > 128 || box_rows > 256 || (swizzle128 && box_cols * elem_bytes != 128))
    return fail(SB_EINVAL, "TMA source must be 16-byte aligned with rows and boxes a multiple of 16 bytes");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * static_cast<uint64_t>(elem_bytes)};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t elem[2] = {1, 1};
  const CUresult r =
      fn(map, elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
         const_cast<void*>(base), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
         swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SB_ECUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(r)) + ")");
  return SB_OK;
}

// ------------------------------------------------------------------ RMSNorm
template <typename T>
__global__ void rms_norm_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y, int dim,
                                float eps) {
  grid_dependency_wait();
  const int row = blockIdx.x;
  const T* xr = x + static_cast<size_t>(row) * dim;
  float ss = 0.f;
  for (int k = threadIdx.x; k < dim; k += blockDim.x) {
    const float v = to_float(xr[k]);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  __shared__ float part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x + 31) / 32 ? part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) part[0] = 1.0f / sqrtf(v / static_cast<float>(dim) + eps);
  }
  __syncthreads();
  const float r = part[0];
  grid_dependency_launch();
  for (int k = threadIdx.x; k < dim; k += blockDim.x)
    y[static_cast<size_t>(row) * dim + k] = from_float<T>(to_float(xr[k]) * r * to_float(w[k]));
}

// ------------------------------------------- INT8 KV append (per token/head)
// One warp per (batch, kv head, token): absmax over D, scale = fp16(absmax/127)
// (fp16 1.0 for a zero row), code = clamp(rint(x / scale), -127, 127).
__global__ void kv_append_kernel(const __nv_bfloat16* __restrict__ k_new, const __nv_bfloat16* __restrict__ v_new,
                                 int8_t* __restrict__ k_cache, __half* __restrict__ k_scale,
                                 int8_t* __restrict__ v_cache, __half* __restrict__ v_scale, int kv_heads, int seq_len,
                                 int head_dim, int capacity, const int* __restrict__ start) {
  grid_dependency_wait();
  const int lane = threadIdx.x & 31;
  const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);  // (b, h, l)
  const int l = item % seq_len;
  const int bh = item / seq_len;
  const int b = bh / kv_heads;
  const int pos = start[b] + l;
  if (pos >= capacity) return;
#pragma unroll
  for (int which = 0; which < 2; ++which) {
    const __nv_bfloat16* src = (which ? v_new : k_new) + (static_cast<size_t>(bh) * seq_len + l) * head_dim;
    int8_t* dst = (which ? v_cache : k_cache) + (static_cast<size_t>(bh) * capacity + pos) * head_dim;
    __half* sdst = (which ? v_scale : k_scale) + static_cast<size_t>(bh) * capacity + pos;
    float amax = 0.f;
    for (int d = lane; d < head_dim; d += 32) amax = fmaxf(amax, fabsf(__bfloat162float(src[d])));
    amax = warp_max(amax);
    __half s16 = __float2half_rn(__fdiv_rn(amax, 127.0f));
    if (__half2float(s16) == 0.f) s16 = __float2half_rn(1.0f);
    const float s = __half2float(s16);
    for (int d = lane; d < head_dim; d += 32) {
      float r = rintf(__fdiv_rn(__bfloat162float(src[d]), s));
      r = fminf(fmaxf(r, -127.0f), 127.0f);
      dst[d] = static_cast<int8_t>(static_cast<int>(r));
    }
    if (lane == 0) *sdst = s16;
  }
}

// -------------------------------------------------------- embedding gather
__global__ void embed_kernel(const __nv_bfloat16* __restrict__ table, const int* __restrict__ ids,
                             __nv_bfloat16* __restrict__ out, int hidden, int vocab) {
  grid_dependency_wait();
  const int row = blockIdx.x;
  int id = ids[row];
  id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);
  const uint4* src = reinterpret_cast<const uint4*>(table + static_cast<size_t>(id) * hidden);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * hidden);
  for (int i = threadIdx.x; i < hidden / 8; i += blockDim.x) dst[i] = src[i];
}

// One CTA per row of an MLX-affine quantized table: each thread dequantizes
// 8 consecutive values (one 32-bit word of 4-bit codes, two of 8-bit codes;
// element j of a word at bits [j*bits, (j+1)*bits)) as bf16(scale * q + bias).
__global__ void embed_affine_kernel(const uint32_t* __restrict__ w, const __nv_bfloat16* __restrict__ scales,
                                    const __nv_bfloat16* __restrict__ biases, const int* __restrict__ ids,
                                    __nv_bfloat16* __restrict__ out, int hidden, int vocab, int group, int bits) {
  grid_dependency_wait();
  const int row = blockIdx.x;
  int id = ids[row];
  id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);
  const int words = hidden * bits / 32, groups = hidden / group;
  const uint32_t* wr = w + static_cast<size_t>(id) * words;
  const __nv_bfloat16* sr = scales + static_cast<size_t>(id) * groups;
  const __nv_bfloat16* br = biases + static_cast<size_t>(id) * groups;
  for (int i = threadIdx.x; i < hidden / 8; i += blockDim.x) {
    const int g = (8 * i) / group;
    const float sc = __bfloat162float(sr[g]), bi = __bfloat162float(br[g]);
    uint32_t q[8];
    if (bits == 4) {
      const uint32_t word = wr[i];
#pragma unroll
      for (int j = 0; j < 8; ++j) q[j] = (word >> (4 * j)) & 15u;
    } else {
      const uint32_t w0 = wr[2 * i], w1 = wr[2 * i + 1];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        q[j] = (w0 >> (8 * j)) & 255u;
        q[4 + j] = (w1 >> (8 * j)) & 255u;
      }
    }
    __align__(16) __nv_bfloat16 o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = __float2bfloat16_rn(__fmaf_rn(sc, static_cast<float>(q[j]), bi));
    *reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * hidden + 8 * i) = *reinterpret_cast<const uint4*>(o);
  }
}

// ------------------------------------------------------------ residual add
__global__ void residual_add_kernel(__nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ y, int n) {
  grid_dependency_wait();
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i >= n) return;
  if (i + 8 <= n) {
    uint4 a = *reinterpret_cast<uint4*>(x + i);
    const uint4 b = *reinterpret_cast<const uint4*>(y + i);
    __nv_bfloat16* av = reinterpret_cast<__nv_bfloat16*>(&a);
    const __nv_bfloat16* bv = reinterpret_cast<const __nv_bfloat16*>(&b);
#pragma unroll
    for (int j = 0; j < 8; ++j) av[j] = __float2bfloat16_rn(__bfloat162float(av[j]) + __bfloat162float(bv[j]));
    *reinterpret_cast<uint4*>(x + i) = a;
  } else {
    for (int j = i; j < n; ++j) x[j] = __float2bfloat16_rn(__bfloat162float(x[j]) + __bfloat162float(y[j]));
  }
}

// ------------------------------------------- greedy token + position advance
// token[b] = argmax index decoded from keys[b]; keys reset; pos[b] += 1.
__global__ void decode_advance_kernel(unsigned long long* keys, int* tokens, int* positions, int batch,
                                      int advance) {
  grid_dependency_wait();
  const int b = threadIdx.x;
  if (b < batch) {
    const unsigned long long k = keys[b];
    tokens[b] = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull));
    keys[b] = 0ull;
    positions[b] += advance;
  }
}

}  // namespace sb

using namespace sb;

// ------------------------------------------------------------------ C ABI
extern "C" int sb_version(void) { return 100; }

extern "C" const char* sb_last_error_message(void) { return g_last_error.c_str(); }

extern "C" int sb_device_supported(int device) {
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return major == 10 ? 1 : 0;
}

namespace {

int weight_format(int bits) {
  if (bits == 4) return W_AFF4;
  if (bits == 8) return W_AFF8;
  return -1;
}

LinearRequest base_request(const void* x, int x_dtype, int64_t M, int64_t N, int64_t K) {
  LinearRequest r{};
  r.x = x;
  r.x_dtype = x_dtype;
  r.ldx = static_cast<int>(K);
  r.M = static_cast<int>(M);
  r.N = static_cast<int>(N);
  r.K = static_cast<int>(K);
  r.ldy = static_cast<int>(N);
  r.epi = EPI_STORE;
  return r;
}

int check_sizes(int64_t M, int64_t N, int64_t K) {
  SB_REQUIRE(M > 0 && N > 0 && K > 0, "Expected nonempty x[M, K] and weight[N, K]");
  SB_REQUIRE(N < (1LL << 31) && K < (1LL << 31) && M < (1LL << 31), "dimensions must fit in int32");
  return SB_OK;
}

size_t act_size(int dtype) { return dtype == SB_DTYPE_F32 ? 4 : 2; }

}  // namespace

extern "C" size_t sb_affine_linear_workspace_size(int64_t M, int64_t N, int64_t K, int group_size, int bits) {
  (void)M;
  (void)bits;
  if (N <= 0 || K <= 0 || group_size <= 0) return 0;
  return linear_workspace_size(EPI_STORE, static_cast<int>(N), static_cast<int>(K), group_size);
}

extern "C" int sb_affine_linear(const void* x, int x_dtype, const uint32_t* w, const void* scales,
                                const void* biases, void* y, int64_t M, int64_t N, int64_t K, int group_size,
                                int bits, void* workspace, size_t workspace_bytes, void* stream) {
  if (int st = check_sizes(M, N, K)) return st;
  SB_REQUIRE(x_dtype == SB_DTYPE_BF16 || x_dtype == SB_DTYPE_F16, "x must be bfloat16 or float16");
  const int wf = weight_format(bits);
  if (wf < 0) return fail(SB_EUNSUPPORTED, "affine bits must be 4 or 8");
  SB_REQUIRE(group_size == 32 || group_size == 64 || group_size == 128, "group_size must be 32, 64 or 128");
  SB_REQUIRE(K % group_size == 0, "K must be a multiple of group_size");
  if (M > 8) {  // tensor-core (tcgen05) kernel when the shapes allow it
    TcRequest t;
    t.tw = bits == 4 ? TW_AFF4 : TW_AFF8;
    t.te = TE_STORE;
    t.act_dtype = x_dtype;
    t.x = x;
    t.M = static_cast<int>(M);
    t.N = static_cast<int>(N);
    t.K = static_cast<int>(K);
    t.w = w;
    t.scales = scales;
    t.biases = biases;
    t.group_size = group_size;
    t.y = y;
    t.ldy = static_cast<int>(N);
    if (tc_linear_supported(t)) return run_tc_linear(t, as_stream(stream));
  }
  for (int64_t m0 = 0; m0 < M; m0 += 8) {
    LinearRequest r = base_request(static_cast<const uint8_t*>(x) + m0 * K * act_size(x_dtype), x_dtype,
                                   std::min<int64_t>(8, M - m0), N, K);
    r.wf = wf;
    r.w0 = w;
    r.s0 = scales;
    r.b0 = biases;
    r.group_size = group_size;
    r.y = static_cast<uint8_t*>(y) + m0 * N * act_size(x_dtype);
    r.workspace = workspace;
    r.workspace_bytes = workspace_bytes;
    if (int st = run_linear(r, as_stream(stream))) return st;
  }
  return SB_OK;
}

extern "C" size_t sb_w8a16_per_channel_workspace_size(int64_t M, int64_t N, int64_t K) {
  (void)M;
  if (N <= 0 || K <= 0) return 0;
  return linear_workspace_size(EPI_STORE, static_cast<int>(N), static_cast<int>(K), 64);
}

extern "C" int sb_w8a16_per_channel(const void* x, int x_dtype, const int8_t* w, const float* scales, void* y,
                                    int64_t M, int64_t N, int64_t K, void* workspace, size_t workspace_bytes,
                                    void* stream) {
  if (int st = check_sizes(M, N, K)) return st;
  SB_REQUIRE(x_dtype == SB_DTYPE_BF16 || x_dtype == SB_DTYPE_F16,
             "w8a16_per_channel x must have dtype bfloat16 or float16.");
  if (K % 64) return fail(SB_EUNSUPPORTED, "this build requires K to be a multiple of 64");
  if (M > 8) {  // tensor-core (tcgen05) kernel when the shapes allow it
    TcRequest t;
    t.tw = TW_I8;
    t.te = TE_CHSCALE;
    t.act_dtype = x_dtype;
    t.x = x;
    t.M = static_cast<int>(M);
    t.N = static_cast<int>(N);
    t.K = static_cast<int>(K);
    t.w = w;
    t.wscale = scales;
    t.y = y;
    t.ldy = static_cast<int>(N);
    if (tc_linear_supported(t)) return run_tc_linear(t, as_stream(stream));
  }
  for (int64_t m0 = 0; m0 < M; m0 += 8) {
    LinearRequest r = base_request(static_cast<const uint8_t*>(x) + m0 * K * act_size(x_dtype), x_dtype,
                                   std::min<int64_t>(8, M - m0), N, K);
    r.wf = W_I8PC;
    r.w0 = w;
    r.s0 = scales;
    r.y = static_cast<uint8_t*>(y) + m0 * N * act_size(x_dtype);
    r.workspace = workspace;
    r.workspace_bytes = workspace_bytes;
    if (int st = run_linear(r, as_stream(stream))) return st;
  }
  return SB_OK;
}

extern "C" size_t sb_qkv_rope_workspace_size(int64_t batch, int64_t seq_len, int64_t hidden, int num_heads,
                                             int num_kv_heads, int head_dim, int group_size, int bits) {
  (void)batch;
  (void)seq_len;
  (void)bits;
  const int64_t n = static_cast<int64_t>(num_heads + 2 * num_kv_heads) * head_dim;
  if (n <= 0 || hidden <= 0 || group_size <= 0) return 0;
  return linear_workspace_size(EPI_ROPE, static_cast<int>(n), static_cast<int>(hidden), group_size);
}

extern "C" int sb_qkv_rope(const void* x, int x_dtype, const uint32_t* w, const void* scales, const void* biases,
                           const int32_t* positions, void* q_out, void* k_out, void* v_out, int64_t batch,
                           int64_t seq_len, int64_t hidden, int num_heads, int num_kv_heads, int head_dim,
                           int rope_dims, float rope_base, int group_size, int bits, void* workspace,
                           size_t workspace_bytes, void* stream) {
  SB_REQUIRE(batch > 0 && seq_len > 0 && hidden > 0, "x must have shape [B, L, hidden] with hidden > 0.");
  SB_REQUIRE(num_heads > 0 && num_kv_heads > 0 && head_dim > 0 && num_heads % num_kv_heads == 0,
             "Invalid head counts, head_dim, q_size, or kv_size.");
  SB_REQUIRE(rope_dims > 0 && rope_dims % 2 == 0 && rope_dims <= head_dim && std::isfinite(rope_base) &&
                 rope_base > 0,
             "rope_dims must be positive, even, and no larger than head_dim; rope_base must be positive and "
             "finite.");
  if (rope_dims != head_dim) return fail(SB_EUNSUPPORTED, "the fused kernel rotates the full head_dim");
  SB_REQUIRE(x_dtype == SB_DTYPE_BF16 || x_dtype == SB_DTYPE_F16, "x must be bfloat16 or float16");
  const int wf = weight_format(bits);
  if (wf < 0) return fail(SB_EUNSUPPORTED, "bits must be 4 or 8 in this build");
  SB_REQUIRE(group_size == 32 || group_size == 64 || group_size == 128, "group_size must be 32, 64, or 128.");
  SB_REQUIRE(hidden % group_size == 0, "Packed weight and quantization metadata shapes do not match x.");
  if (batch * seq_len > 8) {  // tensor-core (tcgen05) kernel, one 128-row weight tile per head
    TcRequest t;
    t.tw = bits == 4 ? TW_AFF4 : TW_AFF8;
    t.te = TE_ROPE;
    t.act_dtype = x_dtype;
    t.x = x;
    t.M = static_cast<int>(batch * seq_len);
    t.N = (num_heads + 2 * num_kv_heads) * head_dim;
    t.K = static_cast<int>(hidden);
    t.w = w;
    t.scales = scales;
    t.biases = biases;
    t.group_size = group_size;
    t.positions = positions;
    t.heads_q = num_heads;
    t.heads_kv = num_kv_heads;
    t.seq_len = static_cast<int>(seq_len);
    t.rope_base = rope_base;
    t.q_out = q_out;
    t.k_out = k_out;
    t.v_out = v_out;
    SB_REQUIRE(positions != nullptr, "positions are required");
    if (head_dim != 128 || !tc_linear_supported(t))
      return fail(SB_EUNSUPPORTED, "QKV + RoPE for more than 8 tokens needs head_dim 128, hidden / group_size a "
                                   "multiple of 8 and 16-byte aligned tensors");
    return run_tc_linear(t, as_stream(stream));
  }
  LinearRequest r = base_request(x, x_dtype, batch * seq_len,
                                 static_cast<int64_t>(num_heads + 2 * num_kv_heads) * head_dim, hidden);
  r.wf = wf;
  r.w0 = w;
  r.s0 = scales;
  r.b0 = biases;
  r.group_size = group_size;
  r.epi = EPI_ROPE;
  r.positions = positions;
  r.heads_q = num_heads;
  r.heads_kv = num_kv_heads;
  r.head_dim = head_dim;
  r.seq_len = static_cast<int>(seq_len);
  r.rope_dims = rope_dims;
  r.rope_base = rope_base;
  r.q_out = q_out;
  r.k_out = k_out;
  r.v_out = v_out;
  r.workspace = workspace;
  r.workspace_bytes = workspace_bytes;
  return run_linear(r, as_stream(stream));
}

extern "C" int sb_rms_norm(const void* x, const void* weight, void* y, int x_dtype, int64_t rows, int64_t dim,
                           float eps, void* stream) {
  SB_REQUIRE(rows > 0 && dim > 0, "x must be nonempty");
  const dim3 grid(static_cast<unsigned>(rows)), block(256);
  switch (x_dtype) {
    case SB_DTYPE_BF16:
      return launch("rms_norm", rms_norm_kernel<__nv_bfloat16>, grid, block, 0, as_stream(stream),
                    static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(weight),
                    static_cast<__nv_bfloat16*>(y), static_cast<int>(dim), eps);
    case SB_DTYPE_F16:
      return launch("rms_norm", rms_norm_kernel<__half>, grid, block, 0, as_stream(stream),
                    static_cast<const __half*>(x), static_cast<const __half*>(weight), static_cast<__half*>(y),
                    static_cast<int>(dim), eps);
    case SB_DTYPE_F32:
      return launch("rms_norm", rms_norm_kernel<float>, grid, block, 0, as_stream(stream),
                    static_cast<const float*>(x), static_cast<const float*>(weight), static_cast<float*>(y),
                    static_cast<int>(dim), eps);
  }
  return fail(SB_EINVAL, "x must be bfloat16, float16 or float32");
}

// ------------------------------------------------------- decoder entry points
extern "C" size_t sb_linear_ex_workspace_size(const sb_linear_ex_desc* d) {
  if (!d || d->N <= 0 || d->K <= 0) return 0;
  const int gk = (d->weight_format == SB_WEIGHT_AFFINE4 || d->weight_format == SB_WEIGHT_AFFINE8) ? d->group_size : 64;
  if (gk <= 0) return 0;
  return linear_workspace_size(d->epilogue, static_cast<int>(d->N), static_cast<int>(d->K), gk);
}

namespace {
int linear_ex(const sb_linear_ex_desc* d, void* stream, int* plan_out) {
  SB_REQUIRE(d != nullptr, "null descriptor");
  if (int st = check_sizes(d->M, d->N, d->K)) return st;
  SB_REQUIRE(d->epilogue >= SB_EPI_STORE && d->epilogue <= SB_EPI_ARGMAX, "unknown epilogue");
  SB_REQUIRE(d->weight_format >= SB_WEIGHT_AFFINE4 && d->weight_format <= SB_WEIGHT_BF16, "unknown weight format");
  LinearRequest r = base_request(d->x, d->x_dtype, d->M, d->N, d->K);
  r.ldx = d->ldx > 0 ? static_cast<int>(d->ldx) : static_cast<int>(d->K);
  r.ldy = d->ldy > 0 ? static_cast<int>(d->ldy) : static_cast<int>(d->N);
  r.wf = d->weight_format;
  r.w0 = d->weight;
  r.s0 = d->scales;
  r.b0 = d->biases;
  r.w1 = d->weight2;
  r.s1 = d->scales2;
  r.b1 = d->biases2;
  r.group_size = d->group_size;
  r.epi = d->epilogue;
  r.norm = d->norm_weight != nullptr;
  r.norm_w = d->norm_weight;
  r.eps = d->norm_eps;
  r.y = d->y;
  r.residual = d->residual;
  r.ldr = d->ldr > 0 ? static_cast<int>(d->ldr) : r.ldy;
  r.positions = d->positions;
  r.heads_q = d->num_heads;
  r.heads_kv = d->num_kv_heads;
  r.head_dim = d->head_dim;
  r.seq_len = d->seq_len > 0 ? d->seq_len : 1;
  r.rope_dims = d->head_dim;
  r.rope_base = d->rope_base;
  r.q_out = d->q_out;
  r.k_out = d->k_out;
  r.v_out = d->v_out;
  r.kv_k_cache = d->kv_k_cache;
  r.kv_k_scale = d->kv_k_scale;
  r.kv_v_cache = d->kv_v_cache;
  r.kv_v_scale = d->kv_v_scale;
  r.kv_capacity = d->kv_capacity;
  r.ar_world = d->ar_world;
  r.ar_rank = d->ar_rank;
  r.ar_channel = d->ar_channel;
  for (int i = 0; i < 8; ++i) r.ar_buffers[i] = d->ar_buffers[i];
  r.argmax_keys = d->argmax_keys;
  r.argmax_offset = d->argmax_offset;
  r.workspace = d->workspace;
  r.workspace_bytes = d->workspace_bytes;
  r.weights_constant = d->weights_constant != 0;
  SB_REQUIRE(d->activation == 0 || d->activation == 1, "activation must be 0 (SiLU) or 1 (GELU)");
  r.activation = d->activation;
  SB_REQUIRE(d->k_chunks >= 0 && d->k_chunks <= 8, "k_chunks must be 0..8");
  SB_REQUIRE(d->plan_rows >= 0 && d->plan_rows < (1LL << 31) && d->plan_k_chunks >= 0 && d->plan_k_chunks <= 8,
             "plan_rows must be >= 0 and plan_k_chunks 0..8");
  r.k_chunks = d->k_chunks;
  r.plan_rows = static_cast<int>(d->plan_rows);
  r.plan_chunks = d->plan_k_chunks;
  SB_REQUIRE(d->y_fp32 == 0 || d->y_fp32 == 1, "y_fp32 must be 0 or 1");
  r.y_f32 = d->y_fp32 != 0;
  SB_REQUIRE(d->scales_ld >= 0 && d->scales_ld < (1LL << 31), "scales_ld must be >= 0");
  r.scales_ld = static_cast<int>(d->scales_ld);
  r.plan_out = plan_out;
  return run_linear(r, as_stream(stream));
}
}  // namespace

extern "C" int sb_linear_ex(const sb_linear_ex_desc* d, void* stream) { return linear_ex(d, stream, nullptr); }

extern "C" int sb_linear_ex_plan(const sb_linear_ex_desc* d, int* plan) {
  SB_REQUIRE(plan != nullptr, "null plan array");
  return linear_ex(d, nullptr, plan);
}

extern "C" int sb_kv_append_int8(const void* k_new, const void* v_new, int8_t* k_cache, void* k_scale,
                                 int8_t* v_cache, void* v_scale, int64_t batch, int num_kv_heads, int64_t seq_len,
                                 int head_dim, int64_t capacity, const int32_t* start, void* stream) {
  SB_REQUIRE(batch > 0 && num_kv_heads > 0 && seq_len > 0 && head_dim > 0 && capacity > 0, "empty KV append");
  const int items = static_cast<int>(batch * num_kv_heads * seq_len);
  const int warps = 4;
  return launch("kv_append", kv_append_kernel, dim3((items + warps - 1) / warps), dim3(32 * warps), 0,
                as_stream(stream), static_cast<const __nv_bfloat16*>(k_new), static_cast<const __nv_bfloat16*>(v_new),
                k_cache, static_cast<__half*>(k_scale), v_cache, static_cast<__half*>(v_scale), num_kv_heads,
                static_cast<int>(seq_len), head_dim, static_cast<int>(capacity), start);
}

extern "C" int sb_embed_rows(const void* table, const int32_t* ids, void* out, int64_t rows, int64_t hidden,
                             int64_t vocab, void* stream) {
  SB_REQUIRE(rows > 0 && hidden > 0 && hidden % 8 == 0 && vocab > 0, "bad embedding shape");
  return launch("embed", embed_kernel, dim3(static_cast<unsigned>(rows)), dim3(128), 0, as_stream(stream),
                static_cast<const __nv_bfloat16*>(table), ids, static_cast<__nv_bfloat16*>(out),
                static_cast<int>(hidden), static_cast<int>(vocab));
}

extern "C" int sb_embed_rows_affine(const void* weight, const void* scales, const void* biases, const int32_t* ids,
                                    void* out, int64_t rows, int64_t hidden, int64_t vocab, int group_size, int bits,
                                    void* stream) {
  SB_REQUIRE(weight && scales && biases && ids && out, "null pointer");
  SB_REQUIRE(bits == 4 || bits == 8, "bits must be 4 or 8");
  SB_REQUIRE(group_size == 32 || group_size == 64 || group_size == 128, "group_size must be 32, 64 or 128");
  SB_REQUIRE(rows > 0 && rows < (1LL << 31) && vocab > 0 && vocab < (1LL << 31) && hidden > 0 &&
                 hidden % group_size == 0 && hidden < (1LL << 24),
             "bad embedding shape (hidden a multiple of group_size)");
  SB_REQUIRE((reinterpret_cast<uintptr_t>(out) & 15) == 0 && (reinterpret_cast<uintptr_t>(weight) & 3) == 0,
             "out must be 16-byte and weight 4-byte aligned");
  return launch("embed_affine", embed_affine_kernel, dim3(static_cast<unsigned>(rows)), dim3(128), 0,
                as_stream(stream), static_cast<const uint32_t*>(weight), static_cast<const __nv_bfloat16*>(scales),
                static_cast<const __nv_bfloat16*>(biases), ids, static_cast<__nv_bfloat16*>(out),
                static_cast<int>(hidden), static_cast<int>(vocab), group_size, bits);
}

extern "C" int sb_decode_advance(unsigned long long* argmax_keys, int32_t* tokens, int32_t* positions, int batch,
                                 int advance, void* stream) {
  SB_REQUIRE(batch > 0 && batch <= 1024, "batch must be in [1, 1024]");
  return launch("decode_advance", decode_advance_kernel, dim3(1), dim3(((batch + 31) / 32) * 32), 0,
                as_stream(stream), argmax_keys, tokens, positions, batch, advance);
}


extern "C" int sb_residual_add(void* x, const void* y, int64_t count, void* stream) {
  SB_REQUIRE(count > 0 && count < (1LL << 31), "bad element count");
  SB_REQUIRE(((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0, "x and y must be 16-byte aligned");
  const int threads = 256;
  const int64_t vecs = (count + 7) / 8;
  return launch("residual_add", residual_add_kernel, dim3(static_cast<unsigned>((vecs + threads - 1) / threads)),
                dim3(threads), 0, as_stream(stream), static_cast<__nv_bfloat16*>(x),
                static_cast<const __nv_bfloat16*>(y), static_cast<int>(count));
}

// ------------------------------------------------------ peer exchange buffers
extern "C" size_t sb_tp_exchange_bytes(int world, int64_t n) {
  if (world < 2 || world > 8 || n <= 0) return 0;
  return 2 * ar_channel_bytes(world, n);
}

extern "C" int sb_peer_buffer_alloc(size_t bytes, void** ptr, void* handle64) {
  SB_REQUIRE(bytes > 0 && ptr != nullptr && handle64 != nullptr, "bad peer buffer request");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  void* p = nullptr;
  cudaError_t err = cudaMalloc(&p, bytes);
  if (err != cudaSuccess) return fail(SB_ECUDA, std::string("peer buffer cudaMalloc: ") + cudaGetErrorString(err));
  err = cudaMemset(p, 0, bytes);
  if (err == cudaSuccess) err = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle64), p);
  if (err != cudaSuccess) {
    cudaFree(p);
    return fail(SB_ECUDA, std::string("peer buffer export: ") + cudaGetErrorString(err));
  }
  *ptr = p;
  return SB_OK;
}

extern "C" int sb_peer_buffer_open(const void* handle64, void** ptr) {
  SB_REQUIRE(handle64 != nullptr && ptr != nullptr, "bad peer buffer handle");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  const cudaError_t err = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) return fail(SB_ECUDA, std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(err));
  return SB_OK;
}

extern "C" int sb_peer_buffer_close(void* ptr) {
  const cudaError_t err = cudaIpcCloseMemHandle(ptr);
  if (err != cudaSuccess) return fail(SB_ECUDA, std::string("cudaIpcCloseMemHandle: ") + cudaGetErrorString(err));
  return SB_OK;
}

extern "C" int sb_peer_buffer_free(void* ptr) {
  const cudaError_t err = cudaFree(ptr);
  if (err != cudaSuccess) return fail(SB_ECUDA, std::string("peer buffer cudaFree: ") + cudaGetErrorString(err));
  return SB_OK;
}
