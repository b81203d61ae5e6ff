// W8A8: per-token INT8 activation quantization, exact INT8 x INT8 -> INT32
// products on the tensor cores (mma.sync m16n8k32 s8), fp32 dequant epilogue.
//
// Arithmetic contract (bit-exact with the reference):
//   quantizer  extensions/spark-mlx-ext/src/kernels/w8a8_quantize.metal:11-27
//              scale = amax > 0 ? amax / 127 : 1 (IEEE fp32 divide),
//              q = clamp(rint(x / scale), -127, 127)   (round half to even)
//   int32 acc  exact (K <= 131040, src/spark_w8a8.cpp:57-61)
//   epilogue   float(acc) * scale_a[m] * scale_w[n] + bias[n], left to right,
//              no contraction (w8a8_matmul.metal:73-74), then one cast.
// The kernel layout mirrors the weight-streaming linear in sb_gemv.cu: a warp
// owns 32 weight rows over a K range, activations (M <= 8) are quantized into
// shared memory by each CTA, K is split across warps when N is small and the
// last warp of a row block reduces the int32 partials.
#include <algorithm>
#include <mutex>

#include "sb_common.cuh"
#include "sb_tcgemm.cuh"

namespace sb {

constexpr int kI8Warps = 4;
constexpr int kI8Tiles = 2;
constexpr int kI8Seg = 4096;  // K values of activations staged in shared memory at a time

struct I8Params {
  const void* x;  // [M][K] (int8 when x_dtype < 0, else float type to quantize)
  int x_dtype;    // -1: int8 input (raw matmul)
  const int8_t* w;
  const float* w_scales;
  const void* bias;
  int bias_dtype;  // -1: none
  void* y;         // int32 (raw) or x dtype
  int M, N, K;
  int splits, groups_total;
  int* partial;    // [splits][rows_padded][8]
  unsigned* counters;
  int rows_padded;
  int early_prefetch;  // 1: weights are constant, stream them before waiting
};

template <typename T>
__device__ __forceinline__ float load_f(const void* p, size_t i) {
  return to_float(static_cast<const T*>(p)[i]);
}

__device__ __forceinline__ float load_any(const void* p, int dtype, size_t i) {
  if (dtype == SB_DTYPE_BF16) return load_f<__nv_bfloat16>(p, i);
  if (dtype == SB_DTYPE_F16) return load_f<__half>(p, i);
  return static_cast<const float*>(p)[i];
}

__device__ __forceinline__ int8_t quantize_value(float v, float scale) {
  float r = rintf(__fdiv_rn(v, scale));
  r = fminf(fmaxf(r, -127.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(r));
}

// One CTA per row: amax reduction, then quantize (reference quantize_per_token).
template <typename T>
__global__ void quantize_per_token_kernel(const T* __restrict__ x, int8_t* __restrict__ q,
                                          float* __restrict__ scales, int K) {
  grid_dependency_wait();
  const int row = blockIdx.x;
  const T* xr = x + static_cast<size_t>(row) * K;
  float amax = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) amax = fmaxf(amax, fabsf(to_float(xr[k])));
  amax = warp_max(amax);
  __shared__ float s_max[32];
  if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x + 31) / 32 ? s_max[threadIdx.x] : 0.f;
    v = warp_max(v);
    if (threadIdx.x == 0) s_max[0] = v;
  }
  __syncthreads();
  const float m = s_max[0];
  const float scale = m > 0.f ? __fdiv_rn(m, 127.0f) : 1.0f;
  if (threadIdx.x == 0) scales[row] = scale;
  grid_dependency_launch();
  for (int k = threadIdx.x; k < K; k += blockDim.x)
    q[static_cast<size_t>(row) * K + k] = quantize_value(to_float(xr[k]), scale);
}

template <bool kQuantize, bool kRaw>
__global__ void __launch_bounds__(kI8Warps * 32, 4) i8_gemv_kernel(const __grid_constant__ I8Params p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ float s_part[kI8Warps][8];
  __shared__ float s_scale[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int split = blockIdx.y;
  const int tiles = (p.N + 15) / 16;
  const int rowblocks = (tiles + kI8Tiles - 1) / kI8Tiles;
  const int rb = blockIdx.x * kI8Warps + warp;
  const bool active = rb < rowblocks;
  const int grp_begin = static_cast<int>((static_cast<long long>(p.groups_total) * split) / p.splits);
  const int grp_end = static_cast<int>((static_cast<long long>(p.groups_total) * (split + 1)) / p.splits);
  const int k_begin = grp_begin * 64, k_count = (grp_end - grp_begin) * 64;
  const int c_begin = grp_begin, c_end = grp_end;  // 64-K chunks

  constexpr int kRows = 2 * kI8Tiles;
  const int8_t* wrow[kRows];
#pragma unroll
  for (int q = 0; q < kRows; ++q) {
    const int row = min((min(rb, rowblocks - 1) * kI8Tiles + (q >> 1)) * 16 + (q & 1) * 8 + g, p.N - 1);
    wrow[q] = p.w + static_cast<size_t>(row) * p.K + t * 16;
  }
  if (!p.early_prefetch) grid_dependency_wait();
  uint32_t wbuf[kRows][4];
  if (active && c_begin < c_end) {
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
      const uint4 v = ldg_stream16(wrow[q] + static_cast<size_t>(c_begin) * 64);
      wbuf[q][0] = v.x;
      wbuf[q][1] = v.y;
      wbuf[q][2] = v.z;
      wbuf[q][3] = v.w;
    }
  }
  grid_dependency_wait();

  // per-token scales over the full row (quantizing path)
  if constexpr (kQuantize) {
    for (int m = 0; m < p.M; ++m) {
      float amax = 0.f;
      for (int k = threadIdx.x; k < p.K; k += kI8Warps * 32)
        amax = fmaxf(amax, fabsf(load_any(p.x, p.x_dtype, static_cast<size_t>(m) * p.K + k)));
      amax = warp_max(amax);
      if (lane == 0) s_part[warp][m] = amax;
    }
    __syncthreads();
    if (threadIdx.x < p.M) {
      float amax = 0.f;
#pragma unroll
      for (int w = 0; w < kI8Warps; ++w) amax = fmaxf(amax, s_part[w][threadIdx.x]);
      s_scale[threadIdx.x] = amax > 0.f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    }
  }

  int8_t* xs = reinterpret_cast<int8_t*>(smem_raw);
  const int xs_ld = kI8Seg + 16;
  int acc[kI8Tiles][4];
#pragma unroll
  for (int r = 0; r < kI8Tiles; ++r)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[r][e] = 0;
  const int8_t* xcol = xs + min(g, p.M - 1) * xs_ld + t * 16;
  for (int seg0 = 0; seg0 < k_count; seg0 += kI8Seg) {
    // stage int8 activations of this K segment (all warps take part)
    const int seg_len = min(kI8Seg, k_count - seg0);
    __syncthreads();
    if constexpr (kQuantize) {
      for (int idx = threadIdx.x; idx < p.M * seg_len; idx += kI8Warps * 32) {
        const int m = idx / seg_len, k = idx % seg_len;
        xs[m * xs_ld + k] = quantize_value(
            load_any(p.x, p.x_dtype, static_cast<size_t>(m) * p.K + k_begin + seg0 + k), s_scale[m]);
      }
    } else {
      const int vecs = seg_len / 16;
      for (int idx = threadIdx.x; idx < p.M * vecs; idx += kI8Warps * 32) {
        const int m = idx / vecs, v = idx % vecs;
        *reinterpret_cast<uint4*>(xs + m * xs_ld + v * 16) = *reinterpret_cast<const uint4*>(
            static_cast<const int8_t*>(p.x) + static_cast<size_t>(m) * p.K + k_begin + seg0 + v * 16);
      }
    }
    __syncthreads();
    if (!active) continue;
    const int cs = c_begin + seg0 / 64, ce = cs + seg_len / 64;
    for (int c = cs; c < ce; ++c) {
      uint32_t cur[kRows][4];
#pragma unroll
      for (int q = 0; q < kRows; ++q)
#pragma unroll
        for (int i = 0; i < 4; ++i) cur[q][i] = wbuf[q][i];
      if (c + 1 < c_end) {
#pragma unroll
        for (int q = 0; q < kRows; ++q) {
          const uint4 v = ldg_stream16(wrow[q] + static_cast<size_t>(c + 1) * 64);
          wbuf[q][0] = v.x;
          wbuf[q][1] = v.y;
          wbuf[q][2] = v.z;
          wbuf[q][3] = v.w;
        }
      }
      const uint4 xv = *reinterpret_cast<const uint4*>(xcol + (c - cs) * 64);
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int r = 0; r < kI8Tiles; ++r) {
          const uint32_t a[4] = {cur[2 * r][2 * j], cur[2 * r + 1][2 * j], cur[2 * r][2 * j + 1],
                                 cur[2 * r + 1][2 * j + 1]};
          mma_s8_16832(acc[r], a, xw[2 * j], xw[2 * j + 1]);
        }
      }
    }
  }
  if (!active) return;
  grid_dependency_launch();

  if (p.splits > 1) {
    int* part = p.partial + (static_cast<size_t>(split) * p.rows_padded + rb * 16 * kI8Tiles) * 8;
#pragma unroll
    for (int r = 0; r < kI8Tiles; ++r)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        if (2 * t < p.M)
          *reinterpret_cast<int2*>(part + (r * 16 + h * 8 + g) * 8 + 2 * t) = make_int2(acc[r][2 * h], acc[r][2 * h + 1]);
    __threadfence();
    __syncwarp();
    unsigned prev = 0;
    if (lane == 0) prev = atomicAdd(p.counters + rb, 1u);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != static_cast<unsigned>(p.splits - 1)) return;
    __threadfence();
#pragma unroll
    for (int r = 0; r < kI8Tiles; ++r)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[r][e] = 0;
    for (int s = 0; s < p.splits; ++s) {
      const int* ps = p.partial + (static_cast<size_t>(s) * p.rows_padded + rb * 16 * kI8Tiles) * 8;
#pragma unroll
      for (int r = 0; r < kI8Tiles; ++r)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          if (2 * t < p.M) {
            const int2 v = __ldcg(reinterpret_cast<const int2*>(ps + (r * 16 + h * 8 + g) * 8 + 2 * t));
            acc[r][2 * h] += v.x;
            acc[r][2 * h + 1] += v.y;
          }
    }
    if (lane == 0) p.counters[rb] = 0u;
  }

#pragma unroll
  for (int r = 0; r < kI8Tiles; ++r) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = (rb * kI8Tiles + r) * 16 + h * 8 + g;
      if (row >= p.N) continue;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int m = 2 * t + e;
        if (m >= p.M) continue;
        const int a = acc[r][2 * h + e];
        const size_t idx = static_cast<size_t>(m) * p.N + row;
        if constexpr (kRaw) {
          static_cast<int32_t*>(p.y)[idx] = a;
        } else {
          float v = __fmul_rn(__fmul_rn(static_cast<float>(a), s_scale[m]), p.w_scales[row]);
          const float b = p.bias_dtype < 0 ? 0.f : load_any(p.bias, p.bias_dtype, row);
          v = __fadd_rn(v, b);
          if (p.x_dtype == SB_DTYPE_BF16) static_cast<__nv_bfloat16*>(p.y)[idx] = __float2bfloat16_rn(v);
          else if (p.x_dtype == SB_DTYPE_F16) static_cast<__half*>(p.y)[idx] = __float2half_rn(v);
          else static_cast<float*>(p.y)[idx] = v;
        }
      }
    }
  }
}

namespace {

int sms() { return device_sm_count(); }

struct I8Plan {
  int rowblocks, groups, splits;
  size_t counter_bytes, partial_bytes;
};

I8Plan plan_i8(int N, int K, bool allow_split) {
  I8Plan pl{};
  pl.rowblocks = ((N + 15) / 16 + kI8Tiles - 1) / kI8Tiles;
  pl.groups = K / 64;
  int s = allow_split ? (sms() * 12 + pl.rowblocks - 1) / pl.rowblocks : 1;
  s = std::min(s, std::max(1, pl.groups / 2));
  s = std::max(1, std::min(s, pl.groups));
  pl.splits = pl.rowblocks > kMaxCounters ? 1 : s;
  pl.counter_bytes = kCounterBytes;
  pl.partial_bytes = pl.splits > 1 ? static_cast<size_t>(pl.splits) * pl.rowblocks * 16 * kI8Tiles * 8 * sizeof(int) : 0;
  return pl;
}

template <bool kQuantize, bool kRaw>
int launch_i8(I8Params& p, const I8Plan& pl, void* ws, size_t ws_bytes, cudaStream_t stream) {
  p.splits = pl.splits;
  p.groups_total = pl.groups;
  p.rows_padded = pl.rowblocks * 16 * kI8Tiles;
  if (pl.splits > 1) {
    p.counters = static_cast<unsigned*>(ws);
    p.partial = reinterpret_cast<int*>(static_cast<uint8_t*>(ws) + pl.counter_bytes);
  }
  const size_t smem = static_cast<size_t>(p.M) * (kI8Seg + 16);
  auto kernel = i8_gemv_kernel<kQuantize, kRaw>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return fail(SB_ECUDA, "w8a8: shared memory opt-in failed");
  dim3 grid((pl.rowblocks + kI8Warps - 1) / kI8Warps, pl.splits);
  return launch("w8a8 gemv", kernel, grid, dim3(kI8Warps * 32), smem, stream, p);
}

int check_i8_shapes(int64_t M, int64_t N, int64_t K) {
  SB_REQUIRE(M > 0 && N > 0 && K > 0, "Expected nonempty x[M, K] and weight[N, K] with matching K.");
  SB_REQUIRE(K % 32 == 0 && K <= 131040, "K must be a multiple of 32 in [32, 131040].");
  SB_REQUIRE(M <= 0x7fffffff && N <= 0x7fffffff, "M and N must fit in int32");
  return SB_OK;
}

}  // namespace

}  // namespace sb

using namespace sb;

extern "C" int sb_quantize_per_token(const void* x, int x_dtype, int8_t* q, float* scales, int64_t M,
                                     int64_t K, void* stream) {
  SB_REQUIRE(M > 0 && K > 0, "x must be a nonempty [M, K] matrix");
  SB_REQUIRE(x && q && scales, "null pointer");
  const int threads = static_cast<int>(std::min<int64_t>(256, ((K + 31) / 32) * 32));
  const dim3 grid(static_cast<unsigned>(M));
  switch (x_dtype) {
    case SB_DTYPE_BF16:
      return launch("quantize_per_token", quantize_per_token_kernel<__nv_bfloat16>, grid, dim3(threads), 0,
                    as_stream(stream), static_cast<const __nv_bfloat16*>(x), q, scales, static_cast<int>(K));
    case SB_DTYPE_F16:
      return launch("quantize_per_token", quantize_per_token_kernel<__half>, grid, dim3(threads), 0,
                    as_stream(stream), static_cast<const __half*>(x), q, scales, static_cast<int>(K));
    case SB_DTYPE_F32:
      return launch("quantize_per_token", quantize_per_token_kernel<float>, grid, dim3(threads), 0,
                    as_stream(stream), static_cast<const float*>(x), q, scales, static_cast<int>(K));
  }
  return fail(SB_EINVAL, "x must have dtype float16, bfloat16, or float32.");
}

extern "C" size_t sb_w8a8_linear_workspace_size(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0 || K % 64) return 0;
  const I8Plan pl = plan_i8(static_cast<int>(N), static_cast<int>(K), true);
  size_t need = pl.counter_bytes + pl.partial_bytes;
  // M > 8: per-token INT8 activations and their scales for the tensor-core kernel
  if (M > 8) need = std::max(need, tc_w8a8_bytes(M, K));
  return need;
}

extern "C" int sb_int8_matmul_int32(const int8_t* x, const int8_t* w, int32_t* out, int64_t M, int64_t N,
                                    int64_t K, void* stream) {
  if (int st = check_i8_shapes(M, N, K)) return st;
  SB_REQUIRE(K % 64 == 0, "this build requires K to be a multiple of 64");
  SB_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0,
             "x and weight must be 16-byte aligned");
  if (M > 8) {  // tensor-core (tcgen05 kind::i8) kernel, exact int32 accumulators
    TcRequest t;
    t.tw = TW_S8;
    t.te = TE_I32;
    t.x = x;
    t.M = static_cast<int>(M);
    t.N = static_cast<int>(N);
    t.K = static_cast<int>(K);
    t.w = w;
    t.y = out;
    t.ldy = static_cast<int>(N);
    if (tc_linear_supported(t)) return run_tc_linear(t, as_stream(stream));
  }
  I8Plan pl = plan_i8(static_cast<int>(N), static_cast<int>(K), false);
  for (int64_t m0 = 0; m0 < M; m0 += 8) {
    I8Params p{};
    p.x = x + m0 * K;
    p.x_dtype = -1;
    p.w = w;
    p.bias_dtype = -1;
    p.y = out + m0 * N;
    p.M = static_cast<int>(std::min<int64_t>(8, M - m0));
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    if (int st = launch_i8<false, true>(p, pl, nullptr, 0, as_stream(stream))) return st;
  }
  return SB_OK;
}

extern "C" int sb_w8a8_linear(const void* x, int x_dtype, const int8_t* w, const float* scales,
                              const void* bias, int bias_dtype, void* y, int64_t M, int64_t N, int64_t K,
                              void* workspace, size_t workspace_bytes, void* stream) {
  if (int st = check_i8_shapes(M, N, K)) return st;
  SB_REQUIRE(K % 64 == 0, "this build requires K to be a multiple of 64");
  SB_REQUIRE(x_dtype == SB_DTYPE_BF16 || x_dtype == SB_DTYPE_F16 || x_dtype == SB_DTYPE_F32,
             "x must have dtype float16, bfloat16, or float32.");
  SB_REQUIRE(bias == nullptr || bias_dtype == SB_DTYPE_BF16 || bias_dtype == SB_DTYPE_F16 ||
                 bias_dtype == SB_DTYPE_F32,
             "bias must have a real floating dtype.");
  SB_REQUIRE((reinterpret_cast<uintptr_t>(w) & 15) == 0, "weight must be 16-byte aligned");
  if (M > 8 && workspace != nullptr && workspace_bytes >= tc_w8a8_bytes(M, K)) {
    // per-token quantization into the workspace (past its counter region), then
    // the tensor-core kernel with the W8A8 epilogue
    int8_t* xq = static_cast<int8_t*>(workspace) + kCounterBytes;
    float* sa = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterBytes + ((M * K + 255) / 256) * 256);
    TcRequest t;
    t.tw = TW_S8;
    t.te = TE_W8A8;
    t.x = xq;
    t.M = static_cast<int>(M);
    t.N = static_cast<int>(N);
    t.K = static_cast<int>(K);
    t.w = w;
    t.y = y;
    t.ldy = static_cast<int>(N);
    t.y_dtype = x_dtype;
    t.wscale = scales;
    t.ascale = sa;
    t.bias = bias;
    t.bias_dtype = bias ? bias_dtype : -1;
    if (tc_linear_supported(t)) {
      if (int st = sb_quantize_per_token(x, x_dtype, xq, sa, M, K, stream)) return st;
      return run_tc_linear(t, as_stream(stream));
    }
  }
  I8Plan pl = plan_i8(static_cast<int>(N), static_cast<int>(K), true);
  if (pl.splits > 1 && (workspace == nullptr || workspace_bytes < pl.counter_bytes + pl.partial_bytes))
    pl = plan_i8(static_cast<int>(N), static_cast<int>(K), false);
  const size_t esize = x_dtype == SB_DTYPE_F32 ? 4 : 2;
  for (int64_t m0 = 0; m0 < M; m0 += 8) {
    I8Params p{};
    p.x = static_cast<const uint8_t*>(x) + m0 * K * esize;
    p.x_dtype = x_dtype;
    p.w = w;
    p.w_scales = scales;
    p.bias = bias;
    p.bias_dtype = bias ? bias_dtype : -1;
    p.y = static_cast<uint8_t*>(y) + m0 * N * esize;
    p.M = static_cast<int>(std::min<int64_t>(8, M - m0));
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    if (int st = launch_i8<true, false>(p, pl, workspace, workspace_bytes, as_stream(stream))) return st;
  }
  return SB_OK;
}
