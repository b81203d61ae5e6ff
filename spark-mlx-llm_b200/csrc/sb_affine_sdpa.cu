// Attention over MLX affine-quantized KV tuples (packed codes, scales, biases):
// the input format of ``int8_quantized_sdpa`` (spark_mlx_ext/
// int8_quantized_sdpa.py:156-287). K and V are uint32-packed codes [B,KH,N,W]
// (element j of a word at bits [j*b, j*b+b)), with per-group (G along the head
// dimension) scale and bias [B,KH,N,D/G] in the query dtype:
//     K[n,d] = sk[n,d/G] * code[n,d] + bk[n,d/G]      (same for V).
// Scores, softmax and P*V accumulate in fp32 (the fused kernels' contract,
// int8_quantized_sdpa.py:178-180), with the bottom-right causal mask for
// multi-token queries.
//
// Layout on B200: one CTA per (query row, token split). A thread scores one
// token per pass (sum over groups of sk * sum(q*code) + bk * sum(q), the
// reassociation of _int8_sdpa_sources.py); the CTA keeps an online softmax
// over 128-token chunks and accumulates P*V with threads across the head
// dimension (coalesced row reads). Splits publish (max, sum, o) partials and
// the last CTA of a query merges them in split order (deterministic).
#include <algorithm>

#include "sb_common.cuh"

namespace sb {

constexpr int kAffSdpaThreads = 128;
constexpr int kAffSdpaMaxDim = 256;
constexpr int kAffSdpaMaxSplits = 64;

struct AffineSdpaParams {
  const void* q;  // [B,H,L,Dk]
  const uint32_t* kp;
  const void* ks;
  const void* kb;
  const uint32_t* vp;
  const void* vs;
  const void* vb;
  void* out;  // [B,H,L,Dv]
  int batch, heads, kv_heads, length, n, dk, dv, group, bits;
  float scale;
  int causal;
  int splits;
  float* partial;      // [B*H*L][splits][dv + 2]
  unsigned* counters;  // [B*H*L]
  unsigned* status;
};

template <typename T>
__device__ __forceinline__ float ldf(const void* p, size_t i) {
  return to_float(static_cast<const T*>(p)[i]);
}

template <typename T>
__global__ void __launch_bounds__(kAffSdpaThreads) affine_sdpa_kernel(const AffineSdpaParams p) {
  __shared__ float q_s[kAffSdpaMaxDim];
  __shared__ float qsum_s[kAffSdpaMaxDim / 32];
  __shared__ float p_s[kAffSdpaThreads];
  __shared__ float red_s[kAffSdpaThreads / 32];
  __shared__ float bcast;

  grid_dependency_wait();
  const int row = blockIdx.x;  // ((b * H + h) * L + l)
  const int split = blockIdx.y;
  const int l = row % p.length;
  const int bh = row / p.length;
  const int h = bh % p.heads, b = bh / p.heads;
  const int kh = h / (p.heads / p.kv_heads);
  const int tid = threadIdx.x;
  const int per_word = 32 / p.bits;
  const uint32_t cmask = (1u << p.bits) - 1u;
  const int wk = p.dk / per_word, wv = p.dv / per_word;  // words per token row
  const int gk = p.dk / p.group, gv = p.dv / p.group;
  // tokens visible to this query (bottom-right causal mask for L > 1)
  const int visible = p.causal ? p.n - p.length + 1 + l : p.n;
  const int t_begin = static_cast<int>(static_cast<long long>(visible) * split / p.splits);
  const int t_end = static_cast<int>(static_cast<long long>(visible) * (split + 1) / p.splits);

  const size_t qoff = static_cast<size_t>(row) * p.dk;
  for (int d = tid; d < p.dk; d += kAffSdpaThreads) q_s[d] = ldf<T>(p.q, qoff + d);
  __syncthreads();
  if (tid < gk) {
    float s = 0.f;
    for (int i = 0; i < p.group; ++i) s += q_s[tid * p.group + i];
    qsum_s[tid] = s;
  }
  __syncthreads();

  const size_t kv_row0 = (static_cast<size_t>(b) * p.kv_heads + kh) * p.n;  // token 0 of this (b, kh)
  float m_run = -INFINITY, l_run = 0.f;
  float o0 = 0.f, o1 = 0.f;  // head-dimension entries tid and tid + 128
  for (int c0 = t_begin; c0 < t_end; c0 += kAffSdpaThreads) {
    const int t = c0 + tid;
    float s = -INFINITY;
    if (t < t_end) {
      const size_t tok = kv_row0 + t;
      const uint32_t* kw = p.kp + tok * wk;
      float acc = 0.f;
      for (int g = 0; g < gk; ++g) {
        float dot = 0.f;
        const int d0 = g * p.group;
        for (int w = d0 / per_word; w < (d0 + p.group) / per_word; ++w) {
          const uint32_t word = kw[w];
          for (int j = 0; j < per_word; ++j)
            dot = fmaf(q_s[w * per_word + j], static_cast<float>((word >> (j * p.bits)) & cmask), dot);
        }
        const float sk = ldf<T>(p.ks, tok * gk + g), bk = ldf<T>(p.kb, tok * gk + g);
        acc = fmaf(sk, dot, fmaf(bk, qsum_s[g], acc));
      }
      s = acc * p.scale;
    }
    // chunk maximum
    float cm = warp_max(s);
    if ((tid & 31) == 0) red_s[tid >> 5] = cm;
    __syncthreads();
    if (tid == 0) {
      float v = red_s[0];
      for (int i = 1; i < kAffSdpaThreads / 32; ++i) v = fmaxf(v, red_s[i]);
      bcast = v;
    }
    __syncthreads();
    const float m_new = fmaxf(m_run, bcast);
    const float alpha = (m_run == -INFINITY) ? 0.f : expf(m_run - m_new);
    const float pt = (t < t_end) ? expf(s - m_new) : 0.f;
    p_s[tid] = pt;
    float cs = warp_sum(pt);
    __syncthreads();  // p_s complete; red_s free
    if ((tid & 31) == 0) red_s[tid >> 5] = cs;
    __syncthreads();
    float chunk_sum = 0.f;
    for (int i = 0; i < kAffSdpaThreads / 32; ++i) chunk_sum += red_s[i];
    l_run = l_run * alpha + chunk_sum;
    m_run = m_new;
    o0 *= alpha;
    o1 *= alpha;
    // P * V over the chunk; thread owns head dims tid and tid + 128
    const int nt = min(kAffSdpaThreads, t_end - c0);
    for (int i = 0; i < nt; ++i) {
      const float pi = p_s[i];
      const size_t tok = kv_row0 + c0 + i;
      const uint32_t* vw = p.vp + tok * wv;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int d = tid + half * kAffSdpaThreads;
        if (d < p.dv) {
          const uint32_t code = (vw[d / per_word] >> ((d % per_word) * p.bits)) & cmask;
          const int g = d / p.group;
          const float v = fmaf(ldf<T>(p.vs, tok * gv + g), static_cast<float>(code), ldf<T>(p.vb, tok * gv + g));
          if (half == 0) o0 = fmaf(pi, v, o0);
          else o1 = fmaf(pi, v, o1);
        }
      }
    }
    __syncthreads();  // p_s / red_s reused next chunk
  }
  grid_dependency_launch();

  const size_t out_off = static_cast<size_t>(row) * p.dv;
  if (p.splits == 1) {
    const float inv = l_run > 0.f ? 1.0f / l_run : 0.f;
    if (tid < p.dv) static_cast<T*>(p.out)[out_off + tid] = from_float<T>(o0 * inv);
    if (tid + kAffSdpaThreads < p.dv) static_cast<T*>(p.out)[out_off + tid + kAffSdpaThreads] = from_float<T>(o1 * inv);
    return;
  }
  // publish this split's partial; the last split of the query merges
  float* part = p.partial + (static_cast<size_t>(row) * p.splits + split) * (p.dv + 2);
  if (tid < p.dv) part[tid] = o0;
  if (tid + kAffSdpaThreads < p.dv) part[tid + kAffSdpaThreads] = o1;
  if (tid == 0) {
    part[p.dv] = m_run;
    part[p.dv + 1] = l_run;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) bcast = __uint_as_float(atomicAdd(p.counters + row, 1u));
  __syncthreads();
  if (__float_as_uint(bcast) != static_cast<unsigned>(p.splits - 1)) return;
  __threadfence();
  float m_all = -INFINITY;
  for (int sp = 0; sp < p.splits; ++sp) {
    const float* ps = p.partial + (static_cast<size_t>(row) * p.splits + sp) * (p.dv + 2);
    m_all = fmaxf(m_all, __ldcg(ps + p.dv));
  }
  float l_all = 0.f, a0 = 0.f, a1 = 0.f;
  for (int sp = 0; sp < p.splits; ++sp) {
    const float* ps = p.partial + (static_cast<size_t>(row) * p.splits + sp) * (p.dv + 2);
    const float ms = __ldcg(ps + p.dv);
    const float w = (ms == -INFINITY) ? 0.f : expf(ms - m_all);
    l_all = fmaf(__ldcg(ps + p.dv + 1), w, l_all);
    if (tid < p.dv) a0 = fmaf(__ldcg(ps + tid), w, a0);
    if (tid + kAffSdpaThreads < p.dv) a1 = fmaf(__ldcg(ps + tid + kAffSdpaThreads), w, a1);
  }
  const float inv = l_all > 0.f ? 1.0f / l_all : 0.f;
  if (tid < p.dv) static_cast<T*>(p.out)[out_off + tid] = from_float<T>(a0 * inv);
  if (tid + kAffSdpaThreads < p.dv) static_cast<T*>(p.out)[out_off + tid + kAffSdpaThreads] = from_float<T>(a1 * inv);
  if (tid == 0) p.counters[row] = 0u;
}

namespace {

int affine_splits(int64_t rows, int64_t n) {
  // about two waves of 4 CTAs per SM, at least 256 tokens per split
  int s = static_cast<int>(std::max<int64_t>(1, (148 * 8) / std::max<int64_t>(rows, 1)));
  s = static_cast<int>(std::min<int64_t>(s, std::max<int64_t>(1, n / 256)));
  return std::max(1, std::min(s, kAffSdpaMaxSplits));
}

size_t affine_ws_bytes(int64_t rows, int splits, int dv) {
  if (splits <= 1) return 0;
  return kCounterBytes + static_cast<size_t>(rows) * splits * (dv + 2) * sizeof(float);
}

}  // namespace

}  // namespace sb

using namespace sb;

extern "C" size_t sb_affine_sdpa_workspace_size(int64_t batch, int num_heads, int64_t length, int64_t n, int dv) {
  const int64_t rows = batch * num_heads * length;
  return affine_ws_bytes(rows, affine_splits(rows, n), dv);
}

extern "C" int sb_affine_sdpa(const void* q, int dtype, const void* k_packed, const void* k_scales,
                              const void* k_biases, const void* v_packed, const void* v_scales, const void* v_biases,
                              void* out, int64_t batch, int num_heads, int num_kv_heads, int64_t length, int64_t n,
                              int dk, int dv, int group_size, int bits, float scale, int causal, void* workspace,
                              size_t workspace_bytes, void* stream) {
  SB_REQUIRE(batch > 0 && num_heads > 0 && num_kv_heads > 0 && length > 0 && n > 0, "nonempty inputs required");
  SB_REQUIRE(num_heads % num_kv_heads == 0, "query heads must be divisible by KV heads");
  SB_REQUIRE(bits == 2 || bits == 4 || bits == 8, "Supported affine formats: bits 2/4/8, group size 32/64/128");
  SB_REQUIRE(group_size == 32 || group_size == 64 || group_size == 128,
             "Supported affine formats: bits 2/4/8, group size 32/64/128");
  SB_REQUIRE(dk > 0 && dv > 0 && dk <= kAffSdpaMaxDim && dv <= kAffSdpaMaxDim && dk % group_size == 0 &&
                 dv % group_size == 0,
             "head dimensions must be multiples of the group size, at most 256");
  SB_REQUIRE(!causal || length <= n, "causal queries need at least as many keys as queries");
  SB_REQUIRE(std::isfinite(scale), "scale must be finite");
  const int64_t rows = batch * num_heads * length;
  SB_REQUIRE(rows < (1LL << 31) && n < (1LL << 31), "inputs too large");
  AffineSdpaParams p{};
  p.q = q;
  p.kp = static_cast<const uint32_t*>(k_packed);
  p.ks = k_scales;
  p.kb = k_biases;
  p.vp = static_cast<const uint32_t*>(v_packed);
  p.vs = v_scales;
  p.vb = v_biases;
  p.out = out;
  p.batch = static_cast<int>(batch);
  p.heads = num_heads;
  p.kv_heads = num_kv_heads;
  p.length = static_cast<int>(length);
  p.n = static_cast<int>(n);
  p.dk = dk;
  p.dv = dv;
  p.group = group_size;
  p.bits = bits;
  p.scale = scale;
  p.causal = causal ? 1 : 0;
  p.splits = affine_splits(rows, n);
  const size_t need = affine_ws_bytes(rows, p.splits, dv);
  if (p.splits > 1 && (workspace == nullptr || workspace_bytes < need || rows > kMaxCounters)) p.splits = 1;
  if (p.splits > 1) {
    p.counters = static_cast<unsigned*>(workspace);
    p.partial = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterBytes);
  }
  const dim3 grid(static_cast<unsigned>(rows), p.splits);
  const dim3 block(kAffSdpaThreads);
  cudaStream_t s = as_stream(stream);
  switch (dtype) {
    case SB_DTYPE_BF16:
      return launch("affine_sdpa", affine_sdpa_kernel<__nv_bfloat16>, grid, block, 0, s, p);
    case SB_DTYPE_F16:
      return launch("affine_sdpa", affine_sdpa_kernel<__half>, grid, block, 0, s, p);
    case SB_DTYPE_F32:
      return launch("affine_sdpa", affine_sdpa_kernel<float>, grid, block, 0, s, p);
  }
  return fail(SB_EUNSUPPORTED, "Q and metadata must be float16, bfloat16 or float32");
}
