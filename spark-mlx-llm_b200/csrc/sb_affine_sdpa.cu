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
// Single-query decode of the common shapes (4- or 8-bit codes, bf16/fp16,
// GQA 1/2/4/8) runs affine_decode_tc_kernel at head_dim 128/256 (tensor cores
// on fp16-dequantized tiles) and affine_decode_kernel at 64 (CUDA cores), both
// one CTA per (batch, KV head, token split), below. Other shapes:
// one CTA per (query row, token split). A thread scores one
// token per pass (sum over groups of sk * sum(q*code) + bk * sum(q), the
// reassociation of _int8_sdpa_sources.py); the CTA keeps an online softmax
// over 128-token chunks and accumulates P*V with threads across the head
// dimension (coalesced row reads). Splits publish (max, sum, o) partials and
// the last CTA of a query merges them in split order (deterministic).
#include <algorithm>
#include <type_traits>

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

// ---- single-query decode (L = 1, dk = dv = D in {64, 128, 256}, 4- or 8-bit codes, bf16/fp16):
// one CTA per (batch, KV head, token split) serves the KV head's G query heads,
// so every K/V byte is read once. Warp w takes tokens t_begin + w + 8i in
// groups of 4 (their loads issued together); lane l owns head dimensions
// [E*l, E*l + E) (E = D / 32: coalesced row reads) and the scale/bias of their
// group. A score is the lanes' partial sums (sk * sum(q*code) + bk * sum(q),
// per lane) added by a butterfly, so every lane holds every head's score; the
// online softmax is in fp32 (exp2); P.V accumulates per lane. Warps merge in
// shared memory and splits through the workspace (the last CTA of a KV head
// adds them in split order). A split's partial is [o (D floats), m, l, pad 2]:
// the stride D + 4 keeps every partial row 16-byte aligned for float4 reads.
constexpr int kAffDecWarps = 8;
constexpr int kAffDecPad = 4;

// the lane's E codes of a row as raw words (unpacked where they are used)
template <int BITS, int E>
__device__ __forceinline__ void load_codes(const uint32_t* row, int lane, uint32_t (&w)[2]) {
  constexpr int kBytes = E * BITS / 8;  // bytes of the lane's codes
  const uint8_t* base = reinterpret_cast<const uint8_t*>(row) + lane * kBytes;
  w[0] = w[1] = 0u;
  if constexpr (kBytes == 8) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(base));
    w[0] = v.x;
    w[1] = v.y;
  } else if constexpr (kBytes == 4) {
    w[0] = __ldg(reinterpret_cast<const uint32_t*>(base));
  } else if constexpr (kBytes == 2) {
    w[0] = __ldg(reinterpret_cast<const uint16_t*>(base));
  } else {
    w[0] = __ldg(base);
  }
}
template <int BITS>
__device__ __forceinline__ float code_at(const uint32_t (&w)[2], int e) {
  const int bit = e * BITS;
  return static_cast<float>((w[bit >> 5] >> (bit & 31)) & ((1u << BITS) - 1u));
}

// The end of a single-query decode CTA: the warp partials in shared memory
// (dsm: [W][G][D] outputs, then [W][G] maxima and [W][G] sums, log2 domain;
// written before a __syncthreads) -> the CTA's output, or its split partial,
// and the last CTA of a (batch, KV head) merges the splits: one warp per query
// head turns the split maxima into weights in shared memory, then each thread
// adds four output columns over the splits with float4 loads.
template <typename T, int G, int D, int W>
__device__ __forceinline__ void affine_decode_finish(const AffineSdpaParams& p, float* dsm, int split, int bkv,
                                                     int b, int kh) {
  constexpr int kThreads = W * 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* so = dsm;
  const float* sm_ = dsm + W * G * D;
  const float* sl_ = sm_ + W * G;
  grid_dependency_launch();
  const bool single = p.splits == 1;
  for (int idx = threadIdx.x; idx < G * D; idx += kThreads) {
    const int gi = idx / D, d = idx % D;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < W; ++w) mm = fmaxf(mm, sm_[w * G + gi]);
    float ll = 0.f, oo = 0.f;
    if (mm != -INFINITY) {
#pragma unroll
      for (int w = 0; w < W; ++w) {
        const float f = sm_[w * G + gi] == -INFINITY ? 0.f : exp2f(sm_[w * G + gi] - mm);
        ll = fmaf(sl_[w * G + gi], f, ll);
        oo = fmaf(so[(w * G + gi) * D + d], f, oo);
      }
    }
    const size_t row = static_cast<size_t>(b) * p.heads + kh * G + gi;
    if (single) {
      static_cast<T*>(p.out)[row * D + d] = from_float<T>(ll > 0.f ? oo / ll : 0.f);
    } else {
      float* part = p.partial + (row * p.splits + split) * (D + kAffDecPad);
      part[d] = oo;
      if (d == 0) {
        part[D] = mm;
        part[D + 1] = ll;
      }
    }
  }
  if (single) return;
  __shared__ unsigned s_prev;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_prev = atomicAdd(p.counters + bkv, 1u);
  __syncthreads();
  if (s_prev != static_cast<unsigned>(p.splits - 1)) return;
  __threadfence();
  constexpr int kPS = D + kAffDecPad;
  const int S = p.splits;
  const size_t row0 = static_cast<size_t>(b) * p.heads + kh * G;
  float* sw = dsm;                             // [G][kAffSdpaMaxSplits]
  float* sden = dsm + G * kAffSdpaMaxSplits;  // [G]
  for (int gi = warp; gi < G; gi += W) {
    const float* base = p.partial + (row0 + gi) * S * kPS;
    float mm = -INFINITY;
    for (int sp = lane; sp < S; sp += 32) mm = fmaxf(mm, __ldcg(base + sp * kPS + D));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, off));
    float ll = 0.f;
    for (int sp = lane; sp < S; sp += 32) {
      const float ms = __ldcg(base + sp * kPS + D);
      const float w = ms == -INFINITY ? 0.f : exp2f(ms - mm);
      sw[gi * kAffSdpaMaxSplits + sp] = w;
      ll = fmaf(__ldcg(base + sp * kPS + D + 1), w, ll);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ll += __shfl_xor_sync(0xffffffffu, ll, off);
    if (lane == 0) sden[gi] = ll;
  }
  __syncthreads();
  for (int v4 = threadIdx.x; v4 < G * D / 4; v4 += kThreads) {
    const int gi = (4 * v4) / D, d = (4 * v4) % D;
    const float* base = p.partial + (row0 + gi) * S * kPS + d;
    const float* w = sw + gi * kAffSdpaMaxSplits;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int sp = 0; sp < S; ++sp) {
      const float4 o4 = __ldcg(reinterpret_cast<const float4*>(base + static_cast<size_t>(sp) * kPS));
      const float ws = w[sp];
      acc.x = fmaf(o4.x, ws, acc.x);
      acc.y = fmaf(o4.y, ws, acc.y);
      acc.z = fmaf(o4.z, ws, acc.z);
      acc.w = fmaf(o4.w, ws, acc.w);
    }
    const float ll = sden[gi];
    T* dst = static_cast<T*>(p.out) + (row0 + gi) * D + d;
    dst[0] = from_float<T>(ll > 0.f ? acc.x / ll : 0.f);
    dst[1] = from_float<T>(ll > 0.f ? acc.y / ll : 0.f);
    dst[2] = from_float<T>(ll > 0.f ? acc.z / ll : 0.f);
    dst[3] = from_float<T>(ll > 0.f ? acc.w / ll : 0.f);
  }
  if (threadIdx.x == 0) p.counters[bkv] = 0u;
}

template <typename T, int BITS, int G, int D>
__global__ void __launch_bounds__(kAffDecWarps * 32, G * D <= 1024 ? 2 : 1)
    affine_decode_kernel(const AffineSdpaParams p) {
  constexpr int E = D / 32;
  constexpr int kU = 4;  // tokens per warp iteration
  extern __shared__ float dsm[];  // [warps][G][D] partial O, then [warps][G] m and l
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, bkv = blockIdx.y;
  const int b = bkv / p.kv_heads, kh = bkv % p.kv_heads;
  const int words = D * BITS / 32, ngroups = D / p.group;
  const int lg = (E * lane) / p.group;  // the lane's group
  grid_dependency_wait();
  const int t_begin = static_cast<int>(static_cast<long long>(p.n) * split / p.splits);
  const int t_end = static_cast<int>(static_cast<long long>(p.n) * (split + 1) / p.splits);
  const float sl2 = p.scale * 1.4426950408889634f;

  float q[G][E], qs[G];
#pragma unroll
  for (int gi = 0; gi < G; ++gi) {
    const size_t qrow = (static_cast<size_t>(b) * p.heads + kh * G + gi) * D + E * lane;
    qs[gi] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      q[gi][e] = ldf<T>(p.q, qrow + e);
      qs[gi] += q[gi][e];
    }
  }
  float m_run[G], l_run[G], o[G][E];
#pragma unroll
  for (int gi = 0; gi < G; ++gi) {
    m_run[gi] = -INFINITY;
    l_run[gi] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) o[gi][e] = 0.f;
  }
  const size_t tok0 = static_cast<size_t>(bkv) * p.n;  // token 0 of this (b, kv head)
  for (int t0 = t_begin + warp; t0 < t_end; t0 += kU * kAffDecWarps) {
    uint32_t kc[kU][2], vc[kU][2];
    float sk[kU], bk[kU], sv[kU], bv[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int t = t0 + u * kAffDecWarps;
      const size_t tok = tok0 + (t < t_end ? t : t_begin);
      load_codes<BITS, E>(p.kp + tok * words, lane, kc[u]);
      load_codes<BITS, E>(p.vp + tok * words, lane, vc[u]);
      sk[u] = ldf<T>(p.ks, tok * ngroups + lg);
      bk[u] = ldf<T>(p.kb, tok * ngroups + lg);
      sv[u] = ldf<T>(p.vs, tok * ngroups + lg);
      bv[u] = ldf<T>(p.vb, tok * ngroups + lg);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const bool live = t0 + u * kAffDecWarps < t_end;
      float sc[G];
#pragma unroll
      for (int gi = 0; gi < G; ++gi) {
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) dot = fmaf(q[gi][e], code_at<BITS>(kc[u], e), dot);
        sc[gi] = fmaf(sk[u], dot, bk[u] * qs[gi]);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
#pragma unroll
        for (int gi = 0; gi < G; ++gi) sc[gi] += __shfl_xor_sync(0xffffffffu, sc[gi], off);
      float v[E];
#pragma unroll
      for (int e = 0; e < E; ++e) v[e] = fmaf(sv[u], code_at<BITS>(vc[u], e), bv[u]);
#pragma unroll
      for (int gi = 0; gi < G; ++gi) {
        if (!live) continue;
        const float s2 = sc[gi] * sl2;
        // rescale only when the maximum rises; the butterfly leaves every lane
        // the same sum, so the branch is uniform across the warp
        if (s2 > m_run[gi]) {
          const float alpha = m_run[gi] == -INFINITY ? 0.f : exp2f(m_run[gi] - s2);
          l_run[gi] *= alpha;
#pragma unroll
          for (int e = 0; e < E; ++e) o[gi][e] *= alpha;
          m_run[gi] = s2;
        }
        const float pr = exp2f(s2 - m_run[gi]);
        l_run[gi] += pr;
#pragma unroll
        for (int e = 0; e < E; ++e) o[gi][e] = fmaf(pr, v[e], o[gi][e]);
      }
    }
  }
  // ---- warps -> CTA (fixed warp order)
  float* so = dsm;
  float* sm_ = dsm + kAffDecWarps * G * D;
  float* sl_ = sm_ + kAffDecWarps * G;
#pragma unroll
  for (int gi = 0; gi < G; ++gi) {
#pragma unroll
    for (int e = 0; e < E; ++e) so[(warp * G + gi) * D + E * lane + e] = o[gi][e];
    if (lane == 0) {
      sm_[warp * G + gi] = m_run[gi];
      sl_[warp * G + gi] = l_run[gi];
    }
  }
  __syncthreads();
  affine_decode_finish<T, G, D, kAffDecWarps>(p, dsm, split, bkv, b, kh);
}

// ---------------------------------------------------------------------------
// Tensor-core single-query decode (head_dim 128 / 256). A CTA of kTcWarps warps
// takes one (batch, KV head, token split); each warp walks its own 16-token
// tiles of the split:
//   1. loads the tile's packed K and V codes (16-byte chunks, one group each)
//      and their scales and biases, and dequantizes them into fp16 rows in its
//      shared-memory tiles: code -> 1024 + code under the fp16 exponent of 1024
//      (prmt), minus 1024 (exact), then one fused s * c + b (fp16, one rounding);
//   2. S = Q K^T with mma.sync m16n8k16: A = the G query heads (rows g < G, the
//      rest zero) as fp16, B = the K tile through ldmatrix -> S[head, token];
//   3. online softmax per head in fp32 (exp2 domain), P rounded to fp16;
//   4. O^T += V^T P: A = the V tile through ldmatrix.trans (dims x tokens),
//      B = P straight from S's accumulator layout -> O^T[dim, head] in fp32.
// The warps' (O, max, sum) then meet in shared memory and the splits in the
// workspace (affine_decode_finish).
constexpr int kTcWarps = 4;
constexpr int kTcTok = 16;  // tokens per warp tile

template <int D>
struct TcGeo {
  static constexpr int kStride = D * 2 + 16;      // bytes per fp16 row (ldmatrix without bank conflicts)
  static constexpr int kTile = kTcTok * kStride;  // one fp16 tile (K or V)
  static constexpr int kWarpBytes = 2 * kTile;
  static constexpr int kSmem = kTcWarps * kWarpBytes;
  static constexpr int kMerge = (kTcWarps * 8 * D + 2 * kTcWarps * 8) * 4;  // finish's [W][G][D] + [W][G] x 2
  static_assert(kMerge <= kSmem, "the merge reuses the tiles' shared memory");
};

__device__ __forceinline__ uint32_t tc_pack_half2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t tc_dequant2(uint32_t biased, __half2 s2, __half2 b2) {
  // biased = (1024 + c0, 1024 + c1) as fp16x2 -> (s c0 + b, s c1 + b)
  const __half2 k1024 = __floats2half2_rn(1024.f, 1024.f);
  const __half2 c = __hsub2(*reinterpret_cast<const __half2*>(&biased), k1024);
  const __half2 r = __hfma2(c, s2, b2);
  return *reinterpret_cast<const uint32_t*>(&r);
}
__device__ __forceinline__ void ldsm4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

template <typename T, int BITS, int G, int D>
__global__ void __launch_bounds__(kTcWarps * 32, 2) affine_decode_tc_kernel(const AffineSdpaParams p) {
  using C = TcGeo<D>;
  constexpr int kRowBytes = D * BITS / 8;        // packed codes of one token
  constexpr int kChunks = kRowBytes / 16;        // 16-byte chunks per token row
  constexpr int kLaneChunks = kTcTok * kChunks / 32;
  constexpr int kChunkDims = 16 * 8 / BITS;      // dims per chunk (16 or 32)
  static_assert(kLaneChunks >= 1 && (kTcTok * kChunks) % 32 == 0, "tile chunks must spread over the lanes");
  extern __shared__ __align__(128) uint8_t tsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int split = blockIdx.x, bkv = blockIdx.y;
  const int b = bkv / p.kv_heads, kh = bkv % p.kv_heads;
  const int ngroups = D / p.group;
  uint8_t* ktile = tsm + warp * C::kWarpBytes;
  uint8_t* vtile = ktile + C::kTile;
  const uint32_t kbase = smem_u32(ktile), vbase = smem_u32(vtile);
  // ldmatrix lane address: matrix (lane / 8) -> token rows 0-7 / 8-15, dims +0 / +8
  const int lm = lane >> 3;
  const uint32_t lrow = static_cast<uint32_t>(((lane & 7) + (lm >> 1) * 8) * C::kStride + (lm & 1) * 16);
  grid_dependency_wait();
  const int t_begin = static_cast<int>(static_cast<long long>(p.n) * split / p.splits);
  const int t_end = static_cast<int>(static_cast<long long>(p.n) * (split + 1) / p.splits);
  const float sl2 = p.scale * 1.4426950408889634f;

  // query rows as the A operand: row g = head g of the group (zero for g >= G)
  uint32_t qa[D / 16][2];
  {
    const T* qrow = static_cast<const T*>(p.q) + (static_cast<size_t>(b) * p.heads + kh * G + (g < G ? g : 0)) * D;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int d0 = 16 * ks + 2 * c;
      qa[ks][0] = g < G ? tc_pack_half2(to_float(qrow[d0]), to_float(qrow[d0 + 1])) : 0u;
      qa[ks][1] = g < G ? tc_pack_half2(to_float(qrow[d0 + 8]), to_float(qrow[d0 + 9])) : 0u;
    }
  }
  float o[D / 16][4];
#pragma unroll
  for (int mt = 0; mt < D / 16; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;  // head g (the same in the four lanes of g)

  const uint8_t* kp = reinterpret_cast<const uint8_t*>(p.kp) + static_cast<size_t>(bkv) * p.n * kRowBytes;
  const uint8_t* vp = reinterpret_cast<const uint8_t*>(p.vp) + static_cast<size_t>(bkv) * p.n * kRowBytes;
  const T* ksc = static_cast<const T*>(p.ks) + static_cast<size_t>(bkv) * p.n * ngroups;
  const T* kbi = static_cast<const T*>(p.kb) + static_cast<size_t>(bkv) * p.n * ngroups;
  const T* vsc = static_cast<const T*>(p.vs) + static_cast<size_t>(bkv) * p.n * ngroups;
  const T* vbi = static_cast<const T*>(p.vb) + static_cast<size_t>(bkv) * p.n * ngroups;

  for (int t0 = t_begin + warp * kTcTok; t0 < t_end; t0 += kTcWarps * kTcTok) {
    // ---- 1. codes -> fp16 rows (tokens past the split repeat its last token; masked below)
    uint4 kc[kLaneChunks], vc[kLaneChunks];
    uint32_t ksb[kLaneChunks], vsb[kLaneChunks];  // scale bits | bias bits << 16
#pragma unroll
    for (int j = 0; j < kLaneChunks; ++j) {
      const int idx = lane + 32 * j, row = idx / kChunks, col = idx % kChunks;
      const int tok = min(t0 + row, t_end - 1);
      const size_t off = static_cast<size_t>(tok) * kRowBytes + col * 16;
      kc[j] = ldg_stream16(kp + off);
      vc[j] = ldg_stream16(vp + off);
      const size_t gi = static_cast<size_t>(tok) * ngroups + (col * kChunkDims) / p.group;
      ksb[j] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(ksc + gi)) |
               static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(kbi + gi)) << 16;
      vsb[j] = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(vsc + gi)) |
               static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(vbi + gi)) << 16;
    }
    __syncwarp();  // the previous tile's ldmatrix reads are done before the tiles are rewritten
#pragma unroll
    for (int j = 0; j < kLaneChunks; ++j) {
      const int idx = lane + 32 * j, row = idx / kChunks, col = idx % kChunks;
#pragma unroll
      for (int kv = 0; kv < 2; ++kv) {
        const uint4 w = kv ? vc[j] : kc[j];
        const uint32_t sb = kv ? vsb[j] : ksb[j], sbits = sb & 0xFFFFu, bbits = sb >> 16;
        float sf, bf;
        if constexpr (std::is_same<T, __half>::value) {
          sf = __half2float(__ushort_as_half(static_cast<unsigned short>(sbits)));
          bf = __half2float(__ushort_as_half(static_cast<unsigned short>(bbits)));
        } else {
          sf = __uint_as_float(sbits << 16);
          bf = __uint_as_float(bbits << 16);
        }
        const __half2 s2 = __float2half2_rn(sf), b2 = __float2half2_rn(bf);
        uint8_t* dst = (kv ? vtile : ktile) + row * C::kStride + col * kChunkDims * 2;
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
        if constexpr (BITS == 8) {
          uint32_t h[8];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            h[2 * i] = tc_dequant2(prmt(ws[i], 0x64646464u, 0x4140u), s2, b2);
            h[2 * i + 1] = tc_dequant2(prmt(ws[i], 0x64646464u, 0x4342u), s2, b2);
          }
          reinterpret_cast<uint4*>(dst)[0] = make_uint4(h[0], h[1], h[2], h[3]);
          reinterpret_cast<uint4*>(dst)[1] = make_uint4(h[4], h[5], h[6], h[7]);
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            // nibble j of the word is dim 8 i + j
            const uint32_t lo = ws[i] & 0x0F0F0F0Fu, hi = (ws[i] >> 4) & 0x0F0F0F0Fu;
            const uint32_t a = prmt(lo, hi, 0x5140u), bb = prmt(lo, hi, 0x7362u);  // nibbles 0-3, 4-7
            reinterpret_cast<uint4*>(dst)[i] =
                make_uint4(tc_dequant2(prmt(a, 0x64646464u, 0x4140u), s2, b2),
                           tc_dequant2(prmt(a, 0x64646464u, 0x4342u), s2, b2),
                           tc_dequant2(prmt(bb, 0x64646464u, 0x4140u), s2, b2),
                           tc_dequant2(prmt(bb, 0x64646464u, 0x4342u), s2, b2));
          }
        }
      }
    }
    __syncwarp();
    // ---- 2. S[head, token] for tokens t0 + (0..7) and t0 + (8..15)
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t kb[4];
      ldsm4(kb, kbase + lrow + ks * 32);
      const uint32_t a[4] = {qa[ks][0], 0u, qa[ks][1], 0u};
      mma_16816<true>(s0, a, kb[0], kb[1]);
      mma_16816<true>(s1, a, kb[2], kb[3]);
    }
    // ---- 3. online softmax of head g over the tile (lanes 4g..4g+3 hold its 16 tokens)
    const int tk = t0 + 2 * c;
    float x[4] = {tk < t_end ? s0[0] * sl2 : -INFINITY, tk + 1 < t_end ? s0[1] * sl2 : -INFINITY,
                  tk + 8 < t_end ? s1[0] * sl2 : -INFINITY, tk + 9 < t_end ? s1[1] * sl2 : -INFINITY};
    float tmax = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
    const float m_new = fmaxf(m_run, tmax);  // finite: token t0 is in the split
    const float alpha = m_run == -INFINITY ? 0.f : exp2f(m_run - m_new);
    float pr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) pr[i] = exp2f(x[i] - m_new);
    l_run = fmaf(l_run, alpha, (pr[0] + pr[1]) + (pr[2] + pr[3]));
    m_run = m_new;
    // O^T columns are heads 2c and 2c + 1: their factors live in lanes 8c and 8c + 4
    const float a0 = __shfl_sync(0xffffffffu, alpha, 8 * c), a1 = __shfl_sync(0xffffffffu, alpha, 8 * c + 4);
    if (__any_sync(0xffffffffu, a0 != 1.f || a1 != 1.f)) {
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) {
        o[mt][0] *= a0;
        o[mt][1] *= a1;
        o[mt][2] *= a0;
        o[mt][3] *= a1;
      }
    }
    // ---- 4. O^T[dim, head] += V^T[dim, token] P[token, head]
    const uint32_t pb0 = tc_pack_half2(pr[0], pr[1]), pb1 = tc_pack_half2(pr[2], pr[3]);
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt) {
      uint32_t va[4];
      ldsm4_trans(va, vbase + lrow + mt * 32);
      mma_16816<true>(o[mt], va, pb0, pb1);
    }
  }
  // ---- warp partials -> shared memory (the tiles are free once every warp is done)
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  __syncthreads();
  float* dsm = reinterpret_cast<float*>(tsm);
  float* so = dsm;
  float* sm_ = dsm + kTcWarps * G * D;
  float* sl_ = sm_ + kTcWarps * G;
#pragma unroll
  for (int mt = 0; mt < D / 16; ++mt) {
    const int d0 = 16 * mt + g;
    if (2 * c < G) {
      so[(warp * G + 2 * c) * D + d0] = o[mt][0];
      so[(warp * G + 2 * c) * D + d0 + 8] = o[mt][2];
    }
    if (2 * c + 1 < G) {
      so[(warp * G + 2 * c + 1) * D + d0] = o[mt][1];
      so[(warp * G + 2 * c + 1) * D + d0 + 8] = o[mt][3];
    }
  }
  if (c == 0 && g < G) {
    sm_[warp * G + g] = m_run;
    sl_[warp * G + g] = l_run;
  }
  __syncthreads();
  affine_decode_finish<T, G, D, kTcWarps>(p, dsm, split, bkv, b, kh);
}

namespace {

template <typename T, int BITS, int G, int D>
int launch_affine_decode(const AffineSdpaParams& p, cudaStream_t s) {
  constexpr int smem = (kAffDecWarps * G * D + 2 * kAffDecWarps * G) * 4;
  auto kernel = affine_decode_kernel<T, BITS, G, D>;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return fail(SB_ECUDA, std::string("affine decode attribute: ") + cudaGetErrorString(e));
  }
  return launch("affine_sdpa_decode", kernel, dim3(p.splits, p.batch * p.kv_heads), dim3(kAffDecWarps * 32), smem,
                s, p);
}

template <typename T, int BITS, int G, int D>
int launch_affine_decode_tc(const AffineSdpaParams& p, cudaStream_t s) {
  constexpr int smem = TcGeo<D>::kSmem;
  auto kernel = affine_decode_tc_kernel<T, BITS, G, D>;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return fail(SB_ECUDA, std::string("affine decode attribute: ") + cudaGetErrorString(e));
  return launch("affine_sdpa_decode_tc", kernel, dim3(p.splits, p.batch * p.kv_heads), dim3(kTcWarps * 32), smem,
                s, p);
}

// head_dim 128 / 256 run the tensor-core kernel, 64 the CUDA-core one
template <typename T, int BITS, int G>
int affine_decode_by_dim(const AffineSdpaParams& p, cudaStream_t s) {
  switch (p.dk) {
    case 64: return launch_affine_decode<T, BITS, G, 64>(p, s);
    case 128: return launch_affine_decode_tc<T, BITS, G, 128>(p, s);
    default: return launch_affine_decode_tc<T, BITS, G, 256>(p, s);
  }
}

template <typename T, int BITS>
int affine_decode_by_gqa(const AffineSdpaParams& p, int G, cudaStream_t s) {
  switch (G) {
    case 1: return affine_decode_by_dim<T, BITS, 1>(p, s);
    case 2: return affine_decode_by_dim<T, BITS, 2>(p, s);
    case 4: return affine_decode_by_dim<T, BITS, 4>(p, s);
    default: return affine_decode_by_dim<T, BITS, 8>(p, s);
  }
}

int affine_splits(int64_t rows, int64_t n) {
  // about two waves of 4 CTAs per SM, at least 256 tokens per split
  int s = static_cast<int>(std::max<int64_t>(1, (148 * 8) / std::max<int64_t>(rows, 1)));
  s = static_cast<int>(std::min<int64_t>(s, std::max<int64_t>(1, n / 256)));
  return std::max(1, std::min(s, kAffSdpaMaxSplits));
}

// Token splits of the single-query decode kernel: one wave of CTAs over the
// (batch, KV head) pairs (two CTAs per SM up to G x D = 1024, else one), at
// least 64 tokens per split, at most kAffSdpaMaxSplits.
int64_t affine_decode_splits(int64_t bkv, int64_t n, int64_t slots) {
  int64_t sp = std::max<int64_t>(1, (slots + bkv - 1) / bkv);
  sp = std::min<int64_t>(sp, std::max<int64_t>(1, n / 64));
  return std::min<int64_t>(sp, kAffSdpaMaxSplits);
}

size_t affine_ws_bytes(int64_t rows, int splits, int dv) {
  if (splits <= 1) return 0;
  // (dv + 4 floats per partial: the decode kernel's aligned stride; the general kernel uses dv + 2)
  return kCounterBytes + static_cast<size_t>(rows) * splits * (dv + kAffDecPad) * sizeof(float);
}

}  // namespace

}  // namespace sb

using namespace sb;

extern "C" size_t sb_affine_sdpa_workspace_size(int64_t batch, int num_heads, int64_t length, int64_t n, int dv) {
  const int64_t rows = batch * num_heads * length;
  int splits = affine_splits(rows, n);
  // single-query decode: the most splits the decode kernel can plan (at least
  // rows / 8 KV-head pairs, 296 CTA slots)
  if (length == 1)
    splits = std::max(splits, static_cast<int>(affine_decode_splits(std::max<int64_t>(1, (rows + 7) / 8), n, 296)));
  return affine_ws_bytes(rows, splits, dv);
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
  cudaStream_t s = as_stream(stream);
  // single-query decode of the common shapes: the KV-head-per-CTA kernel
  const int G = num_heads / num_kv_heads;
  // code rows are read as 8-byte (head_dim 64) or 16-byte (128 / 256, the tensor-core kernel) chunks
  const uintptr_t row_align = dk >= 128 ? 16 : 8;
  const bool rows_aligned = reinterpret_cast<uintptr_t>(k_packed) % row_align == 0 &&
                            reinterpret_cast<uintptr_t>(v_packed) % row_align == 0;
  if (length == 1 && dk == dv && (dk == 64 || dk == 128 || dk == 256) && (bits == 4 || bits == 8) &&
      (G == 1 || G == 2 || G == 4 || G == 8) && (dtype == SB_DTYPE_BF16 || dtype == SB_DTYPE_F16) &&
      rows_aligned && batch * num_kv_heads < 65536) {
    const int64_t bkv = batch * num_kv_heads;
    p.splits = static_cast<int>(affine_decode_splits(bkv, n, 296));  // two CTAs per SM
    // the merge reads the partials as float4: a workspace off 16 bytes (or too small) runs one split
    if (p.splits > 1 && (workspace == nullptr || workspace_bytes < affine_ws_bytes(rows, p.splits, dv) ||
                         rows > kMaxCounters || reinterpret_cast<uintptr_t>(workspace) % 16 != 0))
      p.splits = 1;
    p.counters = p.splits > 1 ? static_cast<unsigned*>(workspace) : nullptr;
    p.partial = p.splits > 1 ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterBytes) : nullptr;
    if (dtype == SB_DTYPE_BF16)
      return bits == 4 ? affine_decode_by_gqa<__nv_bfloat16, 4>(p, G, s) : affine_decode_by_gqa<__nv_bfloat16, 8>(p, G, s);
    return bits == 4 ? affine_decode_by_gqa<__half, 4>(p, G, s) : affine_decode_by_gqa<__half, 8>(p, G, s);
  }
  const dim3 grid(static_cast<unsigned>(rows), p.splits);
  const dim3 block(kAffSdpaThreads);
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
