// INT8-KV single-query decode attention (flash-decoding, split-K) for sm_100a.
//
// Reference: extensions/spark-mlx-ext/spark_mlx_ext/int8_quantized_sdpa.py:156-287
// with the online-softmax kernel _int8_sdpa_sources.py:8-181 and its merge
// :363-376. KV format here: int8 codes [B, KH, cap, D]
// with one fp16 scale per token per head (K = code * scale).
//
// Design (B200): the KV stream is the HBM-bound part (260 bytes per token per
// KV head); everything else lives in registers. One CTA handles one
// (batch, kv head, token range); its 8 warps take 16-token blocks in turn,
// each keeping 3 blocks (K box, V box and the blocks' fp16 scales) in flight
// in its own shared-memory ring (two CTAs per SM: 48 blocks in flight).
// Scores and P.V run on the tensor cores (mma.sync m16n8k16, fp16 operands,
// fp32 accumulate): the G query heads sharing a KV head are the MMA rows
// (GQA reuse: every K/V byte is loaded once for all G heads). int8 codes are
// turned into the exact fp16 values 1024 + (code + 128) by byte permutes; the
// constant 1152 they carry is removed exactly afterwards (for QK with the
// precomputed sum of q, for PV with an MMA of the rounded probabilities
// against ones). q is scaled by a power of two per head so its fp16 copy is
// exact. The head dimension is permuted across lanes so every lane loads
// whole 16-byte segments of K and V rows. Softmax is fp32 (exp2 with log2(e)
// folded into the scale). Partial results of the warps merge in shared
// memory, the CTAs' partials in a workspace; the last CTA of each (batch, kv
// head) merges them in a fixed order (deterministic, one launch).
#include <algorithm>
#include <cmath>
#include <mutex>
#include <string>

#include "sb_common.cuh"

namespace sb {

// Warps per CTA: head_dim 128 runs 6 (two CTAs per SM, up to 170 registers per
// thread: no spills), head_dim 256 runs 8 (one CTA per SM: its ring of 8 KB
// blocks fills the SM). Measured on B200 at head_dim 128 against 8 warps x 2
// CTAs (128 registers, 150 bytes of spills): 32K tokens 0.61 -> 0.63 of HBM at
// batch 8, 0.65 -> 0.66 at batch 32; 4K tokens at batch 8 0.40 -> 0.45.
constexpr int sdpa_warps(int D) { return D == 128 ? 6 : 8; }
// head dims 128 and 256 (a K/V row is one or two 128-byte TMA boxes)
constexpr int part_stride(int D) { return D + 4; }  // O[D], then m, l
constexpr int kSdpaStages = 3;           // 16-token blocks in flight per warp
constexpr int kMaxSplits = 64;           // token splits per (batch, kv head)
constexpr int stage_bytes(int D) { return 2 * 16 * D; }  // swizzled K boxes + V boxes of 16 tokens
constexpr int kSdpaScaleBytes = 64;                 // the block's 16 K scales + 16 V scales (fp16)
constexpr size_t sdpa_smem(int warps, int stages, int D) {
  return 2048 + static_cast<size_t>(warps) * stages * (stage_bytes(D) + kSdpaScaleBytes);
}

struct SdpaParams {
  alignas(64) CUtensorMap kmap;  // K cache as [B*KH*cap rows][128 B], 16-row boxes, 128-B swizzle
  alignas(64) CUtensorMap vmap;
  const __nv_bfloat16* q;  // [B, H, D]
  const int8_t* k;         // [B*KH, cap, D]
  const __half* ks;        // [B*KH, cap]
  const int8_t* v;
  const __half* vs;
  __nv_bfloat16* out;  // [B, H, D]
  int kv_heads, length, capacity, splits;
  const int* length_dev;  // optional per-batch lengths in device memory (+ length_offset)
  int length_offset;
  float scale_log2e;
  float* partial;      // [B*KH][splits][G][D + 4] (global merge)
  unsigned* counters;  // [B*KH]
  unsigned* status;    // device status word or null
  int cluster;         // 1: the splits of a (b, kv head) form a cluster and merge in shared memory
  int early;           // 1: lengths and every cache row but the newest are final before this kernel
  int scale_bulk;      // 1: the blocks' scales stream with the K/V boxes (capacity % 16 == 0, aligned)
  int stages;          // ring depth per warp
};

constexpr int kSdpaMaxClusterSplits = 16;
// cluster merge buffer: [split][G][slice + 2] floats, slice = ceil(D / splits)
constexpr int cluster_buf(int D) { return 8 * D + 3 * 8 * kSdpaMaxClusterSplits; }

// m16n8k16 fp16 MMA keeping only rows 0-7 of the accumulator tile: rows 8-15
// (zero A rows here) start from zero and are discarded, so they hold no
// registers across the loop.
__device__ __forceinline__ void mma_16816_top(float (&d)[2], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  float j0, j1;
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%12};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(j0), "=f"(j1)
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(d[0]), "f"(d[1]), "f"(0.0f));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <int G, bool kBulk, int kSdpaWarps, int D>
__global__ void __launch_bounds__(kSdpaWarps * 32, D == 128 ? 16 / kSdpaWarps : 1)
    sdpa_int8_decode_kernel(const __grid_constant__ SdpaParams p) {
  constexpr int kBoxes = D / 128;           // 128-byte TMA boxes per K/V row
  constexpr int kStageBytes = stage_bytes(D);
  constexpr int kPartStride = part_stride(D);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int split = blockIdx.x;
  const int bkv = blockIdx.y;
  const int b = bkv / p.kv_heads, kvh = bkv % p.kv_heads;
  if (threadIdx.x == 0) {
    prefetch_tmap(&p.kmap);
    prefetch_tmap(&p.vmap);
  }
  // With `early`, the KV blocks that do not hold the newest token stream in
  // while the previous kernel (which writes that token) still runs.
  if (!p.early) grid_dependency_wait();
  const int N = p.length_dev ? min(p.length_dev[b] + p.length_offset, p.capacity) : p.length;
  const int nblk = (N + 15) / 16;
  const int blk_begin = static_cast<int>((static_cast<long long>(nblk) * split) / p.splits);
  const int blk_end = static_cast<int>((static_cast<long long>(nblk) * (split + 1)) / p.splits);
  const size_t kv_base = static_cast<size_t>(bkv) * p.capacity;
  const __half* ksb = p.ks + kv_base;
  const __half* vsb = p.vs + kv_base;

  // ---- running state (row g of the MMA tiles; rows g+8 are unused padding)
  float m_run = -INFINITY, l_run = 0.f;
  float acc[16 * kBoxes][2];  // rows g (the heads) of each 16 x 8 tile; rows g + 8 are padding
  float psum[2] = {0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 16 * kBoxes; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) acc[j][e] = 0.f;
  constexpr uint32_t kOnes = 0x3C003C00u;

  // ---- per-warp ring of 16-token K/V blocks in shared memory (TMA boxes)
  extern __shared__ uint8_t smem_dyn[];
  // 1 KB-aligned start (pointer arithmetic keeps the shared address space known to the compiler)
  uint8_t* sbase = smem_dyn + ((1024u - (smem_u32(smem_dyn) & 1023u)) & 1023u);
  const int NS = p.stages;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sbase) + warp * NS;
  uint8_t* ring = sbase + 1024 + warp * NS * kStageBytes;
  // per-warp ring of the blocks' scales: [stage][k 16 x fp16 | v 16 x fp16]
  uint8_t* sring = sbase + 1024 + kSdpaWarps * NS * kStageBytes + warp * NS * kSdpaScaleBytes;
  const int nb = blk_end - blk_begin;
  const int my_blocks = nb > warp ? (nb - warp + kSdpaWarps - 1) / kSdpaWarps : 0;
  auto block_of = [&](int i) { return blk_begin + warp + i * kSdpaWarps; };
  auto issue = [&](int i, int slot) {
    const int row = static_cast<int>(kv_base) + block_of(i) * 16;
    uint8_t* dst = ring + slot * kStageBytes;
    mbar_arrive_expect_tx(bars + slot, kStageBytes + (kBulk ? kSdpaScaleBytes : 0));
    // [K box 0 | K box 1 ..][V box 0 | V box 1 ..], 16 rows x 128 B each
#pragma unroll
    for (int x = 0; x < kBoxes; ++x) {
      tma_load_2d(dst + x * 2048, &p.kmap, 128 * x, row, bars + slot);
      tma_load_2d(dst + 16 * D + x * 2048, &p.vmap, 128 * x, row, bars + slot);
    }
    if constexpr (kBulk) {
      uint8_t* sdst = sring + slot * kSdpaScaleBytes;
      bulk_copy_g2s(sdst, p.ks + row, 32, bars + slot);
      bulk_copy_g2s(sdst + 32, p.vs + row, 32, bars + slot);
    }
  };
  const int last_blk = nblk - 1;  // holds token N-1, written by the previous kernel
  if (lane == 0) {
    for (int i = 0; i < NS; ++i) mbar_init(bars + i, 1);
    mbar_fence_init();
    for (int i = 0; i < NS && i < my_blocks; ++i)
      if (!p.early || block_of(i) != last_blk) issue(i, i);
  }
  __syncwarp();
  if (p.early) {
    grid_dependency_wait();
    if (lane == 0)
      for (int i = 0; i < NS && i < my_blocks; ++i)
        if (block_of(i) == last_blk) issue(i, i);
    __syncwarp();
  }

  // ---- q fragments: row g = query head kvh*G + g, k-slot d = 32t + 4s + {0..3}
  const bool head_ok = g < G;
  const int head = kvh * G + (head_ok ? g : 0);
  // (box x: d = 128x + 32t + 4s + {0..3}; qv[32x + ...])
  const __nv_bfloat16* qrow = p.q + (static_cast<size_t>(b) * p.kv_heads * G + head) * D + 32 * t;
  float qv[32 * kBoxes];
  {
#pragma unroll
    for (int i = 0; i < 4 * kBoxes; ++i) {
      const uint4 w = *reinterpret_cast<const uint4*>(qrow + 128 * (i >> 2) + 8 * (i & 3));
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        qv[8 * i + 2 * j] = bf16_lo(ww[j]);
        qv[8 * i + 2 * j + 1] = bf16_hi(ww[j]);
      }
    }
  }
  float qmax = 0.f;
#pragma unroll
  for (int i = 0; i < 32 * kBoxes; ++i) qmax = fmaxf(qmax, fabsf(qv[i]));
  qmax = fmaxf(qmax, __shfl_xor_sync(0xffffffffu, qmax, 1));
  qmax = fmaxf(qmax, __shfl_xor_sync(0xffffffffu, qmax, 2));
  int qexp = 0;
  frexpf(qmax, &qexp);  // qmax < 2^qexp
  const float up = qmax > 0.f ? ldexpf(1.0f, 15 - qexp) : 1.0f;     // |q*up| < 2^15
  const float down = qmax > 0.f ? ldexpf(1.0f, qexp - 15) : 1.0f;
  // A operand: a0 = slots (2t, 2t+1) -> d = 32t+4s+{0,1}; a2 = slots (2t+8, 2t+9) -> d = 32t+4s+{2,3}
  uint32_t aq[8 * kBoxes], aq2[8 * kBoxes];
  float qsum = 0.f;
#pragma unroll
  for (int s = 0; s < 8 * kBoxes; ++s) {
    const __half2 lo = __floats2half2_rn(qv[4 * s] * up, qv[4 * s + 1] * up);
    const __half2 hi = __floats2half2_rn(qv[4 * s + 2] * up, qv[4 * s + 3] * up);
    aq[s] = head_ok ? *reinterpret_cast<const uint32_t*>(&lo) : 0u;
    aq2[s] = head_ok ? *reinterpret_cast<const uint32_t*>(&hi) : 0u;
    if (head_ok) {
      const float2 fl = __half22float2(lo), fh = __half22float2(hi);
      qsum += (fl.x + fl.y) + (fh.x + fh.y);
    }
  }
  qsum += __shfl_xor_sync(0xffffffffu, qsum, 1);
  qsum += __shfl_xor_sync(0xffffffffu, qsum, 2);
  const float qoff = 1152.0f * qsum;                 // sum(q' * 1152) over D
  const float fscale = down * p.scale_log2e;         // undo q scaling, softmax scale, log2(e)


  // scales of this lane's 4 tokens, one block ahead
  float sk[4], sv[4], skn[4], svn[4];
  auto load_scales = [&](int i, float* k4, float* v4) {
    const int tb = block_of(i) * 16;
    const int vt[4] = {tb + 2 * t, tb + 2 * t + 1, tb + 2 * t + 8, tb + 2 * t + 9};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int tok = min(vt[j], N - 1);
      k4[j] = __half2float(ksb[tok]);
      v4[j] = __half2float(vsb[tok]);
    }
  };
  if (my_blocks > 0 && !kBulk) load_scales(0, sk, sv);
  bool failed = false;

  int slot = 0;
  uint32_t phase = 0u;
  for (int i = 0; i < my_blocks; ++i) {
    const int tb = block_of(i) * 16;
    if (!kBulk && i + 1 < my_blocks) load_scales(i + 1, skn, svn);
    if (!mbar_wait_bounded(bars + slot, phase)) {
      failed = true;
      break;
    }
    if constexpr (kBulk) {
      // this lane's tokens (2t, 2t+1) and (2t+8, 2t+9) of the block
      const uint8_t* ssl = sring + slot * kSdpaScaleBytes;
      const __half2 k01 = *reinterpret_cast<const __half2*>(ssl + 4 * t);
      const __half2 k89 = *reinterpret_cast<const __half2*>(ssl + 16 + 4 * t);
      const __half2 v01 = *reinterpret_cast<const __half2*>(ssl + 32 + 4 * t);
      const __half2 v89 = *reinterpret_cast<const __half2*>(ssl + 48 + 4 * t);
      sk[0] = __low2float(k01);
      sk[1] = __high2float(k01);
      sk[2] = __low2float(k89);
      sk[3] = __high2float(k89);
      sv[0] = __low2float(v01);
      sv[1] = __high2float(v01);
      sv[2] = __low2float(v89);
      sv[3] = __high2float(v89);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (tb + (j < 2 ? 2 * t + j : 2 * t + 6 + j) >= N) sv[j] = 0.f;  // rows past the length: any bits
    }
    const uint8_t* kst = ring + slot * kStageBytes;
    const uint8_t* vst = kst + 16 * D;
    const int vt[4] = {tb + 2 * t, tb + 2 * t + 1, tb + 2 * t + 8, tb + 2 * t + 9};

    // QK^T: C[u] rows = heads, cols = tokens 8u + (2t, 2t+1); K row (8u + g), bytes 32t..32t+31
    float cqk[2][2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
#pragma unroll
      for (int e = 0; e < 2; ++e) cqk[u][e] = 0.f;
#pragma unroll
      for (int x = 0; x < kBoxes; ++x) {
        const uint4 ka = *reinterpret_cast<const uint4*>(swz128(kst + x * 2048, 8 * u + g, 32 * t));
        const uint4 kb = *reinterpret_cast<const uint4*>(swz128(kst + x * 2048, 8 * u + g, 32 * t + 16));
        const uint32_t kw[8] = {ka.x, ka.y, ka.z, ka.w, kb.x, kb.y, kb.z, kb.w};
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint32_t w = kw[s] ^ 0x80808080u;
          const uint32_t b0 = prmt(w, 0x64646464u, 0x4140u);
          const uint32_t b1 = prmt(w, 0x64646464u, 0x4342u);
          const uint32_t a[4] = {aq[8 * x + s], 0u, aq2[8 * x + s], 0u};
          mma_16816_top(cqk[u], a, b0, b1);
        }
      }
    }
    // scores (log2 domain) for tokens vt[0..3] = (u0: 2t, 2t+1), (u1: 2t+8, 2t+9)
    float sc[4];
    sc[0] = (cqk[0][0] - qoff) * fscale * sk[0];
    sc[1] = (cqk[0][1] - qoff) * fscale * sk[1];
    sc[2] = (cqk[1][0] - qoff) * fscale * sk[2];
    sc[3] = (cqk[1][1] - qoff) * fscale * sk[3];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (vt[j] >= N) sc[j] = -INFINITY;
    float mb = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
    mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, 1));
    mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, 2));
    const float m_new = fmaxf(m_run, mb);
    const float alpha = (m_run == -INFINITY) ? 0.f : exp2f(m_run - m_new);
    float pr[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) pr[j] = (vt[j] < N) ? exp2f(sc[j] - m_new) : 0.f;
    l_run = l_run * alpha + ((pr[0] + pr[1]) + (pr[2] + pr[3]));
    m_run = m_new;
    // rescale only when some row's running maximum moved (alpha == 1 exactly otherwise)
    if (__any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll
      for (int j = 0; j < 16 * kBoxes; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) acc[j][e] *= alpha;
#pragma unroll
      for (int e = 0; e < 2; ++e) psum[e] *= alpha;
    }
    // P' = p * v_scale as the fp16 A operand (rows = heads, k = tokens)
    uint32_t ap[4];
    ap[0] = head_ok ? pack_half2(pr[0] * sv[0], pr[1] * sv[1]) : 0u;
    ap[1] = 0u;
    ap[2] = head_ok ? pack_half2(pr[2] * sv[2], pr[3] * sv[3]) : 0u;
    ap[3] = 0u;
    mma_16816_top(psum, ap, kOnes, kOnes);
    // P'V: n-tile j covers d = 16n + j; the lane's B column n = g reads bytes 16g..16g+15
#pragma unroll
    for (int x = 0; x < kBoxes; ++x) {
      const uint8_t* vbx = vst + x * 2048;  // d = 128x + 16n + j
      const uint4 vr0 = *reinterpret_cast<const uint4*>(swz128(vbx, 2 * t, 16 * g));
      const uint4 vr1 = *reinterpret_cast<const uint4*>(swz128(vbx, 2 * t + 1, 16 * g));
      const uint4 vr2 = *reinterpret_cast<const uint4*>(swz128(vbx, 2 * t + 8, 16 * g));
      const uint4 vr3 = *reinterpret_cast<const uint4*>(swz128(vbx, 2 * t + 9, 16 * g));
      const uint32_t va[4] = {vr0.x, vr0.y, vr0.z, vr0.w}, vb[4] = {vr1.x, vr1.y, vr1.z, vr1.w};
      const uint32_t vc[4] = {vr2.x, vr2.y, vr2.z, vr2.w}, vd[4] = {vr3.x, vr3.y, vr3.z, vr3.w};
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint32_t sel = static_cast<uint32_t>(j & 3) | (static_cast<uint32_t>(4 + (j & 3)) << 8);
        uint32_t b0 = prmt(va[j >> 2], vb[j >> 2], sel);
        uint32_t b1 = prmt(vc[j >> 2], vd[j >> 2], sel);
        b0 = (b0 & 0x00FF00FFu) ^ 0x64806480u;
        b1 = (b1 & 0x00FF00FFu) ^ 0x64806480u;
        mma_16816_top(acc[16 * x + j], ap, b0, b1);
      }
    }
    if constexpr (!kBulk) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sk[j] = skn[j];
        sv[j] = svn[j];
      }
    }
    __syncwarp();
    if (i + NS < my_blocks && lane == 0) {
      fence_proxy_async_smem();
      issue(i + NS, slot);
    }
    if (++slot == NS) {
      slot = 0;
      phase ^= 1u;
    }
  }
  if (failed) {
    if (p.status && lane == 0) atomicOr(p.status, kStatusTimeout);
    for (int i = max(0, my_blocks - NS); i < my_blocks; ++i) mbar_wait_bounded(bars + i % NS, (i / NS) & 1);
    m_run = -INFINITY;
    l_run = 0.f;
  }

  // ---- warp result: o[d] = acc - 1152 * sum(P'); d(j, c0) = 32t + j, d(j, c1) = 32t + 16 + j
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  __shared__ float s_m[kSdpaWarps][8], s_l[kSdpaWarps][8];
  // the warp's partial O [8][D] goes to its own (drained) ring: warp w at ring_of(w)
  auto o_of = [&](int w) {
    return reinterpret_cast<float*>(sbase + 1024 + w * NS * kStageBytes);
  };
  __syncwarp();
  if (head_ok) {
    float* ow = o_of(warp) + g * D;
#pragma unroll
    for (int x = 0; x < kBoxes; ++x)
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        ow[128 * x + 32 * t + j] = acc[16 * x + j][0] - 1152.0f * psum[0];
        ow[128 * x + 32 * t + 16 + j] = acc[16 * x + j][1] - 1152.0f * psum[1];
      }
    if (t == 0) {
      s_m[warp][g] = m_run;
      s_l[warp][g] = l_run;
    }
  }
  __syncthreads();
  grid_dependency_launch();

  // ---- splits of one (b, kv head) in a cluster: reduce-scatter of the CTAs'
  // (m, l, o) over the head dimension in distributed shared memory; rank r
  // merges dims [r*SL, (r+1)*SL) of every head in split order
  if (p.cluster) {
    __shared__ float s_cred[cluster_buf(D)];
    const int S = p.splits, SL = (D + S - 1) / S, stride = SL + 2;
    const uint32_t cred = smem_u32(s_cred);
    for (int idx = threadIdx.x; idx < G * D; idx += kSdpaWarps * 32) {
      const int hh = idx / D, d = idx % D;
      float mm = -INFINITY;
#pragma unroll
      for (int w = 0; w < kSdpaWarps; ++w) mm = fmaxf(mm, s_m[w][hh]);
      float ll = 0.f, oo = 0.f;
      if (mm != -INFINITY) {
#pragma unroll
        for (int w = 0; w < kSdpaWarps; ++w) {
          const float f = s_m[w][hh] == -INFINITY ? 0.f : exp2f(s_m[w][hh] - mm);
          ll += s_l[w][hh] * f;
          oo += o_of(w)[hh * D + d] * f;
        }
      }
      const int r = d / SL;
      const int base = (split * G + hh) * stride;
      st_cluster_f32(cluster_map(cred + 4u * static_cast<uint32_t>(base + d - r * SL), r), oo);
      if (d == 0) {
        for (int rr = 0; rr < S; ++rr) {
          st_cluster_f32(cluster_map(cred + 4u * static_cast<uint32_t>(base + SL), rr), mm);
          st_cluster_f32(cluster_map(cred + 4u * static_cast<uint32_t>(base + SL + 1), rr), ll);
        }
      }
    }
    cluster_sync_all();
    for (int idx = threadIdx.x; idx < G * SL; idx += kSdpaWarps * 32) {
      const int hh = idx / SL, dl = idx % SL, d = split * SL + dl;
      if (d >= D) continue;
      float mm = -INFINITY;
      for (int src = 0; src < S; ++src) mm = fmaxf(mm, s_cred[(src * G + hh) * stride + SL]);
      float ll = 0.f, oo = 0.f;
      if (mm != -INFINITY) {
        for (int src = 0; src < S; ++src) {
          const float ms = s_cred[(src * G + hh) * stride + SL];
          const float w = ms == -INFINITY ? 0.f : exp2f(ms - mm);
          ll += s_cred[(src * G + hh) * stride + SL + 1] * w;
          oo += s_cred[(src * G + hh) * stride + dl] * w;
        }
      }
      p.out[(static_cast<size_t>(b) * p.kv_heads * G + kvh * G + hh) * D + d] =
          __float2bfloat16_rn(ll > 0.f ? oo / ll : 0.f);
    }
    return;
  }

  // ---- CTA merge (fixed warp order) -> partial or final output
  const bool single = p.splits == 1;
  float* part = p.partial + (static_cast<size_t>(bkv) * p.splits + split) * G * kPartStride;
  for (int idx = threadIdx.x; idx < G * D; idx += kSdpaWarps * 32) {
    const int hh = idx / D, d = idx % D;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kSdpaWarps; ++w) mm = fmaxf(mm, s_m[w][hh]);
    float ll = 0.f, oo = 0.f;
    if (mm != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kSdpaWarps; ++w) {
        const float f = s_m[w][hh] == -INFINITY ? 0.f : exp2f(s_m[w][hh] - mm);
        ll += s_l[w][hh] * f;
        oo += o_of(w)[hh * D + d] * f;
      }
    }
    if (single) {
      const float o = ll > 0.f ? oo / ll : 0.f;
      p.out[(static_cast<size_t>(b) * p.kv_heads * G + kvh * G + hh) * D + d] = __float2bfloat16_rn(o);
    } else {
      part[hh * kPartStride + d] = oo;
      if (d == 0) {
        part[hh * kPartStride + D] = mm;
        part[hh * kPartStride + D + 1] = ll;
      }
    }
  }
  if (single) return;

  __threadfence();
  __syncthreads();
  __shared__ unsigned s_prev;
  if (threadIdx.x == 0) s_prev = atomicAdd(p.counters + bkv, 1u);
  __syncthreads();
  if (s_prev != static_cast<unsigned>(p.splits - 1)) return;
  __threadfence();
  const float* all = p.partial + static_cast<size_t>(bkv) * p.splits * G * kPartStride;
  // merge the CTAs' partials in split order: stage (m, l) in shared memory,
  // per-split weights exp2(m_s - M), then O = sum_s w_s * O_s with loads batched
  __shared__ float s_mw[kMaxSplits][8], s_ls[kMaxSplits][8], s_norm[8];
  for (int idx = threadIdx.x; idx < p.splits * G; idx += kSdpaWarps * 32) {
    const int s = idx / G, hh = idx % G;
    s_mw[s][hh] = __ldcg(all + (s * G + hh) * kPartStride + D);
    s_ls[s][hh] = __ldcg(all + (s * G + hh) * kPartStride + D + 1);
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int hh = threadIdx.x;
    float mm = -INFINITY;
    for (int s = 0; s < p.splits; ++s) mm = fmaxf(mm, s_mw[s][hh]);
    float ll = 0.f;
    for (int s = 0; s < p.splits; ++s) {
      const float w = (mm == -INFINITY || s_mw[s][hh] == -INFINITY) ? 0.f : exp2f(s_mw[s][hh] - mm);
      s_mw[s][hh] = w;
      ll += s_ls[s][hh] * w;
    }
    s_norm[hh] = ll > 0.f ? 1.0f / ll : 0.f;
  }
  __syncthreads();
  // every output of this thread loads its next kBatch splits together: one
  // round trip per kBatch splits, not per split and output
  constexpr int kOut = (G * D + kSdpaWarps * 32 - 1) / (kSdpaWarps * 32);
  constexpr int kBatch = 32 / kOut;
  float oo[kOut];
#pragma unroll
  for (int o = 0; o < kOut; ++o) oo[o] = 0.f;
  for (int s0 = 0; s0 < p.splits; s0 += kBatch) {
    float v[kOut][kBatch];
#pragma unroll
    for (int o = 0; o < kOut; ++o) {
      const int idx = threadIdx.x + o * kSdpaWarps * 32;
      const int hh = idx / D, d = idx % D;
#pragma unroll
      for (int j = 0; j < kBatch; ++j)
        v[o][j] = (idx < G * D && s0 + j < p.splits) ? __ldcg(all + ((s0 + j) * G + hh) * kPartStride + d) : 0.f;
    }
#pragma unroll
    for (int o = 0; o < kOut; ++o) {
      const int hh = min((threadIdx.x + o * kSdpaWarps * 32) / D, G - 1);
#pragma unroll
      for (int j = 0; j < kBatch; ++j)
        if (s0 + j < p.splits) oo[o] += v[o][j] * s_mw[s0 + j][hh];
    }
  }
#pragma unroll
  for (int o = 0; o < kOut; ++o) {
    const int idx = threadIdx.x + o * kSdpaWarps * 32;
    if (idx >= G * D) continue;
    const int hh = idx / D, d = idx % D;
    p.out[(static_cast<size_t>(b) * p.kv_heads * G + kvh * G + hh) * D + d] =
        __float2bfloat16_rn(oo[o] * s_norm[hh]);
  }
  if (threadIdx.x == 0) p.counters[bkv] = 0u;
}

namespace {

// Multiprocessor count of the current device (cached per device index).
int sdpa_sms() { return device_sm_count(); }

// Launch plan: warps per CTA (sdpa_warps) and token splits per (batch, kv
// head): one wave of CTAs (two per SM at head_dim 128, one at 256), raised to 16 splits (one thread-block cluster,
// merged in distributed shared memory) when that still puts a CTA on most SMs,
// at least two 16-token blocks per warp. (Measured on B200 at 32K tokens:
// minimising waves per unit of work instead picked 9-15 splits for batch 8-32
// and lost 0-45% to cluster placement and merge cost.)
struct SdpaPlan {
  int warps, splits;
};
SdpaPlan sdpa_plan(int64_t batch, int kv_heads, int64_t length, int D) {
  const int64_t bkv = batch * kv_heads;
  const int64_t nblk = (length + 15) / 16;
  SdpaPlan pl{sdpa_warps(D), 1};
  const int64_t sms = sdpa_sms();
  const int64_t slots = sms * (D == 128 ? 2 : 1);
  int64_t s = (slots + bkv - 1) / bkv;
  // a second wave of a few CTAs costs a whole CTA time: drop to one split less
  // when that still fills three quarters of the slots
  if (s > 1 && bkv * s > slots && bkv * (s - 1) * 4 >= slots * 3) --s;
  // more splits than a cluster holds: keep them (two CTAs per SM, partials
  // merged through the workspace by the last CTA) unless 16 splits already
  // fill nine tenths of the slots (one cluster, merged in shared memory)
  if (s > kSdpaMaxClusterSplits && bkv * kSdpaMaxClusterSplits * 10 >= slots * 9) s = kSdpaMaxClusterSplits;
  s = std::min<int64_t>(s, std::max<int64_t>(1, nblk / (2 * pl.warps)));
  s = std::min<int64_t>(s, kMaxSplits);
  pl.splits = static_cast<int>(std::max<int64_t>(1, s));
  return pl;
}
// splits of the plan the launch uses (workspace sizing)
int sdpa_splits(int64_t batch, int kv_heads, int64_t length, int D) {
  return sdpa_plan(batch, kv_heads, length, D).splits;
}

}  // namespace

size_t sdpa_workspace_bytes(int64_t batch, int num_heads, int num_kv_heads, int64_t length, int D) {
  const int splits = sdpa_splits(batch, num_kv_heads, length, D);
  const int64_t bkv = batch * num_kv_heads;
  const int G = num_heads / num_kv_heads;
  const size_t counters = kCounterBytes;
  return counters + static_cast<size_t>(bkv) * splits * G * part_stride(D) * sizeof(float);
}

int run_sdpa_int8(const void* q, const int8_t* k, const void* k_scale, const int8_t* v, const void* v_scale,
                  void* out, int64_t batch, int num_heads, int num_kv_heads, int64_t length, int64_t capacity,
                  int head_dim, float scale, void* workspace, size_t workspace_bytes, cudaStream_t stream,
                  int force_splits, const int* length_dev, int length_offset, int early = 0,
                  int plan_kv_heads = 0) {
  SB_REQUIRE(head_dim == 128 || head_dim == 256, "head_dim must be 128 or 256");
  SB_REQUIRE(batch > 0 && num_heads > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0,
             "Nonempty inputs and query heads divisible by KV heads required");
  const int G = num_heads / num_kv_heads;
  SB_REQUIRE(G == 1 || G == 2 || G == 4 || G == 8, "query heads per KV head must be 1, 2, 4 or 8");
  SB_REQUIRE(length > 0 && length <= capacity && capacity < (1LL << 31), "need 0 < length <= capacity < 2^31");
  SB_REQUIRE(std::isfinite(scale), "scale must be finite");
  SB_REQUIRE(((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) &
              15) == 0,
             "q, k and v must be 16-byte aligned");
  const bool bulk = capacity % 16 == 0 &&
                    ((reinterpret_cast<uintptr_t>(k_scale) | reinterpret_cast<uintptr_t>(v_scale)) & 15) == 0;
  // plan_kv_heads > 0: split the tokens as for that many KV heads (a tensor-
  // parallel shard planning like the unsharded model, so its heads merge alike)
  const SdpaPlan plan =
      sdpa_plan(batch, plan_kv_heads > 0 ? plan_kv_heads : num_kv_heads, length, head_dim);
  int splits = force_splits > 0 ? force_splits : plan.splits;
  SB_REQUIRE(splits <= kMaxSplits, "at most 64 token splits");
  const int64_t bkv = batch * num_kv_heads;
  const size_t counters = kCounterBytes;
  // one arrival counter per (batch, kv head): more of them than the counter
  // region holds run unsplit
  if (bkv > kMaxCounters) {
    SB_REQUIRE(force_splits <= 1, "a forced split count needs at most 32752 (batch x kv head) rows");
    splits = 1;
  }
  const size_t need = counters + static_cast<size_t>(bkv) * splits * G * part_stride(head_dim) * sizeof(float);
  if (splits > 1 && (workspace == nullptr || workspace_bytes < need)) {
    SB_REQUIRE(force_splits <= 0, "workspace too small for the requested split count");
    splits = 1;
  }
  SdpaParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = k;
  p.ks = static_cast<const __half*>(k_scale);
  p.v = v;
  p.vs = static_cast<const __half*>(v_scale);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.kv_heads = num_kv_heads;
  p.length = static_cast<int>(length);
  p.capacity = static_cast<int>(capacity);
  p.splits = splits;
  p.length_dev = length_dev;
  {
    const uint64_t rows = static_cast<uint64_t>(bkv) * static_cast<uint64_t>(capacity);
    if (rows >= (1ULL << 31)) return fail(SB_EINVAL, "KV cache too large for 32-bit TMA row coordinates");
    if (int st = make_tmap_rows(&p.kmap, k, rows, head_dim, 16)) return st;
    if (int st = make_tmap_rows(&p.vmap, v, rows, head_dim, 16)) return st;
  }
  p.length_offset = length_offset;
  p.scale_bulk = bulk ? 1 : 0;
  p.scale_log2e = scale * 1.4426950408889634f;
  if (splits > 1) {
    p.counters = static_cast<unsigned*>(workspace);
    p.partial = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + counters);
  }
  if (workspace != nullptr && workspace_bytes >= kCounterBytes)
    p.status = static_cast<unsigned*>(workspace) + kStatusWord;
  p.early = early ? 1 : 0;
  const dim3 grid(splits, static_cast<unsigned>(bkv));
  const dim3 block(plan.warps * 32);
  // Ring depth: 3 blocks per warp. (A 6-deep ring when the grid leaves one CTA
  // per SM measured slower on B200 at batch 1 / 32K tokens: 52 vs 40 us.)
  p.stages = kSdpaStages;
  const size_t smem = sdpa_smem(plan.warps, p.stages, head_dim);
  auto go = [&](auto kernel) -> int {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return fail(SB_ECUDA, "int8 sdpa: shared memory opt-in failed");
    // splits of one (batch, kv head) merge inside a thread-block cluster when it can hold them
    p.cluster = 0;
    if (splits > 1 && splits <= kSdpaMaxClusterSplits) {
      bool ok = splits <= 8;
      if (!ok) {
        ok = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
        if (!ok) cudaGetLastError();
      }
      p.cluster = ok ? 1 : 0;
    }
    if (p.cluster) return launch_cluster("int8 sdpa", kernel, grid, block, smem, splits, stream, p);
    return launch("int8 sdpa", kernel, grid, block, smem, stream, p);
  };
  switch (G * 1000 + head_dim) {
#define SB_SDPA_GO(GG, DD)                                                                                  \
  case GG * 1000 + DD:                                                                                     \
    return bulk ? go(sdpa_int8_decode_kernel<GG, true, sdpa_warps(DD), DD>)                                \
                : go(sdpa_int8_decode_kernel<GG, false, sdpa_warps(DD), DD>);
    SB_SDPA_GO(1, 128)
    SB_SDPA_GO(2, 128)
    SB_SDPA_GO(4, 128)
    SB_SDPA_GO(8, 128)
    SB_SDPA_GO(1, 256)
    SB_SDPA_GO(2, 256)
    SB_SDPA_GO(4, 256)
    SB_SDPA_GO(8, 256)
#undef SB_SDPA_GO
    default:
      return fail(SB_EINVAL, "unsupported head_dim / GQA combination");
  }
}

}  // namespace sb

extern "C" size_t sb_int8_sdpa_workspace_size(int64_t batch, int num_heads, int num_kv_heads, int64_t length,
                                              int head_dim) {
  if (batch <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads || length <= 0 ||
      (head_dim != 128 && head_dim != 256))
    return 0;
  return sb::sdpa_workspace_bytes(batch, num_heads, num_kv_heads, length, head_dim);
}

extern "C" int sb_int8_sdpa_decode(const void* q, const int8_t* k, const void* k_scale, const int8_t* v,
                                   const void* v_scale, void* out, int64_t batch, int num_heads, int num_kv_heads,
                                   int64_t length, int64_t capacity, int head_dim, float scale, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  return sb::run_sdpa_int8(q, k, k_scale, v, v_scale, out, batch, num_heads, num_kv_heads, length, capacity,
                           head_dim, scale, workspace, workspace_bytes, sb::as_stream(stream), 0, nullptr, 0);
}

// ---------------------------------------------------------------------------
// Allocation-free variant: the split-K scratch (arrival counters, status word,
// per-split partial results) lives in a file-scope device array instead of a
// caller workspace. Every GPU that loads this library keeps the array until the
// process exits.
namespace {

constexpr size_t kStaticScratchBytes = size_t(4) << 20;  // 4 MiB per device
static __device__ __align__(256) unsigned char g_sdpa_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_static_scratch_mutex;
void* g_static_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device. The host-side name
// g_sdpa_static_scratch is only a stand-in, so the address is looked up once per
// device (with that device current) and cached.
int static_scratch_address(void** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return sb::fail(SB_ECUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(err));
  if (dev < 0 || dev >= kMaxDevices) return sb::fail(SB_EUNSUPPORTED, "device index out of range for the static scratch");
  std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
  if (g_static_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_sdpa_static_scratch);
    if (err != cudaSuccess || ptr == nullptr)
      return sb::fail(SB_ECUDA, std::string("cudaGetSymbolAddress(static scratch): ") + cudaGetErrorString(err));
    g_static_scratch_ptr[dev] = ptr;
  }
  *out = g_static_scratch_ptr[dev];
  return SB_OK;
}

}  // namespace

extern "C" int sb_int8_sdpa_decode_static(const void* q, const int8_t* k, const void* k_scale, const int8_t* v,
                                          const void* v_scale, void* out, int64_t batch, int num_heads,
                                          int num_kv_heads, int64_t length, int64_t capacity, int head_dim,
                                          float scale, void* stream) {
  SB_REQUIRE(batch > 0 && num_kv_heads > 0 && num_heads > 0 && num_heads % num_kv_heads == 0 && length > 0,
             "Nonempty inputs and query heads divisible by KV heads required");
  SB_REQUIRE(head_dim == 128 || head_dim == 256, "head_dim must be 128 or 256");
  const size_t need = sb::sdpa_workspace_bytes(batch, num_heads, num_kv_heads, length, head_dim);
  if (need > kStaticScratchBytes)
    return sb::fail(SB_EINVAL, "sb_int8_sdpa_decode_static: this shape needs " + std::to_string(need) +
                                   " bytes of scratch but the static scratch holds " +
                                   std::to_string(kStaticScratchBytes) +
                                   " bytes; use sb_int8_sdpa_decode with a caller workspace");
  void* scratch = nullptr;
  if (int st = static_scratch_address(&scratch)) return st;
  // The array keeps the previous call's contents: clear the arrival counters and
  // the status word (everything the kernel expects to start at zero).
  cudaError_t err = cudaMemsetAsync(scratch, 0, sb::kCounterBytes, sb::as_stream(stream));
  if (err != cudaSuccess) return sb::fail(SB_ECUDA, std::string("clearing static scratch: ") + cudaGetErrorString(err));
  return sb::run_sdpa_int8(q, k, k_scale, v, v_scale, out, batch, num_heads, num_kv_heads, length, capacity,
                           head_dim, scale, scratch, kStaticScratchBytes, sb::as_stream(stream), 0, nullptr, 0);
}

extern "C" int sb_int8_sdpa_decode_dev(const void* q, const int8_t* k, const void* k_scale, const int8_t* v,
                                       const void* v_scale, void* out, int64_t batch, int num_heads,
                                       int num_kv_heads, const int32_t* lengths, int length_offset,
                                       int64_t max_length, int64_t capacity, int head_dim, float scale,
                                       int prefix_constant, int plan_kv_heads, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  SB_REQUIRE(lengths != nullptr, "lengths must be a device pointer");
  SB_REQUIRE(plan_kv_heads >= 0, "plan_kv_heads must be >= 0");
  return sb::run_sdpa_int8(q, k, k_scale, v, v_scale, out, batch, num_heads, num_kv_heads, max_length, capacity,
                           head_dim, scale, workspace, workspace_bytes, sb::as_stream(stream), 0, lengths,
                           length_offset, prefix_constant, plan_kv_heads);
}
