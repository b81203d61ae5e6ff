// Weight-streaming linear kernels (M <= 8) and their C-ABI entry points.
// The design notes are in sb_gemv.cuh.
#include <algorithm>
#include <cmath>
#include <mutex>

#include "sb_gemv.cuh"

namespace sb {

template <typename TA>
struct ActTraits;
template <>
struct ActTraits<__nv_bfloat16> {
  static constexpr bool kHalf = false;
  static constexpr uint32_t kMagic = 0x43004300u;  // bf16 128.0 | code
  static constexpr uint32_t kOnes = 0x3F803F80u;   // bf16 pair (1.0, 1.0)
  static constexpr float kOffset = 128.0f;
};
template <>
struct ActTraits<__half> {
  static constexpr bool kHalf = true;
  static constexpr uint32_t kMagic = 0x64006400u;  // fp16 1024.0 | code
  static constexpr uint32_t kOnes = 0x3C003C00u;   // fp16 pair (1.0, 1.0)
  static constexpr float kOffset = 1024.0f;
};

template <typename TA, int WF>
struct Fmt {
  static constexpr bool kHalf = ActTraits<TA>::kHalf;
  // Two exact nibble planes are needed for 8-bit codes with bf16 operands.
  static constexpr int kPlanes = ((WF == W_AFF8 || WF == W_I8PC) && !kHalf) ? 2 : 1;
  static constexpr int kBits = WF == W_AFF4 ? 4 : (WF == W_BF16 ? 16 : 8);
  // sum(code * x) = C_lo + 16 * C_hi - kCodeOffset * sum(x)
  static constexpr float kCodeOffset =
      WF == W_BF16 ? 0.0f
                   : (kPlanes == 2 ? ActTraits<TA>::kOffset * 17.0f : ActTraits<TA>::kOffset);
};

// Loads `kWords` consecutive uint32 words (streaming, 4..32 bytes).
template <int kWords>
__device__ __forceinline__ void load_words(const uint8_t* p, uint32_t (&out)[kWords]) {
  if constexpr (kWords == 1) {
    out[0] = ldg_stream4(p);
  } else if constexpr (kWords == 2) {
    uint2 v = ldg_stream8(p);
    out[0] = v.x;
    out[1] = v.y;
  } else {
#pragma unroll
    for (int i = 0; i < kWords; i += 4) {
      uint4 v = ldg_stream16(p + 4 * i);
      out[i] = v.x;
      out[i + 1] = v.y;
      out[i + 2] = v.z;
      out[i + 3] = v.w;
    }
  }
}

// Converts one row segment of packed codes into MMA A-operand pairs.
// Pair order (shared with the x pairs below):
//   4-bit : pair 4w+j holds values (8w+j, 8w+j+4) of the segment
//   8-bit : pair 2w+i holds values (4w+2i, 4w+2i+1)
//   bf16  : pair i holds values (2i, 2i+1)
template <typename TA, int WF, int kWords, int kPairs>
__device__ __forceinline__ void dequant_pairs(const uint32_t (&w)[kWords],
                                              uint32_t (&lo)[kPairs], uint32_t (&hi)[kPairs]) {
  constexpr uint32_t kMagic = ActTraits<TA>::kMagic;
  if constexpr (WF == W_AFF4) {
#pragma unroll
    for (int i = 0; i < kWords; ++i) {
      lo[4 * i + 0] = lop_and_or(w[i], 0x000F000Fu, kMagic);
      lo[4 * i + 1] = lop_and_or(w[i] >> 4, 0x000F000Fu, kMagic);
      lo[4 * i + 2] = lop_and_or(w[i] >> 8, 0x000F000Fu, kMagic);
      lo[4 * i + 3] = lop_and_or(w[i] >> 12, 0x000F000Fu, kMagic);
    }
  } else if constexpr (WF == W_AFF8 || WF == W_I8PC) {
#pragma unroll
    for (int i = 0; i < kWords; ++i) {
      const uint32_t u = (WF == W_I8PC) ? (w[i] ^ 0x80808080u) : w[i];
      if constexpr (ActTraits<TA>::kHalf) {
        lo[2 * i + 0] = prmt(u, 0x64646464u, 0x4140u);
        lo[2 * i + 1] = prmt(u, 0x64646464u, 0x4342u);
      } else {
        const uint32_t t0 = prmt(u, 0u, 0x4140u);
        const uint32_t t1 = prmt(u, 0u, 0x4342u);
        lo[2 * i + 0] = lop_and_or(t0, 0x000F000Fu, kMagic);
        lo[2 * i + 1] = lop_and_or(t1, 0x000F000Fu, kMagic);
        hi[2 * i + 0] = lop_and_or(t0 >> 4, 0x000F000Fu, kMagic);
        hi[2 * i + 1] = lop_and_or(t1 >> 4, 0x000F000Fu, kMagic);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < kWords; ++i) lo[i] = w[i];
  }
}

// x values (bf16/fp16 pairs as stored) -> B-operand pairs in the same order.
template <int WF, int kXWords, int kPairs>
__device__ __forceinline__ void x_pairs(const uint32_t (&xw)[kXWords], uint32_t (&xp)[kPairs]) {
  if constexpr (WF == W_AFF4) {
#pragma unroll
    for (int w = 0; w < kXWords / 4; ++w) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        xp[4 * w + j] = prmt(xw[4 * w + j / 2], xw[4 * w + 2 + j / 2], (j & 1) ? 0x7632u : 0x5410u);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < kPairs; ++i) xp[i] = xw[i];
  }
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int index) {
  uint32_t u = __float_as_uint(v);
  if (v != v) u = 0x007FFFFFu;  // NaN ranks below every number
  else u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<unsigned long long>(u) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(index));
}

template <typename TA>
__device__ __forceinline__ void store_act(void* base, size_t index, float v) {
  static_cast<TA*>(base)[index] = from_float<TA>(v);
}
template <typename TA>
__device__ __forceinline__ float load_act(const void* base, size_t index) {
  return to_float(static_cast<const TA*>(base)[index]);
}
template <typename TA>
__device__ __forceinline__ float round_act(float v) {
  return to_float(from_float<TA>(v));
}

// ---- warp row blocks
// A warp owns 32 weight rows, fetched per stage as two TMA boxes (A and B) of
// 16 rows x 128 bytes. MMA rows 0-7 of tile r come from box A rows 8r + sigma(g),
// MMA rows 8-15 from box B rows 8r + sigma(g). sigma relabels the rows so the
// lanes' reads of the 128-byte-swizzled boxes hit distinct banks.
template <int kBits>
__device__ __forceinline__ int sigma_row(int g) {
  if constexpr (kBits == 4) return ((g & 3) << 1) | (g >> 2);   // 0,2,4,6,1,3,5,7
  else if constexpr (kBits == 8) return ((g & 1) << 2) | (g >> 1);  // 0,4,1,5,2,6,3,7
  else return g;
}

// number of 32-row warp blocks
template <int EPI>
__device__ __forceinline__ int warp_blocks(const GemvParams& p) {
  if constexpr (EPI == EPI_SWIGLU) return (p.N + 15) / 16;
  else if constexpr (EPI == EPI_ROPE) return p.N / 32;
  else return (p.N + 31) / 32;
}

// first weight row of box h (0 = A, 1 = B) of warp block rb
template <int EPI>
__device__ __forceinline__ int box_row0(const GemvParams& p, int rb, int h) {
  if constexpr (EPI == EPI_SWIGLU) {
    return 16 * rb;  // gate rows in A, the same up rows in B
  } else if constexpr (EPI == EPI_ROPE) {
    const int wph = p.head_dim / 32;  // warp blocks per head
    return (rb / wph) * p.head_dim + h * (p.head_dim / 2) + 16 * (rb % wph);
  } else {
    return 32 * rb + 16 * h;
  }
}

template <int kBits>
struct StageGeom {
  static constexpr int kRowBytes = 128;                  // bytes of one weight row per stage
  static constexpr int kStageK = kRowBytes * 8 / kBits;  // K values per stage
  static constexpr int kStages = 4;                      // ring depth per warp
  static constexpr int kStageBytes = 32 * kRowBytes;     // two 16-row boxes
};

template <typename TA, int WF, int KC, int GC, int EPI, bool NORM, int MC>
__global__ void __launch_bounds__(kGemvWarps * 32, 2) gemv_kernel(const __grid_constant__ GemvParams p) {
  using F = Fmt<TA, WF>;
  using SG = StageGeom<F::kBits>;
  constexpr int V = KC / 4;                      // values per lane per row per chunk
  constexpr int kPairs = V / 2;                  // MMA operand pairs per row per chunk
  constexpr int kMma = KC / 16;                  // k16 steps per chunk
  constexpr int kWords = V * F::kBits / 32;      // weight words per lane per row per chunk
  constexpr int kXWords = V / 2;                 // activation words per lane per chunk
  constexpr int kRows = 2 * kGemvTiles;          // weight rows held per lane
  constexpr bool kAffine = (WF == W_AFF4 || WF == W_AFF8);
  constexpr int kGroupK = kAffine ? KC * GC : KC;  // K covered by one split unit
  constexpr int kChunkRowBytes = KC * F::kBits / 8;
  constexpr int kLaneBytes = V * F::kBits / 8;
  constexpr int kChunksPerStage = SG::kStageK / KC;
  // The MMA's 8 n-columns carry (activation column m, group slot) pairs:
  // column n -> m = n % MC, slot = n / MC. An affine "super-group" of kSlots
  // consecutive groups accumulates in separate columns; its scales are applied
  // once at its end. Non-affine formats use one slot (columns = activation rows).
  constexpr int kSlots = kAffine ? 8 / MC : 1;
  constexpr int kSuperChunks = kSlots * GC;
  static_assert(!kAffine || kChunksPerStage % GC == 0, "a stage holds whole groups");

  extern __shared__ uint8_t smem_dyn[];
  __shared__ float s_rms[8];
  __shared__ float s_part[kGemvWarps][8];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;
  const int t = lane & 3;
  const int sg = sigma_row<F::kBits>(g);
  const int split = blockIdx.y;
  const int rowblocks = warp_blocks<EPI>(p);
  const int rb = blockIdx.x * kGemvWarps + warp;
  const bool active = rb < rowblocks;
  const int rbc = min(rb, rowblocks - 1);
  const int mcols = p.M;

  // K range of this split, in whole groups.
  const int grp_begin = static_cast<int>((static_cast<long long>(p.groups_total) * split) / p.splits);
  const int grp_end = static_cast<int>((static_cast<long long>(p.groups_total) * (split + 1)) / p.splits);
  const int k_begin = grp_begin * kGroupK;
  const int k_count = (grp_end - grp_begin) * kGroupK;
  const int nstages = (k_count + SG::kStageK - 1) / SG::kStageK;
  const int nchunks = k_count / KC;
  const int kbyte0 = k_begin * F::kBits / 8;

  // ---- shared memory: barriers, per-warp weight rings (1 KB aligned), x segment, x group sums
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base) + warp * SG::kStages;
  uint8_t* ring = base + 1024 + (warp * SG::kStages) * SG::kStageBytes;
  TA* xs = reinterpret_cast<TA*>(base + 1024 + kGemvWarps * SG::kStages * SG::kStageBytes);
  const int xs_ld = p.x_seg + 8;
  float* xgs = reinterpret_cast<float*>(xs + mcols * xs_ld);  // [M][x_seg / kGroupK]
  const int xg_ld = p.x_seg / kGroupK;
  const int rowA = box_row0<EPI>(p, rbc, 0), rowB = box_row0<EPI>(p, rbc, 1);

  auto issue_stage = [&](int st) {
    const int slot = st % SG::kStages;
    uint8_t* dst = ring + slot * SG::kStageBytes;
    mbar_arrive_expect_tx(bars + slot, SG::kStageBytes);
    const int x = kbyte0 + st * SG::kRowBytes;
    tma_load_2d(dst, &p.tmap0, x, rowA, bars + slot);
    tma_load_2d(dst + 16 * SG::kRowBytes, &p.tmap1, x, rowB, bars + slot);
  };

  if (active && lane == 0) {
    for (int i = 0; i < SG::kStages; ++i) mbar_init(bars + i, 1);
    mbar_fence_init();
  }
  __syncwarp();
  // ---- start streaming weights; with constant weights this may overlap the
  // tail of the previous kernel in the stream
  if (!p.early_prefetch) grid_dependency_wait();
  if (active && lane == 0) {
    for (int st = 0; st < SG::kStages && st < nstages; ++st) issue_stage(st);
  }

  // ---- activations depend on the previous kernel from here on
  grid_dependency_wait();
  if constexpr (NORM) {
    // full-row sum of squares per column (fixed reduction order)
    for (int m = 0; m < mcols; ++m) {
      float ss = 0.f;
      const TA* xr = static_cast<const TA*>(p.x) + static_cast<size_t>(m) * p.ldx;
      for (int k = threadIdx.x * 8; k < p.K; k += kGemvWarps * 32 * 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
        const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float a, b;
          if constexpr (ActTraits<TA>::kHalf) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&vv[i]));
            a = f.x;
            b = f.y;
          } else {
            a = bf16_lo(vv[i]);
            b = bf16_hi(vv[i]);
          }
          ss = fmaf(a, a, ss);
          ss = fmaf(b, b, ss);
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) s_part[warp][m] = ss;
    }
    __syncthreads();
    if (threadIdx.x < mcols) {
      float ss = 0.f;
#pragma unroll
      for (int w = 0; w < kGemvWarps; ++w) ss += s_part[w][threadIdx.x];
      s_rms[threadIdx.x] = 1.0f / sqrtf(ss / static_cast<float>(p.K) + p.eps);
    }
  }

  // B-operand column of this lane: activation column bm, group slot bslot
  const int bm = g % MC;
  const int bslot = g / MC;
  const bool b_live = bm < mcols && (kAffine || bslot == 0);

  constexpr uint32_t kOnes = ActTraits<TA>::kOnes;
  float cacc[kGemvTiles][F::kPlanes][4];
  float xsum[4];
  float res[kGemvTiles][2][2];  // [tile][h][e] affine results per (row, column)
#pragma unroll
  for (int r = 0; r < kGemvTiles; ++r)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
#pragma unroll
      for (int pl = 0; pl < F::kPlanes; ++pl) cacc[r][pl][e] = 0.f;
      res[r][e >> 1][e & 1] = 0.f;
    }
#pragma unroll
  for (int e = 0; e < 4; ++e) xsum[e] = 0.f;

  // scale/bias of this lane's rows (tile r, box h) for its two columns' groups
  auto row_of = [&](int r, int h) { return min((h ? rowB : rowA) + 8 * r + sg, p.N - 1); };
  auto set_of = [&](int h) { return (EPI == EPI_SWIGLU) ? h : 0; };
  uint32_t sbv[kGemvTiles][2][2];  // packed (scale, bias) for [tile][h][e]
  auto load_super_scales = [&](int grp0) {
    if constexpr (kAffine) {
      const int gpr = p.K / p.group_size;
#pragma unroll
      for (int r = 0; r < kGemvTiles; ++r)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int grp = min(grp0 + (2 * t + e) / MC, grp_end - 1);
            const size_t idx = static_cast<size_t>(row_of(r, h)) * gpr + grp;
            const uint16_t s = *reinterpret_cast<const uint16_t*>(static_cast<const TA*>(set_of(h) ? p.s1 : p.s0) + idx);
            const uint16_t b = *reinterpret_cast<const uint16_t*>(static_cast<const TA*>(set_of(h) ? p.b1 : p.b0) + idx);
            sbv[r][h][e] = static_cast<uint32_t>(s) | (static_cast<uint32_t>(b) << 16);
          }
    }
  };
  if (active && nchunks > 0) load_super_scales(grp_begin);

  bool failed = false;
  int chunk = 0;  // chunk index inside the split
  for (int st = 0; st < nstages; ++st) {
    // ---- activation segment staging (all warps of the CTA take part)
    const int kst = st * SG::kStageK;  // offset inside the split
    if (kst % p.x_seg == 0) {
      __syncthreads();
      const int seg_len = min(p.x_seg, k_count - kst);
      const int vecs = seg_len / 8;
      for (int idx = threadIdx.x; idx < mcols * vecs; idx += kGemvWarps * 32) {
        const int m = idx / vecs, v8 = idx % vecs;
        const int kg = k_begin + kst + v8 * 8;
        uint4 v = *reinterpret_cast<const uint4*>(static_cast<const TA*>(p.x) + static_cast<size_t>(m) * p.ldx + kg);
        if constexpr (NORM) {
          const uint4 wv = *reinterpret_cast<const uint4*>(static_cast<const TA*>(p.norm_w) + kg);
          const TA* xv = reinterpret_cast<const TA*>(&v);
          const TA* nv = reinterpret_cast<const TA*>(&wv);
          TA out[8];
          const float r = s_rms[m];
#pragma unroll
          for (int i = 0; i < 8; ++i) out[i] = from_float<TA>(to_float(xv[i]) * r * to_float(nv[i]));
          v = *reinterpret_cast<const uint4*>(out);
        }
        *reinterpret_cast<uint4*>(xs + m * xs_ld + v8 * 8) = v;
      }
      if constexpr (kAffine) {
        __syncthreads();
        // per-group sums of the staged activations (fixed order)
        const int ng = seg_len / kGroupK;
        for (int idx = threadIdx.x; idx < mcols * ng; idx += kGemvWarps * 32) {
          const int m = idx / ng, gi = idx % ng;
          const TA* xp = xs + m * xs_ld + gi * kGroupK;
          float sum = 0.f;
          for (int i = 0; i < kGroupK; ++i) sum += to_float(xp[i]);
          xgs[m * xg_ld + gi] = sum;
        }
      }
      __syncthreads();
    }
    if (!active || failed) continue;

    const int slot = st % SG::kStages;
    if (!mbar_wait_bounded(bars + slot, (st / SG::kStages) & 1)) {
      failed = true;
      continue;
    }
    const uint8_t* stage = ring + slot * SG::kStageBytes;
    const int chunks = min(kChunksPerStage, (k_count - kst) / KC);
    const TA* xbase = xs + min(bm, mcols - 1) * xs_ld + (kst % p.x_seg) + t * V;
#pragma unroll
    for (int cc = 0; cc < kChunksPerStage; ++cc) {
      if (cc < chunks) {
        uint32_t wv[kRows][kWords];
#pragma unroll
        for (int q = 0; q < kRows; ++q) {
          const uint8_t* box = stage + (q & 1) * 16 * SG::kRowBytes;
          const int row = 8 * (q >> 1) + sg;
          const int byte = cc * kChunkRowBytes + t * kLaneBytes;
          if constexpr (kWords == 1) {
            wv[q][0] = *reinterpret_cast<const uint32_t*>(swz128(box, row, byte));
          } else if constexpr (kWords == 2) {
            const uint2 v = *reinterpret_cast<const uint2*>(swz128(box, row, byte));
            wv[q][0] = v.x;
            wv[q][1] = v.y;
          } else {
#pragma unroll
            for (int i = 0; i < kWords; i += 4) {
              const uint4 v = *reinterpret_cast<const uint4*>(swz128(box, row, byte + 4 * i));
              wv[q][i] = v.x;
              wv[q][i + 1] = v.y;
              wv[q][i + 2] = v.z;
              wv[q][i + 3] = v.w;
            }
          }
        }
        uint32_t lo[kRows][kPairs], hi[kRows][kPairs];
#pragma unroll
        for (int q = 0; q < kRows; ++q) dequant_pairs<TA, WF, kWords, kPairs>(wv[q], lo[q], hi[q]);
        // B operand: this lane's column feeds only the group of its slot
        const int gslot = (chunk / GC) % kSlots;
        const bool feed = b_live && (bslot == gslot);
        uint32_t xpair[kPairs];
        if (feed) {
          uint32_t xw[kXWords];
#pragma unroll
          for (int i = 0; i < kXWords; i += 4) {
            const uint4 v = *reinterpret_cast<const uint4*>(xbase + cc * KC + 2 * i);
            xw[i] = v.x;
            xw[i + 1] = v.y;
            xw[i + 2] = v.z;
            xw[i + 3] = v.w;
          }
          x_pairs<WF, kXWords, kPairs>(xw, xpair);
        } else {
#pragma unroll
          for (int i = 0; i < kPairs; ++i) xpair[i] = 0u;
        }
#pragma unroll
        for (int j = 0; j < kMma; ++j) {
          const uint32_t b0 = xpair[2 * j], b1 = xpair[2 * j + 1];
#pragma unroll
          for (int r = 0; r < kGemvTiles; ++r) {
            const uint32_t a_lo[4] = {lo[2 * r][2 * j], lo[2 * r + 1][2 * j], lo[2 * r][2 * j + 1],
                                      lo[2 * r + 1][2 * j + 1]};
            mma_16816<F::kHalf>(cacc[r][0], a_lo, b0, b1);
            if constexpr (F::kPlanes == 2) {
              const uint32_t a_hi[4] = {hi[2 * r][2 * j], hi[2 * r + 1][2 * j], hi[2 * r][2 * j + 1],
                                        hi[2 * r + 1][2 * j + 1]};
              mma_16816<F::kHalf>(cacc[r][1], a_hi, b0, b1);
            }
          }
          if constexpr (WF == W_I8PC) {
            const uint32_t ones[4] = {kOnes, kOnes, kOnes, kOnes};
            mma_16816<F::kHalf>(xsum, ones, b0, b1);
          }
        }
        ++chunk;
        if constexpr (kAffine) {
          if (chunk % kSuperChunks == 0 || chunk == nchunks) {
            // super-group epilogue: res += scale * sum(code*x) + (bias - offset*scale) * sum(x)
            const int grp0 = grp_begin + (chunk - 1) / kSuperChunks * kSlots;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int n = 2 * t + e;
              const int grp = grp0 + n / MC;
              const int m = n % MC;
              const bool ok = grp < grp_end && m < mcols;
              float xg = 0.f;
              if (ok) {
                const int k_in_seg = (grp - grp_begin) * kGroupK - (kst / p.x_seg) * p.x_seg;
                xg = xgs[m * xg_ld + k_in_seg / kGroupK];
              }
#pragma unroll
              for (int r = 0; r < kGemvTiles; ++r)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  const uint32_t v = sbv[r][h][e];
                  float s, b;
                  if constexpr (ActTraits<TA>::kHalf) {
                    s = __half2float(__ushort_as_half(static_cast<unsigned short>(v & 0xFFFFu)));
                    b = __half2float(__ushort_as_half(static_cast<unsigned short>(v >> 16)));
                  } else {
                    s = bf16_lo(v);
                    b = bf16_hi(v);
                  }
                  float d = cacc[r][0][2 * h + e];
                  if constexpr (F::kPlanes == 2) d = fmaf(16.0f, cacc[r][1][2 * h + e], d);
                  const float bb = fmaf(-F::kCodeOffset, s, b);
                  res[r][h][e] = ok ? fmaf(s, d, fmaf(bb, xg, res[r][h][e])) : res[r][h][e];
                }
            }
#pragma unroll
            for (int r = 0; r < kGemvTiles; ++r)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                cacc[r][0][e] = 0.f;
                if constexpr (F::kPlanes == 2) cacc[r][1][e] = 0.f;
              }
            if (chunk < nchunks) load_super_scales(grp0 + kSlots);
          }
        }
      }
    }
    // refill this slot with the stage kStages ahead
    __syncwarp();
    if (st + SG::kStages < nstages && lane == 0) {
      fence_proxy_async_smem();
      issue_stage(st + SG::kStages);
    }
  }
  if (!active) return;
  if (failed) {
    // a TMA load never completed: report, drain what is still in flight, stop
    if (p.status && lane == 0) atomicOr(p.status, kStatusTimeout);
    for (int st = max(0, nstages - SG::kStages); st < nstages; ++st)
      mbar_wait_bounded(bars + st % SG::kStages, (st / SG::kStages) & 1);
    return;
  }

  // ---- per-lane results: value[r][h][e] for activation column m = 2t + e
  // (after reducing the lanes that hold other group slots of the same column)
  float val[kGemvTiles][2][2];
  if constexpr (kAffine) {
#pragma unroll
    for (int r = 0; r < kGemvTiles; ++r)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if constexpr (MC == 1) {
          float v = res[r][h][0] + res[r][h][1];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          val[r][h][0] = v;
          val[r][h][1] = 0.f;
        } else {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float v = res[r][h][e];
            if constexpr (MC == 2) {
              v += __shfl_xor_sync(0xffffffffu, v, 1);
              v += __shfl_xor_sync(0xffffffffu, v, 2);
            } else if constexpr (MC == 4) {
              v += __shfl_xor_sync(0xffffffffu, v, 2);
            }
            val[r][h][e] = v;
          }
        }
      }
  } else {
#pragma unroll
    for (int r = 0; r < kGemvTiles; ++r)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float d = cacc[r][0][2 * h + e];
          if constexpr (F::kPlanes == 2) d = fmaf(16.0f, cacc[r][1][2 * h + e], d);
          if constexpr (WF == W_I8PC) d = fmaf(-(F::kCodeOffset + 128.0f), xsum[e], d);
          val[r][h][e] = d;
        }
  }
  // owner lanes: t < MC/2 (MC == 1: t == 0, e == 0); column m = 2t + e
  const bool owner = (MC == 1) ? (t == 0) : (2 * t < MC);
  auto col_ok = [&](int e) { return owner && (MC == 1 ? e == 0 : true) && (2 * t + e) < mcols; };

  grid_dependency_launch();

  // ---- split-K: publish partials; the last warp of the row block reduces
  if (p.splits > 1) {
    float* part = p.partial + (static_cast<size_t>(split) * p.rows_padded + rb * 32) * 8;
#pragma unroll
    for (int r = 0; r < kGemvTiles; ++r)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int e = 0; e < 2; ++e)
          if (col_ok(e)) part[(r * 16 + h * 8 + g) * 8 + 2 * t + e] = val[r][h][e];
    __threadfence();
    __syncwarp();
    unsigned prev = 0;
    if (lane == 0) prev = atomicAdd(p.counters + rb, 1u);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != static_cast<unsigned>(p.splits - 1)) return;
    __threadfence();
#pragma unroll
    for (int r = 0; r < kGemvTiles; ++r)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int e = 0; e < 2; ++e) val[r][h][e] = 0.f;
    // partial sums in a fixed split order; 8 splits of loads in flight at a time
    for (int s0 = 0; s0 < p.splits; s0 += 8) {
      float v[8][kGemvTiles][2][2];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float* ps = p.partial + (static_cast<size_t>(s0 + j) * p.rows_padded + rb * 32) * 8;
#pragma unroll
        for (int r = 0; r < kGemvTiles; ++r)
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int e = 0; e < 2; ++e)
              v[j][r][h][e] = (s0 + j < p.splits && col_ok(e)) ? __ldcg(ps + (r * 16 + h * 8 + g) * 8 + 2 * t + e) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int r = 0; r < kGemvTiles; ++r)
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int e = 0; e < 2; ++e) val[r][h][e] += v[j][r][h][e];
    }
    if (lane == 0) p.counters[rb] = 0u;
  }

  // ---- final epilogue: (tile r, box h) of this lane is weight row box_row0(h) + 8r + sigma(g)
  if constexpr (EPI == EPI_ARGMAX) {
    // per column m = 2t + e: best (value, row) over this lane's rows, then over g
    float best[2] = {-INFINITY, -INFINITY};
    int best_i[2] = {0x7FFFFFFF, 0x7FFFFFFF};
#pragma unroll
    for (int r = 0; r < kGemvTiles; ++r)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = (h ? rowB : rowA) + 8 * r + sg;
        if (row >= p.N) continue;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float v = val[r][h][e];
          if (v > best[e] || (v == best[e] && row < best_i[e])) {
            best[e] = v;
            best_i[e] = row;
          }
        }
      }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float ov = __shfl_xor_sync(0xffffffffu, best[e], o);
        const int oi = __shfl_xor_sync(0xffffffffu, best_i[e], o);
        if (ov > best[e] || (ov == best[e] && oi < best_i[e])) {
          best[e] = ov;
          best_i[e] = oi;
        }
      }
    }
    if (g == 0) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        if (col_ok(e) && best_i[e] != 0x7FFFFFFF)
          atomicMax(p.argmax_keys + 2 * t + e, argmax_key(best[e], best_i[e] + p.argmax_offset));
      }
    }
    return;
  } else {
    float scale_pc[kRows];
    if constexpr (WF == W_I8PC) {
#pragma unroll
      for (int q = 0; q < kRows; ++q)
        scale_pc[q] = static_cast<const float*>(set_of(q & 1) ? p.s1 : p.s0)[row_of(q >> 1, q & 1)];
    }
#pragma unroll
    for (int r = 0; r < kGemvTiles; ++r) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        if (!col_ok(e)) continue;
        const int m = 2 * t + e;
        float v_lo = val[r][0][e], v_hi = val[r][1][e];
        if constexpr (WF == W_I8PC) {
          v_lo *= scale_pc[2 * r];
          v_hi *= scale_pc[2 * r + 1];
        }
        if constexpr (EPI == EPI_SWIGLU) {
          const int n = rowA + 8 * r + sg;
          if (n < p.N) {
            const float gt = round_act<TA>(v_lo), up = round_act<TA>(v_hi);
            const float silu = gt / (1.0f + expf(-gt));
            store_act<TA>(p.y, static_cast<size_t>(m) * p.ldy + n, silu * up);
          }
        } else if constexpr (EPI == EPI_ROPE) {
          const int wph = p.head_dim / 32;
          const int head = rb / wph;
          const int i = 16 * (rb % wph) + 8 * r + sg;  // rotation pair index
          const int half = p.head_dim / 2;
          float a = round_act<TA>(v_lo), b = round_act<TA>(v_hi);
          void* out;
          int hh, nh;
          if (head < p.heads_q) {
            out = p.q_out;
            hh = head;
            nh = p.heads_q;
          } else if (head < p.heads_q + p.heads_kv) {
            out = p.k_out;
            hh = head - p.heads_q;
            nh = p.heads_kv;
          } else {
            out = p.v_out;
            hh = head - p.heads_q - p.heads_kv;
            nh = p.heads_kv;
          }
          if (head < p.heads_q + p.heads_kv) {
            const float angle = static_cast<float>(p.positions[m]) * p.inv_freq[i];
            float sn, cs;
            sincosf(angle, &sn, &cs);
            const float ra = a * cs - b * sn;
            const float rb2 = b * cs + a * sn;
            a = ra;
            b = rb2;
          }
          const int bi = m / p.seq_len, l = m % p.seq_len;
          const size_t obase = ((static_cast<size_t>(bi) * nh + hh) * p.seq_len + l) * p.head_dim;
          store_act<TA>(out, obase + i, a);
          store_act<TA>(out, obase + half + i, b);
        } else {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int row = (h ? rowB : rowA) + 8 * r + sg;
            if (row >= p.N) continue;
            const float v = h ? v_hi : v_lo;
            const size_t idx = static_cast<size_t>(m) * p.ldy + row;
            if constexpr (EPI == EPI_RESID) {
              const float res_v = load_act<TA>(p.residual, static_cast<size_t>(m) * p.ldr + row);
              store_act<TA>(p.y, idx, res_v + round_act<TA>(v));
            } else {
              store_act<TA>(p.y, idx, v);
            }
          }
        }
      }
    }
  }
}

// ------------------------------------------------------------------ host side

namespace {

int sm_count() {
  static int count = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || count <= 0)
      count = 148;
  });
  return count;
}

struct Plan {
  int tiles, rowblocks, groups, splits, k_group;
  size_t counter_bytes, partial_bytes;
  void* workspace;
  size_t workspace_bytes;
};

constexpr int kMaxGemvSplits = 32;

// Row blocks and groups of a request; the split count is chosen at launch from
// the kernel's occupancy. partial_bytes covers the largest split count allowed.
Plan make_plan(int epi, int N, int K, int group_k, bool allow_split) {
  Plan pl{};
  pl.tiles = 0;
  pl.rowblocks = epi == EPI_SWIGLU ? (N + 15) / 16 : (epi == EPI_ROPE ? N / 32 : (N + 31) / 32);
  pl.k_group = group_k;
  pl.groups = K / group_k;
  const int max_s = (allow_split && pl.rowblocks <= kMaxCounters) ? std::max(1, std::min(kMaxGemvSplits, pl.groups / 2)) : 1;
  pl.splits = max_s;
  pl.counter_bytes = kCounterBytes;
  pl.partial_bytes = max_s > 1 ? static_cast<size_t>(max_s) * pl.rowblocks * 32 * 8 * sizeof(float) : 0;
  return pl;
}

template <typename TA, int WF, int KC, int GC, int EPI, bool NORM, int MC>
int launch_gemv_mc(GemvParams& p, const Plan& plan, cudaStream_t stream) {
  using SG = StageGeom<Fmt<TA, WF>::kBits>;
  constexpr bool kAff = (WF == W_AFF4 || WF == W_AFF8);
  auto kernel = gemv_kernel<TA, WF, KC, GC, EPI, NORM, MC>;
  // activation segment: at most 8 KB of shared memory, whole stages and whole
  // super-groups (so a super-group's group sums are staged together)
  const int super_k = kAff ? (8 / MC) * p.group_size : SG::kStageK;
  const int unit = std::max(SG::kStageK, super_k);
  auto smem_for = [&](int splits) {
    const int max_kunit = (plan.groups + splits - 1) / splits * plan.k_group;
    int seg = (8192 / (p.M * static_cast<int>(sizeof(TA)))) / unit * unit;
    seg = std::max(seg, unit);
    p.x_seg = std::min(seg, ((max_kunit + unit - 1) / unit) * unit);
    const size_t xg_bytes = static_cast<size_t>(p.M) * (p.x_seg / plan.k_group + 1) * sizeof(float);
    return 2048 + static_cast<size_t>(kGemvWarps) * SG::kStages * SG::kStageBytes +
           static_cast<size_t>(p.M) * (p.x_seg + 8) * sizeof(TA) + xg_bytes;
  };
  size_t smem = smem_for(1);
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return fail(SB_ECUDA, "gemv: shared memory opt-in failed");
  // splits: fill the resident CTA slots in one wave (no tail wave)
  int splits = 1;
  const int ctas_per_split = (plan.rowblocks + kGemvWarps - 1) / kGemvWarps;
  if (plan.splits > 1 && plan.workspace != nullptr &&
      plan.workspace_bytes >= plan.counter_bytes + plan.partial_bytes) {
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kGemvWarps * 32, smem) != cudaSuccess || occ < 1)
      occ = 1;
    const int slots = sm_count() * occ;
    splits = std::max(1, std::min(plan.splits, slots / ctas_per_split));
  }
  smem = smem_for(splits);
  p.splits = splits;
  p.groups_total = plan.groups;
  p.rows_padded = plan.rowblocks * 32;
  if (splits > 1) {
    p.counters = static_cast<unsigned*>(plan.workspace);
    p.partial = reinterpret_cast<float*>(static_cast<uint8_t*>(plan.workspace) + plan.counter_bytes);
  }
  dim3 grid(ctas_per_split, splits);
  return launch("gemv", kernel, grid, dim3(kGemvWarps * 32), smem, stream, p);
}

template <typename TA, int WF, int KC, int GC, int EPI, bool NORM>
int launch_gemv(GemvParams& p, const Plan& pl, cudaStream_t stream) {
  if (p.M == 1) return launch_gemv_mc<TA, WF, KC, GC, EPI, NORM, 1>(p, pl, stream);
  if (p.M <= 4) return launch_gemv_mc<TA, WF, KC, GC, EPI, NORM, 4>(p, pl, stream);
  return launch_gemv_mc<TA, WF, KC, GC, EPI, NORM, 8>(p, pl, stream);
}

template <typename TA, int WF, int EPI, bool NORM>
int dispatch_group(GemvParams& p, const Plan& pl, cudaStream_t stream) {
  if constexpr (WF == W_AFF4 || WF == W_AFF8) {
    switch (p.group_size) {
      case 32:
        return launch_gemv<TA, WF, 32, 1, EPI, NORM>(p, pl, stream);
      case 64:
        return launch_gemv<TA, WF, 64, 1, EPI, NORM>(p, pl, stream);
      case 128:
        return launch_gemv<TA, WF, 64, 2, EPI, NORM>(p, pl, stream);
      default:
        return fail(SB_EUNSUPPORTED, "group_size must be 32, 64 or 128");
    }
  } else {
    return launch_gemv<TA, WF, 64, 1, EPI, NORM>(p, pl, stream);
  }
}

template <int EPI, bool NORM>
int dispatch_fmt(int wf, int x_dtype, GemvParams& p, const Plan& pl, cudaStream_t stream) {
  constexpr bool kAffineEpi = EPI != EPI_ARGMAX;
  constexpr bool kI8Epi = EPI == EPI_STORE || EPI == EPI_RESID || EPI == EPI_ROPE;
  constexpr bool kBf16Epi = EPI == EPI_STORE || EPI == EPI_ARGMAX;
  if (x_dtype == SB_DTYPE_BF16) {
    if constexpr (kAffineEpi) {
      if (wf == W_AFF4) return dispatch_group<__nv_bfloat16, W_AFF4, EPI, NORM>(p, pl, stream);
      if (wf == W_AFF8) return dispatch_group<__nv_bfloat16, W_AFF8, EPI, NORM>(p, pl, stream);
    }
    if constexpr (kI8Epi) {
      if (wf == W_I8PC) return dispatch_group<__nv_bfloat16, W_I8PC, EPI, NORM>(p, pl, stream);
    }
    if constexpr (kBf16Epi) {
      if (wf == W_BF16) return dispatch_group<__nv_bfloat16, W_BF16, EPI, NORM>(p, pl, stream);
    }
  } else if (x_dtype == SB_DTYPE_F16) {
    if constexpr (EPI == EPI_STORE || EPI == EPI_ROPE) {
      if (wf == W_AFF4) return dispatch_group<__half, W_AFF4, EPI, NORM>(p, pl, stream);
      if (wf == W_AFF8) return dispatch_group<__half, W_AFF8, EPI, NORM>(p, pl, stream);
      if (wf == W_I8PC) return dispatch_group<__half, W_I8PC, EPI, NORM>(p, pl, stream);
    }
  }
  return fail(SB_EUNSUPPORTED, "unsupported activation dtype / weight format / epilogue combination");
}

}  // namespace

static int group_k_of(const LinearRequest& r) {
  if (r.wf == W_AFF4 || r.wf == W_AFF8) return r.group_size;
  return 64;
}

size_t linear_workspace_size(int epi, int N, int K, int group_k) {
  if (group_k <= 0 || K % group_k) return 0;
  const Plan pl = make_plan(epi, N, K, group_k, true);
  return pl.counter_bytes + pl.partial_bytes;
}

int run_linear(const LinearRequest& r, cudaStream_t stream) {
  SB_REQUIRE(r.M >= 1 && r.M <= 8, "weight-streaming linear supports 1..8 activation rows per call");
  SB_REQUIRE(r.N > 0 && r.K > 0, "N and K must be positive");
  const int gk = group_k_of(r);
  SB_REQUIRE(r.K % gk == 0, "K must be a multiple of the group size (64 for per-channel/bf16 weights)");
  SB_REQUIRE(r.ldx % 8 == 0 && (reinterpret_cast<uintptr_t>(r.x) & 15) == 0,
             "activations must be 16-byte aligned with a row stride that is a multiple of 8");
  SB_REQUIRE((reinterpret_cast<uintptr_t>(r.w0) & 15) == 0 && (r.w1 == nullptr || (reinterpret_cast<uintptr_t>(r.w1) & 15) == 0),
             "weights must be 16-byte aligned");
  SB_REQUIRE((static_cast<int64_t>(r.K) * (r.wf == W_AFF4 ? 4 : (r.wf == W_BF16 ? 16 : 8)) / 8) % 16 == 0,
             "weight rows must be a multiple of 16 bytes");
  if (r.epi == EPI_ROPE) {
    SB_REQUIRE(r.head_dim % 16 == 0 && r.head_dim / 2 <= kMaxRopeHalf, "head_dim must be a multiple of 16, <= 256");
    SB_REQUIRE(r.rope_dims == r.head_dim, "the fused RoPE epilogue rotates the full head_dim");
    SB_REQUIRE(r.N == (r.heads_q + 2 * r.heads_kv) * r.head_dim, "QKV rows must equal (Hq + 2*Hkv) * head_dim");
  }
  if (r.epi == EPI_SWIGLU) SB_REQUIRE(r.N % 8 == 0, "SwiGLU width must be a multiple of 8");

  Plan pl = make_plan(r.epi, r.N, r.K, gk, true);
  pl.workspace = r.workspace;
  pl.workspace_bytes = r.workspace_bytes;

  GemvParams p{};
  p.x = r.x;
  p.ldx = r.ldx;
  p.M = r.M;
  p.N = r.N;
  p.K = r.K;
  p.w0 = r.w0;
  p.s0 = r.s0;
  p.b0 = r.b0;
  p.w1 = r.w1 ? r.w1 : r.w0;
  p.s1 = r.s1 ? r.s1 : r.s0;
  p.b1 = r.b1 ? r.b1 : r.b0;
  p.group_size = r.group_size;
  p.groups_total = pl.groups;
  p.rows_padded = pl.rowblocks * 32;
  {
    const int bits = r.wf == W_AFF4 ? 4 : (r.wf == W_BF16 ? 16 : 8);
    const uint64_t row_bytes = static_cast<uint64_t>(r.K) * bits / 8;
    if (int st = make_tmap_rows(&p.tmap0, r.w0, static_cast<uint64_t>(r.N), row_bytes, 16)) return st;
    if (int st = make_tmap_rows(&p.tmap1, r.w1 ? r.w1 : r.w0, static_cast<uint64_t>(r.N), row_bytes, 16)) return st;
  }
  if (r.workspace != nullptr && r.workspace_bytes >= kCounterBytes)
    p.status = static_cast<unsigned*>(r.workspace) + kStatusWord;
  p.norm_w = r.norm_w;
  p.eps = r.eps;
  p.y = r.y;
  p.ldy = r.ldy;
  p.residual = r.residual;
  p.ldr = r.ldr;
  p.positions = r.positions;
  p.heads_q = r.heads_q;
  p.heads_kv = r.heads_kv;
  p.head_dim = r.head_dim;
  p.seq_len = r.seq_len > 0 ? r.seq_len : 1;
  p.q_out = r.q_out;
  p.k_out = r.k_out;
  p.v_out = r.v_out;
  p.argmax_keys = r.argmax_keys;
  p.argmax_offset = r.argmax_offset;
  p.early_prefetch = r.weights_constant ? 1 : 0;
  if (r.epi == EPI_ROPE) {
    for (int i = 0; i < r.rope_dims / 2; ++i)
      p.inv_freq[i] = static_cast<float>(std::pow(static_cast<double>(r.rope_base), -2.0 * i / r.rope_dims));
  }

  switch (r.epi) {
    case EPI_STORE:
      return r.norm ? dispatch_fmt<EPI_STORE, true>(r.wf, r.x_dtype, p, pl, stream)
                    : dispatch_fmt<EPI_STORE, false>(r.wf, r.x_dtype, p, pl, stream);
    case EPI_RESID:
      return dispatch_fmt<EPI_RESID, false>(r.wf, r.x_dtype, p, pl, stream);
    case EPI_SWIGLU:
      return r.norm ? dispatch_fmt<EPI_SWIGLU, true>(r.wf, r.x_dtype, p, pl, stream)
                    : dispatch_fmt<EPI_SWIGLU, false>(r.wf, r.x_dtype, p, pl, stream);
    case EPI_ROPE:
      return r.norm ? dispatch_fmt<EPI_ROPE, true>(r.wf, r.x_dtype, p, pl, stream)
                    : dispatch_fmt<EPI_ROPE, false>(r.wf, r.x_dtype, p, pl, stream);
    case EPI_ARGMAX:
      return r.norm ? dispatch_fmt<EPI_ARGMAX, true>(r.wf, r.x_dtype, p, pl, stream)
                    : dispatch_fmt<EPI_ARGMAX, false>(r.wf, r.x_dtype, p, pl, stream);
  }
  return fail(SB_EINVAL, "unknown epilogue");
}

}  // namespace sb
