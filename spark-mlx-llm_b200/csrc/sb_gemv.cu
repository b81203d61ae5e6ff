// Weight-streaming linear kernels (M <= 8) and their C-ABI entry points.
// The design notes are in sb_gemv.cuh.
#include <algorithm>
#include <cmath>
#include <mutex>
#include <type_traits>
#include <vector>

#include "sb_gemv.cuh"

namespace sb {

constexpr int cmin(int a, int b) { return a < b ? a : b; }

// Compile-time geometry of one (weight format, group size, column layout).
//
// A stage is 128 weight bytes of each of a warp's 32 rows. The MMA's 8 output
// columns carry (activation row m = n % MC, group slot = n / MC); a stage holds
// kU "super-groups" of kSlots groups each. Within a super-group the 8 operand
// streams of a k16 step (lane quad t = 0..3, half h = 0/1 -> stream 2t+h) are
// pieces of kPB bytes: stream s reads group slot s*kSlots/8, piece
// s % (8/kSlots), so lane quad t always reads the contiguous bytes
// [t*kLaneB, (t+1)*kLaneB) of the super-group, and the B operand of column n is
// non-zero only on the lanes whose stream belongs to n's slot.
template <int WF, int G, int MC>
struct Geo {
  static constexpr int kBits = WF == W_AFF4 ? 4 : (WF == W_BF16 ? 16 : 8);
  static constexpr bool kAffine = WF == W_AFF4 || WF == W_AFF8;
  // fp16 operands with per-group power-of-two activation scaling (all but bf16 weights)
  static constexpr bool kScaled = WF != W_BF16;
  static constexpr int kGroupK = kAffine ? G : 64;  // per-channel/bf16: 64-wide pseudo-groups
  static constexpr int kGB = kGroupK * kBits / 8;   // weight bytes of one group of one row
  static constexpr int kStageK = 128 * 8 / kBits;
  static constexpr int kGPS = 128 / kGB;  // groups per stage
  static constexpr int kSlots = kScaled ? cmin(8 / MC, kGPS) : 1;
  static constexpr int kU = kGPS / kSlots;
  static constexpr int kSGB = kSlots * kGB;  // bytes per super-group per row
  static constexpr int kPB = kSGB / 8;       // bytes per stream piece
  static constexpr int kLaneB = 2 * kPB;     // bytes per lane quad per row per super-group
  static constexpr int kPieceK = kPB * 8 / kBits;
  static constexpr int kSteps = kPieceK / 2;  // k16 MMA steps per super-group
  static constexpr int kQuads = kSteps / 4;   // 4 steps share one 16-byte activation load
  static constexpr int kWQ = kBits / 4;       // weight words per stream per quad
  static constexpr int kWords = kLaneB / 4;   // weight words per lane per row per super-group
  static constexpr int kYG = kGroupK * 2 + 16;  // staged activation bytes per group (+16: bank rotation)
  static_assert(kSteps % 4 == 0 && kLaneB >= 8, "geometry");
};

// Operand encoding of the codes (A = offset + code, exact) and of the staged
// activations, per k16 step j of a quad (4-bit: steps 0 and 2 carry the low
// nibble of each byte, steps 1 and 3 the high nibble):
//   4-bit, bf16 activations: low nibble  bf16 128+q   (0x4300 | q)      x staged as bf16
//                            high nibble fp16 64+q    (0x5400 | q<<4)   x staged as fp16
//   4-bit, fp16 activations: low nibble  fp16 1024+q  (0x6400 | q), high nibble as above
//   8-bit                  : fp16 1024+u  (0x64 | byte; signed int8: u = code+128, offset 1152)
//   bf16 weights           : bf16 as stored
// acc = sum(code * xs) + sum(offset_k * xs_k); the second sum is staged per group.
template <typename TA, int WF>
struct Enc {
  static constexpr bool kMixed = WF == W_AFF4 && !std::is_same<TA, __half>::value;
  __host__ __device__ static constexpr bool half_step(int j) {
    return WF == W_BF16 ? false : (kMixed ? (j & 1) != 0 : true);
  }
  static constexpr uint32_t kLowMagic = kMixed ? 0x43004300u : 0x64006400u;
  static constexpr float kOffEven = WF == W_AFF4 ? (kMixed ? 128.0f : 1024.0f) : (WF == W_I8PC ? 1152.0f : 1024.0f);
  static constexpr float kOffOdd = WF == W_AFF4 ? 64.0f : kOffEven;
};

// Staged-activation layout inside one group: the 8-value vector at k (a
// multiple of 8) holds four operand pairs. When a lane's two streams are
// adjacent pieces of one group (kSlots <= 4), the pairs of the two pieces are
// interleaved (lo j, hi j, lo j+1, hi j+1, ...) so one 16-byte load yields the
// B operands of two k16 steps in register order; otherwise vectors are stored
// in place.
template <typename C>
__device__ __forceinline__ int y_offset(int k) {
  if constexpr (C::kSlots <= 4) {
    const int piece = k / C::kPieceK, qd = (k % C::kPieceK) / 8;
    return (piece >> 1) * C::kPieceK * 4 + qd * 32 + (piece & 1) * 4;
  } else {
    return k * 2;
  }
}
template <typename C>
__device__ __forceinline__ void store_pairs(uint8_t* dst, uint4 v) {
  if constexpr (C::kSlots <= 4) {
    *reinterpret_cast<uint32_t*>(dst) = v.x;
    *reinterpret_cast<uint32_t*>(dst + 8) = v.y;
    *reinterpret_cast<uint32_t*>(dst + 16) = v.z;
    *reinterpret_cast<uint32_t*>(dst + 24) = v.w;
  } else {
    *reinterpret_cast<uint4*>(dst) = v;
  }
}

// Row relabeling inside each 8-row half of a box so that the lanes' reads of
// the 128-byte-swizzled rows fall into distinct banks for their access width.
template <int kLaneB>
__device__ __forceinline__ int sigma_row(int g) {
  if constexpr (kLaneB >= 32) return g;                           // 2 x 16 B per row
  else if constexpr (kLaneB == 16) return ((g & 1) << 2) | (g >> 1);  // 16 B per row
  else return ((g & 3) << 1) | (g >> 2);                          // 8 B per row
}

// Four k16 steps' worth of one stream's weight words -> operand pairs
//   4-bit: word -> pairs (k0,k4) (k1,k5) (k2,k6) (k3,k7)
//   8-bit: 2 words -> pairs (k0,k1) (k2,k3) per word
//   bf16 : 4 words -> pairs as stored
template <typename TA, int WF>
__device__ __forceinline__ void dequant_quad(const uint32_t* w, uint32_t (&p)[4]) {
  if constexpr (WF == W_AFF4) {
    constexpr uint32_t kLow = Enc<TA, WF>::kLowMagic;
    const uint32_t s = w[0] >> 8;
    p[0] = lop_and_or(w[0], 0x000F000Fu, kLow);
    p[1] = lop_and_or(w[0], 0x00F000F0u, 0x54005400u);
    p[2] = lop_and_or(s, 0x000F000Fu, kLow);
    p[3] = lop_and_or(s, 0x00F000F0u, 0x54005400u);
  } else if constexpr (WF == W_AFF8 || WF == W_I8PC) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint32_t u = (WF == W_I8PC) ? (w[i] ^ 0x80808080u) : w[i];
      p[2 * i] = prmt(u, 0x64646464u, 0x4140u);
      p[2 * i + 1] = prmt(u, 0x64646464u, 0x4342u);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = w[i];
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
// 16-bit activation-typed value (bf16 or fp16 bits) -> float
template <typename TA>
__device__ __forceinline__ float bits_to_float(uint32_t b16) {
  if constexpr (std::is_same<TA, __half>::value) return __half2float(__ushort_as_half(static_cast<unsigned short>(b16)));
  else return __uint_as_float(b16 << 16);
}

// ---- warp row blocks
// A warp owns 32 weight rows, fetched per stage as two TMA boxes (A and B) of
// 16 rows x 128 bytes. MMA rows 0-7 of tile r come from box A rows 8r + sigma(g),
// MMA rows 8-15 from box B rows 8r + sigma(g).
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

constexpr int kStageBytes = 32 * 128;  // two 16-row boxes

template <typename TA, int WF, int G, int EPI, bool NORM, int MC>
__global__ void __launch_bounds__(kGemvMaxWarps * 32, 1) gemv_kernel(const __grid_constant__ GemvParams p) {
  using C = Geo<WF, G, MC>;
  constexpr int kVG = C::kGroupK / 8;  // 8-value activation vectors per group
  const int kNT = static_cast<int>(blockDim.x);  // 32 x (4 row blocks x kSub K sub-parts)
  const int nwarps = kNT >> 5;

  extern __shared__ uint8_t smem_dyn[];
  __shared__ float s_rms[8];
  __shared__ float s_part[kGemvMaxWarps][8];
  __shared__ unsigned long long s_keys[8];
  __shared__ unsigned s_kvmax[2][8];  // fused cache append: |K/V| max per (head in group, m)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2;
  const int t = lane & 3;
  const int sg = sigma_row<C::kLaneB>(g);
  const int part = blockIdx.x;  // K part = rank in the cluster
  const int nparts = gridDim.x;
  const int rowblocks = warp_blocks<EPI>(p);
  const int rbi = warp % kGemvWarps;  // row block of this warp inside the CTA
  const int sub = warp / kGemvWarps;  // K sub-part of this warp inside the CTA
  const int nsub = nwarps / kGemvWarps;
  const int rb = blockIdx.y * kGemvWarps + rbi;
  const bool active = rb < rowblocks;
  const int rbc = min(rb, rowblocks - 1);
  const int M = p.M;
  const int gpr = p.K / C::kGroupK;  // groups per row (of this K chunk)
  const int cparts = p.chunk_parts;  // CTAs per K chunk (chunk-major cluster ranks)
  const int zc = part / cparts;      // K chunk of this CTA
  const int cq = part - zc * cparts; // part inside the chunk
  const TA* xz = static_cast<const TA*>(p.x) + static_cast<size_t>(zc) * p.K;

  // stages [st0, st1) of this CTA (of its chunk)
  const int st0 = static_cast<int>((static_cast<long long>(p.stages_total) * cq) / cparts);
  const int st1 = static_cast<int>((static_cast<long long>(p.stages_total) * (cq + 1)) / cparts);
  const int nst = st1 - st0;

  // ---- shared memory: barriers + zero block, per-warp rings, staged x, group meta, reduction buffer
  // 1 KB-aligned start (pointer arithmetic keeps the shared address space known to the compiler)
  uint8_t* base = smem_dyn + ((1024u - (smem_u32(smem_dyn) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base) + warp * kGemvMaxRing;
  const uint8_t* zero_blk = base + 768;
  uint64_t* scbar = reinterpret_cast<uint64_t*>(base + 512);  // scale/bias TMA barrier
  uint8_t* ring = base + 1024 + warp * p.ring * kStageBytes;
  // staged scales and biases (affine): [warp][row h*16 + i][sc_ld] of the current segment
  uint16_t* scs = reinterpret_cast<uint16_t*>(base + 1024 + nwarps * p.ring * kStageBytes);
  uint16_t* scb = scs + kGemvWarps * 32 * p.sc_ld;
  uint8_t* ys = reinterpret_cast<uint8_t*>(scb + kGemvWarps * 32 * p.sc_ld);
  float4* meta = reinterpret_cast<float4*>(ys + M * p.y_ld);
  float* red = reinterpret_cast<float*>(meta + M * p.meta_ld);

  const int rowA = box_row0<EPI>(p, rbc, 0), rowB = box_row0<EPI>(p, rbc, 1);
  auto set_of = [&](int h) { return (EPI == EPI_SWIGLU) ? h : 0; };
  auto issue_stage = [&](int slot, int st) {
    uint8_t* dst = ring + slot * kStageBytes;
    mbar_arrive_expect_tx(bars + slot, kStageBytes);
    const int x = zc * p.chunk_wbytes + (st0 + st) * 128;
    tma_load_2d(dst, &p.tmap0, x, rowA, bars + slot);
    tma_load_2d(dst + 16 * 128, &p.tmap1, x, rowB, bars + slot);
  };

  // Scales and biases of the CTA's 4 x 32 rows for the groups of stages
  // [sb, sb + seg_stages) into shared memory: by TMA (boxes of 16 rows from the
  // group G0 rounded down to 8; sc_off = G0 % 8) when the tables allow it, else
  // by 4-byte asynchronous copies or plain loads, with the columns past the
  // range zeroed. Completion: scbar (TMA) or cp.async.wait_all, both at the
  // end of the segment's activation staging.
  int sc_off = 0;
  auto stage_scales = [&](int sb) {
    if constexpr (C::kAffine) {
      const int G0 = (st0 + sb) * C::kGPS;
      if (p.sc_tma) {
        const int Ga = zc * gpr + G0;  // group in the table row
        sc_off = Ga & 7;
        if (threadIdx.x == 0) {
          fence_proxy_async_smem();
          mbar_arrive_expect_tx(scbar, static_cast<uint32_t>(2 * kGemvWarps * 32 * p.sc_ld * 2));
          for (int w = 0; w < kGemvWarps; ++w) {
            const int rbw = min(static_cast<int>(blockIdx.y) * kGemvWarps + w, rowblocks - 1);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int row0 = box_row0<EPI>(p, rbw, h);
              const int o = (w * 32 + h * 16) * p.sc_ld;
              tma_load_2d(scs + o, set_of(h) ? &p.smap1 : &p.smap0, Ga - sc_off, row0, scbar);
              tma_load_2d(scb + o, set_of(h) ? &p.bmap1 : &p.bmap0, Ga - sc_off, row0, scbar);
            }
          }
        }
        return;
      }
      const int G1 = min(min(st0 + sb + p.seg_stages, st1) * C::kGPS, gpr);
      const int ng = max(G1 - G0, 0);
      const bool async = (C::kGPS % 2 == 0) && p.pair_scales;
      const int per_row = async ? ng / 2 : ng;  // copies per row and array
      const int total = 2 * kGemvWarps * 32 * per_row;
      for (int idx = threadIdx.x; idx < total; idx += kNT) {
        const int which = idx / (kGemvWarps * 32 * per_row);  // 0 scales, 1 biases
        const int rem = idx - which * (kGemvWarps * 32 * per_row);
        const int wr = rem / per_row, c = rem - (rem / per_row) * per_row;
        const int w = wr >> 5, row = wr & 31, h = row >> 4;
        const int rbw = min(static_cast<int>(blockIdx.y) * kGemvWarps + w, rowblocks - 1);
        const int grow = min(box_row0<EPI>(p, rbw, h) + (row & 15), p.N - 1);
        const uint16_t* src = static_cast<const uint16_t*>(which ? (set_of(h) ? p.b1 : p.b0) : (set_of(h) ? p.s1 : p.s0)) +
                              static_cast<size_t>(grow) * p.sc_stride + zc * gpr + G0;
        uint16_t* dst = (which ? scb : scs) + wr * p.sc_ld;
        if (async) cp_async4(dst + 2 * c, src + 2 * c);
        else dst[c] = src[c];
      }
      // zero the padding columns [ng, sc_ld) of every row
      const int pad = p.sc_ld - ng;
      for (int idx = threadIdx.x; idx < 2 * kGemvWarps * 32 * pad; idx += kNT) {
        const int which = idx / (kGemvWarps * 32 * pad);
        const int rem = idx - which * (kGemvWarps * 32 * pad);
        const int wr = rem / pad, c = ng + rem - (rem / pad) * pad;
        (which ? scb : scs)[wr * p.sc_ld + c] = 0;
      }
      cp_async_commit();
    }
  };
  int sc_phase = 0;
  auto wait_scales = [&]() {
    if constexpr (C::kAffine) {
      if (p.sc_tma) {
        if (!mbar_wait_bounded(scbar, static_cast<uint32_t>(sc_phase))) {
          if (p.status && threadIdx.x == 0) atomicOr(p.status, kStatusTimeout);
        }
        sc_phase ^= 1;
      } else {
        cp_async_wait_all();
      }
    }
  };

  // the weight (and scale/bias) tensor maps: start the descriptor fetches
  // before the barriers are set up (a first copy otherwise waits for them)
  if (threadIdx.x == 0) {
    prefetch_tmap(&p.tmap0);
    prefetch_tmap(&p.tmap1);
    if (C::kAffine && p.sc_tma) {
      prefetch_tmap(&p.smap0);
      prefetch_tmap(&p.bmap0);
      prefetch_tmap(&p.smap1);
      prefetch_tmap(&p.bmap1);
    }
  }
  if (active && lane == 0) {
    for (int i = 0; i < p.ring; ++i) mbar_init(bars + i, 1);
    mbar_fence_init();
  }
  if (C::kAffine && threadIdx.x == 0) {
    mbar_init(scbar, 1);
    mbar_fence_init();
  }
  __syncwarp();
  // ---- start streaming weights; with constant weights this may overlap the
  // tail of the previous kernel in the stream
  if (!p.early_prefetch) grid_dependency_wait();
  // this warp's stages [ws0, ws1) of the CTA's range
  const int ws0 = nst * sub / nsub, ws1 = nst * (sub + 1) / nsub;
  if (active && lane == 0) {
    for (int i = 0; i < p.ring && ws0 + i < ws1; ++i) issue_stage(i, ws0 + i);
  }
  if (p.early_prefetch && nst > 0) stage_scales(0);
  if (threadIdx.x < 16) reinterpret_cast<uint4*>(base + 768)[threadIdx.x] = make_uint4(0u, 0u, 0u, 0u);
  if (threadIdx.x < 8) s_keys[threadIdx.x] = 0ull;
  if (threadIdx.x < 16) s_kvmax[threadIdx.x >> 3][threadIdx.x & 7] = 0u;

  // ---- activations depend on the previous kernel from here on
  grid_dependency_wait();
  // the first two staging passes of the first segment load their activations
  // (and norm weights) now, together with the norm statistics' loads, so the
  // prologue costs one memory round trip
  uint4 pre_x[2], pre_w[2];
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    pre_x[it] = make_uint4(0u, 0u, 0u, 0u);
    pre_w[it] = make_uint4(0u, 0u, 0u, 0u);
    const int k0 = st0 * C::kStageK;
    const int k1 = min(min(st0 + p.seg_stages, st1) * C::kStageK, p.K);
    const int nvec = max(k1 - k0, 0) / 8;
    const int idx = it * kNT + static_cast<int>(threadIdx.x);
    if (idx < M * nvec) {
      const int m = idx / nvec, k = k0 + 8 * (idx - m * nvec);
      pre_x[it] = *reinterpret_cast<const uint4*>(xz + static_cast<size_t>(m) * p.ldx + k);
      if constexpr (NORM) pre_w[it] = *reinterpret_cast<const uint4*>(static_cast<const TA*>(p.norm_w) + k);
    }
  }
  if constexpr (NORM) {
    // full-row sum of squares per activation row (fixed reduction order); a
    // thread's loads are issued together so the pass costs one round trip
    constexpr int kU4 = 4;
    const int nv = p.K / 8;  // 8-value vectors per row
    float ss[MC];
#pragma unroll
    for (int m = 0; m < MC; ++m) ss[m] = 0.f;
    for (int i0 = threadIdx.x; i0 < M * nv; i0 += kNT * kU4) {
      uint4 v[kU4];
#pragma unroll
      for (int u = 0; u < kU4; ++u) {
        const int i = i0 + u * kNT;
        const int m = i / nv;
        v[u] = i < M * nv ? *reinterpret_cast<const uint4*>(static_cast<const TA*>(p.x) + static_cast<size_t>(m) * p.ldx +
                                                             8 * (i - m * nv))
                          : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < kU4; ++u) {
        const int m = (i0 + u * kNT) / nv;
        const TA* e = reinterpret_cast<const TA*>(&v[u]);
        float a2 = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) a2 = fmaf(to_float(e[i]), to_float(e[i]), a2);
#pragma unroll
        for (int mm = 0; mm < MC; ++mm)
          if (mm == m) ss[mm] += a2;
      }
    }
#pragma unroll
    for (int m = 0; m < MC; ++m) {
      if (m < M) {
        const float w = warp_sum(ss[m]);
        if (lane == 0) s_part[warp][m] = w;
      }
    }
    __syncthreads();
    if (threadIdx.x < M) {
      float t2 = 0.f;
#pragma unroll
      for (int w = 0; w < kGemvMaxWarps; ++w)
        if (w < nwarps) t2 += s_part[w][threadIdx.x];
      s_rms[threadIdx.x] = 1.0f / sqrtf(t2 / static_cast<float>(p.K) + p.eps);
    }
  }

  // ---- activation staging of stages [sb, sb + seg_stages) (all threads):
  // xs = x * 2^e per group in the operand type of its k (exact), laid out in
  // the operand pair order; meta = {2^-e, sum(offset_k * xs_k), sum(x)} per group.
  auto stage_x = [&](int sb) {
    if (sb > 0 || !p.early_prefetch) stage_scales(sb);
    const int k0 = (st0 + sb) * C::kStageK;
    const int k1 = min(min(st0 + sb + p.seg_stages, st1) * C::kStageK, p.K);
    const int nvec = max(k1 - k0, 0) / 8;
    const int total = M * nvec;
    for (int b0 = 0; b0 < total; b0 += kNT) {
      const int idx = b0 + threadIdx.x;
      const bool ok = idx < total;
      const int m = ok ? idx / nvec : 0;
      const int v = ok ? idx - m * nvec : 0;
      const int k = k0 + 8 * v;
      float f[8];
      if (ok) {
        const bool pre = sb == 0 && b0 < 2 * kNT;
        const uint4 xv = pre ? (b0 == 0 ? pre_x[0] : pre_x[1])
                             : *reinterpret_cast<const uint4*>(xz + static_cast<size_t>(m) * p.ldx + k);
        const TA* xe = reinterpret_cast<const TA*>(&xv);
        if constexpr (NORM) {
          const uint4 wv = pre ? (b0 == 0 ? pre_w[0] : pre_w[1])
                               : *reinterpret_cast<const uint4*>(static_cast<const TA*>(p.norm_w) + k);
          const TA* we = reinterpret_cast<const TA*>(&wv);
          const float r = s_rms[m];
#pragma unroll
          for (int i = 0; i < 8; ++i) f[i] = round_act<TA>(to_float(xe[i]) * r * to_float(we[i]));
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) f[i] = to_float(xe[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = 0.f;
      }
      const int grp = (8 * v) / C::kGroupK;  // group inside the segment
      uint8_t* dst = ys + m * p.y_ld + grp * C::kYG + y_offset<C>((8 * v) % C::kGroupK);
      if constexpr (C::kScaled) {
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[i]));
#pragma unroll
        for (int o = 1; o < kVG; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        // power of two putting the group's largest |x| into [2^14, 2^15)
        const int ex = static_cast<int>((__float_as_uint(amax) >> 23) & 0xFFu);
        const int e = max(-126, min(126, 141 - ex));
        const float sc = __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
        uint16_t hb[8];
        float osum = 0.f, xsum = 0.f;  // sum(offset_k * xs_k), sum(x)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float ys = f[i] * sc;
          float yv;
          if (Enc<TA, WF>::kMixed && (i & 1) == 0) {
            const __nv_bfloat16 b = __float2bfloat16_rn(ys);
            hb[i] = __bfloat16_as_ushort(b);
            yv = __bfloat162float(b);
          } else {
            const __half h = __float2half_rn(ys);
            hb[i] = __half_as_ushort(h);
            yv = __half2float(h);
          }
          osum = fmaf((i & 1) ? Enc<TA, WF>::kOffOdd : Enc<TA, WF>::kOffEven, yv, osum);
          xsum += f[i];
        }
#pragma unroll
        for (int o = 1; o < kVG; o <<= 1) {
          osum += __shfl_xor_sync(0xffffffffu, osum, o);
          xsum += __shfl_xor_sync(0xffffffffu, xsum, o);
        }
        uint4 out;
        if constexpr (WF == W_AFF4) {
          // pair order of the 4-bit operand: (k0,k4) (k1,k5) (k2,k6) (k3,k7)
          out.x = static_cast<uint32_t>(hb[0]) | (static_cast<uint32_t>(hb[4]) << 16);
          out.y = static_cast<uint32_t>(hb[1]) | (static_cast<uint32_t>(hb[5]) << 16);
          out.z = static_cast<uint32_t>(hb[2]) | (static_cast<uint32_t>(hb[6]) << 16);
          out.w = static_cast<uint32_t>(hb[3]) | (static_cast<uint32_t>(hb[7]) << 16);
        } else {
          out = *reinterpret_cast<const uint4*>(hb);
        }
        if (ok) {
          store_pairs<C>(dst, out);
          if ((v % kVG) == 0) {
            const float inv = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);
            meta[m * p.meta_ld + grp] = make_float4(inv, osum, xsum, 0.f);
          }
        }
      } else {
        if (ok) {
          __nv_bfloat16 hb[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) hb[i] = __float2bfloat16_rn(f[i]);
          store_pairs<C>(dst, *reinterpret_cast<const uint4*>(hb));
        }
      }
    }
    wait_scales();
  };

  // ---- per-lane operand geometry
  const int bm = g % MC;      // activation row of this lane's B column
  const int bslot = g / MC;   // group slot of this lane's B column
  const bool col_live = bm < M;
  constexpr bool kPaired = C::kSlots <= 4;  // a lane's two streams are adjacent pieces of one group
  constexpr int kP8 = 8 / C::kSlots;        // pieces per group
  const int slot_lo = (2 * t) * C::kSlots / 8, slot_hi = (2 * t + 1) * C::kSlots / 8;
  const bool act_lo = col_live && bslot == slot_lo;
  const bool act_hi = col_live && bslot == slot_hi;
  // staged-activation byte offset of the lane's streams inside their group
  const int ypo_lo = kPaired ? (((2 * t) % kP8) >> 1) * C::kPieceK * 4 : 0;
  // this lane's bytes of row 8r+sg of a box, per super-group u and 16-byte load i
  constexpr int kLoads = C::kLaneB >= 16 ? C::kLaneB / 16 : 1;
  int aoff[C::kU][kLoads];
#pragma unroll
  for (int u = 0; u < C::kU; ++u)
#pragma unroll
    for (int i = 0; i < kLoads; ++i) {
      const int byte = u * C::kSGB + t * C::kLaneB + 16 * i;
      aoff[u][i] = sg * 128 + ((((byte >> 4) ^ sg) << 4) | (byte & 15));
    }

  // scale/bias of the lane's rows for the groups of its two accumulator columns
  const int ss0 = (MC == 1) ? 2 * t : (2 * t) / MC;  // slot of column 2t
  constexpr bool kPairCols = (MC == 1) && (C::kSlots >= 2);  // columns 2t, 2t+1 = two groups
  // two accumulator sets (even / odd k16 steps) halve the MMA dependency chains
  float cacc[2][2][4];
  float res[2][2][2];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      cacc[0][r][e] = 0.f;
      cacc[1][r][e] = 0.f;
      res[r][e >> 1][e & 1] = 0.f;
    }

  bool failed = false;
  int done = ws0;  // stages consumed by this warp (the next one to wait for)
  // The first activation segment is staged before the loop by all threads; a
  // CTA whose K sub-parts split its range (nsub > 1) has a single segment, so
  // only single-part CTAs meet the in-loop segment barriers (uniform trip count).
  __syncthreads();
  stage_x(0);
  __syncthreads();
  int seg_first = 0, seg_left = p.seg_stages;
  int slot = 0;
  uint32_t phase = 0;
  for (int st = ws0; st < ws1; ++st) {
    if (seg_left == 0) {
      __syncthreads();
      stage_x(st);
      __syncthreads();
      seg_first = st;
      seg_left = p.seg_stages;
    }
    --seg_left;
    if (!active || failed) continue;

    if (!mbar_wait_bounded(bars + slot, phase)) {
      failed = true;
      continue;
    }
    done = st + 1;
    const uint8_t* stage = ring + slot * kStageBytes;
#pragma unroll
    for (int u = 0; u < C::kU; ++u) {
      // weight words of this super-group: rows q = 2r + h (tile r, box h)
      uint32_t aw[4][C::kWords];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint8_t* rowp = stage + (q & 1) * 2048 + (q >> 1) * 1024;
        if constexpr (C::kLaneB >= 16) {
#pragma unroll
          for (int i = 0; i < kLoads; ++i) {
            const uint4 v = *reinterpret_cast<const uint4*>(rowp + aoff[u][i]);
            aw[q][4 * i] = v.x;
            aw[q][4 * i + 1] = v.y;
            aw[q][4 * i + 2] = v.z;
            aw[q][4 * i + 3] = v.w;
          }
        } else {
          const uint2 v = *reinterpret_cast<const uint2*>(rowp + aoff[u][0]);
          aw[q][0] = v.x;
          aw[q][1] = v.y;
        }
      }
      // staged activations of the lane's two streams (zeros when the lane's column is elsewhere)
      const int gseg = (st - seg_first) * C::kGPS + u * C::kSlots;  // group of slot 0 in the segment
      const int gabs = (st0 + st) * C::kGPS + u * C::kSlots;        // absolute group of slot 0
      const uint8_t* yrow = ys + bm * p.y_ld + gseg * C::kYG;
      const uint8_t* yl = (act_lo && gabs + slot_lo < gpr) ? yrow + slot_lo * C::kYG + ypo_lo : zero_blk;
      const uint8_t* yh = (act_hi && gabs + slot_hi < gpr) ? yrow + slot_hi * C::kYG : zero_blk;
#pragma unroll
      for (int qd = 0; qd < C::kQuads; ++qd) {
        uint32_t bvv[8];  // B operands: step j uses (bvv[2j], bvv[2j+1])
        if constexpr (kPaired) {
          const uint4 b0 = *reinterpret_cast<const uint4*>(yl + 32 * qd);
          const uint4 b1 = *reinterpret_cast<const uint4*>(yl + 32 * qd + 16);
          bvv[0] = b0.x; bvv[1] = b0.y; bvv[2] = b0.z; bvv[3] = b0.w;
          bvv[4] = b1.x; bvv[5] = b1.y; bvv[6] = b1.z; bvv[7] = b1.w;
        } else {
          const uint4 bl = *reinterpret_cast<const uint4*>(yl + 16 * qd);
          const uint4 bh = *reinterpret_cast<const uint4*>(yh + 16 * qd);
          bvv[0] = bl.x; bvv[2] = bl.y; bvv[4] = bl.z; bvv[6] = bl.w;
          bvv[1] = bh.x; bvv[3] = bh.y; bvv[5] = bh.z; bvv[7] = bh.w;
        }
        uint32_t pl[4][4], ph[4][4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          dequant_quad<TA, WF>(&aw[q][qd * C::kWQ], pl[q]);
          dequant_quad<TA, WF>(&aw[q][C::kWords / 2 + qd * C::kWQ], ph[q]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            const uint32_t a[4] = {pl[2 * r][j], pl[2 * r + 1][j], ph[2 * r][j], ph[2 * r + 1][j]};
            if (Enc<TA, WF>::half_step(j)) mma_16816<true>(cacc[j & 1][r], a, bvv[2 * j], bvv[2 * j + 1]);
            else mma_16816<false>(cacc[j & 1][r], a, bvv[2 * j], bvv[2 * j + 1]);
          }
      }
      if constexpr (C::kScaled) {
        // super-group epilogue for the lane's columns 2t+e: group gabs + slot
        float4 mt[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int n = 2 * t + e;
          const int m = n % MC, sl = n / MC;
          const bool ok = m < M && sl < C::kSlots && gabs + sl < gpr;
          mt[e] = *reinterpret_cast<const float4*>(ok ? reinterpret_cast<const uint8_t*>(meta + m * p.meta_ld + gseg + sl)
                                                      : zero_blk);
        }
        uint32_t sv[2][2], bv[2][2];  // [tile][h]: (s of col 2t) | (s of col 2t+1) << 16, same for bias
        if constexpr (C::kAffine) {
#pragma unroll
          for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int o = (rbi * 32 + h * 16 + 8 * r + sg) * p.sc_ld + gseg + ss0 + sc_off;
              if constexpr (kPairCols) {
                if ((sc_off & 1) == 0) {
                  sv[r][h] = *reinterpret_cast<const uint32_t*>(scs + o);
                  bv[r][h] = *reinterpret_cast<const uint32_t*>(scb + o);
                } else {  // a K chunk starting at an odd group: the pair straddles 4 bytes
                  sv[r][h] = static_cast<uint32_t>(scs[o]) | (static_cast<uint32_t>(scs[o + 1]) << 16);
                  bv[r][h] = static_cast<uint32_t>(scb[o]) | (static_cast<uint32_t>(scb[o + 1]) << 16);
                }
              } else {
                sv[r][h] = scs[o];
                bv[r][h] = scb[o];
              }
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const float d = (cacc[0][r][2 * h + e] + cacc[1][r][2 * h + e]) - mt[e].y;
              if constexpr (C::kAffine) {
                const uint32_t s16 = (kPairCols && e) ? (sv[r][h] >> 16) : (sv[r][h] & 0xFFFFu);
                const uint32_t b16 = (kPairCols && e) ? (bv[r][h] >> 16) : (bv[r][h] & 0xFFFFu);
                const float sf = bits_to_float<TA>(s16), bf = bits_to_float<TA>(b16);
                res[r][h][e] = fmaf(sf * mt[e].x, d, fmaf(bf, mt[e].z, res[r][h][e]));
              } else {
                res[r][h][e] = fmaf(mt[e].x, d, res[r][h][e]);
              }
              cacc[0][r][2 * h + e] = 0.f;
              cacc[1][r][2 * h + e] = 0.f;
            }
      }
    }
    // refill this slot with the stage `ring` ahead
    __syncwarp();
    if (st + p.ring < ws1 && lane == 0) {
      fence_proxy_async_smem();
      issue_stage(slot, st + p.ring);
    }
    if (++slot == p.ring) {
      slot = 0;
      phase ^= 1u;
    }
  }
  if (active && failed) {
    // a TMA load never completed: report and drain what is still in flight
    if (p.status && lane == 0) atomicOr(p.status, kStatusTimeout);
    for (int st = done; st < min(ws1, done + p.ring); ++st)
      mbar_wait_bounded(bars + (st - ws0) % p.ring, ((st - ws0) / p.ring) & 1);
  }
  grid_dependency_launch();

  // ---- per-lane results for activation row m of column 2t+e, summed over group slots
  float val[2][2][2];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int e = 0; e < 2; ++e)
        val[r][h][e] = C::kScaled ? res[r][h][e] : cacc[0][r][2 * h + e] + cacc[1][r][2 * h + e];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if constexpr (MC == 1) {
        float v = val[r][h][0] + val[r][h][1];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        val[r][h][0] = v;
      } else if constexpr (MC == 4) {
#pragma unroll
        for (int e = 0; e < 2; ++e) val[r][h][e] += __shfl_xor_sync(0xffffffffu, val[r][h][e], 2);
      }
    }
  // owner lanes of activation row m = 2t + e (MC == 1: t == 0, e == 0)
  auto own = [&](int e) {
    if constexpr (MC == 1) return t == 0 && e == 0;
    else return 2 * t < MC && 2 * t + e < M;
  };

  // ---- reduction over the K parts: pair P = warp*16 + 8r + g (rows of box A and B)
  // of this CTA belongs to part P / ppc, which sums red[src][P % ppc][h][m] over src.
  // With the fused cache append every pair belongs to part 0 (a head's
  // absolute maximum needs all of its pairs in one CTA).
  const bool kv_fused = (EPI == EPI_ROPE) && p.kv_k_cache != nullptr;
  const int ppc = kv_fused ? 64 : 64 / nparts;
  if (active) {
    const uint32_t red_u32 = smem_u32(red);
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          if (!own(e)) continue;
          const int m = (MC == 1) ? 0 : 2 * t + e;
          const int P = rbi * 16 + 8 * r + g;
          const int owner = kv_fused ? 0 : P / ppc;
          const int src = part * nsub + sub;
          const uint32_t addr = red_u32 + static_cast<uint32_t>((((src * ppc + P % ppc) * 2 + h) * M + m) * 4);
          if (nparts == 1) st_shared_f32(addr, val[r][h][e]);
          else st_cluster_f32(cluster_map(addr, owner), val[r][h][e]);
        }
  }
  if (nparts > 1) cluster_sync_all();
  else __syncthreads();

  // ---- final epilogue over this part's pairs
  const int own_pairs = (kv_fused && part != 0) ? 0 : ppc;
  // fused all-reduce: this CTA's exchange epoch (the same on every rank)
  const size_t ar_chan_bytes = static_cast<size_t>(p.ar_world) * p.ar_np * 64 + static_cast<size_t>(kArCtas) * 4;
  __shared__ unsigned s_epoch;
  unsigned* ar_seen = nullptr;
  if (EPI == EPI_RESID && p.ar_world > 1) {
    ar_seen = reinterpret_cast<unsigned*>(p.ar_buf[p.ar_rank] + p.ar_channel * ar_chan_bytes +
                                          static_cast<size_t>(p.ar_world) * p.ar_np * 64) +
              (blockIdx.y * gridDim.x + blockIdx.x);
    if (threadIdx.x == 0) s_epoch = *ar_seen + 1u;
    __syncthreads();
  }
  // value of pair pl (box h) for activation row m: per K chunk the chunk's
  // parts added in rank order from zero, times the per-channel scale (a
  // rounded product, never fused into a later add: the value a launch over
  // that chunk alone produces); the chunks' values then meet in the balanced
  // tree of tree_sum8
  const int nchunks = p.chunks;
  const int sstride = ppc * 2 * M;  // floats between sources in `red`
  auto pair_row = [&](int pl, int h) {
    const int P = part * ppc + pl;
    const int rbx = blockIdx.y * kGemvWarps + (P >> 4);
    return rbx < rowblocks ? box_row0<EPI>(p, rbx, h) + 8 * ((P >> 3) & 1) + sigma_row<C::kLaneB>(P & 7) : p.N;
  };
  if (nchunks > 1) {
    // chunk values in parallel, each into its chunk's first source slot
    const int per = cparts * nsub;
    const int items = own_pairs * M * 2 * nchunks;
    for (int idx = threadIdx.x; idx < items; idx += kNT) {
      const int z = idx % nchunks;
      const int rest = idx / nchunks;
      const int h = rest & 1, m = (rest >> 1) % M, pl = (rest >> 1) / M;
      float* rd = red + pl * 2 * M + h * M + m;
      float v = 0.f;
      for (int src = z * per; src < (z + 1) * per; ++src) v += rd[src * sstride];
      if constexpr (WF == W_I8PC) {
        const int row = pair_row(pl, h);
        if (row < p.N) v = __fmul_rn(v, static_cast<const float*>(p.s0)[row]);
      }
      rd[z * per * sstride] = v;
    }
    __syncthreads();
  }
  auto part_sum = [&](int pl, int m, int h, int row) {
    const float* rd = red + pl * 2 * M + h * M + m;  // source src at rd[src * sstride]
    if (nchunks == 1) {
      float v = 0.f;
      for (int src = 0; src < nparts * nsub; ++src) v += rd[src * sstride];
      if constexpr (WF == W_I8PC) {
        if (row < p.N) v = __fmul_rn(v, static_cast<const float*>(p.s0)[row]);
      }
      return v;
    }
    const int per = cparts * nsub;
    float c[8];
#pragma unroll
    for (int z = 0; z < 8; ++z) c[z] = z < nchunks ? rd[z * per * sstride] : 0.f;
    return tree_sum8(c, nchunks);
  };

  bool gave_up = false;  // fused all-reduce: a wait of this thread ran out
  for (int idx = threadIdx.x; idx < own_pairs * M; idx += kNT) {
    const int pl = idx / M, m = idx - (idx / M) * M;
    const int P = (kv_fused ? 0 : part * ppc) + pl;
    const int w = P >> 4, r = (P >> 3) & 1, gg = P & 7;
    const int rbx = blockIdx.y * kGemvWarps + w;
    if (rbx >= rowblocks) continue;
    const int sgg = sigma_row<C::kLaneB>(gg);
    const int row_lo = box_row0<EPI>(p, rbx, 0) + 8 * r + sgg;
    const int row_hi = box_row0<EPI>(p, rbx, 1) + 8 * r + sgg;
    float v_lo = part_sum(pl, m, 0, row_lo);
    float v_hi = part_sum(pl, m, 1, row_hi);
    if constexpr (EPI == EPI_ARGMAX) {
      unsigned long long best = 0ull;
      if (row_lo < p.N) best = argmax_key(v_lo, row_lo + p.argmax_offset);
      if (row_hi < p.N) {
        const unsigned long long k2 = argmax_key(v_hi, row_hi + p.argmax_offset);
        best = k2 > best ? k2 : best;
      }
      if (best) atomicMax(&s_keys[m], best);
    } else if constexpr (EPI == EPI_SWIGLU) {
      const int n = row_lo;  // gate row n (set 0) pairs with up row n (set 1)
      if (n < p.N) {
        const float gt = round_act<TA>(v_lo), up = round_act<TA>(v_hi);
        const float act = p.act ? 0.5f * gt * (1.0f + erff(gt * 0.70710678118654752f)) : gt / (1.0f + expf(-gt));
        store_act<TA>(p.y, static_cast<size_t>(m + p.m0) * p.ldy + n, act * up);
      }
    } else if constexpr (EPI == EPI_ROPE) {
      const int wph = p.head_dim / 32;
      const int head = rbx / wph;
      const int i = 16 * (rbx % wph) + 8 * r + sgg;  // rotation pair index
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
        const float angle = static_cast<float>(p.positions[m + p.m0]) * p.inv_freq[i];
        float sn, cs;
        sincosf(angle, &sn, &cs);
        const float ra = a * cs - b * sn;
        const float rb2 = b * cs + a * sn;
        a = ra;
        b = rb2;
      }
      if (kv_fused && head >= p.heads_q) {
        // stash the stored-precision values in this pair's own slot of source 0
        a = round_act<TA>(a);
        b = round_act<TA>(b);
        red[((0 * ppc + pl) * 2 + 0) * M + m] = a;
        red[((0 * ppc + pl) * 2 + 1) * M + m] = b;
        atomicMax(&s_kvmax[w / wph][m], __float_as_uint(fmaxf(fabsf(a), fabsf(b))));
        continue;
      }
      const int bi = (m + p.m0) / p.seq_len, l = (m + p.m0) % p.seq_len;
      const size_t obase = ((static_cast<size_t>(bi) * nh + hh) * p.seq_len + l) * p.head_dim;
      store_act<TA>(out, obase + i, a);
      store_act<TA>(out, obase + half + i, b);
    } else {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = h ? row_hi : row_lo;
        if (row >= p.N) continue;
        const float v = h ? v_hi : v_lo;
        const size_t o = static_cast<size_t>(m + p.m0) * p.ldy + row;
        if constexpr (EPI == EPI_RESID) {
          if (p.ar_world > 1) {
            // fused all-reduce: post this rank's fp32 partial with the epoch in
            // slot [ar_rank] of every other rank, wait for the other ranks'
            // partials of the same output element here, add them in tree order
            const unsigned epoch = s_epoch;
            const size_t col = (static_cast<size_t>(row) * 8 + m + p.m0) * 8;
            const size_t chan = p.ar_channel * ar_chan_bytes;
            for (int q = 0; q < p.ar_world; ++q)
              if (q != p.ar_rank)
                st_slot(p.ar_buf[q] + chan + static_cast<size_t>(p.ar_rank) * p.ar_np * 64 + col, v, epoch);
            // the ranks' partials, added in the balanced tree of the K chunks
            // (rank r holds chunks [r*c, (r+1)*c)), so every degree rounds alike
            float pv[8];
            for (int q = 0; q < 8; ++q) pv[q] = 0.f;
            for (int q = 0; q < p.ar_world; ++q) {
              if (q == p.ar_rank) {
                pv[q] = v;
                continue;
              }
              const uint8_t* slot = p.ar_buf[p.ar_rank] + chan + static_cast<size_t>(q) * p.ar_np * 64 + col;
              unsigned long long w = ld_slot(slot);
              if (static_cast<unsigned>(w >> 32) != epoch && !gave_up) {
                // once any wait of this or an earlier launch has run out (the
                // status word persists in the workspace), every later wait is
                // skipped: a dead peer costs one bound, not one per element
                if (p.status && (ld_volatile_u32(p.status) & kStatusTimeout)) {
                  gave_up = true;
                } else {
                  const long long start = clock64();
                  while (static_cast<unsigned>((w = ld_slot(slot)) >> 32) != epoch) {
                    if (clock64() - start > (1LL << 31)) {
                      if (p.status) atomicOr(p.status, kStatusTimeout);
                      gave_up = true;
                      break;
                    }
                    if (p.status && (ld_volatile_u32(p.status) & kStatusTimeout)) {
                      gave_up = true;
                      break;
                    }
                  }
                }
              }
              pv[q] = __uint_as_float(static_cast<unsigned>(w));
            }
            const float sum = tree_sum8(pv, p.ar_world);
            const float res_v = load_act<TA>(p.residual, static_cast<size_t>(m + p.m0) * p.ldr + row);
            store_act<TA>(p.y, o, res_v + round_act<TA>(sum));
            continue;
          }
          const float res_v = load_act<TA>(p.residual, static_cast<size_t>(m + p.m0) * p.ldr + row);
          store_act<TA>(p.y, o, res_v + round_act<TA>(v));
        } else {
          if (p.y_f32) static_cast<float*>(p.y)[o] = v;
          else store_act<TA>(p.y, o, v);
        }
      }
    }
  }
  if constexpr (EPI == EPI_ARGMAX) {
    __syncthreads();
    if (threadIdx.x < M && s_keys[threadIdx.x]) atomicMax(p.argmax_keys + p.m0 + threadIdx.x, s_keys[threadIdx.x]);
  }
  if (EPI == EPI_RESID && p.ar_world > 1 && threadIdx.x == 0) *ar_seen = s_epoch;
  if constexpr (EPI == EPI_ROPE) {
    if (kv_fused) {
      // symmetric INT8 per (token, KV head): scale = fp16(max|x| / 127) (1 for
      // a zero row), code = clamp(rint(x / scale), -127, 127) - the arithmetic
      // of sb_kv_append_int8 on the values k_out / v_out would have held
      __syncthreads();
      const int wph = p.head_dim / 32, half = p.head_dim / 2;
      for (int idx = threadIdx.x; idx < own_pairs * M; idx += kNT) {
        const int pl = idx / M, m = idx - (idx / M) * M;
        const int P = pl, w = P >> 4, r = (P >> 3) & 1;
        const int rbx = blockIdx.y * kGemvWarps + w;
        if (rbx >= rowblocks) continue;
        const int head = rbx / wph;
        if (head < p.heads_q) continue;
        const bool is_k = head < p.heads_q + p.heads_kv;
        const int kh = head - p.heads_q - (is_k ? 0 : p.heads_kv);
        const int bi = (m + p.m0) / p.seq_len;
        const int pos = p.positions[m + p.m0];
        if (pos < 0 || pos >= p.kv_capacity) continue;
        const int i = 16 * (rbx % wph) + 8 * r + sigma_row<C::kLaneB>(P & 7);
        __half s16 = __float2half_rn(__fdiv_rn(__uint_as_float(s_kvmax[w / wph][m]), 127.0f));
        if (__half2float(s16) == 0.f) s16 = __float2half_rn(1.0f);
        const float sc = __half2float(s16);
        const size_t row = (static_cast<size_t>(bi) * p.heads_kv + kh) * p.kv_capacity + pos;
        int8_t* codes = (is_k ? p.kv_k_cache : p.kv_v_cache) + row * p.head_dim;
        const float a = red[((0 * ppc + pl) * 2 + 0) * M + m], b = red[((0 * ppc + pl) * 2 + 1) * M + m];
        codes[i] = static_cast<int8_t>(static_cast<int>(fminf(fmaxf(rintf(__fdiv_rn(a, sc)), -127.f), 127.f)));
        codes[half + i] = static_cast<int8_t>(static_cast<int>(fminf(fmaxf(rintf(__fdiv_rn(b, sc)), -127.f), 127.f)));
        if (i == 0) (is_k ? p.kv_k_scale : p.kv_v_scale)[row] = s16;
      }
    }
  }
}

// ------------------------------------------------------------------ host side

namespace {

constexpr int kMaxParts = 16;  // CTAs per cluster sharing one row group's K range

struct ClusterFit {
  const void* kernel;
  int device, parts, threads;
  size_t smem;
  int clusters;
};

// Largest number of co-resident clusters of `parts` CTAs (cached per kernel, size and device).
int max_active_clusters(const void* kernel, int parts, int threads, size_t smem, int row_groups) {
  static std::mutex mu;
  static std::vector<ClusterFit> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const ClusterFit& c : cache)
      if (c.kernel == kernel && c.device == dev && c.parts == parts && c.threads == threads && c.smem == smem)
        return c.clusters;
  }
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(parts, std::max(1, row_groups));
  config.blockDim = dim3(threads);
  config.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(parts);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  config.attrs = attr;
  config.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &config) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  std::lock_guard<std::mutex> lock(mu);
  cache.push_back({kernel, dev, parts, threads, smem, n});
  return n;
}

// Function attributes, once per kernel and device: the shared-memory opt-in and
// cluster sizes above 8.
bool prepare_kernel(const void* kernel, bool* large_clusters) {
  struct Prepared {
    const void* kernel;
    int device;
    bool large;
  };
  static std::mutex mu;
  static std::vector<Prepared> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  for (const Prepared& d : done)
    if (d.kernel == kernel && d.device == dev) {
      *large_clusters = d.large;
      return true;
    }
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  bool large = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
  if (!large) cudaGetLastError();
  done.push_back({kernel, dev, large});
  *large_clusters = large;
  return true;
}

int rowblocks_of(int epi, int N) {
  return epi == EPI_SWIGLU ? (N + 15) / 16 : (epi == EPI_ROPE ? N / 32 : (N + 31) / 32);
}

template <typename TA, int WF, int G, int EPI, bool NORM, int MC>
int launch_gemv_mc(GemvParams& p, cudaStream_t stream) {
  using C = Geo<WF, G, MC>;
  auto kernel = gemv_kernel<TA, WF, G, EPI, NORM, MC>;
  bool large_clusters = false;
  if (!prepare_kernel(reinterpret_cast<const void*>(kernel), &large_clusters))
    return fail(SB_ECUDA, "gemv: shared memory opt-in failed");
  const int row_groups = (rowblocks_of(EPI, p.N) + kGemvWarps - 1) / kGemvWarps;
  // the K split is chosen for the planned shape (the rows and K chunks of the
  // unsharded matrix, its clusters all resident at once), so shards of it sum alike
  const int plan_groups = (rowblocks_of(EPI, p.plan_rows > 0 ? p.plan_rows : p.N) + kGemvWarps - 1) / kGemvWarps;
  const int pchunks = std::max(1, p.plan_chunks > 0 ? p.plan_chunks : p.chunks);
  const int row_bytes = static_cast<int>(static_cast<int64_t>(p.K) * C::kBits / 8);
  p.stages_total = (row_bytes + 127) / 128;

  // Scales/biases come by TMA when each table row is a multiple of 16 bytes and
  // the tables are 16-byte aligned.
  const int gpr = C::kAffine ? p.K / C::kGroupK : 0;
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  // (a K chunk may start at any group: the box then starts at the group rounded
  // down to 8, and a planned launch reserves the 7 columns that can cost
  // whether or not its tables allow TMA, so its plan does not depend on them)
  const bool planned = pchunks > 1;
  const bool tma_ok = C::kAffine && (gpr % 8 == 0 || planned) && p.sc_stride % 8 == 0 && al16(p.s0) && al16(p.b0) &&
                      al16(p.s1) && al16(p.b1);
  // Per candidate (cluster size, K sub-parts per CTA, ring depth): activation
  // segment and shared memory; 0 when the sub-parts cannot share one segment.
  auto configure = [&](int parts, int nsub, int ring) -> size_t {
    const int per = (p.stages_total + parts - 1) / parts;  // most stages of one CTA
    const int per_warp = (per + nsub - 1) / nsub;
    p.ring = std::max(1, std::min(per_warp, ring));
    // staged x + meta (per activation row) and scales/biases (128 rows) per stage
    const int per_stage = C::kGPS * (C::kYG + 16) * p.M + (C::kAffine ? C::kGPS * 128 * 4 : 0);
    p.seg_stages = std::max(1, std::min(per, (16 * 1024) / per_stage));
    if (nsub > 1 && (p.seg_stages < per || per < nsub)) return 0;
    const int seg_groups = p.seg_stages * C::kGPS;
    p.y_ld = seg_groups * C::kYG;
    if (((p.y_ld / 16) & 1) == 0) p.y_ld += 16;  // rows of different m start in different banks
    p.meta_ld = seg_groups;
    // staged scales: lanes read up to column seg_groups - kSlots + 7 (M = 1);
    // a multiple of 8 elements with an odd number of 8s makes the lanes' 4-byte
    // reads of 8 rows x 4 columns hit 32 distinct banks
    p.sc_ld = 0;
    if (C::kAffine) {
      // TMA boxes start at the group rounded down to 8 (up to 6 more columns)
      const int need = seg_groups + (MC == 1 ? std::max(0, 8 - C::kSlots) : 0) + (planned ? 7 : (tma_ok ? 6 : 0));
      int q = (need + 7) / 8;
      if ((q & 1) == 0) ++q;
      p.sc_ld = 8 * q;
    }
    return static_cast<size_t>(2048) + static_cast<size_t>(kGemvWarps) * nsub * p.ring * kStageBytes +
           static_cast<size_t>(p.M) * p.y_ld + static_cast<size_t>(p.M) * p.meta_ld * 16 +
           static_cast<size_t>(128) * p.M * nsub * (p.kv_k_cache != nullptr ? parts : 1) * sizeof(float) +
           static_cast<size_t>(2) * kGemvWarps * 32 * p.sc_ld * sizeof(uint16_t);
  };
  // Largest cluster (K split across CTAs) whose clusters are all co-resident,
  // each CTA with at least two stages; within it, two K sub-parts per CTA (8
  // warps) when they fit, and the deepest ring (4..2) that fits. One CTA of 4
  // warps per row group when the row groups alone fill the GPU. With K chunks
  // the cluster is chunks x (CTAs per chunk), planned for the unsharded chunk
  // count; `parts` below counts the CTAs of one chunk.
  int parts = 1, nsub = 1;
  size_t smem = 0;
  bool chosen = false;
  for (int cand = kMaxParts / pchunks; cand >= (pchunks > 1 ? 1 : 2) && !chosen; cand >>= 1) {
    const int cl = cand * pchunks;
    if (p.stages_total < 2 * cand || (cl > 8 && !large_clusters)) continue;
    for (int ns = 2; ns >= 1 && !chosen; --ns)
      for (int ring = 4; ring >= 2 && !chosen; --ring) {
        smem = configure(cand, ns, ring);
        if (smem == 0) continue;
        if (max_active_clusters(reinterpret_cast<const void*>(kernel), cl, 32 * kGemvWarps * ns, smem, plan_groups) >=
            plan_groups) {
          parts = cand;
          nsub = ns;
          chosen = true;
        }
      }
  }
  if (!chosen) smem = configure(1, 1, 4);
  p.chunk_parts = parts;
  const int cluster = parts * std::max(1, p.chunks);
  p.sc_tma = 0;
  if (tma_ok && p.sc_ld <= 256) {
    p.sc_tma = 1;
    const uint64_t n = static_cast<uint64_t>(p.N);
    if (int st = make_tmap_u16(&p.smap0, p.s0, n, p.sc_stride, p.sc_ld, 16)) return st;
    if (int st = make_tmap_u16(&p.bmap0, p.b0, n, p.sc_stride, p.sc_ld, 16)) return st;
    if (int st = make_tmap_u16(&p.smap1, p.s1, n, p.sc_stride, p.sc_ld, 16)) return st;
    if (int st = make_tmap_u16(&p.bmap1, p.b1, n, p.sc_stride, p.sc_ld, 16)) return st;
  }
  if (p.ar_world > 1 && cluster * row_groups > kArCtas)
    return fail(SB_EUNSUPPORTED, "fused all-reduce: too many CTAs for the exchange counters");
  if (cluster > 8 && !large_clusters) return fail(SB_EUNSUPPORTED, "K chunks: cluster larger than 8 CTAs unavailable");
  dim3 grid(cluster, row_groups);
  if (p.plan_out) {
    const int plan[8] = {cluster, row_groups, kGemvWarps * 32 * nsub, static_cast<int>(smem), parts, nsub, p.ring,
                         p.stages_total};
    for (int i = 0; i < 8; ++i) p.plan_out[i] = plan[i];
    return SB_OK;
  }
  return launch_cluster("gemv", kernel, grid, dim3(kGemvWarps * 32 * nsub), smem, cluster, stream, p);
}

template <typename TA, int WF, int G, int EPI, bool NORM>
int launch_gemv(GemvParams& p, cudaStream_t stream) {
  if (p.M == 1) return launch_gemv_mc<TA, WF, G, EPI, NORM, 1>(p, stream);
  if (p.M <= 4) return launch_gemv_mc<TA, WF, G, EPI, NORM, 4>(p, stream);
  if constexpr (G == 32 && (WF == W_AFF4 || WF == W_AFF8)) {
    // a 32-wide group has too few codes per lane for the 8-column layout:
    // activation rows 0-3 and 4.. go as two launches of the 4-column layout
    GemvParams hi = p;
    p.M = 4;
    if (int st = launch_gemv_mc<TA, WF, G, EPI, NORM, 4>(p, stream)) return st;
    hi.M -= 4;
    hi.m0 += 4;
    hi.x = static_cast<const TA*>(hi.x) + static_cast<size_t>(4) * hi.ldx;
    return launch_gemv_mc<TA, WF, G, EPI, NORM, 4>(hi, stream);
  } else {
    return launch_gemv_mc<TA, WF, G, EPI, NORM, 8>(p, stream);
  }
}

template <typename TA, int WF, int EPI, bool NORM>
int dispatch_group(GemvParams& p, cudaStream_t stream) {
  if constexpr (WF == W_AFF4 || WF == W_AFF8) {
    switch (p.group_size) {
      case 32:
        return launch_gemv<TA, WF, 32, EPI, NORM>(p, stream);
      case 64:
        return launch_gemv<TA, WF, 64, EPI, NORM>(p, stream);
      case 128:
        return launch_gemv<TA, WF, 128, EPI, NORM>(p, stream);
      default:
        return fail(SB_EUNSUPPORTED, "group_size must be 32, 64 or 128");
    }
  } else {
    return launch_gemv<TA, WF, 64, EPI, NORM>(p, stream);
  }
}

template <int EPI, bool NORM>
int dispatch_fmt(int wf, int x_dtype, GemvParams& p, cudaStream_t stream) {
  constexpr bool kAffineEpi = EPI != EPI_ARGMAX;
  constexpr bool kI8Epi = EPI == EPI_STORE || EPI == EPI_RESID || EPI == EPI_ROPE;
  constexpr bool kBf16Epi = EPI == EPI_STORE || EPI == EPI_ARGMAX;
  if (x_dtype == SB_DTYPE_BF16) {
    if constexpr (kAffineEpi) {
      if (wf == W_AFF4) return dispatch_group<__nv_bfloat16, W_AFF4, EPI, NORM>(p, stream);
      if (wf == W_AFF8) return dispatch_group<__nv_bfloat16, W_AFF8, EPI, NORM>(p, stream);
    }
    if constexpr (kI8Epi) {
      if (wf == W_I8PC) return dispatch_group<__nv_bfloat16, W_I8PC, EPI, NORM>(p, stream);
    }
    if constexpr (kBf16Epi) {
      if (wf == W_BF16) return dispatch_group<__nv_bfloat16, W_BF16, EPI, NORM>(p, stream);
    }
  } else if (x_dtype == SB_DTYPE_F16) {
    if constexpr (EPI == EPI_STORE || EPI == EPI_ROPE) {
      if (wf == W_AFF4) return dispatch_group<__half, W_AFF4, EPI, NORM>(p, stream);
      if (wf == W_AFF8) return dispatch_group<__half, W_AFF8, EPI, NORM>(p, stream);
      if (wf == W_I8PC) return dispatch_group<__half, W_I8PC, EPI, NORM>(p, stream);
    }
  }
  return fail(SB_EUNSUPPORTED, "unsupported activation dtype / weight format / epilogue combination");
}

}  // namespace

static int group_k_of(const LinearRequest& r) {
  if (r.wf == W_AFF4 || r.wf == W_AFF8) return r.group_size;
  return 64;
}

// The weight-streaming kernels need no scratch: the K split reduces through
// distributed shared memory. The workspace only carries the status word.
size_t linear_workspace_size(int epi, int N, int K, int group_k) {
  (void)epi;
  (void)N;
  if (group_k <= 0 || K % group_k) return 0;
  return kCounterBytes;
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
  if (r.norm) SB_REQUIRE((reinterpret_cast<uintptr_t>(r.norm_w) & 15) == 0, "norm weight must be 16-byte aligned");
  if (r.epi == EPI_ROPE) {
    SB_REQUIRE(r.head_dim % 32 == 0 && r.head_dim / 2 <= kMaxRopeHalf, "head_dim must be a multiple of 32, <= 256");
    SB_REQUIRE(r.rope_dims == r.head_dim, "the fused RoPE epilogue rotates the full head_dim");
    SB_REQUIRE(r.N == (r.heads_q + 2 * r.heads_kv) * r.head_dim, "QKV rows must equal (Hq + 2*Hkv) * head_dim");
  }
  if (r.epi == EPI_SWIGLU) SB_REQUIRE(r.N % 8 == 0, "SwiGLU width must be a multiple of 8");
  if (r.ar_world > 1) {
    SB_REQUIRE(r.epi == EPI_RESID, "the fused all-reduce belongs to the residual epilogue");
    SB_REQUIRE(r.ar_world <= 8 && r.ar_rank >= 0 && r.ar_rank < r.ar_world, "ar_world must be 2..8, 0 <= ar_rank < ar_world");
    SB_REQUIRE(r.ar_channel == 0 || r.ar_channel == 1, "ar_channel must be 0 or 1");
    for (int q = 0; q < r.ar_world; ++q) SB_REQUIRE(r.ar_buffers[q] != nullptr, "every rank's exchange buffer is required");
  }
  if (r.kv_k_cache != nullptr) {
    SB_REQUIRE(r.epi == EPI_ROPE, "the fused cache append belongs to the RoPE epilogue");
    SB_REQUIRE(r.head_dim == 64 || r.head_dim == 128, "the fused cache append needs head_dim 64 or 128");
    SB_REQUIRE(r.kv_k_scale && r.kv_v_cache && r.kv_v_scale && r.kv_capacity > 0 && r.kv_capacity < (1LL << 31),
               "fused cache append: every cache pointer and a positive capacity are required");
    SB_REQUIRE(r.positions != nullptr, "fused cache append needs positions");
  }

  const int bits = r.wf == W_AFF4 ? 4 : (r.wf == W_BF16 ? 16 : 8);
  const int chunks = r.k_chunks > 1 ? r.k_chunks : 1;
  if (chunks > 1) {
    SB_REQUIRE(chunks <= 8, "k_chunks must be 1..8");
    SB_REQUIRE(r.epi == EPI_RESID || r.epi == EPI_STORE, "K chunks belong to the STORE and RESID epilogues");
    SB_REQUIRE(!r.norm, "K chunks do not combine with the fused RMSNorm");
    SB_REQUIRE(r.plan_chunks == 0 || r.plan_chunks >= chunks, "plan_k_chunks must cover k_chunks");
    SB_REQUIRE(r.K % (chunks * gk) == 0, "K must split into k_chunks chunks of whole groups");
    SB_REQUIRE((static_cast<int64_t>(r.K / chunks) * bits / 8) % 16 == 0,
               "each K chunk must hold a multiple of 16 weight bytes per row");
  }

  GemvParams p{};
  p.x = r.x;
  p.ldx = r.ldx;
  p.M = r.M;
  p.N = r.N;
  p.K = r.K / chunks;
  p.chunks = chunks;
  p.chunk_wbytes = static_cast<int>(static_cast<int64_t>(p.K) * bits / 8);
  SB_REQUIRE(r.scales_ld == 0 || r.scales_ld >= r.K / gk, "scales_ld must cover K / group_size groups");
  p.sc_stride = r.scales_ld > 0 ? r.scales_ld : r.K / gk;
  p.plan_rows = r.plan_rows;
  p.plan_chunks = r.plan_chunks;
  SB_REQUIRE(!r.y_f32 || r.epi == EPI_STORE, "fp32 outputs belong to the STORE epilogue");
  p.y_f32 = r.y_f32 ? 1 : 0;
  p.plan_out = r.plan_out;

  p.w0 = r.w0;
  p.s0 = r.s0;
  p.b0 = r.b0;
  p.w1 = r.w1 ? r.w1 : r.w0;
  p.s1 = r.s1 ? r.s1 : r.s0;
  p.b1 = r.b1 ? r.b1 : r.b0;
  p.group_size = r.group_size;
  {
    const int gpr = p.K / gk;
    auto al4 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 3) == 0; };
    p.pair_scales = (gpr % 2 == 0) && (p.sc_stride % 2 == 0) && al4(p.s0) && al4(p.b0) && al4(p.s1) && al4(p.b1) ? 1 : 0;
  }
  {
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
  p.kv_k_cache = r.kv_k_cache;
  p.kv_k_scale = static_cast<__half*>(r.kv_k_scale);
  p.kv_v_cache = r.kv_v_cache;
  p.kv_v_scale = static_cast<__half*>(r.kv_v_scale);
  p.kv_capacity = static_cast<int>(r.kv_capacity);
  p.ar_world = r.ar_world > 1 ? r.ar_world : 0;
  p.ar_rank = r.ar_rank;
  p.ar_channel = r.ar_channel;
  p.ar_np = static_cast<int>(ar_np(r.N));
  for (int q = 0; q < 8; ++q) p.ar_buf[q] = static_cast<uint8_t*>(r.ar_buffers[q]);
  p.argmax_keys = r.argmax_keys;
  p.argmax_offset = r.argmax_offset;
  p.early_prefetch = r.weights_constant ? 1 : 0;
  p.act = r.activation;
  if (r.epi == EPI_ROPE) {
    for (int i = 0; i < r.rope_dims / 2; ++i)
      p.inv_freq[i] = static_cast<float>(std::pow(static_cast<double>(r.rope_base), -2.0 * i / r.rope_dims));
  }

  switch (r.epi) {
    case EPI_STORE:
      return r.norm ? dispatch_fmt<EPI_STORE, true>(r.wf, r.x_dtype, p, stream)
                    : dispatch_fmt<EPI_STORE, false>(r.wf, r.x_dtype, p, stream);
    case EPI_RESID:
      return dispatch_fmt<EPI_RESID, false>(r.wf, r.x_dtype, p, stream);
    case EPI_SWIGLU:
      return r.norm ? dispatch_fmt<EPI_SWIGLU, true>(r.wf, r.x_dtype, p, stream)
                    : dispatch_fmt<EPI_SWIGLU, false>(r.wf, r.x_dtype, p, stream);
    case EPI_ROPE:
      return r.norm ? dispatch_fmt<EPI_ROPE, true>(r.wf, r.x_dtype, p, stream)
                    : dispatch_fmt<EPI_ROPE, false>(r.wf, r.x_dtype, p, stream);
    case EPI_ARGMAX:
      return r.norm ? dispatch_fmt<EPI_ARGMAX, true>(r.wf, r.x_dtype, p, stream)
                    : dispatch_fmt<EPI_ARGMAX, false>(r.wf, r.x_dtype, p, stream);
  }
  return fail(SB_EINVAL, "unknown epilogue");
}

}  // namespace sb
