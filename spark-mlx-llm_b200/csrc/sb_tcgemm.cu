// Tensor-core linear for M >= 9 activation rows on the 5th-generation tensor
// cores (tcgen05.mma with TMEM accumulators), sm_100a.
//
// Tile: 128 weight rows (MMA M = 128, one TMEM lane per weight row) by BN
// activation rows (MMA N = BN in 16..256, one TMEM column per activation row).
// The product is computed "weights as A": D[n, m] = sum_k W[n, k] * x[m, k],
// both operands K-major in 128-byte-swizzled shared memory, so the weight tile
// is the 128-row operand that the tensor core reads once per K step, and small
// activation counts (16, 64) still use full-height MMAs.
//
// Warp roles (320 threads):
//   warps 0-7  convert the streamed weight stage into the MMA operand (affine
//              codes -> scale * q + bias rounded to the activation dtype, or
//              int8 -> exact 16-bit), then read TMEM in the epilogue
//   warp 8     TMA producer: weight stage (packed codes or int8), the stage's
//              scale/bias boxes, the activation box; one mbarrier per stage
//   warp 9     allocates TMEM, one elected lane issues the MMAs and commits
//              each stage's completion to the stage's "empty" barrier
// A K split over the CTAs of a thread-block cluster (when N alone gives too few
// tiles to fill the 148 SMs) is reduced through distributed shared memory in
// rank order: deterministic, exact for int32, no global workspace.
//
// Every mbarrier wait is bounded; a wait that gives up sets a CTA-wide abort
// flag and the device status word, the producer waits (bounded) for its copies
// in flight, TMEM is freed and the kernel returns.
#include <algorithm>
#include <cmath>
#include <string>

#include "sb_tcgemm.cuh"

namespace sb {

namespace {

constexpr int kBM = 128;          // weight rows per tile
constexpr int kConvWarps = 8;      // conversion + epilogue warps
constexpr int kWProducerWarp = 8;  // weight stages + scale chunks
constexpr int kMmaWarp = 9;
constexpr int kXProducerWarp = 10;  // activation stages
constexpr int kTcThreads = 352;
constexpr int kATile = kBM * 128;  // one 128-byte-swizzled A operand tile (bytes)
constexpr int kMaxSplit = 8;
constexpr size_t kTcSmemMax = 202u << 10;  // above every plan (one-CTA plans are built within 200 KB)

struct TcParams {
  alignas(64) CUtensorMap wmap;  // weight rows [N][row bytes]: box {wraw bytes, 128} (TW_S8: SW128 {128, 128})
  alignas(64) CUtensorMap smap;  // scales [N][K/G] u16, box {8, 128} (affine)
  alignas(64) CUtensorMap bmap;  // biases, same
  alignas(64) CUtensorMap xmap;  // activations [M][K], SW128 box {128 bytes, BN}
  int M, N, K, G;
  int lg_g;  // log2(G): groups are 32, 64 or 128 K values
  int bn, na, nx, nw, ksteps;
  void* y;
  int ldy, y_dtype;
  const float* wscale;
  const float* ascale;
  const void* bias;
  int bias_dtype;
  const int* positions;
  int heads_q, heads_kv, seq_len;
  void* q_out;
  void* k_out;
  void* v_out;
  unsigned* status;
  float inv_freq[64];
};

// ---------------------------------------------------------------- tcgen05 PTX
// Shared-memory matrix descriptor (sm_100 format): K-major operand in the
// canonical 128-byte-swizzle layout, rows of 128 bytes, 8-row core groups
// 1024 bytes apart (SBO), version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1) << 16;           // leading byte offset (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;   // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;           // descriptor version
  d |= static_cast<uint64_t>(2) << 61;           // 128-byte swizzle
  return d;
}
// Instruction descriptor: D format (1 f32, 2 s32), A/B formats (kind::f16:
// 0 f16, 1 bf16; kind::i8: 1 signed), both K-major, N >> 3, M >> 4.
__host__ __device__ constexpr uint32_t umma_idesc(uint32_t dfmt, uint32_t abfmt, uint32_t n, uint32_t m) {
  return (dfmt << 4) | (abfmt << 7) | (abfmt << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

template <bool kI8>
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  if constexpr (kI8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}
// Arrive on `bar` once every tcgen05 operation issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// 32 lanes x 16 consecutive 32-bit TMEM columns starting at `taddr` (lane base in bits 31:16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ uint32_t ld_cluster_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}

// Bounded wait that also gives up as soon as another role of the CTA aborted.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, unsigned* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > (1LL << 31)) {
      *abort_flag = 1;
      if (status) atomicOr(status, kStatusTimeout);
      return false;
    }
  }
  return true;
}

// ------------------------------------------------------------ conversions
__device__ __forceinline__ float bits16_to_float(uint32_t b, bool half) {
  return half ? __half2float(__ushort_as_half(static_cast<unsigned short>(b))) : __uint_as_float(b << 16);
}
template <bool kHalf>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (kHalf) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}
// Eight 4-bit codes (one uint32 word, code e at bits 4e) -> eight 16-bit
// values scale * q + bias, each rounded once (fused multiply-add in the
// operand type), in K order. The codes become exact 16-bit numbers by OR-ing
// them into the mantissa of 128 (bf16) or 1024 (fp16) and subtracting it.
// s2 / b2 hold the scale / bias bits in both halves.
template <bool kHalf>
__device__ __forceinline__ uint4 dequant8_w4(uint32_t w, uint32_t s2, uint32_t b2) {
  constexpr uint32_t kMagic = kHalf ? 0x64006400u : 0x43004300u;
  uint32_t t[4];
  t[0] = lop_and_or(w, 0x000F000Fu, kMagic);        // (q0, q4)
  t[1] = lop_and_or(w >> 4, 0x000F000Fu, kMagic);   // (q1, q5)
  t[2] = lop_and_or(w >> 8, 0x000F000Fu, kMagic);   // (q2, q6)
  t[3] = lop_and_or(w >> 12, 0x000F000Fu, kMagic);  // (q3, q7)
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (kHalf) {
      const __half2 q = __hsub2(*reinterpret_cast<const __half2*>(&t[i]), *reinterpret_cast<const __half2*>(&kMagic));
      const __half2 r = __hfma2(q, *reinterpret_cast<const __half2*>(&s2), *reinterpret_cast<const __half2*>(&b2));
      t[i] = *reinterpret_cast<const uint32_t*>(&r);
    } else {
      const __nv_bfloat162 q =
          __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&t[i]), *reinterpret_cast<const __nv_bfloat162*>(&kMagic));
      const __nv_bfloat162 r = __hfma2(q, *reinterpret_cast<const __nv_bfloat162*>(&s2),
                                       *reinterpret_cast<const __nv_bfloat162*>(&b2));
      t[i] = *reinterpret_cast<const uint32_t*>(&r);
    }
  }
  return make_uint4(prmt(t[0], t[1], 0x5410u), prmt(t[2], t[3], 0x5410u), prmt(t[0], t[1], 0x7632u),
                    prmt(t[2], t[3], 0x7632u));
}

// exact float of an unsigned integer below 2^23
__device__ __forceinline__ float u2f(uint32_t c) { return __uint_as_float(0x4B000000u | c) - 8388608.0f; }

__device__ __forceinline__ void store_typed(void* base, size_t i, float v, int dtype) {
  if (dtype == SB_DTYPE_BF16) static_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
  else if (dtype == SB_DTYPE_F16) static_cast<__half*>(base)[i] = __float2half_rn(v);
  else static_cast<float*>(base)[i] = v;
}
__device__ __forceinline__ float load_typed(const void* base, size_t i, int dtype) {
  if (dtype == SB_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[i]);
  if (dtype == SB_DTYPE_F16) return __half2float(static_cast<const __half*>(base)[i]);
  return static_cast<const float*>(base)[i];
}

template <int TW>
constexpr int wraw_bytes() {  // weight bytes per row per MMA stage (16-bit kinds: 64 K values)
  return TW == TW_AFF4 ? 32 : (TW == TW_S8 ? 128 : 64);
}

// ------------------------------------------------------------------ kernel
template <int TW, bool kHalf, int TE>
__global__ void __launch_bounds__(kTcThreads, 2) tc_linear_kernel(const __grid_constant__ TcParams p) {
  constexpr bool kS8 = TW == TW_S8;
  constexpr bool kAffine = TW == TW_AFF4 || TW == TW_AFF8;
  // converted kinds stream the weights in 128-byte-wide, 128-byte-swizzled boxes
  // of 128 rows, each covering kSub MMA stages of kWStage bytes per row
  constexpr int kWStage = wraw_bytes<TW>();
  constexpr int kSub = kS8 ? 1 : 128 / kWStage;
  constexpr int kRawTile = kS8 ? 0 : kBM * 128;
  constexpr int kScTile = 2 * kBM * 16;             // scales + biases of 8 groups x 128 rows
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = gridDim.x, rank = blockIdx.x;
  const int n0 = blockIdx.y * kBM, m0 = blockIdx.z * p.bn;
  const int ks0 = static_cast<int>(static_cast<long long>(p.ksteps) * rank / S);
  const int ks1 = static_cast<int>(static_cast<long long>(p.ksteps) * (rank + 1) / S);
  const int nk = ks1 - ks0;
  const int BN = p.bn, NA = p.na, NX = p.nx, NW = p.nw;

  extern __shared__ uint8_t smem_dyn[];
  uint8_t* base = smem_dyn + ((1024u - (smem_u32(smem_dyn) & 1023u)) & 1023u);
  uint8_t* a_ring = base;                     // NA x 16 KB: SW128 A operand (TW_S8: loaded by TMA, NA = NX)
  uint8_t* x_ring = a_ring + NA * kATile;     // NX x BN * 128: SW128 activations
  uint8_t* w_ring = x_ring + NX * BN * 128;   // NW x streamed weight stage
  uint8_t* sc_ring = w_ring + NW * kRawTile;  // 2 x scale/bias chunk [2][128][8] u16 (affine)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sc_ring + (kAffine ? 2 * kScTile : 0));
  uint64_t* xfull = bars;           // activation (+ TW_S8 weight) stage landed
  uint64_t* xempty = xfull + NX;    // MMAs of the stage done
  uint64_t* afull = xempty + NX;    // A slot converted (8 warps)
  uint64_t* aempty = afull + NA;    // MMAs reading the A slot done
  uint64_t* wfull = aempty + NA;    // weight stage landed
  uint64_t* wempty = wfull + NW;    // weight stage converted (8 warps)
  uint64_t* scfull = wempty + NW;   // scale chunk landed
  uint64_t* scempty = scfull + 2;   // scale chunk used up (8 warps)
  uint64_t* done = scempty + 2;     // every MMA done
  uint32_t* red = reinterpret_cast<uint32_t*>(a_ring);  // epilogue: [128][BN + 1] 32-bit over the drained rings
  const int rs = BN + 1;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  volatile int* abort_flag = &s_abort;
  const uint32_t tmem_cols = BN <= 32 ? 32u : (BN <= 64 ? 64u : (BN <= 128 ? 128u : 256u));
  // scale chunk (8 groups) of K stage ks (64 K values per stage)
  // (ring slots and phases advance incrementally: no division by a runtime
  // ring depth or group size in the loops)
  auto chunk_of = [&](int ks) { return ((ks * 64) >> p.lg_g) >> 3; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < NX; ++s) {
      mbar_init(xfull + s, 1);
      mbar_init(xempty + s, 1);
    }
    for (int s = 0; s < NA; ++s) {
      mbar_init(afull + s, kConvWarps);
      mbar_init(aempty + s, 1);
    }
    for (int s = 0; s < NW; ++s) {
      mbar_init(wfull + s, 1);
      mbar_init(wempty + s, kConvWarps);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(scfull + s, 1);
      mbar_init(scempty + s, kConvWarps);
    }
    mbar_init(done, 1);
    mbar_fence_init();
    s_abort = 0;
  }
  // the producers' tensor maps: fetch the descriptors while TMEM and the barriers are set up
  if (threadIdx.x == kWProducerWarp * 32 && !kS8) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.wmap)) : "memory");
    if (kAffine) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.smap)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.bmap)) : "memory");
    }
  }
  if (threadIdx.x == kXProducerWarp * 32) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.xmap)) : "memory");
    if (kS8) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.wmap)) : "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  // activations (and positions) may come from the previous kernel in the stream
  grid_dependency_wait();

  if (warp == kWProducerWarp) {
    // ---- weight stages (and scale chunks) into their rings, as far ahead as the rings allow
    if (lane == 0 && !kS8) {
      int issued = 0, chunks = 0, cur = -1;
      int s = 0;
      uint32_t ph = 0u;
      bool stop = false;
      const int nbox = (nk + kSub - 1) / kSub;
      for (int bx = 0; bx < nbox && !stop; ++bx) {
        const int i0 = bx * kSub;
        if constexpr (kAffine) {
          // scale chunks of the box's stages, in stage order
          for (int i = i0; i < min(nk, i0 + kSub); ++i) {
            const int ch = chunk_of(ks0 + i);
            if (ch == cur) continue;
            cur = ch;
            const int cs = chunks & 1, cu = chunks >> 1;
            if (cu > 0 && !tc_wait(scempty + cs, (cu - 1) & 1, abort_flag, p.status)) {
              stop = true;
              break;
            }
            mbar_arrive_expect_tx(scfull + cs, kScTile);
            tma_load_2d(sc_ring + cs * kScTile, &p.smap, ch * 8, n0, scfull + cs);
            tma_load_2d(sc_ring + cs * kScTile + kBM * 16, &p.bmap, ch * 8, n0, scfull + cs);
            ++chunks;
          }
          if (stop) break;
        }
        if (bx >= NW && !tc_wait(wempty + s, ph ^ 1u, abort_flag, p.status)) break;
        mbar_arrive_expect_tx(wfull + s, kRawTile);
        tma_load_2d(w_ring + s * kRawTile, &p.wmap, (ks0 + i0) * kWStage, n0, wfull + s);
        ++issued;
        if (++s == NW) {
          s = 0;
          ph ^= 1u;
        }
      }
      // copies still in flight (only after an abort) land before the memory is reused
      for (int s = 0; s < NW && s < issued; ++s) mbar_wait_bounded(wfull + s, ((issued - 1 - s) / NW) & 1);
      for (int c = 0; c < 2 && c < chunks; ++c) mbar_wait_bounded(scfull + c, ((chunks - 1 - c) / 2) & 1);
    }
  } else if (warp == kXProducerWarp) {
    // ---- activation stages (TW_S8: with the int8 weight tile)
    if (lane == 0) {
      const uint32_t bytes = static_cast<uint32_t>(BN * 128 + (kS8 ? kATile : 0));
      int issued = 0, s = 0;
      uint32_t ph = 0u;
      for (int i = 0; i < nk; ++i) {
        const int ks = ks0 + i;
        if (i >= NX && !tc_wait(xempty + s, ph ^ 1u, abort_flag, p.status)) break;
        mbar_arrive_expect_tx(xfull + s, bytes);
        if constexpr (kS8) tma_load_2d(a_ring + s * kATile, &p.wmap, ks * 128, n0, xfull + s);
        tma_load_2d(x_ring + s * BN * 128, &p.xmap, kS8 ? ks * 128 : ks * 64, m0, xfull + s);
        ++issued;
        if (++s == NX) {
          s = 0;
          ph ^= 1u;
        }
      }
      for (int s = 0; s < NX && s < issued; ++s) mbar_wait_bounded(xfull + s, ((issued - 1 - s) / NX) & 1);
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      const uint32_t idesc = kS8 ? umma_idesc(2, 1, BN, kBM) : umma_idesc(1, kHalf ? 0 : 1, BN, kBM);
      int sx = 0, sa = 0;
      uint32_t px = 0u, pa = 0u;
      for (int i = 0; i < nk; ++i) {
        if (!tc_wait(xfull + sx, px, abort_flag, p.status)) break;
        if (!kS8 && !tc_wait(afull + sa, pa, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(a_ring + sa * kATile), b0 = smem_u32(x_ring + sx * BN * 128);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)  // 4 MMA K steps of 32 bytes inside the 128-byte atom
          tc_mma<kS8>(tmem, umma_desc_sw128(a0 + 32 * kk), umma_desc_sw128(b0 + 32 * kk), idesc,
                      (i > 0 || kk > 0) ? 1u : 0u);
        tc_commit(xempty + sx);
        if (!kS8) tc_commit(aempty + sa);
        if (++sx == NX) {
          sx = 0;
          px ^= 1u;
        }
        if (kS8) {
          sa = sx;
        } else if (++sa == NA) {
          sa = 0;
          pa ^= 1u;
        }
      }
      tc_commit(done);
    }
    __syncwarp();
  } else if constexpr (!kS8) {
    // ---- conversion: thread -> (row r, half h) = 32 K values of the 64 in a stage;
    // the two threads of a row read its stage bytes from the swizzled weight box
    const int r = threadIdx.x >> 1, h = threadIdx.x & 1;
    int chunks = 0, cur = -1;
    int sw = 0, sub = 0, sa = 0;
    uint32_t pw = 0u, pa = 0u;
    for (int i = 0; i < nk; ++i) {
      const int ks = ks0 + i;
      if (sub == 0 && !tc_wait(wfull + sw, pw, abort_flag, p.status)) break;
      int ch = 0;
      if constexpr (kAffine) {
        ch = chunk_of(ks);
        if (ch != cur) {
          cur = ch;
          if (!tc_wait(scfull + (chunks & 1), (chunks >> 1) & 1, abort_flag, p.status)) break;
          ++chunks;
        }
      }
      if (i >= NA && !tc_wait(aempty + sa, pa ^ 1u, abort_flag, p.status)) break;
      // 16-byte chunk c of row r sits at chunk c ^ (r % 8) (128-byte swizzle)
      const uint8_t* wrow = w_ring + sw * kRawTile + r * 128;
      const int c16 = (sub * kWStage + h * (kWStage / 2)) >> 4;
      uint8_t* arow = a_ring + sa * kATile + r * 128;
      // scale / bias of this thread's 32 K values [32h, 32h + 32) (one group: G >= 32)
      float sc = 1.f, bi = 0.f;
      uint32_t s2 = 0u, b2 = 0u;
      if constexpr (kAffine) {
        const int gi = ((ks * 64 + 32 * h) >> p.lg_g) & 7;  // group inside the chunk
        const uint16_t* st = reinterpret_cast<const uint16_t*>(sc_ring + ((chunks - 1) & 1) * kScTile);
        const uint32_t sb = st[r * 8 + gi], bb = st[kBM * 8 + r * 8 + gi];
        sc = bits16_to_float(sb, kHalf);
        bi = bits16_to_float(bb, kHalf);
        s2 = sb | (sb << 16);
        b2 = bb | (bb << 16);
      }
      if constexpr (TW == TW_AFF4) {
        const uint4 w = *reinterpret_cast<const uint4*>(wrow + ((c16 ^ (r & 7)) << 4));
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int j = 4 * h + c;
          *reinterpret_cast<uint4*>(arow + ((j ^ (r & 7)) << 4)) = dequant8_w4<kHalf>(ww[c], s2, b2);
        }
      } else {
        const uint4 wa = *reinterpret_cast<const uint4*>(wrow + ((c16 ^ (r & 7)) << 4));
        const uint4 wb = *reinterpret_cast<const uint4*>(wrow + (((c16 + 1) ^ (r & 7)) << 4));
        const uint32_t ww[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int j = 4 * h + c;
          float f[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if constexpr (TW == TW_AFF8) {
              f[e] = fmaf(u2f((ww[2 * c] >> (8 * e)) & 255u), sc, bi);
              f[4 + e] = fmaf(u2f((ww[2 * c + 1] >> (8 * e)) & 255u), sc, bi);
            } else {  // TW_I8: signed bytes, exact
              f[e] = static_cast<float>(static_cast<int8_t>((ww[2 * c] >> (8 * e)) & 255u));
              f[4 + e] = static_cast<float>(static_cast<int8_t>((ww[2 * c + 1] >> (8 * e)) & 255u));
            }
          }
          uint4 o;
          o.x = pack2<kHalf>(f[0], f[1]);
          o.y = pack2<kHalf>(f[2], f[3]);
          o.z = pack2<kHalf>(f[4], f[5]);
          o.w = pack2<kHalf>(f[6], f[7]);
          *reinterpret_cast<uint4*>(arow + ((j ^ (r & 7)) << 4)) = o;
        }
      }
      fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(afull + sa);
        if (sub == kSub - 1 || i + 1 == nk) mbar_arrive(wempty + sw);
        if (kAffine && (i + 1 == nk || chunk_of(ks + 1) != ch)) mbar_arrive(scempty + ((chunks - 1) & 1));
      }
      if (++sub == kSub) {
        sub = 0;
        if (++sw == NW) {
          sw = 0;
          pw ^= 1u;
        }
      }
      if (++sa == NA) {
        sa = 0;
        pa ^= 1u;
      }
    }
  }
  __syncthreads();

  // ---- accumulators: TMEM -> shared memory [row][BN + 1] (warps 0-7: lane quarter warp % 4)
  if (warp < kConvWarps) {
    if (!mbar_wait_bounded(done, 0)) {
      *abort_flag = 1;
      if (p.status && lane == 0) atomicOr(p.status, kStatusTimeout);
    }
    tc_fence_after();
    const int q = warp & 3, hh = warp >> 2;
    const int row = 32 * q + lane;
    for (int c0 = 16 * hh; c0 < BN; c0 += 32) {
      uint32_t v[16];
      tmem_ld16(tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(c0), v);
#pragma unroll
      for (int e = 0; e < 16; ++e) red[row * rs + c0 + e] = v[e];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols) : "memory");
  }
  if (S > 1) cluster_sync_all();

  // ---- final epilogue over this rank's row pairs (d, d + 64), summed over the cluster in rank order
  const int d0 = 64 * rank / S, d1 = 64 * (rank + 1) / S, P = d1 - d0;
  const int mcount = min(BN, p.M - m0);
  const bool aborted = *abort_flag != 0;
  const uint32_t red_u32 = smem_u32(red);
  for (int idx = threadIdx.x; !aborted && idx < P * mcount; idx += kTcThreads) {
    const int c = idx / P, d = d0 + idx % P;
    const int m = m0 + c;
    uint32_t lo_bits[kMaxSplit], hi_bits[kMaxSplit];
    const uint32_t off_lo = red_u32 + static_cast<uint32_t>((d * rs + c) * 4);
    const uint32_t off_hi = red_u32 + static_cast<uint32_t>(((d + 64) * rs + c) * 4);
    if (S == 1) {
      lo_bits[0] = red[d * rs + c];
      hi_bits[0] = red[(d + 64) * rs + c];
    } else {
#pragma unroll
      for (int q = 0; q < kMaxSplit; ++q)
        if (q < S) {
          lo_bits[q] = ld_cluster_u32(cluster_map(off_lo, q));
          hi_bits[q] = ld_cluster_u32(cluster_map(off_hi, q));
        }
    }
    const int n_lo = n0 + d, n_hi = n0 + 64 + d;
    if constexpr (kS8) {
      int a_lo = 0, a_hi = 0;
#pragma unroll
      for (int q = 0; q < kMaxSplit; ++q)
        if (q < S) {
          a_lo += static_cast<int>(lo_bits[q]);
          a_hi += static_cast<int>(hi_bits[q]);
        }
#pragma unroll
      for (int hsel = 0; hsel < 2; ++hsel) {
        const int n = hsel ? n_hi : n_lo;
        if (n >= p.N) continue;
        const int acc = hsel ? a_hi : a_lo;
        const size_t o = static_cast<size_t>(m) * p.ldy + n;
        if constexpr (TE == TE_I32) {
          static_cast<int32_t*>(p.y)[o] = acc;
        } else {
          float v = __fmul_rn(__fmul_rn(static_cast<float>(acc), p.ascale[m]), p.wscale[n]);
          const float b = p.bias_dtype < 0 ? 0.f : load_typed(p.bias, n, p.bias_dtype);
          v = __fadd_rn(v, b);
          store_typed(p.y, o, v, p.y_dtype);
        }
      }
    } else {
      float v_lo = 0.f, v_hi = 0.f;
#pragma unroll
      for (int q = 0; q < kMaxSplit; ++q)
        if (q < S) {
          v_lo += __uint_as_float(lo_bits[q]);
          v_hi += __uint_as_float(hi_bits[q]);
        }
      const int adt = kHalf ? SB_DTYPE_F16 : SB_DTYPE_BF16;
      if constexpr (TE == TE_ROPE) {
        const int head = n0 / kBM;
        float a = kHalf ? __half2float(__float2half_rn(v_lo)) : round_bf16(v_lo);
        float b = kHalf ? __half2float(__float2half_rn(v_hi)) : round_bf16(v_hi);
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
          const float angle = static_cast<float>(p.positions[m]) * p.inv_freq[d];
          float sn, cs;
          sincosf(angle, &sn, &cs);
          const float ra = a * cs - b * sn;
          const float rb = b * cs + a * sn;
          a = ra;
          b = rb;
        }
        const int bi = m / p.seq_len, l = m % p.seq_len;
        const size_t obase = ((static_cast<size_t>(bi) * nh + hh) * p.seq_len + l) * kBM;
        store_typed(out, obase + d, a, adt);
        store_typed(out, obase + 64 + d, b, adt);
      } else {
#pragma unroll
        for (int hsel = 0; hsel < 2; ++hsel) {
          const int n = hsel ? n_hi : n_lo;
          if (n >= p.N) continue;
          float v = hsel ? v_hi : v_lo;
          if constexpr (TE == TE_CHSCALE) v = __fmul_rn(v, p.wscale[n]);
          store_typed(p.y, static_cast<size_t>(m) * p.ldy + n, v, adt);
        }
      }
    }
  }
  // remote CTAs read this CTA's shared memory until here
  if (S > 1) cluster_sync_all();
}

// ---------------------------------------------------------------- host side
struct TcPlan {
  int bn, na, nx, nw, split, tiles_n, tiles_m;
  size_t smem;
};

int sm_count() { return device_sm_count(); }

int raw_tile_bytes(int tw) { return tw == TW_S8 ? 0 : kBM * 128; }

size_t tc_smem_bytes(int tw, int bn, int na, int nx, int nw) {
  const bool affine = tw == TW_AFF4 || tw == TW_AFF8;
  return 1024 + static_cast<size_t>(na) * kATile + static_cast<size_t>(nx) * bn * 128 +
         static_cast<size_t>(nw) * raw_tile_bytes(tw) + (affine ? 2 * 2 * kBM * 16 : 0) +
         static_cast<size_t>(2 * nx + 2 * na + 2 * nw + 5) * 8;
}

// Tile and ring plan. Tiles up to 128 activation rows run two CTAs per SM
// (<= 110 KB of shared memory each), 256-row tiles one. The weight ring is
// deepest (it streams from HBM), then the activation ring (L2-resident), then
// the converted-operand ring. The epilogue's [128][bn + 1] staging reuses the
// drained rings.
TcPlan plan_tc(const TcRequest& r) {
  TcPlan pl{};
  const int kstage = r.tw == TW_S8 ? 128 : 64;
  const int ksteps = (r.K + kstage - 1) / kstage;
  pl.tiles_n = (r.N + kBM - 1) / kBM;
  const int bn = r.M <= 256 ? ((r.M + 15) / 16) * 16 : 256;
  pl.bn = bn;
  pl.tiles_m = (r.M + bn - 1) / bn;
  // small activation tiles (HBM-bound) run two CTAs per SM; larger ones one,
  // with deeper rings
  int occ = bn <= 64 ? 2 : 1;
  const size_t budget = occ == 2 ? (112u << 10) : (200u << 10);
  const bool s8 = r.tw == TW_S8;
  int na = 2, nx = 2, nw = s8 ? 0 : 2;
  auto size = [&](int a, int x, int w) { return tc_smem_bytes(r.tw, bn, s8 ? x : a, x, w); };
  auto fits = [&](int a, int x, int w) { return size(a, x, w) <= budget; };
  if (s8) {
    while (nx < 8 && fits(0, nx + 1, 0)) ++nx;
    na = nx;
  } else {
    // The converted-operand ring bounds the rate: a slot returns only after
    // conversion -> MMA issue -> MMA completion -> commit (about 2 us per round
    // trip measured on B200), so it gets depth first, then the activation ring
    // (L2-resident boxes), then the weight ring (each slot covers 2-4 stages).
    if (fits(na + 1, nx, nw)) ++na;
    if (fits(na, nx + 1, nw)) ++nx;
    if (fits(na + 1, nx, nw)) ++na;
    while (nx < 4 && fits(na, nx + 1, nw)) ++nx;
    while (na < 6 && fits(na + 1, nx, nw)) ++na;
    while (nx < 6 && fits(na, nx + 1, nw)) ++nx;
    while (nw < 4 && fits(na, nx, nw + 1)) ++nw;
  }
  const size_t ring_bytes = static_cast<size_t>(s8 ? nx : na) * kATile + static_cast<size_t>(nx) * bn * 128 +
                            static_cast<size_t>(nw) * raw_tile_bytes(r.tw);
  size_t red = static_cast<size_t>(kBM) * (bn + 1) * 4;
  for (int extra = 0; red > ring_bytes + static_cast<size_t>(extra) * bn * 128; ++extra) nx = nx + 1;
  if (s8) na = nx;
  pl.na = na;
  pl.nx = nx;
  pl.nw = nw;
  pl.smem = tc_smem_bytes(r.tw, bn, na, nx, nw);
  if (pl.smem > (113u << 10)) occ = 1;
  // K split over a cluster: fill one wave of CTAs, at least two stages per CTA
  const int tiles = pl.tiles_n * pl.tiles_m;
  int split = 1;
  for (int s = 2; s <= kMaxSplit; ++s)
    if (tiles * s <= sm_count() * occ && ksteps / s >= 2) split = s;
  pl.split = split;
  return pl;
}

template <int TW, bool kHalf, int TE>
int launch_tc(const TcParams& p, const TcPlan& pl, cudaStream_t stream) {
  auto kernel = tc_linear_kernel<TW, kHalf, TE>;
  // opt in to the largest dynamic shared memory any plan uses (kTcSmemMax), once per device
  if (pl.smem > kTcSmemMax) return fail(SB_EINVAL, "tensor-core linear: tile plan exceeds shared memory");
  static int opted[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !opted[dev]) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kTcSmemMax)) !=
        cudaSuccess)
      return fail(SB_ECUDA, "tensor-core linear: shared memory opt-in failed");
    if (dev >= 0 && dev < 64) opted[dev] = 1;
  }
  const dim3 grid(pl.split, pl.tiles_n, pl.tiles_m);
  return launch_cluster("tensor-core linear", kernel, grid, dim3(kTcThreads), pl.smem, pl.split, stream, p);
}

}  // namespace

bool tc_linear_supported(const TcRequest& r) {
  if (r.M < 9 || r.N <= 0 || r.K <= 0) return false;
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!al16(r.x) || !al16(r.w)) return false;
  if (r.tw == TW_S8) return r.K % 16 == 0;
  if (r.act_dtype != SB_DTYPE_BF16 && r.act_dtype != SB_DTYPE_F16) return false;
  if (r.K % 64) return false;
  if (r.tw == TW_AFF4 || r.tw == TW_AFF8) {
    if (r.group_size != 32 && r.group_size != 64 && r.group_size != 128) return false;
    if (r.K % r.group_size || (r.K / r.group_size) % 8 || !al16(r.scales) || !al16(r.biases)) return false;
  }
  if (r.te == TE_ROPE) {
    if (r.N != (r.heads_q + 2 * r.heads_kv) * kBM) return false;  // head_dim 128: one tile per head
  }
  return true;
}

int run_tc_linear(const TcRequest& r, cudaStream_t stream) {
  if (!tc_linear_supported(r)) return fail(SB_EUNSUPPORTED, "tensor-core linear: unsupported shape or alignment");
  const TcPlan pl = plan_tc(r);
  TcParams p{};
  p.M = r.M;
  p.N = r.N;
  p.K = r.K;
  p.G = r.group_size > 0 ? r.group_size : 64;
  p.lg_g = p.G == 32 ? 5 : (p.G == 128 ? 7 : 6);
  p.bn = pl.bn;
  p.na = pl.na;
  p.nx = pl.nx;
  p.nw = pl.nw;
  const int kstage = r.tw == TW_S8 ? 128 : 64;
  p.ksteps = (r.K + kstage - 1) / kstage;
  // weights
  if (r.tw == TW_S8) {
    if (int st = make_tmap_2d(&p.wmap, r.w, 1, r.N, r.K, r.K, 128, kBM, true)) return st;
  } else {
    const int row_bytes = r.tw == TW_AFF4 ? r.K / 2 : r.K;
    if (int st = make_tmap_2d(&p.wmap, r.w, 1, r.N, row_bytes, row_bytes, 128, kBM, true)) return st;
  }
  if (r.tw == TW_AFF4 || r.tw == TW_AFF8) {
    const int gpr = r.K / r.group_size;
    if (int st = make_tmap_2d(&p.smap, r.scales, 2, r.N, gpr, gpr, 8, kBM, false)) return st;
    if (int st = make_tmap_2d(&p.bmap, r.biases, 2, r.N, gpr, gpr, 8, kBM, false)) return st;
  }
  // activations: 128-byte boxes (64 16-bit values or 128 int8) of BN rows
  if (r.tw == TW_S8) {
    if (int st = make_tmap_2d(&p.xmap, r.x, 1, r.M, r.K, r.K, 128, pl.bn, true)) return st;
  } else {
    if (int st = make_tmap_2d(&p.xmap, r.x, 2, r.M, r.K, r.K, 64, pl.bn, true)) return st;
  }
  p.y = r.y;
  p.ldy = r.ldy > 0 ? r.ldy : r.N;
  p.y_dtype = r.y_dtype;
  p.wscale = r.wscale;
  p.ascale = r.ascale;
  p.bias = r.bias;
  p.bias_dtype = r.bias ? r.bias_dtype : -1;
  p.positions = r.positions;
  p.heads_q = r.heads_q;
  p.heads_kv = r.heads_kv;
  p.seq_len = r.seq_len > 0 ? r.seq_len : 1;
  p.q_out = r.q_out;
  p.k_out = r.k_out;
  p.v_out = r.v_out;
  if (r.te == TE_ROPE) {
    for (int i = 0; i < 64; ++i)
      p.inv_freq[i] = static_cast<float>(std::pow(static_cast<double>(r.rope_base), -2.0 * i / 128.0));
  }
  const bool half = r.act_dtype == SB_DTYPE_F16;
  switch (r.tw) {
    case TW_AFF4:
      if (r.te == TE_ROPE) return half ? launch_tc<TW_AFF4, true, TE_ROPE>(p, pl, stream)
                                       : launch_tc<TW_AFF4, false, TE_ROPE>(p, pl, stream);
      return half ? launch_tc<TW_AFF4, true, TE_STORE>(p, pl, stream) : launch_tc<TW_AFF4, false, TE_STORE>(p, pl, stream);
    case TW_AFF8:
      if (r.te == TE_ROPE) return half ? launch_tc<TW_AFF8, true, TE_ROPE>(p, pl, stream)
                                       : launch_tc<TW_AFF8, false, TE_ROPE>(p, pl, stream);
      return half ? launch_tc<TW_AFF8, true, TE_STORE>(p, pl, stream) : launch_tc<TW_AFF8, false, TE_STORE>(p, pl, stream);
    case TW_I8:
      return half ? launch_tc<TW_I8, true, TE_CHSCALE>(p, pl, stream) : launch_tc<TW_I8, false, TE_CHSCALE>(p, pl, stream);
    case TW_S8:
      if (r.te == TE_I32) return launch_tc<TW_S8, false, TE_I32>(p, pl, stream);
      return launch_tc<TW_S8, false, TE_W8A8>(p, pl, stream);
  }
  return fail(SB_EINVAL, "tensor-core linear: unknown weight kind");
}

}  // namespace sb
