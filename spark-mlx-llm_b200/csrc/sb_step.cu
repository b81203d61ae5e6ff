// Persistent decode step (batch 1): the whole step - every layer's RMSNorm +
// QKV + RoPE, INT8-KV attention, o_proj + residual, RMSNorm + gate/up +
// SwiGLU, down + residual, then RMSNorm + lm_head + greedy argmax - as ONE
// cooperative kernel with one CTA per SM. Interface: include/spark_b200_step.h.
//
// Structure of a CTA (kConsumers + 1 warps):
// * the producer warp walks this CTA's share of every weight stream in
//   consumption order and copies each tile (one 16-row block x one K chunk,
//   8-11 KB, contiguous in the stream) into a ring of shared-memory slots with
//   one 1-D bulk async copy (mbarrier complete_tx, L2 evict-first). Weights do
//   not depend on activations, so it runs ahead across operator and layer
//   boundaries, limited only by free slots - HBM keeps streaming while the
//   consumers wait for the previous operator's outputs;
// * consumer warps take the CTA's tiles round-robin, compute each tile's
//   per-row partial sums on the tensor cores (mma.sync m16n8k16 on exact
//   integer code operands, fp32 accumulation), release the slot, and the warp
//   that completes a row block sums its chunk partials in chunk order and
//   runs the operator's epilogue (RoPE, residual, SwiGLU, argmax). A row
//   block whose chunks are split between CTAs is finished by whichever CTA
//   arrives last (global counter; partials through L2).
// * operators are separated by a grid-wide arrival counter (bounded spin).
//
// Tile arithmetic (per lane L = 4g + c; rows g, g+8 of the block):
//   W8  : byte u = int8 + 128 -> fp16 1024 + u (byte permute), minus 1152 in
//         fp16 (exact) = the signed code; x staged as fp16 (exact for the
//         decoder's activations); one accumulator chain over the chunk; the
//         row's fp32 scale multiplies the chunk-ordered sum.
//   W4  : code q -> bf16 128+q (low nibbles) and fp16 64+q (high nibbles),
//         one LOP3 each after one shift per word; x staged as bf16 / fp16
//         pairs in the matching order; the 8 MMA columns carry 8 groups, so
//         the affine epilogue  s*(acc - O) + b*X  (O = sum of offset*x,
//         X = sum of x per group, staged with x) runs once per 8 groups.
//   BF16: weights are the A operand as stored.
#include <algorithm>
#include <cmath>
#include <initializer_list>
#include <mutex>
#include <string>

#include "sb_common.cuh"
#include "spark_b200_step.h"

namespace sb {
namespace step {

constexpr int kConsumers = 11;               // consumer warps per CTA (+1 producer: 384 threads at <= 160 registers)
constexpr int kConsumerThreads = kConsumers * 32;
constexpr int kThreads = kConsumerThreads + 32;  // + the producer warp
constexpr int kMaxSlots = 16;                // ring slots (upper bound)
constexpr int kPartSlots = 64;               // per-tile partial slots
constexpr int kRbSlots = 128;                // row-block completion counters
constexpr int kMaxK = 10240;                 // staged activation values
constexpr int kMaxGroups = kMaxK / 64;
constexpr int kChunks = 8;                   // K chunks of o/down/lm_head (tensor-parallel unit)
constexpr int kAttnChunk = 128;              // tokens per attention work item
constexpr int kMaxLayers = 128;

// shared-memory layout (offsets from a 1024-byte aligned base)
constexpr int kOffBars = 0;            // full[16], empty[16]
constexpr int kOffRbCnt = 256;         // u32 [128]
constexpr int kOffReady = 768;         // u32 [64]: next tile index allowed into a partial slot
constexpr int kOffZero = 1024;         // 256 zero bytes
constexpr int kOffMisc = 1280;         // abort, rms, key, warp sums
constexpr int kOffMeta = 2048;         // float2 [kMaxGroups] (O, X) per staged group
constexpr int kOffPart = kOffMeta + kMaxGroups * 8;               // float [64][32]
constexpr int kOffXs = kOffPart + kPartSlots * 32 * 4;             // staged activations
constexpr int kOffRing = ((kOffXs + kMaxK * 2 + 1023) / 1024) * 1024;

struct Misc {
  int abort;
  float rms;
  unsigned long long key;
  float warp_ss[kConsumers];
};

struct Layer {
  const uint8_t* qkv;
  const float* qkv_scale;
  const uint8_t* o;
  const float* o_scale;
  const uint8_t* gateup;
  const uint8_t* down;
  const __nv_bfloat16* in_norm;
  const __nv_bfloat16* post_norm;
  int8_t* k_cache;
  __half* k_scale;
  int8_t* v_cache;
  __half* v_scale;
};
static_assert(sizeof(Layer) == sizeof(sb_step_layer), "layer table layout");

// Geometry of one weight stream (one operator of one layer).
struct Stream {
  int rbs;      // 16-row blocks
  int chunks;   // K chunks per row block held by this rank
  int tile;     // bytes per tile
  int ck;       // K values per chunk (W8 / BF16) or groups per chunk (W4)
};

struct Params {
  const Layer* layers;
  int num_layers, hidden, heads, kv_heads, inter, vocab, vocab_offset, capacity, vocab_total;
  float eps, attn_scale;
  float inv_freq[64];
  const __nv_bfloat16* embed;
  const uint8_t* head;
  const __nv_bfloat16* final_norm;
  const int* tokens;
  const int* positions;
  __nv_bfloat16* x;
  __nv_bfloat16* q;
  __nv_bfloat16* kv_new;
  __nv_bfloat16* attn;
  __nv_bfloat16* act;
  unsigned long long* keys;
  unsigned* sync;     // workspace word 0: grid arrival counter
  unsigned* status;   // workspace word 1
  unsigned* gcount;   // row-block counters of split row blocks
  unsigned* acount;   // attention per-KV-head counters
  float* gpart;       // split row-block partials [rb][kChunks][32]
  float* apart;       // attention partials [kv head][chunk][G][132]
  int attn_max_chunks;
  Stream sq, so, sgu, sdn, slm;
  int slot_bytes, slots;
};

// ------------------------------------------------------------- small helpers
__device__ __forceinline__ void named_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerThreads) : "memory");
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ float ldcg_f(const float* p) { return __ldcg(p); }
__device__ __forceinline__ float ldcg_bf(const __nv_bfloat16* p) {
  return __uint_as_float(static_cast<uint32_t>(__ldcg(reinterpret_cast<const unsigned short*>(p))) << 16);
}
__device__ __forceinline__ uint4 ldcg16(const void* p) {
  return __ldcg(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ float bfr(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
__device__ __forceinline__ unsigned long long argmax_key(float v, int index) {
  uint32_t u = __float_as_uint(v);
  if (v != v) u = 0x007FFFFFu;
  else u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<unsigned long long>(u) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(index));
}

// Bounded wait on a phase of an mbarrier; on timeout records the status and
// raises the CTA's abort flag.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, const Params& p, Misc* misc) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*reinterpret_cast<volatile int*>(&misc->abort)) return false;
    if (clock64() - start > (1LL << 31)) {
      atomicOr(p.status, kStatusTimeout);
      *reinterpret_cast<volatile int*>(&misc->abort) = 1;
      return false;
    }
  }
  return true;
}

// Grid-wide join between operators: all consumer threads of the CTA finish
// the operator, thread 0 adds this CTA's arrival, waits (bounded) until every
// CTA has arrived `target` times in total, and releases the consumers.
__device__ void grid_join(const Params& p, Misc* misc, unsigned target) {
  named_sync();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(p.sync, 1u);
    if (!*reinterpret_cast<volatile int*>(&misc->abort)) {
      const long long start = clock64();
      while (ld_volatile_u32(p.sync) < target) {
        if (clock64() - start > (1LL << 31) || ld_volatile_u32(p.status) != 0u) {
          atomicOr(p.status, kStatusTimeout);
          misc->abort = 1;
          break;
        }
      }
    }
    __threadfence();
  }
  named_sync();
}

// ------------------------------------------------------------------ tiles
// W8 tile: `kb` blocks of 32 columns. Returns the rows' partial sums.
__device__ __forceinline__ void w8_tile(const uint8_t* tile, const uint8_t* xs, int kb_count, int lane, float& og,
                                        float& oh) {
  const int c = lane & 3;
  float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
  const uint8_t* a_ptr = tile + lane * 16;
  const uint8_t* x_ptr = xs + c * 16;
  constexpr uint32_t kMagic = 0x64646464u;
  constexpr uint32_t kOff = 0x64806480u;  // fp16 1152 in both halves
#pragma unroll 4
  for (int kb = 0; kb < kb_count; ++kb) {
    const uint4 a = lds128(a_ptr + kb * 512);
    const uint4 b = lds128(x_ptr + kb * 64);
    const uint32_t f0[4] = {hsub2_u32(prmt(a.x, kMagic, 0x4140u), kOff), hsub2_u32(prmt(a.y, kMagic, 0x4140u), kOff),
                            hsub2_u32(prmt(a.x, kMagic, 0x4342u), kOff), hsub2_u32(prmt(a.y, kMagic, 0x4342u), kOff)};
    mma_16816<true>(acc0, f0, b.x, b.y);
    const uint32_t f1[4] = {hsub2_u32(prmt(a.z, kMagic, 0x4140u), kOff), hsub2_u32(prmt(a.w, kMagic, 0x4140u), kOff),
                            hsub2_u32(prmt(a.z, kMagic, 0x4342u), kOff), hsub2_u32(prmt(a.w, kMagic, 0x4342u), kOff)};
    mma_16816<true>(acc1, f1, b.z, b.w);
  }
  og = acc0[0] + acc1[0];
  oh = acc0[2] + acc1[2];
}

// BF16 tile: `mmas` blocks of 16 columns.
__device__ __forceinline__ void bf16_tile(const uint8_t* tile, const uint8_t* xs, int mmas, int lane, float& og,
                                          float& oh) {
  const int c = lane & 3;
  float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
  const uint8_t* a_ptr = tile + lane * 16;
  const uint8_t* x_ptr = xs + c * 8;
  int j = 0;
#pragma unroll 2
  for (; j + 1 < mmas; j += 2) {
    const uint4 a0 = lds128(a_ptr + j * 512);
    const uint2 b0 = *reinterpret_cast<const uint2*>(x_ptr + j * 32);
    const uint4 a1 = lds128(a_ptr + (j + 1) * 512);
    const uint2 b1 = *reinterpret_cast<const uint2*>(x_ptr + (j + 1) * 32);
    const uint32_t f0[4] = {a0.x, a0.y, a0.z, a0.w};
    const uint32_t f1[4] = {a1.x, a1.y, a1.z, a1.w};
    mma_16816<false>(acc0, f0, b0.x, b0.y);
    mma_16816<false>(acc1, f1, b1.x, b1.y);
  }
  if (j < mmas) {
    const uint4 a0 = lds128(a_ptr + j * 512);
    const uint2 b0 = *reinterpret_cast<const uint2*>(x_ptr + j * 32);
    const uint32_t f0[4] = {a0.x, a0.y, a0.z, a0.w};
    mma_16816<false>(acc0, f0, b0.x, b0.y);
  }
  og = acc0[0] + acc1[0];
  oh = acc0[2] + acc1[2];
}

// 4-bit word -> (bf16 128+n0, 128+n4), (fp16 64+n1, 64+n5), (bf16 n2,n6), (fp16 n3,n7)
__device__ __forceinline__ void w4_convert(uint32_t w, uint32_t (&t)[4]) {
  const uint32_t s = w >> 8;
  t[0] = lop_and_or(w, 0x000F000Fu, 0x43004300u);
  t[1] = lop_and_or(w, 0x00F000F0u, 0x54005400u);
  t[2] = lop_and_or(s, 0x000F000Fu, 0x43004300u);
  t[3] = lop_and_or(s, 0x00F000F0u, 0x54005400u);
}

// W4 tile of MATS matrices (1 = down, 2 = gate+up) over `ngroups` groups of
// 64. xs points at the chunk's first staged group, om at its (O, X) pairs.
template <int MATS>
__device__ __forceinline__ void w4_tile(const uint8_t* tile, int ngroups, const uint8_t* xs, const float2* om,
                                        const uint8_t* zero, int lane, float (&out)[MATS][2]) {
  const int g = lane >> 2, c = lane & 3;
  const uint8_t* a_ptr = tile + lane * 16;
  const int rounds = (ngroups + 7) >> 3;
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(tile + MATS * ngroups * 512);
  const uint16_t* bi = sc + rounds * MATS * 128;
  float res[MATS][2];
#pragma unroll
  for (int m = 0; m < MATS; ++m) res[m][0] = res[m][1] = 0.f;
  for (int r = 0; r < rounds; ++r) {
    float acc[MATS][4];
#pragma unroll
    for (int m = 0; m < MATS; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;
    const int jn = min(8, ngroups - 8 * r);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j < jn) {
        const int gi = 8 * r + j;
        const uint8_t* bp = (g == j) ? xs + gi * 128 : zero;
        const uint4 b0 = lds128(bp + c * 16);
        const uint4 b1 = lds128(bp + 64 + c * 16);
#pragma unroll
        for (int m = 0; m < MATS; ++m) {
          const uint4 a = lds128(a_ptr + (gi * MATS + m) * 512);
          uint32_t tg[4], th[4];
          w4_convert(a.x, tg);
          w4_convert(a.y, th);
          {
            const uint32_t fa[4] = {tg[0], th[0], tg[2], th[2]};
            const uint32_t fb[4] = {tg[1], th[1], tg[3], th[3]};
            mma_16816<false>(acc[m], fa, b0.x, b0.y);
            mma_16816<true>(acc[m], fb, b0.z, b0.w);
          }
          w4_convert(a.z, tg);
          w4_convert(a.w, th);
          {
            const uint32_t fa[4] = {tg[0], th[0], tg[2], th[2]};
            const uint32_t fb[4] = {tg[1], th[1], tg[3], th[3]};
            mma_16816<false>(acc[m], fa, b1.x, b1.y);
            mma_16816<true>(acc[m], fb, b1.z, b1.w);
          }
        }
      }
    }
    // affine epilogue of this round: the lane's columns 2c, 2c+1 = groups 8r+2c, 8r+2c+1
    float4 o4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (2 * c < jn) {
      const float2 e0 = om[8 * r + 2 * c];
      const float2 e1 = (2 * c + 1 < jn) ? om[8 * r + 2 * c + 1] : make_float2(0.f, 0.f);
      o4 = make_float4(e0.x, e0.y, e1.x, e1.y);
    }
#pragma unroll
    for (int m = 0; m < MATS; ++m) {
      const int base = (r * MATS + m) * 128;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = g + 8 * h;
        const uint32_t s2 = *reinterpret_cast<const uint32_t*>(sc + base + row * 8 + 2 * c);
        const uint32_t b2 = *reinterpret_cast<const uint32_t*>(bi + base + row * 8 + 2 * c);
        const float s0 = bf16_lo(s2), s1 = bf16_hi(s2), b0 = bf16_lo(b2), b1 = bf16_hi(b2);
        float v = res[m][h];
        v = fmaf(s0, acc[m][2 * h] - o4.x, fmaf(b0, o4.y, v));
        v = fmaf(s1, acc[m][2 * h + 1] - o4.z, fmaf(b1, o4.w, v));
        res[m][h] = v;
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MATS; ++m)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float v = res[m][h];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      out[m][h] = v;
    }
}

// ---------------------------------------------------------------- staging
// Sum of squares of x[0..n) over the consumer threads in a fixed order, then
// r = 1/sqrt(mean + eps) in misc->rms (every CTA computes the same value).
__device__ void rms_stat(const __nv_bfloat16* x, int n, float eps, Misc* misc, bool from_l2) {
  const int tid = threadIdx.x;
  float ss = 0.f;
  for (int v = tid; v < n / 8; v += kConsumerThreads) {
    const uint4 w = from_l2 ? ldcg16(x + v * 8) : *reinterpret_cast<const uint4*>(x + v * 8);
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = bf16_lo(u[i]), b = bf16_hi(u[i]);
      ss = fmaf(a, a, ss);
      ss = fmaf(b, b, ss);
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) misc->warp_ss[tid >> 5] = ss;
  named_sync();
  if (tid == 0) {
    float t = 0.f;
    for (int w = 0; w < kConsumers; ++w) t += misc->warp_ss[w];
    misc->rms = 1.0f / sqrtf(t / static_cast<float>(n) + eps);
  }
  named_sync();
}

// 8 activation values of vector v (optionally RMS-normalised and rounded to bf16)
__device__ __forceinline__ void load8(const __nv_bfloat16* x, const __nv_bfloat16* w, float r, int v, bool from_l2,
                                      float (&f)[8]) {
  const uint4 xv = from_l2 ? ldcg16(x + v * 8) : *reinterpret_cast<const uint4*>(x + v * 8);
  const uint32_t u[4] = {xv.x, xv.y, xv.z, xv.w};
  if (w != nullptr) {
    const uint4 wv = *reinterpret_cast<const uint4*>(w + v * 8);
    const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = bfr(bf16_lo(u[i]) * r * bf16_lo(wu[i]));
      f[2 * i + 1] = bfr(bf16_hi(u[i]) * r * bf16_hi(wu[i]));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = bf16_lo(u[i]);
      f[2 * i + 1] = bf16_hi(u[i]);
    }
  }
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  return static_cast<uint32_t>(__half_as_ushort(__float2half_rn(a))) |
         (static_cast<uint32_t>(__half_as_ushort(__float2half_rn(b))) << 16);
}
__device__ __forceinline__ uint32_t pack_b2(float a, float b) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(a))) |
         (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(b))) << 16);
}

// Stage x[0..n) for W8 tiles: fp16 in natural order.
__device__ void stage_w8(const __nv_bfloat16* x, const __nv_bfloat16* w, int n, bool from_l2, float r, uint8_t* xs) {
  for (int v = threadIdx.x; v < n / 8; v += kConsumerThreads) {
    float f[8];
    load8(x, w, r, v, from_l2, f);
    *reinterpret_cast<uint4*>(xs + v * 16) =
        make_uint4(pack_h2(f[0], f[1]), pack_h2(f[2], f[3]), pack_h2(f[4], f[5]), pack_h2(f[6], f[7]));
  }
}

// Stage x[0..n) for BF16 tiles: bf16 in natural order.
__device__ void stage_bf16(const __nv_bfloat16* x, const __nv_bfloat16* w, int n, bool from_l2, float r,
                           uint8_t* xs) {
  for (int v = threadIdx.x; v < n / 8; v += kConsumerThreads) {
    float f[8];
    load8(x, w, r, v, from_l2, f);
    *reinterpret_cast<uint4*>(xs + v * 16) =
        make_uint4(pack_b2(f[0], f[1]), pack_b2(f[2], f[3]), pack_b2(f[4], f[5]), pack_b2(f[6], f[7]));
  }
}

// Stage x[0..n) for W4 tiles: per 8-value word [bf16 (x0,x4) | bf16 (x2,x6) |
// fp16 (x1,x5) | fp16 (x3,x7)], and per group of 64 the offset sum
// O = 128*sum(even) + 64*sum(odd) and X = sum(x) (fixed reduction order).
__device__ void stage_w4(const __nv_bfloat16* x, const __nv_bfloat16* w, int n, bool from_l2, float r, uint8_t* xs,
                         float2* om) {
  // kConsumerThreads is a multiple of 8, so the 8 words of a group sit in 8 consecutive lanes
  for (int v0 = 0; v0 < n / 8; v0 += kConsumerThreads) {
    const int v = v0 + threadIdx.x;
    float O = 0.f, X = 0.f;
    if (v < n / 8) {
      float f[8];
      load8(x, w, r, v, from_l2, f);
      float h[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) h[i] = (i & 1) ? __half2float(__float2half_rn(f[i])) : f[i];
      *reinterpret_cast<uint4*>(xs + v * 16) =
          make_uint4(pack_b2(f[0], f[4]), pack_b2(f[2], f[6]), pack_h2(f[1], f[5]), pack_h2(f[3], f[7]));
      O = 128.f * (((h[0] + h[2]) + h[4]) + h[6]) + 64.f * (((h[1] + h[3]) + h[5]) + h[7]);
#pragma unroll
      for (int i = 0; i < 8; ++i) X += f[i];
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      O += __shfl_xor_sync(0xffffffffu, O, o);
      X += __shfl_xor_sync(0xffffffffu, X, o);
    }
    if (v < n / 8 && (v & 7) == 0) om[v >> 3] = make_float2(O, X);
  }
}

// -------------------------------------------------------------- operators
enum Kind : int { K_W8 = 0, K_W4 = 1, K_W4PAIR = 2, K_BF16 = 3 };
enum Epi : int { E_QKV = 0, E_OPROJ = 1, E_SWIGLU = 2, E_DOWN = 3, E_ARGMAX = 4 };

struct Smem {
  uint64_t* full;
  uint64_t* empty;
  unsigned* rbcnt;
  unsigned* ready;
  const uint8_t* zero;
  Misc* misc;
  float2* om;
  float* part;
  uint8_t* xs;
  uint8_t* ring;
};

// Epilogue of a finished row block: lane r < rows holds the chunk-ordered sum of row r.
template <int EPI>
__device__ void finish_rows(const Params& p, const Layer& L, int rb, float total, int lane, int pos, Misc* misc) {
  if constexpr (EPI == E_QKV) {
    // rows g and g+8 of the block are dims d and d+64 of one head (d = 8*(rb%8) + g)
    const int hd = rb >> 3, i0 = (rb & 7) * 8;
    const float s = L.qkv_scale[rb * 16 + (lane & 15)];
    const float v = bfr(total * s);
    const float partner = __shfl_down_sync(0xffffffffu, v, 8);
    if (lane < 8) {
      const int d = i0 + lane;
      float a = v, b = partner;
      if (hd < p.heads + p.kv_heads) {
        const float angle = static_cast<float>(pos) * p.inv_freq[d];
        float sn, cs;
        sincosf(angle, &sn, &cs);
        const float ra = a * cs - b * sn;
        const float rb2 = b * cs + a * sn;
        a = ra;
        b = rb2;
      }
      __nv_bfloat16* dst;
      if (hd < p.heads) dst = p.q + hd * 128;
      else if (hd < p.heads + p.kv_heads) dst = p.kv_new + (hd - p.heads) * 128;
      else dst = p.kv_new + (p.kv_heads + hd - p.heads - p.kv_heads) * 128;
      dst[d] = __float2bfloat16_rn(a);
      dst[d + 64] = __float2bfloat16_rn(b);
    }
  } else if constexpr (EPI == E_OPROJ) {
    if (lane < 16) {
      const int n = rb * 16 + lane;
      const float v = bfr(total * L.o_scale[n]);
      p.x[n] = __float2bfloat16_rn(ldcg_bf(p.x + n) + v);
    }
  } else if constexpr (EPI == E_SWIGLU) {
    const float v = bfr(total);
    const float up = __shfl_down_sync(0xffffffffu, v, 16);
    if (lane < 16) {
      const float silu = v / (1.0f + expf(-v));
      p.act[rb * 16 + lane] = __float2bfloat16_rn(silu * up);
    }
  } else if constexpr (EPI == E_DOWN) {
    if (lane < 16) {
      const int n = rb * 16 + lane;
      p.x[n] = __float2bfloat16_rn(ldcg_bf(p.x + n) + bfr(total));
    }
  } else {  // E_ARGMAX
    const int n = rb * 16 + lane;
    unsigned long long key = (lane < 16 && n < p.vocab) ? argmax_key(total, n + p.vocab_offset) : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
      key = k2 > key ? k2 : key;
    }
    if (lane == 0 && key) atomicMax(&misc->key, key);
  }
}

// One operator over this CTA's share of a weight stream.
template <int KIND, int EPI>
__device__ void run_op(const Params& p, const Layer& L, const Smem& s, const Stream& st, const uint8_t* stream,
                       uint32_t& seq, int pos) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int W = gridDim.x, cta = blockIdx.x;
  const int T = st.rbs * st.chunks;
  const int t0 = static_cast<int>((static_cast<long long>(T) * cta) / W);
  const int t1 = static_cast<int>((static_cast<long long>(T) * (cta + 1)) / W);
  constexpr int kRows = (KIND == K_W4PAIR) ? 32 : 16;
  // reset the partial-slot gates for this operator
  for (int i = threadIdx.x; i < kPartSlots; i += kConsumerThreads) s.ready[i] = i;
  named_sync();
  const int rb_first = t0 / max(st.chunks, 1);
  for (int t = t0; t < t1; ++t) {
    const uint32_t q = seq + static_cast<uint32_t>(t - t0);
    if (static_cast<int>(q % kConsumers) != warp) continue;
    if (*reinterpret_cast<volatile int*>(&s.misc->abort)) break;
    const int slot = static_cast<int>(q % static_cast<uint32_t>(p.slots));
    if (!wait_bar(s.full + slot, (q / static_cast<uint32_t>(p.slots)) & 1u, p, s.misc)) break;
    const uint8_t* tile = s.ring + static_cast<size_t>(slot) * p.slot_bytes;
    const int rb = t / st.chunks, ch = t % st.chunks;
    float vals[2][2];
    if constexpr (KIND == K_W8) {
      w8_tile(tile, s.xs + ch * st.ck * 2, st.ck / 32, lane, vals[0][0], vals[0][1]);
    } else if constexpr (KIND == K_BF16) {
      bf16_tile(tile, s.xs + ch * st.ck * 2, st.ck / 16, lane, vals[0][0], vals[0][1]);
    } else if constexpr (KIND == K_W4) {
      float o[1][2];
      w4_tile<1>(tile, st.ck, s.xs + ch * st.ck * 128, s.om + ch * st.ck, s.zero, lane, o);
      vals[0][0] = o[0][0];
      vals[0][1] = o[0][1];
    } else {
      w4_tile<2>(tile, st.ck, s.xs + ch * st.ck * 128, s.om + ch * st.ck, s.zero, lane, vals);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(s.empty + slot);
    // partials of this tile into its slot (after the slot's previous tile was consumed)
    const int li = t - t0;
    const int ps = li % kPartSlots;
    if (lane == 0) {
      const long long start = clock64();
      while (static_cast<int>(*reinterpret_cast<volatile unsigned*>(s.ready + ps)) < li) {
        if (clock64() - start > (1LL << 31)) {
          atomicOr(p.status, kStatusTimeout);
          s.misc->abort = 1;
          break;
        }
      }
    }
    __syncwarp();
    float* part = s.part + ps * 32;
    const int g = lane >> 2;
    if ((lane & 3) == 0) {
      part[g] = vals[0][0];
      part[g + 8] = vals[0][1];
      if constexpr (kRows == 32) {
        part[16 + g] = vals[1][0];
        part[16 + g + 8] = vals[1][1];
      }
    }
    __threadfence_block();
    __syncwarp();
    // local tiles of this row block inside [t0, t1)
    const int cl0 = max(rb * st.chunks, t0), cl1 = min((rb + 1) * st.chunks, t1);
    const int need = cl1 - cl0;
    unsigned done = 0;
    const int rslot = (rb - rb_first) % kRbSlots;
    if (lane == 0) done = atomicAdd(s.rbcnt + rslot, 1u) + 1u;
    done = __shfl_sync(0xffffffffu, done, 0);
    if (static_cast<int>(done) != need) continue;
    // ---- this warp finishes the row block
    __threadfence_block();
    if (lane == 0) s.rbcnt[rslot] = 0u;
    const bool split = need != st.chunks;
    bool last = true;
    if (split) {
      // publish the local chunk partials; the CTA that brings the row block's count to `chunks` finishes it
      float* gp = p.gpart + static_cast<size_t>(rb) * kChunks * 32;
      for (int c = cl0; c < cl1; ++c) {
        const float v = s.part[((c - t0) % kPartSlots) * 32 + lane];
        if (lane < kRows) gp[(c - rb * st.chunks) * 32 + lane] = v;
      }
      __threadfence();
      __syncwarp();
      unsigned old = 0;
      if (lane == 0) old = atomicAdd(p.gcount + rb, static_cast<unsigned>(need));
      old = __shfl_sync(0xffffffffu, old, 0);
      last = static_cast<int>(old) + need == st.chunks;
      if (last) __threadfence();
    }
    float total = 0.f;
    if (last) {
      for (int c = 0; c < st.chunks; ++c) {
        const int gc = rb * st.chunks + c;
        float v;
        if (gc >= cl0 && gc < cl1) v = s.part[((gc - t0) % kPartSlots) * 32 + lane];
        else v = ldcg_f(p.gpart + (static_cast<size_t>(rb) * kChunks + c) * 32 + lane);
        total += v;  // chunk order
      }
      if (split && lane == 0) p.gcount[rb] = 0u;
    }
    // release the partial slots of this row block's local tiles
    __syncwarp();
    if (lane == 0) {
      for (int c = cl0; c < cl1; ++c) {
        const int l = c - t0;
        s.ready[l % kPartSlots] = static_cast<unsigned>(l + kPartSlots);
      }
    }
    if (last) finish_rows<EPI>(p, L, rb, total, lane, pos, s.misc);
  }
  seq += static_cast<uint32_t>(t1 - t0);
}

// ------------------------------------------------------------- attention
// INT8-KV attention of the new token (position pos) for every (KV head,
// 128-token chunk) work item, one warp per item; the items of a KV head are
// merged in chunk order by the warp that completes the last one. The warp
// holding the newest position quantizes the new K/V row into the cache
// (symmetric per token per head, fp16 scale = absmax / 127).
template <int G>
__device__ void attention_items(const Params& p, const Layer& L, int pos, float* qs_all) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = pos + 1;
  const int nchunks = (n + kAttnChunk - 1) / kAttnChunk;
  const int items = p.kv_heads * nchunks;
  const int gw = blockIdx.x * kConsumers + warp;
  const int stride = gridDim.x * kConsumers;
  float* qs = qs_all + warp * G * 128;
  const size_t cap = static_cast<size_t>(p.capacity);
  for (int item = gw; item < items; item += stride) {
    const int h = item / nchunks, ck = item % nchunks;
    const int tb = ck * kAttnChunk;
    // queries of the G heads sharing KV head h (fp32 in shared memory)
    for (int i = lane; i < G * 128; i += 32) qs[i] = ldcg_bf(p.q + (h * G) * 128 + i);
    int8_t* kc = L.k_cache + static_cast<size_t>(h) * cap * 128;
    int8_t* vc = L.v_cache + static_cast<size_t>(h) * cap * 128;
    __half* ksc = L.k_scale + static_cast<size_t>(h) * cap;
    __half* vsc = L.v_scale + static_cast<size_t>(h) * cap;
    if (pos >= tb && pos < tb + kAttnChunk) {
      // the new token's row: quantize K and V into the cache
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const __nv_bfloat16* src = p.kv_new + (which * p.kv_heads + h) * 128;
        float v4[4];
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          v4[i] = ldcg_bf(src + lane * 4 + i);
          amax = fmaxf(amax, fabsf(v4[i]));
        }
        amax = warp_max(amax);
        __half s16 = __float2half_rn(__fdiv_rn(amax, 127.0f));
        if (__half2float(s16) == 0.f) s16 = __float2half_rn(1.0f);
        const float sf = __half2float(s16);
        char4 q4;
        int8_t* qq = reinterpret_cast<int8_t*>(&q4);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float rr = fminf(fmaxf(rintf(__fdiv_rn(v4[i], sf)), -127.f), 127.f);
          qq[i] = static_cast<int8_t>(static_cast<int>(rr));
        }
        int8_t* dst = (which ? vc : kc) + static_cast<size_t>(pos) * 128;
        *reinterpret_cast<char4*>(dst + lane * 4) = q4;
        if (lane == 0) (which ? vsc : ksc)[pos] = s16;
      }
      __syncwarp();
      __threadfence_block();
    }
    __syncwarp();
    // scores: lane owns tokens tb + lane + 32*i
    float sc[4][G];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = tb + lane + 32 * i;
#pragma unroll
      for (int hh = 0; hh < G; ++hh) sc[i][hh] = -INFINITY;
      if (t < n) {
        const int8_t* krow = kc + static_cast<size_t>(t) * 128;
        float dot[G];
#pragma unroll
        for (int hh = 0; hh < G; ++hh) dot[hh] = 0.f;
#pragma unroll
        for (int seg = 0; seg < 8; ++seg) {
          const uint4 kv = (t == pos) ? ldcg16(krow + seg * 16) : *reinterpret_cast<const uint4*>(krow + seg * 16);
          const int8_t* kb = reinterpret_cast<const int8_t*>(&kv);
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float kf = static_cast<float>(kb[e]);
#pragma unroll
            for (int hh = 0; hh < G; ++hh) dot[hh] = fmaf(qs[hh * 128 + seg * 16 + e], kf, dot[hh]);
          }
        }
        const float ks = __half2float(t == pos ? __ushort_as_half(__ldcg(reinterpret_cast<const unsigned short*>(ksc + t)))
                                               : ksc[t]);
#pragma unroll
        for (int hh = 0; hh < G; ++hh) sc[i][hh] = dot[hh] * ks * p.attn_scale;
      }
    }
    float m[G], l[G];
#pragma unroll
    for (int hh = 0; hh < G; ++hh) {
      float mx = fmaxf(fmaxf(sc[0][hh], sc[1][hh]), fmaxf(sc[2][hh], sc[3][hh]));
      m[hh] = warp_max(mx);
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sc[i][hh] = (sc[i][hh] == -INFINITY) ? 0.f : expf(sc[i][hh] - m[hh]);
        sum += sc[i][hh];
      }
      l[hh] = warp_sum(sum);
    }
    // P.V: lane owns dims 4*lane .. 4*lane+3
    float acc[G][4];
#pragma unroll
    for (int hh = 0; hh < G; ++hh) acc[hh][0] = acc[hh][1] = acc[hh][2] = acc[hh][3] = 0.f;
    const int tend = min(n - tb, kAttnChunk);
    for (int tt = 0; tt < tend; ++tt) {
      const int t = tb + tt;
      const int owner = tt & 31, idx = tt >> 5;
      const char4 v4 = (t == pos) ? *reinterpret_cast<const char4*>(&reinterpret_cast<const int*>(vc + static_cast<size_t>(t) * 128)[lane])
                                  : reinterpret_cast<const char4*>(vc + static_cast<size_t>(t) * 128)[lane];
      const float vs = __half2float(vsc[t]);
      float pv[G];
#pragma unroll
      for (int hh = 0; hh < G; ++hh) {
        float pt = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float cand = __shfl_sync(0xffffffffu, sc[i][hh], owner);
          if (i == idx) pt = cand;
        }
        pv[hh] = pt * vs;
      }
      const float vf[4] = {static_cast<float>(v4.x), static_cast<float>(v4.y), static_cast<float>(v4.z),
                           static_cast<float>(v4.w)};
#pragma unroll
      for (int hh = 0; hh < G; ++hh)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[hh][e] = fmaf(pv[hh], vf[e], acc[hh][e]);
    }
    // partial of this item
    float* ap = p.apart + (static_cast<size_t>(h) * p.attn_max_chunks + ck) * G * 132;
#pragma unroll
    for (int hh = 0; hh < G; ++hh) {
      *reinterpret_cast<float4*>(ap + hh * 132 + lane * 4) = make_float4(acc[hh][0], acc[hh][1], acc[hh][2], acc[hh][3]);
      if (lane == 0) {
        ap[hh * 132 + 128] = m[hh];
        ap[hh * 132 + 129] = l[hh];
      }
    }
    __threadfence();
    __syncwarp();
    unsigned old = 0;
    if (lane == 0) old = atomicAdd(p.acount + h, 1u);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (static_cast<int>(old) + 1 != nchunks) continue;
    // ---- last item of KV head h: merge the chunks in order
    __threadfence();
    if (lane == 0) p.acount[h] = 0u;
    const float* base = p.apart + static_cast<size_t>(h) * p.attn_max_chunks * G * 132;
#pragma unroll
    for (int hh = 0; hh < G; ++hh) {
      float M = -INFINITY;
      for (int c = 0; c < nchunks; ++c) M = fmaxf(M, ldcg_f(base + (c * G + hh) * 132 + 128));
      float Lsum = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
      for (int c = 0; c < nchunks; ++c) {
        const float* e = base + (c * G + hh) * 132;
        const float w = expf(ldcg_f(e + 128) - M);
        Lsum = fmaf(ldcg_f(e + 129), w, Lsum);
        const float4 a = __ldcg(reinterpret_cast<const float4*>(e + lane * 4));
        o[0] = fmaf(a.x, w, o[0]);
        o[1] = fmaf(a.y, w, o[1]);
        o[2] = fmaf(a.z, w, o[2]);
        o[3] = fmaf(a.w, w, o[3]);
      }
      const float inv = Lsum > 0.f ? 1.0f / Lsum : 0.f;
      __nv_bfloat16* dst = p.attn + (h * G + hh) * 128 + lane * 4;
#pragma unroll
      for (int e = 0; e < 4; ++e) dst[e] = __float2bfloat16_rn(o[e] * inv);
    }
  }
}

// --------------------------------------------------------------- producer
__device__ void produce_op(const Params& p, const Smem& s, const Stream& st, const uint8_t* stream, uint32_t& seq,
                           uint64_t pol) {
  const int W = gridDim.x, cta = blockIdx.x;
  const int T = st.rbs * st.chunks;
  const int t0 = static_cast<int>((static_cast<long long>(T) * cta) / W);
  const int t1 = static_cast<int>((static_cast<long long>(T) * (cta + 1)) / W);
  for (int t = t0; t < t1; ++t, ++seq) {
    if (*reinterpret_cast<volatile int*>(&s.misc->abort)) return;
    const int slot = static_cast<int>(seq % static_cast<uint32_t>(p.slots));
    const uint32_t use = seq / static_cast<uint32_t>(p.slots);
    if (use > 0 && !wait_bar(s.empty + slot, (use - 1) & 1u, p, s.misc)) return;
    mbar_arrive_expect_tx(s.full + slot, static_cast<uint32_t>(st.tile));
    bulk_g2s_hint(s.ring + static_cast<size_t>(slot) * p.slot_bytes, stream + static_cast<size_t>(t) * st.tile,
                  static_cast<uint32_t>(st.tile), s.full + slot, pol);
  }
}

__global__ void __maxnreg__(160) step_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  Smem s;
  s.full = reinterpret_cast<uint64_t*>(base + kOffBars);
  s.empty = s.full + kMaxSlots;
  s.rbcnt = reinterpret_cast<unsigned*>(base + kOffRbCnt);
  s.ready = reinterpret_cast<unsigned*>(base + kOffReady);
  s.zero = base + kOffZero;
  s.misc = reinterpret_cast<Misc*>(base + kOffMisc);
  s.om = reinterpret_cast<float2*>(base + kOffMeta);
  s.part = reinterpret_cast<float*>(base + kOffPart);
  s.xs = base + kOffXs;
  s.ring = base + kOffRing;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.slots; ++i) {
      mbar_init(s.full + i, 1);
      mbar_init(s.empty + i, 1);
    }
    mbar_fence_init();
    s.misc->abort = 0;
    s.misc->key = 0ull;
  }
  for (int i = threadIdx.x; i < kRbSlots; i += blockDim.x) s.rbcnt[i] = 0u;
  for (int i = threadIdx.x; i < 64; i += blockDim.x) reinterpret_cast<uint32_t*>(base + kOffZero)[i] = 0u;
  __syncthreads();

  const int pos = p.positions[0];
  if (warp == kConsumers) {
    // ---------------- producer warp (one lane issues)
    if (lane == 0) {
      const uint64_t pol = evict_first_policy();
      uint32_t seq = 0;
      for (int l = 0; l < p.num_layers; ++l) {
        const Layer& L = p.layers[l];
        produce_op(p, s, p.sq, L.qkv, seq, pol);
        produce_op(p, s, p.so, L.o, seq, pol);
        produce_op(p, s, p.sgu, L.gateup, seq, pol);
        produce_op(p, s, p.sdn, L.down, seq, pol);
      }
      produce_op(p, s, p.slm, p.head, seq, pol);
      // no copy may be in flight when the CTA exits: wait for the last issued ones
      const uint32_t nslots = static_cast<uint32_t>(p.slots);
      for (uint32_t q = seq > nslots ? seq - nslots : 0u; q < seq; ++q) {
        const int slot = static_cast<int>(q % nslots);
        if (!mbar_wait_bounded(s.full + slot, (q / nslots) & 1u)) atomicOr(p.status, kStatusTimeout);
      }
    }
    return;
  }

  // ---------------- consumer warps
  const int W = gridDim.x;
  const int token = p.tokens[0];
  const __nv_bfloat16* emb = p.embed + static_cast<size_t>(min(max(token, 0), p.vocab_total - 1)) * p.hidden;
  if (blockIdx.x == 0) {
    for (int v = threadIdx.x; v < p.hidden / 8; v += kConsumerThreads)
      reinterpret_cast<uint4*>(p.x)[v] = reinterpret_cast<const uint4*>(emb)[v];
  }
  uint32_t seq = 0;
  unsigned joins = 0;
  const int G = p.heads / p.kv_heads;
  for (int l = 0; l < p.num_layers; ++l) {
    const Layer& L = p.layers[l];
    // RMSNorm + QKV + RoPE
    const bool first = l == 0;
    const __nv_bfloat16* xin = first ? emb : p.x;
    rms_stat(xin, p.hidden, p.eps, s.misc, !first);
    stage_w8(xin, L.in_norm, p.hidden, !first, s.misc->rms, s.xs);
    named_sync();
    run_op<K_W8, E_QKV>(p, L, s, p.sq, L.qkv, seq, pos);
    grid_join(p, s.misc, (++joins) * W);
    // attention (q/k/v of all heads are final)
    float* qs = reinterpret_cast<float*>(base + kOffPart);
    switch (G) {
      case 1: attention_items<1>(p, L, pos, qs); break;
      case 2: attention_items<2>(p, L, pos, qs); break;
      case 4: attention_items<4>(p, L, pos, qs); break;
      default: attention_items<8>(p, L, pos, qs); break;
    }
    grid_join(p, s.misc, (++joins) * W);
    // o_proj + residual
    stage_w8(p.attn, nullptr, p.heads * 128, true, 1.f, s.xs);
    named_sync();
    run_op<K_W8, E_OPROJ>(p, L, s, p.so, L.o, seq, pos);
    grid_join(p, s.misc, (++joins) * W);
    // RMSNorm + gate/up + SwiGLU
    rms_stat(p.x, p.hidden, p.eps, s.misc, true);
    stage_w4(p.x, L.post_norm, p.hidden, true, s.misc->rms, s.xs, s.om);
    named_sync();
    run_op<K_W4PAIR, E_SWIGLU>(p, L, s, p.sgu, L.gateup, seq, pos);
    grid_join(p, s.misc, (++joins) * W);
    // down + residual
    stage_w4(p.act, nullptr, p.inter, true, 1.f, s.xs, s.om);
    named_sync();
    run_op<K_W4, E_DOWN>(p, L, s, p.sdn, L.down, seq, pos);
    grid_join(p, s.misc, (++joins) * W);
  }
  // final RMSNorm + lm_head + greedy argmax
  rms_stat(p.x, p.hidden, p.eps, s.misc, true);
  stage_bf16(p.x, p.final_norm, p.hidden, true, s.misc->rms, s.xs);
  named_sync();
  run_op<K_BF16, E_ARGMAX>(p, p.layers[0], s, p.slm, p.head, seq, pos);
  named_sync();
  if (threadIdx.x == 0 && s.misc->key) atomicMax(p.keys, s.misc->key);
}

// ------------------------------------------------------------------- host
struct Geometry {
  Stream sq, so, sgu, sdn, slm;
  int max_rbs;
  int attn_chunks;
  size_t ws_bytes;
  int slot_bytes;
};

int geometry(const sb_step_desc* d, Geometry* g) {
  SB_REQUIRE(d != nullptr, "null descriptor");
  SB_REQUIRE(d->head_dim == 128, "the decode-step kernel supports head_dim 128");
  SB_REQUIRE(d->world == 1 && d->rank == 0, "the decode-step kernel in this build runs one rank");
  SB_REQUIRE(d->num_layers > 0 && d->num_layers <= kMaxLayers, "1..128 layers");
  SB_REQUIRE(d->hidden > 0 && d->hidden % 512 == 0 && d->hidden <= kMaxK, "hidden must be a multiple of 512, <= 10240");
  SB_REQUIRE(d->num_heads > 0 && d->num_kv_heads > 0 && d->num_heads % d->num_kv_heads == 0, "heads");
  const int G = d->num_heads / d->num_kv_heads;
  SB_REQUIRE(G == 1 || G == 2 || G == 4 || G == 8, "query heads per KV head must be 1, 2, 4 or 8");
  const int qk = d->num_heads * 128;  // o_proj K (this rank)
  SB_REQUIRE(qk <= kMaxK && qk % (kChunks * 32 / d->world) == 0, "o_proj K must split into 8 chunks of 32-multiples");
  SB_REQUIRE(d->inter > 0 && d->inter % 16 == 0 && d->inter <= kMaxK, "inter must be a multiple of 16, <= 10240");
  SB_REQUIRE(d->inter_total % (kChunks * 64) == 0, "intermediate size must be a multiple of 512");
  SB_REQUIRE(d->vocab > 0 && d->capacity > 0 && d->capacity % 16 == 0, "vocab and capacity");
  SB_REQUIRE(d->hidden % (kChunks * 16) == 0, "hidden must split into 8 chunks of 16-multiples");
  g->sq = {(d->num_heads + 2 * d->num_kv_heads) * 128 / 16, d->hidden / 512, 16 * 512, 512};
  const int ock = qk / (kChunks / d->world);
  g->so = {d->hidden / 16, kChunks / d->world, 16 * ock, ock};
  g->sgu = {d->inter / 16, d->hidden / 512, 2 * 16 * 8 * 32 + 2 * 2 * 128 * 2, 8};
  const int dg = d->inter_total / 64 / kChunks;  // groups per down chunk
  const int drounds = (dg + 7) / 8;
  g->sdn = {d->hidden / 16, kChunks / d->world, 16 * dg * 32 + 2 * drounds * 128 * 2, dg};
  const int lck = d->hidden / kChunks;
  g->slm = {(d->vocab + 15) / 16, kChunks, 16 * lck * 2, lck};
  int tmax = 0;
  for (const Stream* st : {&g->sq, &g->so, &g->sgu, &g->sdn, &g->slm}) tmax = tmax > st->tile ? tmax : st->tile;
  g->slot_bytes = (tmax + 127) / 128 * 128;
  g->max_rbs = std::max({g->sq.rbs, g->so.rbs, g->sgu.rbs, g->sdn.rbs, g->slm.rbs});
  g->attn_chunks = (d->capacity + kAttnChunk - 1) / kAttnChunk;
  size_t off = 256;  // header words
  off += static_cast<size_t>(g->max_rbs) * 4;  // gcount
  off = (off + 255) / 256 * 256;
  off += 64 * 4;  // acount
  off = (off + 255) / 256 * 256;
  off += static_cast<size_t>(g->max_rbs) * kChunks * 32 * 4;  // gpart
  off += static_cast<size_t>(d->num_kv_heads) * g->attn_chunks * G * 132 * 4;  // apart
  g->ws_bytes = off;
  return SB_OK;
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

}  // namespace step
}  // namespace sb

using namespace sb;
using namespace sb::step;

extern "C" size_t sb_step_workspace_size(const sb_step_desc* d) {
  Geometry g;
  if (geometry(d, &g) != SB_OK) return 0;
  return g.ws_bytes;
}

extern "C" int sb_step_tile_bytes(const sb_step_desc* d, int64_t out[5]) {
  Geometry g;
  if (int st = geometry(d, &g)) return st;
  out[0] = g.sq.tile;
  out[1] = g.so.tile;
  out[2] = g.sgu.tile;
  out[3] = g.sdn.tile;
  out[4] = g.slm.tile;
  return SB_OK;
}

extern "C" int sb_step_run(const sb_step_desc* d, void* stream) {
  Geometry g;
  if (int st = geometry(d, &g)) return st;
  SB_REQUIRE(d->workspace != nullptr && d->workspace_bytes >= g.ws_bytes, "workspace too small");
  SB_REQUIRE(d->layers && d->embed && d->head && d->final_norm && d->tokens && d->positions && d->x && d->q &&
                 d->kv_new && d->attn && d->act && d->argmax_key,
             "null pointer in the step descriptor");
  Params p{};
  p.layers = reinterpret_cast<const Layer*>(d->layers);
  p.num_layers = d->num_layers;
  p.hidden = d->hidden;
  p.heads = d->num_heads;
  p.kv_heads = d->num_kv_heads;
  p.inter = d->inter;
  p.vocab = d->vocab;
  p.vocab_offset = d->vocab_offset;
  p.capacity = d->capacity;
  p.vocab_total = d->vocab_total;
  p.eps = d->rms_eps;
  p.attn_scale = 1.0f / std::sqrt(128.0f);
  for (int i = 0; i < 64; ++i)
    p.inv_freq[i] = static_cast<float>(std::pow(static_cast<double>(d->rope_theta), -2.0 * i / 128.0));
  p.embed = static_cast<const __nv_bfloat16*>(d->embed);
  p.head = static_cast<const uint8_t*>(d->head);
  p.final_norm = static_cast<const __nv_bfloat16*>(d->final_norm);
  p.tokens = d->tokens;
  p.positions = d->positions;
  p.x = static_cast<__nv_bfloat16*>(d->x);
  p.q = static_cast<__nv_bfloat16*>(d->q);
  p.kv_new = static_cast<__nv_bfloat16*>(d->kv_new);
  p.attn = static_cast<__nv_bfloat16*>(d->attn);
  p.act = static_cast<__nv_bfloat16*>(d->act);
  p.keys = d->argmax_key;
  unsigned* ws = static_cast<unsigned*>(d->workspace);
  p.sync = ws;
  p.status = ws + 1;
  uint8_t* wb = static_cast<uint8_t*>(d->workspace);
  size_t off = 256;
  p.gcount = reinterpret_cast<unsigned*>(wb + off);
  off += static_cast<size_t>(g.max_rbs) * 4;
  off = (off + 255) / 256 * 256;
  p.acount = reinterpret_cast<unsigned*>(wb + off);
  off += 64 * 4;
  off = (off + 255) / 256 * 256;
  p.gpart = reinterpret_cast<float*>(wb + off);
  off += static_cast<size_t>(g.max_rbs) * kChunks * 32 * 4;
  p.apart = reinterpret_cast<float*>(wb + off);
  p.attn_max_chunks = g.attn_chunks;
  p.sq = g.sq;
  p.so = g.so;
  p.sgu = g.sgu;
  p.sdn = g.sdn;
  p.slm = g.slm;
  p.slot_bytes = g.slot_bytes;
  int max_smem = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const int fixed = kOffRing + 1024;  // + alignment slack
  p.slots = std::min(kMaxSlots, (max_smem - fixed) / g.slot_bytes);
  SB_REQUIRE(p.slots >= 4, "not enough shared memory for the weight ring");
  const size_t smem = static_cast<size_t>(fixed) + static_cast<size_t>(p.slots) * g.slot_bytes;
  static std::once_flag attr_once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once, [&] {
    attr_err = cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
    if (attr_err == cudaSuccess)
      attr_err = cudaFuncSetAttribute(step_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                      cudaSharedmemCarveoutMaxShared);
  });
  if (attr_err != cudaSuccess) return fail(SB_ECUDA, std::string("step kernel attribute: ") + cudaGetErrorString(attr_err));
  {
    // every CTA must be resident at once (grid-wide joins): one per SM
    int per_sm = 0;
    cudaError_t oe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, step_kernel, kThreads, smem);
    if (oe != cudaSuccess || per_sm < 1) {
      cudaFuncAttributes fa{};
      cudaFuncGetAttributes(&fa, step_kernel);
      return fail(SB_ECUDA, "decode step kernel does not fit on an SM (" + std::to_string(per_sm) +
                                " per SM; " + std::to_string(fa.numRegs) + " registers x " +
                                std::to_string(kThreads) + " threads, max threads " +
                                std::to_string(fa.maxThreadsPerBlock) + ", " + std::to_string(smem) +
                                " B dynamic + " + std::to_string(fa.sharedSizeBytes) + " B static shared memory)");
    }
  }
  // the arrival counter starts at zero for every step
  cudaError_t err = cudaMemsetAsync(d->workspace, 0, 4, as_stream(stream));
  if (err != cudaSuccess) return fail(SB_ECUDA, std::string("step counter reset: ") + cudaGetErrorString(err));
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(static_cast<unsigned>(sm_count()));
  config.blockDim = dim3(kThreads);
  config.dynamicSmemBytes = smem;
  config.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  config.attrs = attr;
  config.numAttrs = 1;
  err = cudaLaunchKernelEx(&config, step_kernel, p);
  if (err != cudaSuccess) return fail(SB_ECUDA, std::string("decode step launch: ") + cudaGetErrorString(err));
  return SB_OK;
}
