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
constexpr int kMaxHidden = 4096;             // residual stream kept in shared memory
constexpr int kMaxGroups = kMaxK / 64;
constexpr int kChunks = 8;                   // K chunks of o/down/lm_head (tensor-parallel unit)
constexpr int kAttnChunk = 16;               // tokens of an attention slice (one warp)
constexpr int kAttnRbk = kAttnChunk / 16;    // 16-token MMA row blocks per slice
constexpr int kMaxLayers = 128;
constexpr unsigned kStatusRange = 2u;        // status bit: position outside the KV cache
// Workspace header (zeroed before every launch): word 0 the grid arrival
// counter; words [64, 128) QKV tiles finished per head (stream order),
// [128, 192) attention finished per KV head (layer + 1), [192, 256) gate/up
// tiles finished per down K chunk. After the header, a persistent block that
// launches do not zero: word 0 the status (sticky until the caller clears it).
constexpr int kHdrQkv = 64, kHdrAttn = 128, kHdrGu = 192;
constexpr int kMaxCtas = 256;
constexpr size_t kHdrBytes = 1024;
constexpr size_t kPersistBytes = 256;
static_assert(kHdrBytes == SB_STEP_STATUS_OFFSET, "status word offset");
constexpr int kMarksPerLayer = 9;  // trace marks per layer
constexpr int kAttnMarks = 4;      // extra trace marks per layer inside an attention item
constexpr int kTlEvents = 96;      // timeline events per consumer warp (one traced layer)
constexpr int kTlSlots = kConsumers * kTlEvents / 2;  // trace slots (4 x u64) holding the timeline

// shared-memory layout (offsets from a 1024-byte aligned base)
constexpr int kOffBars = 0;            // full[16], empty[16]
constexpr int kOffRbCnt = 256;         // u32 [128]
constexpr int kOffReady = 768;         // u32 [64]: next tile index allowed into a partial slot
constexpr int kOffZero = 1024;         // 256 zero bytes
constexpr int kOffMisc = 1280;         // abort, rms, key, warp sums
constexpr int kOffMeta = 2048;         // float2 [kMaxGroups] (O, X) per staged group
constexpr int kOffXres = ((kOffMeta + kMaxGroups * 8 + 255) / 256) * 256;  // bf16 [kMaxHidden] residual stream
constexpr int kOffPart = kOffXres + kMaxHidden * 2;                // float [64][32] (lm_head partials)
constexpr int kOffXs = kOffPart + kPartSlots * 32 * 4;             // staged activations
constexpr int kOffRing = ((kOffXs + kMaxK * 2 + 1023) / 1024) * 1024;
// attention scratch (aliases part + xs, unused during attention): q of the
// G heads as fp16 [4][128], then per warp its partial [4 heads][132] floats
// (the warp's probabilities [32][4] live there until the partial is written)
static_assert(kOffPart + 1024 + kConsumers * 4 * 132 * 4 + (kConsumers + 2) * 4 * 4 <= kOffRing, "attention scratch");

struct Misc {
  int abort;
  float rms;
  unsigned long long key;
  float warp_ss[kConsumers];
  int last;                    // attention: this CTA merges the KV head's spans
  unsigned long long wait_ns;  // tracing: consumer time waiting for tiles (sum over warps)
  unsigned long long busy_ns;  // tracing: consumer time computing tiles
  int tl_on;                   // tracing: this layer's events go to the per-warp timeline
  unsigned tl_n[kConsumers];   // tracing: timeline events recorded per consumer warp
};
static_assert(sizeof(Misc) <= 768, "misc block");

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
  unsigned* status;   // persistent word 0 (after the header)
  unsigned* hdr;      // workspace header words (per-head / per-chunk progress counters)
  unsigned* gcount;   // lm_head: counters of row blocks split between CTAs
  unsigned* acount;   // attention per-KV-head counters
  float* gpart;       // lm_head: split row-block partials [rb][kChunks][32]
  float* apart;       // attention partials [kv head][chunk][G][132]
  // per-chunk partial sums of the projections (L2): [row][8] (gate/up: [row][2][8])
  float* pqkv;
  float* po;
  float* pgu;
  float* pdn;
  int attn_max_chunks;
  Stream sq, so, sgu, sdn, slm;
  int slot_bytes, slots;
  unsigned long long* trace;  // optional [CTA][trace_slots][2] globaltimer stamps
  int trace_slots;
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

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Release-ordered add (this thread's earlier writes, and those ordered before
// them by a barrier, are visible to whoever observes the new value).
__device__ __forceinline__ void red_release_add(unsigned* addr, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* addr) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_volatile_u32(unsigned* addr, unsigned v) {
  asm volatile("st.volatile.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

// Bounded wait until *addr >= target (another CTA's progress). The load that
// observes the target is an acquire at GPU scope: the waiting thread's later
// loads, and those of the threads it releases through a CTA barrier, see the
// writes ordered before the matching release (the other CTA's red.release).
// On timeout, or when another CTA has already recorded a failure, records it
// and raises the CTA's abort flag.
__device__ bool spin_geq(const Params& p, Misc* misc, const unsigned* addr, unsigned target) {
  if (*reinterpret_cast<volatile int*>(&misc->abort)) return false;
  if (ld_acquire_u32(addr) < target) {
    const long long start = clock64();
    while (ld_acquire_u32(addr) < target) {
      if (clock64() - start > (1LL << 31) || ld_volatile_u32(p.status) != 0u) {
        atomicOr(p.status, kStatusTimeout);
        *reinterpret_cast<volatile int*>(&misc->abort) = 1;
        return false;
      }
    }
  }
  return true;
}

// Bounded wait until the QKV progress counters of KV head h's G query heads -
// and, when `with_kv`, of its new K and V rows - are all >= target, polling
// them together (acquire loads); same failure handling as spin_geq.
template <int G>
__device__ bool spin_heads(const Params& p, Misc* misc, int h, bool with_kv, unsigned target) {
  if (*reinterpret_cast<volatile int*>(&misc->abort)) return false;
  const unsigned* q0 = p.hdr + kHdrQkv + G * h;
  const unsigned* kq = p.hdr + kHdrQkv + p.heads + h;
  const unsigned* vq = kq + p.kv_heads;
  const long long start = clock64();
  while (true) {
    unsigned v[G + 2];
#pragma unroll
    for (int i = 0; i < G; ++i) v[i] = ld_acquire_u32(q0 + i);
    v[G] = with_kv ? ld_acquire_u32(kq) : target;
    v[G + 1] = with_kv ? ld_acquire_u32(vq) : target;
    bool ok = true;
#pragma unroll
    for (int i = 0; i < G + 2; ++i) ok = ok && v[i] >= target;
    if (ok) return true;
    if (clock64() - start > (1LL << 31) || ld_volatile_u32(p.status) != 0u) {
      atomicOr(p.status, kStatusTimeout);
      *reinterpret_cast<volatile int*>(&misc->abort) = 1;
      return false;
    }
  }
}

// Tracing (thread 0): mark `slot` of this CTA with (t0, t1) and the tile
// wait/compute time accumulated since the previous mark.
__device__ void trace_mark(const Params& p, Misc* misc, int slot, unsigned long long t0, unsigned long long t1) {
  if (p.trace == nullptr || slot >= p.trace_slots) return;
  unsigned long long* tr = p.trace + (static_cast<size_t>(blockIdx.x) * p.trace_slots + slot) * 4;
  tr[0] = t0;
  tr[1] = t1;
  tr[2] = misc->wait_ns;
  tr[3] = misc->busy_ns;
  misc->wait_ns = 0;
  misc->busy_ns = 0;
}
// Timeline event (tracing, layer num_layers / 2 only): lane 0 of a consumer warp
// records (code, aux) with the SM clock; the analysis reads it per CTA and warp.
__device__ __forceinline__ void tl_event(const Params& p, const Misc* misc, int code, int aux = 0) {
  if (p.trace == nullptr) return;
  if ((threadIdx.x & 31) != 0 || !misc->tl_on) return;
  const int warp = threadIdx.x >> 5;
  Misc* m = const_cast<Misc*>(misc);
  const unsigned i = m->tl_n[warp]++;
  if (i >= static_cast<unsigned>(kTlEvents)) return;
  unsigned long long* ev = p.trace + (static_cast<size_t>(blockIdx.x) * p.trace_slots + p.trace_slots - kTlSlots) * 4 +
                           (static_cast<size_t>(warp) * kTlEvents + i) * 2;
  ev[0] = static_cast<unsigned long long>(code) | (static_cast<unsigned long long>(static_cast<unsigned>(aux)) << 32);
  ev[1] = static_cast<unsigned long long>(clock64());
}
// A trace mark at a point where the CTA's warps are not otherwise joined.
__device__ void mark(const Params& p, Misc* misc, int slot) {
  if (p.trace == nullptr) return;
  named_sync();
  if (threadIdx.x == 0) {
    const unsigned long long t = global_ns();
    trace_mark(p, misc, slot, t, t);
  }
}

// Grid-wide join between operators (join `idx`, 1-based, monotonic within a
// launch): the CTA's consumer threads finish the operator; thread 0 adds the
// CTA's arrival (release) and waits (bounded, acquire) until every CTA has
// arrived idx times, then releases its consumers.
__device__ void grid_join(const Params& p, Misc* misc, unsigned idx, int slot) {
  tl_event(p, misc, 40);
  named_sync();
  if (threadIdx.x == 0) {
    const unsigned long long t0 = p.trace != nullptr ? global_ns() : 0ull;
    tl_event(p, misc, 41);
    red_release_add(p.sync, 1u);
    tl_event(p, misc, 42);
    spin_geq(p, misc, p.sync, idx * gridDim.x);
    tl_event(p, misc, 43);
    if (p.trace != nullptr) trace_mark(p, misc, slot, t0, global_ns());
  }
  named_sync();
  tl_event(p, misc, 44);
}

// ------------------------------------------------------------------ tiles
// W8 tile: `kb` blocks of 32 columns. Returns the rows' partial sums.
// NKB > 0: the block count is a compile-time constant (loop fully unrolled, every
// load hoisted); 0: kb_count at run time.
template <int NKB>
__device__ __forceinline__ void w8_tile(const uint8_t* tile, const uint8_t* xs, int kb_count, int lane, float& og,
                                        float& oh) {
  constexpr int kUnroll = NKB > 0 ? NKB : 4;
  if (NKB > 0) kb_count = NKB;
  const int c = lane & 3;
  float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
  const uint8_t* a_ptr = tile + lane * 16;
  const uint8_t* x_ptr = xs + c * 16;
  constexpr uint32_t kMagic = 0x64646464u;
  constexpr uint32_t kOff = 0x64806480u;  // fp16 1152 in both halves
#pragma unroll kUnroll
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

// The MMAs of one round (up to 8 groups) of a W4 tile; FULL rounds have no
// per-group predicate, so loads of later groups can be scheduled early.
template <int MATS, bool FULL>
__device__ __forceinline__ void w4_round(const uint8_t* a_ptr, const uint8_t* xs, const uint8_t* zero, int gi0, int jn,
                                         int g, int c, float (&acc)[MATS][4], float (&acc2)[MATS][4]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (FULL || j < jn) {
      const int gi = gi0 + j;
      const uint8_t* bp = (g == j) ? xs + gi * 128 : zero;
      const uint4 b0 = lds128(bp + c * 16);
      const uint4 b1 = lds128(bp + 64 + c * 16);
      uint4 a[MATS];
#pragma unroll
      for (int m = 0; m < MATS; ++m) a[m] = lds128(a_ptr + (gi * MATS + m) * 512);
#pragma unroll
      for (int m = 0; m < MATS; ++m) {
        uint32_t tg[4], th[4];
        w4_convert(a[m].x, tg);
        w4_convert(a[m].y, th);
        {
          const uint32_t fa[4] = {tg[0], th[0], tg[2], th[2]};
          const uint32_t fb[4] = {tg[1], th[1], tg[3], th[3]};
          mma_16816<false>(acc[m], fa, b0.x, b0.y);
          mma_16816<true>(acc2[m], fb, b0.z, b0.w);
        }
        w4_convert(a[m].z, tg);
        w4_convert(a[m].w, th);
        {
          const uint32_t fa[4] = {tg[0], th[0], tg[2], th[2]};
          const uint32_t fb[4] = {tg[1], th[1], tg[3], th[3]};
          mma_16816<false>(acc[m], fa, b1.x, b1.y);
          mma_16816<true>(acc2[m], fb, b1.z, b1.w);
        }
      }
    }
  }
}

// W4 tile of MATS matrices (1 = down, 2 = gate+up) over `ngroups` groups of
// 64. xs points at the chunk's first staged group, om at its (O, X) pairs.
template <int MATS, int NG>
__device__ __forceinline__ void w4_tile(const uint8_t* tile, int ngroups, const uint8_t* xs, const float2* om,
                                        const uint8_t* zero, int lane, float (&out)[MATS][2]) {
  constexpr int kRoundUnroll = NG > 0 ? (NG + 7) / 8 : 1;
  if (NG > 0) ngroups = NG;
  const int g = lane >> 2, c = lane & 3;
  const uint8_t* a_ptr = tile + lane * 16;
  const int rounds = (ngroups + 7) >> 3;
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(tile + MATS * ngroups * 512);
  const uint16_t* bi = sc + rounds * MATS * 128;
  float res[MATS][2];
#pragma unroll
  for (int m = 0; m < MATS; ++m) res[m][0] = res[m][1] = 0.f;
#pragma unroll kRoundUnroll
  for (int r = 0; r < rounds; ++r) {
    // two accumulator chains per matrix (bf16 and fp16 MMAs), summed in the epilogue
    float acc[MATS][4], acc2[MATS][4];
#pragma unroll
    for (int m = 0; m < MATS; ++m)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[m][e] = acc2[m][e] = 0.f;
    const int jn = min(8, ngroups - 8 * r);
    if (jn == 8) w4_round<MATS, true>(a_ptr, xs, zero, 8 * r, 8, g, c, acc, acc2);
    else w4_round<MATS, false>(a_ptr, xs, zero, 8 * r, jn, g, c, acc, acc2);
#pragma unroll
    for (int m = 0; m < MATS; ++m)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[m][e] += acc2[m][e];
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
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  return static_cast<uint32_t>(__half_as_ushort(__float2half_rn(a))) |
         (static_cast<uint32_t>(__half_as_ushort(__float2half_rn(b))) << 16);
}
__device__ __forceinline__ uint32_t pack_b2(float a, float b) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(a))) |
         (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(b))) << 16);
}

// RMS of the residual from the per-thread sums of squares: fixed reduction
// order, so every CTA computes the same value.
__device__ void finish_rms(float ss, int n, float eps, Misc* misc) {
  const int tid = threadIdx.x;
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

// Residual stream <- embedding row (layer 0), with its RMS.
__device__ void load_residual(const __nv_bfloat16* src, int n, float eps, __nv_bfloat16* xres, Misc* misc) {
  float ss = 0.f;
  for (int v = threadIdx.x; v < n / 8; v += kConsumerThreads) {
    const uint4 w = *reinterpret_cast<const uint4*>(src + v * 8);
    *reinterpret_cast<uint4*>(xres + v * 8) = w;
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = bf16_lo(u[i]), b = bf16_hi(u[i]);
      ss = fmaf(a, a, ss);
      ss = fmaf(b, b, ss);
    }
  }
  finish_rms(ss, n, eps, misc);
}

// Residual stream += a row-split projection: x[n] = bf16(x[n] + bf16(S)) with
// S = (sum over the 8 K chunks, in chunk order, of P[n][c]) (* scale[n]), then
// the RMS of the new stream. Every CTA folds the same partials identically.
__device__ void fold_residual(const float* P, const float* scale, int n, float eps, __nv_bfloat16* xres, Misc* misc) {
  float ss = 0.f;
  // rows r = tid + k * threads, 4 per batch; all loads of a batch are issued before any is used
  constexpr int kBatch = 4;
  for (int r0 = 0; r0 < n; r0 += kBatch * kConsumerThreads) {
    float4 a[kBatch], b[kBatch];
    float sc[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int r = r0 + threadIdx.x + k * kConsumerThreads;
      if (r < n) {
        a[k] = __ldcg(reinterpret_cast<const float4*>(P + r * 8));
        b[k] = __ldcg(reinterpret_cast<const float4*>(P + r * 8 + 4));
        sc[k] = scale != nullptr ? scale[r] : 1.f;
      }
    }
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int r = r0 + threadIdx.x + k * kConsumerThreads;
      if (r >= n) break;
      float acc = ((((((a[k].x + a[k].y) + a[k].z) + a[k].w) + b[k].x) + b[k].y) + b[k].z) + b[k].w;
      if (scale != nullptr) acc *= sc[k];
      const float x = bfr(__bfloat162float(xres[r]) + bfr(acc));
      xres[r] = __float2bfloat16_rn(x);
      ss = fmaf(x, x, ss);
    }
  }
  named_sync();  // xres complete before anyone stages from it
  finish_rms(ss, n, eps, misc);
}

// 8 values of word v of the residual, RMS-normalised with weight w and rounded to bf16.
__device__ __forceinline__ void norm8(const __nv_bfloat16* xres, const __nv_bfloat16* w, float r, int v,
                                      float (&f)[8]) {
  const uint4 xv = *reinterpret_cast<const uint4*>(xres + v * 8);
  const uint4 wv = *reinterpret_cast<const uint4*>(w + v * 8);
  const uint32_t u[4] = {xv.x, xv.y, xv.z, xv.w};
  const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = bfr(bf16_lo(u[i]) * r * bf16_lo(wu[i]));
    f[2 * i + 1] = bfr(bf16_hi(u[i]) * r * bf16_hi(wu[i]));
  }
}
// 8 values of word v of a bf16 vector in global memory (written by other CTAs).
__device__ __forceinline__ void plain8(const __nv_bfloat16* x, int v, float (&f)[8]) {
  const uint4 xv = ldcg16(x + v * 8);
  const uint32_t u[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = bf16_lo(u[i]);
    f[2 * i + 1] = bf16_hi(u[i]);
  }
}

// W8 tiles read fp16 activations in natural order.
__device__ __forceinline__ void put_w8(uint8_t* xs, int v, const float (&f)[8]) {
  *reinterpret_cast<uint4*>(xs + v * 16) =
      make_uint4(pack_h2(f[0], f[1]), pack_h2(f[2], f[3]), pack_h2(f[4], f[5]), pack_h2(f[6], f[7]));
}
// BF16 tiles read bf16 activations in natural order.
__device__ __forceinline__ void put_bf16(uint8_t* xs, int v, const float (&f)[8]) {
  *reinterpret_cast<uint4*>(xs + v * 16) =
      make_uint4(pack_b2(f[0], f[1]), pack_b2(f[2], f[3]), pack_b2(f[4], f[5]), pack_b2(f[6], f[7]));
}
// W4 tiles read per 8-value word [bf16 (x0,x4) | bf16 (x2,x6) | fp16 (x1,x5) |
// fp16 (x3,x7)] and per group of 64 the offset sum O = 128*sum(even) +
// 64*sum(odd) and X = sum(x). Called by all consumer threads for words
// v0 + tid (v0 a multiple of kConsumerThreads, itself a multiple of 8, so the 8
// words of a group sit in 8 consecutive lanes); `valid` is false past the end.
__device__ __forceinline__ void put_w4(uint8_t* xs, float2* om, int v, bool valid, const float (&f)[8]) {
  float O = 0.f, X = 0.f;
  if (valid) {
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
  if (valid && (v & 7) == 0) om[v >> 3] = make_float2(O, X);
}

// -------------------------------------------------------------- operators
enum Kind : int { K_W8 = 0, K_W4 = 1, K_W4PAIR = 2, K_BF16 = 3 };

struct Smem {
  uint64_t* full;
  uint64_t* empty;
  unsigned* rbcnt;
  unsigned* ready;
  const uint8_t* zero;
  Misc* misc;
  float2* om;
  __nv_bfloat16* xres;
  float* part;
  uint8_t* xs;
  uint8_t* ring;
};

// Tile range [t0, t1) of this CTA in a stream of T tiles (balanced, contiguous).
// First tile index >= t0 of consumer warp `warp` when tiles t0, t0 + 1, ... are
// dealt round-robin from ring sequence number seq (tile t has sequence number
// seq + t - t0 and goes to warp (seq + t - t0) % kConsumers).
__device__ __forceinline__ int first_tile(int t0, uint32_t seq, int warp) {
  return t0 + (warp + kConsumers - static_cast<int>(seq % kConsumers)) % kConsumers;
}

__device__ __forceinline__ void cta_range(int T, int& t0, int& t1) {
  t0 = static_cast<int>((static_cast<long long>(T) * blockIdx.x) / gridDim.x);
  t1 = static_cast<int>((static_cast<long long>(T) * (blockIdx.x + 1)) / gridDim.x);
}

// Tile range of this CTA in a weight stream. Row-block-major streams split their
// tiles evenly. K-chunk-major streams (o_proj, down_proj) give every K chunk its
// own CTAs - chunk c: CTAs [ceil(c W / C), ceil((c + 1) W / C)) - which split the
// chunk's row blocks evenly, so that no CTA needs the activations of two chunks.
__device__ __forceinline__ void stream_range(const Stream& st, bool chunk_major, int& t0, int& t1) {
  const int C = st.chunks, W = static_cast<int>(gridDim.x), b = static_cast<int>(blockIdx.x);
  if (!chunk_major || W < C) {
    cta_range(st.rbs * C, t0, t1);
    return;
  }
  const int c = (b * C) / W;
  const int first = (c * W + C - 1) / C, count = ((c + 1) * W + C - 1) / C - first;
  const int i = b - first;
  t0 = c * st.rbs + (i * st.rbs) / count;
  t1 = c * st.rbs + ((i + 1) * st.rbs) / count;
}

// One projection over this CTA's share of its weight stream: every tile's
// per-row partial sums go to P[row * pstride + matrix * 8 + chunk] in L2 (the
// consumer of the projection sums the chunks in order). Tiles are taken
// round-robin by the consumer warps in stream order (the ring order).
// When `cnt` is set, each finished tile also adds one to cnt[rb / cnt_rbs]
// (progress that the next operator's consumers wait for).
// NK > 0: the stream's chunk size (W8: K blocks of 32; W4: groups) as a
// compile-time constant for the tile loops; 0: st.ck at run time.
template <int KIND, int NK>
__device__ void run_partials(const Params& p, const Smem& s, const Stream& st, bool chunk_major, float* P,
                             int pstride, int chunk0, uint32_t& seq, unsigned* cnt = nullptr, int cnt_rbs = 1) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int t0, t1;
  stream_range(st, chunk_major, t0, t1);
  const int g = lane >> 2;
  const int tl_op = KIND * 2 + (chunk_major ? 1 : 0);
  // progress of this warp's tiles not yet published: counter index and count
  int pend_idx = -1;
  unsigned pend_cnt = 0;
  auto publish = [&]() {
    if (cnt != nullptr && pend_cnt != 0u) {
      tl_event(p, s.misc, 13);
      __syncwarp();
      if (lane == 0) red_release_add(cnt + pend_idx, pend_cnt);
      pend_cnt = 0;
      tl_event(p, s.misc, 14);
    }
  };
  for (int t = first_tile(t0, seq, warp); t < t1; t += kConsumers) {
    const uint32_t q = seq + static_cast<uint32_t>(t - t0);
    if (*reinterpret_cast<volatile int*>(&s.misc->abort)) break;
    const int slot = static_cast<int>(q % static_cast<uint32_t>(p.slots));
    tl_event(p, s.misc, 10, tl_op * 65536 + (t - t0));
    if (!wait_bar(s.full + slot, (q / static_cast<uint32_t>(p.slots)) & 1u, p, s.misc)) break;
    tl_event(p, s.misc, 11);
    const uint8_t* tile = s.ring + static_cast<size_t>(slot) * p.slot_bytes;
    const int rb = chunk_major ? t % st.rbs : t / st.chunks;
    const int ch = chunk_major ? t / st.rbs : t % st.chunks;
    float vals[2][2];
    if constexpr (KIND == K_W8) {
      w8_tile<NK>(tile, s.xs + ch * st.ck * 2, st.ck / 32, lane, vals[0][0], vals[0][1]);
    } else if constexpr (KIND == K_W4) {
      float o[1][2];
      w4_tile<1, NK>(tile, st.ck, s.xs + ch * st.ck * 128, s.om + ch * st.ck, s.zero, lane, o);
      vals[0][0] = o[0][0];
      vals[0][1] = o[0][1];
    } else {
      w4_tile<2, NK>(tile, st.ck, s.xs + ch * st.ck * 128, s.om + ch * st.ck, s.zero, lane, vals);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(s.empty + slot);
    tl_event(p, s.misc, 12);
    if ((lane & 3) == 0) {
      float* out = P + static_cast<size_t>(rb * 16 + g) * pstride + chunk0 + ch;
      out[0] = vals[0][0];
      out[8 * pstride] = vals[0][1];
      if constexpr (KIND == K_W4PAIR) {
        out[8] = vals[1][0];
        out[8 * pstride + 8] = vals[1][1];
      }
    }
    if (cnt != nullptr) {
      const int idx = rb / cnt_rbs;
      if (idx != pend_idx) {
        publish();
        pend_idx = idx;
      }
      ++pend_cnt;
    }
  }
  publish();
  tl_event(p, s.misc, 15);
  seq += static_cast<uint32_t>(t1 - t0);
}

// lm_head + greedy argmax: the warp that completes a row block sums its chunk
// partials in chunk order; a block split between CTAs is finished by the CTA
// that brings its global counter to the chunk count.
__device__ void run_lm(const Params& p, const Smem& s, uint32_t& seq) {
  const Stream& st = p.slm;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = st.rbs * st.chunks;
  int t0, t1;
  cta_range(T, t0, t1);
  for (int i = threadIdx.x; i < kPartSlots; i += kConsumerThreads) s.ready[i] = i;
  named_sync();
  const int rb_first = t0 / st.chunks;
  for (int t = first_tile(t0, seq, warp); t < t1; t += kConsumers) {
    const uint32_t q = seq + static_cast<uint32_t>(t - t0);
    if (*reinterpret_cast<volatile int*>(&s.misc->abort)) break;
    const int slot = static_cast<int>(q % static_cast<uint32_t>(p.slots));
    if (!wait_bar(s.full + slot, (q / static_cast<uint32_t>(p.slots)) & 1u, p, s.misc)) break;
    const uint8_t* tile = s.ring + static_cast<size_t>(slot) * p.slot_bytes;
    const int rb = t / st.chunks, ch = t % st.chunks;
    float og, oh;
    bf16_tile(tile, s.xs + ch * st.ck * 2, st.ck / 16, lane, og, oh);
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
    if ((lane & 3) == 0) {
      part[lane >> 2] = og;
      part[(lane >> 2) + 8] = oh;
    }
    __threadfence_block();
    __syncwarp();
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
      float* gp = p.gpart + static_cast<size_t>(rb) * kChunks * 32;
      for (int c = cl0; c < cl1; ++c) {
        const float v = s.part[((c - t0) % kPartSlots) * 32 + lane];
        if (lane < 16) gp[(c - rb * st.chunks) * 32 + lane] = v;
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
    if (last) {
      const int n = rb * 16 + lane;
      unsigned long long key = (lane < 16 && n < p.vocab) ? argmax_key(total, n + p.vocab_offset) : 0ull;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
        key = k2 > key ? k2 : key;
      }
      if (lane == 0 && key) atomicMax(&s.misc->key, key);
    }
  }
  seq += static_cast<uint32_t>(t1 - t0);
}

// Sum, in chunk order, of the first n (<= 8) per-chunk partials of a row
// stored as 8 floats (written by other CTAs: read through L2).
// Sum of the first n (<= 8) chunk partials a.x .. b.w, in chunk order.
__device__ __forceinline__ float sum_loaded(const float4& a, const float4& b, int n) {
  const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  float acc = v[0];
#pragma unroll
  for (int i = 1; i < 8; ++i)
    if (i < n) acc += v[i];
  return acc;
}
__device__ __forceinline__ float sum_chunks(const float* row, int n) {
  const float4 a = __ldcg(reinterpret_cast<const float4*>(row));
  float v[8] = {a.x, a.y, a.z, a.w, 0.f, 0.f, 0.f, 0.f};
  if (n > 4) {
    const float4 b = __ldcg(reinterpret_cast<const float4*>(row + 4));
    v[4] = b.x;
    v[5] = b.y;
    v[6] = b.z;
    v[7] = b.w;
  }
  float acc = v[0];
#pragma unroll
  for (int i = 1; i < 8; ++i)
    if (i < n) acc += v[i];
  return acc;
}

// ------------------------------------------------------------- attention
// The row pairs (d, d+64) of one head from the QKV partials (stream row order:
// block 8*hd + i holds dims 8i..8i+7 in rows 0-7 and their partners in rows
// 8-15): the 5 K chunks summed in order, the per-row scale, bf16 rounding, and
// for query/key heads the rotation at position pos. Lane L covers dims
// d = 8*(L>>2) + 2*(L&3) + {0, 1} and d + 64.
__device__ __forceinline__ void head_rows(const Params& p, const Layer& L, int hd, bool rope, const float (&cs)[2],
                                          const float (&sn)[2], int lane, float (&lo)[2], float (&hi)[2]) {
  const int i = lane >> 2, gg = (lane & 3) * 2;
  const int base = (hd * 8 + i) * 16;
  // the four rows' chunk partials and scales, all loads issued before any is used
  float4 pa[4], pb[4];
  float sc[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = base + gg + (k >> 1) + 8 * (k & 1);
    pa[k] = __ldcg(reinterpret_cast<const float4*>(p.pqkv + r * 8));
    pb[k] = __ldcg(reinterpret_cast<const float4*>(p.pqkv + r * 8 + 4));
    sc[k] = L.qkv_scale[r];
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    float x0 = bfr(sum_loaded(pa[2 * e], pb[2 * e], p.sq.chunks) * sc[2 * e]);
    float x1 = bfr(sum_loaded(pa[2 * e + 1], pb[2 * e + 1], p.sq.chunks) * sc[2 * e + 1]);
    if (rope) {
      const float ra = x0 * cs[e] - x1 * sn[e];
      const float rb2 = x1 * cs[e] + x0 * sn[e];
      x0 = bfr(ra);
      x1 = bfr(rb2);
    }
    lo[e] = x0;
    hi[e] = x1;
  }
}

// INT8 K/V row quantization (symmetric per token per head, fp16 scale =
// absmax / 127, 1 for a zero row; code = clamp(rint(x / scale), +-127)) of
// the lane's 4 values of a head, written to the cache at position pos.
__device__ __forceinline__ void quantize_row(const float (&lo)[2], const float (&hi)[2], int lane, int8_t* row,
                                             __half* scale_slot, int8_t* srow, __half* sscale) {
  float amax = fmaxf(fmaxf(fabsf(lo[0]), fabsf(lo[1])), fmaxf(fabsf(hi[0]), fabsf(hi[1])));
  amax = warp_max(amax);
  __half s16 = __float2half_rn(__fdiv_rn(amax, 127.0f));
  if (__half2float(s16) == 0.f) s16 = __float2half_rn(1.0f);
  const float sf = __half2float(s16);
  auto q = [&](float v) {
    return static_cast<int8_t>(static_cast<int>(fminf(fmaxf(rintf(__fdiv_rn(v, sf)), -127.f), 127.f)));
  };
  const int d = 8 * (lane >> 2) + 2 * (lane & 3);
  const int8_t q0 = q(lo[0]), q1 = q(lo[1]), q2 = q(hi[0]), q3 = q(hi[1]);
  row[d] = q0;
  row[d + 1] = q1;
  row[d + 64] = q2;
  row[d + 65] = q3;
  srow[d] = q0;
  srow[d + 1] = q1;
  srow[d + 64] = q2;
  srow[d + 65] = q3;
  if (lane == 0) {
    *scale_slot = s16;
    *sscale = s16;
  }
}

// Attention of the new token (position pos) over the INT8 cache. Work item =
// (KV head, span of kAttnSpan tokens), one CTA each (the span count depends
// only on the context length, so the summation structure is the same at every
// tensor-parallel degree). The CTA rebuilds q of the head's G query heads from
// the QKV partials; each consumer warp takes one kAttnChunk-token slice: QK^T on the
// tensor cores (K rows as the A operand, exact int8 -> fp16; q as B with one
// column per head), softmax partials, P.V on the CUDA cores (lane = 4 dims).
// The warps' partials merge in shared memory in token order; spans of one KV
// head merge, in span order, in the CTA that completes the last span. The warp
// whose slice holds pos builds the new K/V row and writes it into the cache.
constexpr int kAttnSpan = kConsumers * kAttnChunk;
constexpr int kAttnPart = 132;  // floats per (head) partial: acc[128], m, l, pad

// Ring slot layout of one attention slice (kAttnChunk tokens of one KV head): K
// rows [kAttnChunk][128] int8, V rows likewise, K scales [kAttnChunk] fp16, V
// scales likewise (every part starts on a 16-byte boundary).
constexpr int kSliceK = 0, kSliceV = kAttnChunk * 128, kSliceKs = 2 * kAttnChunk * 128,
              kSliceVs = kSliceKs + kAttnChunk * 2, kSliceBytes = kSliceVs + kAttnChunk * 2;
static_assert(kAttnChunk % 16 == 0 && (kAttnChunk * 2) % 16 == 0, "slice layout");

// Number of slices of attention item `item` (tokens [span*kAttnSpan, n)).
__device__ __forceinline__ int attn_slices(int item, int spans, int n) {
  const int tspan = (item % spans) * kAttnSpan;
  return min(kConsumers, (n - tspan + kAttnChunk - 1) / kAttnChunk);
}

template <int G>
__device__ void attention_step(const Params& p, const Smem& sm, const Layer& L, int layer, int pos, uint8_t* scratch,
                               uint32_t& seq, const float (&cs)[2], const float (&sn)[2]) {
  Misc* misc = sm.misc;
  // tracing: thread 0 stamps item milestones (heads ready, q built, computed, published)
  unsigned long long* astamp = (p.trace != nullptr && threadIdx.x == 0)
                                   ? p.trace + (static_cast<size_t>(blockIdx.x) * p.trace_slots +
                                                p.num_layers * kMarksPerLayer + 2 + layer * kAttnMarks) * 4
                                   : nullptr;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int g = lane >> 2, c = lane & 3;
  const int n = pos + 1;
  const int spans = (n + kAttnSpan - 1) / kAttnSpan;
  const int items = p.kv_heads * spans;
  const size_t cap = static_cast<size_t>(p.capacity);
  __half* qs = reinterpret_cast<__half*>(scratch);                                    // [G][128] fp16
  float* wpart = reinterpret_cast<float*>(scratch + 1024) + warp * G * kAttnPart;      // this warp's partial
  float* pw = wpart;  // [kAttnChunk][4] probabilities (before the partial)
  float* allpart = reinterpret_cast<float*>(scratch + 1024);
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const int h = item / spans, span = item % spans;
    const int tspan = span * kAttnSpan;
    const int tb = tspan + warp * kAttnChunk;  // this warp's slice
    const int slices = attn_slices(item, spans, n);
    const bool has_slice = warp < slices;
    // this warp's ring slot: K/V rows of the slice below pos (copied by the producer)
    const uint32_t q_slot = seq + static_cast<uint32_t>(warp);
    const int slot = static_cast<int>(q_slot % static_cast<uint32_t>(p.slots));
    uint8_t* tile = sm.ring + static_cast<size_t>(slot) * p.slot_bytes;
    if (has_slice) wait_bar(sm.full + slot, (q_slot / static_cast<uint32_t>(p.slots)) & 1u, p, misc);
    tl_event(p, misc, 20, item);
    const bool span_has_pos = pos >= tspan && pos < tspan + kAttnSpan;
    int8_t* kc = L.k_cache + static_cast<size_t>(h) * cap * 128;
    int8_t* vc = L.v_cache + static_cast<size_t>(h) * cap * 128;
    __half* ksc = L.k_scale + static_cast<size_t>(h) * cap;
    __half* vsc = L.v_scale + static_cast<size_t>(h) * cap;
    // ---- the QKV tiles of the heads this span reads
    if (tid == 0) {
      const unsigned need = static_cast<unsigned>((layer + 1) * 8 * p.sq.chunks);
      // the G query heads' rows, and the new K and V rows when this span holds pos
      spin_heads<G>(p, misc, h, span_has_pos, need);
      if (astamp) astamp[0] = global_ns();
      tl_event(p, misc, 21);
    }
    named_sync();
    // (after a failed wait the item still runs through every barrier; its output is invalid and
    // the status word reports it)
    // ---- q of the G query heads (warp j builds head j), fp16 (exact for these bf16 values)
    const int d0 = 8 * (lane >> 2) + 2 * (lane & 3);
    if (warp < G) {
      float lo[2], hi[2];
      head_rows(p, L, G * h + warp, true, cs, sn, lane, lo, hi);
      *reinterpret_cast<__half2*>(qs + warp * 128 + d0) = __floats2half2_rn(lo[0], lo[1]);
      *reinterpret_cast<__half2*>(qs + warp * 128 + d0 + 64) = __floats2half2_rn(hi[0], hi[1]);
    }
    if (span_has_pos) {
      // the new token's K row (its slice's warp) and V row (the next warp): into the cache and
      // into the slice, after the slice's copies have landed
      const int wn = (pos - tspan) / kAttnChunk;
      const int wv = wn + 1 < kConsumers ? wn + 1 : 0;
      if (warp == wn || warp == wv) {
        const bool is_k = warp == wn;
        const uint32_t qn = seq + static_cast<uint32_t>(wn);
        const int sn2 = static_cast<int>(qn % static_cast<uint32_t>(p.slots));
        uint8_t* tn = sm.ring + static_cast<size_t>(sn2) * p.slot_bytes;
        if (!is_k) wait_bar(sm.full + sn2, (qn / static_cast<uint32_t>(p.slots)) & 1u, p, misc);
        const int r = pos - (tspan + wn * kAttnChunk);
        float lo[2], hi[2];
        head_rows(p, L, is_k ? p.heads + h : p.heads + p.kv_heads + h, is_k, cs, sn, lane, lo, hi);
        if (is_k)
          quantize_row(lo, hi, lane, kc + static_cast<size_t>(pos) * 128, ksc + pos,
                       reinterpret_cast<int8_t*>(tn + kSliceK) + r * 128, reinterpret_cast<__half*>(tn + kSliceKs) + r);
        else
          quantize_row(lo, hi, lane, vc + static_cast<size_t>(pos) * 128, vsc + pos,
                       reinterpret_cast<int8_t*>(tn + kSliceV) + r * 128, reinterpret_cast<__half*>(tn + kSliceVs) + r);
      }
    }
    named_sync();
    tl_event(p, misc, 22);
    if (astamp) astamp[4] = global_ns();
    float m2[2] = {-INFINITY, -INFINITY}, l2[2] = {0.f, 0.f};
    float2 acc[G][2];  // dims (4 lane, +1), (4 lane + 2, +3)
#pragma unroll
    for (int hh = 0; hh < G; ++hh) acc[hh][0] = acc[hh][1] = make_float2(0.f, 0.f);
    if (tb < n) {
      tl_event(p, misc, 26);
      // ---- B fragments: column g < G is query head g; dims of MMA s for lane quad c: 32c + 4s + {0..3}
      uint32_t bq[8][2];
#pragma unroll
      for (int s2 = 0; s2 < 8; ++s2) {
        if (g < G) {
          const uint2 v = *reinterpret_cast<const uint2*>(qs + g * 128 + 32 * c + 4 * s2);
          bq[s2][0] = v.x;
          bq[s2][1] = v.y;
        } else {
          bq[s2][0] = bq[s2][1] = 0u;
        }
      }
      // ---- scores of the slice's tokens (16-token MMA row blocks)
      float sc[kAttnRbk][4];
#pragma unroll
      for (int rbk = 0; rbk < kAttnRbk; ++rbk) {
        float ac[4] = {0.f, 0.f, 0.f, 0.f};
        const int rg = rbk * 16 + g, rh = rg + 8;  // rows of the slice
        const int tg = tb + rg, th = tb + rh;
        const uint8_t* kr_g = tile + kSliceK + rg * 128 + 32 * c;
        const uint8_t* kr_h = tile + kSliceK + rh * 128 + 32 * c;
        const uint4 kg0 = lds128(kr_g), kg1 = lds128(kr_g + 16), kh0 = lds128(kr_h), kh1 = lds128(kr_h + 16);
        const __half* ks_s = reinterpret_cast<const __half*>(tile + kSliceKs);
        const float kgs = tg < n ? __half2float(ks_s[rg]) : 0.f;
        const float khs = th < n ? __half2float(ks_s[rh]) : 0.f;
        const uint32_t wg[8] = {kg0.x, kg0.y, kg0.z, kg0.w, kg1.x, kg1.y, kg1.z, kg1.w};
        const uint32_t wh[8] = {kh0.x, kh0.y, kh0.z, kh0.w, kh1.x, kh1.y, kh1.z, kh1.w};
        constexpr uint32_t kMagic = 0x64646464u, kOff = 0x64806480u;
#pragma unroll
        for (int s2 = 0; s2 < 8; ++s2) {
          const uint32_t ug = wg[s2] ^ 0x80808080u, uh = wh[s2] ^ 0x80808080u;
          const uint32_t a[4] = {hsub2_u32(prmt(ug, kMagic, 0x4140u), kOff), hsub2_u32(prmt(uh, kMagic, 0x4140u), kOff),
                                 hsub2_u32(prmt(ug, kMagic, 0x4342u), kOff), hsub2_u32(prmt(uh, kMagic, 0x4342u), kOff)};
          mma_16816<true>(ac, a, bq[s2][0], bq[s2][1]);
        }
        // lane holds tokens tg (ac 0,1) and th (ac 2,3) for heads 2c, 2c+1
        sc[rbk][0] = tg < n ? ac[0] * kgs * p.attn_scale : -INFINITY;
        sc[rbk][1] = tg < n ? ac[1] * kgs * p.attn_scale : -INFINITY;
        sc[rbk][2] = th < n ? ac[2] * khs * p.attn_scale : -INFINITY;
        sc[rbk][3] = th < n ? ac[3] * khs * p.attn_scale : -INFINITY;
      }
      tl_event(p, misc, 27);
      // ---- softmax partials per head (column 2c + e), over the slice's tokens
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float mx = fmaxf(sc[0][e], sc[0][e + 2]);
#pragma unroll
        for (int rbk = 1; rbk < kAttnRbk; ++rbk) mx = fmaxf(mx, fmaxf(sc[rbk][e], sc[rbk][e + 2]));
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        m2[e] = mx;
        float sum = 0.f;
#pragma unroll
        for (int rbk = 0; rbk < kAttnRbk; ++rbk)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const float v = sc[rbk][e + 2 * hh];
            const float pe = v == -INFINITY ? 0.f : expf(v - mx);
            sc[rbk][e + 2 * hh] = pe;
            sum += pe;
          }
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        l2[e] = sum;
      }
      if (2 * c < G) {
#pragma unroll
        for (int rbk = 0; rbk < kAttnRbk; ++rbk)
#pragma unroll
          for (int e = 0; e < 2; ++e)
            if (2 * c + e < G) {
              pw[(rbk * 16 + g) * 4 + 2 * c + e] = sc[rbk][e];
              pw[(rbk * 16 + g + 8) * 4 + 2 * c + e] = sc[rbk][e + 2];
            }
      }
      __syncwarp();
      tl_event(p, misc, 28);
      // ---- P.V: lane owns dims 4*lane .. 4*lane+3; V words and scales 8 tokens at a time
      const int tend = min(n - tb, kAttnChunk);
      const __half* vs_s = reinterpret_cast<const __half*>(tile + kSliceVs);
      for (int t0 = 0; t0 < tend; t0 += 8) {
        int vw[8];
        float vs[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int tt = t0 + j;
          vw[j] = 0;
          vs[j] = 0.f;
          if (tt < tend) {
            vw[j] = *reinterpret_cast<const int*>(tile + kSliceV + tt * 128 + lane * 4);
            vs[j] = __half2float(vs_s[tt]);
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (t0 + j >= tend) break;
          const float4 p4 = *reinterpret_cast<const float4*>(pw + (t0 + j) * 4);
          const float pr[4] = {p4.x * vs[j], p4.y * vs[j], p4.z * vs[j], p4.w * vs[j]};
          // codes -> fp32 exactly: the biased byte b = code + 128 under exponent 2^23 is 2^23 + b,
          // minus 2^23 + 128 (both exact), two lanes of a packed fp32 pair at a time
          const uint32_t u = static_cast<uint32_t>(vw[j]) ^ 0x80808080u;
          const float2 kBias = make_float2(-8388736.0f, -8388736.0f);
          const float2 v01 = __fadd2_rn(make_float2(__uint_as_float(prmt(u, 0x4B000000u, 0x7540u)),
                                                    __uint_as_float(prmt(u, 0x4B000000u, 0x7541u))), kBias);
          const float2 v23 = __fadd2_rn(make_float2(__uint_as_float(prmt(u, 0x4B000000u, 0x7542u)),
                                                    __uint_as_float(prmt(u, 0x4B000000u, 0x7543u))), kBias);
#pragma unroll
          for (int hh = 0; hh < G; ++hh) {
            const float2 ph = make_float2(pr[hh], pr[hh]);
            acc[hh][0] = __ffma2_rn(ph, v01, acc[hh][0]);
            acc[hh][1] = __ffma2_rn(ph, v23, acc[hh][1]);
          }
        }
      }
      __syncwarp();  // pw is overwritten by the partial below
    }
    if (has_slice && lane == 0) mbar_arrive(sm.empty + slot);
    tl_event(p, misc, 23);
    // ---- this warp's partial into shared memory: [head][acc 128 | m | l]
#pragma unroll
    for (int hh = 0; hh < G; ++hh) {
      *reinterpret_cast<float4*>(wpart + hh * kAttnPart + lane * 4) =
          make_float4(acc[hh][0].x, acc[hh][0].y, acc[hh][1].x, acc[hh][1].y);
      if (lane == hh / 2) {  // lane (g = 0, c = hh/2) holds column hh = 2c + e
        wpart[hh * kAttnPart + 128] = m2[hh & 1];
        wpart[hh * kAttnPart + 129] = l2[hh & 1];
      }
    }
    named_sync();
    if (astamp) astamp[8] = global_ns();
    // ---- merge the warps' partials in token order into this span's partial (L2); thread -> (head, dim)
    float* gp0 = p.apart + ((static_cast<size_t>(h) * p.attn_max_chunks + span) * G) * kAttnPart;
    float* wts = allpart + kConsumers * G * kAttnPart;  // [kConsumers][G] weights, then [G] max, [G] sum
    if (tid < G) {
      const int hh = tid;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) M = fmaxf(M, allpart[(w * G + hh) * kAttnPart + 128]);
      float Lsum = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) {
        const float* e = allpart + (w * G + hh) * kAttnPart;
        const float wt = e[128] == -INFINITY ? 0.f : expf(e[128] - M);
        Lsum = fmaf(e[129], wt, Lsum);
        wts[w * G + hh] = wt;
      }
      wts[kConsumers * G + hh] = M;
      wts[kConsumers * G + G + hh] = Lsum;
    }
    named_sync();
    for (int o = tid; o < G * 128; o += kConsumerThreads) {
      const int hh = o >> 7, d = o & 127;
      float A = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) A = fmaf(allpart[(w * G + hh) * kAttnPart + d], wts[w * G + hh], A);
      float* gp = gp0 + hh * kAttnPart;
      gp[d] = A;
      if (d == 0) {
        gp[128] = wts[kConsumers * G + hh];
        gp[129] = wts[kConsumers * G + G + hh];
      }
    }
    // ---- one more span of KV head h is published (the o_proj prologue merges the spans)
    tl_event(p, misc, 24);
    named_sync();
    if (tid == 0) red_release_add(p.hdr + kHdrAttn + h, 1u);
    tl_event(p, misc, 25);
    if (astamp) astamp[12] = global_ns();
    named_sync();  // the scratch is reused by the next item
    seq += static_cast<uint32_t>(slices);
  }
}

// --------------------------------------------------------------- producer
// Attention slices of this CTA's items: the cache rows below pos (the new row is
// built by the consumer) are copied into one ring slot per slice, so the
// attention reads K and V from shared memory. Slots holding no rows complete
// without a copy.
__device__ void produce_attention(const Params& p, const Smem& s, const Layer& L, int pos, uint32_t& seq,
                                  uint64_t pol) {
  const int n = pos + 1;
  const int spans = (n + kAttnSpan - 1) / kAttnSpan;
  const int items = p.kv_heads * spans;
  const size_t cap = static_cast<size_t>(p.capacity);
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const int h = item / spans, tspan = (item % spans) * kAttnSpan;
    const int slices = attn_slices(item, spans, n);
    for (int w = 0; w < slices; ++w, ++seq) {
      if (*reinterpret_cast<volatile int*>(&s.misc->abort)) return;
      const int slot = static_cast<int>(seq % static_cast<uint32_t>(p.slots));
      const uint32_t use = seq / static_cast<uint32_t>(p.slots);
      if (use > 0 && !wait_bar(s.empty + slot, (use - 1) & 1u, p, s.misc)) return;
      const int tb = tspan + w * kAttnChunk;
      const int cnt = min(kAttnChunk, pos - tb);  // rows below the new token
      if (cnt <= 0) {
        mbar_arrive_expect_tx(s.full + slot, 0u);
        continue;
      }
      const int cnt8 = (cnt + 7) & ~7;  // scale copies in 16-byte units (capacity is a multiple of 16)
      uint8_t* dst = s.ring + static_cast<size_t>(slot) * p.slot_bytes;
      mbar_arrive_expect_tx(s.full + slot, static_cast<uint32_t>(2 * cnt * 128 + 2 * cnt8 * 2));
      const size_t row0 = static_cast<size_t>(h) * cap + tb;
      (void)pol;  // cache rows are read again next step: no evict-first hint
      bulk_copy_g2s(dst + kSliceK, L.k_cache + row0 * 128, static_cast<uint32_t>(cnt * 128), s.full + slot);
      bulk_copy_g2s(dst + kSliceV, L.v_cache + row0 * 128, static_cast<uint32_t>(cnt * 128), s.full + slot);
      bulk_copy_g2s(dst + kSliceKs, L.k_scale + row0, static_cast<uint32_t>(cnt8 * 2), s.full + slot);
      bulk_copy_g2s(dst + kSliceVs, L.v_scale + row0, static_cast<uint32_t>(cnt8 * 2), s.full + slot);
    }
  }
}

__device__ void produce_op(const Params& p, const Smem& s, const Stream& st, bool chunk_major, const uint8_t* stream,
                           uint32_t& seq, uint64_t pol) {
  int t0, t1;
  stream_range(st, chunk_major, t0, t1);
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
  s.xres = reinterpret_cast<__nv_bfloat16*>(base + kOffXres);
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
    s.misc->wait_ns = 0ull;
    s.misc->busy_ns = 0ull;
    s.misc->tl_on = 0;
    for (int w = 0; w < kConsumers; ++w) s.misc->tl_n[w] = 0u;
  }
  for (int i = threadIdx.x; i < kRbSlots; i += blockDim.x) s.rbcnt[i] = 0u;
  for (int i = threadIdx.x; i < 64; i += blockDim.x) reinterpret_cast<uint32_t*>(base + kOffZero)[i] = 0u;
  __syncthreads();

  const int pos = p.positions[0];
  if (pos < 0 || pos >= p.capacity) {
    // the new token's K/V row would fall outside the cache: nothing is read or
    // written; the step reports it (uniform for every thread of every CTA)
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(p.status, kStatusRange);
    return;
  }
  if (warp == kConsumers) {
    // ---------------- producer warp (one lane issues)
    if (lane == 0) {
      const uint64_t pol = evict_first_policy();
      uint32_t seq = 0;
      for (int l = 0; l < p.num_layers; ++l) {
        const Layer& L = p.layers[l];
        produce_op(p, s, p.sq, false, L.qkv, seq, pol);
        produce_attention(p, s, L, pos, seq, pol);
        produce_op(p, s, p.so, true, L.o, seq, pol);
        produce_op(p, s, p.sgu, false, L.gateup, seq, pol);
        produce_op(p, s, p.sdn, true, L.down, seq, pol);
      }
      produce_op(p, s, p.slm, false, p.head, seq, pol);
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
  const int tid = threadIdx.x;
  if (p.trace != nullptr && tid == 0)
  {
    unsigned long long* st0 = p.trace + (static_cast<size_t>(blockIdx.x) * p.trace_slots + p.num_layers * kMarksPerLayer + 1) * 4;
    st0[0] = global_ns();
    st0[1] = static_cast<unsigned long long>(clock64());
  }
  const int token = p.tokens[0];
  const __nv_bfloat16* emb = p.embed + static_cast<size_t>(min(max(token, 0), p.vocab_total - 1)) * p.hidden;
  uint32_t seq = 0;
  unsigned joins = 0;
  const int G = p.heads / p.kv_heads;
  const int nwords = p.hidden / 8;
  const int act_chunk = p.sdn.ck * 64;       // activation values per down K chunk
  const int gu_rbs_per_chunk = act_chunk / 16;
  load_residual(emb, p.hidden, p.eps, s.xres, s.misc);
  // RoPE angles of this position for the lane's two dims (the same in every layer)
  float rope_cs[2], rope_sn[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int d = 8 * ((tid & 31) >> 2) + 2 * (tid & 3) + e;
    sincosf(static_cast<float>(pos) * p.inv_freq[d], &rope_sn[e], &rope_cs[e]);
  }
  for (int l = 0; l < p.num_layers; ++l) {
    const Layer& L = p.layers[l];
    const int mk = l * kMarksPerLayer;
    if (p.trace != nullptr) {
      if (tid == 0) s.misc->tl_on = l == p.num_layers / 2;
      named_sync();
      tl_event(p, s.misc, 1);
    }
    // ---- RMSNorm + QKV projection (per-chunk partials; RoPE happens in the attention items)
    if (l > 0) fold_residual(p.pdn, nullptr, p.hidden, p.eps, s.xres, s.misc);
    tl_event(p, s.misc, 2);
    for (int v = tid; v < nwords; v += kConsumerThreads) {
      float f[8];
      norm8(s.xres, L.in_norm, s.misc->rms, v, f);
      put_w8(s.xs, v, f);
    }
    named_sync();
    tl_event(p, s.misc, 3);
    mark(p, s.misc, mk + 0);
    run_partials<K_W8, 0>(p, s, p.sq, false, p.pqkv, 8, 0, seq, p.hdr + kHdrQkv, 8);
    mark(p, s.misc, mk + 1);
    // ---- attention of the new token (items wait for their heads' QKV tiles)
    named_sync();  // the attention scratch aliases the staged activations
    uint8_t* scratch = base + kOffPart;
    if (G == 1) attention_step<1>(p, s, L, l, pos, scratch, seq, rope_cs, rope_sn);
    else if (G == 2) attention_step<2>(p, s, L, l, pos, scratch, seq, rope_cs, rope_sn);
    else attention_step<4>(p, s, L, l, pos, scratch, seq, rope_cs, rope_sn);
    mark(p, s.misc, mk + 2);
    named_sync();
    // ---- o_proj: this CTA's tiles (K-chunk-major) need the attention output of their chunks' KV heads
    {
      const Stream& st = p.so;
      int t0, t1;
      stream_range(st, true, t0, t1);
      if (t1 > t0) {
        const int c0 = t0 / st.rbs, c1 = (t1 - 1) / st.rbs;
        const int spans = (pos + kAttnSpan) / kAttnSpan;  // ceil((pos + 1) / kAttnSpan)
        if (tid == 0) {
          // every span of the KV heads whose query heads feed K values [c0*ck, (c1+1)*ck)
          const int h0 = (c0 * st.ck) / (128 * G), h1 = ((c1 + 1) * st.ck - 1) / (128 * G);
          tl_event(p, s.misc, 30);
          for (int h = h0; h <= h1; ++h)
            if (!spin_geq(p, s.misc, p.hdr + kHdrAttn + h, static_cast<unsigned>((l + 1) * spans))) break;
          tl_event(p, s.misc, 31);
        }
        named_sync();
        // attention output: the spans' partials merged in span order, rounded to bf16
        for (int v = c0 * st.ck / 8 + tid; v < (c1 + 1) * st.ck / 8; v += kConsumerThreads) {
          const int qh = (v * 8) >> 7, d0 = (v * 8) & 127;
          const int h = qh / G, hh = qh % G;
          const float* e0 = p.apart + (static_cast<size_t>(h) * p.attn_max_chunks * G + hh) * kAttnPart;
          const size_t jstride = static_cast<size_t>(G) * kAttnPart;
          // spans in batches of 4, every load of a batch issued before any is used; the first
          // batch is loaded together with the maxima of the rest (one round of loads up to 4 spans)
          float4 a0[4], a1[4];
          float mj[4], lj[4];
          auto load_batch = [&](int j0) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float* e = e0 + (j0 + j) * jstride;
              const bool ok = j0 + j < spans;
              a0[j] = ok ? __ldcg(reinterpret_cast<const float4*>(e + d0)) : make_float4(0.f, 0.f, 0.f, 0.f);
              a1[j] = ok ? __ldcg(reinterpret_cast<const float4*>(e + d0 + 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
              mj[j] = ok ? ldcg_f(e + 128) : -INFINITY;
              lj[j] = ok ? ldcg_f(e + 129) : 0.f;
            }
          };
          load_batch(0);
          float M = fmaxf(fmaxf(mj[0], mj[1]), fmaxf(mj[2], mj[3]));
          for (int j0 = 4; j0 < spans; j0 += 4) {
            float mv[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) mv[j] = j0 + j < spans ? ldcg_f(e0 + (j0 + j) * jstride + 128) : -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) M = fmaxf(M, mv[j]);
          }
          float Lsum = 0.f, A[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          for (int j0 = 0; j0 < spans; j0 += 4) {
            if (j0 > 0) load_batch(j0);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float wt = mj[j] == -INFINITY ? 0.f : expf(mj[j] - M);
              Lsum = fmaf(lj[j], wt, Lsum);
              const float av[8] = {a0[j].x, a0[j].y, a0[j].z, a0[j].w, a1[j].x, a1[j].y, a1[j].z, a1[j].w};
#pragma unroll
              for (int i = 0; i < 8; ++i) A[i] = fmaf(av[i], wt, A[i]);
            }
          }
          const float inv = Lsum > 0.f ? 1.0f / Lsum : 0.f;
          float f[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) f[i] = bfr(A[i] * inv);
          put_w8(s.xs, v, f);
        }
      }
    }
    tl_event(p, s.misc, 32);
    named_sync();
    tl_event(p, s.misc, 33);
    if (p.trace != nullptr && tid == 0) trace_mark(p, s.misc, mk + 3, global_ns(), global_ns());
    run_partials<K_W8, 0>(p, s, p.so, true, p.po, 8, 0, seq);
    grid_join(p, s.misc, ++joins, mk + 4);
    // ---- residual += o; RMSNorm + gate/up (partials; progress per down K chunk)
    tl_event(p, s.misc, 50);
    fold_residual(p.po, L.o_scale, p.hidden, p.eps, s.xres, s.misc);
    tl_event(p, s.misc, 51);
    for (int v0 = 0; v0 < nwords; v0 += kConsumerThreads) {
      const int v = v0 + tid;
      float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (v < nwords) norm8(s.xres, L.post_norm, s.misc->rms, v, f);
      put_w4(s.xs, s.om, v, v < nwords, f);
    }
    named_sync();
    tl_event(p, s.misc, 52);
    mark(p, s.misc, mk + 5);
    run_partials<K_W4PAIR, 0>(p, s, p.sgu, false, p.pgu, 16, 0, seq, p.hdr + kHdrGu, gu_rbs_per_chunk);
    mark(p, s.misc, mk + 6);
    // ---- SwiGLU of the K chunks this CTA's down tiles read (once their gate/up tiles are done), then down
    named_sync();
    {
      const Stream& st = p.sdn;
      int t0, t1;
      stream_range(st, true, t0, t1);
      if (t1 > t0) {
        const int c0 = t0 / st.rbs, c1 = (t1 - 1) / st.rbs;
        if (tid == 0) {
          const unsigned need = static_cast<unsigned>((l + 1) * gu_rbs_per_chunk * p.sgu.chunks);
          tl_event(p, s.misc, 60);
          for (int c = c0; c <= c1; ++c)
            if (!spin_geq(p, s.misc, p.hdr + kHdrGu + c, need)) break;
          tl_event(p, s.misc, 61);
        }
        named_sync();
        // SwiGLU values of the chunks into shared memory (thread per value: its gate and up
        // chunk partials are 64 contiguous bytes, loaded in one round) ...
        const int a0 = c0 * act_chunk, a1 = (c1 + 1) * act_chunk;
        __nv_bfloat16* actv = reinterpret_cast<__nv_bfloat16*>(base + kOffPart);
        for (int r = a0 + tid; r < a1; r += kConsumerThreads) {
          const float* pr = p.pgu + static_cast<size_t>(r) * 16;
          const float4 g0 = __ldcg(reinterpret_cast<const float4*>(pr));
          const float4 g1 = __ldcg(reinterpret_cast<const float4*>(pr + 4));
          const float4 u0 = __ldcg(reinterpret_cast<const float4*>(pr + 8));
          const float4 u1 = __ldcg(reinterpret_cast<const float4*>(pr + 12));
          const float gt = bfr(sum_loaded(g0, g1, p.sgu.chunks));
          const float up = bfr(sum_loaded(u0, u1, p.sgu.chunks));
          actv[r - a0] = __float2bfloat16_rn(gt / (1.0f + expf(-gt)) * up);
        }
        named_sync();
        // ... then staged for the W4 tiles, 8 values per thread
        const int w0 = a0 / 8, w1 = a1 / 8;
        for (int v0 = w0 & ~7; v0 < w1; v0 += kConsumerThreads) {
          const int v = v0 + tid;
          const bool valid = v >= w0 && v < w1;
          float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          if (valid) {
            const uint4 w = *reinterpret_cast<const uint4*>(actv + (v * 8 - a0));
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ws[i]));
              f[2 * i] = t.x;
              f[2 * i + 1] = t.y;
            }
          }
          put_w4(s.xs, s.om, v, valid, f);
        }
      }
    }
    named_sync();
    tl_event(p, s.misc, 62);
    if (p.trace != nullptr && tid == 0) trace_mark(p, s.misc, mk + 7, global_ns(), global_ns());
    run_partials<K_W4, 0>(p, s, p.sdn, true, p.pdn, 8, 0, seq);
    grid_join(p, s.misc, ++joins, mk + 8);
  }
  // ---- residual += down; final RMSNorm + lm_head + greedy argmax
  fold_residual(p.pdn, nullptr, p.hidden, p.eps, s.xres, s.misc);
  for (int v = tid; v < nwords; v += kConsumerThreads) {
    float f[8];
    norm8(s.xres, p.final_norm, s.misc->rms, v, f);
    put_bf16(s.xs, v, f);
  }
  named_sync();
  run_lm(p, s, seq);
  named_sync();
  if (tid == 0) {
    if (s.misc->key) atomicMax(p.keys, s.misc->key);
    if (p.trace != nullptr) trace_mark(p, s.misc, p.num_layers * kMarksPerLayer, global_ns(), global_ns());
  }
  // the residual stream of this step, for callers that inspect it (CTA 0)
  if (blockIdx.x == 0)
    for (int v = tid; v < nwords; v += kConsumerThreads)
      reinterpret_cast<uint4*>(p.x)[v] = reinterpret_cast<const uint4*>(s.xres)[v];
}

// ------------------------------------------------------------------- host
// Workspace layout (byte offsets): header words (arrival counter, status),
// lm_head split-block counters and partials, attention counters and
// partials, and the projections' per-chunk partial sums.
struct Workspace {
  size_t gcount, acount, gpart, apart, pqkv, po, pgu, pdn, total;
};

struct Geometry {
  Stream sq, so, sgu, sdn, slm;
  int attn_chunks;
  Workspace ws;
  int slot_bytes;
};

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

int geometry(const sb_step_desc* d, Geometry* g) {
  SB_REQUIRE(d != nullptr, "null descriptor");
  SB_REQUIRE(d->head_dim == 128, "the decode-step kernel supports head_dim 128");
  SB_REQUIRE(d->world == 1 && d->rank == 0, "the decode-step kernel in this build runs one rank");
  SB_REQUIRE(d->num_layers > 0 && d->num_layers <= kMaxLayers, "1..128 layers");
  SB_REQUIRE(d->hidden > 0 && d->hidden % 512 == 0 && d->hidden <= kMaxHidden,
             "hidden must be a multiple of 512, <= 4096");
  SB_REQUIRE(d->num_heads > 0 && d->num_kv_heads > 0 && d->num_heads % d->num_kv_heads == 0, "heads");
  const int G = d->num_heads / d->num_kv_heads;
  SB_REQUIRE(G == 1 || G == 2 || G == 4, "query heads per KV head must be 1, 2 or 4");
  SB_REQUIRE(d->num_heads + 2 * d->num_kv_heads <= 64, "at most 64 attention heads (query + key + value) per rank");
  SB_REQUIRE(sm_count() <= kMaxCtas, "at most 256 SMs");
  const int qk = d->num_heads * 128;  // o_proj K (this rank)
  SB_REQUIRE(qk <= kMaxK && qk % (kChunks * 32 / d->world) == 0, "o_proj K must split into 8 chunks of 32-multiples");
  SB_REQUIRE(d->inter > 0 && d->inter % 16 == 0 && d->inter <= kMaxK, "inter must be a multiple of 16, <= 10240");
  SB_REQUIRE(d->inter_total % (kChunks * 64) == 0, "intermediate size must be a multiple of 512");
  SB_REQUIRE(2 * (d->inter_total / kChunks) * 2 <= kPartSlots * 32 * 4,
             "two K chunks of down_proj activations must fit the shared staging area");
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
  tmax = tmax > kSliceBytes ? tmax : kSliceBytes;
  g->slot_bytes = (tmax + 127) / 128 * 128;
  g->attn_chunks = (d->capacity + kAttnSpan - 1) / kAttnSpan;
  Workspace& w = g->ws;
  size_t off = kHdrBytes + kPersistBytes;  // header words, persistent words
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = (off + bytes + 255) / 256 * 256;
    return at;
  };
  w.gcount = take(static_cast<size_t>(g->slm.rbs) * 4);
  w.acount = take(64 * 4);
  w.gpart = take(static_cast<size_t>(g->slm.rbs) * kChunks * 32 * 4);
  w.apart = take(static_cast<size_t>(d->num_kv_heads) * g->attn_chunks * G * kAttnPart * 4);
  w.pqkv = take(static_cast<size_t>(g->sq.rbs) * 16 * 8 * 4);
  w.po = take(static_cast<size_t>(d->hidden) * 8 * 4);
  w.pgu = take(static_cast<size_t>(d->inter) * 16 * 4);
  w.pdn = take(static_cast<size_t>(d->hidden) * 8 * 4);
  w.total = off;
  return SB_OK;
}



}  // namespace step
}  // namespace sb

using namespace sb;
using namespace sb::step;

extern "C" size_t sb_step_status_offset(void) { return kHdrBytes; }

extern "C" int sb_step_trace_slots(int num_layers) {
  return num_layers * (kMarksPerLayer + kAttnMarks) + 2 + kTlSlots;
}

extern "C" size_t sb_step_workspace_size(const sb_step_desc* d) {
  Geometry g;
  if (geometry(d, &g) != SB_OK) return 0;
  return g.ws.total;
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
  SB_REQUIRE(d->workspace != nullptr && d->workspace_bytes >= g.ws.total, "workspace too small");
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
  p.status = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(d->workspace) + kHdrBytes);
  p.hdr = ws;
  uint8_t* wb = static_cast<uint8_t*>(d->workspace);
  p.gcount = reinterpret_cast<unsigned*>(wb + g.ws.gcount);
  p.acount = reinterpret_cast<unsigned*>(wb + g.ws.acount);
  p.gpart = reinterpret_cast<float*>(wb + g.ws.gpart);
  p.apart = reinterpret_cast<float*>(wb + g.ws.apart);
  p.pqkv = reinterpret_cast<float*>(wb + g.ws.pqkv);
  p.po = reinterpret_cast<float*>(wb + g.ws.po);
  p.pgu = reinterpret_cast<float*>(wb + g.ws.pgu);
  p.pdn = reinterpret_cast<float*>(wb + g.ws.pdn);
  p.attn_max_chunks = g.attn_chunks;
  p.sq = g.sq;
  p.so = g.so;
  p.sgu = g.sgu;
  p.sdn = g.sdn;
  p.slm = g.slm;
  p.slot_bytes = g.slot_bytes;
  p.trace = d->trace;
  p.trace_slots = sb_step_trace_slots(d->num_layers);
  int max_smem = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  {
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, step_kernel) == cudaSuccess) max_smem -= static_cast<int>(fa.sharedSizeBytes);
  }
  const int fixed = kOffRing + 1024;  // + alignment slack
  p.slots = std::min(kMaxSlots, (max_smem - fixed) / g.slot_bytes);
  SB_REQUIRE(p.slots >= 4, "not enough shared memory for the weight ring");
  const size_t smem = static_cast<size_t>(fixed) + static_cast<size_t>(p.slots) * g.slot_bytes;
  {
    // the attributes are per function and device: set them once per device index
    static std::atomic<int> attr_done[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attr_done[dev].load(std::memory_order_relaxed)) {
      cudaError_t attr_err = cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
      if (attr_err == cudaSuccess)
        attr_err = cudaFuncSetAttribute(step_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                        cudaSharedmemCarveoutMaxShared);
      if (attr_err != cudaSuccess)
        return fail(SB_ECUDA, std::string("step kernel attribute: ") + cudaGetErrorString(attr_err));
      if (dev >= 0 && dev < 64) attr_done[dev].store(1, std::memory_order_relaxed);
    }
  }
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
  // the header counters start at zero for every step (the status word after the header persists)
  cudaError_t err = cudaMemsetAsync(d->workspace, 0, kHdrBytes, as_stream(stream));
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
