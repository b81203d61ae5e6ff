// INT8-KV multi-query (prefill) attention and the batched-prompt helpers for sm_100a.
//
// Reference: the prefill route of int8_quantized_sdpa
// (extensions/spark-mlx-ext/spark_mlx_ext/int8_quantized_sdpa_prefill.py:44-57,
// kernel _int8_prefill_sources.py:7-154: query rows interleaved across the GQA
// heads share each KV tile; QK, online softmax and PV in one dispatch; fp32
// scores, normalizers and accumulators) and its staged recipe
// int8_quantized_sdpa.py:122-153 (bottom-right causal mask: query l of L sees
// keys [0, N - L + l]). KV format here: the BASELINE int8 codes [B, KH, cap, D]
// with one fp16 scale per token per head (K = code * scale), D = 128.
//
// Design (B200): one CTA = 64 query rows (position-major, the G heads of a KV
// head interleaved) x one KV head; four warps of 16 rows. KV tiles of 64
// tokens stream through a double-buffered shared-memory stage (cp.async), are
// converted once per CTA to fp16 codes (exact: |code| <= 127) and read by the
// tensor cores (mma.sync m16n8k16, fp16 operands, fp32 accumulators) through
// ldmatrix (K as the column-major B of QK^T, V transposed by ldmatrix.trans
// for PV). The K scale multiplies each score column, the V scale each
// probability before it is rounded to fp16 for PV; softmax is online in fp32
// (exp2 with log2 e folded into the score scale). Tiles past a CTA's last
// query position are skipped (causal), the diagonal tile is masked per row.
#include <algorithm>
#include <cmath>
#include <string>

#include "sb_common.cuh"
#include "spark_b200_decoder.h"

namespace sb {
namespace prefill {

constexpr int kRows = 64;        // query rows per CTA
constexpr int kWarps = 4;        // 16 query rows each
constexpr int kThreads = kWarps * 32;

// Per head dimension D (128 or 256): keys per tile (64 at 128; 32 at 256, where
// a warp's 16 x 256 fp32 accumulator alone takes 128 registers), the 16-bit tile
// row stride (bytes; ldmatrix without bank conflicts) and the shared-memory
// layout. At 256 the query tile stays in shared memory and each k step reads its
// fragments with ldmatrix instead of holding all of them in registers.
template <int D>
struct Geo {
  static constexpr int kKeys = D == 128 ? 64 : 32;
  static constexpr bool kQSmem = D > 128;
  static constexpr int kHStride = D * 2 + 16;
  static constexpr int kHTile = kKeys * kHStride;  // one 16-bit tile (K or V)
  static constexpr int kRawTile = kKeys * D;       // one int8 tile (K or V)
  static constexpr int kQTile = kQSmem ? kRows * kHStride : 0;
  // INT8 KV: [K | V] 16-bit code tiles, [2 buffers][K | V] int8 tiles, the
  // tile's K and V scales (fp32), [the query tile]
  static constexpr int kOffKh = 0;
  static constexpr int kOffVh = kHTile;
  static constexpr int kOffRaw = 2 * kHTile;
  static constexpr int kOffScale = kOffRaw + 2 * 2 * kRawTile;
  static constexpr int kOffQI8 = kOffScale + 2 * kKeys * 4;
  static constexpr int kSmemI8 = kOffQI8 + kQTile;
  // bf16 KV: [2 buffers][K | V] bf16 tiles (loaded straight into the padded layout), [the query tile]
  static constexpr int kOffQBf = 2 * 2 * kHTile;
  static constexpr int kSmemBf = kOffQBf + kQTile;
};

struct Params {
  const __nv_bfloat16* q;
  const void* k;  // int8 codes or bf16 values [B, KH, cap, D]
  const __half* ks;
  const void* v;
  const __half* vs;
  __nv_bfloat16* out;
  const uint8_t* mask;  // optional [q_len, mask_ld] bytes, nonzero = visible (broadcast over batch and heads)
  int mask_ld;
  int heads, kv_heads, q_len, length, capacity;
  int causal, window, layout;  // window > 0: keys (pos - window, pos] (with causal); layout 0: [B, H, L, D], 1: [B, L, H, D]
  float scale_log2;            // softmax scale * log2(e)
  int tiles;                   // query tiles per (batch, kv head)
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit_group() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// Four int8 codes (one 32-bit word) -> two fp16x2 words of the same values, exactly:
// byte b = code + 128 under the fp16 exponent of 1024 is 1024 + b; minus 1152.
__device__ __forceinline__ void codes_to_half(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  const __half2 off = __floats2half2_rn(1152.f, 1152.f);
  const uint32_t a = prmt(u, 0x64646464u, 0x4140u), b = prmt(u, 0x64646464u, 0x4342u);
  const __half2 ha = __hsub2(*reinterpret_cast<const __half2*>(&a), off);
  const __half2 hb = __hsub2(*reinterpret_cast<const __half2*>(&b), off);
  lo = *reinterpret_cast<const uint32_t*>(&ha);
  hi = *reinterpret_cast<const uint32_t*>(&hb);
}

// KVB: bf16 K/V (no scales; bf16 operands, probabilities as a bf16 hi + lo pair for P.V);
// else INT8 codes + fp16 scales (fp16 code tiles, probabilities times the V scale in fp16).
template <int G, bool KVB, int D>
__global__ void __launch_bounds__(kThreads) prefill_kernel(const __grid_constant__ Params p) {
  using C = Geo<D>;
  constexpr int kD = D, kKeys = C::kKeys, kHStride = C::kHStride, kHTile = C::kHTile, kRawTile = C::kRawTile;
  constexpr int kOffKh = C::kOffKh, kOffVh = C::kOffVh, kOffRaw = C::kOffRaw, kOffScale = C::kOffScale;
  extern __shared__ __align__(128) uint8_t sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int g = lane >> 2, c = lane & 3;
  const int tile = p.tiles - 1 - static_cast<int>(blockIdx.x);  // latest (longest) query tiles first
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int nrows = p.q_len * G;  // query row r = l * G + (head in group)
  const int row0 = tile * kRows;
  const int qoff = p.length - p.q_len;  // position of query l is qoff + l (bottom-right)
  const int last_row = min(row0 + kRows, nrows) - 1;
  // keys this CTA reads: [kbeg, kend)
  const int kend = p.causal ? min(p.length, qoff + last_row / G + 1) : p.length;
  const int kbeg = p.window > 0 ? max(0, qoff + row0 / G - p.window + 1) : 0;
  const int kt0 = kbeg / kKeys;
  const int ntiles = (kend + kKeys - 1) / kKeys;
  const size_t head_base = (static_cast<size_t>(b) * p.kv_heads + kvh) * p.capacity;
  const uint8_t* kbase = static_cast<const uint8_t*>(p.k) + head_base * kD * (KVB ? 2 : 1);
  const uint8_t* vbase = static_cast<const uint8_t*>(p.v) + head_base * kD * (KVB ? 2 : 1);
  float* sks = reinterpret_cast<float*>(sm + kOffScale);
  float* svs = sks + kKeys;

  // this warp's two rows per lane (g, g + 8) and their positions / pointers
  const int wr0 = row0 + warp * 16;
  const int ra = wr0 + g, rb = ra + 8;
  auto qkv_offset = [&](int r) -> size_t {
    const int l = r / G, head = kvh * G + r % G;
    return p.layout == 0 ? ((static_cast<size_t>(b) * p.heads + head) * p.q_len + l) * kD
                         : ((static_cast<size_t>(b) * p.q_len + l) * p.heads + head) * kD;
  };
  const int la = ra / G, lb = rb / G;
  const int pos_a = qoff + la, pos_b = qoff + lb;
  const int kend_a = p.causal ? min(p.length, pos_a + 1) : p.length;
  const int kend_b = p.causal ? min(p.length, pos_b + 1) : p.length;
  const int kbeg_a = p.window > 0 ? pos_a - p.window + 1 : 0;
  const int kbeg_b = p.window > 0 ? pos_b - p.window + 1 : 0;
  const uint8_t* mrow_a = (p.mask && la < p.q_len) ? p.mask + static_cast<size_t>(la) * p.mask_ld : nullptr;
  const uint8_t* mrow_b = (p.mask && lb < p.q_len) ? p.mask + static_cast<size_t>(lb) * p.mask_ld : nullptr;
  const int warp_last = qoff + min(wr0 + 15, nrows - 1) / G;  // latest position among the warp's rows
  const int warp_first = qoff + wr0 / G;
  const bool warp_live = wr0 < nrows;

  grid_dependency_wait();

  auto load_tile = [&](int kt, int buf) {
    const int key0 = kt * kKeys;
    if constexpr (KVB) {
      uint8_t* dst0 = sm + buf * 2 * kHTile;
      for (int i = tid; i < 2 * kKeys * (kD * 2 / 16); i += kThreads) {
        const int mat = i / (kKeys * (kD * 2 / 16)), rem = i % (kKeys * (kD * 2 / 16));
        const int key = rem / (kD * 2 / 16), ch = rem % (kD * 2 / 16);
        uint8_t* dst = dst0 + mat * kHTile + key * kHStride + ch * 16;
        if (key0 + key < kend && key0 + key >= kbeg)
          cp_async16(dst, (mat ? vbase : kbase) + static_cast<size_t>(key0 + key) * kD * 2 + ch * 16);
        else
          *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
      }
    } else {
      int8_t* rk = reinterpret_cast<int8_t*>(sm + kOffRaw + buf * 2 * kRawTile);
      for (int i = tid; i < 2 * kKeys * (kD / 16); i += kThreads) {
        const int mat = i / (kKeys * (kD / 16)), rem = i % (kKeys * (kD / 16));
        const int key = rem / (kD / 16), ch = rem % (kD / 16);
        int8_t* dst = rk + mat * kRawTile + key * kD + ch * 16;
        if (key0 + key < kend && key0 + key >= kbeg)
          cp_async16(dst, (mat ? vbase : kbase) + static_cast<size_t>(key0 + key) * kD + ch * 16);
        else
          *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    cp_async_commit_group();
  };

  // q rows of the warp as A fragments (fp16 for INT8 KV, bf16 as stored for bf16 KV;
  // rows beyond the query count are zero): in registers at D = 128, else the
  // CTA's query tile in shared memory (the same values, read per k step)
  uint32_t qa[C::kQSmem ? 1 : kD / 16][4];
  const uint32_t q_base = smem_u32(sm + (KVB ? C::kOffQBf : C::kOffQI8));
  if constexpr (C::kQSmem) {
    uint8_t* qs = sm + (KVB ? C::kOffQBf : C::kOffQI8);
    for (int i = tid; i < kRows * (kD / 8); i += kThreads) {
      const int r = i / (kD / 8), ch = i % (kD / 8);
      uint4 w = make_uint4(0u, 0u, 0u, 0u);
      if (row0 + r < nrows) w = *reinterpret_cast<const uint4*>(p.q + qkv_offset(row0 + r) + ch * 8);
      if constexpr (!KVB) {
        w.x = pack_half2(bf16_lo(w.x), bf16_hi(w.x));
        w.y = pack_half2(bf16_lo(w.y), bf16_hi(w.y));
        w.z = pack_half2(bf16_lo(w.z), bf16_hi(w.z));
        w.w = pack_half2(bf16_lo(w.w), bf16_hi(w.w));
      }
      *reinterpret_cast<uint4*>(qs + r * kHStride + ch * 16) = w;  // read after the loop's first barrier
    }
  } else {
    const __nv_bfloat16* qra = ra < nrows ? p.q + qkv_offset(ra) : nullptr;
    const __nv_bfloat16* qrb = rb < nrows ? p.q + qkv_offset(rb) : nullptr;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int d = ks * 16 + h * 8 + 2 * c;
        const uint32_t wa = qra ? *reinterpret_cast<const uint32_t*>(qra + d) : 0u;
        const uint32_t wb = qrb ? *reinterpret_cast<const uint32_t*>(qrb + d) : 0u;
        qa[ks][2 * h] = KVB ? wa : pack_half2(bf16_lo(wa), bf16_hi(wa));
        qa[ks][2 * h + 1] = KVB ? wb : pack_half2(bf16_lo(wb), bf16_hi(wb));
      }
  }
  float o[kD / 8][4];
#pragma unroll
  for (int n = 0; n < kD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

  if (kt0 < ntiles) load_tile(kt0, kt0 & 1);
  for (int kt = kt0; kt < ntiles; ++kt) {
    const int key0 = kt * kKeys;
    if (kt + 1 < ntiles) load_tile(kt + 1, (kt + 1) & 1);
    else cp_async_commit_group();  // an empty group keeps the wait count uniform
    cp_async_wait_group<1>();
    __syncthreads();
    uint32_t kh_base, vh_base;
    if constexpr (KVB) {
      kh_base = smem_u32(sm + (kt & 1) * 2 * kHTile);
      vh_base = kh_base + kHTile;
    } else {
      // ---- int8 tile -> fp16 codes (exact), and the tile's scales
      const int8_t* rk = reinterpret_cast<const int8_t*>(sm + kOffRaw + (kt & 1) * 2 * kRawTile);
      for (int i = tid; i < 2 * kKeys * (kD / 16); i += kThreads) {
        const int mat = i / (kKeys * (kD / 16)), rem = i % (kKeys * (kD / 16));
        const int key = rem / (kD / 16), ch = rem % (kD / 16);
        const uint4 w = *reinterpret_cast<const uint4*>(rk + mat * kRawTile + key * kD + ch * 16);
        uint32_t h[8];
        codes_to_half(w.x, h[0], h[1]);
        codes_to_half(w.y, h[2], h[3]);
        codes_to_half(w.z, h[4], h[5]);
        codes_to_half(w.w, h[6], h[7]);
        uint8_t* dst = sm + (mat ? kOffVh : kOffKh) + key * kHStride + ch * 32;
        *reinterpret_cast<uint4*>(dst) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(dst + 16) = make_uint4(h[4], h[5], h[6], h[7]);
      }
      if (tid < 2 * kKeys) {
        const int key = key0 + (tid & (kKeys - 1));
        const __half* src = tid < kKeys ? p.ks : p.vs;
        const float sc = (key < kend && key >= kbeg) ? __half2float(src[head_base + key]) : 0.f;
        (tid < kKeys ? sks : svs)[tid & (kKeys - 1)] = sc;
      }
      __syncthreads();
      kh_base = smem_u32(sm + kOffKh);
      vh_base = smem_u32(sm + kOffVh);
    }
    // a warp skips the tiles its rows cannot see: past its last position (causal)
    // or before its first window (sliding); without the causal mask every tile counts
    if (warp_live && (!p.causal || key0 <= warp_last) &&
        (p.window <= 0 || key0 + kKeys > warp_first - p.window + 1)) {
      // ---- scores S = q . K^T for the warp's 16 rows x 64 keys
      float s[kKeys / 8][4];
#pragma unroll
      for (int nt = 0; nt < kKeys / 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
      for (int ks2 = 0; ks2 < kD / 32; ++ks2) {
        uint32_t qf[2][4];
        if constexpr (C::kQSmem) {
#pragma unroll
          for (int h = 0; h < 2; ++h)
            ldsm_x4(qf[h], q_base + (warp * 16 + (lane & 15)) * kHStride + ((2 * ks2 + h) * 16 + (lane >> 4) * 8) * 2);
        }
#pragma unroll
        for (int nt = 0; nt < kKeys / 8; ++nt) {
          uint32_t bk[4];
          ldsm_x4(bk, kh_base + (nt * 8 + (lane & 7)) * kHStride + (ks2 * 32 + (lane >> 3) * 8) * 2);
          if constexpr (C::kQSmem) {
            mma_16816<!KVB>(s[nt], qf[0], bk[0], bk[1]);
            mma_16816<!KVB>(s[nt], qf[1], bk[2], bk[3]);
          } else {
            mma_16816<!KVB>(s[nt], qa[2 * ks2], bk[0], bk[1]);
            mma_16816<!KVB>(s[nt], qa[2 * ks2 + 1], bk[2], bk[3]);
          }
        }
      }
      // ---- scale, mask, online softmax (log2 domain)
      float mx[2] = {m_run[0], m_run[1]};
#pragma unroll
      for (int nt = 0; nt < kKeys / 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int kk = nt * 8 + 2 * c + (e & 1);
          const int key = key0 + kk;
          const bool row_a = e < 2;
          const uint8_t* mrow = row_a ? mrow_a : mrow_b;
          const bool ok = key < (row_a ? kend_a : kend_b) && key >= (row_a ? kbeg_a : kbeg_b) &&
                          (mrow == nullptr || mrow[key] != 0);
          const float v = KVB ? s[nt][e] * p.scale_log2 : s[nt][e] * sks[kk] * p.scale_log2;
          s[nt][e] = ok ? v : -INFINITY;
          mx[e >> 1] = fmaxf(mx[e >> 1], s[nt][e]);
        }
      float corr[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
        mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
        corr[i] = mx[i] == -INFINITY ? 1.f : exp2f(m_run[i] - mx[i]);
        m_run[i] = mx[i];
        l_run[i] *= corr[i];
      }
#pragma unroll
      for (int n = 0; n < kD / 8; ++n) {
        o[n][0] *= corr[0];
        o[n][1] *= corr[0];
        o[n][2] *= corr[1];
        o[n][3] *= corr[1];
      }
      // probabilities as the A operand of P.V
      uint32_t pa[kKeys / 16][4], pl[kKeys / 16][4];
#pragma unroll
      for (int nt = 0; nt < kKeys / 8; ++nt) {
        float pr[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float mrow = m_run[e >> 1];
          const float pe = s[nt][e] == -INFINITY ? 0.f : exp2f(s[nt][e] - mrow);
          l_run[e >> 1] += pe;
          pr[e] = KVB ? pe : pe * svs[nt * 8 + 2 * c + (e & 1)];
        }
        if constexpr (KVB) {
          // P = hi + lo in bf16 (about 16 significant bits)
          const __nv_bfloat162 h01 = __floats2bfloat162_rn(pr[0], pr[1]), h23 = __floats2bfloat162_rn(pr[2], pr[3]);
          const __nv_bfloat162 l01 = __floats2bfloat162_rn(pr[0] - __low2float(h01), pr[1] - __high2float(h01));
          const __nv_bfloat162 l23 = __floats2bfloat162_rn(pr[2] - __low2float(h23), pr[3] - __high2float(h23));
          pa[nt >> 1][(nt & 1) * 2] = *reinterpret_cast<const uint32_t*>(&h01);
          pa[nt >> 1][(nt & 1) * 2 + 1] = *reinterpret_cast<const uint32_t*>(&h23);
          pl[nt >> 1][(nt & 1) * 2] = *reinterpret_cast<const uint32_t*>(&l01);
          pl[nt >> 1][(nt & 1) * 2 + 1] = *reinterpret_cast<const uint32_t*>(&l23);
        } else {
          pa[nt >> 1][(nt & 1) * 2] = pack_half2(pr[0], pr[1]);
          pa[nt >> 1][(nt & 1) * 2 + 1] = pack_half2(pr[2], pr[3]);
        }
      }
      // ---- O += P . V (V transposed by ldmatrix.trans)
#pragma unroll
      for (int j = 0; j < kKeys / 16; ++j)
#pragma unroll
        for (int np = 0; np < kD / 16; ++np) {
          uint32_t bv[4];
          ldsm_x4_trans(bv, vh_base + (j * 16 + ((lane >> 3) & 1) * 8 + (lane & 7)) * kHStride +
                                (np * 16 + (lane >> 4) * 8) * 2);
          mma_16816<!KVB>(o[2 * np], pa[j], bv[0], bv[1]);
          mma_16816<!KVB>(o[2 * np + 1], pa[j], bv[2], bv[3]);
          if constexpr (KVB) {
            mma_16816<false>(o[2 * np], pl[j], bv[0], bv[1]);
            mma_16816<false>(o[2 * np + 1], pl[j], bv[2], bv[3]);
          }
        }
    }
    __syncthreads();  // the tiles and scales are rewritten by the next tile
  }
  cp_async_wait_group<0>();
  // ---- normalize and store (rows past the query count are not stored; fully masked rows are 0)
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    l_run[i] += __shfl_xor_sync(0xffffffffu, l_run[i], 1);
    l_run[i] += __shfl_xor_sync(0xffffffffu, l_run[i], 2);
  }
  if (!warp_live) return;
  const float inv_a = l_run[0] > 0.f ? 1.0f / l_run[0] : 0.f;
  const float inv_b = l_run[1] > 0.f ? 1.0f / l_run[1] : 0.f;
  __nv_bfloat16* oa = ra < nrows ? p.out + qkv_offset(ra) : nullptr;
  __nv_bfloat16* ob = rb < nrows ? p.out + qkv_offset(rb) : nullptr;
#pragma unroll
  for (int n = 0; n < kD / 8; ++n) {
    const int d = n * 8 + 2 * c;
    if (oa) *reinterpret_cast<__nv_bfloat162*>(oa + d) = __floats2bfloat162_rn(o[n][0] * inv_a, o[n][1] * inv_a);
    if (ob) *reinterpret_cast<__nv_bfloat162*>(ob + d) = __floats2bfloat162_rn(o[n][2] * inv_b, o[n][3] * inv_b);
  }
}

// ------------------------------------------- batched prompt: RoPE + split + KV append
// One warp per (token m, head j of the H + 2 KH heads of a QKV projection row):
// query heads rotate into q_out [M, H, D]; key heads rotate and, like value
// heads, are quantized into the INT8 cache at the token's position. The
// arithmetic is the single-token path's (the QKV projection's bf16 outputs are
// rotated in fp32 with sincosf(pos * inv_freq[i]) and stored as bf16; K/V rows
// are quantized from those bf16 values with fp16 scale = absmax / 127, 1 for a
// zero row, code = clamp(rint(x / scale), -127, 127)).
struct RopeParams {
  const __nv_bfloat16* qkv;
  int64_t ld;  // qkv row stride (elements)
  const int32_t* positions;
  __nv_bfloat16* q_out;
  int8_t* k_cache;
  __half* k_scale;
  int8_t* v_cache;
  __half* v_scale;
  int rows, seq_len, heads, kv_heads, capacity, rope_pairs;
  int ring;  // > 0: the cache rows are a ring of `ring` slots (position p -> slot p % ring)
  float inv_freq[128];  // theta^(-2i / rope_dims), i < rope_pairs
};

// One warp per (row, head) of the projected qkv: RoPE on the first 2 * rope_pairs
// features of q and k heads (non-traditional: feature e < rope_pairs pairs with
// e + rope_pairs), the rest unchanged; q heads to q_out, k/v heads quantized into
// the INT8 cache (symmetric per token and head, fp16 scale = absmax / 127).
template <int D>
__global__ void rope_append_kernel(const __grid_constant__ RopeParams p) {
  constexpr int E = D / 32;  // features per lane: e = lane + 32 t
  grid_dependency_wait();
  const int lane = threadIdx.x & 31;
  const int nh = p.heads + 2 * p.kv_heads;
  const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item >= p.rows * nh) return;
  const int m = item / nh, j = item % nh;
  const int bi = m / p.seq_len;
  const int pos = p.positions[m];
  const __nv_bfloat16* src = p.qkv + static_cast<size_t>(m) * p.ld + static_cast<size_t>(j) * D;
  const int half = p.rope_pairs;
  float v[E];
#pragma unroll
  for (int t = 0; t < E; ++t) v[t] = __bfloat162float(src[lane + 32 * t]);
  if (j < p.heads + p.kv_heads) {
#pragma unroll
    for (int t = 0; t < E; ++t) {
      const int e = lane + 32 * t;
      if (e >= 2 * half) continue;
      const bool lo = e < half;
      const int i = lo ? e : e - half;  // rotation pair (i, i + half)
      const float o = __bfloat162float(src[lo ? e + half : e - half]);
      float sn, cs;
      sincosf(static_cast<float>(pos) * p.inv_freq[i], &sn, &cs);
      const float r = lo ? v[t] * cs - o * sn : v[t] * cs + o * sn;
      v[t] = __bfloat162float(__float2bfloat16_rn(r));
    }
  }
  if (j < p.heads) {
    __nv_bfloat16* dst = p.q_out + (static_cast<size_t>(m) * p.heads + j) * D;
#pragma unroll
    for (int t = 0; t < E; ++t) dst[lane + 32 * t] = __float2bfloat16_rn(v[t]);
    return;
  }
  const bool is_k = j < p.heads + p.kv_heads;
  const int h = is_k ? j - p.heads : j - p.heads - p.kv_heads;
  if (pos < 0 || (p.ring == 0 && pos >= p.capacity)) return;  // never write outside the cache
  const int slot = p.ring > 0 ? pos % p.ring : pos;
  float amax = 0.f;
#pragma unroll
  for (int t = 0; t < E; ++t) amax = fmaxf(amax, fabsf(v[t]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  __half s16 = __float2half_rn(__fdiv_rn(amax, 127.0f));
  if (__half2float(s16) == 0.f) s16 = __float2half_rn(1.0f);
  const float sc = __half2float(s16);
  const size_t row = (static_cast<size_t>(bi) * p.kv_heads + h) * p.capacity + slot;
  int8_t* dst = (is_k ? p.k_cache : p.v_cache) + row * D;
#pragma unroll
  for (int t = 0; t < E; ++t)
    dst[lane + 32 * t] = static_cast<int8_t>(static_cast<int>(fminf(fmaxf(rintf(__fdiv_rn(v[t], sc)), -127.f), 127.f)));
  if (lane == 0) (is_k ? p.k_scale : p.v_scale)[row] = s16;
}

// ------------------------------------------------- gated activations (elementwise)
// out = bf16(act(g) * u) with g, u the bf16 gate / up projections and act SiLU
// (act 0) or the exact GELU (act 1) - the single-token path's fused gate/up
// epilogue (sb_gemv.cu EPI_SWIGLU).
__device__ __forceinline__ float gate_act(float g, int act) {
  return act ? 0.5f * g * (1.0f + erff(g * 0.70710678118654752f)) : g / (1.0f + expf(-g));
}

__global__ void swiglu_kernel(const __nv_bfloat16* __restrict__ gate, const __nv_bfloat16* __restrict__ up,
                              __nv_bfloat16* __restrict__ out, int64_t count, int act) {
  grid_dependency_wait();
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (i >= count) return;
  if (i + 8 <= count) {
    const uint4 gv = *reinterpret_cast<const uint4*>(gate + i), uv = *reinterpret_cast<const uint4*>(up + i);
    const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
    uint32_t r[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float o2[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float g = e ? bf16_hi(gw[k]) : bf16_lo(gw[k]);
        const float u = e ? bf16_hi(uw[k]) : bf16_lo(uw[k]);
        o2[e] = gate_act(g, act) * u;
      }
      const __nv_bfloat162 h = __floats2bfloat162_rn(o2[0], o2[1]);
      r[k] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(out + i) = make_uint4(r[0], r[1], r[2], r[3]);
  } else {
    for (int64_t k = i; k < count; ++k) {
      const float g = __bfloat162float(gate[k]), u = __bfloat162float(up[k]);
      out[k] = __float2bfloat16_rn(gate_act(g, act) * u);
    }
  }
}

// --------------------------------------------------------- attention-output head gate
// One warp per (row m, head h): the reference's sigmoid head gate
// (spark_mlx_llm/ops/attention_output.py:91-95): d = bf16(x[m] . gate_w[h]) (fp32
// accumulation), gate = bf16(sigmoid(d)) in fp32, out[m, h, :] = bf16(attn[m, h, :] * gate).
__global__ void head_gate_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                 const __nv_bfloat16* attn, __nv_bfloat16* out, int rows, int hidden, int heads,
                                 int head_dim) {
  grid_dependency_wait();
  const int lane = threadIdx.x & 31;
  const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item >= rows * heads) return;
  const int m = item / heads, h = item % heads;
  const __nv_bfloat16* xr = x + static_cast<size_t>(m) * hidden;
  const __nv_bfloat16* wr = w + static_cast<size_t>(h) * hidden;
  float acc = 0.f;
  for (int k = lane * 8; k < hidden; k += 256) {
    const uint4 xa = *reinterpret_cast<const uint4*>(xr + k), wa = *reinterpret_cast<const uint4*>(wr + k);
    const uint32_t xs[4] = {xa.x, xa.y, xa.z, xa.w}, ws[4] = {wa.x, wa.y, wa.z, wa.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc = fmaf(bf16_lo(xs[i]), bf16_lo(ws[i]), acc);
      acc = fmaf(bf16_hi(xs[i]), bf16_hi(ws[i]), acc);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  const float d = __bfloat162float(__float2bfloat16_rn(acc));
  const float gate = __bfloat162float(__float2bfloat16_rn(1.0f / (1.0f + expf(-d))));
  const size_t base = (static_cast<size_t>(m) * heads + h) * head_dim;
  for (int i = lane; i < head_dim; i += 32) out[base + i] = __float2bfloat16_rn(__bfloat162float(attn[base + i]) * gate);
}

}  // namespace prefill
}  // namespace sb

using namespace sb;
using namespace sb::prefill;

namespace {

template <int G, bool KVB, int D>
int launch_prefill(const Params& p, int batch, int kv_heads, cudaStream_t stream) {
  constexpr int smem = KVB ? Geo<D>::kSmemBf : Geo<D>::kSmemI8;
  // the shared-memory opt-in is per function and device: once per device index
  static std::atomic<int> attr_done[64];
  int dev = 0;
  cudaGetDevice(&dev);
  const bool cached = dev >= 0 && dev < 64 && attr_done[dev].load(std::memory_order_relaxed);
  if (!cached) {
    const cudaError_t e =
        cudaFuncSetAttribute(prefill_kernel<G, KVB, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return fail(SB_ECUDA, std::string("prefill attention attribute: ") + cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) attr_done[dev].store(1, std::memory_order_relaxed);
  }
  return launch(KVB ? "bf16_sdpa_multiquery" : "int8_sdpa_prefill", prefill_kernel<G, KVB, D>,
                dim3(p.tiles, kv_heads, batch), dim3(kThreads), smem, stream, p);
}

template <bool KVB>
int launch_any(Params& p, int64_t batch, int num_kv_heads, int G, int64_t q_len, int head_dim, cudaStream_t s) {
  const int64_t tiles = (q_len * G + kRows - 1) / kRows;
  SB_REQUIRE(tiles <= 0x7fffffff, "too many query rows");
  p.tiles = static_cast<int>(tiles);
  const int b = static_cast<int>(batch);
  if (head_dim == 256) {
    switch (G) {
      case 1: return launch_prefill<1, KVB, 256>(p, b, num_kv_heads, s);
      case 2: return launch_prefill<2, KVB, 256>(p, b, num_kv_heads, s);
      case 4: return launch_prefill<4, KVB, 256>(p, b, num_kv_heads, s);
      default: return launch_prefill<8, KVB, 256>(p, b, num_kv_heads, s);
    }
  }
  switch (G) {
    case 1: return launch_prefill<1, KVB, 128>(p, b, num_kv_heads, s);
    case 2: return launch_prefill<2, KVB, 128>(p, b, num_kv_heads, s);
    case 4: return launch_prefill<4, KVB, 128>(p, b, num_kv_heads, s);
    default: return launch_prefill<8, KVB, 128>(p, b, num_kv_heads, s);
  }
}

// Checks shared by both entry points; fills the common fields.
int common_params(Params& p, const void* q, const void* k, const void* v, void* out, int64_t batch, int num_heads,
                  int num_kv_heads, int64_t q_len, int64_t length, int64_t capacity, int head_dim, float scale,
                  int causal, int layout) {
  SB_REQUIRE(q && k && v && out, "null pointer");
  SB_REQUIRE(head_dim == 128 || head_dim == 256, "head_dim must be 128 or 256");
  SB_REQUIRE(batch >= 1 && batch <= 65535, "batch must be in [1, 65535]");
  SB_REQUIRE(num_kv_heads >= 1 && num_kv_heads <= 65535 && num_heads % num_kv_heads == 0, "heads");
  const int G = num_heads / num_kv_heads;
  SB_REQUIRE(G == 1 || G == 2 || G == 4 || G == 8, "query heads per KV head must be 1, 2, 4 or 8");
  SB_REQUIRE(q_len >= 1 && q_len <= length && length <= capacity && capacity <= (1LL << 30),
             "need 1 <= q_len <= length <= capacity");
  SB_REQUIRE(layout == 0 || layout == 1, "layout must be 0 ([B,H,L,D]) or 1 ([B,L,H,D])");
  SB_REQUIRE(reinterpret_cast<uintptr_t>(k) % 16 == 0 && reinterpret_cast<uintptr_t>(v) % 16 == 0,
             "the K/V caches must be 16-byte aligned");
  SB_REQUIRE(reinterpret_cast<uintptr_t>(q) % 4 == 0 && reinterpret_cast<uintptr_t>(out) % 4 == 0,
             "q and out must be 4-byte aligned");
  SB_REQUIRE(head_dim == 128 || reinterpret_cast<uintptr_t>(q) % 16 == 0, "q must be 16-byte aligned at head_dim 256");
  p = Params{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = k;
  p.v = v;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.heads = num_heads;
  p.kv_heads = num_kv_heads;
  p.q_len = static_cast<int>(q_len);
  p.length = static_cast<int>(length);
  p.capacity = static_cast<int>(capacity);
  p.causal = causal != 0;
  p.layout = layout;
  p.scale_log2 = scale * 1.4426950408889634f;
  return SB_OK;
}

}  // namespace

extern "C" int sb_int8_sdpa_prefill(const void* q, const int8_t* k, const void* k_scale, const int8_t* v,
                                    const void* v_scale, void* out, int64_t batch, int num_heads, int num_kv_heads,
                                    int64_t q_len, int64_t length, int64_t capacity, int head_dim, float scale,
                                    int causal, int layout, void* stream) {
  SB_REQUIRE(k_scale && v_scale, "null pointer");
  Params p;
  if (int st = common_params(p, q, k, v, out, batch, num_heads, num_kv_heads, q_len, length, capacity, head_dim,
                             scale, causal, layout))
    return st;
  p.ks = static_cast<const __half*>(k_scale);
  p.vs = static_cast<const __half*>(v_scale);
  return launch_any<false>(p, batch, num_kv_heads, num_heads / num_kv_heads, q_len, head_dim, as_stream(stream));
}

extern "C" int sb_int8_sdpa_prefill_window(const void* q, const int8_t* k, const void* k_scale, const int8_t* v,
                                           const void* v_scale, void* out, int64_t batch, int num_heads,
                                           int num_kv_heads, int64_t q_len, int64_t length, int64_t capacity,
                                           int head_dim, float scale, int window, int layout, void* stream) {
  SB_REQUIRE(k_scale && v_scale, "null pointer");
  SB_REQUIRE(window >= 0, "window must be >= 0");
  Params p;
  if (int st = common_params(p, q, k, v, out, batch, num_heads, num_kv_heads, q_len, length, capacity, head_dim,
                             scale, 1, layout))
    return st;
  p.ks = static_cast<const __half*>(k_scale);
  p.vs = static_cast<const __half*>(v_scale);
  p.window = window;
  return launch_any<false>(p, batch, num_kv_heads, num_heads / num_kv_heads, q_len, head_dim, as_stream(stream));
}

extern "C" int sb_bf16_sdpa_multiquery(const void* q, const void* k, const void* v, void* out, int64_t batch,
                                       int num_heads, int num_kv_heads, int64_t q_len, int64_t length,
                                       int64_t capacity, int head_dim, float scale, int causal, int window,
                                       const uint8_t* mask, int64_t mask_ld, int layout, void* stream) {
  Params p;
  if (int st = common_params(p, q, k, v, out, batch, num_heads, num_kv_heads, q_len, length, capacity, head_dim,
                             scale, causal, layout))
    return st;
  SB_REQUIRE(window >= 0, "window must be >= 0");
  SB_REQUIRE(window == 0 || causal, "a sliding window applies with the causal mask");
  SB_REQUIRE(mask == nullptr || (mask_ld >= length && mask_ld <= (1LL << 30)), "mask row stride must be >= length");
  p.window = window;
  p.mask = mask;
  p.mask_ld = static_cast<int>(mask ? mask_ld : 0);
  return launch_any<true>(p, batch, num_kv_heads, num_heads / num_kv_heads, q_len, head_dim, as_stream(stream));
}

namespace {
int rope_kv_append(const void* qkv, int64_t ld, const int32_t* positions, void* q_out, int8_t* k_cache,
                   void* k_scale, int8_t* v_cache, void* v_scale, int64_t batch, int64_t seq_len, int num_heads,
                   int num_kv_heads, int head_dim, int64_t capacity, int rope_dims, float rope_base, int64_t ring,
                   void* stream) {
  SB_REQUIRE(qkv && positions && q_out && k_cache && k_scale && v_cache && v_scale, "null pointer");
  SB_REQUIRE(head_dim == 64 || head_dim == 128 || head_dim == 256, "head_dim must be 64, 128 or 256");
  SB_REQUIRE(rope_dims >= 2 && rope_dims <= head_dim && rope_dims % 2 == 0, "rope_dims must be even, 2..head_dim");
  SB_REQUIRE(batch >= 1 && seq_len >= 1 && num_heads >= 1 && num_kv_heads >= 1, "shape");
  SB_REQUIRE(ld >= static_cast<int64_t>(num_heads + 2 * num_kv_heads) * head_dim, "qkv row stride too small");
  SB_REQUIRE(capacity >= 1 && capacity <= (1LL << 30), "capacity");
  const int64_t rows = batch * seq_len;
  const int64_t items = rows * (num_heads + 2 * num_kv_heads);
  SB_REQUIRE(items <= (1LL << 31) - 1, "too many rows");
  RopeParams p;
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
  p.ld = ld;
  p.positions = positions;
  p.q_out = static_cast<__nv_bfloat16*>(q_out);
  p.k_cache = k_cache;
  p.k_scale = static_cast<__half*>(k_scale);
  p.v_cache = v_cache;
  p.v_scale = static_cast<__half*>(v_scale);
  p.rows = static_cast<int>(rows);
  p.seq_len = static_cast<int>(seq_len);
  p.heads = num_heads;
  p.kv_heads = num_kv_heads;
  p.capacity = static_cast<int>(capacity);
  p.rope_pairs = rope_dims / 2;
  SB_REQUIRE(ring >= 0 && ring <= capacity, "ring must be 0 (linear cache) or 1..capacity slots");
  SB_REQUIRE(ring == 0 || seq_len <= ring, "a chunk's positions must map to distinct ring slots (seq_len <= ring)");
  p.ring = static_cast<int>(ring);
  for (int i = 0; i < 128; ++i)
    p.inv_freq[i] = i < rope_dims / 2 ? static_cast<float>(std::pow(static_cast<double>(rope_base), -2.0 * i / rope_dims))
                                      : 0.f;
  constexpr int kWarpsPerBlock = 8;
  const dim3 grid(static_cast<unsigned>((items + kWarpsPerBlock - 1) / kWarpsPerBlock)), block(32 * kWarpsPerBlock);
  if (head_dim == 64) return launch("rope_kv_append", rope_append_kernel<64>, grid, block, 0, as_stream(stream), p);
  if (head_dim == 128) return launch("rope_kv_append", rope_append_kernel<128>, grid, block, 0, as_stream(stream), p);
  return launch("rope_kv_append", rope_append_kernel<256>, grid, block, 0, as_stream(stream), p);
}
}  // namespace

extern "C" int sb_rope_kv_append(const void* qkv, int64_t ld, const int32_t* positions, void* q_out,
                                 int8_t* k_cache, void* k_scale, int8_t* v_cache, void* v_scale, int64_t batch,
                                 int64_t seq_len, int num_heads, int num_kv_heads, int head_dim, int64_t capacity,
                                 int rope_dims, float rope_base, void* stream) {
  return rope_kv_append(qkv, ld, positions, q_out, k_cache, k_scale, v_cache, v_scale, batch, seq_len, num_heads,
                        num_kv_heads, head_dim, capacity, rope_dims, rope_base, 0, stream);
}

extern "C" int sb_rope_kv_append_ring(const void* qkv, int64_t ld, const int32_t* positions, void* q_out,
                                      int8_t* k_cache, void* k_scale, int8_t* v_cache, void* v_scale, int64_t batch,
                                      int64_t seq_len, int num_heads, int num_kv_heads, int head_dim,
                                      int64_t capacity, int rope_dims, float rope_base, int64_t ring, void* stream) {
  SB_REQUIRE(ring >= 1, "ring must be at least 1 slot");
  return rope_kv_append(qkv, ld, positions, q_out, k_cache, k_scale, v_cache, v_scale, batch, seq_len, num_heads,
                        num_kv_heads, head_dim, capacity, rope_dims, rope_base, ring, stream);
}

extern "C" int sb_swiglu(const void* gate, const void* up, void* out, int64_t count, void* stream) {
  SB_REQUIRE(gate && up && out, "null pointer");
  SB_REQUIRE(count >= 0, "count");
  if (count == 0) return SB_OK;
  SB_REQUIRE(reinterpret_cast<uintptr_t>(gate) % 16 == 0 && reinterpret_cast<uintptr_t>(up) % 16 == 0 &&
                 reinterpret_cast<uintptr_t>(out) % 16 == 0,
             "gate, up and out must be 16-byte aligned");
  const int64_t threads = (count + 7) / 8;
  return launch("swiglu", swiglu_kernel, dim3(static_cast<unsigned>((threads + 255) / 256)), dim3(256), 0,
                as_stream(stream), static_cast<const __nv_bfloat16*>(gate), static_cast<const __nv_bfloat16*>(up),
                static_cast<__nv_bfloat16*>(out), count, 0);
}

extern "C" int sb_gated_activation(const void* gate, const void* up, void* out, int64_t count, int activation,
                                   void* stream) {
  SB_REQUIRE(gate && up && out, "null pointer");
  SB_REQUIRE(count >= 0, "count");
  SB_REQUIRE(activation == 0 || activation == 1, "activation must be 0 (SiLU) or 1 (GELU)");
  if (count == 0) return SB_OK;
  SB_REQUIRE(reinterpret_cast<uintptr_t>(gate) % 16 == 0 && reinterpret_cast<uintptr_t>(up) % 16 == 0 &&
                 reinterpret_cast<uintptr_t>(out) % 16 == 0,
             "gate, up and out must be 16-byte aligned");
  const int64_t threads = (count + 7) / 8;
  return launch("gated_activation", swiglu_kernel, dim3(static_cast<unsigned>((threads + 255) / 256)), dim3(256), 0,
                as_stream(stream), static_cast<const __nv_bfloat16*>(gate), static_cast<const __nv_bfloat16*>(up),
                static_cast<__nv_bfloat16*>(out), count, activation);
}

extern "C" int sb_head_gate(const void* x, const void* gate_weight, const void* attn, void* out, int64_t rows,
                            int64_t hidden, int num_heads, int head_dim, void* stream) {
  SB_REQUIRE(x && gate_weight && attn && out, "null pointer");
  SB_REQUIRE(rows >= 1 && num_heads >= 1 && head_dim >= 1 && hidden >= 8 && hidden % 8 == 0, "shape");
  SB_REQUIRE(rows * num_heads <= (1LL << 31) - 1 && hidden <= (1LL << 30), "too large");
  SB_REQUIRE(reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(gate_weight) % 16 == 0,
             "x and gate_weight must be 16-byte aligned");
  const int64_t items = rows * num_heads;
  return launch("head_gate", head_gate_kernel, dim3(static_cast<unsigned>((items + 7) / 8)), dim3(256), 0,
                as_stream(stream), static_cast<const __nv_bfloat16*>(x),
                static_cast<const __nv_bfloat16*>(gate_weight), static_cast<const __nv_bfloat16*>(attn),
                static_cast<__nv_bfloat16*>(out), static_cast<int>(rows), static_cast<int>(hidden), num_heads,
                head_dim);
}
