// Shared device/host helpers for the spark_b200 CUDA library (sm_100a).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "spark_b200.h"

namespace sb {

// ---------------------------------------------------------------- host side
void set_error(const std::string& message);
int fail(int status, const std::string& message);
int check_launch(const char* what);

#define SB_REQUIRE(cond, msg)                         \
  do {                                                \
    if (!(cond)) return ::sb::fail(SB_EINVAL, (msg)); \
  } while (0)

inline cudaStream_t as_stream(void* stream) { return static_cast<cudaStream_t>(stream); }

// Multiprocessor count of the current device, cached per device index (one
// process may drive several GPUs with different counts); 148 if the query fails.
inline int device_sm_count() {
  constexpr int kDevs = 64;
  static std::atomic<int> counts[kDevs];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < kDevs) {
    const int cached = counts[dev].load(std::memory_order_relaxed);
    if (cached > 0) return cached;
  }
  int count = 0;
  if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || count <= 0) count = 148;
  if (dev >= 0 && dev < kDevs) counts[dev].store(count, std::memory_order_relaxed);
  return count;
}

// 2-D TMA descriptor over a row-major byte matrix [rows][row_bytes] with a
// [box_rows x 128 B] box and the 128-byte swizzle (16-byte units of row i are
// permuted by XOR with i % 8 in shared memory). Out-of-range reads fill zeros.
int make_tmap_rows(CUtensorMap* map, const void* base, uint64_t rows, uint64_t row_bytes, uint32_t box_rows);
// 2-D TMA descriptor over a row-major uint16 matrix [rows][cols] (no swizzle),
// box [box_rows x box_cols]; out-of-range reads fill zeros.
int make_tmap_u16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_cols,
                  uint32_t box_rows);
// General 2-D TMA descriptor over a row-major matrix [rows][cols] of 1- or
// 2-byte elements with row stride `ld` elements, box [box_rows x box_cols],
// optional 128-byte swizzle (box_cols * elem_bytes must then be 128); reads
// outside the matrix fill zeros.
int make_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t rows, uint64_t cols, uint64_t ld,
                 uint32_t box_cols, uint32_t box_rows, bool swizzle128);

// Every workspace starts with a fixed-size region of arrival counters (zero
// between calls), followed by the call's partial results. The fixed size keeps
// one call's partials from ever overlapping another call's counters when
// different operators share one workspace.
constexpr size_t kCounterBytes = 128 * 1024;
// The last 16 words of the counter region are reserved: word kStatusWord holds
// a device-side status (nonzero when a bounded wait gave up).
constexpr int kMaxCounters = static_cast<int>(kCounterBytes / sizeof(unsigned)) - 16;
constexpr int kStatusWord = static_cast<int>(kCounterBytes / sizeof(unsigned)) - 1;
constexpr unsigned kStatusTimeout = 1u;

// Launch helper: every kernel is launched with programmatic stream
// serialization allowed, so a dependent kernel may start its weight prefetch
// while the previous kernel drains (it waits with griddepcontrol.wait before
// touching the previous kernel's outputs).
template <typename Kernel, typename... Args>
int launch(const char* what, Kernel kernel, dim3 grid, dim3 block, size_t smem,
           cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attr;
  config.numAttrs = 1;
  cudaError_t err = cudaLaunchKernelEx(&config, kernel, args...);
  if (err != cudaSuccess) {
    return fail(SB_ECUDA, std::string(what) + ": " + cudaGetErrorString(err));
  }
  return SB_OK;
}

// Same, with the grid's x dimension grouped into thread-block clusters of
// `cluster_x` CTAs (1 = no cluster attribute).
template <typename Kernel, typename... Args>
int launch_cluster(const char* what, Kernel kernel, dim3 grid, dim3 block, size_t smem, int cluster_x,
                   cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = static_cast<unsigned>(cluster_x);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  config.attrs = attr;
  config.numAttrs = cluster_x > 1 ? 2 : 1;
  cudaError_t err = cudaLaunchKernelEx(&config, kernel, args...);
  if (err != cudaSuccess) {
    return fail(SB_ECUDA, std::string(what) + ": " + cudaGetErrorString(err));
  }
  return SB_OK;
}

// -------------------------------------------------------------- device side
// Wait until the previous kernel in the stream (launched with programmatic
// serialization) has completed and its memory is visible.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
// Allow the next kernel in the stream to begin launching.
__device__ __forceinline__ void grid_dependency_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------ mbarrier + bulk async copy
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
// Waits for the phase with parity `phase`; gives up after ~2^31 clock cycles
// (about a second) and returns false instead of hanging.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t phase) {
  if (mbar_try_wait(bar, phase)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, phase)) {
    if (clock64() - start > (1LL << 31)) return false;
  }
  return true;
}
// 2-D tiled TMA load (no multicast) of one box at (x bytes, y rows) into shared memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// Start fetching a TMA descriptor (kernel parameter) into the descriptor cache,
// so the first copy that uses it does not wait for the fetch.
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// Byte `byte` of row `row` inside a 128-byte-swizzled box.
__device__ __forceinline__ const uint8_t* swz128(const uint8_t* box, int row, int byte) {
  return box + row * 128 + ((((byte >> 4) ^ (row & 7)) << 4) | (byte & 15));
}

// Order earlier generic-proxy accesses of shared memory before later async-proxy ones.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 1-D bulk copy global -> shared, completing `bytes` on the mbarrier (16-B aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Ampere-style asynchronous 4-byte global -> shared copy (no registers held).
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ------------------------------------ 8-byte (value, epoch) slots between GPUs
// A naturally aligned 64-bit access is single-copy atomic, so a reader that
// sees the expected epoch in a slot also sees the value stored with it: no
// fence or flag is needed (volatile accesses bypass the non-coherent L1).
__device__ __forceinline__ void st_slot(void* addr, float v, unsigned epoch) {
  const unsigned long long w = (static_cast<unsigned long long>(epoch) << 32) | __float_as_uint(v);
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(addr), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_slot(const void* addr) {
  unsigned long long w;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(addr) : "memory");
  return w;
}

// Uncached 32-bit load of a word other threads or launches may have written.
__device__ __forceinline__ unsigned ld_volatile_u32(const unsigned* addr) {
  unsigned v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// ------------------------------------------------- thread-block cluster (DSMEM)
// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t cluster_map(uint32_t local, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void st_shared_f32(uint32_t addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
// All threads of all CTAs in the cluster; release/acquire orders the
// distributed shared-memory stores before the loads after it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t mask, uint32_t bits) {
  // (a & mask) | bits in one LOP3
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(bits));
  return d;
}

// Read-only streaming loads (do not allocate in L1; weights are used once).
__device__ __forceinline__ uint4 ldg_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ldg_stream8(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ldg_stream4(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// D = A*B + C for m16n8k16 with bf16 or fp16 operands, fp32 accumulators.
template <bool kHalf>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  if constexpr (kHalf) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, "
        "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, "
        "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// D = A*B + C for m16n8k32 int8 x int8 -> int32 (exact).
__device__ __forceinline__ void mma_s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, "
      "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_float(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_float(float v) { return v; }

template <typename T>
__device__ __forceinline__ T from_float(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half from_float<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ float from_float<float>(float v) {
  return v;
}

__device__ __forceinline__ float round_bf16(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace sb
