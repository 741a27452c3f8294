// Shared helpers for the libspk.so kernels: status reporting, element types,
// and thin inline-PTX wrappers for the sm_100a features the kernels use
// (mbarrier, TMA tensor copies, tcgen05 MMA / TMEM).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/spk.h"

namespace spk {

// ---------------------------------------------------------------- errors

int fail(int code, const char* fmt, ...);  // records the message, returns code
int check_launch(const char* what);        // cudaGetLastError -> status
int check_stream_device(void* stream);     // device must be sm_100

#define SPK_REQUIRE(cond, code, ...)            \
  do {                                          \
    if (!(cond)) return ::spk::fail(code, __VA_ARGS__); \
  } while (0)

inline bool aligned(const void* p, int bytes) {
  return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}

inline int dtype_size(int dt) {
  switch (dt) {
    case SPK_F32: return 4;
    case SPK_F16: return 2;
    case SPK_BF16: return 2;
    case SPK_U8: return 1;
    case SPK_FP8: return 1;
    default: return 0;
  }
}

int num_sms();  // SM count of the current device (cached per device)

// Reads and clears the device-side error flag of the calling translation unit
// (see g_spk_device_error below); returns SPK_ERR_TIMEOUT if it was raised.
#define SPK_DEFINE_ERROR_READER(fn_name)                                                               \
  int fn_name(cudaStream_t stream) {                                                                   \
    int h = 0;                                                                                         \
    cudaError_t e = cudaMemcpyFromSymbolAsync(&h, g_spk_device_error, sizeof(int), 0,                  \
                                              cudaMemcpyDeviceToHost, stream);                         \
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);                                           \
    if (e != cudaSuccess) return ::spk::fail(SPK_ERR_CUDA, "reading device error flag: %s",           \
                                             cudaGetErrorString(e));                                   \
    if (h != 0) {                                                                                      \
      int z = 0;                                                                                       \
      cudaMemcpyToSymbolAsync(g_spk_device_error, &z, sizeof(int), 0, cudaMemcpyHostToDevice, stream); \
      cudaStreamSynchronize(stream);                                                                   \
      return ::spk::fail(SPK_ERR_TIMEOUT, "a device-side wait gave up (code %d)", h);                 \
    }                                                                                                  \
    return SPK_OK;                                                                                     \
  }

// ---------------------------------------------------------------- elements

template <int DT> struct Elem;
template <> struct Elem<SPK_F32> {
  using T = float;
  __device__ static float load(const T* p) { return *p; }
  __device__ static T make(float v) { return v; }
};
template <> struct Elem<SPK_F16> {
  using T = __half;
  __device__ static float load(const T* p) { return __half2float(*p); }
  __device__ static T make(float v) { return __float2half_rn(v); }
};
template <> struct Elem<SPK_BF16> {
  using T = __nv_bfloat16;
  __device__ static float load(const T* p) { return __bfloat162float(*p); }
  __device__ static T make(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<SPK_U8> {
  using T = uint8_t;
  __device__ static float load(const T* p) { return (float)(*p); }
  __device__ static T make(float v) { return (uint8_t)(v != 0.0f); }
};
// fp8 e4m3 spikes: 1.0 is the byte 0x38 (exponent 7 = bias, mantissa 0), 0.0
// the byte 0; spike tensors hold nothing else, so any non-zero magnitude
// byte reads as 1.
template <> struct Elem<SPK_FP8> {
  using T = uint8_t;
  __device__ static float load(const T* p) { return (*p & 0x7f) ? 1.0f : 0.0f; }
  __device__ static T make(float v) { return v != 0.0f ? (uint8_t)0x38 : (uint8_t)0; }
};

// ---------------------------------------------------------------- PTX: sync

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded waits.  A wait polls its mbarrier until the phase completes or about
// kWaitLimitNs of wall time (%globaltimer) has passed; on give-up it records
// `code` in the per-file device error flag and returns false, and the caller
// abandons its work loop, drains what it has in flight (also with bounded
// waits) and exits normally.  Host code turns the flag into SPK_ERR_TIMEOUT.
static __device__ int g_spk_device_error = 0;
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, int code, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && global_ns() - t0 > limit_ns) {
      atomicExch(&g_spk_device_error, code);
      return false;
    }
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code = 1) {
  return mbar_wait_for(bar, parity, code, kWaitLimitNs);
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ uint32_t elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t.reg .b32 r;\n\t"
      "elect.sync r|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred;
}

// ---------------------------------------------------------------- PTX: TMA

__device__ __forceinline__ void tma_prefetch_desc(const void* desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(desc) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const void* desc, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(desc), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const void* desc, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(desc), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// ---------------------------------------------------------------- PTX: tcgen05

// Shared-memory matrix descriptor (sm_100 layout): start address, leading and
// stride byte offsets (16-byte units), version 1 at bit 46, swizzle mode in
// bits 61-63 (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t swizzle) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)(swizzle & 7) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 accumulate.
// a_mn / b_mn select MN-major operands (bits 15/16); N>>3 at bits 17-22,
// M>>4 at bits 24-28.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, int a_mn, int b_mn) {
  return (1u << 4)                    // D format f32
         | (1u << 7)                  // A bf16
         | (1u << 10)                 // B bf16
         | ((uint32_t)a_mn << 15)     // A major
         | ((uint32_t)b_mn << 16)     // B major
         | ((uint32_t)(N >> 3) << 17) // N
         | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bits, 16 consecutive columns: thread i of the warp receives
// row (lane base + i), columns [col, col+16).  Waits for completion; the
// wait names the destination registers so no use is hoisted above it.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  tmem_ld16(taddr, v);
  tmem_ld16(taddr + 16, v + 16);
}

// ---------------------------------------------------------------- host: TMA maps

// Encodes a tiled tensor map (bf16 elements, 128-byte swizzle).  dims/strides
// are innermost first; strides in bytes for dims 1..rank-1.
int make_tmap_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                   const uint64_t* strides_bytes, const uint32_t* box, bool swizzle128);
// The same with the swizzle span in bytes (0, 32, 64 or 128).
int make_tmap_bf16_sw(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes);

}  // namespace spk

namespace spk {

// ---------------------------------------------------------------- PTX: clusters

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// all threads of all CTAs of the cluster
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// address of the same shared variable in CTA `rank` of this cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f32x2(uint32_t addr, float a, float b) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_cluster() { asm volatile("fence.acq_rel.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int code = 2) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 255u) == 0 && global_ns() - t0 > kWaitLimitNs) {
      atomicExch(&g_spk_device_error, code);
      return false;
    }
  }
}

}  // namespace spk

namespace spk {

// ---------------------------------------------------------------- TMEM loads, pipelined
// tmem_ld16_raw issues the load; the registers are only valid after
// tmem_wait_ld_fence(r), which names them as read-write operands so the
// compiler cannot move their uses above the wait.
__device__ __forceinline__ void tmem_ld16_raw(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld_fence(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
}

// one column of the calling thread's lane, raw issue (valid after a wait that names it)
__device__ __forceinline__ void tmem_ld1_raw(uint32_t taddr, uint32_t& r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
}

// After a bare tcgen05.wait::ld: makes the registers of one more 16-column load
// read-write at this point, so that no use of them moves above the wait.
__device__ __forceinline__ void reg_fence16(uint32_t (&r)[16]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
}

// two buffers in flight: waits for both, fences both
__device__ __forceinline__ void tmem_wait_ld_fence2(uint32_t (&a)[16], uint32_t (&b)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                 "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]), "+r"(a[14]),
                 "+r"(a[15]), "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]),
                 "+r"(b[7]), "+r"(b[8]), "+r"(b[9]), "+r"(b[10]), "+r"(b[11]), "+r"(b[12]), "+r"(b[13]),
                 "+r"(b[14]), "+r"(b[15])
               :
               : "memory");
}

// ---------------------------------------------------------------- spike tiles
// number of ones in row r of a 128B-swizzled tile of bf16 spikes (first n
// elements, n % 8 == 0).  A spike is 0x0000 or 0x3F80, so bit 7 of each half
// word counts it: the masked words add up to 0x80 per one in each half (at
// most 32 ones per half, no carry into the other half).
__device__ __forceinline__ int row_count_sw128(const uint8_t* tile, int r, int n) {
  constexpr uint32_t kBit = 0x00800080u;
  uint32_t acc = 0u;
  const int chunks = n >> 3;
  for (int c = 0; c < chunks; ++c) {
    const uint4 w = *reinterpret_cast<const uint4*>(tile + r * 128 + ((c ^ (r & 7)) << 4));
    acc += (w.x & kBit) + (w.y & kBit);
    acc += (w.z & kBit) + (w.w & kBit);
  }
  return (int)(((acc & 0xFFFFu) + (acc >> 16)) >> 7);
}

// 32-byte global store (sm_100): the address must be 32-byte aligned
__device__ __forceinline__ void st_global_v8(void* ptr, uint4 lo, uint4 hi) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(ptr), "r"(lo.x), "r"(lo.y),
               "r"(lo.z), "r"(lo.w), "r"(hi.x), "r"(hi.y), "r"(hi.z), "r"(hi.w)
               : "memory");
}

// ---------------------------------------------------------------- packed fp32x2 arithmetic (sm_100)
// Each operation rounds like its scalar fp32 counterpart (round to nearest).
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  uint64_t x = *reinterpret_cast<uint64_t*>(&a), y = *reinterpret_cast<uint64_t*>(&b), z;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(z) : "l"(x), "l"(y));
  return *reinterpret_cast<float2*>(&z);
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  uint64_t x = *reinterpret_cast<uint64_t*>(&a), y = *reinterpret_cast<uint64_t*>(&b), z;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(z) : "l"(x), "l"(y));
  return *reinterpret_cast<float2*>(&z);
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  uint64_t x = *reinterpret_cast<uint64_t*>(&a), y = *reinterpret_cast<uint64_t*>(&b),
           w = *reinterpret_cast<uint64_t*>(&c), z;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(z) : "l"(x), "l"(y), "l"(w));
  return *reinterpret_cast<float2*>(&z);
}

}  // namespace spk

namespace spk {

// ---------------------------------------------------------------- TMEM stores / A-from-TMEM MMA
// 32 lanes x 32 bits, 32 consecutive columns from the calling thread's registers
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// 32 lanes x 32 bits, 16 consecutive columns from the calling thread's registers
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D (TMEM) [+]= A (TMEM, K-major, two bf16 per 32-bit column) x B (shared memory descriptor)
__device__ __forceinline__ void umma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

}  // namespace spk

namespace spk {

// 32 lanes x 32 bits x 32 columns, raw issue (valid after tmem_wait_ld_fence32)
__device__ __forceinline__ void tmem_ld32_raw(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld_fence32(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

}  // namespace spk

namespace spk {

// Asynchronous store of two floats into (possibly remote) cluster shared
// memory; completion is signalled on the destination CTA's mbarrier as
// transaction bytes (8), so no fence is needed before the receiver's wait.
__device__ __forceinline__ void st_async_f32x2(uint32_t cluster_addr, float a, float b, uint32_t cluster_mbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(
                   cluster_addr),
               "f"(a), "f"(b), "r"(cluster_mbar)
               : "memory");
}

}  // namespace spk

namespace spk {

// ---------------------------------------------------------------- PTX: transposed TMEM reads, matrix
// shared-memory moves, TMA stores

// 16 lanes x 256 bits, four column repeats: thread i receives, for repeat j,
// r[4j], r[4j+1] = lane (base + i/4), columns 8j + 2(i%4) and +1, and
// r[4j+2], r[4j+3] = lane (base + i/4 + 8), the same columns.  Raw issue:
// valid after a tcgen05.wait::ld that names the registers.
__device__ __forceinline__ void tmem_ld16x256_x4_raw(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Four 8x8 b16 matrices from registers into shared memory: lane i gives the
// address of row i%8 of matrix i/8; register k of thread i holds row i/4,
// columns 2(i%4) and +1 of matrix k.
__device__ __forceinline__ void stmatrix_x4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b),
               "r"(c), "r"(d)
               : "memory");
}

// The inverse of stmatrix_x4 (same addresses, same register layout).
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const void* desc, uint64_t* bar, int x, int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(desc), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// shared -> global tile store, tracked by the issuing thread's bulk groups
__device__ __forceinline__ void tma_store_3d(const void* desc, const void* src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(desc),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// at most N of this thread's bulk groups still reading their shared-memory source
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// at most N of this thread's bulk groups not yet complete
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace spk

namespace spk {

// ---------------------------------------------------------------- programmatic dependent launch
// A kernel launched with programmatic stream serialisation may be scheduled before the previous
// kernel in the stream has finished.  pdl_wait() blocks until that grid has completed and its
// memory is visible; every CTA calls it before reading anything an earlier kernel wrote, so the
// completion of a grid implies the completion of all earlier ones.  Without the launch
// attribute both instructions are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// lets the next kernel in the stream be scheduled once every CTA of this grid has issued it
// (or exited); its CTAs then take SMs as this grid's CTAs leave them
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// adds programmatic stream serialisation to a launch configuration's attribute list
inline void add_pdl_attr(cudaLaunchConfig_t& cfg, cudaLaunchAttribute* attrs) {
  cudaLaunchAttribute& a = attrs[cfg.numAttrs++];
  a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  a.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
}

}  // namespace spk
