// Shared helpers of libasap: error reporting, geometry arithmetic, PTX wrappers for sm_100a.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/asap.h"

namespace asap {

// ------------------------------------------------------------------ host-side error plumbing
void set_error(const char* fmt, ...);
int cuda_fail(cudaError_t err, const char* what);

#define ASAP_CUDA(call)                                        \
  do {                                                         \
    cudaError_t err__ = (call);                                \
    if (err__ != cudaSuccess) return asap::cuda_fail(err__, #call); \
  } while (0)

#define ASAP_CHECK_LAUNCH(what)                                \
  do {                                                         \
    cudaError_t err__ = cudaGetLastError();                    \
    if (err__ != cudaSuccess) return asap::cuda_fail(err__, what); \
  } while (0)

// ------------------------------------------------------------------ geometry (transport/layout.py)
constexpr uint64_t kAlign = 256;
constexpr uint64_t kFlagStride = 64;
constexpr uint64_t kFlagsPage = 2ull << 20;
constexpr uint64_t kBellStride = 64;
constexpr uint32_t kMaxTokens = (1u << 17) - 1;
constexpr uint32_t kMaxLayer = (1u << 10) - 1;
constexpr uint32_t kMaxEpoch = (1u << 5) - 1;

__host__ __device__ inline uint64_t align_up(uint64_t n, uint64_t a) { return (n + a - 1) / a * a; }

struct Offsets {
  uint64_t ids_off, w_off, region_bytes, recv_bytes, host_bytes, flags_bytes, seg_bytes, result_bytes;
};

__host__ __device__ inline Offsets offsets_of(const asap_geometry_t& g) {
  Offsets o;
  const uint64_t nm = (uint64_t)g.n_max;
  o.ids_off = align_up(nm * g.hidden * 2, kAlign);
  o.w_off = o.ids_off + align_up(nm * g.topk * 4, kAlign);
  o.region_bytes = o.w_off + align_up(nm * g.topk * 4, kAlign);
  o.recv_bytes = (uint64_t)g.num_a * g.slots * o.region_bytes;
  o.host_bytes = align_up((uint64_t)g.num_a * g.slots * kBellStride, 4096);
  o.flags_bytes = align_up((uint64_t)g.num_f * g.slots * kFlagStride, kFlagsPage);
  o.seg_bytes = align_up(nm * g.hidden * 2, kAlign);
  o.result_bytes = o.flags_bytes + (uint64_t)g.num_f * g.slots * o.seg_bytes;
  return o;
}

__host__ __device__ inline uint64_t region_off(const asap_geometry_t& g, const Offsets& o, int a, int s) {
  return ((uint64_t)a * g.slots + s) * o.region_bytes;
}
__host__ __device__ inline uint64_t bell_off(const asap_geometry_t& g, int a, int s) {
  return ((uint64_t)a * g.slots + s) * kBellStride;
}
__host__ __device__ inline uint64_t done_off(const asap_geometry_t& g, int f, int s) {
  return ((uint64_t)f * g.slots + s) * kFlagStride;
}
__host__ __device__ inline uint64_t seg_off(const asap_geometry_t& g, const Offsets& o, int f, int s) {
  return o.flags_bytes + ((uint64_t)f * g.slots + s) * o.seg_bytes;
}

__host__ __device__ inline uint64_t pack_doorbell(uint32_t seq, uint32_t n, uint32_t layer, uint32_t epoch) {
  return (uint64_t)seq | ((uint64_t)n << 32) | ((uint64_t)layer << 49) | ((uint64_t)epoch << 59);
}

__host__ __device__ inline uint64_t status_word(uint32_t code, uint32_t f, uint32_t slot, uint32_t seq) {
  return (uint64_t)(code & 0xff) | ((uint64_t)(f & 0xff) << 8) | ((uint64_t)(slot & 0xff) << 16) |
         ((uint64_t)seq << 32);
}

// ------------------------------------------------------------------ device helpers
#ifdef __CUDACC__

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// First failure wins; a status pointer of 0 disables reporting.
__device__ __forceinline__ void report(uint64_t status, uint64_t word) {
  if (status) atomicCAS(reinterpret_cast<unsigned long long*>(status), 0ull, (unsigned long long)word);
}

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false when `deadline` (globaltimer ns) passed or *abort was raised by another warp.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t deadline,
                                          volatile int* abort) {
  uint32_t it = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++it & 255u) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() > deadline) {
        *abort = 1;
        return false;
      }
    }
  }
  return true;
}

// ---- TMA (tensor maps live in kernel parameter space: __grid_constant__)
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int32_t x, int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---- tcgen05
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
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// smem (32 rows x 128 bit) -> TMEM lanes of all four sub-partitions (scale-factor copy)
__device__ __forceinline__ void tc_cp_32x128b_warpx4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
// D(tmem) (+)= A(smem) * B(smem), MXF8F6F4 block-scaled, E8M0 scale per 32 along K.
__device__ __forceinline__ void tc_mma_mxf8f6f4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate, uint32_t sfa_tmem, uint32_t sfb_tmem) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
// D (TMEM, fp32) (+)= A * B, kind::f8f6f4 without block scaling (A, B E4M3, both K-major in shared memory).
__device__ __forceinline__ void tc_mma_f8f6f4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem), "l"(adesc), "l"(bdesc),
      "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---- MX quantisation (OCP Microscaling v1.0, section 6.3: shared exponent = floor(log2(amax)) - emax_elem)
// E8M0 scale byte for a block whose absolute maximum is `amax`, element type E4M3 (emax_elem = 8).
__device__ __forceinline__ uint32_t mx_e4m3_scale_byte(float amax) {
  const int biased = (int)((__float_as_uint(amax) >> 23) & 0xff);  // 0 for zero / subnormal amax
  int s = biased - 8;
  return (uint32_t)(s < 0 ? 0 : s);
}
// Multiplier that maps a block to the element range: 2^(127 - scale_byte), exact in fp32 (subnormal at 254).
__device__ __forceinline__ float mx_inv_scale(uint32_t sbyte) {
  const int e = 254 - (int)sbyte;  // biased exponent of 2^(127 - sbyte)
  return e > 0 ? __uint_as_float((uint32_t)e << 23) : __uint_as_float(0x00400000u);
}
// Two fp32 -> two E4M3 bytes (round to nearest even, saturate to +-448), packed lo = a, hi = b.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float a, float b) {
  uint16_t r;
  asm volatile("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;" : "=h"(r) : "f"(a), "f"(b));
  return r;
}

#endif  // __CUDACC__

}  // namespace asap
