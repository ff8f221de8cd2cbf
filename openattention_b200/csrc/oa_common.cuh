// Shared device helpers and host-side error plumbing for the OpenAttention B200 kernels.
//
// Layout conventions used by every kernel in this library (all row-major, contiguous unless a
// stride argument says otherwise):
//   D   = 128 (head dimension), G = 4 query heads per KV head, RQ = 32 (QGS rank), RC = 16 (QGC rank)
//   row r        = b * 32 + h          (one query head of one request)
//   kv row       = b * 8 + h / 4       (the KV head that query head reads)
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <math.h>

#include <algorithm>

namespace oa {

constexpr int kD = 128;
constexpr int kG = 4;
constexpr int kRQ = 32;
constexpr int kRC = 16;
constexpr int kHQ = 32;
constexpr int kHKV = 8;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Round-to-nearest-even fp32 -> bf16 bits (no NaN inputs occur on these paths; +-inf preserved).
__device__ __forceinline__ uint16_t f2bf_bits(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float bf_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// 16-byte read-only streaming load (K/V rows are touched once per row).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- 16-byte asynchronous copies global -> shared (both addresses 16-byte aligned; through L2 only).
// The data never passes through registers; cp_async_wait_all returns once this thread's copies have
// landed (a hardware wait on the thread's own copies, no polling), and a barrier then publishes them.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// ---- TMA bulk copies (cp.async.bulk, no multicast) completing on an mbarrier, with bounded waits
__device__ __forceinline__ void mbar_init(uint32_t bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(1) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// one thread: expect `bytes` on the barrier and start the copy (16-byte aligned, size % 16 == 0)
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
// several copies on one barrier: announce the total first, then start each copy
__device__ __forceinline__ void mbar_expect(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
// Bounded wait for phase `parity`; false after kSpinLimit polls (the caller reports and bails out).
constexpr uint32_t kSpinLimit = 1u << 26;
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  for (uint32_t it = 0; it < kSpinLimit; ++it) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

}  // namespace oa

// ---------------------------------------------------------------- host error plumbing
enum {
  OA_OK = 0,
  OA_ERR_INVALID = 1,
  OA_ERR_UNSUPPORTED = 2,
  OA_ERR_CUDA = 3,
};

int oa_fail(int code, const char* fmt, ...);
int oa_check_launch(const char* what);
// Raise a kernel's dynamic shared-memory limit when its static arrays plus `dyn` bytes pass the
// 48 KB default (the opt-in counts the static part too).  With max_carveout, the kernel also asks
// for the largest shared-memory share of the SM's L1 (for kernels whose occupancy is set by shared
// memory and that do not rely on L1).  Returns an OA status.
int oa_smem_opt_in(const void* kernel, size_t dyn, const char* what, bool max_carveout = false);

#define OA_REQUIRE(cond, ...)                      \
  do {                                             \
    if (!(cond)) return oa_fail(OA_ERR_INVALID, __VA_ARGS__); \
  } while (0)

static inline bool oa_aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// hkv: KV heads per request held by this call's arrays (8 = whole requests; fewer = a KV-head shard of
// each request, whose query heads are the 4 hkv that read those KV heads)
#define OA_REQUIRE_HKV(fn, hkv) \
  OA_REQUIRE((hkv) >= 1 && (hkv) <= oa::kHKV, "%s: hkv=%lld outside [1, %d]", fn, (long long)(hkv), oa::kHKV)
