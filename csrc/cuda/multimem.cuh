// NVLink multicast (NVLS) memory operations, written from the PTX ISA's
// multimem.* description.  `mc_addr` is an address inside a multicast mapping:
// a store reaches the same offset in every GPU's buffer bound to the object, a
// ld_reduce returns the sum over those buffers, computed in the NVSwitch.
// Only threads issue these; no TMA or bulk copy addresses a multicast range.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace mb {

__device__ __forceinline__ void mc_store_release_u32(uint64_t mc_addr, uint32_t v) {
  asm volatile("multimem.st.release.sys.global.u32 [%0], %1;" ::"l"(mc_addr), "r"(v) : "memory");
}

__device__ __forceinline__ void mc_store_u32(uint64_t mc_addr, uint32_t v) {
  asm volatile("multimem.st.relaxed.sys.global.u32 [%0], %1;" ::"l"(mc_addr), "r"(v) : "memory");
}

__device__ __forceinline__ void mc_store_f32(uint64_t mc_addr, float v) {
  asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(mc_addr), "f"(v) : "memory");
}

// 16 bytes to every replica.
__device__ __forceinline__ void mc_store_16(uint64_t mc_addr, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc_addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// Sum over every replica of 8 bf16 at mc_addr, accumulated in fp32 by the switch.
__device__ __forceinline__ uint4 mc_ld_reduce_bf16x8(uint64_t mc_addr) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(mc_addr)
               : "memory");
  return r;
}

__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

}  // namespace mb
