// Bulk asynchronous copies and shared-memory mbarriers (sm_90+, used here on
// sm_100a), in inline PTX.
//
// * `bulk_g2s` issues one 1-D bulk copy global -> shared through the TMA
//   engine (`cp.async.bulk ... .mbarrier::complete_tx::bytes`): no tensor
//   map, any contiguous span whose source address, destination address and
//   size are multiples of 16 bytes.  Its completion is counted on an mbarrier
//   in bytes.  Only this GPU's own global memory is ever the source here, and
//   the copies are plain (one destination CTA).
// * mbarrier helpers: init, arrive, arrive with an expected byte count, and a
//   parity try-wait (phase-parity protocol: a wait for parity P returns once
//   the phase with parity P has completed; a freshly initialised barrier is in
//   phase 0, so a wait for parity 1 returns at once).
// * `fence_proxy_async_global` orders this thread's earlier generic-proxy
//   view of global memory (e.g. data a peer stored and this thread then
//   acquired through a flag) before its later async-proxy (bulk copy) reads.
#pragma once

#include <stdint.h>

namespace bitscom_b200 {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Makes mbarrier initialisations visible to the async proxy (bulk copies).
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_addr(bar)),
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
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0u;
}

// One bulk copy of `bytes` (multiple of 16) from this GPU's global memory to
// this CTA's shared memory; completion is signalled on `bar` as transaction
// bytes.  Both addresses must be 16-byte aligned.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Bulk prefetch of `bytes` (multiple of 16, 16-byte aligned source) of this
// GPU's global memory into L2: no destination, no completion to wait for.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Shared-memory atomic add with acquire-release semantics at CTA scope.
__device__ __forceinline__ uint32_t atom_add_acq_rel_cta(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(smem_addr(p)), "r"(v) : "memory");
  return old;
}

// Shared-memory vector loads.
__device__ __forceinline__ uint4 lds_v4(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_addr(p)));
  return v;
}

__device__ __forceinline__ uint2 lds_v2(const void* p) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(smem_addr(p)));
  return v;
}

__device__ __forceinline__ uint32_t lds_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_addr(p)));
  return v;
}

}  // namespace bitscom_b200
