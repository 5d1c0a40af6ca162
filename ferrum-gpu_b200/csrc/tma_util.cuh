// Bulk-copy (TMA) and mbarrier helpers for the sm_100a kernels: bounded
// mbarrier waits (%globaltimer), 1D bulk copies, tiled 2D tensor copies
// between global and shared memory, and L2 prefetches. Every source and
// destination is this GPU's own memory; no copy uses cluster multicast.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace ferrum {

constexpr uint64_t kWaitTimeoutNs = 1000000000ull;  // 1 s per wait
constexpr int kErrWaitTimeout = 1;

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return done != 0;
}

// Bounded wait for `phase` of `bar`; false after kWaitTimeoutNs.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t phase) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, phase)) {
    if (global_ns() - t0 > kWaitTimeoutNs) return false;
  }
  return true;
}

// Global -> shared bulk copy of `bytes` (multiple of 16, both addresses
// 16-byte aligned) completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Contiguous bytes into the L2 (address and size multiples of 16).
__device__ __forceinline__ void l2_prefetch_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Box {x, y} of a 2D tensor map into the L2 (x: element within a row, y: row).
__device__ __forceinline__ void l2_prefetch_tile2d(const CUtensorMap* map, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map),
               "r"(x), "r"(y)
               : "memory");
}

// Box {x, y} of a 2D tensor map into shared memory, completing on `bar`. x
// times the element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_tile2d(void* dst_smem, const CUtensorMap* map, int32_t x,
                                                int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst_smem)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Box {x, y} of a 2D tensor map from shared memory (x, y >= 0 and x times
// the element size a multiple of 16 bytes), in the current bulk group.
__device__ __forceinline__ void tma_store_tile2d(const CUtensorMap* map, int32_t x, int32_t y,
                                                 const void* src_smem) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   map),
               "r"(x), "r"(y), "r"(smem_u32(src_smem))
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Every committed bulk store has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Every committed bulk store has completed (its writes are performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Orders this thread's generic-proxy shared-memory accesses before later
// async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

}  // namespace ferrum
