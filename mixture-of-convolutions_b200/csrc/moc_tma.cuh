// Tensor Memory Accelerator (TMA) staging for sm_100a: 2-D tiled bulk copies
// global -> shared completed on an mbarrier, with bounded waits.
//
// Loads here are never multicast across a cluster: each CTA fetches its own tiles.  Every wait
// on an mbarrier gives up after kSpinLimit polls; the kernel then records an error in its
// translation unit's device status word (read by moc_device_status()), waits once more,
// again bounded, for the copies it issued, and returns.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace moc {

constexpr uint32_t kSpinLimit = 1u << 22;

// device status bits
constexpr int kStatusWaitTimeout = 1;

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}

// Polls the mbarrier phase `parity` at most kSpinLimit times; true once it completed.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint32_t limit = kSpinLimit) {
  for (uint32_t i = 0; i < limit; ++i) {
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

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Byte offset of the 16-byte chunk `chunk` (0..7) of row `row` inside a tile written by
// TMA with CU_TENSOR_MAP_SWIZZLE_128B (128-byte rows; tile base 1024-byte aligned).
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}

// Shared -> global tiled store of the box at `src` (same box and swizzle as the map's loads),
// tracked by the issuing thread's bulk groups.  Rows and columns past the tensor's extent are
// not written.  c0 * 2 bytes must be a multiple of 16, and neither coordinate negative.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int c0, int c1, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];\n" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(src)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }

// Waits until this thread's bulk groups, all but the newest N, have finished reading shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;\n" ::"n"(N) : "memory");
}

// Waits until this thread's bulk groups, all but the newest N, have completed (writes performed).
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;\n" ::"n"(N) : "memory");
}

// Orders this thread's (and, after a CTA barrier, the CTA's) generic-proxy shared-memory
// accesses before its following async-proxy (TMA) writes to the same memory.
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

// Host: 2-D bf16 tensor map over a row-major [outer, inner] array with a row pitch of
// `row_bytes`, box [box_outer, box_inner], zero fill out of bounds.  swizzle_bytes is the
// shared-memory swizzle span: 128 (the 16-byte chunk index of a 128-byte row XOR row % 8),
// 64 (chunk of a 64-byte row XOR (row / 2) % 4), 32 (chunk of a 32-byte row XOR (row / 4)
// % 2), or 0 (dense rows).  The box's inner extent must not exceed the span.
int make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                      uint32_t box_inner, uint32_t box_outer, int swizzle_bytes = 128);

}  // namespace moc
