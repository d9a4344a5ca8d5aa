// Inline-PTX wrappers for the warp-level tensor-core kernels: ldmatrix / movmatrix /
// mma.sync (m16n8k16, bf16 in, fp32 accumulate) and cp.async staging.
//
// Fragment layouts used throughout (g = lane/4, q = lane%4):
//   A 16x16 row-major : a0=(g, 2q..2q+1) a1=(g+8, 2q..) a2=(g, 2q+8..) a3=(g+8, 2q+8..)
//   B 16x8  "col"     : b0=(k 2q..2q+1, n g)            b1=(k 2q+8.., n g)
//   C 16x8            : c0,c1=(g, 2q..2q+1)             c2,c3=(g+8, 2q..2q+1)
// ldmatrix.x4 returns matrix i (rows addressed by lanes 8i..8i+7) in register i with
// thread t holding (row t/4, cols 2(t%4), 2(t%4)+1); the .trans form holds the
// transposed pair (rows 2(t%4), 2(t%4)+1 of column t/4).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace moc {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Stores four 8x8 b16 matrices (register i = matrix i, thread t holding row t/4, columns
// 2(t%4)..+1); lanes 8i..8i+7 give the row addresses of matrix i.
__device__ __forceinline__ void stsm_x4(uint32_t addr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1,%2,%3,%4};\n" ::"r"(addr), "r"(r0), "r"(r1),
               "r"(r2), "r"(r3)
               : "memory");
}

// d += a * b  (m16n8k16, bf16 x bf16 -> fp32)
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// d = a * b  (m16n8k16, bf16 x bf16 -> fp32, zero accumulator)
__device__ __forceinline__ void mma_bf16_z(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}

// Transpose one 8x8 b16 fragment held one register per thread.
__device__ __forceinline__ uint32_t movm_t(uint32_t v) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(r) : "r"(v));
  return r;
}

__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// Round two floats to bf16 (nearest even) and pack: lo in bits 0-15, hi in 16-31.
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// (d0, d1) += (a0, a1) * (b0, b1) as one packed fp32x2 FMA (sm_100 FFMA2).
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  const float2 r = __ffma2_rn(make_float2(a0, a1), make_float2(b0, b1), make_float2(d0, d1));
  d0 = r.x;
  d1 = r.y;
}

// Elementwise bf16x2 product rounded to bf16 (nearest even).  For bf16 inputs the exact
// product fits fp32, so this equals rounding the fp32 product once.
__device__ __forceinline__ uint32_t hmul2_bf16(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// 16-byte async copy global -> shared; src_bytes = 0 writes zeros without reading.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

}  // namespace moc
