// Warp-level tensor-core helpers shared by the attention kernels (sm_100a): cp.async copies,
// ldmatrix fragment loads and mma.m16n8k16 with bf16 operands and fp32 accumulators.
//
// Fragment layouts (PTX ISA, mma.m16n8k16): thread (g, t) = (lane / 4, lane % 4).
//   A (16 x 16, row-major), 4 registers of two bf16: (row g, cols 2t..2t+1),
//     (row g + 8, cols 2t..), (row g, cols 2t + 8..), (row g + 8, cols 2t + 8..).
//   B (16 x 8, column-major), 2 registers: (rows 2t..2t+1, col g), (rows 2t + 8.., col g).
//   C / D (16 x 8, fp32), 4 values: (row g, cols 2t, 2t + 1), (row g + 8, cols 2t, 2t + 1).
// ldmatrix.x4: lanes 8i .. 8i + 7 give the row addresses of 8x8 matrix i; register i of a
// thread holds (row g, cols 2t..2t+1) of matrix i, or with .trans (rows 2t..2t+1, col g).
#pragma once

#include "common.cuh"  // smem_u32

namespace dsm {

// 16 bytes global -> shared; when !valid nothing is read and the 16 bytes are zero-filled
// (src must still be a mapped address)
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
// all but the most recent commit group have landed (for this thread)
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;\n" ::); }
// all but the N most recent commit groups have landed (for this thread)
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// c += a (16 x 16, row-major) * b (16 x 8, column-major); bf16 in, fp32 accumulate
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// two fp32 values rounded to bf16, lo in the low half (the lower column / row index)
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

}  // namespace dsm
