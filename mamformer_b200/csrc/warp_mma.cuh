// Warp-level tensor-core helpers shared by the attention-style kernels: ldmatrix fragment loads,
// mma.sync m16n8k16 (bf16 in, fp32 accumulate) and cp.async 16-byte copies.
//
// Fragment layouts (m16n8k16, per lane with g = lane / 4, t = lane % 4):
//   A (16 x 16, row-major): a0 (row g, k 2t..2t+1), a1 (row g+8, k 2t..), a2 (row g, k 2t+8..), a3 (row g+8, k 2t+8..)
//   B (16 x 8,  "col"):     b0 (k 2t..2t+1, n g),  b1 (k 2t+8.., n g)
//   C (16 x 8):             c0 c1 (row g, n 2t, 2t+1), c2 c3 (row g+8, n 2t, 2t+1)
// Two C tiles of adjacent n (keys 16j..16j+15) form the A fragment of the next product
// (c0c1 of tile 2j -> a0, c2c3 -> a1, tile 2j+1 -> a2, a3).
#pragma once
#include "common.cuh"

namespace mamf {
namespace wm {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_addr(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_addr(p)));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
               "{%0,%1,%2,%3};"
               : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Row / column offsets a lane supplies to ldmatrix.x4 for the three operand patterns.
//   A operand (rows r0.., k c0..):                 row r0 + (l&7) + ((l>>3)&1)*8, col c0 + (l>>4)*8
//   B operand from [n][k] storage (non-trans):    row n0 + (l&7) + (l>>4)*8,     col k0 + ((l>>3)&1)*8
//   B operand from [k][n] storage (trans):        row k0 + (l&7) + ((l>>3)&1)*8, col n0 + (l>>4)*8
//   A operand from [k][m] storage (trans):        row k0 + (l&7) + (l>>4)*8,     col m0 + ((l>>3)&1)*8
__device__ __forceinline__ int a_row(int l) { return (l & 7) + ((l >> 3) & 1) * 8; }
__device__ __forceinline__ int a_col(int l) { return (l >> 4) * 8; }
__device__ __forceinline__ int bn_row(int l) { return (l & 7) + (l >> 4) * 8; }
__device__ __forceinline__ int bn_col(int l) { return ((l >> 3) & 1) * 8; }
__device__ __forceinline__ int bt_row(int l) { return (l & 7) + ((l >> 3) & 1) * 8; }
__device__ __forceinline__ int bt_col(int l) { return (l >> 4) * 8; }
__device__ __forceinline__ int at_row(int l) { return (l & 7) + (l >> 4) * 8; }
__device__ __forceinline__ int at_col(int l) { return ((l >> 3) & 1) * 8; }

__device__ __forceinline__ void cp16(void* dst, const void* src, bool ok) {
  const int n = ok ? 16 : 0;   // src-size 0 -> zero fill
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

}  // namespace wm
}  // namespace mamf
