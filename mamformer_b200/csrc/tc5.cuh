// tcgen05 / TMA / mbarrier building blocks shared by the attention kernels (csrc/flash_tc.cu,
// csrc/flash_tc_bwd.cu).  Inline PTX for sm_100a:
//   * mbarrier init / arrive / expect_tx / bounded parity wait (clock64 limit, error word);
//   * TMA: 2-D / 3-D tiled loads (no multicast: every map covers this GPU's memory only);
//   * UMMA shared-memory descriptors (128-byte swizzle) and kind::f16 instruction descriptors;
//   * tcgen05.mma with A from shared memory or from tensor memory, tcgen05.commit;
//   * tcgen05.ld / st of 32 lanes x 16 / 32 / 64 columns.
#pragma once

#include "common.cuh"

#include <cudaTypedefs.h>

namespace mamf {
namespace tc5 {

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// ---- mbarrier ------------------------------------------------------------------------------------
__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n));
}
__device__ __forceinline__ void bar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
// One try: the thread is suspended until the phase completes or about 1 ms passes (the
// suspend-time hint), so waiting warps take no issue slots from the warps doing the work.
__device__ __forceinline__ bool bar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
               : "=r"(ok) : "r"(su32(b)), "r"(parity), "r"(1000000u) : "memory");
  return ok != 0;
}
// Wait for the phase with the given parity to complete, for at most `limit` clock64 cycles.
// Returns false on timeout (code recorded in *err unless a code is already there) or once
// another role of the grid has recorded an error.  The error word is a global load (an L2 round
// trip): it and the clock are read only every 64th unsuccessful try, so a waiting thread notices
// a completed phase within one try_wait instead of after a global load.
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity, int code, int* err, long long limit) {
  if (bar_try(b, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t n = 1;; ++n) {
    if (bar_try(b, parity)) return true;
    if ((n & 63u) == 0) {
      if (*((volatile int*)err) != 0) return false;
      if (clock64() - t0 > limit) { atomicCAS(err, 0, code); return false; }
    }
  }
}

// ---- TMA -----------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(su32(dst)), "l"(map), "r"(su32(bar)), "r"(c0), "r"(c1), "r"(c2) : "memory");
}
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(su32(dst)), "l"(map), "r"(su32(bar)), "r"(c0), "r"(c1) : "memory");
}
// generic-proxy shared-memory writes made visible to the async proxy (TMA / tcgen05 reads)
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---- UMMA descriptors ----------------------------------------------------------------------------
// Shared-memory matrix descriptor (sm100: version 1 at bit 46, 128-byte swizzle at bits 61-63).
// K-major operands: lbo unused (16), sbo = 1024 (8 rows of 128 B).  MN-major operands: lbo = the
// byte stride between 64-element chunks along M / N, sbo = 1024 (8 K-rows of 128 B).
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// kind::f16 instruction descriptor: bf16 x bf16 -> f32, shape M x N, A / B K-major or MN-major
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// ---- tcgen05 -------------------------------------------------------------------------------------
// D[tmem] (+)= A[smem] * B[smem]
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
               ::"r"(d), "l"(a), "l"(b), "r"(id), "r"(acc));
}
// D[tmem] (+)= A[tmem] * B[smem]
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n"
               ::"r"(d), "r"(a_tmem), "l"(b), "r"(id), "r"(acc));
}
// arrive on the mbarrier once every tcgen05 operation issued so far by this thread has completed
__device__ __forceinline__ void commit(uint64_t* b) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

#define MAMF_TC5_LD32(DST, ADDR)                                                                           \
  asm volatile(                                                                                            \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"     \
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                           \
      : "=r"(DST[0]), "=r"(DST[1]), "=r"(DST[2]), "=r"(DST[3]), "=r"(DST[4]), "=r"(DST[5]), "=r"(DST[6]),   \
        "=r"(DST[7]), "=r"(DST[8]), "=r"(DST[9]), "=r"(DST[10]), "=r"(DST[11]), "=r"(DST[12]),             \
        "=r"(DST[13]), "=r"(DST[14]), "=r"(DST[15]), "=r"(DST[16]), "=r"(DST[17]), "=r"(DST[18]),          \
        "=r"(DST[19]), "=r"(DST[20]), "=r"(DST[21]), "=r"(DST[22]), "=r"(DST[23]), "=r"(DST[24]),          \
        "=r"(DST[25]), "=r"(DST[26]), "=r"(DST[27]), "=r"(DST[28]), "=r"(DST[29]), "=r"(DST[30]),          \
        "=r"(DST[31])                                                                                      \
      : "r"(ADDR))

__device__ __forceinline__ void tld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tst_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 consecutive columns of this thread's lane (the warp's 32 lanes), waited
__device__ __forceinline__ void tld32(uint32_t taddr, float (&r)[32]) {
  uint32_t v[32];
  MAMF_TC5_LD32(v, taddr);
  tld_wait();
#pragma unroll
  for (int i = 0; i < 32; ++i) r[i] = __uint_as_float(v[i]);
}
// two 32-column loads in flight, one wait
__device__ __forceinline__ void tld32x2(uint32_t a0, uint32_t a1, float* r0, float* r1) {
  uint32_t v[32], w[32];
  MAMF_TC5_LD32(v, a0);
  MAMF_TC5_LD32(w, a1);
  tld_wait();
#pragma unroll
  for (int i = 0; i < 32; ++i) { r0[i] = __uint_as_float(v[i]); r1[i] = __uint_as_float(w[i]); }
}
__device__ __forceinline__ void tld64(uint32_t taddr, float* r) { tld32x2(taddr, taddr + 32u, r, r + 32); }

__device__ __forceinline__ void tst32(uint32_t taddr, const float (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(__float_as_uint(r[0])), "r"(__float_as_uint(r[1])), "r"(__float_as_uint(r[2])),
        "r"(__float_as_uint(r[3])), "r"(__float_as_uint(r[4])), "r"(__float_as_uint(r[5])), "r"(__float_as_uint(r[6])),
        "r"(__float_as_uint(r[7])), "r"(__float_as_uint(r[8])), "r"(__float_as_uint(r[9])), "r"(__float_as_uint(r[10])),
        "r"(__float_as_uint(r[11])), "r"(__float_as_uint(r[12])), "r"(__float_as_uint(r[13])), "r"(__float_as_uint(r[14])),
        "r"(__float_as_uint(r[15])), "r"(__float_as_uint(r[16])), "r"(__float_as_uint(r[17])), "r"(__float_as_uint(r[18])),
        "r"(__float_as_uint(r[19])), "r"(__float_as_uint(r[20])), "r"(__float_as_uint(r[21])), "r"(__float_as_uint(r[22])),
        "r"(__float_as_uint(r[23])), "r"(__float_as_uint(r[24])), "r"(__float_as_uint(r[25])), "r"(__float_as_uint(r[26])),
        "r"(__float_as_uint(r[27])), "r"(__float_as_uint(r[28])), "r"(__float_as_uint(r[29])), "r"(__float_as_uint(r[30])),
        "r"(__float_as_uint(r[31]))
      : "memory");
  tst_wait();
}
// 16 columns (e.g. 32 bf16 values packed in pairs), not waited: call tst_wait() after the last one
__device__ __forceinline__ void tst16_nowait(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace tc5

// ---- host: tensor maps -----------------------------------------------------------------------------
using TmaEncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline TmaEncodeFn tc5_encode_fn() {
  static TmaEncodeFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    MAMF_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && ptr, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<TmaEncodeFn>(ptr);
  }
  return fn;
}

// (B, L, heads, 128) bf16 -> 3-D map (dim, head, B*L rows), box 64 dims x 1 head x `rows` rows,
// 128-byte swizzle (one 64-dim chunk of a row = one 128-byte swizzle row).
inline CUtensorMap tc5_head_map(const at::Tensor& t, uint32_t rows, const char* what) {
  TORCH_CHECK(t.is_contiguous() && t.dim() == 4 && t.size(3) == 128 && t.scalar_type() == at::kBFloat16,
              what, ": contiguous bf16 (B, L, heads, 128) tensors");
  TORCH_CHECK(aligned16(t.data_ptr()), what, ": 16-byte aligned base");
  const int64_t heads = t.size(2);
  CUtensorMap m;
  cuuint64_t gd[3] = {(cuuint64_t)128, (cuuint64_t)heads, (cuuint64_t)(t.size(0) * t.size(1))};
  cuuint64_t gs[2] = {(cuuint64_t)128 * 2, (cuuint64_t)(heads * 128 * 2)};
  cuuint32_t bx[3] = {64u, 1u, rows}, es[3] = {1, 1, 1};
  CUresult r = tc5_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, t.data_ptr(), gd, gs, bx, es,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (", what, ") failed: ", (int)r);
  return m;
}

// (rows, cols) row-major fp32 -> 2-D map, box `box_cols` x 1 row, no swizzle
inline CUtensorMap tc5_rows_map_f32(const float* base, int64_t rows, int64_t cols, uint32_t box_cols,
                                    const char* what) {
  TORCH_CHECK(aligned16(base) && (cols * 4) % 16 == 0 && (box_cols * 4) % 16 == 0 && box_cols <= 256, what,
              ": fp32 row map alignment");
  CUtensorMap m;
  cuuint64_t gd[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t gs[1] = {(cuuint64_t)cols * 4};
  cuuint32_t bx[2] = {box_cols, 1u}, es[2] = {1, 1};
  CUresult r = tc5_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), gd, gs, bx, es,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (", what, ") failed: ", (int)r);
  return m;
}

}  // namespace mamf
