// Persistent tcgen05 GEMM for sm_100a: dense, grouped-M (MoE forward / data-gradient) and
// grouped-K (MoE weight-gradient) problems.
//
//   D[M, N] (+)= alpha * sum_k A(m, k) * B(n, k)    bf16 operands, fp32 accumulation in TMEM
//
// Operand layouts (per operand, compile-time):
//   K-major : A stored [M][K] / B stored [N][K]      (contraction dim contiguous)
//   MN-major: A stored [K][M] / B stored [K][N]      (the M / N dim contiguous)
// Modes:
//   0 dense     : one problem.
//   1 grouped-M : A rows (and D rows) are split into groups by `seg` (row offsets, multiples of
//                 64); group g multiplies by B[g] (3-D B).  MoE: X_perm @ W_e^T and dH @ W_e.
//   2 grouped-K : the contraction dim is split by `seg`; group g writes D[g] (3-D D).
//                 MoE: dW_e = dY_e^T X_e.  `seg` must be 64-aligned (zero-padded rows).
//   3 gathered-A: tensor-parallel all-gather -> GEMM.  A's rows are split into shards of
//                 `shard_rows`; shard r is read by TMA (no multicast) from tensor map r, which
//                 covers rank r's symmetric buffer (peer memory over NVLink); each rank starts
//                 with its own shard, so the remote tiles stream in while local tiles compute.
//   4 scattered-D: GEMM -> reduce-scatter.  Rows of shard r are written by the epilogue to
//                 d_ptrs[r] (rank r's staging slot for this rank, peer memory over NVLink);
//                 each rank starts with the next rank's shard and does its own last.
//
// Structure (one CTA per SM, 192 threads):
//   warp 0      TMA producer (one lane): A/B tiles -> a STAGES-deep shared-memory ring,
//               128-byte swizzle, completion counted on mbarriers (expect_tx).  No multicast.
//   warp 1      TMEM allocator + MMA issuer (one lane): tcgen05.mma.cta_group::1.kind::f16,
//               M=128 x N=BN x K=16 per instruction, 4 per 64-wide k-block; tcgen05.commit
//               releases the smem stage and, at tile end, publishes the accumulator.
//   warps 2..5  epilogue: tcgen05.ld 32x32b.x32 from a double-buffered accumulator (2*BN TMEM
//               columns), scale, convert; dense / grouped modes: stage 32 x 128-byte blocks in shared
//               memory and write them with bulk tensor stores, or bulk tensor reduce-adds that
//               accumulate straight into fp32 gradient buffers at L2; TP modes: per-thread
//               stores.
// Grouped-M launches use an upper bound on the tile count (no host synchronisation); tiles past
// the device-side tile table are skipped identically by all three roles.
// Every wait is bounded (clock64); on timeout the CTA records an error code in g_mamf_gemm_err,
// stops issuing work, waits a bounded time for in-flight copies, frees its TMEM and returns.
#include "common.cuh"

#include <cudaTypedefs.h>

namespace mamf {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int NUM_THREADS = 192;
constexpr long long WAIT_CYCLES = 4000000000LL;   // ~2 s at 1.9 GHz

__device__ int g_mamf_gemm_err = 0;

struct Params {
  int M, N, K;          // dense sizes (grouped-M: M = total rows; grouped-K: K = total rows)
  int G;                // groups (1 for dense)
  const int* seg;       // [G+1] group offsets (grouped modes), multiples of 64
  const int* tile_off;  // [G+1] cumulative m-tile counts (grouped-M)
  int n_tiles_n;
  int total_tiles;
  int group_m;          // dense: tile raster walks group_m m-tiles before the next n-tile
  int shard_rows;       // modes 3 / 4: rows per rank shard (multiple of BM)
  int rank_shift;       // modes 3 / 4: m-tile rotation (start position of this rank)
  void* d_ptrs[8];      // mode 4: per-shard output base
  void* D;
  int64_t ldd;          // row stride of D (elements)
  int64_t d_gstride;    // grouped-K: stride between D[g] (elements)
  float alpha;
};

// ---- PTX helpers ------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// One try; the thread is suspended until the phase completes or about 1 ms passes (suspend-time
// hint), so waiting warps leave the issue slots to the epilogue warps.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u) : "memory");
  return ok != 0;
}
// Bounded wait.  Returns false (and records `code`) on timeout or if another role already failed.
// The error word (a global load) and the clock are read every 64th unsuccessful try only.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t n = 1;; ++n) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((n & 63u) == 0) {
      if (*((volatile int*)&g_mamf_gemm_err) != 0) return false;
      if (clock64() - t0 > WAIT_CYCLES) {
        atomicCAS(&g_mamf_gemm_err, 0, code);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1) : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2) : "memory");
}

// Bulk tensor store / reduce-add from shared memory (epilogue of the dense and grouped-K modes).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];"
               ::"l"(map), "r"(smem_u32(src)), "r"(c0), "r"(c1) : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];"
               ::"l"(map), "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2) : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];"
               ::"l"(map), "r"(smem_u32(src)), "r"(c0), "r"(c1) : "memory");
}
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];"
               ::"l"(map), "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// UMMA shared-memory descriptor (sm100 layout: version 1 at bits 46-47, swizzle at 61-63).
//   K-major SW128 : LBO = 16 B (unused), SBO = 1024 B (8 rows x 128 B); +32 B per K=16 step.
//   MN-major SW128: LBO = bytes between 64-element MN groups, SBO = 1024 B per 8 K-rows;
//                   +2048 B (16 K-rows) per K=16 step.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;            // version = 1 (Blackwell)
  d |= (uint64_t)2 << 61;            // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: bf16 x bf16 -> f32, M=128, N=n.
__host__ __device__ constexpr uint32_t instr_desc(int n, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&r)[32]) {
  uint32_t v[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) r[i] = __uint_as_float(v[i]);
}

// ---- tile scheduling ---------------------------------------------------------------------------
struct Tile { int g, m0, n0, m_end; };   // g < 0: no tile;  m_end: first row not owned by the group

template <int MODE>
__device__ __forceinline__ Tile tile_of(const Params& p, int t) {
  Tile r;
  if (MODE == 1) {
    const int tm = t / p.n_tiles_n, tn = t - tm * p.n_tiles_n;
    if (tm >= p.tile_off[p.G]) { r.g = -1; r.m0 = r.n0 = r.m_end = 0; return r; }
    int lo = 0, hi = p.G;   // find g with tile_off[g] <= tm < tile_off[g+1]
    while (hi - lo > 1) { const int mid = (lo + hi) >> 1; if (p.tile_off[mid] <= tm) lo = mid; else hi = mid; }
    r.g = lo;
    r.m0 = p.seg[lo] + (tm - p.tile_off[lo]) * BM;
    r.m_end = p.seg[lo + 1];
    r.n0 = tn;
  } else if (MODE == 0 || MODE == 3 || MODE == 4) {
    // grouped raster: the CTAs running at one time share a panel of group_m m-tiles (A rows stay
    // in L2) and a few n-tiles, so each B tile is fetched from DRAM about once per panel
    const int m_tiles = (p.M + BM - 1) / BM;
    const int span = p.group_m * p.n_tiles_n;
    const int grp = t / span, first = grp * p.group_m;
    const int gm = min(p.group_m, m_tiles - first);
    const int local = t - grp * span;
    int tm = first + local % gm;
    const int tn = local / gm;
    if (MODE >= 3) tm = (tm + p.rank_shift) % m_tiles;
    r.g = (MODE >= 3) ? (tm * BM) / p.shard_rows : 0;
    r.m0 = tm * BM;
    r.m_end = p.M;
    r.n0 = tn;
  } else {
    const int per_g = ((p.M + BM - 1) / BM) * p.n_tiles_n;
    r.g = t / per_g;
    const int tt = t - r.g * per_g;
    const int tm = tt / p.n_tiles_n, tn = tt - tm * p.n_tiles_n;
    r.m0 = tm * BM;
    r.m_end = p.M;
    r.n0 = tn;
  }
  return r;
}

template <int MODE>
__device__ __forceinline__ void k_range(const Params& p, const Tile& tl, int& k0, int& nk) {
  if (MODE == 2) {
    k0 = p.seg[tl.g];
    nk = (p.seg[tl.g + 1] - k0 + BK - 1) / BK;
  } else {
    k0 = 0;
    nk = (p.K + BK - 1) / BK;
  }
}

// ---- the kernel -----------------------------------------------------------------------------------
struct MapSet { CUtensorMap m[8]; };   // mode 3: one A tensor map per rank shard; modes 0/2: m[0] = D map

// Dense, grouped-M and grouped-K tiles are written by bulk tensor stores (bf16 / fp32) or bulk
// tensor reduce-adds (fp32 accumulation into gradient buffers, performed at L2 without a round
// trip through the SM): each epilogue warp stages a 32-row x 128-byte block in shared memory
// (128-byte swizzle, two buffers per warp) and one lane issues the copy.  Grouped-M groups start
// and end on 64-row boundaries, so a warp's 32 rows lie entirely inside or entirely past its
// group's end; warps past the end issue nothing.  The tensor-parallel modes keep per-thread
// stores (their outputs may be peer memory).
template <int MODE, typename OutT, bool ACCUM>
__host__ __device__ constexpr bool tma_epilogue() {
  return (MODE == 0 || MODE == 1 || MODE == 2) && !(sizeof(OutT) == 2 && ACCUM);
}
constexpr int EPI_BUF_BYTES = 32 * 128;                      // 32 rows x 128 bytes
constexpr int EPI_STAGE_BYTES = 4 * 2 * EPI_BUF_BYTES;       // 4 epilogue warps x 2 buffers

template <int BN, int STAGES, bool A_MN, bool B_MN, int MODE, typename OutT, bool ACCUM>
__global__ void __launch_bounds__(NUM_THREADS, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p,
            const __grid_constant__ MapSet tmAs) {
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int B_BYTES = BN * BK * 2;
  constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t IDESC = instr_desc(BN, A_MN, B_MN);
  constexpr int TMEM_COLS = 2 * BN <= 32 ? 32 : (2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512)));
  constexpr bool TMA_EPI = tma_epilogue<MODE, OutT, ACCUM>();
  constexpr int EPI_BYTES = TMA_EPI ? EPI_STAGE_BYTES : 0;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi = smem + STAGES * STAGE_BYTES;                 // epilogue staging (1024-aligned)
  uint64_t* full = reinterpret_cast<uint64_t*>(epi + EPI_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;     // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], 128); }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(tmem_slot)), "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------- TMA producer -------------------------------
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
      const Tile tl = tile_of<MODE>(p, t);
      if (tl.g < 0) continue;
      const int n0 = tl.n0 * BN;
      int k0, nk;
      k_range<MODE>(p, tl, k0, nk);
      for (int kb = 0; kb < nk; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, 1)) { ok = false; break; }
        uint8_t* sA = smem + stage * STAGE_BYTES;
        uint8_t* sB = sA + A_BYTES;
        mbar_expect_tx(&full[stage], STAGE_BYTES);
        const int kk = k0 + kb * BK;
        if (MODE == 3) {
          tma_load_2d(sA, &tmAs.m[tl.g], &full[stage], kk, tl.m0 - tl.g * p.shard_rows);
        } else if (!A_MN) {
          tma_load_2d(sA, &tmA, &full[stage], kk, tl.m0);
        } else {
#pragma unroll
          for (int h = 0; h < BM / 64; ++h) tma_load_2d(sA + h * 64 * BK * 2, &tmA, &full[stage], tl.m0 + 64 * h, kk);
        }
        if (!B_MN) {
          if (MODE == 1) tma_load_3d(sB, &tmB, &full[stage], kk, n0, tl.g);
          else tma_load_2d(sB, &tmB, &full[stage], kk, n0);
        } else {
#pragma unroll
          for (int h = 0; h < BN / 64; ++h) {
            if (MODE == 1) tma_load_3d(sB + h * 64 * BK * 2, &tmB, &full[stage], n0 + 64 * h, kk, tl.g);
            else tma_load_2d(sB + h * 64 * BK * 2, &tmB, &full[stage], n0 + 64 * h, kk);
          }
        }
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------- MMA issuer -------------------------------
    int stage = 0;
    uint32_t phase = 0;
    int local = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
      const Tile tl = tile_of<MODE>(p, t);
      if (tl.g < 0) continue;
      int k0, nk;
      k_range<MODE>(p, tl, k0, nk);
      const int buf = local & 1;
      const uint32_t use = (uint32_t)(local >> 1);
      if (!mbar_wait(&acc_empty[buf], (use & 1) ^ 1, 2)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
      for (int kb = 0; kb < nk; ++kb) {
        if (!mbar_wait(&full[stage], phase, 3)) { ok = false; break; }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + stage * STAGE_BYTES);
        const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint64_t ad = !A_MN ? smem_desc(a_addr + k * 32, 16, 1024)
                                    : smem_desc(a_addr + k * 16 * 128, 64 * BK * 2, 1024);
          const uint64_t bd = !B_MN ? smem_desc(b_addr + k * 32, 16, 1024)
                                    : smem_desc(b_addr + k * 16 * 128, 64 * BK * 2, 1024);
          umma_bf16(d_tmem, ad, bd, IDESC, (kb | k) ? 1u : 0u);
        }
        umma_commit(&empty[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      umma_commit(&acc_full[buf]);
      ++local;
    }
  } else if (warp >= 2) {
    // ------------------------------- epilogue -------------------------------
    const int sub = warp & 3;                  // TMEM lane quarter accessible to this warp
    const int row_in_tile = sub * 32 + lane;
    int local = 0;
    int epi_buf = 0;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x) {
      const Tile tl = tile_of<MODE>(p, t);
      if (tl.g < 0) continue;
      int k0, nk;
      k_range<MODE>(p, tl, k0, nk);
      const int buf = local & 1;
      const uint32_t use = (uint32_t)(local >> 1);
      ++local;
      if (!mbar_wait(&acc_full[buf], use & 1, 4)) break;
      tc_fence_after();
      const int row = tl.m0 + row_in_tile;
      const bool row_ok = row < tl.m_end;
      OutT* dbase = (MODE == 4)
          ? reinterpret_cast<OutT*>(p.d_ptrs[tl.g]) + (int64_t)(row - tl.g * p.shard_rows) * p.ldd
          : reinterpret_cast<OutT*>(p.D) + (MODE == 2 ? (int64_t)tl.g * p.d_gstride : 0) + (int64_t)row * p.ldd;
      const int n_base = tl.n0 * BN;
      if (nk == 0) {
        // empty contraction (a group without rows): the accumulator was never written
        if (!ACCUM && row_ok)
          for (int c = n_base; c < min(p.N, n_base + BN); ++c) dbase[c] = from_f<OutT>(0.f);
        tc_fence_before();
        mbar_arrive(&acc_empty[buf]);
        continue;
      }
      if constexpr (TMA_EPI) {
        // stage 32 rows x 128 bytes per copy: 32 fp32 columns, or 64 bf16 columns
        constexpr int COLS = 128 / (int)sizeof(OutT);
        const int row0 = tl.m0 + sub * 32;
        const bool warp_rows = MODE != 1 || row0 < tl.m_end;    // grouped-M: rows of this group
#pragma unroll 1
        for (int c = 0; c < BN && warp_rows; c += COLS) {
          float r[COLS];
          tmem_ld32(tmem_base + ((uint32_t)(sub * 32) << 16) + (uint32_t)(buf * BN + c),
                    *reinterpret_cast<float(*)[32]>(&r[0]));
          if constexpr (COLS == 64)
            tmem_ld32(tmem_base + ((uint32_t)(sub * 32) << 16) + (uint32_t)(buf * BN + c + 32),
                      *reinterpret_cast<float(*)[32]>(&r[32]));
          if (lane == 0) bulk_wait_read<1>();        // the copy that last read this buffer is done
          __syncwarp();
          uint8_t* sb = epi + (sub * 2 + epi_buf) * EPI_BUF_BYTES + lane * 128;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            uint4 v;
            if constexpr (sizeof(OutT) == 4) {
              v.x = __float_as_uint(p.alpha * r[4 * q]);     v.y = __float_as_uint(p.alpha * r[4 * q + 1]);
              v.z = __float_as_uint(p.alpha * r[4 * q + 2]); v.w = __float_as_uint(p.alpha * r[4 * q + 3]);
            } else {
              __nv_bfloat162 b0 = __floats2bfloat162_rn(p.alpha * r[8 * q], p.alpha * r[8 * q + 1]);
              __nv_bfloat162 b1 = __floats2bfloat162_rn(p.alpha * r[8 * q + 2], p.alpha * r[8 * q + 3]);
              __nv_bfloat162 b2 = __floats2bfloat162_rn(p.alpha * r[8 * q + 4], p.alpha * r[8 * q + 5]);
              __nv_bfloat162 b3 = __floats2bfloat162_rn(p.alpha * r[8 * q + 6], p.alpha * r[8 * q + 7]);
              v.x = *reinterpret_cast<uint32_t*>(&b0); v.y = *reinterpret_cast<uint32_t*>(&b1);
              v.z = *reinterpret_cast<uint32_t*>(&b2); v.w = *reinterpret_cast<uint32_t*>(&b3);
            }
            *reinterpret_cast<uint4*>(sb + ((q ^ (lane & 7)) << 4)) = v;   // 128-byte swizzle
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            const void* src = epi + (sub * 2 + epi_buf) * EPI_BUF_BYTES;
            const int col = n_base + c;
            if constexpr (MODE == 2) {
              if (ACCUM) tma_reduce_add_3d(&tmAs.m[0], src, col, row0, tl.g);
              else tma_store_3d(&tmAs.m[0], src, col, row0, tl.g);
            } else {
              if (ACCUM) tma_reduce_add_2d(&tmAs.m[0], src, col, row0);
              else tma_store_2d(&tmAs.m[0], src, col, row0);
            }
            bulk_commit();
          }
          epi_buf ^= 1;
        }
      } else {
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        float r[32];
        tmem_ld32(tmem_base + ((uint32_t)(sub * 32) << 16) + (uint32_t)(buf * BN + c), r);
        if (row_ok) {
          const int col0 = n_base + c;
          if (col0 + 32 <= p.N) {
            if constexpr (sizeof(OutT) == 2) {
              if (ACCUM) {
#pragma unroll
                for (int i = 0; i < 32; ++i) dbase[col0 + i] = from_f<OutT>(to_f(dbase[col0 + i]) + p.alpha * r[i]);
              } else {
                Vec16<OutT> v[4];
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i / 8].v[i % 8] = from_f<OutT>(p.alpha * r[i]);
#pragma unroll
                for (int q = 0; q < 4; ++q) st16(dbase + col0 + 8 * q, v[q]);
              }
            } else {
              float4* d4 = reinterpret_cast<float4*>(dbase + col0);
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                float4 o = make_float4(p.alpha * r[4 * q], p.alpha * r[4 * q + 1], p.alpha * r[4 * q + 2], p.alpha * r[4 * q + 3]);
                if (ACCUM) { const float4 x = d4[q]; o.x += x.x; o.y += x.y; o.z += x.z; o.w += x.w; }
                d4[q] = o;
              }
            }
          } else {
            for (int i = 0; i < 32 && col0 + i < p.N; ++i) {
              const float v = p.alpha * r[i];
              if (ACCUM) dbase[col0 + i] = from_f<OutT>(to_f(dbase[col0 + i]) + v);
              else dbase[col0 + i] = from_f<OutT>(v);
            }
          }
        }
      }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
    if (TMA_EPI && lane == 0) bulk_wait_all();    // every staged block written before exit
  }

  __syncwarp();
  if (*((volatile int*)&g_mamf_gemm_err) != 0) {
    // a role gave up: let any bulk copy already issued by this CTA land before teardown
    const long long t0 = clock64();
    while (clock64() - t0 < 20000000LL) { }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
  }
}

// ---- host side -----------------------------------------------------------------------------------
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    MAMF_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && ptr, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeFn>(ptr);
  }
  return fn;
}

// bf16 tensor map.  dims/strides innermost first; strides in bytes for dims >= 1.
static CUtensorMap make_map(const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
                            uint32_t box0, uint32_t box1) {
  TORCH_CHECK(aligned16(base), "tcgen05 gemm: operand base must be 16-byte aligned");
  for (int i = 0; i < rank - 1; ++i) TORCH_CHECK(strides_bytes[i] % 16 == 0, "tcgen05 gemm: strides must be 16-byte multiples");
  CUtensorMap m;
  cuuint64_t gd[3], gs[2];
  cuuint32_t bx[3] = {box0, box1, 1}, es[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) gd[i] = dims[i];
  for (int i = 0; i < rank - 1; ++i) gs[i] = strides_bytes[i];
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), gd, gs, bx, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

// Output tensor map for the bulk-store epilogue: box = 128 bytes x 32 rows, 128-byte swizzle.
// dims/strides innermost first (strides in bytes for dims >= 1).
static CUtensorMap make_map_d(const at::Tensor& D, int rank, const uint64_t* dims, const uint64_t* strides_bytes) {
  const bool f32 = D.scalar_type() == at::kFloat;
  TORCH_CHECK(f32 || D.scalar_type() == at::kBFloat16, "tcgen05 gemm: bf16 or fp32 output");
  TORCH_CHECK(aligned16(D.data_ptr()), "tcgen05 gemm: output base must be 16-byte aligned");
  for (int i = 0; i < rank - 1; ++i) TORCH_CHECK(strides_bytes[i] % 16 == 0, "tcgen05 gemm: output strides must be 16-byte multiples");
  CUtensorMap m;
  cuuint64_t gd[3], gs[2];
  cuuint32_t bx[3] = {f32 ? 32u : 64u, 32u, 1u}, es[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) gd[i] = dims[i];
  for (int i = 0; i < rank - 1; ++i) gs[i] = strides_bytes[i];
  CUresult r = encode_fn()(&m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank,
                           D.data_ptr(), gd, gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (output) failed: ", (int)r);
  return m;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int MODE, typename OutT, bool ACCUM>
static void launch(const CUtensorMap& a, const CUtensorMap& b, const Params& p, const MapSet& as) {
  auto k = gemm_kernel<BN, STAGES, A_MN, B_MN, MODE, OutT, ACCUM>;
  const int smem = STAGES * (BM * BK * 2 + BN * BK * 2) + 1024 + 256 +
                   (tma_epilogue<MODE, OutT, ACCUM>() ? EPI_STAGE_BYTES : 0);
  MAMF_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int grid = std::max(1, std::min(p.total_tiles, num_sms()));
  k<<<grid, NUM_THREADS, smem, stream()>>>(a, b, p, as);
  MAMF_LAUNCH_CHECK();
}

template <bool A_MN, bool B_MN, int MODE>
static void dispatch_out(const CUtensorMap& a, const CUtensorMap& b, const Params& p, at::ScalarType out,
                         bool accum, int bn, const MapSet& as = MapSet{}) {
  auto run = [&](auto bnc) {
    constexpr int BNV = decltype(bnc)::value;
    // stages: as many A + B k-blocks as fit next to the 32 KB epilogue staging in 227 KB
    constexpr int ST = BNV == 256 ? 4 : (BNV == 192 ? 4 : 6);
    if (MODE >= 3) {
      TORCH_CHECK(out == at::kBFloat16 && !accum, "tensor-parallel gemm: bf16 output without accumulation");
      return launch<BNV, ST, A_MN, B_MN, MODE, __nv_bfloat16, false>(a, b, p, as);
    } else {
      if (out == at::kBFloat16 && !accum) return launch<BNV, ST, A_MN, B_MN, MODE, __nv_bfloat16, false>(a, b, p, as);
      if (out == at::kFloat && !accum) return launch<BNV, ST, A_MN, B_MN, MODE, float, false>(a, b, p, as);
      if (out == at::kFloat && accum) return launch<BNV, ST, A_MN, B_MN, MODE, float, true>(a, b, p, as);
    }
    TORCH_CHECK(false, "tcgen05 gemm: unsupported output configuration");
  };
  if (bn == 256) run(std::integral_constant<int, 256>{});
  else if (bn == 192) run(std::integral_constant<int, 192>{});
  else run(std::integral_constant<int, 128>{});
}

}  // namespace gemm

// ---------------------------------------------------------------------------------------------------
// gemm_tn(A, a_mn, B, b_mn, D, accumulate, seg, tile_off, mode, alpha)
//   mode 0 dense:     A [M,K] | [K,M];  B [N,K] | [K,N];        D [M,N]
//   mode 1 grouped-M: A [Mt,K];         B [G,N,K] | [G,K,N];    D [Mt,N]; seg, tile_off [G+1] int32 (device)
//   mode 2 grouped-K: A [Kt,M] (MN);    B [Kt,N] (MN);          D [G,M,N]; seg [G+1] int32 (device)
void gemm_tn(at::Tensor A, bool a_mn, at::Tensor B, bool b_mn, at::Tensor D, bool accumulate,
             c10::optional<at::Tensor> seg, c10::optional<at::Tensor> tile_off, int64_t mode, double alpha) {
  using namespace gemm;
  c10::cuda::CUDAGuard guard(A.device());
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm: bf16 operands");
  TORCH_CHECK(A.stride(-1) == 1 && B.stride(-1) == 1 && D.stride(-1) == 1, "gemm: unit inner strides");
  Params p{};
  p.alpha = (float)alpha;
  p.D = D.data_ptr();
  p.G = 1;
  CUtensorMap ma, mb;
  const uint64_t esz = 2;
  int M, N, K;
  if (mode == 0 || mode == 1) {
    if (!a_mn) { M = A.size(0); K = A.size(1); } else { K = A.size(0); M = A.size(1); }
    if (mode == 0) {
      if (!b_mn) { N = B.size(0); TORCH_CHECK(B.size(1) == K, "gemm: K mismatch"); }
      else { N = B.size(1); TORCH_CHECK(B.size(0) == K, "gemm: K mismatch"); }
    } else {
      TORCH_CHECK(!a_mn, "grouped-M gemm: A must be K-major");
      p.G = B.size(0);
      if (!b_mn) { N = B.size(1); TORCH_CHECK(B.size(2) == K, "gemm: K mismatch"); }
      else { N = B.size(2); TORCH_CHECK(B.size(1) == K, "gemm: K mismatch"); }
    }
    TORCH_CHECK(D.dim() == 2 && D.size(0) == M && D.size(1) == N, "gemm: D shape");
    p.ldd = D.stride(0);
  } else {
    TORCH_CHECK(a_mn && b_mn, "grouped-K gemm: A and B must be MN-major");
    K = A.size(0); M = A.size(1); N = B.size(1);
    TORCH_CHECK(B.size(0) == K, "grouped-K gemm: rows mismatch");
    p.G = D.size(0);
    TORCH_CHECK(D.dim() == 3 && D.size(1) == M && D.size(2) == N, "grouped-K gemm: D shape");
    p.ldd = D.stride(1);
    p.d_gstride = D.stride(0);
  }
  p.M = M; p.N = N; p.K = K;
  // TMA needs the contiguous (innermost) dimension of every operand to be 16-byte aligned
  TORCH_CHECK((a_mn && b_mn) || K % 8 == 0, "gemm: K must be a multiple of 8 for K-major operands");
  TORCH_CHECK(!a_mn || M % 8 == 0, "gemm: M must be a multiple of 8 for an MN-major A");
  TORCH_CHECK(!b_mn || N % 8 == 0, "gemm: N must be a multiple of 8 for an MN-major B");
  const int64_t esz_d = D.element_size();
  TORCH_CHECK(aligned16(D.data_ptr()) && (p.ldd * esz_d) % 16 == 0 && (p.d_gstride * esz_d) % 16 == 0,
              "gemm: D must be 16-byte aligned with 16-byte-multiple row strides");
  // tile width: the one of 128 / 192 / 256 that pads N least (ties -> the wider tile, which reads
  // fewer A bytes per FLOP); grouped-K keeps 128 (more tiles per group).  192 serves the MoE expert
  // width 576 and the MTP FFN width 1152 without a padded tail.
  const int pad128 = (N + 127) / 128 * 128, pad192 = (N + 191) / 192 * 192, pad256 = (N + 255) / 256 * 256;
  int bn = 128;
  if (mode != 2 && N >= 192) {
    if (N >= 256 && pad256 <= pad192 && pad256 <= pad128) bn = 256;
    else if (pad192 <= pad128) bn = 192;
  }
  p.n_tiles_n = (N + bn - 1) / bn;
  if (!a_mn) {
    uint64_t dims[2] = {(uint64_t)K, (uint64_t)M}, st[1] = {(uint64_t)A.stride(0) * esz};
    ma = make_map(A.data_ptr(), 2, dims, st, BK, BM);
  } else {
    uint64_t dims[2] = {(uint64_t)M, (uint64_t)K}, st[1] = {(uint64_t)A.stride(0) * esz};
    ma = make_map(A.data_ptr(), 2, dims, st, 64, BK);
  }
  if (mode == 1) {
    if (!b_mn) {
      uint64_t dims[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)p.G};
      uint64_t st[2] = {(uint64_t)B.stride(1) * esz, (uint64_t)B.stride(0) * esz};
      mb = make_map(B.data_ptr(), 3, dims, st, BK, bn);
    } else {
      uint64_t dims[3] = {(uint64_t)N, (uint64_t)K, (uint64_t)p.G};
      uint64_t st[2] = {(uint64_t)B.stride(1) * esz, (uint64_t)B.stride(0) * esz};
      mb = make_map(B.data_ptr(), 3, dims, st, 64, BK);
    }
  } else if (!b_mn) {
    uint64_t dims[2] = {(uint64_t)K, (uint64_t)N}, st[1] = {(uint64_t)B.stride(0) * esz};
    mb = make_map(B.data_ptr(), 2, dims, st, BK, bn);
  } else {
    uint64_t dims[2] = {(uint64_t)N, (uint64_t)K}, st[1] = {(uint64_t)B.stride(0) * esz};
    mb = make_map(B.data_ptr(), 2, dims, st, 64, BK);
  }
  if (mode == 1) {
    TORCH_CHECK(seg.has_value() && tile_off.has_value(), "grouped gemm needs seg and tile_off (device int32)");
    TORCH_CHECK(seg->scalar_type() == at::kInt && tile_off->scalar_type() == at::kInt, "grouped gemm: int32 tables");
    TORCH_CHECK(seg->numel() == p.G + 1 && tile_off->numel() == p.G + 1, "grouped gemm: table sizes");
    p.seg = seg->data_ptr<int>();
    p.tile_off = tile_off->data_ptr<int>();
    p.total_tiles = ((M + BM - 1) / BM + p.G) * p.n_tiles_n;   // upper bound; extra tiles skipped
  } else if (mode == 2) {
    TORCH_CHECK(seg.has_value() && seg->scalar_type() == at::kInt && seg->numel() == p.G + 1,
                "grouped-K gemm needs seg [G+1] int32");
    p.seg = seg->data_ptr<int>();
    p.total_tiles = p.G * ((M + BM - 1) / BM) * p.n_tiles_n;
  } else {
    p.total_tiles = ((M + BM - 1) / BM) * p.n_tiles_n;
    const int64_t panel_bytes = (int64_t)BM * K * 2;           // one m-tile of A
    const int m_tiles = (M + BM - 1) / BM;
    p.group_m = (int)std::max<int64_t>(1, std::min<int64_t>({(int64_t)m_tiles, 32, (48ll << 20) / std::max<int64_t>(1, panel_bytes)}));
  }
  if (p.total_tiles == 0) return;
  const auto out = D.scalar_type();
  // dense / grouped-K outputs are written by bulk tensor stores (reduce-adds when accumulating)
  MapSet dm{};
  if (mode == 0 || mode == 1) {
    uint64_t dims[2] = {(uint64_t)N, (uint64_t)M}, st[1] = {(uint64_t)(p.ldd * esz_d)};
    dm.m[0] = make_map_d(D, 2, dims, st);
  } else if (mode == 2) {
    uint64_t dims[3] = {(uint64_t)N, (uint64_t)M, (uint64_t)p.G};
    uint64_t st[2] = {(uint64_t)(p.ldd * esz_d), (uint64_t)(p.d_gstride * esz_d)};
    dm.m[0] = make_map_d(D, 3, dims, st);
  }
  if (mode == 0) {
    if (!a_mn && !b_mn) dispatch_out<false, false, 0>(ma, mb, p, out, accumulate, bn, dm);
    else if (!a_mn && b_mn) dispatch_out<false, true, 0>(ma, mb, p, out, accumulate, bn, dm);
    else if (a_mn && b_mn) dispatch_out<true, true, 0>(ma, mb, p, out, accumulate, bn, dm);
    else dispatch_out<true, false, 0>(ma, mb, p, out, accumulate, bn, dm);
  } else if (mode == 1) {
    if (!b_mn) dispatch_out<false, false, 1>(ma, mb, p, out, accumulate, bn, dm);
    else dispatch_out<false, true, 1>(ma, mb, p, out, accumulate, bn, dm);
  } else {
    dispatch_out<true, true, 2>(ma, mb, p, out, accumulate, bn, dm);
  }
}

// ---- tensor-parallel fused GEMMs -------------------------------------------------------------------
static void tp_common(gemm::Params& p, int M, int N, int K, int shard_rows, int rank, int P, bool b_mn,
                      const at::Tensor& B, CUtensorMap& mb, int& bn) {
  using namespace gemm;
  TORCH_CHECK(P >= 1 && P <= 8 && rank >= 0 && rank < P, "tensor-parallel gemm: 1..8 ranks");
  TORCH_CHECK(shard_rows % BM == 0 && M == shard_rows * P, "tensor-parallel gemm: shard rows must be a multiple of 128");
  TORCH_CHECK(K % 8 == 0 && N % 8 == 0, "tensor-parallel gemm: K and N multiples of 8");
  p.M = M; p.N = N; p.K = K; p.G = 1;
  p.shard_rows = shard_rows;
  const int pad128 = (N + 127) / 128 * 128, pad256 = (N + 255) / 256 * 256;
  bn = (N >= 256 && pad256 <= pad128) ? 256 : 128;
  p.n_tiles_n = (N + bn - 1) / bn;
  const int m_tiles = M / BM;
  p.total_tiles = m_tiles * p.n_tiles_n;
  p.group_m = (int)std::max<int64_t>(1, std::min<int64_t>({(int64_t)m_tiles, 32, (48ll << 20) / ((int64_t)BM * K * 2)}));
  const uint64_t esz = 2;
  if (!b_mn) {
    TORCH_CHECK(B.size(0) == N && B.size(1) == K, "tensor-parallel gemm: B (N, K)");
    uint64_t dims[2] = {(uint64_t)K, (uint64_t)N}, st[1] = {(uint64_t)B.stride(0) * esz};
    mb = make_map(B.data_ptr(), 2, dims, st, BK, bn);
  } else {
    TORCH_CHECK(B.size(0) == K && B.size(1) == N, "tensor-parallel gemm: B (K, N)");
    uint64_t dims[2] = {(uint64_t)N, (uint64_t)K}, st[1] = {(uint64_t)B.stride(0) * esz};
    mb = make_map(B.data_ptr(), 2, dims, st, 64, BK);
  }
}

// All-gather -> GEMM: D (P*shard_rows, N) = [A_0; ...; A_{P-1}] B^T, A_r = rows at a_ptrs[r] (bf16,
// row stride lda elements, K columns; peer pointers of a symmetric buffer).
void gemm_ag(std::vector<int64_t> a_ptrs, int64_t shard_rows, int64_t lda, int64_t rank, at::Tensor B, bool b_mn,
             at::Tensor D) {
  using namespace gemm;
  c10::cuda::CUDAGuard guard(D.device());
  const int P = (int)a_ptrs.size();
  TORCH_CHECK(B.scalar_type() == at::kBFloat16 && D.scalar_type() == at::kBFloat16 && B.stride(-1) == 1 &&
              D.is_contiguous(), "gemm_ag: bf16 operands");
  const int K = b_mn ? B.size(0) : B.size(1), N = D.size(1), M = D.size(0);
  Params p{};
  CUtensorMap mb;
  int bn;
  tp_common(p, M, N, K, (int)shard_rows, (int)rank, P, b_mn, B, mb, bn);
  p.D = D.data_ptr();
  p.ldd = D.stride(0);
  p.alpha = 1.f;
  p.rank_shift = (int)(rank * (shard_rows / BM));
  MapSet as{};
  for (int r = 0; r < P; ++r) {
    TORCH_CHECK(a_ptrs[r] % 16 == 0 && (lda * 2) % 16 == 0, "gemm_ag: 16-byte aligned shards");
    uint64_t dims[2] = {(uint64_t)K, (uint64_t)shard_rows}, st[1] = {(uint64_t)lda * 2};
    as.m[r] = make_map(reinterpret_cast<void*>(a_ptrs[r]), 2, dims, st, BK, BM);
  }
  if (!b_mn) dispatch_out<false, false, 3>(as.m[0], mb, p, at::kBFloat16, false, bn, as);
  else dispatch_out<false, true, 3>(as.m[0], mb, p, at::kBFloat16, false, bn, as);
}

// GEMM -> reduce-scatter: rows of shard r of A B^T are written to d_ptrs[r] (bf16, row stride ldd).
void gemm_rs(at::Tensor A, at::Tensor B, bool b_mn, std::vector<int64_t> d_ptrs, int64_t shard_rows, int64_t ldd,
             int64_t rank) {
  using namespace gemm;
  c10::cuda::CUDAGuard guard(A.device());
  const int P = (int)d_ptrs.size();
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16 && A.stride(-1) == 1 &&
              B.stride(-1) == 1, "gemm_rs: bf16 operands");
  const int M = A.size(0), K = A.size(1), N = b_mn ? B.size(1) : B.size(0);
  Params p{};
  CUtensorMap mb;
  int bn;
  tp_common(p, M, N, K, (int)shard_rows, (int)rank, P, b_mn, B, mb, bn);
  p.ldd = ldd;
  p.alpha = 1.f;
  TORCH_CHECK((ldd * 2) % 16 == 0, "gemm_rs: 16-byte row stride");
  for (int r = 0; r < P; ++r) {
    TORCH_CHECK(d_ptrs[r] % 16 == 0, "gemm_rs: 16-byte aligned outputs");
    p.d_ptrs[r] = reinterpret_cast<void*>(d_ptrs[r]);
  }
  // start with the next rank's shard, finish with this rank's own
  p.rank_shift = (int)(((rank + 1) % P) * (shard_rows / BM));
  uint64_t dims[2] = {(uint64_t)K, (uint64_t)M}, st[1] = {(uint64_t)A.stride(0) * 2};
  CUtensorMap ma = make_map(A.data_ptr(), 2, dims, st, BK, BM);
  if (!b_mn) dispatch_out<false, false, 4>(ma, mb, p, at::kBFloat16, false, bn);
  else dispatch_out<false, true, 4>(ma, mb, p, at::kBFloat16, false, bn);
}

int64_t gemm_error() {
  int v = 0;
  MAMF_CUDA_CHECK(cudaMemcpyFromSymbol(&v, gemm::g_mamf_gemm_err, sizeof(int)));
  return v;
}

void gemm_clear_error() {
  int z = 0;
  MAMF_CUDA_CHECK(cudaMemcpyToSymbol(gemm::g_mamf_gemm_err, &z, sizeof(int)));
}

}  // namespace mamf
