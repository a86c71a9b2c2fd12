// Flash attention backward on the 5th-generation tensor cores (tcgen05 / TMEM / TMA).
//
// Gradients of softmax attention at head_dim 128 for one or two query streams that share the K / V
// tensors (csrc/flash_tc.cu is the matching forward):
//   plain / GQA:    one stream, O = softmax(Q K^T s) V
//   differential:   two streams Q1, Q2 with out = (O1 - lam O2) / (1 - lam + 1e-8), so
//                   dO1 = c1 dout, dO2 = c2 dout with c1 = 1 / (1 - lam + 1e-8), c2 = -lam c1;
//                   the per-stream, per-head factor c is applied inside the kernel, so dout is
//                   read once and dK / dV of both maps accumulate in the same tensor memory.
// Reference semantics: mamformer/layers/kda_diff.py:826-862 (autograd through the two
// materialised S x S softmax maps and the lambda combine), dsa.py:276-317, attention.py:157-181.
// Masking is the band lo <= key - (query + Skv - S) <= hi (causal: lo = -inf, hi = 0).
//
// Math per (key block, query tile), s = softmax scale, L = row log-sum-exp of the forward,
// D = rowsum(dO . O):
//   S^T = K Q^T,  P^T = exp(s S^T - L),  dP^T = V dO^T,  dS^T = P^T (dP^T - D)
//   dV += c P^T dout,  dK += s c dS^T Q,  dQ += s c dS K
//
// One CTA = 128 keys of one KV head (the TMEM lanes); it loops over the query heads of that KV
// head (GQA), the streams, and the 64-query tiles that reach its keys, so dK and dV accumulate in
// tensor memory without atomics.  14 warps:
//   warps 0-7   softmax gradient (thread = key row; warps w and w + 4 share the lanes of TMEM
//               subpartition w and take query columns 0-31 / 32-63): read S^T and dP^T with
//               tcgen05.ld, write c P^T and c dS^T as packed bf16 back into the S^T columns
//               (the A operands of the dV / dK products) and c dS^T into shared memory (the B
//               operand of the dQ product);
//   warps 8-11  dQ epilogue (thread = head dimension): read dQ^T from TMEM and add it to the fp32
//               dQ accumulator (B, H, S, 128) with fp32 reductions at L2 (one 128-byte line per
//               warp instruction: the 32 lanes are 32 consecutive dimensions of one query);
//   warp 12     TMA producer (one lane): K / V once, then Q, dO and the tile's {L, D} row for
//               each tile into a 4-deep ring (no multicast: every map covers this GPU's memory
//               only), so tile t + 1 is loaded while tiles t - 2 .. t still hold their stages;
//   warp 13     TMEM allocator + MMA issuer (one lane).
// MMAs per tile (M 128): S^T = K Q^T and dP^T = V dO^T (N 64, K 128, both operands K-major);
// dQ^T = K^T dS^T (N 64, K 128 keys; A = the K tile read MN-major, B = dS^T from shared memory);
// dV += (cP^T) dO and dK += (c dS^T) Q (N 128, K 64; A from TMEM, B MN-major).
// TMEM (512 columns): region r = 0, 1 (double-buffered tiles) at r * 128: S^T in columns 0-63
// (each softmax warp overwrites its own 32 columns with 16 of packed c P^T and 16 of packed
// c dS^T), dP^T in 64-127 (overwritten by dQ^T);
// dV at 256-383, dK at 384-511.  The MMA thread issues dQ^T before dV / dK so the dQ epilogue of a
// tile overlaps the tile's last two products, and a region is reused (S^T of tile t + 2) only
// after the epilogue has read dQ^T of tile t.  The tensor pipe runs one thread's MMAs in order,
// and tcgen05.commit arrives only when every earlier MMA has completed, so a region's bf16
// operands are free once the next S^T of that region is done.  The single dS^T shared-memory
// buffer is rewritten for tile t + 1 only after the dQ^T product of tile t has completed (its
// commit barrier), which the softmax warps wait for after their exponentials.
// Waiting threads sleep in mbarrier.try_wait (suspend-time hint) and read the error word only
// every 64th try, so they neither take issue slots nor add an L2 round trip to a hand-off.
// Every wait is bounded (clock64); a timeout records a code in g_mamf_fa5b_err, stops the CTA's
// work, waits a bounded time for its copies in flight, frees TMEM and returns.  Every global
// access computed from the tile indices is checked against its tensor's size; a bad index is
// recorded (code >= 100) and the access skipped.
#include "tc5.cuh"

namespace mamf {
namespace fa5b {

using namespace tc5;

constexpr int BK = 128;            // keys per CTA
constexpr int BQ = 64;             // queries per tile
constexpr int HD = 128;            // head dim
constexpr int QS = 4;              // Q / dO / {L, D} ring depth
constexpr int NT = 448;            // 14 warps
constexpr long long WAIT_CYCLES = 4000000000LL;   // ~2 s

__device__ int g_mamf_fa5b_err = 0;

constexpr int KV_BYTES = BK * HD * 2;     // 32 KB (two 16 KB chunks of 64 dims)
constexpr int QT_BYTES = BQ * HD * 2;     // 16 KB (two 8 KB chunks)
constexpr int DS_BYTES = BK * BQ * 2;     // 16 KB: c dS^T, 128 key rows x 64 queries, 128-byte swizzle
constexpr int LD_BYTES = BQ * 8;          // {L * log2 e, D} of 64 queries
constexpr int OFF_K = 0, OFF_V = KV_BYTES;
constexpr int OFF_Q = 2 * KV_BYTES;                      // [QS]
constexpr int OFF_DO = OFF_Q + QS * QT_BYTES;            // [QS]
constexpr int OFF_DS = OFF_DO + QS * QT_BYTES;           // one buffer
constexpr int OFF_LD = OFF_DS + DS_BYTES;                // [QS]
constexpr int OFF_BAR = OFF_LD + QS * LD_BYTES;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;

struct Params {
  int B, S, Skv, H, G, off, lo, hi, Spad, nstream;
  float scale_log2;            // softmax scale * log2(e)
  float scale;                 // softmax scale (applied to dK here and to dQ by the convert pass)
  const float* coef;           // (nstream, H) factor of dout per stream and head, or null (1)
  float* dq;                   // (nstream, B, H, Spad, HD) fp32 accumulators, zeroed
  __nv_bfloat16* dk;           // (B, Skv, G, HD)
  __nv_bfloat16* dv;
  int64_t dq_n, kv_n;          // element counts of dq and dk / dv (checked indices)
  int skip_dq_red;             // profiling switch (MAMF_FA5B_SKIP_DQ_RED=1): drop the dQ reductions
};
// ld: the {L * log2 e (+inf: no key / padding), D} pairs as rows (stream, b, h) of 2 * Spad fp32
struct Maps { CUtensorMap q0, q1, k, v, dout, ld; };

// false (and the code recorded) when i is outside [0, n)
__device__ __forceinline__ bool in_range(int64_t i, int64_t n, int code) {
  if (i >= 0 && i < n) return true;
  atomicCAS(&g_mamf_fa5b_err, 0, code);
  return false;
}

__device__ __forceinline__ bool wait(uint64_t* b, uint32_t parity, int code) {
  return tc5::bar_wait(b, parity, code, &g_mamf_fa5b_err, WAIT_CYCLES);
}

// tile t of this CTA -> (stream, query head, first query)
struct Tile { int s, h, q0; };
__device__ __forceinline__ Tile tile_of(int t, int nqt, int qt0, int hpg, int g) {
  const int per_s = hpg * nqt;
  Tile r;
  r.s = t / per_s;
  const int rem = t - r.s * per_s;
  const int hh = rem / nqt;
  r.h = g * hpg + hh;
  r.q0 = (qt0 + rem - hh * nqt) * BQ;
  return r;
}

__global__ void __launch_bounds__(NT, 1) fa5_bwd_kernel(const __grid_constant__ Maps mp, Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* kv_full = bars;              // 1
  uint64_t* qd_full = bars + 1;          // [QS]
  uint64_t* qd_empty = qd_full + QS;     // [QS]
  uint64_t* s_full = qd_empty + QS;      // [2] S^T, dP^T of the region's tile are in TMEM
  uint64_t* p_full = s_full + 2;         // [2] c P^T, c dS^T written (256 arrivals)
  uint64_t* dq_full = p_full + 2;        // [2] dQ^T in TMEM
  uint64_t* r_free = dq_full + 2;        // [2] dQ^T read out (128 arrivals)
  uint64_t* acc_full = r_free + 2;       // dV, dK complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x, b = blockIdx.y, kb = blockIdx.z;   // key blocks slowest: heavy (causal) first
  const int hpg = p.H / p.G;
  const int k0 = kb * BK;
  const int krows = min(BK, p.Skv - k0);
  // queries reached by these keys: key - (q + off) in [lo, hi]
  const int qmin = max(0, k0 - p.off - p.hi);
  const int qmax = min(p.S - 1, k0 + krows - 1 - p.off - p.lo);
  const int qt0 = qmin / BQ;
  const int nqt = qmax >= qmin ? qmax / BQ - qt0 + 1 : 0;
  const int ntile = p.nstream * hpg * nqt;

  if (threadIdx.x == 0) {
    bar_init(kv_full, 1);
    for (int i = 0; i < QS; ++i) { bar_init(&qd_full[i], 1); bar_init(&qd_empty[i], 1); }
    for (int i = 0; i < 2; ++i) {
      bar_init(&s_full[i], 1); bar_init(&p_full[i], 256); bar_init(&dq_full[i], 1); bar_init(&r_free[i], 128);
    }
    bar_init(acc_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 13) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(su32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 12) {
    // ------------------------------- producer -------------------------------
    if (lane == 0 && ntile > 0) {
      bar_expect_tx(kv_full, 2 * KV_BYTES);
      for (int c = 0; c < 2; ++c) {
        tma_3d(sm + OFF_K + c * (KV_BYTES / 2), &mp.k, kv_full, c * 64, g, b * p.Skv + k0);
        tma_3d(sm + OFF_V + c * (KV_BYTES / 2), &mp.v, kv_full, c * 64, g, b * p.Skv + k0);
      }
      int issued = 0;
      for (int t = 0; t < ntile; ++t) {
        const int st = t % QS;
        if (!wait(&qd_empty[st], (uint32_t)(((t / QS) & 1) ^ 1), 31)) break;
        const Tile tl = tile_of(t, nqt, qt0, hpg, g);
        const CUtensorMap* qm = tl.s ? &mp.q1 : &mp.q0;
        bar_expect_tx(&qd_full[st], 2 * QT_BYTES + LD_BYTES);
        for (int c = 0; c < 2; ++c) {
          tma_3d(sm + OFF_Q + st * QT_BYTES + c * (QT_BYTES / 2), qm, &qd_full[st], c * 64, tl.h, b * p.S + tl.q0);
          tma_3d(sm + OFF_DO + st * QT_BYTES + c * (QT_BYTES / 2), &mp.dout, &qd_full[st], c * 64, tl.h, b * p.S + tl.q0);
        }
        // {L, D} of the tile's 64 queries: 128 fp32 of row (stream, b, h) from column 2 * q0
        tma_2d(sm + OFF_LD + st * LD_BYTES, &mp.ld, &qd_full[st], 2 * tl.q0, (tl.s * p.B + b) * p.H + tl.h);
        ++issued;
      }
      if (*((volatile int*)&g_mamf_fa5b_err) != 0) {   // error exit: let the copies in flight land
        wait(kv_full, 0, 0);
        for (int t = 0; t < issued; ++t) wait(&qd_full[t % QS], (uint32_t)((t / QS) & 1), 0);
      }
    }
  } else if (warp == 13) {
    // ------------------------------- MMA issuer -------------------------------
    if (lane == 0 && ntile > 0) {
      constexpr uint32_t ID_S = idesc_bf16(128, BQ, false, false);    // S^T, dP^T
      constexpr uint32_t ID_DQ = idesc_bf16(128, BQ, true, true);     // dQ^T = K^T dS^T
      constexpr uint32_t ID_KV = idesc_bf16(128, HD, false, true);    // dV, dK (A from TMEM)
      const uint32_t sK = su32(sm + OFF_K), sV = su32(sm + OFF_V);
      bool ok = wait(kv_full, 0, 32);
      fence_after();
      auto issue_sdp = [&](int t) -> bool {
        const int st = t % QS, r = t & 1;
        if (!wait(&qd_full[st], (uint32_t)((t / QS) & 1), 33)) return false;
        if (t >= 2 && !wait(&r_free[r], (uint32_t)(((t - 2) >> 1) & 1), 34)) return false;
        fence_after();
        const uint32_t sQ = su32(sm + OFF_Q + st * QT_BYTES), sO = su32(sm + OFF_DO + st * QT_BYTES);
        const uint32_t dS = tmem + (uint32_t)(r * 128), dP = dS + 64u;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t ko = (k >> 2) * (KV_BYTES / 2) + (k & 3) * 32, qo = (k >> 2) * (QT_BYTES / 2) + (k & 3) * 32;
          mma_ss(dS, sdesc(sK + ko, 16, 1024), sdesc(sQ + qo, 16, 1024), ID_S, k > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint32_t ko = (k >> 2) * (KV_BYTES / 2) + (k & 3) * 32, qo = (k >> 2) * (QT_BYTES / 2) + (k & 3) * 32;
          mma_ss(dP, sdesc(sV + ko, 16, 1024), sdesc(sO + qo, 16, 1024), ID_S, k > 0 ? 1u : 0u);
        }
        commit(&s_full[r]);
        return true;
      };
      if (ok) ok = issue_sdp(0);
      for (int t = 0; t < ntile && ok; ++t) {
        if (t + 1 < ntile && !issue_sdp(t + 1)) { ok = false; break; }
        const int st = t % QS, r = t & 1;
        if (!wait(&p_full[r], (uint32_t)((t >> 1) & 1), 35)) { ok = false; break; }
        fence_after();
        const uint32_t sQ = su32(sm + OFF_Q + st * QT_BYTES), sO = su32(sm + OFF_DO + st * QT_BYTES);
        const uint32_t sDS = su32(sm + OFF_DS);
        const uint32_t reg = tmem + (uint32_t)(r * 128);
        // dQ^T (128 dims x 64 queries) = K^T dS^T over the 128 keys, into the dP^T columns
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          mma_ss(reg + 64u, sdesc(sK + k * 2048, KV_BYTES / 2, 1024), sdesc(sDS + k * 2048, DS_BYTES, 1024), ID_DQ,
                 k > 0 ? 1u : 0u);
        commit(&dq_full[r]);
        // dV += (c P^T) dO, dK += (c dS^T) Q over the 64 queries
        // (queries 16k .. 16k+15: packed columns (k >> 1) * 32 + (k & 1) * 8, c dS^T 16 further)
#pragma unroll
        for (int k = 0; k < BQ / 16; ++k) {
          const uint32_t acc = (t > 0 || k > 0) ? 1u : 0u;
          const uint32_t pc = reg + (uint32_t)((k >> 1) * 32 + (k & 1) * 8);
          mma_ts(tmem + 256u, pc, sdesc(sO + k * 2048, QT_BYTES / 2, 1024), ID_KV, acc);
          mma_ts(tmem + 384u, pc + 16u, sdesc(sQ + k * 2048, QT_BYTES / 2, 1024), ID_KV, acc);
        }
        commit(&qd_empty[st]);
      }
      // acc_full also tells this thread that no MMA is in flight when TMEM is freed
      commit(acc_full);
      wait(acc_full, 0, ok ? 36 : 0);
    }
  } else if (warp < 8) {
    // ------------------------------- softmax gradient -------------------------------
    const int hf = warp >> 2;                         // query columns hf*32 .. hf*32+31
    const int r = (warp & 3) * 32 + lane;             // key row = TMEM lane
    const int key = k0 + r;
    const bool key_ok = r < krows;
    const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    bool ok = true;
    for (int t = 0; t < ntile && ok; ++t) {
      const int st = t % QS, rg = t & 1;
      const Tile tt = tile_of(t, nqt, qt0, hpg, g);
      ok = __all_sync(0xffffffffu, wait(&s_full[rg], (uint32_t)((t >> 1) & 1), 41) &&
                                   wait(&qd_full[st], (uint32_t)((t / QS) & 1), 42));
      if (!ok) break;
      fence_after();
      // S^T first; dP^T's load stays in flight while the exponentials run
      uint32_t sr[32], dr[32];
      MAMF_TC5_LD32(sr, tl + (uint32_t)(rg * 128 + hf * 32));
      tld_wait();
      MAMF_TC5_LD32(dr, tl + (uint32_t)(rg * 128 + 64 + hf * 32));
      const float c = p.coef ? __ldg(p.coef + tt.s * p.H + tt.h) : 1.f;
      const float4* ld4 = reinterpret_cast<const float4*>(sm + OFF_LD + st * LD_BYTES) + hf * 16;   // {L, D} pairs
      const int qa = tt.q0 + hf * 32;                 // first query of this thread's columns
      // the whole 32 x 32 block inside the band and the key range: no per-element mask
      const bool full = key_ok && (key - (qa + 31) - p.off >= p.lo) && (key - qa - p.off <= p.hi);
      const bool mask = __any_sync(0xffffffffu, !full);
      float pv[32], dd[32];
#pragma unroll
      for (int j2 = 0; j2 < 16; ++j2) {
        const float4 L = ld4[j2];                     // {L, D} of queries 2 j2, 2 j2 + 1
        pv[2 * j2] = ex2(fmaf(__uint_as_float(sr[2 * j2]), p.scale_log2, -L.x));   // L = +inf gives 0
        pv[2 * j2 + 1] = ex2(fmaf(__uint_as_float(sr[2 * j2 + 1]), p.scale_log2, -L.z));
        dd[2 * j2] = L.y;
        dd[2 * j2 + 1] = L.w;
      }
      if (mask) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int d = key - (qa + j) - p.off;
          pv[j] = (key_ok && d >= p.lo && d <= p.hi) ? pv[j] : 0.f;
        }
      }
      tld_wait();
      uint32_t pk[16], dk[16];
#pragma unroll
      for (int j2 = 0; j2 < 16; ++j2) {
        const float p0 = pv[2 * j2] * c, p1 = pv[2 * j2 + 1] * c;
        pk[j2] = pack_bf16(p0, p1);
        dk[j2] = pack_bf16(p0 * (__uint_as_float(dr[2 * j2]) - dd[2 * j2]),
                           p1 * (__uint_as_float(dr[2 * j2 + 1]) - dd[2 * j2 + 1]));
      }
      // over this warp's own S^T columns (hf*32 .. hf*32+31, already read): c P^T in the first 16,
      // c dS^T in the last 16, so the two warps sharing these lanes never overwrite each other
      tst16_nowait(tl + (uint32_t)(rg * 128 + hf * 32), pk);
      tst16_nowait(tl + (uint32_t)(rg * 128 + hf * 32 + 16), dk);
      // c dS^T row r into shared memory (128-byte swizzle: 16-byte chunk c of row r at c ^ (r & 7)),
      // once the dQ^T product of the previous tile, which reads the buffer, has completed
      if (t > 0) {
        ok = __all_sync(0xffffffffu, wait(&dq_full[(t - 1) & 1], (uint32_t)(((t - 1) >> 1) & 1), 44));
        if (!ok) { tst_wait(); break; }
      }
      uint8_t* dsrow = sm + OFF_DS + r * 128;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int ch = hf * 4 + i;
        *reinterpret_cast<uint4*>(dsrow + ((ch ^ (r & 7)) << 4)) = make_uint4(dk[4 * i], dk[4 * i + 1], dk[4 * i + 2], dk[4 * i + 3]);
      }
      tst_wait();
      fence_async_smem();
      fence_before();
      bar_arrive(&p_full[rg]);
    }
    // ---- dV (warps 0-3) and dK (warps 4-7) of this thread's key row ----
    if (ok && ntile > 0) ok = __all_sync(0xffffffffu, wait(acc_full, 0, 43));
    if (ok) {
      fence_after();
      __nv_bfloat16* dst = hf ? p.dk : p.dv;
      const float f = hf ? p.scale : 1.f;
      const int64_t row = (((int64_t)b * p.Skv + key) * p.G + g) * HD;
#pragma unroll 1
      for (int cc = 0; cc < HD; cc += 32) {
        float o[32];
        if (ntile > 0) tld32(tl + (uint32_t)(256 + hf * 128 + cc), o);
        else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (key_ok && in_range(row + cc + 31, p.kv_n, 102)) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(dst + row + cc + 8 * q) =
                make_uint4(pack_bf16(o[8 * q] * f, o[8 * q + 1] * f), pack_bf16(o[8 * q + 2] * f, o[8 * q + 3] * f),
                           pack_bf16(o[8 * q + 4] * f, o[8 * q + 5] * f), pack_bf16(o[8 * q + 6] * f, o[8 * q + 7] * f));
        }
      }
    }
  } else {
    // ------------------------------- dQ epilogue (warps 8-11) -------------------------------
    const int d = (warp - 8) * 32 + lane;             // head dimension = TMEM lane
    const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    bool ok = true;
    for (int t = 0; t < ntile && ok; ++t) {
      const int rg = t & 1;
      const Tile tt = tile_of(t, nqt, qt0, hpg, g);
      ok = __all_sync(0xffffffffu, wait(&dq_full[rg], (uint32_t)((t >> 1) & 1), 51));
      if (!ok) break;
      fence_after();
      float v[64];
      tld64(tl + (uint32_t)(rg * 128 + 64), v);
      fence_before();
      bar_arrive(&r_free[rg]);
      // rows q0 .. q0+63 of the (stream, b, h) slab; rows past S land in its padding
      const int64_t base = ((((int64_t)tt.s * p.B + b) * p.H + tt.h) * p.Spad + tt.q0) * HD + d;
      if (!p.skip_dq_red && in_range(base + (int64_t)(BQ - 1) * HD, p.dq_n, 103)) {
#pragma unroll
        for (int j = 0; j < BQ; ++j) atomicAdd(p.dq + base + (int64_t)j * HD, v[j]);
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 13) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}

// {L * log2 e, D = rowsum(dout . o)} per (stream, b, h, query), padded rows {+inf, 0}; one warp per row
__global__ void fa5_bwd_prep_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ o0,
                                    const __nv_bfloat16* __restrict__ o1, const float* __restrict__ lse0,
                                    const float* __restrict__ lse1, float2* __restrict__ ld, int nstream, int B,
                                    int S, int H, int Spad) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)nstream * B * H * Spad;
  if (row >= rows) return;
  const int q = (int)(row % Spad);
  const int64_t sbh = row / Spad;
  const int h = (int)(sbh % H);
  const int64_t sb = sbh / H;
  const int bb = (int)(sb % B), s = (int)(sb / B);
  if (q >= S) {
    if (lane == 0) ld[row] = make_float2(INFINITY, 0.f);
    return;
  }
  const int64_t off = (((int64_t)bb * S + q) * H + h) * HD + lane * 4;
  if (!in_range(off + 3, (int64_t)B * S * H * HD, 104)) return;
  const __nv_bfloat16* o = s ? o1 : o0;
  const uint2 a = *reinterpret_cast<const uint2*>(dout + off);
  const uint2 c = *reinterpret_cast<const uint2*>(o + off);
  const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
  const __nv_bfloat162* c2 = reinterpret_cast<const __nv_bfloat162*>(&c);
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float2 x = __bfloat1622float2(a2[i]), y = __bfloat1622float2(c2[i]);
    acc = fmaf(x.x, y.x, fmaf(x.y, y.y, acc));
  }
  acc = warp_sum(acc);
  if (lane == 0) {
    const float l = (s ? lse1 : lse0)[((int64_t)bb * H + h) * S + q];
    ld[row] = make_float2(l * 1.4426950408889634f, acc);   // +inf (a row without keys) stays +inf
  }
}

// dq (B, S, H, HD) bf16 = scale * acc (B, H, Spad, HD) fp32; 4 elements per thread
__global__ void fa5_bwd_dq_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq, int B, int S, int H,
                                  int Spad, float scale) {
  const int64_t n4 = (int64_t)B * S * H * (HD / 4);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const int c4 = (int)(i % (HD / 4));
    const int64_t bqh = i / (HD / 4);
    const int h = (int)(bqh % H);
    const int64_t bq = bqh / H;
    const int q = (int)(bq % S), bb = (int)(bq / S);
    const int64_t src = (((int64_t)bb * H + h) * Spad + q) * HD + c4 * 4;
    if (!in_range(src + 3, (int64_t)B * H * Spad * HD, 105)) continue;
    const float4 v = *reinterpret_cast<const float4*>(acc + src);
    *reinterpret_cast<uint2*>(dq + i * 4) = make_uint2(tc5::pack_bf16(v.x * scale, v.y * scale),
                                                       tc5::pack_bf16(v.z * scale, v.w * scale));
  }
}

}  // namespace fa5b

// q1 (B, S, H, 128), q2 like q1 or none; k, v (B, Skv, G, 128); o1 (o2) the normalised stream
// outputs of the forward, lse1 (lse2) (B, H, S) natural-log row log-sum-exp; dout (B, S, H, 128);
// coef (nstream, H) fp32 factors of dout per stream and head, or none (1).
// Returns (dq1, dk, dv) or (dq1, dq2, dk, dv).
std::vector<at::Tensor> flash_tc_bwd(at::Tensor q1, c10::optional<at::Tensor> q2, at::Tensor k, at::Tensor v,
                                     at::Tensor o1, c10::optional<at::Tensor> o2, at::Tensor lse1,
                                     c10::optional<at::Tensor> lse2, at::Tensor dout, c10::optional<at::Tensor> coef,
                                     int64_t lo, int64_t hi, double scale) {
  using namespace fa5b;
  c10::cuda::CUDAGuard guard(q1.device());
  const int ns = q2.has_value() ? 2 : 1;
  Params p{};
  p.B = q1.size(0); p.S = q1.size(1); p.H = q1.size(2); p.Skv = k.size(1); p.G = k.size(2);
  TORCH_CHECK(k.sizes() == v.sizes() && k.size(0) == p.B && p.G > 0 && p.H % p.G == 0, "tcgen05 attention bwd: shapes");
  TORCH_CHECK(p.S <= p.Skv, "tcgen05 attention bwd: S <= Skv");
  TORCH_CHECK(dout.sizes() == q1.sizes() && o1.sizes() == q1.sizes() && lse1.numel() == (int64_t)p.B * p.H * p.S,
              "tcgen05 attention bwd: dout / o / lse like q");
  TORCH_CHECK(p.B <= 65535 && p.G <= 65535 && (p.Skv + BK - 1) / BK <= 65535, "tcgen05 attention bwd: grid limits");
  p.off = p.Skv - p.S;
  p.lo = (int)std::max<int64_t>(lo, -(1LL << 30));
  p.hi = (int)std::min<int64_t>(hi, (1LL << 30));
  p.scale = (float)scale;
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  p.Spad = (p.S + BQ - 1) / BQ * BQ;
  p.nstream = ns;
  dout = dout.contiguous();
  o1 = o1.contiguous();
  at::Tensor lse1c = lse1.to(at::kFloat).contiguous(), lse2c, o2c;
  Maps mp{};
  mp.q0 = tc5_head_map(q1, BQ, "tcgen05 attention bwd");
  mp.q1 = mp.q0;
  if (ns == 2) {
    TORCH_CHECK(q2->sizes() == q1.sizes() && o2.has_value() && o2->sizes() == q1.sizes() && lse2.has_value() &&
                lse2->numel() == lse1.numel(), "tcgen05 attention bwd: second stream like the first");
    mp.q1 = tc5_head_map(*q2, BQ, "tcgen05 attention bwd");
    o2c = o2->contiguous();
    lse2c = lse2->to(at::kFloat).contiguous();
  }
  mp.k = tc5_head_map(k.contiguous(), BK, "tcgen05 attention bwd");
  mp.v = tc5_head_map(v.contiguous(), BK, "tcgen05 attention bwd");
  mp.dout = tc5_head_map(dout, BQ, "tcgen05 attention bwd");
  at::Tensor coefc;
  if (coef.has_value()) {
    coefc = coef->to(at::kFloat).contiguous();
    TORCH_CHECK(coefc.numel() == (int64_t)ns * p.H, "tcgen05 attention bwd: coef (nstream, H)");
    p.coef = coefc.data_ptr<float>();
  }
  auto f32 = q1.options().dtype(at::kFloat);
  at::Tensor ld = at::empty({(int64_t)ns * p.B * p.H * p.Spad * 2}, f32);
  at::Tensor acc = at::zeros({(int64_t)ns * p.B * p.H * p.Spad * HD}, f32);
  at::Tensor dk = at::empty_like(k), dv = at::empty_like(v);
  mp.ld = tc5_rows_map_f32(ld.data_ptr<float>(), (int64_t)ns * p.B * p.H, 2 * (int64_t)p.Spad, 2 * BQ,
                           "tcgen05 attention bwd");
  p.dq = acc.data_ptr<float>();
  p.dk = (__nv_bfloat16*)dk.data_ptr();
  p.dv = (__nv_bfloat16*)dv.data_ptr();
  p.dq_n = acc.numel();
  p.kv_n = dk.numel();
  const bool dbg = std::getenv("MAMF_FA5B_DEBUG") != nullptr;   // host progress marks (stderr)
  p.skip_dq_red = std::getenv("MAMF_FA5B_SKIP_DQ_RED") != nullptr;  // timing experiments only: dq is wrong
  auto mark = [&](const char* what) {
    if (dbg) { fprintf(stderr, "[flash_tc_bwd] %s\n", what); fflush(stderr); }
  };
  mark("buffers and tensor maps ready");
  std::vector<at::Tensor> dqs;
  for (int s = 0; s < ns; ++s) dqs.push_back(at::empty_like(q1));
  if (p.S > 0 && p.B > 0) {
    const int64_t rows = (int64_t)ns * p.B * p.H * p.Spad;
    fa5_bwd_prep_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, stream()>>>(
        (const __nv_bfloat16*)dout.data_ptr(), (const __nv_bfloat16*)o1.data_ptr(),
        ns == 2 ? (const __nv_bfloat16*)o2c.data_ptr() : nullptr, lse1c.data_ptr<float>(),
        ns == 2 ? lse2c.data_ptr<float>() : nullptr, reinterpret_cast<float2*>(ld.data_ptr<float>()), ns, p.B, p.S,
        p.H, p.Spad);
    MAMF_LAUNCH_CHECK();
    mark("prep launched");
  }
  if (p.Skv > 0 && p.B > 0) {
    auto kfn = fa5_bwd_kernel;
    MAMF_CUDA_CHECK(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    mark("smem attribute set");
    dim3 grid((unsigned)p.G, (unsigned)p.B, (unsigned)((p.Skv + BK - 1) / BK));
    kfn<<<grid, NT, SMEM_BYTES, stream()>>>(mp, p);
    MAMF_LAUNCH_CHECK();
    mark("main kernel launched");
  }
  if (p.S > 0 && p.B > 0) {
    const int64_t n4 = (int64_t)p.B * p.S * p.H * (HD / 4);
    const unsigned blocks = (unsigned)std::min<int64_t>((n4 + 255) / 256, (int64_t)num_sms() * 16);
    for (int s = 0; s < ns; ++s) {
      fa5_bwd_dq_kernel<<<blocks, 256, 0, stream()>>>(acc.data_ptr<float>() + (int64_t)s * p.B * p.H * p.Spad * HD,
                                                      (__nv_bfloat16*)dqs[s].data_ptr(), p.B, p.S, p.H, p.Spad,
                                                      p.scale);
      MAMF_LAUNCH_CHECK();
    }
  }
  mark("dq conversion launched");
  std::vector<at::Tensor> out = dqs;
  out.push_back(dk);
  out.push_back(dv);
  return out;
}

int64_t flash_tc_bwd_error() {
  int v = 0;
  MAMF_CUDA_CHECK(cudaMemcpyFromSymbol(&v, fa5b::g_mamf_fa5b_err, sizeof(int)));
  if (v) {
    int z = 0;
    MAMF_CUDA_CHECK(cudaMemcpyToSymbol(fa5b::g_mamf_fa5b_err, &z, sizeof(int)));
  }
  return v;
}

}  // namespace mamf
