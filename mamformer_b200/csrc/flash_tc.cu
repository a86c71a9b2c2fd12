// Flash attention forward on the 5th-generation tensor cores (tcgen05 / TMEM / TMA), two query
// streams per CTA sharing one K/V stream:
//
//   differential mode (KDA-Diff full attention, DSA):  streams A = Q1[h], B = Q2[h]
//       out = (softmax(Q1 K^T s) V - lam[h] softmax(Q2 K^T s) V) / (1 - lam[h] + 1e-8)
//   pair mode (GQA):  streams A = Q[h0], B = Q[h0 + 1], two query heads of one KV head
//       out[h] = softmax(Q[h] K^T s) V
//
// Reference semantics: mamformer/layers/kda_diff.py:826-862 (two materialised S x S softmax
// maps, then the lambda combine), dsa.py:276-317, attention.py:157-181.  Masking is the band
// lo <= key - (query + Skv - S) <= hi of csrc/flash_attn.cu (causal: lo = -inf, hi = 0); a row
// without any key gives 0 and lse = +inf.  The per-stream row log-sum-exp (natural log) and the
// normalised per-stream outputs are kept for the backward (csrc/flash_attn.cu's kernels).
//
// One CTA = 128 query rows of one head (or head pair); 10 warps:
//   warps 0-3  softmax of stream A, warps 4-7 softmax of stream B (thread = query row: its S row
//              is read from TMEM with tcgen05.ld and its P row is written back as packed bf16
//              over the first 32 columns of the same S buffer with tcgen05.st);
//   warp 8     TMA producer (one lane): Q_A, Q_B once, then K / V tiles of 64 keys into a 5-deep
//              ring (no multicast; the maps cover this GPU's memory only);
//   warp 9     TMEM allocator + MMA issuer (one lane): S = Q K^T (M 128, N 64, K 128) into a
//              double-buffered S region per stream, O += P V (M 128, N 128, K 64) with P read
//              from TMEM (the A-in-tensor-memory form of tcgen05.mma) and V from shared memory.
// TMEM (512 columns): S_A[2] 0..127, S_B[2] 128..255, O_A 256..383, O_B 384..511 (fp32).
// The MMA thread issues O += P(j) V before S(j + 2) = Q K^T into the same buffer, and the tensor
// pipe runs one thread's MMAs in order, so P needs no buffer of its own and no proxy fence.
// Online softmax with lazy rescaling: a row's running max is raised (and its O rescaled in TMEM
// with tcgen05.ld / st) only when a new score exceeds it by more than 8 in log2 units, so P stays
// below 2^8 and most tiles need no rescale.
// Every wait is bounded (clock64); a timeout records a code in g_mamf_fa5_err, stops the CTA's
// work, waits a bounded time for its TMA copies, frees TMEM and returns.
#include "tc5.cuh"

namespace mamf {
namespace fa5 {

constexpr int BM = 128;            // query rows per stream
constexpr int BN = 64;             // keys per tile
constexpr int HD = 128;            // head dim
constexpr int ST = 5;              // K / V ring depth (four tiles of TMA prefetch)
constexpr int NT = 320;            // 10 warps
constexpr long long WAIT_CYCLES = 4000000000LL;   // ~2 s
constexpr float RESCALE_LOG2 = 8.f;

__device__ int g_mamf_fa5_err = 0;

// shared-memory layout (bytes, from a 1024-aligned base)
constexpr int Q_BYTES = BM * HD * 2;                     // 32 KB per stream (2 chunks of 64 dims)
constexpr int K_BYTES = BN * HD * 2;                     // 16 KB per tile
constexpr int OFF_QA = 0, OFF_QB = Q_BYTES;
constexpr int OFF_K = 2 * Q_BYTES;                       // [ST] K tiles
constexpr int OFF_V = OFF_K + ST * K_BYTES;              // [ST] V tiles
constexpr int OFF_BAR = OFF_V + ST * K_BYTES;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;         // barriers + alignment slack

struct Params {
  int B, S, Skv, H, G, off, lo, hi;
  float scale_log2;
  int pair;                    // 1: GQA head pairs, 0: differential (two query tensors)
  const float* lam;            // (H,) differential lambda (already clamped), null in pair mode
  __nv_bfloat16* out;          // (B, S, H, HD): combined (differential) or per-head (pair)
  __nv_bfloat16* oa;           // differential: normalised stream outputs (B, S, H, HD); null in pair mode
  __nv_bfloat16* ob;
  __nv_bfloat16* od;           // differential: o_a - o_b computed in fp32 (the d lambda term; the
                               // difference of the two bf16-rounded maps would lose it to cancellation)
  float* lse_a;                // (B, H, S) natural-log row log-sum-exp
  float* lse_b;
};

// ---- PTX helpers (csrc/tc5.cuh) -----------------------------------------------------------------
using namespace tc5;
// Bounded wait; false on timeout (code recorded) or when another role already failed.
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity, int code) {
  return tc5::bar_wait(b, parity, code, &g_mamf_fa5_err, WAIT_CYCLES);
}
// kind::f16 instruction descriptor: bf16 x bf16 -> f32, M = 128, N = n, A K-major
__host__ __device__ constexpr uint32_t idesc(int n, bool b_mn) { return idesc_bf16(BM, n, false, b_mn); }
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) { mma_ss(d, a, b, id, acc); }

// ---- the kernel ---------------------------------------------------------------------------------
struct Maps { CUtensorMap qa, qb, k, v; };

__global__ void __launch_bounds__(NT, 1) fa5_fwd_kernel(const __grid_constant__ Maps mp, Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;          // [ST]
  uint64_t* kv_empty = bars + 1 + ST;    // [ST]
  uint64_t* s_full = bars + 1 + 2 * ST;  // [stream][buf]
  uint64_t* p_full = s_full + 4;         // P of tile j in TMEM (128 arrivals)
  uint64_t* o_done = p_full + 4;
  uint64_t* ex_full = o_done + 4;        // stream B's normalised rows are in shared memory
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ex_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, q0 = blockIdx.x * BM;
  const int hpg = p.H / p.G;
  const int hA = p.pair ? 2 * blockIdx.y : blockIdx.y;
  const int hB = p.pair ? hA + 1 : hA;
  const int g = hA / hpg;
  const int qrows = min(BM, p.S - q0);
  const int kmin = max(0, q0 + p.off + p.lo);
  const int kmax = min(p.Skv - 1, q0 + qrows - 1 + p.off + p.hi);
  const int kt0 = kmax >= kmin ? kmin / BN : 0;
  const int ntile = kmax >= kmin ? kmax / BN - kt0 + 1 : 0;

  if (threadIdx.x == 0) {
    bar_init(q_full, 1);
    for (int s = 0; s < ST; ++s) { bar_init(&kv_full[s], 1); bar_init(&kv_empty[s], 1); }
    for (int i = 0; i < 4; ++i) {
      bar_init(&s_full[i], 1); bar_init(&p_full[i], 128); bar_init(&o_done[i], 1);
    }
    bar_init(ex_full, 128);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(su32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ------------------------------- TMA producer -------------------------------
    if (lane == 0 && ntile > 0) {
      bar_expect_tx(q_full, 2 * Q_BYTES);
      const CUtensorMap* mqb = p.pair ? &mp.qa : &mp.qb;
      for (int c = 0; c < 2; ++c) {
        tma_3d(sm + OFF_QA + c * (Q_BYTES / 2), &mp.qa, q_full, c * 64, hA, b * p.S + q0);
        tma_3d(sm + OFF_QB + c * (Q_BYTES / 2), mqb, q_full, c * 64, hB, b * p.S + q0);
      }
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int j = 0; j < ntile; ++j) {
        if (!bar_wait(&kv_empty[stage], phase ^ 1, 11)) break;
        bar_expect_tx(&kv_full[stage], 2 * K_BYTES);
        const int key0 = b * p.Skv + (kt0 + j) * BN;
        uint8_t* sK = sm + OFF_K + stage * K_BYTES;
        uint8_t* sV = sm + OFF_V + stage * K_BYTES;
        for (int c = 0; c < 2; ++c) {
          tma_3d(sK + c * (K_BYTES / 2), &mp.k, &kv_full[stage], c * 64, g, key0);
          tma_3d(sV + c * (K_BYTES / 2), &mp.v, &kv_full[stage], c * 64, g, key0);
        }
        ++issued;
        if (++stage == ST) { stage = 0; phase ^= 1; }
      }
      // on an error exit, wait (bounded) for the copies still in flight before the CTA can end
      if (*((volatile int*)&g_mamf_fa5_err) != 0) {
        bar_wait(q_full, 0, 0);
        for (int j = 0; j < issued; ++j) bar_wait(&kv_full[j % ST], (uint32_t)((j / ST) & 1), 0);
      }
    }
  } else if (warp == 9) {
    // ------------------------------- MMA issuer -------------------------------
    if (lane == 0 && ntile > 0) {
      bool ok = bar_wait(q_full, 0, 12);
      fence_after();
      constexpr uint32_t ID_QK = idesc(BN, false), ID_PV = idesc(HD, true);
      auto issue_qk = [&](int j) -> bool {
        const int st = j % ST, buf = j & 1;
        // S buffer `buf` last held P(j - 2), read by O += P V issued earlier by this thread
        if (!bar_wait(&kv_full[st], (uint32_t)((j / ST) & 1), 13)) return false;
        fence_after();
        const uint32_t kb = su32(sm + OFF_K + st * K_BYTES);
        for (int s = 0; s < 2; ++s) {
          const uint32_t qb = su32(sm + (s ? OFF_QB : OFF_QA));
          const uint32_t d = tmem + (uint32_t)(s * 128 + buf * 64);
#pragma unroll
          for (int k = 0; k < HD / 16; ++k) {
            const uint64_t a = sdesc(qb + (k >> 2) * (Q_BYTES / 2) + (k & 3) * 32, 16, 1024);
            const uint64_t bd = sdesc(kb + (k >> 2) * (K_BYTES / 2) + (k & 3) * 32, 16, 1024);
            mma(d, a, bd, ID_QK, k > 0 ? 1u : 0u);
          }
          commit(&s_full[s * 2 + buf]);
        }
        return true;
      };
      if (ok) ok = issue_qk(0);
      for (int j = 0; j < ntile && ok; ++j) {
        if (j + 1 < ntile && !issue_qk(j + 1)) { ok = false; break; }
        const int st = j % ST, buf = j & 1;
        const uint32_t vb = su32(sm + OFF_V + st * K_BYTES);
        for (int s = 0; s < 2 && ok; ++s) {
          if (!bar_wait(&p_full[s * 2 + buf], (uint32_t)((j >> 1) & 1), 15)) { ok = false; break; }
          fence_after();
          const uint32_t pa = tmem + (uint32_t)(s * 128 + buf * 64);     // P: 32 columns of bf16 pairs
          const uint32_t d = tmem + (uint32_t)(256 + s * 128);
#pragma unroll
          for (int k = 0; k < BN / 16; ++k) {
            const uint64_t bd = sdesc(vb + k * 2048, K_BYTES / 2, 1024);
            mma_ts(d, pa + (uint32_t)(k * 8), bd, ID_PV, (j > 0 || k > 0) ? 1u : 0u);
          }
          commit(&o_done[s * 2 + buf]);
        }
        if (ok) commit(&kv_empty[st]);
      }
    }
  } else {
    // ------------------------------- softmax (warps 0-3: A, 4-7: B) -------------------------------
    const int s = warp >> 2;
    const int r = (warp & 3) * 32 + lane;                 // query row in the tile = TMEM lane
    const int qi = q0 + r;
    const bool row_ok = qi < p.S;
    const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const int klo = qi + p.off + p.lo, khi = qi + p.off + p.hi;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < ntile && ok; ++j) {
      const int buf = j & 1;
      ok = __all_sync(0xffffffffu, bar_wait(&s_full[s * 2 + buf], (uint32_t)((j >> 1) & 1), 21));
      if (!ok) break;
      fence_after();
      float sv[BN];
      tld64(tl + (uint32_t)(s * 128 + buf * 64), sv);
      const int kbase = (kt0 + j) * BN;
      const bool full = row_ok && klo <= kbase && khi >= kbase + BN - 1 && kbase + BN - 1 < p.Skv;
      if (__any_sync(0xffffffffu, !full)) {           // band edge or sequence end: mask raw scores
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          const int key = kbase + c;
          sv[c] = (row_ok && key >= klo && key <= khi && key < p.Skv) ? sv[c] : -INFINITY;
        }
      }
      // row max of the raw scores with 8 independent chains (the scale is positive)
      float mq[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mq[i] = sv[i];
#pragma unroll
      for (int c = 8; c < BN; ++c) mq[c & 7] = fmaxf(mq[c & 7], sv[c]);
#pragma unroll
      for (int i = 0; i < 4; ++i) mq[i] = fmaxf(mq[i], mq[i + 4]);
      const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * p.scale_log2;
      const float m_new = fmaxf(m, mx);
      const bool need = m_new > m + RESCALE_LOG2;          // also true for the first key of a row
      if (__any_sync(0xffffffffu, need && m != -INFINITY)) {
        // O of this stream holds earlier tiles: wait for the last P V product, then rescale rows
        ok = __all_sync(0xffffffffu, bar_wait(&o_done[s * 2 + ((j - 1) & 1)], (uint32_t)(((j - 1) >> 1) & 1), 22));
        if (!ok) break;
        fence_after();
        const float f = (need && m != -INFINITY) ? ex2(m - m_new) : 1.f;
#pragma unroll 1
        for (int cc = 0; cc < HD; cc += 32) {
          float o[32];
          tld32(tl + (uint32_t)(256 + s * 128 + cc), o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= f;
          tst32(tl + (uint32_t)(256 + s * 128 + cc), o);
        }
      }
      if (need) {
        l = (m == -INFINITY) ? 0.f : l * ex2(m - m_new);
        m = m_new;
      }
      // p = 2^(s * scale_log2 - m); masked scores are -inf and give 0.  A row without any key so
      // far (m = -inf) has only masked scores, so subtracting 0 instead keeps it at 0.
      const float neg_m = (m == -INFINITY) ? 0.f : -m;
      float rq[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      float pk[BN / 2];                                   // P as bf16 pairs, bit patterns in fp32 slots
#pragma unroll
      for (int c2 = 0; c2 < BN / 2; ++c2) {
        const float e0 = ex2(fmaf(sv[2 * c2], p.scale_log2, neg_m));
        const float e1 = ex2(fmaf(sv[2 * c2 + 1], p.scale_log2, neg_m));
        rq[(2 * c2) & 7] += e0;
        rq[(2 * c2 + 1) & 7] += e1;
        __nv_bfloat162 h = __floats2bfloat162_rn(e0, e1);
        pk[c2] = __uint_as_float(*reinterpret_cast<uint32_t*>(&h));
      }
      l += ((rq[0] + rq[1]) + (rq[2] + rq[3])) + ((rq[4] + rq[5]) + (rq[6] + rq[7]));
      tst32(tl + (uint32_t)(s * 128 + buf * 64), pk);     // over this row's S(j), already in registers
      fence_before();
      bar_arrive(&p_full[s * 2 + buf]);
    }
    // ---- epilogue ----
    if (ok && ntile > 0)
      ok = __all_sync(0xffffffffu, bar_wait(&o_done[s * 2 + ((ntile - 1) & 1)], (uint32_t)(((ntile - 1) >> 1) & 1), 24));
    if (ok) {
      fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int h = s ? hB : hA;
      float* xrow = reinterpret_cast<float*>(sm) + r * (HD + 4);   // stream B's rows (Q / K area is free now)
      __nv_bfloat16* own = nullptr;
      if (p.pair) own = p.out;
      else own = s ? p.ob : p.oa;
      const int64_t orow = (((int64_t)b * p.S + qi) * p.H + h) * HD;
#pragma unroll 1
      for (int cc = 0; cc < HD; cc += 32) {
        float o[32];
        if (ntile > 0) tld32(tl + (uint32_t)(256 + s * 128 + cc), o);
        else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] *= inv;
        if (row_ok) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 v;
            __nv_bfloat162 h0 = __floats2bfloat162_rn(o[8 * q], o[8 * q + 1]), h1 = __floats2bfloat162_rn(o[8 * q + 2], o[8 * q + 3]);
            __nv_bfloat162 h2 = __floats2bfloat162_rn(o[8 * q + 4], o[8 * q + 5]), h3 = __floats2bfloat162_rn(o[8 * q + 6], o[8 * q + 7]);
            v.x = *reinterpret_cast<uint32_t*>(&h0); v.y = *reinterpret_cast<uint32_t*>(&h1);
            v.z = *reinterpret_cast<uint32_t*>(&h2); v.w = *reinterpret_cast<uint32_t*>(&h3);
            *reinterpret_cast<uint4*>(own + orow + cc + 8 * q) = v;
          }
        }
        if (!p.pair && s == 1) {
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(xrow + cc + 4 * q) = make_float4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
        }
        if (!p.pair && s == 0) {
          // keep stream A's normalised values in registers for the combine: stash in the O_A
          // columns (this thread's own TMEM row) so no extra registers are held across chunks
          tst32(tl + (uint32_t)(256 + cc), o);
        }
      }
      float* lse = s ? p.lse_b : p.lse_a;
      if (row_ok) lse[((int64_t)b * p.H + h) * p.S + qi] = l > 0.f ? (m + __log2f(l)) * 0.6931471805599453f : INFINITY;
      if (!p.pair) {
        if (s == 1) {
          fence_before();
          bar_arrive(ex_full);
        } else {
          ok = __all_sync(0xffffffffu, bar_wait(ex_full, 0, 25));
          if (ok) {
            const float lam = p.lam[hA];
            const float den = 1.f / (1.f - lam + 1e-8f);
            const float* brow = reinterpret_cast<const float*>(sm) + r * (HD + 4);
#pragma unroll 1
            for (int cc = 0; cc < HD; cc += 32) {
              float a[32];
              tld32(tl + (uint32_t)(256 + cc), a);
              if (row_ok) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  float c8[8], d8[8];
#pragma unroll
                  for (int i = 0; i < 8; ++i) {
                    const float bv = brow[cc + 8 * q + i];
                    c8[i] = (a[8 * q + i] - lam * bv) * den;
                    d8[i] = a[8 * q + i] - bv;
                  }
                  uint4 v, w;
                  __nv_bfloat162 h0 = __floats2bfloat162_rn(c8[0], c8[1]), h1 = __floats2bfloat162_rn(c8[2], c8[3]);
                  __nv_bfloat162 h2 = __floats2bfloat162_rn(c8[4], c8[5]), h3 = __floats2bfloat162_rn(c8[6], c8[7]);
                  v.x = *reinterpret_cast<uint32_t*>(&h0); v.y = *reinterpret_cast<uint32_t*>(&h1);
                  v.z = *reinterpret_cast<uint32_t*>(&h2); v.w = *reinterpret_cast<uint32_t*>(&h3);
                  *reinterpret_cast<uint4*>(p.out + orow + cc + 8 * q) = v;
                  h0 = __floats2bfloat162_rn(d8[0], d8[1]); h1 = __floats2bfloat162_rn(d8[2], d8[3]);
                  h2 = __floats2bfloat162_rn(d8[4], d8[5]); h3 = __floats2bfloat162_rn(d8[6], d8[7]);
                  w.x = *reinterpret_cast<uint32_t*>(&h0); w.y = *reinterpret_cast<uint32_t*>(&h1);
                  w.z = *reinterpret_cast<uint32_t*>(&h2); w.w = *reinterpret_cast<uint32_t*>(&h3);
                  *reinterpret_cast<uint4*>(p.od + orow + cc + 8 * q) = w;
                }
              }
            }
          }
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 9) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}

}  // namespace fa5

// ---- host side ------------------------------------------------------------------------------------
static CUtensorMap fa5_map(const at::Tensor& t, uint32_t rows) { return tc5_head_map(t, rows, "tcgen05 attention"); }

// Differential mode: q1, q2 (B, S, H, 128), k, v (B, Skv, G, 128), lam (H,) fp32.
//   returns (out, o1, o2, lse1, lse2, od): out = (o1 - lam o2) / (1 - lam + 1e-8), o1 / o2 the
//   normalised stream outputs, lse (B, H, S), od = o1 - o2 formed in fp32.
// Pair mode (q2 undefined): q (B, S, H, 128), H / G even; returns (out, lse).
std::vector<at::Tensor> flash_tc_fwd(at::Tensor q1, c10::optional<at::Tensor> q2, at::Tensor k, at::Tensor v,
                                     c10::optional<at::Tensor> lam, int64_t lo, int64_t hi, double scale) {
  using namespace fa5;
  c10::cuda::CUDAGuard guard(q1.device());
  const bool diff = q2.has_value();
  Params p{};
  p.B = q1.size(0); p.S = q1.size(1); p.H = q1.size(2); p.Skv = k.size(1); p.G = k.size(2);
  TORCH_CHECK(k.sizes() == v.sizes() && k.size(0) == p.B && p.H % p.G == 0, "tcgen05 attention: shapes");
  TORCH_CHECK(p.S <= p.Skv, "tcgen05 attention: S <= Skv");
  p.off = p.Skv - p.S;
  p.lo = (int)std::max<int64_t>(lo, -(1LL << 30));
  p.hi = (int)std::min<int64_t>(hi, (1LL << 30));
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  p.pair = diff ? 0 : 1;
  auto f32 = q1.options().dtype(at::kFloat);
  at::Tensor out = at::empty_like(q1), o1, o2, od;
  at::Tensor lse1 = at::empty({p.B, p.H, p.S}, f32), lse2;
  Maps mp{};
  mp.qa = fa5_map(q1, BM);
  mp.k = fa5_map(k.contiguous(), BN);
  mp.v = fa5_map(v.contiguous(), BN);
  if (diff) {
    TORCH_CHECK(q2->sizes() == q1.sizes() && lam.has_value() && lam->numel() == p.H &&
                lam->scalar_type() == at::kFloat, "tcgen05 attention: q2 like q1, lam (H,) fp32");
    mp.qb = fa5_map(*q2, BM);
    o1 = at::empty_like(q1);
    o2 = at::empty_like(q1);
    od = at::empty_like(q1);
    lse2 = at::empty({p.B, p.H, p.S}, f32);
    p.od = (__nv_bfloat16*)od.data_ptr();
    p.lam = lam->data_ptr<float>();
    p.oa = (__nv_bfloat16*)o1.data_ptr();
    p.ob = (__nv_bfloat16*)o2.data_ptr();
    p.lse_b = lse2.data_ptr<float>();
  } else {
    TORCH_CHECK((p.H / p.G) % 2 == 0, "tcgen05 attention (pair mode): an even number of query heads per KV head");
    mp.qb = mp.qa;
    p.lse_b = lse1.data_ptr<float>();
  }
  p.out = (__nv_bfloat16*)out.data_ptr();
  p.lse_a = lse1.data_ptr<float>();
  if (p.S > 0) {
    auto kfn = fa5_fwd_kernel;
    MAMF_CUDA_CHECK(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    dim3 grid((unsigned)((p.S + BM - 1) / BM), (unsigned)(diff ? p.H : p.H / 2), (unsigned)p.B);
    kfn<<<grid, NT, SMEM_BYTES, stream()>>>(mp, p);
    MAMF_LAUNCH_CHECK();
  }
  if (diff) return {out, o1, o2, lse1, lse2, od};
  return {out, lse1};
}

int64_t flash_tc_error() {
  int v = 0;
  MAMF_CUDA_CHECK(cudaMemcpyFromSymbol(&v, fa5::g_mamf_fa5_err, sizeof(int)));
  if (v) {
    int z = 0;
    MAMF_CUDA_CHECK(cudaMemcpyToSymbol(fa5::g_mamf_fa5_err, &z, sizeof(int)));
  }
  return v;
}

}  // namespace mamf
