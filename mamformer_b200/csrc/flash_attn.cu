// Fused softmax attention (GQA, causal / sliding-window bounds), forward and backward, for the
// full-attention paths: GQA attention (dense configs, MTP blocks) and the two softmax maps of
// KDA-Diff / DSA differential attention.
//
// Reference semantics (mamformer/layers/attention.py:157-181, kda_diff.py:826-886,
// kernels/flash_attention.py:66-270): out = softmax(Q K^T * scale + mask) V with the K/V head
// h / (H/G) for query head h.  The mask is a band on the key-minus-query distance:
// lo <= key - (query + Skv - S) <= hi (causal: lo = -inf, hi = 0; causal window W: lo = 1 - W;
// the reference's window quirks map to other bands).  Rows without any key produce 0.
//
// Tensor-core tiles use the warp-level mma.sync m16n8k16 bf16 instruction with fp32
// accumulation; operands are staged in shared memory with cp.async and read with ldmatrix
// (rows padded by 16 bytes, so the eight rows of each 8x8 matrix fall in different banks).
// Forward (one CTA = 64 query rows of one head, 4 warps x 16 rows): online softmax over 64-key
// blocks with the running max / sum in registers; K/V blocks double-buffered.  The row
// log-sum-exp is kept for the backward.
// Backward (one CTA = 64 keys of one KV head, looping over its query heads and the query blocks
// the band reaches): P recomputed from the saved log-sum-exp; dV += P^T dO, dP = dO V^T,
// dS = P (dP - D) with D = rowsum(dO * O); dK += dS^T Q in registers; dQ += dS K is summed
// over key blocks with fp32 reductions into a global accumulator.
#include "common.cuh"

namespace mamf {
namespace fa {

constexpr int BM = 64, BN = 64, NW = 4, NT = NW * 32;

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
__device__ __forceinline__ void cp16(void* dst, const void* src, bool ok) {
  const int n = ok ? 16 : 0;     // src-size 0 -> zero fill
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

struct Params {
  const __nv_bfloat16 *q, *k, *v, *o, *dout;
  __nv_bfloat16 *out, *dq, *dk, *dv;
  float *lse, *dpre, *dq_acc;
  int B, S, Skv, H, G, off;     // off = Skv - S (queries aligned to the last key positions)
  int lo, hi;                   // band on key - query position
  float scale_log2;             // scale * log2(e)
  float scale;
};

// rows x HD tile of a (B, len, heads, HD) tensor into smem [rows][HD + 8] (zero past `valid`)
template <int HD>
__device__ __forceinline__ void load_tile(__nv_bfloat16* dst, const __nv_bfloat16* src, int b, int r0, int valid,
                                          int len, int head, int heads) {
  constexpr int LD = HD + 8, CH = HD / 8;
  for (int i = threadIdx.x; i < 64 * CH; i += NT) {
    const int r = i / CH, c = (i % CH) * 8;
    const bool ok = r < valid;
    const __nv_bfloat16* g = src + (((int64_t)b * len + r0 + (ok ? r : 0)) * heads + head) * HD + c;
    cp16(dst + r * LD + c, g, ok);
  }
}

// ---- forward -----------------------------------------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(NT) fa_fwd_kernel(Params p) {
  constexpr int LD = HD + 8;
  extern __shared__ __align__(16) unsigned char smraw[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smraw);
  __nv_bfloat16* sK = sQ + BM * LD;        // [2][BN][LD]
  __nv_bfloat16* sV = sK + 2 * BN * LD;    // [2][BN][LD]
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int g = h / (p.H / p.G);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int q0 = qb * BM;
  const int qrows = min(BM, p.S - q0);
  // key range reached by this query block
  const int kmin = max(0, q0 + p.off + p.lo);
  const int kmax = min(p.Skv - 1, q0 + qrows - 1 + p.off + p.hi);
  const int kb0 = kmax >= kmin ? kmin / BN : 0, kb1 = kmax >= kmin ? kmax / BN : -1;

  load_tile<HD>(sQ, p.q, b, q0, qrows, p.S, h, p.H);
  if (kb0 <= kb1) {
    load_tile<HD>(sK, p.k, b, kb0 * BN, min(BN, p.Skv - kb0 * BN), p.Skv, g, p.G);
    load_tile<HD>(sV, p.v, b, kb0 * BN, min(BN, p.Skv - kb0 * BN), p.Skv, g, p.G);
  }
  cp_commit();

  float o[HD / 8][4];
#pragma unroll
  for (int n = 0; n < HD / 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[n][e] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const int gq = lane >> 2, tq = lane & 3;
  // query positions of this thread's two rows
  const int qi0 = q0 + w * 16 + gq, qi1 = qi0 + 8;
  uint32_t qf[HD / 16][4];

  for (int kb = kb0, it = 0; kb <= kb1; ++kb, ++it) {
    const int buf = it & 1;
    if (kb + 1 <= kb1) {
      const int nb = (kb + 1) * BN;
      load_tile<HD>(sK + (buf ^ 1) * BN * LD, p.k, b, nb, min(BN, p.Skv - nb), p.Skv, g, p.G);
      load_tile<HD>(sV + (buf ^ 1) * BN * LD, p.v, b, nb, min(BN, p.Skv - nb), p.Skv, g, p.G);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (it == 0) {
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        const int r = w * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(qf[kk], sQ + r * LD + c);
      }
    }
    const __nv_bfloat16* K = sK + buf * BN * LD;
    const __nv_bfloat16* V = sV + buf * BN * LD;
    // S = Q K^T  (16 rows x 64 keys per warp)
    float s[BN / 8][4];
#pragma unroll
    for (int n = 0; n < BN / 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
      for (int n = 0; n < BN / 8; n += 2) {
        uint32_t bf[4];
        const int key = n * 8 + (lane & 7) + (lane >> 4) * 8, c = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(bf, K + key * LD + c);
        mma16816(s[n], qf[kk], bf[0], bf[1]);
        mma16816(s[n + 1], qf[kk], bf[2], bf[3]);
      }
    }
    // mask, scale, online softmax (rows qi0 / qi1; each row spread over the 4 lanes of a quad)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < BN / 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kb * BN + n * 8 + 2 * tq + (e & 1);
        const int qi = (e < 2) ? qi0 : qi1;
        const int dist = key - (qi + p.off);
        const bool ok = key < p.Skv && qi < p.S && dist >= p.lo && dist <= p.hi;
        s[n][e] = ok ? s[n][e] * p.scale_log2 : -INFINITY;
        mx[e >> 1] = fmaxf(mx[e >> 1], s[n][e]);
      }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mnew = fmaxf(m_r[r], mx[r]);
      alpha[r] = (mnew == -INFINITY) ? 1.f : exp2f(m_r[r] - mnew);
      m_r[r] = mnew;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int n = 0; n < BN / 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mm = m_r[e >> 1];
        const float pv = (mm == -INFINITY) ? 0.f : exp2f(s[n][e] - mm);
        s[n][e] = pv;
        rs[e >> 1] += pv;
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_r[r] = l_r[r] * alpha[r] + rs[r];
    }
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) {
      o[n][0] *= alpha[0]; o[n][1] *= alpha[0];
      o[n][2] *= alpha[1]; o[n][3] *= alpha[1];
    }
    // O += P V
#pragma unroll
    for (int j = 0; j < BN / 16; ++j) {
      uint32_t pa[4] = {pack_bf16(s[2 * j][0], s[2 * j][1]), pack_bf16(s[2 * j][2], s[2 * j][3]),
                        pack_bf16(s[2 * j + 1][0], s[2 * j + 1][1]), pack_bf16(s[2 * j + 1][2], s[2 * j + 1][3])};
#pragma unroll
      for (int n = 0; n < HD / 8; n += 2) {
        uint32_t bf[4];
        const int key = j * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = n * 8 + (lane >> 4) * 8;
        ldsm_x4_t(bf, V + key * LD + c);
        mma16816(o[n], pa, bf[0], bf[1]);
        mma16816(o[n + 1], pa, bf[2], bf[3]);
      }
    }
    __syncthreads();
  }
  cp_wait<0>();
  // epilogue: normalise, store O and the row log-sum-exp (natural log)
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = r == 0 ? qi0 : qi1;
    if (qi >= p.S) continue;
    const float inv = l_r[r] > 0.f ? 1.f / l_r[r] : 0.f;
    __nv_bfloat16* dst = p.out + (((int64_t)b * p.S + qi) * p.H + h) * HD;
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) {
      const int c = n * 8 + 2 * tq;
      *reinterpret_cast<__nv_bfloat162*>(dst + c) = __floats2bfloat162_rn(o[n][2 * r] * inv, o[n][2 * r + 1] * inv);
    }
    if (tq == 0)
      p.lse[((int64_t)b * p.H + h) * p.S + qi] =
          l_r[r] > 0.f ? (m_r[r] + __log2f(l_r[r])) * 0.6931471805599453f : INFINITY;
  }
}

// ---- backward -------------------------------------------------------------------------------------
// D[b, h, q] = sum_d dO * O
template <int HD>
__global__ void fa_bwd_pre_kernel(Params p) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);   // (b, q, h)
  const int lane = threadIdx.x & 31;
  if (row >= (int64_t)p.B * p.S * p.H) return;
  const int h = row % p.H;
  const int64_t bq = row / p.H;
  const int q = bq % p.S, b = bq / p.S;
  float acc = 0.f;
  for (int c = lane; c < HD; c += 32)
    acc += __bfloat162float(p.dout[row * HD + c]) * __bfloat162float(p.o[row * HD + c]);
  acc = warp_sum(acc);
  if (lane == 0) p.dpre[((int64_t)b * p.H + h) * p.S + q] = acc;
}

template <int HD>
__global__ void __launch_bounds__(NT) fa_bwd_kernel(Params p) {
  constexpr int LD = HD + 8, LS = BM + 8;
  extern __shared__ __align__(16) unsigned char smraw[];
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(smraw);   // [BN][LD]
  __nv_bfloat16* sV = sK + BN * LD;
  __nv_bfloat16* sQ = sV + BN * LD;                              // [BM][LD]
  __nv_bfloat16* sdO = sQ + BM * LD;
  __nv_bfloat16* sdS = sdO + BM * LD;                            // [BN][LS]  (dS^T: key rows)
  float* sL = reinterpret_cast<float*>(sdS + BN * LS);           // [BM] lse * log2e
  float* sD = sL + BM;                                           // [BM]
  const int kb = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int groups = p.H / p.G;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const int k0 = kb * BN, krows = min(BN, p.Skv - k0);
  load_tile<HD>(sK, p.k, b, k0, krows, p.Skv, g, p.G);
  load_tile<HD>(sV, p.v, b, k0, krows, p.Skv, g, p.G);
  cp_commit();
  // queries reached by this key block: key - (q + off) in [lo, hi]  ->  q in [key - off - hi, key - off - lo]
  const int qmin = max(0, k0 - p.off - p.hi);
  const int qmax = min(p.S - 1, k0 + krows - 1 - p.off - p.lo);
  float dk[HD / 8][4], dv[HD / 8][4];
#pragma unroll
  for (int n = 0; n < HD / 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) { dk[n][e] = 0.f; dv[n][e] = 0.f; }
  const int key_r0 = k0 + w * 16 + gq, key_r1 = key_r0 + 8;   // this thread's two key rows

  for (int hh = 0; hh < groups && qmin <= qmax; ++hh) {
    const int h = g * groups + hh;
    for (int qb = qmin / BM; qb <= qmax / BM; ++qb) {
      const int q0 = qb * BM, qrows = min(BM, p.S - q0);
      __syncthreads();
      load_tile<HD>(sQ, p.q, b, q0, qrows, p.S, h, p.H);
      load_tile<HD>(sdO, p.dout, b, q0, qrows, p.S, h, p.H);
      cp_commit();
      for (int i = threadIdx.x; i < BM; i += NT) {
        const bool ok = i < qrows;
        sL[i] = ok ? p.lse[((int64_t)b * p.H + h) * p.S + q0 + i] * 1.4426950408889634f : INFINITY;
        sD[i] = ok ? p.dpre[((int64_t)b * p.H + h) * p.S + q0 + i] : 0.f;
      }
      cp_wait<0>();
      __syncthreads();
      // S^T (16 keys x 64 queries) = K_w Q^T ; dP^T = V_w dO^T
      float st[BM / 8][4], dpt[BM / 8][4];
#pragma unroll
      for (int n = 0; n < BM / 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) { st[n][e] = 0.f; dpt[n][e] = 0.f; }
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        uint32_t ka[4], va[4];
        const int r = w * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(ka, sK + r * LD + c);
        ldsm_x4(va, sV + r * LD + c);
#pragma unroll
        for (int n = 0; n < BM / 8; n += 2) {
          uint32_t qbf[4], obf[4];
          const int qr = n * 8 + (lane & 7) + (lane >> 4) * 8, qc = kk * 16 + ((lane >> 3) & 1) * 8;
          ldsm_x4(qbf, sQ + qr * LD + qc);
          ldsm_x4(obf, sdO + qr * LD + qc);
          mma16816(st[n], ka, qbf[0], qbf[1]);
          mma16816(st[n + 1], ka, qbf[2], qbf[3]);
          mma16816(dpt[n], va, obf[0], obf[1]);
          mma16816(dpt[n + 1], va, obf[2], obf[3]);
        }
      }
      // P^T and dS^T (scaled for the raw logits)
#pragma unroll
      for (int n = 0; n < BM / 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int ql = n * 8 + 2 * tq + (e & 1);
          const int qi = q0 + ql;
          const int key = (e < 2) ? key_r0 : key_r1;
          const int dist = key - (qi + p.off);
          const bool ok = qi < p.S && key < p.Skv && dist >= p.lo && dist <= p.hi;
          const float pv = ok ? exp2f(st[n][e] * p.scale_log2 - sL[ql]) : 0.f;
          st[n][e] = pv;
          dpt[n][e] = pv * (dpt[n][e] - sD[ql]) * p.scale;
        }
      // dV += P^T dO ; dK += dS^T Q ; stage dS^T for dQ
#pragma unroll
      for (int j = 0; j < BM / 16; ++j) {
        uint32_t pa[4] = {pack_bf16(st[2 * j][0], st[2 * j][1]), pack_bf16(st[2 * j][2], st[2 * j][3]),
                          pack_bf16(st[2 * j + 1][0], st[2 * j + 1][1]), pack_bf16(st[2 * j + 1][2], st[2 * j + 1][3])};
        uint32_t da[4] = {pack_bf16(dpt[2 * j][0], dpt[2 * j][1]), pack_bf16(dpt[2 * j][2], dpt[2 * j][3]),
                          pack_bf16(dpt[2 * j + 1][0], dpt[2 * j + 1][1]), pack_bf16(dpt[2 * j + 1][2], dpt[2 * j + 1][3])};
#pragma unroll
        for (int n = 0; n < HD / 8; n += 2) {
          uint32_t ob[4], qbt[4];
          const int qr = j * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = n * 8 + (lane >> 4) * 8;
          ldsm_x4_t(ob, sdO + qr * LD + c);
          ldsm_x4_t(qbt, sQ + qr * LD + c);
          mma16816(dv[n], pa, ob[0], ob[1]);
          mma16816(dv[n + 1], pa, ob[2], ob[3]);
          mma16816(dk[n], da, qbt[0], qbt[1]);
          mma16816(dk[n + 1], da, qbt[2], qbt[3]);
        }
        // dS^T rows (keys w*16 + gq, +8), columns (queries j*16 + 2tq .. , +8)
        __nv_bfloat16* d0 = sdS + (w * 16 + gq) * LS + j * 16 + 2 * tq;
        __nv_bfloat16* d1 = d0 + 8 * LS;
        *reinterpret_cast<uint32_t*>(d0) = da[0];
        *reinterpret_cast<uint32_t*>(d1) = da[1];
        *reinterpret_cast<uint32_t*>(d0 + 8) = da[2];
        *reinterpret_cast<uint32_t*>(d1 + 8) = da[3];
      }
      __syncthreads();
      // dQ (warp: queries w*16.., all HD) += dS K  with dS = (dS^T)^T from smem
      {
        float dq[HD / 8][4];
#pragma unroll
        for (int n = 0; n < HD / 8; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) dq[n][e] = 0.f;
#pragma unroll
        for (int ks = 0; ks < BN / 16; ++ks) {
          uint32_t sa[4];
          const int key = ks * 16 + (lane & 7) + (lane >> 4) * 8, qc = w * 16 + ((lane >> 3) & 1) * 8;
          ldsm_x4_t(sa, sdS + key * LS + qc);
#pragma unroll
          for (int n = 0; n < HD / 8; n += 2) {
            uint32_t kbf[4];
            const int kr = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, c = n * 8 + (lane >> 4) * 8;
            ldsm_x4_t(kbf, sK + kr * LD + c);
            mma16816(dq[n], sa, kbf[0], kbf[1]);
            mma16816(dq[n + 1], sa, kbf[2], kbf[3]);
          }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int qi = q0 + w * 16 + gq + 8 * r;
          if (qi >= p.S) continue;
          float* dst = p.dq_acc + (((int64_t)b * p.S + qi) * p.H + h) * HD;
#pragma unroll
          for (int n = 0; n < HD / 8; ++n) {
            atomicAdd(dst + n * 8 + 2 * tq, dq[n][2 * r]);
            atomicAdd(dst + n * 8 + 2 * tq + 1, dq[n][2 * r + 1]);
          }
        }
      }
    }
  }
  cp_wait<0>();
  // dK, dV rows of this warp
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int key = (r == 0) ? key_r0 : key_r1;
    if (key >= p.Skv) continue;
    const int64_t base = (((int64_t)b * p.Skv + key) * p.G + g) * HD;
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) {
      const int c = n * 8 + 2 * tq;
      *reinterpret_cast<__nv_bfloat162*>(p.dk + base + c) = __floats2bfloat162_rn(dk[n][2 * r], dk[n][2 * r + 1]);
      *reinterpret_cast<__nv_bfloat162*>(p.dv + base + c) = __floats2bfloat162_rn(dv[n][2 * r], dv[n][2 * r + 1]);
    }
  }
}

template <int HD>
constexpr int fwd_smem() { return (BM + 4 * BN) * (HD + 8) * 2; }
template <int HD>
constexpr int bwd_smem() { return (2 * BN + 2 * BM) * (HD + 8) * 2 + BN * (BM + 8) * 2 + 2 * BM * 4; }

}  // namespace fa

static fa::Params fa_params(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, int64_t lo, int64_t hi,
                            double scale) {
  for (const at::Tensor* t : {&q, &k, &v})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->is_contiguous() && t->dim() == 4,
                "flash attention: contiguous bf16 (B, S, heads, head_dim) tensors");
  TORCH_CHECK(k.sizes() == v.sizes() && q.size(0) == k.size(0) && q.size(3) == k.size(3) && q.size(2) % k.size(2) == 0 &&
              q.size(1) <= k.size(1), "flash attention: shapes");
  fa::Params p{};
  p.q = (const __nv_bfloat16*)q.data_ptr();
  p.k = (const __nv_bfloat16*)k.data_ptr();
  p.v = (const __nv_bfloat16*)v.data_ptr();
  p.B = q.size(0); p.S = q.size(1); p.Skv = k.size(1); p.H = q.size(2); p.G = k.size(2);
  p.off = p.Skv - p.S;
  p.lo = (int)std::max<int64_t>(lo, -(int64_t)(1 << 30));
  p.hi = (int)std::min<int64_t>(hi, (int64_t)(1 << 30));
  p.scale = (float)scale;
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  return p;
}

template <typename F>
static void fa_dispatch(int hd, F&& f) {
  if (hd == 128) f(std::integral_constant<int, 128>{});
  else if (hd == 64) f(std::integral_constant<int, 64>{});
  else TORCH_CHECK(false, "flash attention: head_dim must be 64 or 128");
}

// returns (out, lse (B, H, S) fp32)
std::vector<at::Tensor> flash_attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, int64_t lo, int64_t hi, double scale) {
  c10::cuda::CUDAGuard guard(q.device());
  fa::Params p = fa_params(q, k, v, lo, hi, scale);
  auto out = at::empty_like(q);
  auto lse = at::empty({p.B, p.H, p.S}, q.options().dtype(at::kFloat));
  p.out = (__nv_bfloat16*)out.data_ptr();
  p.lse = lse.data_ptr<float>();
  fa_dispatch(q.size(3), [&](auto hc) {
    constexpr int HD = decltype(hc)::value;
    constexpr int sm = fa::fwd_smem<HD>();
    MAMF_CUDA_CHECK(cudaFuncSetAttribute(fa::fa_fwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
    dim3 grid((p.S + fa::BM - 1) / fa::BM, p.H, p.B);
    fa::fa_fwd_kernel<HD><<<grid, fa::NT, sm, stream()>>>(p);
    MAMF_LAUNCH_CHECK();
  });
  return {out, lse};
}

// returns (dq, dk, dv)
std::vector<at::Tensor> flash_attn_bwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out, at::Tensor lse,
                                       at::Tensor dout, int64_t lo, int64_t hi, double scale) {
  c10::cuda::CUDAGuard guard(q.device());
  fa::Params p = fa_params(q, k, v, lo, hi, scale);
  TORCH_CHECK(dout.sizes() == q.sizes() && dout.is_contiguous() && dout.scalar_type() == at::kBFloat16 &&
              out.is_contiguous(), "flash attention backward: dout / out like q");
  auto f32 = q.options().dtype(at::kFloat);
  auto dq_acc = at::zeros(q.sizes(), f32);
  auto dpre = at::empty({p.B, p.H, p.S}, f32);
  auto dk = at::empty_like(k), dv = at::empty_like(v);
  p.o = (const __nv_bfloat16*)out.data_ptr();
  p.dout = (const __nv_bfloat16*)dout.data_ptr();
  p.lse = lse.data_ptr<float>();
  p.dpre = dpre.data_ptr<float>();
  p.dq_acc = dq_acc.data_ptr<float>();
  p.dk = (__nv_bfloat16*)dk.data_ptr();
  p.dv = (__nv_bfloat16*)dv.data_ptr();
  fa_dispatch(q.size(3), [&](auto hc) {
    constexpr int HD = decltype(hc)::value;
    const int64_t rows = (int64_t)p.B * p.S * p.H;
    fa::fa_bwd_pre_kernel<HD><<<(unsigned)((rows + 7) / 8), 256, 0, stream()>>>(p);
    MAMF_LAUNCH_CHECK();
    constexpr int sm = fa::bwd_smem<HD>();
    MAMF_CUDA_CHECK(cudaFuncSetAttribute(fa::fa_bwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
    dim3 grid((p.Skv + fa::BN - 1) / fa::BN, p.G, p.B);
    fa::fa_bwd_kernel<HD><<<grid, fa::NT, sm, stream()>>>(p);
    MAMF_LAUNCH_CHECK();
  });
  return {dq_acc.to(at::kBFloat16), dk, dv};
}

}  // namespace mamf
