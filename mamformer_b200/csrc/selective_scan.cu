// Diagonal selective scan (the reference's Mamba2Block recurrence), forward and backward.
//
//   h[t,c,n] = exp(-A[n] dt[t,c]) h[t-1,c,n] + B[t,n] dt[t,c] x[t,c]
//   y[t,c]   = (sum_n C[t,n] h[t,c,n] + D[c] x[t,c]) * silu(z[t,c])        (GATE)
//   hs[t,n]  = mean_c h[t,c,n]                                             (HS)
// with A = exp(clamp(A_log, -5, 5)) and dt = softplus(dt_raw) (SOFTPLUS).
// Reference semantics: mamformer/layers/mamba2.py:70-130 (scan), 249-368 (block).
//
// Work split (sm_100a, 148 SMs): one CTA per (batch, 32-channel block); warp w owns states
// [16w, 16w+16) of all 32 channels (N/16 warps per CTA); lane = channel.  Each thread keeps
// its 16 states in registers as 8 fp32x2 pairs, so the time recurrence is 16 independent chains
// per thread issued as packed FFMA2/FMUL2 instructions, and the decay exp2 runs on the MUFU pipe.  Inputs of a 32-step chunk are staged in shared
// memory (B/C rows are broadcast reads); the forward loads the next chunk into registers while
// the current chunk's recurrence runs.  Reductions over channels (h_states, dB, dC) use an
// in-warp reduce-scatter after which lanes 2s, 2s+1 hold the 32-channel sum for state 16w+s;
// the per-block partial rows are written to [batch, channel-block, S, N] and summed by the
// caller.  Forward per-warp partial outputs go to separate shared rows (no atomics).
//
// Backward: the forward stores the state at every 32-step chunk start (fp32).  The backward
// walks chunks in reverse: phase A recomputes the chunk forward (saving 4-step
// sub-checkpoints to a per-CTA global scratch area and producing y, dz, dC); phase B walks
// the 4-step sub-chunks in reverse: B1 runs the adjoint recurrence
// G[t] = a[t+1] G[t+1] + C[t] dy'[t] + dhs[t]/Di (fp32 carry in registers, G copied to shared
// memory as bf16), B2 recomputes h from the sub-checkpoint and forms the decay gradients
// sum_n G a h[t-1] A[n] (-> ddt) and sum G a h[t-1] dt (-> dA).
#include "common.cuh"

namespace mamf {
namespace scan {

constexpr int CK = 32;      // checkpoint / staging chunk (time steps)
constexpr int SUB = 4;      // backward sub-chunk (time steps between sub-checkpoints)
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr int SW = 16;      // states per warp (lane = channel, 32 channels per CTA)

// ---- packed fp32x2 state arithmetic --------------------------------------------------------------
// sm_100 issues two fp32 FMAs / multiplies / adds per instruction (FFMA2 & co.), which halves the
// instruction count of the per-state recurrence.  A thread's 16 states are 8 float2 pairs.
//
// Register permutation.  Register k of lane l holds state k ^ (qx(l) << 2), qx(l) = (l >> 3) & 3:
// every group of 4 states (one float4 of a B / C row) is loaded from float4 index q ^ qx.  With
// this layout the first two rounds of the channel reduce-scatter (partners l ^ 16, l ^ 8) need no
// lane-dependent selects: every lane keeps registers [0, 8) (then [0, 4)) and adds the partner's
// registers [8, 16) (then [4, 8)), which hold the same states in the partner's permutation.
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 ex2x2(float2 x) { return make_float2(ex2(x.x), ex2(x.y)); }
__device__ __forceinline__ int perm_q(int lane) { return (lane >> 3) & 3; }
__device__ __forceinline__ int state_of(int k, int lane) { return k ^ (perm_q(lane) << 2); }

// 16 consecutive shared-memory floats (16-byte aligned) in the lane's register permutation
__device__ __forceinline__ void ld_row16p(float2 (&r)[8], const float* src, int qx) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 v = s4[q ^ qx];
    r[2 * q] = make_float2(v.x, v.y);
    r[2 * q + 1] = make_float2(v.z, v.w);
  }
}
// the same for 16 fp32 values in global memory (checkpoint rows)
__device__ __forceinline__ void ld_state16p(float2 (&r)[8], const float* src, int qx) { ld_row16p(r, src, qx); }
__device__ __forceinline__ void st_state16p(float* dst, const float2 (&r)[8], int qx) {
  float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) d4[q ^ qx] = make_float4(r[2 * q].x, r[2 * q].y, r[2 * q + 1].x, r[2 * q + 1].y);
}

// Sum over the 32 lanes (channels) of the 16 permuted state values; afterwards lanes 2s and 2s+1
// hold the sum for state s (s = lane >> 1).  v is destroyed.
__device__ __forceinline__ float reduce_scatter16p(float2 (&v)[8], int lane) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
    v[i] = add2(v[i], make_float2(__shfl_xor_sync(0xffffffffu, v[i + 4].x, 16), __shfl_xor_sync(0xffffffffu, v[i + 4].y, 16)));
#pragma unroll
  for (int i = 0; i < 2; ++i)
    v[i] = add2(v[i], make_float2(__shfl_xor_sync(0xffffffffu, v[i + 2].x, 8), __shfl_xor_sync(0xffffffffu, v[i + 2].y, 8)));
  {
    const bool up = lane & 4;
    const float2 send = up ? v[0] : v[1], keep = up ? v[1] : v[0];
    v[0] = add2(keep, make_float2(__shfl_xor_sync(0xffffffffu, send.x, 4), __shfl_xor_sync(0xffffffffu, send.y, 4)));
  }
  const bool up = lane & 2;
  const float send = up ? v[0].x : v[0].y, keep = up ? v[0].y : v[0].x;
  const float r = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  return r + __shfl_xor_sync(0xffffffffu, r, 1);
}

struct Params {
  int Bsz, S, Di, N, G, nck;
  // inputs: [b, t, c] / [b, t, n] with unit inner stride
  const void* x;  int64_t x_bs, x_ts;
  const void* dt; int64_t dt_bs, dt_ts;
  const void* Bm; int64_t B_bs, B_ts;
  const void* Cm; int64_t C_bs, C_ts;
  const void* z;  int64_t z_bs, z_ts;
  const float* A_log;
  const float* D;
  const float* h0;          // [Bsz, Di, N] or null
  // forward outputs
  void* y; int64_t y_bs, y_ts;
  float* hs_part;           // [Bsz, G, S, N]
  float* ckpt;              // [Bsz, nck, Di, N]
  float* final_state;       // [Bsz, Di, N] or null
  // backward
  const void* dy; int64_t dy_bs, dy_ts;
  const float* dhs;         // [Bsz, S, N] or null
  void* dx; void* ddt; void* dz;   // contiguous [b, t, c]
  float* dB_part; float* dC_part;  // [Bsz, G, S, N]
  float* dA;                // [N]   (d loss / d A[n])
  float* dD;                // [Di]
  float* scratch;           // per CTA: [CK/SUB][SW][NT]
};

template <typename T>
__device__ __forceinline__ float ldf(const void* base, int64_t off) {
  return to_f<T>(reinterpret_cast<const T*>(base)[off]);
}

// ---------------------------------------------------------------------------------------------
// Per-thread register staging of the next chunk's inputs (issued before the current chunk's
// time loop, so the global-load latency overlaps the recurrence).
template <typename T, int NT, int N>
struct Stage {
  static constexpr int NBC = (CK * N + NT - 1) / NT;     // B / C elements per thread
  static constexpr int NXD = (CK * 32 + NT - 1) / NT;    // dt / x elements per thread
  float b[NBC], c[NBC], d[NXD], x[NXD];

  __device__ __forceinline__ void load(const Params& p, int b_, int cblk, int t0, int L) {
#pragma unroll
    for (int k = 0; k < NBC; ++k) {
      const int i = threadIdx.x + k * NT;
      const int tt = i / N, n = i - tt * N;
      const bool ok = i < CK * N && tt < L;
      b[k] = ok ? ldf<T>(p.Bm, (int64_t)b_ * p.B_bs + (int64_t)(t0 + tt) * p.B_ts + n) : 0.f;
      c[k] = ok ? ldf<T>(p.Cm, (int64_t)b_ * p.C_bs + (int64_t)(t0 + tt) * p.C_ts + n) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < NXD; ++k) {
      const int i = threadIdx.x + k * NT;
      const int tt = i >> 5, cc = cblk * 32 + (i & 31);
      const bool ok = i < CK * 32 && tt < L && cc < p.Di;
      d[k] = ok ? ldf<T>(p.dt, (int64_t)b_ * p.dt_bs + (int64_t)(t0 + tt) * p.dt_ts + cc) : 0.f;
      x[k] = ok ? ldf<T>(p.x, (int64_t)b_ * p.x_bs + (int64_t)(t0 + tt) * p.x_ts + cc) : 0.f;
    }
  }
  template <bool SOFTPLUS>
  __device__ __forceinline__ void store(float* sB, float* sC, float* sDt, float* sDtx) const {
#pragma unroll
    for (int k = 0; k < NBC; ++k) {
      const int i = threadIdx.x + k * NT;
      if (i < CK * N) { sB[i] = b[k]; sC[i] = c[k]; }
    }
#pragma unroll
    for (int k = 0; k < NXD; ++k) {
      const int i = threadIdx.x + k * NT;
      if (i < CK * 32) {
        const float dd = SOFTPLUS ? softplus_f(d[k]) : d[k];
        sDt[i] = dd;
        sDtx[i] = dd * x[k];
      }
    }
  }
};

template <typename T, int NW, bool SOFTPLUS, bool GATE, bool HS, int UNR>
__global__ void __launch_bounds__(NW * 32, 2) scan_fwd_kernel(Params p) {
  constexpr int NT = NW * 32;
  constexpr int N = NW * SW;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int b = blockIdx.y, cblk = blockIdx.x;
  const int c = cblk * 32 + lane;
  const bool cvalid = c < p.Di;

  extern __shared__ float smem[];
  float* sB = smem;                 // [CK][N]
  float* sC = sB + CK * N;          // [CK][N]
  float* sDt = sC + CK * N;         // [CK][32]
  float* sDtx = sDt + CK * 32;      // [CK][32]
  float* sYw = sDtx + CK * 32;      // [NW][CK][32] per-warp partial outputs

  const int qx = perm_q(lane);
  float2 A2[SW / 2];
#pragma unroll
  for (int j = 0; j < SW; ++j) {
    const float al = fminf(fmaxf(p.A_log[w * SW + state_of(j, lane)], -5.f), 5.f);
    const float v = -__expf(al) * LOG2E;
    if (j & 1) A2[j >> 1].y = v; else A2[j >> 1].x = v;
  }
  float2 h[SW / 2];
  if (p.h0 && cvalid) ld_state16p(h, p.h0 + ((int64_t)b * p.Di + c) * N + w * SW, qx);
  else {
#pragma unroll
    for (int j = 0; j < SW / 2; ++j) h[j] = f2(0.f);
  }

  Stage<T, NT, N> st;
  st.load(p, b, cblk, 0, min(CK, p.S));
  for (int t0 = 0, ck = 0; t0 < p.S; t0 += CK, ++ck) {
    const int L = min(CK, p.S - t0);
    if (p.ckpt && cvalid) st_state16p(p.ckpt + (((int64_t)b * p.nck + ck) * p.Di + c) * N + w * SW, h, qx);
    __syncthreads();
    st.template store<SOFTPLUS>(sB, sC, sDt, sDtx);
    __syncthreads();
    if (t0 + CK < p.S) st.load(p, b, cblk, t0 + CK, min(CK, p.S - t0 - CK));   // next chunk in flight
    float* yw = sYw + w * CK * 32;
#pragma unroll UNR
    for (int tt = 0; tt < L; ++tt) {
      const float2 dd = f2(sDt[tt * 32 + lane]), dx2 = f2(sDtx[tt * 32 + lane]);
      float2 Bt[SW / 2], Ct[SW / 2];
      ld_row16p(Bt, sB + tt * N + w * SW, qx);
      ld_row16p(Ct, sC + tt * N + w * SW, qx);
      float2 yq[2] = {f2(0.f), f2(0.f)};        // 4 independent partial sums (short FMA chains)
#pragma unroll
      for (int j = 0; j < SW / 2; ++j) {
        const float2 a = ex2x2(mul2(A2[j], dd));
        h[j] = fma2(a, h[j], mul2(Bt[j], dx2));
        yq[j & 1] = fma2(Ct[j], h[j], yq[j & 1]);
      }
      yw[tt * 32 + lane] = (yq[0].x + yq[0].y) + (yq[1].x + yq[1].y);
      if (HS) {
        float2 tmp[SW / 2];
#pragma unroll
        for (int j = 0; j < SW / 2; ++j) tmp[j] = h[j];
        const float r = reduce_scatter16p(tmp, lane);
        if ((lane & 1) == 0)
          p.hs_part[(((int64_t)b * p.G + cblk) * p.S + t0 + tt) * N + w * SW + (lane >> 1)] = r;
      }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < L * 32; i += NT) {
      const int tt = i >> 5, cc = cblk * 32 + (i & 31);
      if (cc >= p.Di) continue;
      float yv = 0.f;
#pragma unroll
      for (int ww = 0; ww < NW; ++ww) yv += sYw[ww * CK * 32 + i];
      const float xv = ldf<T>(p.x, (int64_t)b * p.x_bs + (int64_t)(t0 + tt) * p.x_ts + cc);
      yv += p.D[cc] * xv;
      if (GATE) yv *= silu_f(ldf<T>(p.z, (int64_t)b * p.z_bs + (int64_t)(t0 + tt) * p.z_ts + cc));
      reinterpret_cast<T*>(p.y)[(int64_t)b * p.y_bs + (int64_t)(t0 + tt) * p.y_ts + cc] = from_f<T>(yv);
    }
  }
  if (p.final_state && cvalid) st_state16p(p.final_state + ((int64_t)b * p.Di + c) * N + w * SW, h, qx);
}

// ---------------------------------------------------------------------------------------------
template <typename T, int NW, bool SOFTPLUS, bool GATE, bool HS, int UNR>
__global__ void __launch_bounds__(NW * 32, 2) scan_bwd_kernel(Params p) {
  constexpr int NT = NW * 32;
  constexpr int N = NW * SW;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int b = blockIdx.y, cblk = blockIdx.x;
  const int c = cblk * 32 + lane;
  const bool cvalid = c < p.Di;
  const float inv_di = 1.f / (float)p.Di;

  extern __shared__ float smem[];
  float* sB = smem;                       // [CK][N]
  float* sC = sB + CK * N;                // [CK][N]
  float* sDhs = sC + CK * N;              // [CK][N]  (HS)
  float* sDt = sDhs + (HS ? CK * N : 0);  // [CK][32]
  float* sDtx = sDt + CK * 32;
  float* sX = sDtx + CK * 32;
  float* sDyp = sX + CK * 32;
  float* sY = sDyp + CK * 32;
  float* sDU = sY + CK * 32;
  float* sDD = sDU + CK * 32;
  float* sA2 = sDD + CK * 32;             // [N]
  float* sDsum = sA2 + N;                 // [32]
  __nv_bfloat16* sG = reinterpret_cast<__nv_bfloat16*>(sDsum + 32);   // [SUB][SW][NT]

  for (int i = tid; i < N; i += NT) {
    float al = fminf(fmaxf(p.A_log[i], -5.f), 5.f);
    sA2[i] = -__expf(al) * LOG2E;
  }
  if (tid < 32) sDsum[tid] = 0.f;
  float* scratch = p.scratch + ((int64_t)blockIdx.y * gridDim.x + blockIdx.x) * (CK / SUB) * SW * NT;

  const int qx = perm_q(lane);
  float2 P[SW / 2], dAacc[SW / 2], A2[SW / 2];
#pragma unroll
  for (int j = 0; j < SW / 2; ++j) { P[j] = f2(0.f); dAacc[j] = f2(0.f); }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < SW; ++j) {
    const float v = sA2[w * SW + state_of(j, lane)];
    if (j & 1) A2[j >> 1].y = v; else A2[j >> 1].x = v;
  }

  for (int ck = p.nck - 1; ck >= 0; --ck) {
    const int t0 = ck * CK;
    const int L = min(CK, p.S - t0);
    __syncthreads();
    for (int i = tid; i < L * N; i += NT) {
      const int tt = i / N, n = i - tt * N;
      sB[i] = ldf<T>(p.Bm, (int64_t)b * p.B_bs + (int64_t)(t0 + tt) * p.B_ts + n);
      sC[i] = ldf<T>(p.Cm, (int64_t)b * p.C_bs + (int64_t)(t0 + tt) * p.C_ts + n);
      if (HS) sDhs[i] = p.dhs[((int64_t)b * p.S + t0 + tt) * N + n] * inv_di;
    }
    for (int i = tid; i < L * 32; i += NT) {
      const int tt = i >> 5, cc = cblk * 32 + (i & 31);
      float d = 0.f, xv = 0.f, dyp = 0.f;
      if (cc < p.Di) {
        d = ldf<T>(p.dt, (int64_t)b * p.dt_bs + (int64_t)(t0 + tt) * p.dt_ts + cc);
        if (SOFTPLUS) d = softplus_f(d);
        xv = ldf<T>(p.x, (int64_t)b * p.x_bs + (int64_t)(t0 + tt) * p.x_ts + cc);
        dyp = ldf<T>(p.dy, (int64_t)b * p.dy_bs + (int64_t)(t0 + tt) * p.dy_ts + cc);
        if (GATE) dyp *= silu_f(ldf<T>(p.z, (int64_t)b * p.z_bs + (int64_t)(t0 + tt) * p.z_ts + cc));
      }
      sDt[i] = d; sDtx[i] = d * xv; sX[i] = xv; sDyp[i] = dyp;
      sY[i] = 0.f; sDU[i] = 0.f; sDD[i] = 0.f;
    }
    __syncthreads();

    // ---- phase A: recompute the chunk forward --------------------------------------------
    {
      float2 h[SW / 2];
      if (cvalid) ld_state16p(h, p.ckpt + (((int64_t)b * p.nck + ck) * p.Di + c) * N + w * SW, qx);
      else {
#pragma unroll
        for (int j = 0; j < SW / 2; ++j) h[j] = f2(0.f);
      }
#pragma unroll UNR
      for (int tt = 0; tt < L; ++tt) {
        if ((tt % SUB) == 0) {
          float2* dst = reinterpret_cast<float2*>(scratch + (int64_t)(tt / SUB) * SW * NT);
#pragma unroll
          for (int j = 0; j < SW / 2; ++j) dst[j * NT + tid] = h[j];
        }
        const float2 dd = f2(sDt[tt * 32 + lane]), dx2 = f2(sDtx[tt * 32 + lane]), dy2 = f2(sDyp[tt * 32 + lane]);
        float2 Bt[SW / 2], Ct[SW / 2];
        ld_row16p(Bt, sB + tt * N + w * SW, qx);
        ld_row16p(Ct, sC + tt * N + w * SW, qx);
        float2 yq[2] = {f2(0.f), f2(0.f)};
        float2 tmp[SW / 2];
#pragma unroll
        for (int j = 0; j < SW / 2; ++j) {
          const float2 a = ex2x2(mul2(A2[j], dd));
          h[j] = fma2(a, h[j], mul2(Bt[j], dx2));
          yq[j & 1] = fma2(Ct[j], h[j], yq[j & 1]);
          tmp[j] = mul2(h[j], dy2);
        }
        atomicAdd(&sY[tt * 32 + lane], (yq[0].x + yq[0].y) + (yq[1].x + yq[1].y));
        const float r = reduce_scatter16p(tmp, lane);
        if ((lane & 1) == 0)
          p.dC_part[(((int64_t)b * p.G + cblk) * p.S + t0 + tt) * N + w * SW + (lane >> 1)] = r;
      }
    }
    __syncthreads();
    // epilogue A: dz and dD
    for (int i = tid; i < L * 32; i += NT) {
      const int tt = i >> 5, cl = i & 31, cc = cblk * 32 + cl;
      if (cc >= p.Di) continue;
      const float xv = sX[i];
      atomicAdd(&sDsum[cl], sDyp[i] * xv);
      if (GATE) {
        const int64_t off = (int64_t)b * p.z_bs + (int64_t)(t0 + tt) * p.z_ts + cc;
        const float zv = ldf<T>(p.z, off);
        const float sg = sigmoid_f(zv);
        const float yfull = sY[i] + p.D[cc] * xv;
        const float dyg = ldf<T>(p.dy, (int64_t)b * p.dy_bs + (int64_t)(t0 + tt) * p.dy_ts + cc);
        const float dz = dyg * yfull * (sg * (1.f + zv * (1.f - sg)));
        reinterpret_cast<T*>(p.dz)[((int64_t)b * p.S + t0 + tt) * p.Di + cc] = from_f<T>(dz);
      }
    }

    // ---- phase B: adjoint over sub-chunks in reverse ---------------------------------------
    const int nsub = (L + SUB - 1) / SUB;
    for (int sub = nsub - 1; sub >= 0; --sub) {
      const int s0 = sub * SUB, s1 = min(s0 + SUB, L);
      // B1: G recurrence (reverse)
      for (int tt = s1 - 1; tt >= s0; --tt) {
        const float2 dd = f2(sDt[tt * 32 + lane]), dx2 = f2(sDtx[tt * 32 + lane]), dy2 = f2(sDyp[tt * 32 + lane]);
        float2 Bt[SW / 2], Ct[SW / 2], Ht[SW / 2];
        ld_row16p(Bt, sB + tt * N + w * SW, qx);
        ld_row16p(Ct, sC + tt * N + w * SW, qx);
        if (HS) ld_row16p(Ht, sDhs + tt * N + w * SW, qx);
        float2 duq[2] = {f2(0.f), f2(0.f)};
        float2 gb[SW / 2];
        uint32_t* gdst = reinterpret_cast<uint32_t*>(sG) + (int64_t)(tt - s0) * (SW / 2) * NT + tid;
#pragma unroll
        for (int j = 0; j < SW / 2; ++j) {
          float2 G = fma2(Ct[j], dy2, P[j]);
          if (HS) G = add2(G, Ht[j]);
          __nv_bfloat162 gp = __floats2bfloat162_rn(G.x, G.y);
          gdst[j * NT] = *reinterpret_cast<uint32_t*>(&gp);
          duq[j & 1] = fma2(G, Bt[j], duq[j & 1]);
          gb[j] = mul2(G, dx2);
          P[j] = mul2(ex2x2(mul2(A2[j], dd)), G);
        }
        atomicAdd(&sDU[tt * 32 + lane], (duq[0].x + duq[0].y) + (duq[1].x + duq[1].y));
        const float r = reduce_scatter16p(gb, lane);
        if ((lane & 1) == 0)
          p.dB_part[(((int64_t)b * p.G + cblk) * p.S + t0 + tt) * N + w * SW + (lane >> 1)] = r;
      }
      // B2: recompute h over the sub-chunk and form the decay gradients
      {
        float2 h[SW / 2];
        const float2* src = reinterpret_cast<const float2*>(scratch + (int64_t)sub * SW * NT);
#pragma unroll
        for (int j = 0; j < SW / 2; ++j) h[j] = src[j * NT + tid];
        for (int tt = s0; tt < s1; ++tt) {
          const float d = sDt[tt * 32 + lane];
          const float2 dd = f2(d), mdd = f2(-d), dx2 = f2(sDtx[tt * 32 + lane]);
          float2 Bt[SW / 2];
          ld_row16p(Bt, sB + tt * N + w * SW, qx);
          const uint32_t* gsrc = reinterpret_cast<const uint32_t*>(sG) + (int64_t)(tt - s0) * (SW / 2) * NT + tid;
          float2 ddq[2] = {f2(0.f), f2(0.f)};
#pragma unroll
          for (int j = 0; j < SW / 2; ++j) {
            const uint32_t gw = gsrc[j * NT];
            const float2 gf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gw));
            const float2 v = mul2(ex2x2(mul2(A2[j], dd)), h[j]);
            h[j] = fma2(Bt[j], dx2, v);
            const float2 gv = mul2(gf, v);
            ddq[j & 1] = fma2(gv, A2[j], ddq[j & 1]);
            dAacc[j] = fma2(gv, mdd, dAacc[j]);
          }
          atomicAdd(&sDD[tt * 32 + lane], (ddq[0].x + ddq[0].y) + (ddq[1].x + ddq[1].y));
        }
      }
    }
    __syncthreads();
    // epilogue B: dx, ddt
    for (int i = tid; i < L * 32; i += NT) {
      const int tt = i >> 5, cc = cblk * 32 + (i & 31);
      if (cc >= p.Di) continue;
      const float d = sDt[i], xv = sX[i], du = sDU[i];
      float ddt = sDD[i] * LN2 + xv * du;       // decay part uses A2 = -A*log2(e)
      const float dxo = d * du + p.D[cc] * sDyp[i];
      if (SOFTPLUS) {
        const float raw = ldf<T>(p.dt, (int64_t)b * p.dt_bs + (int64_t)(t0 + tt) * p.dt_ts + cc);
        ddt *= (raw > 20.f) ? 1.f : sigmoid_f(raw);
      }
      const int64_t off = ((int64_t)b * p.S + t0 + tt) * p.Di + cc;
      reinterpret_cast<T*>(p.dx)[off] = from_f<T>(dxo);
      reinterpret_cast<T*>(p.ddt)[off] = from_f<T>(ddt);
    }
  }
  __syncthreads();
  {
    const float r = reduce_scatter16p(dAacc, lane);
    if ((lane & 1) == 0) atomicAdd(&p.dA[w * SW + (lane >> 1)], r);
  }
  if (tid < 32 && cvalid) atomicAdd(&p.dD[c], sDsum[tid]);
}

// ---------------------------------------------------------------------------------------------
inline size_t fwd_smem(int N) { return (size_t)(2 * CK * N + 2 * CK * 32 + (N / SW) * CK * 32) * sizeof(float); }
inline size_t bwd_smem(int N, bool hs) {
  size_t f = (size_t)(2 * CK * N + (hs ? CK * N : 0) + 7 * CK * 32 + N + 32) * sizeof(float);
  return f + (size_t)SUB * 32 * N * sizeof(__nv_bfloat16);
}

template <typename T, int NW, bool SP, bool GATE, bool HS>
void launch_fwd(const Params& p) {
  auto k = scan_fwd_kernel<T, NW, SP, GATE, HS, 1>;      // unrolling the time loop was slower (2.70 vs 2.51 ms)
  size_t sm = fwd_smem(NW * SW);
  MAMF_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
  dim3 grid((p.Di + 31) / 32, p.Bsz);
  k<<<grid, NW * 32, sm, stream()>>>(p);
  MAMF_LAUNCH_CHECK();
}

template <typename T, int NW, bool SP, bool GATE, bool HS>
void launch_bwd(const Params& p) {
  auto k = scan_bwd_kernel<T, NW, SP, GATE, HS, 2>;      // phase A unrolled by 2: 8.37 -> 8.10 ms
  size_t sm = bwd_smem(NW * SW, HS);
  MAMF_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
  dim3 grid((p.Di + 31) / 32, p.Bsz);
  k<<<grid, NW * 32, sm, stream()>>>(p);
  MAMF_LAUNCH_CHECK();
}

template <bool FWD, typename T, int NW>
void dispatch_flags(const Params& p, bool sp, bool gate, bool hs) {
#define MAMF_SCAN_CASE(SP, GT, H)                                               \
  if (sp == SP && gate == GT && hs == H) {                                      \
    if (FWD) launch_fwd<T, NW, SP, GT, H>(p); else launch_bwd<T, NW, SP, GT, H>(p); \
    return;                                                                     \
  }
  MAMF_SCAN_CASE(true, true, true) MAMF_SCAN_CASE(true, true, false)
  MAMF_SCAN_CASE(false, false, true) MAMF_SCAN_CASE(false, false, false)
#undef MAMF_SCAN_CASE
  TORCH_CHECK(false, "selective scan: unsupported flag combination (softplus and gate go together)");
}

template <bool FWD, typename T>
void dispatch_nw(const Params& p, bool sp, bool gate, bool hs) {
  switch (p.N) {
    case 32: dispatch_flags<FWD, T, 2>(p, sp, gate, hs); break;
    case 64: dispatch_flags<FWD, T, 4>(p, sp, gate, hs); break;
    case 128: dispatch_flags<FWD, T, 8>(p, sp, gate, hs); break;
    default: TORCH_CHECK(false, "selective scan: d_state must be 32, 64 or 128, got ", p.N);
  }
}

}  // namespace scan

// Python-facing entry points --------------------------------------------------------------------
using scan::Params;

static void fill_common(Params& p, const at::Tensor& x, const at::Tensor& dt, const at::Tensor& Bm,
                        const at::Tensor& Cm, const c10::optional<at::Tensor>& z,
                        const at::Tensor& A_log, const at::Tensor& D) {
  TORCH_CHECK(x.dim() == 3 && x.stride(2) == 1 && dt.stride(2) == 1 && Bm.stride(2) == 1 && Cm.stride(2) == 1,
              "selective scan: inputs must be (B, S, C) with unit inner stride");
  p.Bsz = x.size(0); p.S = x.size(1); p.Di = x.size(2); p.N = Bm.size(2);
  TORCH_CHECK(A_log.numel() == p.N && D.numel() == p.Di && A_log.dtype() == at::kFloat && D.dtype() == at::kFloat,
              "selective scan: A_log (N,) and D (Di,) must be fp32");
  p.G = (p.Di + 31) / 32;
  p.nck = (p.S + scan::CK - 1) / scan::CK;
  p.x = x.data_ptr(); p.x_bs = x.stride(0); p.x_ts = x.stride(1);
  p.dt = dt.data_ptr(); p.dt_bs = dt.stride(0); p.dt_ts = dt.stride(1);
  p.Bm = Bm.data_ptr(); p.B_bs = Bm.stride(0); p.B_ts = Bm.stride(1);
  p.Cm = Cm.data_ptr(); p.C_bs = Cm.stride(0); p.C_ts = Cm.stride(1);
  if (z.has_value()) {
    TORCH_CHECK(z->stride(2) == 1, "selective scan: z needs unit inner stride");
    p.z = z->data_ptr(); p.z_bs = z->stride(0); p.z_ts = z->stride(1);
  } else {
    p.z = nullptr; p.z_bs = p.z_ts = 0;
  }
  p.A_log = A_log.data_ptr<float>();
  p.D = D.data_ptr<float>();
}

// Returns (y, hs or empty, ckpt, final or empty)
std::vector<at::Tensor> selective_scan_fwd(at::Tensor x, at::Tensor dt, at::Tensor A_log, at::Tensor Bm,
                                           at::Tensor Cm, at::Tensor D, c10::optional<at::Tensor> z,
                                           c10::optional<at::Tensor> h0, bool softplus, bool need_hs,
                                           bool need_final) {
  c10::cuda::CUDAGuard g(x.device());
  Params p{};
  fill_common(p, x, dt, Bm, Cm, z, A_log, D);
  auto f32 = x.options().dtype(at::kFloat);
  at::Tensor y = at::empty({p.Bsz, p.S, p.Di}, x.options());
  at::Tensor ckpt = at::empty({p.Bsz, p.nck, p.Di, p.N}, f32);
  at::Tensor part, fin;
  p.y = y.data_ptr(); p.y_bs = y.stride(0); p.y_ts = y.stride(1);
  p.ckpt = ckpt.data_ptr<float>();
  if (need_hs) { part = at::empty({p.Bsz, p.G, p.S, p.N}, f32); p.hs_part = part.data_ptr<float>(); }
  if (need_final) { fin = at::empty({p.Bsz, p.Di, p.N}, f32); p.final_state = fin.data_ptr<float>(); }
  at::Tensor h0c;
  if (h0.has_value()) { h0c = h0->to(at::kFloat).contiguous(); p.h0 = h0c.data_ptr<float>(); }
  if (x.scalar_type() == at::kBFloat16) scan::dispatch_nw<true, __nv_bfloat16>(p, softplus, z.has_value(), need_hs);
  else if (x.scalar_type() == at::kFloat) scan::dispatch_nw<true, float>(p, softplus, z.has_value(), need_hs);
  else TORCH_CHECK(false, "selective scan: bf16 or fp32 inputs");
  at::Tensor hs;
  if (need_hs) hs = part.sum(1).div_((double)p.Di);
  return {y, hs, ckpt, fin};
}

// Returns (dx, ddt, dB, dC, dz or empty, dA (N,), dD (Di,))
std::vector<at::Tensor> selective_scan_bwd(at::Tensor x, at::Tensor dt, at::Tensor A_log, at::Tensor Bm,
                                           at::Tensor Cm, at::Tensor D, c10::optional<at::Tensor> z,
                                           at::Tensor ckpt, at::Tensor dy, c10::optional<at::Tensor> dhs,
                                           bool softplus) {
  c10::cuda::CUDAGuard g(x.device());
  Params p{};
  fill_common(p, x, dt, Bm, Cm, z, A_log, D);
  TORCH_CHECK(dy.stride(2) == 1, "selective scan bwd: dy needs unit inner stride");
  auto f32 = x.options().dtype(at::kFloat);
  p.ckpt = ckpt.data_ptr<float>();
  p.dy = dy.data_ptr(); p.dy_bs = dy.stride(0); p.dy_ts = dy.stride(1);
  at::Tensor dhs_c;
  if (dhs.has_value()) { dhs_c = dhs->to(at::kFloat).contiguous(); p.dhs = dhs_c.data_ptr<float>(); }
  at::Tensor dx = at::empty({p.Bsz, p.S, p.Di}, x.options());
  at::Tensor ddt = at::empty({p.Bsz, p.S, p.Di}, x.options());
  at::Tensor dz;
  if (z.has_value()) { dz = at::empty({p.Bsz, p.S, p.Di}, x.options()); p.dz = dz.data_ptr(); }
  at::Tensor dBp = at::empty({p.Bsz, p.G, p.S, p.N}, f32);
  at::Tensor dCp = at::empty({p.Bsz, p.G, p.S, p.N}, f32);
  at::Tensor dA = at::zeros({p.N}, f32);
  at::Tensor dD = at::zeros({p.Di}, f32);
  at::Tensor scratch = at::empty({(int64_t)p.Bsz * p.G * (scan::CK / scan::SUB) * 32 * p.N}, f32);
  p.dx = dx.data_ptr(); p.ddt = ddt.data_ptr();
  p.dB_part = dBp.data_ptr<float>(); p.dC_part = dCp.data_ptr<float>();
  p.dA = dA.data_ptr<float>(); p.dD = dD.data_ptr<float>();
  p.scratch = scratch.data_ptr<float>();
  if (x.scalar_type() == at::kBFloat16) scan::dispatch_nw<false, __nv_bfloat16>(p, softplus, z.has_value(), dhs.has_value());
  else if (x.scalar_type() == at::kFloat) scan::dispatch_nw<false, float>(p, softplus, z.has_value(), dhs.has_value());
  else TORCH_CHECK(false, "selective scan: bf16 or fp32 inputs");
  return {dx, ddt, dBp.sum(1), dCp.sum(1), dz, dA, dD};
}

}  // namespace mamf
