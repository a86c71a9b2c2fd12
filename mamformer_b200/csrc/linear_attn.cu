// KDA-Diff causal linear attention (dual query, shared K/V, differential combine), forward and
// backward, chunked for sm_100a.
//
// Reference semantics (mamformer/layers/kda_diff.py:357-478, kernels/triton_ssd.py:59-181):
//   phi(x) = elu(x[:K]) + 1
//   o_m,i  = phi(q_m,i) S_i / (phi(q_m,i) . z_i + 1e-8),  S_i = sum_{j<=i} phi(k_j)^T v_j,
//            z_i = sum_{j<=i} phi(k_j)                                   (m = 1, 2)
//   out_i  = (o_1,i - lam o_2,i) / (1 - lam + 1e-8)
// K/V heads are shared by H/G query heads (GQA).  Accumulation is fp32 throughout (the
// reference keeps bf16 intermediates; the fp32 form is the oracle of the tests).
//
// Chunked algorithm (chunk C = 64 rows):
//   la_state   per (b, kv-head g, chunk c): dS_c = Pk_c^T V_c, dz_c = sum Pk_c         (fp32)
//   la_prefix  exclusive prefix over chunks, in place: S_c = sum_{c' < c} dS_c'
//   la_fwd     per (b, q-head h, chunk c): A_m = tril(Pq_m Pk^T); N_m = A_m V + Pq_m S_c;
//              D_m = rowsum A_m + Pq_m . z_c; out = (N_1/D_1 - lam N_2/D_2)/(1 - lam)
// Backward (o_m = N_m / D_m, do_m = c_m dout with c_1 = 1/(1-lam), c_2 = -lam/(1-lam)):
//   dN = do / D, dD = -(do . o) / D, dA_ij = dN_i . v_j + dD_i (j <= i)
//   dPq_i = sum_j dA_ij Pk_j + S_i dN_i + dD_i z_i
//   dPk_j = sum_{m, i >= j} dA_ij Pq_i = intra + R_j v_j + r_j,   dv_j = intra + R_j^T Pk_j
//   with the reverse states R_j = sum_{m, i > chunk(j)} Pq_i dN_i^T, r_j = sum dD_i Pq_i.
//   la_bwd_dn     per (b, h, c): recompute o_m; store dN_m, dD_m; chunk partials dR, dr; dlam
//   la_rprefix    reverse exclusive prefix over chunks, summing the group's query heads
//   la_bwd_dqkv   per (b, g, c): loop over the group's heads and both queries: dq_m, and the
//                 chunk's dk, dv (intra + reverse-state terms)
// The per-thread work is a 4 x (cols/16) register tile of each 64 x cols product (rows and
// columns strided by 16 over the threads; shared-memory rows padded by one word).
#include "common.cuh"
#include "warp_mma.cuh"

namespace mamf {
namespace la {

constexpr int C = 64;
constexpr int NT = 256;

__device__ __forceinline__ float phi_f(float x) { return x > 0.f ? x + 1.f : __expf(x); }
__device__ __forceinline__ float dphi_f(float x) { return x > 0.f ? 1.f : __expf(x); }

struct Params {
  const __nv_bfloat16 *q1, *q2, *k, *v;   // (B,S,H,HD) / (B,S,G,HD)
  __nv_bfloat16* out;                     // (B,S,H,HD)
  const float* lam;                       // (H,)
  float *st, *zs;                         // (B,G,NC,K,HD), (B,G,NC,K): prefix states
  // backward
  const __nv_bfloat16* dout;
  float *dN, *dD;                         // (B,S,H,2,HD), (B,S,H,2)
  float *R, *r;                           // (B,H,NC,K,HD) partials -> (B,G,NC,K,HD) reverse states
  float *Rg, *rg;
  __nv_bfloat16 *dq1, *dq2, *dk, *dv;
  float* dlam;                            // (H,) accumulated
  int B, S, H, G, NC;
};

// Shared-memory tiles are row-padded (stride cols + 1) and every thread owns rows r, r + 16,
// r + 32, r + 48 and columns c, c + 16, ...: the 16 threads that read different rows of one
// column hit 16 different banks, and threads that share a row read one broadcast word.
template <int COLS>
struct Pad { static constexpr int v = COLS + 1; };

// Load `rows` rows (<= C) of an (B,S,heads,HD) tensor at (b, s0, head) into smem [C][COLS+1] as
// fp32, applying phi when PHI (only the first COLS columns are loaded).
template <int COLS, bool PHI>
__device__ __forceinline__ void load_rows(float* dst, const __nv_bfloat16* src, int b, int s0, int rows, int head,
                                          int heads, int HD, int S) {
  constexpr int LDS = Pad<COLS>::v;
  for (int idx = threadIdx.x; idx < C * COLS; idx += NT) {
    const int i = idx / COLS, c = idx % COLS;
    float x = 0.f;
    if (i < rows) {
      x = __bfloat162float(src[(((int64_t)b * S + s0 + i) * heads + head) * HD + c]);
      if (PHI) x = phi_f(x);
    }
    dst[i * LDS + c] = x;
  }
}

// ---- forward ------------------------------------------------------------------------------------
template <int K, int HD>
__global__ void __launch_bounds__(NT) la_state_kernel(Params p) {
  extern __shared__ float sm[];
  constexpr int LK = Pad<K>::v, LD = Pad<HD>::v;
  float* sK = sm;                 // C x LK
  float* sV = sK + C * LK;        // C x LD
  const int c = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int s0 = c * C, rows = min(C, p.S - s0);
  load_rows<K, true>(sK, p.k, b, s0, rows, g, p.G, HD, p.S);
  load_rows<HD, false>(sV, p.v, b, s0, rows, g, p.G, HD, p.S);
  __syncthreads();
  constexpr int RK = K / 16, RD = HD / 16;
  const int tk = threadIdx.x / 16, td = threadIdx.x % 16;
  float acc[RK][RD];
#pragma unroll
  for (int a = 0; a < RK; ++a)
#pragma unroll
    for (int e = 0; e < RD; ++e) acc[a][e] = 0.f;
  for (int j = 0; j < rows; ++j) {
    float kk[RK], vv[RD];
#pragma unroll
    for (int a = 0; a < RK; ++a) kk[a] = sK[j * LK + tk + 16 * a];
#pragma unroll
    for (int e = 0; e < RD; ++e) vv[e] = sV[j * LD + td + 16 * e];
#pragma unroll
    for (int a = 0; a < RK; ++a)
#pragma unroll
      for (int e = 0; e < RD; ++e) acc[a][e] += kk[a] * vv[e];
  }
  float* S = p.st + ((((int64_t)b * p.G + g) * p.NC + c) * K) * HD;
#pragma unroll
  for (int a = 0; a < RK; ++a)
#pragma unroll
    for (int e = 0; e < RD; ++e) S[(tk + 16 * a) * HD + td + 16 * e] = acc[a][e];
  if (threadIdx.x < K) {
    float s = 0.f;
    for (int j = 0; j < rows; ++j) s += sK[j * LK + threadIdx.x];
    p.zs[(((int64_t)b * p.G + g) * p.NC + c) * K + threadIdx.x] = s;
  }
}

// exclusive prefix (forward) or reverse exclusive prefix over chunks; `sum_heads` > 1 sums that
// many consecutive source heads (the query heads of one KV group) into one destination.
__global__ void la_prefix_kernel(float* dst, const float* src, int64_t elems, int NC, int sum_heads, bool reverse,
                                 int G) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= elems) return;
  const int bg = blockIdx.y;                       // b * G + g
  const int b = bg / G, g = bg % G;
  float run = 0.f;
  for (int t = 0; t < NC; ++t) {
    const int c = reverse ? NC - 1 - t : t;
    float add = 0.f;
    for (int hh = 0; hh < sum_heads; ++hh) {
      const int64_t sh = (int64_t)b * G * sum_heads + g * sum_heads + hh;
      add += src[(sh * NC + c) * elems + e];
    }
    dst[((int64_t)bg * NC + c) * elems + e] = run;
    run += add;
  }
}

// A = tril(Pq Pk^T): thread (ti, tj) owns rows ti + 16x and columns tj + 16y
template <int K>
__device__ __forceinline__ void tile_A(float* sA, const float* sQ, const float* sK, int rows) {
  constexpr int LK = Pad<K>::v, LC = Pad<C>::v;
  const int ti = threadIdx.x / 16, tj = threadIdx.x % 16;
  float a[4][4];
#pragma unroll
  for (int x = 0; x < 4; ++x)
#pragma unroll
    for (int y = 0; y < 4; ++y) a[x][y] = 0.f;
  for (int kk = 0; kk < K; ++kk) {
    float q[4], k[4];
#pragma unroll
    for (int x = 0; x < 4; ++x) q[x] = sQ[(ti + 16 * x) * LK + kk];
#pragma unroll
    for (int y = 0; y < 4; ++y) k[y] = sK[(tj + 16 * y) * LK + kk];
#pragma unroll
    for (int x = 0; x < 4; ++x)
#pragma unroll
      for (int y = 0; y < 4; ++y) a[x][y] += q[x] * k[y];
  }
#pragma unroll
  for (int x = 0; x < 4; ++x)
#pragma unroll
    for (int y = 0; y < 4; ++y) {
      const int i = ti + 16 * x, j = tj + 16 * y;
      sA[i * LC + j] = (j <= i && i < rows && j < rows) ? a[x][y] : 0.f;
    }
}

// N (rows ti + 16x, columns td + 16e) = A V + Pq S; D (per row, in sD) = rowsum A + Pq . z
template <int K, int HD>
__device__ __forceinline__ void num_den(float (&n)[4][HD / 16], float* sD, const float* sA, const float* sV,
                                        const float* sQ, const float* S, const float* z, bool has_state) {
  constexpr int RD = HD / 16, LK = Pad<K>::v, LD = Pad<HD>::v, LC = Pad<C>::v;
  const int ti = threadIdx.x / 16, td = threadIdx.x % 16;
#pragma unroll
  for (int x = 0; x < 4; ++x)
#pragma unroll
    for (int e = 0; e < RD; ++e) n[x][e] = 0.f;
  for (int j = 0; j < C; ++j) {
    float a[4], v[RD];
#pragma unroll
    for (int x = 0; x < 4; ++x) a[x] = sA[(ti + 16 * x) * LC + j];
#pragma unroll
    for (int e = 0; e < RD; ++e) v[e] = sV[j * LD + td + 16 * e];
#pragma unroll
    for (int x = 0; x < 4; ++x)
#pragma unroll
      for (int e = 0; e < RD; ++e) n[x][e] += a[x] * v[e];
  }
  if (has_state) {
    for (int kk = 0; kk < K; ++kk) {
      float q[4], s[RD];
#pragma unroll
      for (int x = 0; x < 4; ++x) q[x] = sQ[(ti + 16 * x) * LK + kk];
#pragma unroll
      for (int e = 0; e < RD; ++e) s[e] = S[kk * HD + td + 16 * e];
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int e = 0; e < RD; ++e) n[x][e] += q[x] * s[e];
    }
  }
  if (threadIdx.x < C) {
    const int i = threadIdx.x;
    float d = 0.f;
    for (int j = 0; j < C; ++j) d += sA[i * LC + j];
    if (has_state)
      for (int kk = 0; kk < K; ++kk) d += sQ[i * LK + kk] * z[kk];
    sD[i] = d + 1e-8f;
  }
}

template <int K, int HD>
__global__ void __launch_bounds__(NT) la_fwd_kernel(Params p) {
  extern __shared__ float sm[];
  constexpr int LK = Pad<K>::v, LD = Pad<HD>::v, LC = Pad<C>::v;
  float* sQ = sm;                   // C x LK
  float* sK = sQ + C * LK;          // C x LK
  float* sV = sK + C * LK;          // C x LD
  float* sA = sV + C * LD;          // C x LC
  float* sD = sA + C * LC;          // C
  constexpr int RD = HD / 16;
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int g = h / (p.H / p.G);
  const int s0 = c * C, rows = min(C, p.S - s0);
  const float* S = p.st + ((((int64_t)b * p.G + g) * p.NC + c) * K) * HD;
  const float* z = p.zs + (((int64_t)b * p.G + g) * p.NC + c) * K;
  load_rows<K, true>(sK, p.k, b, s0, rows, g, p.G, HD, p.S);
  load_rows<HD, false>(sV, p.v, b, s0, rows, g, p.G, HD, p.S);
  const float lam = p.lam[h];
  const float inv = 1.f / (1.f - lam + 1e-8f);
  float o[4][RD];
  const int ti = threadIdx.x / 16, td = threadIdx.x % 16;
  for (int m = 0; m < 2; ++m) {
    __syncthreads();
    load_rows<K, true>(sQ, m == 0 ? p.q1 : p.q2, b, s0, rows, h, p.H, HD, p.S);
    __syncthreads();
    tile_A<K>(sA, sQ, sK, rows);
    __syncthreads();
    float n[4][RD];
    num_den<K, HD>(n, sD, sA, sV, sQ, S, z, c > 0);
    __syncthreads();
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      const float rd = 1.f / sD[ti + 16 * x];
#pragma unroll
      for (int e = 0; e < RD; ++e) {
        const float val = n[x][e] * rd;
        o[x][e] = (m == 0) ? val : (o[x][e] - lam * val) * inv;
      }
    }
  }
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    const int i = ti + 16 * x;
    if (i >= rows) continue;
    __nv_bfloat16* dst = p.out + (((int64_t)b * p.S + s0 + i) * p.H + h) * HD;
#pragma unroll
    for (int e = 0; e < RD; ++e) dst[td + 16 * e] = __float2bfloat16(o[x][e]);
  }
}

// ---- backward ------------------------------------------------------------------------------------
template <int K, int HD>
__global__ void __launch_bounds__(NT) la_bwd_dn_kernel(Params p) {
  extern __shared__ float sm[];
  constexpr int LK = Pad<K>::v, LD = Pad<HD>::v, LC = Pad<C>::v;
  float* sQ = sm;                   // C x LK  (query m)
  float* sK = sQ + C * LK;
  float* sV = sK + C * LK;          // C x LD
  float* sA = sV + C * LD;          // C x LC
  float* sD = sA + C * LC;          // C
  float* sdN = sD + C;              // C x LD (dN of query m)
  float* sdD = sdN + C * LD;        // C
  float* sRed = sdD + C;            // 32
  constexpr int RD = HD / 16, RK = K / 16;
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int g = h / (p.H / p.G);
  const int s0 = c * C, rows = min(C, p.S - s0);
  const float* S = p.st + ((((int64_t)b * p.G + g) * p.NC + c) * K) * HD;
  const float* z = p.zs + (((int64_t)b * p.G + g) * p.NC + c) * K;
  load_rows<K, true>(sK, p.k, b, s0, rows, g, p.G, HD, p.S);
  load_rows<HD, false>(sV, p.v, b, s0, rows, g, p.G, HD, p.S);
  const float lam = p.lam[h];
  const float inv = 1.f / (1.f - lam + 1e-8f);
  const int ti = threadIdx.x / 16, td = threadIdx.x % 16;
  float dout[4][RD], o1[4][RD];
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    const int i = ti + 16 * x;
#pragma unroll
    for (int e = 0; e < RD; ++e)
      dout[x][e] = (i < rows) ? __bfloat162float(p.dout[(((int64_t)b * p.S + s0 + i) * p.H + h) * HD + td + 16 * e])
                              : 0.f;
  }
  // chunk partial of the reverse state for this query head: dR = sum_m Pq_m^T dN_m, dr = sum_m Pq_m^T dD_m
  const int tk = threadIdx.x / 16;
  float accR[RK][RD];
#pragma unroll
  for (int a = 0; a < RK; ++a)
#pragma unroll
    for (int e = 0; e < RD; ++e) accR[a][e] = 0.f;
  float accr = 0.f;
  float dl = 0.f;
  for (int m = 0; m < 2; ++m) {
    __syncthreads();
    load_rows<K, true>(sQ, m == 0 ? p.q1 : p.q2, b, s0, rows, h, p.H, HD, p.S);
    __syncthreads();
    tile_A<K>(sA, sQ, sK, rows);
    __syncthreads();
    float n[4][RD];
    num_den<K, HD>(n, sD, sA, sV, sQ, S, z, c > 0);
    __syncthreads();
    const float cm = (m == 0) ? inv : -lam * inv;
    // dN = cm dout / D;  dD = -(cm dout . o) / D  (row reduction over the 16 threads of a row)
#pragma unroll
    for (int x = 0; x < 4; ++x) {
      const int i = ti + 16 * x;
      const float rd = 1.f / sD[i];
      float part = 0.f;
#pragma unroll
      for (int e = 0; e < RD; ++e) {
        const float o = n[x][e] * rd;
        if (m == 0) o1[x][e] = o;
        else dl += dout[x][e] * (o1[x][e] - o);
        sdN[i * LD + td + 16 * e] = cm * dout[x][e] * rd;
        part += cm * dout[x][e] * o;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
      if (td == 0) sdD[i] = (i < rows) ? -part * rd : 0.f;
    }
    __syncthreads();
    // store dN, dD for the dq/dk/dv kernel
    for (int idx = threadIdx.x; idx < rows * HD; idx += NT) {
      const int i = idx / HD, e = idx % HD;
      p.dN[((((int64_t)b * p.S + s0 + i) * p.H + h) * 2 + m) * HD + e] = sdN[i * LD + e];
    }
    if (threadIdx.x < rows) p.dD[(((int64_t)b * p.S + s0 + threadIdx.x) * p.H + h) * 2 + m] = sdD[threadIdx.x];
    // accumulate dR += Pq^T dN, dr += Pq^T dD over the chunk rows
    for (int i = 0; i < rows; ++i) {
      float q[RK], dn[RD];
#pragma unroll
      for (int a = 0; a < RK; ++a) q[a] = sQ[i * LK + tk + 16 * a];
#pragma unroll
      for (int e = 0; e < RD; ++e) dn[e] = sdN[i * LD + td + 16 * e];
#pragma unroll
      for (int a = 0; a < RK; ++a)
#pragma unroll
        for (int e = 0; e < RD; ++e) accR[a][e] += q[a] * dn[e];
    }
    if (threadIdx.x < K)
      for (int i = 0; i < rows; ++i) accr += sQ[i * LK + threadIdx.x] * sdD[i];
  }
  float* R = p.R + ((((int64_t)b * p.H + h) * p.NC + c) * K) * HD;
#pragma unroll
  for (int a = 0; a < RK; ++a)
#pragma unroll
    for (int e = 0; e < RD; ++e) R[(tk + 16 * a) * HD + td + 16 * e] = accR[a][e];
  if (threadIdx.x < K) p.r[(((int64_t)b * p.H + h) * p.NC + c) * K + threadIdx.x] = accr;
  // dlam = sum dout . (o1 - o2) / (1 - lam)^2
  dl = warp_sum(dl);
  if ((threadIdx.x & 31) == 0) sRed[threadIdx.x >> 5] = dl;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < NT / 32; ++w) t += sRed[w];
    atomicAdd(p.dlam + h, t * inv * inv);
  }
}

template <int K, int HD>
__global__ void __launch_bounds__(NT) la_bwd_dqkv_kernel(Params p) {
  extern __shared__ float sm[];
  constexpr int LK = Pad<K>::v, LD = Pad<HD>::v, LC = Pad<C>::v;
  float* sK = sm;                   // C x LK (phi k)
  float* sV = sK + C * LK;          // C x LD
  float* sQ = sV + C * LD;          // C x LK (phi q of the current head / query)
  float* sdN = sQ + C * LK;         // C x LD
  float* sA = sdN + C * LD;         // C x LC
  float* sdA = sA + C * LC;         // C x LC
  float* sdD = sdA + C * LC;        // C
  constexpr int RD = HD / 16, RK = K / 16;
  const int c = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int groups = p.H / p.G;
  const int s0 = c * C, rows = min(C, p.S - s0);
  const float* S = p.st + ((((int64_t)b * p.G + g) * p.NC + c) * K) * HD;
  const float* z = p.zs + (((int64_t)b * p.G + g) * p.NC + c) * K;
  const float* Rn = p.Rg + ((((int64_t)b * p.G + g) * p.NC + c) * K) * HD;
  const float* rn = p.rg + (((int64_t)b * p.G + g) * p.NC + c) * K;
  load_rows<K, true>(sK, p.k, b, s0, rows, g, p.G, HD, p.S);
  load_rows<HD, false>(sV, p.v, b, s0, rows, g, p.G, HD, p.S);
  const int ti = threadIdx.x / 16, tc = threadIdx.x % 16;
  float dPk[4][RK], dVv[4][RD];
#pragma unroll
  for (int x = 0; x < 4; ++x) {
#pragma unroll
    for (int a = 0; a < RK; ++a) dPk[x][a] = 0.f;
#pragma unroll
    for (int e = 0; e < RD; ++e) dVv[x][e] = 0.f;
  }
  for (int hh = 0; hh < groups; ++hh) {
    const int h = g * groups + hh;
    for (int m = 0; m < 2; ++m) {
      __syncthreads();
      load_rows<K, true>(sQ, m == 0 ? p.q1 : p.q2, b, s0, rows, h, p.H, HD, p.S);
      for (int idx = threadIdx.x; idx < C * HD; idx += NT) {
        const int i = idx / HD, e = idx % HD;
        sdN[i * LD + e] = (i < rows) ? p.dN[((((int64_t)b * p.S + s0 + i) * p.H + h) * 2 + m) * HD + e] : 0.f;
      }
      if (threadIdx.x < C)
        sdD[threadIdx.x] = (threadIdx.x < rows) ? p.dD[(((int64_t)b * p.S + s0 + threadIdx.x) * p.H + h) * 2 + m] : 0.f;
      __syncthreads();
      tile_A<K>(sA, sQ, sK, rows);
      // dA = tril(dN V^T + dD)
      {
        float a[4][4];
#pragma unroll
        for (int x = 0; x < 4; ++x)
#pragma unroll
          for (int y = 0; y < 4; ++y) a[x][y] = 0.f;
        for (int e = 0; e < HD; ++e) {
          float dn[4], vv[4];
#pragma unroll
          for (int x = 0; x < 4; ++x) dn[x] = sdN[(ti + 16 * x) * LD + e];
#pragma unroll
          for (int y = 0; y < 4; ++y) vv[y] = sV[(tc + 16 * y) * LD + e];
#pragma unroll
          for (int x = 0; x < 4; ++x)
#pragma unroll
            for (int y = 0; y < 4; ++y) a[x][y] += dn[x] * vv[y];
        }
#pragma unroll
        for (int x = 0; x < 4; ++x)
#pragma unroll
          for (int y = 0; y < 4; ++y) {
            const int i = ti + 16 * x, j = tc + 16 * y;
            sdA[i * LC + j] = (j <= i && i < rows && j < rows) ? a[x][y] + sdD[i] : 0.f;
          }
      }
      __syncthreads();
      // dPq (rows ti + 16x, columns tc + 16a) = dA Pk + dN S^T + dD z  ->  dq
      {
        float dq[4][RK];
#pragma unroll
        for (int x = 0; x < 4; ++x)
#pragma unroll
          for (int a = 0; a < RK; ++a) dq[x][a] = 0.f;
        for (int j = 0; j < C; ++j) {
          float da[4], kk[RK];
#pragma unroll
          for (int x = 0; x < 4; ++x) da[x] = sdA[(ti + 16 * x) * LC + j];
#pragma unroll
          for (int a = 0; a < RK; ++a) kk[a] = sK[j * LK + tc + 16 * a];
#pragma unroll
          for (int x = 0; x < 4; ++x)
#pragma unroll
            for (int a = 0; a < RK; ++a) dq[x][a] += da[x] * kk[a];
        }
        if (c > 0) {
          for (int e = 0; e < HD; ++e) {
            float dn[4], s[RK];
#pragma unroll
            for (int x = 0; x < 4; ++x) dn[x] = sdN[(ti + 16 * x) * LD + e];
#pragma unroll
            for (int a = 0; a < RK; ++a) s[a] = S[(tc + 16 * a) * HD + e];
#pragma unroll
            for (int x = 0; x < 4; ++x)
#pragma unroll
              for (int a = 0; a < RK; ++a) dq[x][a] += dn[x] * s[a];
          }
#pragma unroll
          for (int x = 0; x < 4; ++x)
#pragma unroll
            for (int a = 0; a < RK; ++a) dq[x][a] += sdD[ti + 16 * x] * z[tc + 16 * a];
        }
        __nv_bfloat16* dqp = (m == 0) ? p.dq1 : p.dq2;
        const __nv_bfloat16* qp = (m == 0) ? p.q1 : p.q2;
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          const int i = ti + 16 * x;
          if (i >= rows) continue;
          const int64_t base = (((int64_t)b * p.S + s0 + i) * p.H + h) * HD;
#pragma unroll
          for (int a = 0; a < RK; ++a) {
            const int col = tc + 16 * a;
            dqp[base + col] = __float2bfloat16(dq[x][a] * dphi_f(__bfloat162float(qp[base + col])));
          }
          for (int col = K + tc; col < HD; col += 16) dqp[base + col] = __float2bfloat16(0.f);
        }
      }
      // dPk += dA^T Pq ;  dV += A^T dN   (rows j = ti + 16x of this thread)
      for (int i = 0; i < C; ++i) {
        float da[4], aa[4], q[RK], dn[RD];
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          da[x] = sdA[i * LC + ti + 16 * x];
          aa[x] = sA[i * LC + ti + 16 * x];
        }
#pragma unroll
        for (int a = 0; a < RK; ++a) q[a] = sQ[i * LK + tc + 16 * a];
#pragma unroll
        for (int e = 0; e < RD; ++e) dn[e] = sdN[i * LD + tc + 16 * e];
#pragma unroll
        for (int x = 0; x < 4; ++x) {
#pragma unroll
          for (int a = 0; a < RK; ++a) dPk[x][a] += da[x] * q[a];
#pragma unroll
          for (int e = 0; e < RD; ++e) dVv[x][e] += aa[x] * dn[e];
        }
      }
    }
  }
  // reverse-state terms: dPk_j += R v_j + r ;  dv_j += R^T Pk_j
  if (c + 1 < p.NC) {
    for (int e = 0; e < HD; ++e) {
      float vv[4], Rr[RK];
#pragma unroll
      for (int x = 0; x < 4; ++x) vv[x] = sV[(ti + 16 * x) * LD + e];
#pragma unroll
      for (int a = 0; a < RK; ++a) Rr[a] = Rn[(tc + 16 * a) * HD + e];
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int a = 0; a < RK; ++a) dPk[x][a] += Rr[a] * vv[x];
    }
#pragma unroll
    for (int x = 0; x < 4; ++x)
#pragma unroll
      for (int a = 0; a < RK; ++a) dPk[x][a] += rn[tc + 16 * a];
    for (int kk = 0; kk < K; ++kk) {
      float pk[4], Rr[RD];
#pragma unroll
      for (int x = 0; x < 4; ++x) pk[x] = sK[(ti + 16 * x) * LK + kk];
#pragma unroll
      for (int e = 0; e < RD; ++e) Rr[e] = Rn[kk * HD + tc + 16 * e];
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int e = 0; e < RD; ++e) dVv[x][e] += pk[x] * Rr[e];
    }
  }
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    const int j = ti + 16 * x;
    if (j >= rows) continue;
    const int64_t base = (((int64_t)b * p.S + s0 + j) * p.G + g) * HD;
#pragma unroll
    for (int a = 0; a < RK; ++a) {
      const int col = tc + 16 * a;
      p.dk[base + col] = __float2bfloat16(dPk[x][a] * dphi_f(__bfloat162float(p.k[base + col])));
    }
    for (int col = K + tc; col < HD; col += 16) p.dk[base + col] = __float2bfloat16(0.f);
#pragma unroll
    for (int e = 0; e < RD; ++e) p.dv[base + tc + 16 * e] = __float2bfloat16(dVv[x][e]);
  }
}

template <int K, int HD>
constexpr int fwd_smem() { return (2 * C * Pad<K>::v + C * Pad<HD>::v + C * Pad<C>::v + C) * 4; }
template <int K, int HD>
constexpr int dn_smem() { return (2 * C * Pad<K>::v + 2 * C * Pad<HD>::v + C * Pad<C>::v + 2 * C + 32) * 4; }
template <int K, int HD>
constexpr int dqkv_smem() { return (2 * C * Pad<K>::v + 2 * C * Pad<HD>::v + 2 * C * Pad<C>::v + C) * 4; }

template <typename F>
static void set_smem(F k, int bytes) {
  MAMF_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

template <int K, int HD>
static void run_states(Params& p) {
  dim3 gs(p.NC, p.G, p.B);
  const int sm_state = (C * Pad<K>::v + C * Pad<HD>::v) * 4;
  set_smem(la_state_kernel<K, HD>, sm_state);
  la_state_kernel<K, HD><<<gs, NT, sm_state, stream()>>>(p);
  MAMF_LAUNCH_CHECK();
  // in-place exclusive prefix (each thread walks its element over the chunks)
  const int64_t eS = (int64_t)K * HD, ez = K;
  la_prefix_kernel<<<dim3((unsigned)((eS + 255) / 256), p.B * p.G), 256, 0, stream()>>>(p.st, p.st, eS, p.NC, 1, false, p.G);
  la_prefix_kernel<<<dim3((unsigned)((ez + 255) / 256), p.B * p.G), 256, 0, stream()>>>(p.zs, p.zs, ez, p.NC, 1, false, p.G);
  MAMF_LAUNCH_CHECK();
}


// =================================================================================================
// Tensor-core path (K = HD = 128): the same chunk algorithm with every chunk product on warp-level
// mma.sync tiles (bf16 operands, fp32 accumulation).  4 warps x 16 rows per 64-row chunk.  The chunk
// state S (and z as an extra column) enters as a bf16 operand.
namespace tc {
constexpr int C = 64, NT = 128, D = 128;
constexpr int LB = D + 8;          // bf16 tile row stride (elements)
constexpr int LSX = D + 24;        // state tile [K][D + 16 (z column, zero pad)] + 8
constexpr int LC = C + 8;          // 64-wide tiles

// rows x 128 bf16 tile of (B, S, heads, 128) into smem (zero past `rows`), phi applied when PHI
template <bool PHI>
__device__ __forceinline__ void load_bf(__nv_bfloat16* dst, const __nv_bfloat16* src, int b, int s0, int rows,
                                        int head, int heads, int S) {
#pragma unroll
  for (int i = threadIdx.x; i < C * (D / 8); i += NT) {
    const int r = i / (D / 8), c = (i % (D / 8)) * 8;
    int4 v = make_int4(0, 0, 0, 0);
    if (r < rows) v = *reinterpret_cast<const int4*>(src + (((int64_t)b * S + s0 + r) * heads + head) * D + c);
    if (PHI) {
      __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&v);
#pragma unroll
      for (int k = 0; k < 8; ++k) e[k] = __float2bfloat16(r < rows ? phi_f(__bfloat162float(e[k])) : 0.f);
    }
    *reinterpret_cast<int4*>(dst + r * LB + c) = v;
  }
}
// fp32 (K x D) state rows -> bf16 smem rows of stride ld: 16-byte loads, eight in flight per thread
__device__ __forceinline__ void load_state_rows(__nv_bfloat16* dst, int ld, const float* S, bool has) {
#pragma unroll 8
  for (int i = threadIdx.x; i < D * (D / 4); i += NT) {
    const int r = i / (D / 4), c = (i % (D / 4)) * 4;
    const float4 v = has ? *reinterpret_cast<const float4*>(S + r * D + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    uint2 o;
    o.x = wm::pack_bf16(v.x, v.y);
    o.y = wm::pack_bf16(v.z, v.w);
    *reinterpret_cast<uint2*>(dst + r * ld + c) = o;
  }
}
// fp32 state (K x D) (+ z column, zero pad to D + 16) -> bf16 smem [K][LSX]
__device__ __forceinline__ void load_state(__nv_bfloat16* dst, const float* S, const float* z, bool has) {
  load_state_rows(dst, LSX, S, has);
  for (int i = threadIdx.x; i < D * 16; i += NT) {
    const int r = i / 16, c = D + i % 16;
    dst[r * LSX + c] = __float2bfloat16((has && c == D && z) ? z[r] : 0.f);
  }
}

// Q fragments (this warp's 16 rows, K = 128)
__device__ __forceinline__ void q_frags(uint32_t (&qf)[8][4], const __nv_bfloat16* sQ, int w, int lane) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) wm::ldsm_x4(qf[kk], sQ + (w * 16 + wm::a_row(lane)) * LB + kk * 16 + wm::a_col(lane));
}
// a (16 x 64) = tril(Q K^T) for this warp's rows
__device__ __forceinline__ void scores(float (&a)[8][4], const uint32_t (&qf)[8][4], const __nv_bfloat16* sK, int w,
                                       int lane, int rows) {
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) a[n][e] = 0.f;
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
#pragma unroll
    for (int n = 0; n < 8; n += 2) {
      uint32_t bf[4];
      wm::ldsm_x4(bf, sK + (n * 8 + wm::bn_row(lane)) * LB + kk * 16 + wm::bn_col(lane));
      wm::mma16816(a[n], qf[kk], bf[0], bf[1]);
      wm::mma16816(a[n + 1], qf[kk], bf[2], bf[3]);
    }
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = w * 16 + g + (e >> 1) * 8, j = n * 8 + 2 * t + (e & 1);
      if (!(j <= i && i < rows && j < rows)) a[n][e] = 0.f;
    }
}
// u (16 x 144) = A V + Q [S | z]; u[:, 128] = Q . z
__device__ __forceinline__ void numer(float (&u)[18][4], const float (&a)[8][4], const uint32_t (&qf)[8][4],
                                      const __nv_bfloat16* sV, const __nv_bfloat16* sS, int lane, bool has) {
#pragma unroll
  for (int n = 0; n < 18; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) u[n][e] = 0.f;
  // A enters as hi + lo bf16 parts: the scores of the positive feature map are nearly uniform, so
  // the two reads' outputs are close and the differential combination (and d lambda) would
  // otherwise inherit the 2^-9 rounding of A.
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t pa[4], pl[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float x0 = a[2 * j + (e >> 1)][(e & 1) * 2], x1 = a[2 * j + (e >> 1)][(e & 1) * 2 + 1];
      const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
      const float2 hf = __bfloat1622float2(h);
      pa[e] = *reinterpret_cast<const uint32_t*>(&h);
      pl[e] = wm::pack_bf16(x0 - hf.x, x1 - hf.y);
    }
#pragma unroll
    for (int n = 0; n < 16; n += 2) {
      uint32_t bf[4];
      wm::ldsm_x4_t(bf, sV + (j * 16 + wm::bt_row(lane)) * LB + n * 8 + wm::bt_col(lane));
      wm::mma16816(u[n], pa, bf[0], bf[1]);
      wm::mma16816(u[n + 1], pa, bf[2], bf[3]);
      wm::mma16816(u[n], pl, bf[0], bf[1]);
      wm::mma16816(u[n + 1], pl, bf[2], bf[3]);
    }
  }
  if (has) {
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
#pragma unroll
      for (int n = 0; n < 18; n += 2) {
        uint32_t bf[4];
        wm::ldsm_x4_t(bf, sS + (kk * 16 + wm::bt_row(lane)) * LSX + n * 8 + wm::bt_col(lane));
        wm::mma16816(u[n], qf[kk], bf[0], bf[1]);
        wm::mma16816(u[n + 1], qf[kk], bf[2], bf[3]);
      }
  }
}
// per-row denominators of this lane's two rows: rowsum(a) + (Q . z)
__device__ __forceinline__ void denom(float (&den)[2], const float (&a)[8][4], const float (&u)[18][4], int lane) {
  float rs[2] = {0.f, 0.f};
#pragma unroll
  for (int n = 0; n < 8; ++n) { rs[0] += a[n][0] + a[n][1]; rs[1] += a[n][2] + a[n][3]; }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
    rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
    const float zq = __shfl_sync(0xffffffffu, u[16][2 * r], lane & ~3);   // column 128 sits in lane t = 0
    den[r] = rs[r] + zq + 1e-8f;
  }
}

__global__ void __launch_bounds__(NT) fwd_kernel(Params p) {
  extern __shared__ __align__(16) unsigned char smraw[];
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(smraw);
  __nv_bfloat16* sV = sK + C * LB;
  __nv_bfloat16* sQ = sV + C * LB;
  __nv_bfloat16* sS = sQ + C * LB;     // [D][LSX]
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int g = h / (p.H / p.G);
  const int s0 = c * C, rows = min(C, p.S - s0);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, gq = lane >> 2, tq = lane & 3;
  load_bf<true>(sK, p.k, b, s0, rows, g, p.G, p.S);
  load_bf<false>(sV, p.v, b, s0, rows, g, p.G, p.S);
  const bool has = c > 0;
  if (has)
    load_state(sS, p.st + ((((int64_t)b * p.G + g) * p.NC + c) * D) * D, p.zs + (((int64_t)b * p.G + g) * p.NC + c) * D, true);
  const float lam = p.lam[h];
  const float inv = 1.f / (1.f - lam + 1e-8f);
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[n][e] = 0.f;
  for (int m = 0; m < 2; ++m) {
    __syncthreads();
    load_bf<true>(sQ, m == 0 ? p.q1 : p.q2, b, s0, rows, h, p.H, p.S);
    __syncthreads();
    uint32_t qf[8][4];
    q_frags(qf, sQ, w, lane);
    float a[8][4];
    scores(a, qf, sK, w, lane, rows);
    float u[18][4];
    numer(u, a, qf, sV, sS, lane, has);
    float den[2];
    denom(den, a, u, lane);
    const float cm = (m == 0) ? inv : -lam * inv;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] += cm * u[n][0] / den[0]; o[n][1] += cm * u[n][1] / den[0];
      o[n][2] += cm * u[n][2] / den[1]; o[n][3] += cm * u[n][3] / den[1];
    }
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int i = w * 16 + gq + 8 * r;
    if (i >= rows) continue;
    __nv_bfloat16* dst = p.out + (((int64_t)b * p.S + s0 + i) * p.H + h) * D;
#pragma unroll
    for (int n = 0; n < 16; ++n)
      *reinterpret_cast<__nv_bfloat162*>(dst + n * 8 + 2 * tq) = __floats2bfloat162_rn(o[n][2 * r], o[n][2 * r + 1]);
  }
}

// Backward part 1 (per b, query head h, chunk c): dN_m = c_m dout / D_m (bf16), dD_m = -(c_m dout . o_m) / D_m,
// chunk partial of the reverse state R += sum_m Pq_m^T dN_m, r += sum_m Pq_m^T dD_m, and dlam.
__global__ void __launch_bounds__(NT) dn_kernel(Params p, __nv_bfloat16* dNb) {
  extern __shared__ __align__(16) unsigned char smraw[];
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(smraw);
  __nv_bfloat16* sV = sK + C * LB;
  __nv_bfloat16* sQ = sV + C * LB;          // [2][C][LB]
  __nv_bfloat16* sdN = sQ + 2 * C * LB;     // [2][C][LB]
  __nv_bfloat16* sS = sdN + 2 * C * LB;     // [D][LSX]
  float* sdD = reinterpret_cast<float*>(sS + D * LSX);   // [2][C]
  float* sRed = sdD + 2 * C;                               // [NT / 32]
  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int g = h / (p.H / p.G);
  const int s0 = c * C, rows = min(C, p.S - s0);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, gq = lane >> 2, tq = lane & 3;
  load_bf<true>(sK, p.k, b, s0, rows, g, p.G, p.S);
  load_bf<false>(sV, p.v, b, s0, rows, g, p.G, p.S);
  load_bf<true>(sQ, p.q1, b, s0, rows, h, p.H, p.S);
  load_bf<true>(sQ + C * LB, p.q2, b, s0, rows, h, p.H, p.S);
  const bool has = c > 0;
  if (has)
    load_state(sS, p.st + ((((int64_t)b * p.G + g) * p.NC + c) * D) * D, p.zs + (((int64_t)b * p.G + g) * p.NC + c) * D, true);
  __syncthreads();
  const float lam = p.lam[h];
  const float inv = 1.f / (1.f - lam + 1e-8f);
  // dout in the accumulator layout of this warp's rows
  float dout[16][4];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int i = w * 16 + gq + 8 * r;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      float2 v = make_float2(0.f, 0.f);
      if (i < rows) v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(
                          p.dout + (((int64_t)b * p.S + s0 + i) * p.H + h) * D + n * 8 + 2 * tq));
      dout[n][2 * r] = v.x; dout[n][2 * r + 1] = v.y;
    }
  }
  float dl = 0.f;
  for (int m = 0; m < 2; ++m) {
    const __nv_bfloat16* sQm = sQ + m * C * LB;
    uint32_t qf[8][4];
    q_frags(qf, sQm, w, lane);
    float a[8][4];
    scores(a, qf, sK, w, lane, rows);
    float u[18][4];
    numer(u, a, qf, sV, sS, lane, has);
    float den[2];
    denom(den, a, u, lane);
    const float cm = (m == 0) ? inv : -lam * inv;
    float part[2] = {0.f, 0.f};
#pragma unroll
    for (int n = 0; n < 16; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float o = u[n][e] / den[e >> 1];
        part[e >> 1] += cm * dout[n][e] * o;
        dl += (m == 0 ? 1.f : -1.f) * dout[n][e] * o;
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      part[r] += __shfl_xor_sync(0xffffffffu, part[r], 1);
      part[r] += __shfl_xor_sync(0xffffffffu, part[r], 2);
      const int i = w * 16 + gq + 8 * r;
      const float dd = (i < rows) ? -part[r] / den[r] : 0.f;
      if (tq == 0) sdD[m * C + i] = dd;
      if (tq == 0 && i < rows) p.dD[(((int64_t)b * p.S + s0 + i) * p.H + h) * 2 + m] = dd;
      __nv_bfloat16* row_s = sdN + (m * C + i) * LB;
      __nv_bfloat16* row_g = dNb + ((((int64_t)b * p.S + s0 + i) * p.H + h) * 2 + m) * D;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        const float rd = (i < rows) ? cm / den[r] : 0.f;
        const __nv_bfloat162 v = __floats2bfloat162_rn(dout[n][2 * r] * rd, dout[n][2 * r + 1] * rd);
        *reinterpret_cast<__nv_bfloat162*>(row_s + n * 8 + 2 * tq) = v;
        if (i < rows) *reinterpret_cast<__nv_bfloat162*>(row_g + n * 8 + 2 * tq) = v;
      }
    }
  }
  __syncthreads();
  // R partial (K x D) = sum_m Pq_m^T dN_m : warp w owns K rows [32w, 32w + 32)
  {
    float acc[2][16][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int n = 0; n < 16; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[mt][n][e] = 0.f;
    for (int m = 0; m < 2; ++m) {
      const __nv_bfloat16* sQm = sQ + m * C * LB;
      const __nv_bfloat16* sdNm = sdN + m * C * LB;
#pragma unroll
      for (int ks = 0; ks < C / 16; ++ks) {
        uint32_t af[2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
          wm::ldsm_x4_t(af[mt], sQm + (ks * 16 + wm::at_row(lane)) * LB + w * 32 + mt * 16 + wm::at_col(lane));
#pragma unroll
        for (int n = 0; n < 16; n += 2) {
          uint32_t bf[4];
          wm::ldsm_x4_t(bf, sdNm + (ks * 16 + wm::bt_row(lane)) * LB + n * 8 + wm::bt_col(lane));
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {
            wm::mma16816(acc[mt][n], af[mt], bf[0], bf[1]);
            wm::mma16816(acc[mt][n + 1], af[mt], bf[2], bf[3]);
          }
        }
      }
    }
    float* R = p.R + ((((int64_t)b * p.H + h) * p.NC + c) * D) * D;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int k = w * 32 + mt * 16 + gq + 8 * r;
#pragma unroll
        for (int n = 0; n < 16; ++n)
          *reinterpret_cast<float2*>(R + k * D + n * 8 + 2 * tq) = make_float2(acc[mt][n][2 * r], acc[mt][n][2 * r + 1]);
      }
  }
  {
    const int k = threadIdx.x;   // 128 threads = K
    float accr = 0.f;
    for (int m = 0; m < 2; ++m)
      for (int i = 0; i < rows; ++i) accr += __bfloat162float(sQ[(m * C + i) * LB + k]) * sdD[m * C + i];
    p.r[(((int64_t)b * p.H + h) * p.NC + c) * D + k] = accr;
  }
  dl = warp_sum(dl);
  if (lane == 0) sRed[w] = dl;
  __syncthreads();
  if (threadIdx.x == 0) atomicAdd(p.dlam + h, (sRed[0] + sRed[1] + sRed[2] + sRed[3]) * inv * inv);
}

// Backward part 2 (per b, KV head g, chunk c): for each query head of the group and both queries,
// dq; accumulated dk, dv including the reverse-state terms.
__global__ void __launch_bounds__(NT) dqkv_kernel(Params p, const __nv_bfloat16* dNb) {
  extern __shared__ __align__(16) unsigned char smraw[];
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(smraw);
  __nv_bfloat16* sV = sK + C * LB;
  __nv_bfloat16* sQ = sV + C * LB;
  __nv_bfloat16* sdN = sQ + C * LB;
  __nv_bfloat16* sS = sdN + C * LB;       // [D][LB]  state S (no z column)
  __nv_bfloat16* sR = sS + D * LB;        // [D][LB]  reverse state
  __nv_bfloat16* sA = sR + D * LB;        // [C][LC]
  __nv_bfloat16* sdA = sA + C * LC;       // [C][LC]
  float* sdD = reinterpret_cast<float*>(sdA + C * LC);    // [C]
  float* sz = sdD + C;                                    // [D]
  float* srn = sz + D;                                    // [D]
  const int c = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int groups = p.H / p.G;
  const int s0 = c * C, rows = min(C, p.S - s0);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, gq = lane >> 2, tq = lane & 3;
  const bool has = c > 0, hasR = c + 1 < p.NC;
  load_bf<true>(sK, p.k, b, s0, rows, g, p.G, p.S);
  load_bf<false>(sV, p.v, b, s0, rows, g, p.G, p.S);
  {
    const float* S = p.st + ((((int64_t)b * p.G + g) * p.NC + c) * D) * D;
    const float* R = p.Rg + ((((int64_t)b * p.G + g) * p.NC + c) * D) * D;
    load_state_rows(sS, LB, S, has);
    load_state_rows(sR, LB, R, hasR);
    sz[threadIdx.x] = has ? p.zs[(((int64_t)b * p.G + g) * p.NC + c) * D + threadIdx.x] : 0.f;
    srn[threadIdx.x] = hasR ? p.rg[(((int64_t)b * p.G + g) * p.NC + c) * D + threadIdx.x] : 0.f;
  }
  float dk[16][4], dv[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) { dk[n][e] = 0.f; dv[n][e] = 0.f; }
  for (int hh = 0; hh < groups; ++hh) {
    const int h = g * groups + hh;
    for (int m = 0; m < 2; ++m) {
      __syncthreads();
      load_bf<true>(sQ, m == 0 ? p.q1 : p.q2, b, s0, rows, h, p.H, p.S);
      for (int i = threadIdx.x; i < C * (D / 8); i += NT) {
        const int r = i / (D / 8), col = (i % (D / 8)) * 8;
        int4 v = make_int4(0, 0, 0, 0);
        if (r < rows) v = *reinterpret_cast<const int4*>(dNb + ((((int64_t)b * p.S + s0 + r) * p.H + h) * 2 + m) * D + col);
        *reinterpret_cast<int4*>(sdN + r * LB + col) = v;
      }
      if (threadIdx.x < C)
        sdD[threadIdx.x] = threadIdx.x < rows ? p.dD[(((int64_t)b * p.S + s0 + threadIdx.x) * p.H + h) * 2 + m] : 0.f;
      __syncthreads();
      uint32_t qf[8][4];
      q_frags(qf, sQ, w, lane);
      // A (masked) -> smem
      {
        float a[8][4];
        scores(a, qf, sK, w, lane, rows);
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
          for (int r = 0; r < 2; ++r)
            *reinterpret_cast<__nv_bfloat162*>(sA + (w * 16 + gq + 8 * r) * LC + n * 8 + 2 * tq) =
                __floats2bfloat162_rn(a[n][2 * r], a[n][2 * r + 1]);
      }
      // dA = tril(dN V^T + dD) -> smem and A fragments
      uint32_t daf[4][4];
      {
        float da[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) da[n][e] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          uint32_t af[4];
          wm::ldsm_x4(af, sdN + (w * 16 + wm::a_row(lane)) * LB + kk * 16 + wm::a_col(lane));
#pragma unroll
          for (int n = 0; n < 8; n += 2) {
            uint32_t bf[4];
            wm::ldsm_x4(bf, sV + (n * 8 + wm::bn_row(lane)) * LB + kk * 16 + wm::bn_col(lane));
            wm::mma16816(da[n], af, bf[0], bf[1]);
            wm::mma16816(da[n + 1], af, bf[2], bf[3]);
          }
        }
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i = w * 16 + gq + (e >> 1) * 8, j = n * 8 + 2 * tq + (e & 1);
            da[n][e] = (j <= i && i < rows && j < rows) ? da[n][e] + sdD[i] : 0.f;
          }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          daf[j][0] = wm::pack_bf16(da[2 * j][0], da[2 * j][1]);
          daf[j][1] = wm::pack_bf16(da[2 * j][2], da[2 * j][3]);
          daf[j][2] = wm::pack_bf16(da[2 * j + 1][0], da[2 * j + 1][1]);
          daf[j][3] = wm::pack_bf16(da[2 * j + 1][2], da[2 * j + 1][3]);
        }
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
          for (int r = 0; r < 2; ++r)
            *reinterpret_cast<__nv_bfloat162*>(sdA + (w * 16 + gq + 8 * r) * LC + n * 8 + 2 * tq) =
                __floats2bfloat162_rn(da[n][2 * r], da[n][2 * r + 1]);
      }
      // dPq = dA Pk + dN S^T + dD z  ->  dq
      {
        float dq[16][4];
#pragma unroll
        for (int n = 0; n < 16; ++n)
#pragma unroll
          for (int e = 0; e < 4; ++e) dq[n][e] = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int n = 0; n < 16; n += 2) {
            uint32_t bf[4];
            wm::ldsm_x4_t(bf, sK + (j * 16 + wm::bt_row(lane)) * LB + n * 8 + wm::bt_col(lane));
            wm::mma16816(dq[n], daf[j], bf[0], bf[1]);
            wm::mma16816(dq[n + 1], daf[j], bf[2], bf[3]);
          }
        if (has) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            uint32_t af[4];
            wm::ldsm_x4(af, sdN + (w * 16 + wm::a_row(lane)) * LB + kk * 16 + wm::a_col(lane));
#pragma unroll
            for (int n = 0; n < 16; n += 2) {
              uint32_t bf[4];     // B[k = d][n = K] = S[K][d]: non-transposed load of S rows
              wm::ldsm_x4(bf, sS + (n * 8 + wm::bn_row(lane)) * LB + kk * 16 + wm::bn_col(lane));
              wm::mma16816(dq[n], af, bf[0], bf[1]);
              wm::mma16816(dq[n + 1], af, bf[2], bf[3]);
            }
          }
        }
        __nv_bfloat16* dqp = (m == 0) ? p.dq1 : p.dq2;
        const __nv_bfloat16* qp = (m == 0) ? p.q1 : p.q2;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int i = w * 16 + gq + 8 * r;
          if (i >= rows) continue;
          const float ddr = sdD[i];
          const int64_t base = (((int64_t)b * p.S + s0 + i) * p.H + h) * D;
#pragma unroll
          for (int n = 0; n < 16; ++n) {
            const int col = n * 8 + 2 * tq;
            const float2 qv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(qp + base + col));
            const float v0 = (dq[n][2 * r] + ddr * sz[col]) * dphi_f(qv.x);
            const float v1 = (dq[n][2 * r + 1] + ddr * sz[col + 1]) * dphi_f(qv.y);
            *reinterpret_cast<__nv_bfloat162*>(dqp + base + col) = __floats2bfloat162_rn(v0, v1);
          }
        }
      }
      __syncthreads();
      // dPk (keys w*16..) += dA^T Pq ;  dV += A^T dN
#pragma unroll
      for (int ks = 0; ks < C / 16; ++ks) {
        uint32_t a1[4], a2[4];
        wm::ldsm_x4_t(a1, sdA + (ks * 16 + wm::at_row(lane)) * LC + w * 16 + wm::at_col(lane));
        wm::ldsm_x4_t(a2, sA + (ks * 16 + wm::at_row(lane)) * LC + w * 16 + wm::at_col(lane));
#pragma unroll
        for (int n = 0; n < 16; n += 2) {
          uint32_t bq[4], bn[4];
          wm::ldsm_x4_t(bq, sQ + (ks * 16 + wm::bt_row(lane)) * LB + n * 8 + wm::bt_col(lane));
          wm::ldsm_x4_t(bn, sdN + (ks * 16 + wm::bt_row(lane)) * LB + n * 8 + wm::bt_col(lane));
          wm::mma16816(dk[n], a1, bq[0], bq[1]);
          wm::mma16816(dk[n + 1], a1, bq[2], bq[3]);
          wm::mma16816(dv[n], a2, bn[0], bn[1]);
          wm::mma16816(dv[n + 1], a2, bn[2], bn[3]);
        }
      }
    }
  }
  // reverse-state terms: dPk += V R^T + r ;  dV += Pk R
  if (hasR) {
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t av[4], ak[4];
      wm::ldsm_x4(av, sV + (w * 16 + wm::a_row(lane)) * LB + kk * 16 + wm::a_col(lane));
      wm::ldsm_x4(ak, sK + (w * 16 + wm::a_row(lane)) * LB + kk * 16 + wm::a_col(lane));
#pragma unroll
      for (int n = 0; n < 16; n += 2) {
        uint32_t br[4], bt[4];
        wm::ldsm_x4(br, sR + (n * 8 + wm::bn_row(lane)) * LB + kk * 16 + wm::bn_col(lane));     // R^T
        wm::ldsm_x4_t(bt, sR + (kk * 16 + wm::bt_row(lane)) * LB + n * 8 + wm::bt_col(lane));   // R
        wm::mma16816(dk[n], av, br[0], br[1]);
        wm::mma16816(dk[n + 1], av, br[2], br[3]);
        wm::mma16816(dv[n], ak, bt[0], bt[1]);
        wm::mma16816(dv[n + 1], ak, bt[2], bt[3]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int j = w * 16 + gq + 8 * r;
    if (j >= rows) continue;
    const int64_t base = (((int64_t)b * p.S + s0 + j) * p.G + g) * D;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      const int col = n * 8 + 2 * tq;
      const float2 kv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p.k + base + col));
      const float k0 = (dk[n][2 * r] + srn[col]) * dphi_f(kv.x);
      const float k1 = (dk[n][2 * r + 1] + srn[col + 1]) * dphi_f(kv.y);
      *reinterpret_cast<__nv_bfloat162*>(p.dk + base + col) = __floats2bfloat162_rn(k0, k1);
      *reinterpret_cast<__nv_bfloat162*>(p.dv + base + col) = __floats2bfloat162_rn(dv[n][2 * r], dv[n][2 * r + 1]);
    }
  }
}

constexpr int fwd_smem = (3 * C * LB + D * LSX) * 2;
constexpr int dn_smem = (6 * C * LB + D * LSX) * 2 + (2 * C + NT / 32) * 4;
constexpr int dqkv_smem = (4 * C * LB + 2 * D * LB + 2 * C * LC) * 2 + (C + 2 * D) * 4;
}  // namespace tc
}  // namespace la

static void la_check(const at::Tensor& q1, const at::Tensor& q2, const at::Tensor& k, const at::Tensor& v) {
  for (const at::Tensor* t : {&q1, &q2, &k, &v})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->is_contiguous() && t->dim() == 4,
                "linear attention: contiguous bf16 (B, S, heads, head_dim) tensors");
  TORCH_CHECK(q1.sizes() == q2.sizes() && k.sizes() == v.sizes() && q1.size(0) == k.size(0) && q1.size(1) == k.size(1) &&
              q1.size(3) == k.size(3) && q1.size(2) % k.size(2) == 0, "linear attention: shapes");
}

template <typename F>
static void la_dispatch(int K, int HD, F&& f) {
  if (K == 128 && HD == 128) f(std::integral_constant<int, 128>{}, std::integral_constant<int, 128>{});
  else if (K == 64 && HD == 128) f(std::integral_constant<int, 64>{}, std::integral_constant<int, 128>{});
  else if (K == 64 && HD == 64) f(std::integral_constant<int, 64>{}, std::integral_constant<int, 64>{});
  else TORCH_CHECK(false, "linear attention: (kernel_dim, head_dim) must be (128,128), (64,128) or (64,64)");
}

static la::Params la_params(const at::Tensor& q1, const at::Tensor& q2, const at::Tensor& k, const at::Tensor& v,
                            const at::Tensor& lam32, const at::Tensor& Sst, const at::Tensor& zst) {
  la::Params p{};
  p.q1 = (const __nv_bfloat16*)q1.data_ptr();
  p.q2 = (const __nv_bfloat16*)q2.data_ptr();
  p.k = (const __nv_bfloat16*)k.data_ptr();
  p.v = (const __nv_bfloat16*)v.data_ptr();
  p.lam = lam32.data_ptr<float>();
  p.st = Sst.data_ptr<float>();
  p.zs = zst.data_ptr<float>();
  p.B = q1.size(0); p.S = q1.size(1); p.H = q1.size(2); p.G = k.size(2);
  p.NC = (p.S + la::C - 1) / la::C;
  return p;
}

// returns (out, S_states, z_states); the states are kept for the backward pass
std::vector<at::Tensor> linear_attn_fwd(at::Tensor q1, at::Tensor q2, at::Tensor k, at::Tensor v, at::Tensor lam,
                                        int64_t kernel_dim) {
  c10::cuda::CUDAGuard guard(q1.device());
  la_check(q1, q2, k, v);
  const int B = q1.size(0), S = q1.size(1), H = q1.size(2), HD = q1.size(3), G = k.size(2), K = kernel_dim;
  const int NC = (S + la::C - 1) / la::C;
  auto f32 = q1.options().dtype(at::kFloat);
  auto out = at::empty_like(q1);
  auto Sst = at::empty({B, G, NC, K, HD}, f32);
  auto zst = at::empty({B, G, NC, K}, f32);
  auto lam32 = lam.to(at::kFloat).contiguous();
  la::Params p = la_params(q1, q2, k, v, lam32, Sst, zst);
  p.out = (__nv_bfloat16*)out.data_ptr();
  if (K == 128 && HD == 128) {
    la::run_states<128, 128>(p);
    la::set_smem(la::tc::fwd_kernel, la::tc::fwd_smem);
    la::tc::fwd_kernel<<<dim3(NC, H, B), la::tc::NT, la::tc::fwd_smem, stream()>>>(p);
    MAMF_LAUNCH_CHECK();
    return {out, Sst, zst};
  }
  la_dispatch(K, HD, [&](auto kc, auto hc) {
    constexpr int KK = decltype(kc)::value, HH = decltype(hc)::value;
    la::run_states<KK, HH>(p);
    constexpr int sm = la::fwd_smem<KK, HH>();
    la::set_smem(la::la_fwd_kernel<KK, HH>, sm);
    la::la_fwd_kernel<KK, HH><<<dim3(NC, H, B), la::NT, sm, stream()>>>(p);
    MAMF_LAUNCH_CHECK();
  });
  return {out, Sst, zst};
}

// returns (dq1, dq2, dk, dv, dlam)
std::vector<at::Tensor> linear_attn_bwd(at::Tensor q1, at::Tensor q2, at::Tensor k, at::Tensor v, at::Tensor lam,
                                        int64_t kernel_dim, at::Tensor Sst, at::Tensor zst, at::Tensor dout) {
  c10::cuda::CUDAGuard guard(q1.device());
  la_check(q1, q2, k, v);
  TORCH_CHECK(dout.sizes() == q1.sizes() && dout.scalar_type() == at::kBFloat16 && dout.is_contiguous(),
              "linear attention backward: dout like q");
  const int B = q1.size(0), S = q1.size(1), H = q1.size(2), HD = q1.size(3), G = k.size(2), K = kernel_dim;
  const int NC = (S + la::C - 1) / la::C;
  auto f32 = q1.options().dtype(at::kFloat);
  auto lam32 = lam.to(at::kFloat).contiguous();
  auto dN = (K == 128 && HD == 128) ? at::empty({0}, f32) : at::empty({B, S, H, 2, HD}, f32);
  auto dD = at::empty({B, S, H, 2}, f32);
  auto Rp = at::empty({B, H, NC, K, HD}, f32);
  auto rp = at::empty({B, H, NC, K}, f32);
  auto Rg = at::empty({B, G, NC, K, HD}, f32);
  auto rg = at::empty({B, G, NC, K}, f32);
  auto dq1 = at::empty_like(q1), dq2 = at::empty_like(q2), dk = at::empty_like(k), dv = at::empty_like(v);
  auto dlam = at::zeros({H}, f32);
  la::Params p = la_params(q1, q2, k, v, lam32, Sst, zst);
  p.dout = (const __nv_bfloat16*)dout.data_ptr();
  p.dN = dN.data_ptr<float>(); p.dD = dD.data_ptr<float>();
  p.R = Rp.data_ptr<float>(); p.r = rp.data_ptr<float>();
  p.Rg = Rg.data_ptr<float>(); p.rg = rg.data_ptr<float>();
  p.dq1 = (__nv_bfloat16*)dq1.data_ptr(); p.dq2 = (__nv_bfloat16*)dq2.data_ptr();
  p.dk = (__nv_bfloat16*)dk.data_ptr(); p.dv = (__nv_bfloat16*)dv.data_ptr();
  p.dlam = dlam.data_ptr<float>();
  if (K == 128 && HD == 128) {
    auto dNb = at::empty({B, S, H, 2, HD}, q1.options());
    la::set_smem(la::tc::dn_kernel, la::tc::dn_smem);
    la::tc::dn_kernel<<<dim3(NC, H, B), la::tc::NT, la::tc::dn_smem, stream()>>>(p, (__nv_bfloat16*)dNb.data_ptr());
    MAMF_LAUNCH_CHECK();
    const int64_t eR = 128 * 128, er = 128;
    const int grp = H / G;
    la::la_prefix_kernel<<<dim3((unsigned)((eR + 255) / 256), B * G), 256, 0, stream()>>>(p.Rg, p.R, eR, NC, grp, true, G);
    la::la_prefix_kernel<<<dim3((unsigned)((er + 255) / 256), B * G), 256, 0, stream()>>>(p.rg, p.r, er, NC, grp, true, G);
    MAMF_LAUNCH_CHECK();
    la::set_smem(la::tc::dqkv_kernel, la::tc::dqkv_smem);
    la::tc::dqkv_kernel<<<dim3(NC, G, B), la::tc::NT, la::tc::dqkv_smem, stream()>>>(p, (const __nv_bfloat16*)dNb.data_ptr());
    MAMF_LAUNCH_CHECK();
    return {dq1, dq2, dk, dv, dlam};
  }
  la_dispatch(K, HD, [&](auto kc, auto hc) {
    constexpr int KK = decltype(kc)::value, HH = decltype(hc)::value;
    constexpr int sm1 = la::dn_smem<KK, HH>();
    la::set_smem(la::la_bwd_dn_kernel<KK, HH>, sm1);
    la::la_bwd_dn_kernel<KK, HH><<<dim3(NC, H, B), la::NT, sm1, stream()>>>(p);
    MAMF_LAUNCH_CHECK();
    const int64_t eR = (int64_t)KK * HH, er = KK;
    const int grp = H / G;
    la::la_prefix_kernel<<<dim3((unsigned)((eR + 255) / 256), B * G), 256, 0, stream()>>>(p.Rg, p.R, eR, NC, grp, true, G);
    la::la_prefix_kernel<<<dim3((unsigned)((er + 255) / 256), B * G), 256, 0, stream()>>>(p.rg, p.r, er, NC, grp, true, G);
    MAMF_LAUNCH_CHECK();
    constexpr int sm2 = la::dqkv_smem<KK, HH>();
    la::set_smem(la::la_bwd_dqkv_kernel<KK, HH>, sm2);
    la::la_bwd_dqkv_kernel<KK, HH><<<dim3(NC, G, B), la::NT, sm2, stream()>>>(p);
    MAMF_LAUNCH_CHECK();
  });
  return {dq1, dq2, dk, dv, dlam};
}

}  // namespace mamf
