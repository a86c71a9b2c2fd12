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
  auto dN = at::empty({B, S, H, 2, HD}, f32);
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
