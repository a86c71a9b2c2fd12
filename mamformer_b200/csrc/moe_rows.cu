// Row movement for the routed experts: dispatch (token rows -> expert-grouped rows), combine
// (gate-weighted sum of each token's k expert rows) and its backward, on one GPU and across the
// expert-parallel group through NVLink peer memory.
//
// Reference semantics (mamformer/layers/moe.py:310-332, parallelism/expert_parallel.py:178-340):
//   out[t] = sum_j gate[t, j] * expert_{idx[t, j]}(x[t]).
// The reference gathers/scatters rows with Python loops and index ops per expert, and moves them
// across ranks with padded all_to_all_single (twice per top-k slot).  Here:
//
//   moe_scatter_rows   dst[dst_idx[q]] = src[q / k]                   (dispatch into the grouped
//                                                                       buffer, or the send stage)
//   moe_combine        out[t] = sum_j w[q] * table[owner[q]][pos[q]]  (q = t*k + j; `table` holds up
//                      to 8 row bases: this GPU's expert outputs, or every EP peer's stage, read
//                      over NVLink with plain 16-byte loads), optionally keeping the k rows
//   moe_combine_bwd    dgate[q] = <dout[t], y[q]>,  dy[dy_idx[q]] = gate[q] * dout[t]
//   ep_pull_runs       dst[run.dst + i] = table[run.src_rank][run.src + i]   (owner pulls its
//                      tokens, already expert-sorted by the sender, from every peer's stage)
//   ep_barrier         flag exchange on the symmetric-memory signal pads: each rank stores an
//                      epoch to every peer (st.release.sys) and waits for every peer's store
//                      (ld.acquire.sys) with a bounded spin; a timeout records an error code in
//                      g_mamf_comm_err and returns instead of hanging.
// No TMA and no multicast: peer memory is only read with ordinary loads.
#include "common.cuh"

namespace mamf {

constexpr int MAX_PEERS = 8;
struct PtrTable { const void* p[MAX_PEERS]; };

__device__ int g_mamf_comm_err = 0;

// ---- 16-byte row chunks ---------------------------------------------------------------------
template <typename T> struct Chunk;            // 8 elements
template <> struct Chunk<__nv_bfloat16> {
  __device__ static void load(const __nv_bfloat16* p, float* f) {
    const int4 v = *reinterpret_cast<const int4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) { const float2 t = __bfloat1622float2(h[i]); f[2 * i] = t.x; f[2 * i + 1] = t.y; }
  }
  __device__ static void store(__nv_bfloat16* p, const float* f) {
    int4 v;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    *reinterpret_cast<int4*>(p) = v;
  }
};
template <> struct Chunk<__half> {
  __device__ static void load(const __half* p, float* f) {
    const int4 v = *reinterpret_cast<const int4*>(p);
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) { const float2 t = __half22float2(h[i]); f[2 * i] = t.x; f[2 * i + 1] = t.y; }
  }
  __device__ static void store(__half* p, const float* f) {
    int4 v;
    __half2* h = reinterpret_cast<__half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    *reinterpret_cast<int4*>(p) = v;
  }
};
template <> struct Chunk<float> {
  __device__ static void load(const float* p, float* f) {
    const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
  __device__ static void store(float* p, const float* f) {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
};

static int row_threads(int64_t d) { return (int)std::min<int64_t>(256, std::max<int64_t>(32, d / 8)); }

// ---- dispatch scatter -------------------------------------------------------------------------
template <typename T>
__global__ void scatter_rows_kernel(T* __restrict__ dst, int64_t ld_dst, int64_t dst_rows,
                                    const int64_t* __restrict__ dst_idx, const T* __restrict__ src, int64_t ld_src,
                                    int k, int64_t d) {
  const int64_t q = blockIdx.x;
  const int64_t t = q / k;
  const int64_t r = dst_idx[q];
  if (!MAMF_BOUND(r >= 0 && r < dst_rows, 1101)) return;
  const int4* s = reinterpret_cast<const int4*>(src + t * ld_src);
  int4* o = reinterpret_cast<int4*>(dst + r * ld_dst);
  const int64_t nv = d * (int64_t)sizeof(T) / 16;
  for (int64_t i = threadIdx.x; i < nv; i += blockDim.x) o[i] = s[i];
}

void moe_scatter_rows(at::Tensor dst, at::Tensor dst_idx, at::Tensor src, int64_t k) {
  c10::cuda::CUDAGuard guard(src.device());
  const int64_t Q = dst_idx.numel(), d = src.size(1);
  if (Q == 0) return;
  TORCH_CHECK(dst.scalar_type() == src.scalar_type() && dst_idx.scalar_type() == at::kLong, "scatter_rows: types");
  TORCH_CHECK(src.size(0) * k == Q && dst.size(1) == d, "scatter_rows: shapes");
  TORCH_CHECK((d * src.element_size()) % 16 == 0 && aligned16(src.data_ptr()) && aligned16(dst.data_ptr()) &&
              (src.stride(0) * src.element_size()) % 16 == 0 && (dst.stride(0) * dst.element_size()) % 16 == 0,
              "scatter_rows: 16-byte aligned rows");
  MAMF_DISPATCH_FLOAT_BF16(src.scalar_type(), "scatter_rows", [&] {
    scatter_rows_kernel<scalar_t><<<(unsigned)Q, row_threads(d), 0, stream()>>>(
        (scalar_t*)dst.data_ptr(), dst.stride(0), dst.size(0), dst_idx.data_ptr<int64_t>(),
        (const scalar_t*)src.data_ptr(), src.stride(0), (int)k, d);
  });
  MAMF_LAUNCH_CHECK();
}

// ---- combine: out[t] = sum_j w[q] * row(q) ---------------------------------------------------------
template <typename S, typename O>
__global__ void combine_kernel(O* __restrict__ out, PtrTable tab, int n_tab, int64_t ld_src, int64_t src_rows,
                               const int32_t* __restrict__ owner, const int64_t* __restrict__ pos,
                               const float* __restrict__ w, int k, int64_t d, S* __restrict__ rows_out) {
  const int64_t t = blockIdx.x;
  for (int64_t c = (int64_t)threadIdx.x * 8; c < d; c += (int64_t)blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const int64_t q = t * k + j;
      const int o = owner ? owner[q] : 0;
      if (!MAMF_BOUND(o >= 0 && o < n_tab && pos[q] >= 0 && pos[q] < src_rows, 1102)) continue;
      const S* base = static_cast<const S*>(tab.p[o]);
      float f[8];
      Chunk<S>::load(base + pos[q] * ld_src + c, f);
      const float g = w ? w[q] : 1.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += g * f[i];
      if (rows_out) Chunk<S>::store(rows_out + q * d + c, f);
    }
    Chunk<O>::store(out + t * d + c, acc);
  }
}

// table: up to 8 base pointers (int64) of row arrays with row stride ld_src (elements), src_rows
// rows each and dtype `src_dtype`; owner (Q,) int32 or None (all rows in table[0]); pos (Q,)
// int64; w (Q,) fp32 or None.
void moe_combine(at::Tensor out, std::vector<int64_t> table, int64_t ld_src, int64_t src_rows,
                 at::ScalarType src_dtype, c10::optional<at::Tensor> owner, at::Tensor pos,
                 c10::optional<at::Tensor> w, int64_t k, c10::optional<at::Tensor> rows_out) {
  c10::cuda::CUDAGuard guard(out.device());
  const int64_t T = out.size(0), d = out.size(1);
  if (T == 0) return;
  TORCH_CHECK(!table.empty() && (int)table.size() <= MAX_PEERS, "combine: 1..8 row tables");
  TORCH_CHECK(out.is_contiguous() && d % 8 == 0 && pos.numel() == T * k && pos.scalar_type() == at::kLong,
              "combine: shapes");
  TORCH_CHECK(!owner || (owner->scalar_type() == at::kInt && owner->numel() == T * k), "combine: owner int32 (Q,)");
  TORCH_CHECK(!w || (w->scalar_type() == at::kFloat && w->numel() == T * k && w->is_contiguous()), "combine: w fp32 (Q,)");
  PtrTable tab{};
  for (size_t i = 0; i < table.size(); ++i) {
    tab.p[i] = reinterpret_cast<const void*>(table[i]);
    TORCH_CHECK(table[i] % 16 == 0, "combine: 16-byte aligned tables");
  }
  const int thr = row_threads(d);
  auto go = [&](auto s_tag, auto o_tag) {
    using S = decltype(s_tag);
    using O = decltype(o_tag);
    TORCH_CHECK((ld_src * (int64_t)sizeof(S)) % 16 == 0, "combine: 16-byte row stride");
    S* ro = nullptr;
    if (rows_out) {
      TORCH_CHECK(rows_out->scalar_type() == src_dtype && rows_out->is_contiguous() && rows_out->numel() == T * k * d,
                  "combine: rows_out (Q, d) of the source dtype");
      ro = (S*)rows_out->data_ptr();
    }
    combine_kernel<S, O><<<(unsigned)T, thr, 0, stream()>>>(
        (O*)out.data_ptr(), tab, (int)table.size(), ld_src, src_rows,
        owner ? owner->data_ptr<int32_t>() : nullptr, pos.data_ptr<int64_t>(),
        w ? w->data_ptr<float>() : nullptr, (int)k, d, ro);
  };
  const bool o_bf = out.scalar_type() == at::kBFloat16;
  TORCH_CHECK(o_bf || out.scalar_type() == at::kFloat, "combine: bf16 or fp32 output");
  if (src_dtype == at::kBFloat16) {
    if (o_bf) go(__nv_bfloat16{}, __nv_bfloat16{}); else go(__nv_bfloat16{}, float{});
  } else {
    TORCH_CHECK(src_dtype == at::kFloat, "combine: bf16 or fp32 rows");
    if (o_bf) go(float{}, __nv_bfloat16{}); else go(float{}, float{});
  }
  MAMF_LAUNCH_CHECK();
}

// ---- combine backward -----------------------------------------------------------------------------
constexpr int CB_MAXK = 16;
template <typename T>
__global__ void combine_bwd_kernel(const T* __restrict__ dout, const T* __restrict__ y, const int64_t* __restrict__ y_idx,
                                   int64_t y_rows, const float* __restrict__ gate, float* __restrict__ dgate,
                                   T* __restrict__ dy, const int64_t* __restrict__ dy_idx, int64_t dy_rows, int k,
                                   int64_t d) {
  __shared__ float red[32 * CB_MAXK];
  const int64_t t = blockIdx.x;
  float part[CB_MAXK];
#pragma unroll
  for (int j = 0; j < CB_MAXK; ++j) part[j] = 0.f;
  for (int64_t c = (int64_t)threadIdx.x * 8; c < d; c += (int64_t)blockDim.x * 8) {
    float g[8];
    Chunk<T>::load(dout + t * d + c, g);
#pragma unroll
    for (int j = 0; j < CB_MAXK; ++j) {
      if (j >= k) break;
      const int64_t q = t * k + j;
      const int64_t yr = y_idx ? y_idx[q] : q, dr = dy_idx ? dy_idx[q] : q;
      if (!MAMF_BOUND(yr >= 0 && yr < y_rows && dr >= 0 && dr < dy_rows, 1103)) continue;
      float f[8];
      Chunk<T>::load(y + yr * d + c, f);
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) s += f[i] * g[i];
      part[j] += s;
      const float gw = gate[q];
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = gw * g[i];
      Chunk<T>::store(dy + dr * d + c, o);
    }
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int j = 0; j < CB_MAXK; ++j) {
    if (j >= k) break;
    const float v = warp_sum(part[j]);
    if (lane == 0) red[wid * CB_MAXK + j] = v;
  }
  __syncthreads();
  if (threadIdx.x < k) {
    float s = 0.f;
    for (int w = 0; w < nw; ++w) s += red[w * CB_MAXK + threadIdx.x];
    dgate[t * k + threadIdx.x] = s;
  }
}

// Fixed top-k form (K known at compile time, the flagship's 8): a thread reads its K row indices
// and gates once, then issues the K row loads of a column chunk together before using any of
// them, so K independent 16-byte loads are in flight per thread (the generic kernel above waits
// for each routed row in turn).
template <typename T, int K>
__global__ void combine_bwd_k_kernel(const T* __restrict__ dout, const T* __restrict__ y, const int64_t* __restrict__ y_idx,
                                     int64_t y_rows, const float* __restrict__ gate, float* __restrict__ dgate,
                                     T* __restrict__ dy, const int64_t* __restrict__ dy_idx, int64_t dy_rows, int64_t d) {
  __shared__ float red[32 * K];
  const int64_t t = blockIdx.x;
  int64_t yr[K], dr[K];
  float gw[K], part[K];
  bool ok[K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    const int64_t q = t * K + j;
    yr[j] = y_idx ? y_idx[q] : q;
    dr[j] = dy_idx ? dy_idx[q] : q;
    ok[j] = MAMF_BOUND(yr[j] >= 0 && yr[j] < y_rows && dr[j] >= 0 && dr[j] < dy_rows, 1103);
    gw[j] = gate[q];
    part[j] = 0.f;
  }
  for (int64_t c = (int64_t)threadIdx.x * 8; c < d; c += (int64_t)blockDim.x * 8) {
    float g[8], f[K][8];
    Chunk<T>::load(dout + t * d + c, g);
#pragma unroll
    for (int j = 0; j < K; ++j) {
      if (ok[j]) Chunk<T>::load(y + yr[j] * d + c, f[j]);
    }
#pragma unroll
    for (int j = 0; j < K; ++j) {
      if (!ok[j]) continue;
      float sacc = 0.f, o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) { sacc = fmaf(f[j][i], g[i], sacc); o[i] = gw[j] * g[i]; }
      part[j] += sacc;
      Chunk<T>::store(dy + dr[j] * d + c, o);
    }
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int j = 0; j < K; ++j) {
    const float v = warp_sum(part[j]);
    if (lane == 0) red[wid * K + j] = v;
  }
  __syncthreads();
  if (threadIdx.x < K) {
    float sum = 0.f;
    for (int w = 0; w < nw; ++w) sum += red[w * K + threadIdx.x];
    dgate[t * K + threadIdx.x] = sum;
  }
}

// dout (T, d); y rows (indexed by y_idx[q] or q); gate (Q,) fp32 -> dgate (Q,) fp32,
// dy rows (written at dy_idx[q] or q).
void moe_combine_bwd(at::Tensor dout, at::Tensor y, c10::optional<at::Tensor> y_idx, at::Tensor gate,
                     at::Tensor dgate, at::Tensor dy, c10::optional<at::Tensor> dy_idx, int64_t k) {
  c10::cuda::CUDAGuard guard(dout.device());
  const int64_t T = dout.size(0), d = dout.size(1);
  if (T == 0) return;
  TORCH_CHECK(k >= 1 && k <= CB_MAXK, "combine_bwd: top-k up to 16");
  TORCH_CHECK(dout.is_contiguous() && y.is_contiguous() && dy.is_contiguous() && d % 8 == 0, "combine_bwd: layout");
  TORCH_CHECK(y.scalar_type() == dout.scalar_type() && dy.scalar_type() == dout.scalar_type(), "combine_bwd: dtypes");
  TORCH_CHECK(gate.scalar_type() == at::kFloat && dgate.scalar_type() == at::kFloat && gate.numel() == T * k &&
              dgate.numel() == T * k, "combine_bwd: gate / dgate fp32 (Q,)");
  const int thr = std::max(32, row_threads(d) / 32 * 32);
  MAMF_DISPATCH_FLOAT_BF16(dout.scalar_type(), "combine_bwd", [&] {
    if (k == 8) {
      combine_bwd_k_kernel<scalar_t, 8><<<(unsigned)T, thr, 0, stream()>>>(
          (const scalar_t*)dout.data_ptr(), (const scalar_t*)y.data_ptr(), y_idx ? y_idx->data_ptr<int64_t>() : nullptr,
          y.size(0), gate.data_ptr<float>(), dgate.data_ptr<float>(), (scalar_t*)dy.data_ptr(),
          dy_idx ? dy_idx->data_ptr<int64_t>() : nullptr, dy.size(0), d);
      return;
    }
    combine_bwd_kernel<scalar_t><<<(unsigned)T, thr, 0, stream()>>>(
        (const scalar_t*)dout.data_ptr(), (const scalar_t*)y.data_ptr(), y_idx ? y_idx->data_ptr<int64_t>() : nullptr,
        y.size(0), gate.data_ptr<float>(), dgate.data_ptr<float>(), (scalar_t*)dy.data_ptr(),
        dy_idx ? dy_idx->data_ptr<int64_t>() : nullptr, dy.size(0), (int)k, d);
  });
  MAMF_LAUNCH_CHECK();
}

// ---- expert-parallel pull of contiguous runs -------------------------------------------------------
constexpr int PULL_ROWS = 16;
__global__ void pull_runs_kernel(__nv_bfloat16* __restrict__ dst, int64_t ld_dst, PtrTable tab, int64_t ld_src,
                                 const int64_t* __restrict__ runs, int64_t d) {
  const int64_t* r = runs + 4 * (int64_t)blockIdx.x;
  const int64_t dst0 = r[0], src_rank = r[1], src0 = r[2], len = r[3];
  const int64_t i0 = (int64_t)blockIdx.y * PULL_ROWS;
  if (i0 >= len) return;
  const int64_t i1 = min(len, i0 + PULL_ROWS);
  const __nv_bfloat16* base = static_cast<const __nv_bfloat16*>(tab.p[src_rank]);
  const int64_t nv = d / 8;
  for (int64_t i = i0; i < i1; ++i) {
    const int4* s = reinterpret_cast<const int4*>(base + (src0 + i) * ld_src);
    int4* o = reinterpret_cast<int4*>(dst + (dst0 + i) * ld_dst);
    for (int64_t v = threadIdx.x; v < nv; v += blockDim.x) o[v] = s[v];
  }
}

// runs: (R, 4) int64 device tensor of (dst_row, src_rank, src_row, n_rows); max_len = max n_rows.
void ep_pull_runs(at::Tensor dst, std::vector<int64_t> table, int64_t ld_src, at::Tensor runs, int64_t max_len) {
  c10::cuda::CUDAGuard guard(dst.device());
  const int64_t R = runs.size(0), d = dst.size(1);
  if (R == 0 || max_len == 0) return;
  TORCH_CHECK(dst.scalar_type() == at::kBFloat16 && d % 8 == 0 && (dst.stride(0) * 2) % 16 == 0 && (ld_src * 2) % 16 == 0,
              "pull_runs: bf16 16-byte aligned rows");
  TORCH_CHECK(runs.scalar_type() == at::kLong && runs.is_contiguous() && runs.size(1) == 4, "pull_runs: runs (R, 4) int64");
  TORCH_CHECK(!table.empty() && (int)table.size() <= MAX_PEERS, "pull_runs: 1..8 peers");
  PtrTable tab{};
  for (size_t i = 0; i < table.size(); ++i) tab.p[i] = reinterpret_cast<const void*>(table[i]);
  dim3 grid((unsigned)R, (unsigned)((max_len + PULL_ROWS - 1) / PULL_ROWS));
  pull_runs_kernel<<<grid, row_threads(d), 0, stream()>>>((__nv_bfloat16*)dst.data_ptr(), dst.stride(0), tab, ld_src,
                                                          runs.data_ptr<int64_t>(), d);
  MAMF_LAUNCH_CHECK();
}

// ---- bounded signal-pad barrier -------------------------------------------------------------------
constexpr long long BARRIER_WAIT_CYCLES = 4000000000LL;   // ~2 s at 1.9 GHz

__global__ void ep_barrier_kernel(PtrTable sig, int me, int P, uint32_t epoch, int slot0) {
  const int p = threadIdx.x;
  if (p < P) {
    uint32_t* remote = static_cast<uint32_t*>(const_cast<void*>(sig.p[p])) + slot0 + me;
    __threadfence_system();
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(remote), "r"(epoch) : "memory");
    const uint32_t* mine = static_cast<const uint32_t*>(sig.p[me]) + slot0 + p;
    const long long t0 = clock64();
    while (true) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if ((int32_t)(v - epoch) >= 0) break;
      if (clock64() - t0 > BARRIER_WAIT_CYCLES) { atomicExch(&g_mamf_comm_err, 100 + p); break; }
      if (*((volatile int*)&g_mamf_comm_err) != 0) break;
      __nanosleep(64);
    }
  }
  __syncthreads();
}

// signal: per-rank signal-pad base pointers (uint32 words); the barrier uses words
// [slot0, slot0 + P) of every pad.  epoch must increase by one per call, identically on every rank.
void ep_barrier(std::vector<int64_t> signal, int64_t me, int64_t epoch, int64_t slot0) {
  const int P = (int)signal.size();
  TORCH_CHECK(P >= 1 && P <= MAX_PEERS && me >= 0 && me < P, "ep_barrier: 1..8 ranks");
  PtrTable sig{};
  for (int i = 0; i < P; ++i) sig.p[i] = reinterpret_cast<const void*>(signal[i]);
  ep_barrier_kernel<<<1, 32, 0, stream()>>>(sig, (int)me, P, (uint32_t)epoch, (int)slot0);
  MAMF_LAUNCH_CHECK();
}

int64_t comm_error() {
  int v = 0;
  MAMF_CUDA_CHECK(cudaMemcpyFromSymbol(&v, g_mamf_comm_err, sizeof(int)));
  return v;
}

void comm_clear_error() {
  int z = 0;
  MAMF_CUDA_CHECK(cudaMemcpyToSymbol(g_mamf_comm_err, &z, sizeof(int)));
}


// =================================================================================================
// Device-side routing plans (no host round trip)
//
//   moe_sort_plan   counting sort of the T*k top-k assignments by expert, stable in assignment
//                   order: per-warp histograms (shared-memory atomics) -> one block turns them into
//                   per-warp base offsets -> every warp ranks its assignments again in order with
//                   __match_any_sync.  Gives srow[q] (position in the expert-sorted order), the
//                   per-expert counts and exclusive starts, and - for the single-GPU layout - the
//                   64-aligned segment table, the GEMM tile table and pos[q] in the padded buffer.
//   ep_exchange     pushes this rank's per-expert counts into row `me` of every peer's count matrix
//                   (P2P stores into symmetric memory), then runs the bounded signal-pad barrier, so
//                   each rank holds the full (P, E) matrix locally.
//   ep_layout       one block: from the count matrix, every owner's 64-aligned segments (so each
//                   rank knows where its rows land in every owner's buffer), this rank's owner
//                   tables (segments, GEMM tiles, per-(sender, expert) offsets) and the capacity
//                   check.  A problem larger than the fixed capacity sets a status word and is
//                   clamped so that every access stays inside the buffers; the host reads the status
//                   once per optimizer step and reruns that step with a larger capacity.
//   ep_pos          pos[q] / owner[q] of every assignment in the owners' buffers (for the combine).
//   ep_pull_rows    owner side: one warp per destination row of the expert-grouped GEMM operand,
//                   read with 16-byte loads from the sender's stage over NVLink; pad rows are
//                   written as zeros (the weight-gradient GEMM contracts over them).
// =================================================================================================
constexpr int SORT_WARPS = 8;
constexpr int SORT_MAXE = 256;

__device__ int g_mamf_plan_err = 0;     // sort saw an expert id < 0 (1) or >= E (2); 0 = none

__global__ void sort_hist_kernel(const int64_t* __restrict__ idx, int64_t Q, int E, int64_t chunk,
                                 int* __restrict__ hist) {
  __shared__ int cnt[SORT_WARPS][SORT_MAXE];
  const int lw = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < SORT_WARPS * SORT_MAXE; i += blockDim.x) (&cnt[0][0])[i] = 0;
  __syncthreads();
  const int64_t w = (int64_t)blockIdx.x * SORT_WARPS + lw;
  const int64_t q0 = w * chunk, q1 = min(Q, q0 + chunk);
  for (int64_t q = q0 + lane; q < q1; q += 32) {
    const int64_t e = idx[q];
    if (e < 0 || e >= E) { atomicCAS(&g_mamf_plan_err, 0, e < 0 ? 1 : 2); continue; }
    atomicAdd(&cnt[lw][e], 1);
  }
  __syncwarp();
  for (int e = lane; e < E; e += 32) hist[w * E + e] = cnt[lw][e];
}

// hist (W, E): per-warp counts in, per-warp base offsets out.  counts (E), start (E+1).
// seg / tile_off (E+1) are written when non-null (single-GPU padded layout, 128-row GEMM tiles).
__global__ void sort_scan_kernel(int* __restrict__ hist, int W, int E, int* __restrict__ counts,
                                 int* __restrict__ start, int* __restrict__ seg, int* __restrict__ tile_off) {
  __shared__ int tot[SORT_MAXE];
  __shared__ int st[SORT_MAXE + 1];
  const int e = threadIdx.x;
  if (e < E) {
    int run = 0;
    for (int w = 0; w < W; ++w) {
      const int c = hist[(int64_t)w * E + e];
      hist[(int64_t)w * E + e] = run;
      run += c;
    }
    tot[e] = run;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int s = 0, sp = 0, sT = 0;
    for (int i = 0; i < E; ++i) {
      st[i] = s;
      start[i] = s;
      counts[i] = tot[i];
      if (seg) { seg[i] = sp; tile_off[i] = sT; }
      const int pad = (tot[i] + 63) / 64 * 64;
      s += tot[i];
      sp += pad;
      sT += (pad + 127) / 128;
    }
    st[E] = s;
    start[E] = s;
    if (seg) { seg[E] = sp; tile_off[E] = sT; }
  }
  __syncthreads();
  if (e < E) {
    const int b = st[e];
    for (int w = 0; w < W; ++w) hist[(int64_t)w * E + e] += b;
  }
}

// srow[q]: stable position of assignment q in the expert-sorted order.  pos[q] (optional):
// seg[e] + rank of q inside expert e (single-GPU padded layout).
__global__ void sort_rank_kernel(const int64_t* __restrict__ idx, int64_t Q, int E, int64_t chunk,
                                 const int* __restrict__ base, const int* __restrict__ start,
                                 const int* __restrict__ seg, int64_t* __restrict__ srow,
                                 int64_t* __restrict__ pos) {
  __shared__ int cnt[SORT_WARPS][SORT_MAXE];
  const int lw = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t w = (int64_t)blockIdx.x * SORT_WARPS + lw;
  for (int e = lane; e < E; e += 32) cnt[lw][e] = base[w * E + e];
  __syncwarp();
  const int64_t q0 = w * chunk, q1 = min(Q, q0 + chunk);
  for (int64_t b0 = q0; b0 < q1; b0 += 32) {
    const int64_t q = b0 + lane;
    int e = q < q1 ? (int)idx[q] : -1;
    if (e < 0 || e >= E) e = -1 - lane;              // unmatched key: the lane takes no part
    const unsigned mask = __match_any_sync(0xffffffffu, e);
    const int r = __popc(mask & ((1u << lane) - 1u));
    const int b = e >= 0 ? cnt[lw][e] : 0;
    __syncwarp();
    if (e >= 0) {
      const int row = b + r;
      srow[q] = row;
      if (pos) pos[q] = (int64_t)seg[e] + (row - start[e]);
      if (r == 0) cnt[lw][e] = b + __popc(mask);
    } else if (q < q1) {
      srow[q] = 0;                                   // bad id (recorded by the histogram pass):
      if (pos) pos[q] = 0;                           // keep every later access in bounds
    }
    __syncwarp();
  }
}

// idx (Q,) int64 expert ids -> srow (Q,) int64, counts (E,) int32, start (E+1) int32 and, with
// `padded`, seg (E+1) int32, tile_off (E+1) int32, pos (Q,) int64.
std::vector<at::Tensor> moe_sort_plan(at::Tensor idx, int64_t E, bool padded) {
  c10::cuda::CUDAGuard guard(idx.device());
  TORCH_CHECK(idx.is_cuda() && idx.scalar_type() == at::kLong, "moe_sort_plan: int64 CUDA expert ids");
  TORCH_CHECK(E >= 1 && E <= SORT_MAXE, "moe_sort_plan: 1 <= E <= 256");
  auto ic = idx.contiguous().view({-1});
  const int64_t Q = ic.numel();
  auto i32 = idx.options().dtype(at::kInt);
  const int64_t want_warps = std::max<int64_t>(1, std::min<int64_t>(1024, (Q + 255) / 256));
  const int64_t blocks = (want_warps + SORT_WARPS - 1) / SORT_WARPS;
  const int64_t W = blocks * SORT_WARPS;
  const int64_t chunk = std::max<int64_t>(1, (Q + W - 1) / W);
  auto hist = at::empty({W, E}, i32);
  auto counts = at::empty({E}, i32);
  auto start = at::empty({E + 1}, i32);
  auto srow = at::empty({Q}, idx.options());
  at::Tensor seg, tile_off, pos;
  if (padded) {
    seg = at::empty({E + 1}, i32);
    tile_off = at::empty({E + 1}, i32);
    pos = at::empty({Q}, idx.options());
  }
  sort_hist_kernel<<<(unsigned)blocks, SORT_WARPS * 32, 0, stream()>>>(ic.data_ptr<int64_t>(), Q, (int)E, chunk,
                                                                       hist.data_ptr<int>());
  MAMF_LAUNCH_CHECK();
  sort_scan_kernel<<<1, SORT_MAXE, 0, stream()>>>(hist.data_ptr<int>(), (int)W, (int)E, counts.data_ptr<int>(),
                                                   start.data_ptr<int>(), padded ? seg.data_ptr<int>() : nullptr,
                                                   padded ? tile_off.data_ptr<int>() : nullptr);
  MAMF_LAUNCH_CHECK();
  sort_rank_kernel<<<(unsigned)blocks, SORT_WARPS * 32, 0, stream()>>>(
      ic.data_ptr<int64_t>(), Q, (int)E, chunk, hist.data_ptr<int>(), start.data_ptr<int>(),
      padded ? seg.data_ptr<int>() : nullptr, srow.data_ptr<int64_t>(), padded ? pos.data_ptr<int64_t>() : nullptr);
  MAMF_LAUNCH_CHECK();
  if (padded) return {srow, counts, start, seg, tile_off, pos};
  return {srow, counts, start};
}

int64_t plan_error() {
  int v = 0;
  MAMF_CUDA_CHECK(cudaMemcpyFromSymbol(&v, g_mamf_plan_err, sizeof(int)));
  if (v) {
    int z = 0;
    MAMF_CUDA_CHECK(cudaMemcpyToSymbol(g_mamf_plan_err, &z, sizeof(int)));
  }
  return v;
}

// ---- expert parallelism: count exchange, layout, positions, row pull -----------------------------
constexpr int EP_MAXP = MAX_PEERS;

__device__ __forceinline__ void signal_wait_all(PtrTable sig, int me, int P, uint32_t epoch, int slot0) {
  const int p = threadIdx.x;
  if (p < P) {
    uint32_t* remote = static_cast<uint32_t*>(const_cast<void*>(sig.p[p])) + slot0 + me;
    __threadfence_system();
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(remote), "r"(epoch) : "memory");
    const uint32_t* mine = static_cast<const uint32_t*>(sig.p[me]) + slot0 + p;
    const long long t0 = clock64();
    while (true) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if ((int32_t)(v - epoch) >= 0) break;
      if (clock64() - t0 > BARRIER_WAIT_CYCLES) { atomicExch(&g_mamf_comm_err, 100 + p); break; }
      if (*((volatile int*)&g_mamf_comm_err) != 0) break;
      __nanosleep(64);
    }
  }
  __syncthreads();
}

// Push counts into row `me` of every peer's (P, E) matrix, then the barrier.
__global__ void ep_exchange_kernel(PtrTable mats, PtrTable sig, const int* __restrict__ counts, int me, int P, int E,
                                   uint32_t epoch, int slot0) {
  for (int i = threadIdx.x; i < P * E; i += blockDim.x) {
    const int p = i / E, e = i - p * E;
    static_cast<int*>(const_cast<void*>(mats.p[p]))[me * E + e] = counts[e];
  }
  __syncthreads();
  signal_wait_all(sig, me, P, epoch, slot0);
}

void ep_exchange_counts(std::vector<int64_t> mats, std::vector<int64_t> signal, at::Tensor counts, int64_t me,
                        int64_t epoch, int64_t slot0) {
  c10::cuda::CUDAGuard guard(counts.device());
  const int P = (int)mats.size();
  TORCH_CHECK(P >= 1 && P <= EP_MAXP && (int)signal.size() == P && me >= 0 && me < P, "ep_exchange: 1..8 ranks");
  TORCH_CHECK(counts.scalar_type() == at::kInt && counts.is_contiguous(), "ep_exchange: int32 counts");
  PtrTable m{}, sg{};
  for (int i = 0; i < P; ++i) {
    m.p[i] = reinterpret_cast<const void*>(mats[i]);
    sg.p[i] = reinterpret_cast<const void*>(signal[i]);
  }
  ep_exchange_kernel<<<1, 256, 0, stream()>>>(m, sg, counts.data_ptr<int>(), (int)me, P, (int)counts.numel(),
                                              (uint32_t)epoch, (int)slot0);
  MAMF_LAUNCH_CHECK();
}

// Plan buffer (int32) of one EP layer, offsets for El local experts, P ranks, E = P * El:
//   [0, El]            seg   (this rank's 64-aligned expert segments; seg[El] = rows used)
//   [El+1, 2El+1]      tile  (cumulative 128-row GEMM tiles)
//   [2El+2, 3El+1]     tot   (rows per local expert, all senders)
//   next P*El          before[s][le]  rows of senders < s for local expert le
//   next P*El          src[s][le]     first row of expert me*El+le in sender s's sorted stage
//   next E             base[e]        where this rank's rows of expert e start in its owner's buffer
struct PlanOff {
  int seg, tile, tot, before, src, base, total;
  __host__ __device__ PlanOff(int P, int El) {
    seg = 0; tile = El + 1; tot = 2 * El + 2; before = 3 * El + 2; src = before + P * El; base = src + P * El;
    total = base + P * El;
  }
};

// status[0]: 1 if some owner needs more rows than `cap`;  status[1]: max rows any owner needs.
__global__ void ep_layout_kernel(const int* __restrict__ C, int P, int El, int me, int cap, int* __restrict__ plan,
                                 int* __restrict__ status) {
  const int E = P * El;
  const PlanOff o(P, El);
  __shared__ int tot[SORT_MAXE];
  __shared__ int segall[EP_MAXP][SORT_MAXE + 1];
  const int e = threadIdx.x;
  if (e < E) {
    int t = 0;
    for (int s = 0; s < P; ++s) t += C[s * E + e];
    tot[e] = t;
  }
  __syncthreads();
  if (threadIdx.x < P) {                          // owner r = threadIdx.x: its segments
    const int r = threadIdx.x;
    int sp = 0;
    for (int le = 0; le < El; ++le) { segall[r][le] = sp; sp += (tot[r * El + le] + 63) / 64 * 64; }
    segall[r][El] = sp;
    if (sp > cap) atomicExch(status, 1);
    atomicMax(status + 1, sp);
  }
  __syncthreads();
  if (e < E) {
    // this rank as a sender: rows of expert e start at owner segment + rows of lower senders
    const int r = e / El, le = e - r * El;
    int before_me = 0;
    for (int s = 0; s < me; ++s) before_me += C[s * E + e];
    plan[o.base + e] = segall[r][le] + before_me;
  }
  if (e < El) {                                   // this rank as owner
    const int ge = me * El + e;
    const int t = tot[ge];
    plan[o.tot + e] = t;
    int run = 0;
    for (int s = 0; s < P; ++s) {
      plan[o.before + s * El + e] = run;
      run += C[s * E + ge];
      int sstart = 0;                             // sender s's sorted start of expert ge
      for (int x = 0; x < ge; ++x) sstart += C[s * E + x];
      plan[o.src + s * El + e] = sstart;
    }
  }
  if (threadIdx.x == 0) {
    int tiles = 0;
    for (int le = 0; le <= El; ++le) {
      const int sg = min(segall[me][le], cap);   // clamped: an overflowing step is discarded
      plan[o.seg + le] = sg;
      plan[o.tile + le] = tiles;
      if (le < El) tiles += (min(segall[me][le + 1], cap) - sg + 127) / 128;
    }
  }
}

// C (P, E) int32 (this rank's copy after the exchange) -> plan (int32, PlanOff(P, El).total).
void ep_layout(at::Tensor C, int64_t me, int64_t cap, at::Tensor plan, at::Tensor status) {
  c10::cuda::CUDAGuard guard(C.device());
  const int P = (int)C.size(0), E = (int)C.size(1);
  TORCH_CHECK(P >= 1 && P <= EP_MAXP && E % P == 0 && E <= SORT_MAXE && C.scalar_type() == at::kInt, "ep_layout: C");
  const int El = E / P;
  TORCH_CHECK(plan.scalar_type() == at::kInt && plan.numel() >= PlanOff(P, El).total, "ep_layout: plan buffer");
  TORCH_CHECK(status.scalar_type() == at::kInt && status.numel() >= 2, "ep_layout: status");
  TORCH_CHECK(cap > 0 && cap < (1LL << 30), "ep_layout: capacity");
  ep_layout_kernel<<<1, SORT_MAXE, 0, stream()>>>(C.data_ptr<int>(), P, El, (int)me, (int)cap, plan.data_ptr<int>(),
                                                  status.data_ptr<int>());
  MAMF_LAUNCH_CHECK();
}

// pos[q] = base[e] + srow[q] - start[e] (clamped into the owner's capacity), owner[q] = e / El.
__global__ void ep_pos_kernel(const int64_t* __restrict__ idx, const int64_t* __restrict__ srow,
                              const int* __restrict__ start, const int* __restrict__ base, int64_t Q, int El, int E,
                              int cap, int64_t* __restrict__ pos, int32_t* __restrict__ owner) {
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < Q; q += (int64_t)gridDim.x * blockDim.x) {
    int64_t e = idx[q];
    if (e < 0 || e >= E) e = 0;
    const int64_t p = (int64_t)base[e] + srow[q] - start[e];
    pos[q] = p < 0 ? 0 : (p >= cap ? (int64_t)cap - 1 : p);
    owner[q] = (int32_t)(e / El);
  }
}

void ep_positions(at::Tensor idx, at::Tensor srow, at::Tensor start, at::Tensor plan, int64_t P, int64_t cap,
                  at::Tensor pos, at::Tensor owner) {
  c10::cuda::CUDAGuard guard(idx.device());
  const int64_t Q = idx.numel();
  const int E = (int)start.numel() - 1, El = E / (int)P;
  if (Q == 0) return;
  TORCH_CHECK(idx.is_contiguous() && srow.numel() == Q && pos.numel() == Q && owner.numel() == Q &&
              owner.scalar_type() == at::kInt && pos.scalar_type() == at::kLong, "ep_positions: shapes");
  const PlanOff o((int)P, El);
  ep_pos_kernel<<<(unsigned)std::min<int64_t>((Q + 255) / 256, 4 * num_sms()), 256, 0, stream()>>>(
      idx.data_ptr<int64_t>(), srow.data_ptr<int64_t>(), start.data_ptr<int>(), plan.data_ptr<int>() + o.base, Q, El,
      E, (int)cap, pos.data_ptr<int64_t>(), owner.data_ptr<int32_t>());
  MAMF_LAUNCH_CHECK();
}

// Owner pull: dst rows [0, seg[El]) of the expert-grouped operand, one warp per row.
__global__ void ep_pull_rows_kernel(__nv_bfloat16* __restrict__ dst, int64_t ld_dst, int64_t dst_rows, PtrTable tab,
                                    int64_t ld_src, int64_t src_rows, const int* __restrict__ plan, int P, int El,
                                    int64_t d) {
  const PlanOff o(P, El);
  __shared__ int seg[SORT_MAXE + 1], tot[SORT_MAXE], before[SORT_MAXE], src[SORT_MAXE];
  for (int i = threadIdx.x; i <= El; i += blockDim.x) seg[i] = plan[o.seg + i];
  for (int i = threadIdx.x; i < El; i += blockDim.x) tot[i] = plan[o.tot + i];
  for (int i = threadIdx.x; i < P * El; i += blockDim.x) { before[i] = plan[o.before + i]; src[i] = plan[o.src + i]; }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t rows = (int64_t)seg[El] < dst_rows ? (int64_t)seg[El] : dst_rows;
  const int64_t nv = d / 8;
  for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < rows; i += warps) {
    int lo = 0, hi = El;
    while (hi - lo > 1) { const int mid = (lo + hi) >> 1; if (seg[mid] <= i) lo = mid; else hi = mid; }
    const int le = lo, j = (int)i - seg[le];
    int4* out = reinterpret_cast<int4*>(dst + i * ld_dst);
    if (j >= tot[le]) {
      for (int64_t v = lane; v < nv; v += 32) out[v] = make_int4(0, 0, 0, 0);
      continue;
    }
    int s = 0;
    while (s + 1 < P && before[(s + 1) * El + le] <= j) ++s;
    const int64_t row = (int64_t)src[s * El + le] + (j - before[s * El + le]);
    if (!MAMF_BOUND(row >= 0 && row < src_rows, 1104)) continue;
    const int4* in = reinterpret_cast<const int4*>(static_cast<const __nv_bfloat16*>(tab.p[s]) + row * ld_src);
    for (int64_t v = lane; v < nv; v += 32) out[v] = in[v];
  }
}

// dst (>= seg[El] rows, bf16); table: every rank's stage base (row stride ld_src, src_rows rows);
// plan from ep_layout.
void ep_pull_rows(at::Tensor dst, std::vector<int64_t> table, int64_t ld_src, int64_t src_rows, at::Tensor plan,
                  int64_t P) {
  c10::cuda::CUDAGuard guard(dst.device());
  const int64_t d = dst.size(1);
  TORCH_CHECK(dst.scalar_type() == at::kBFloat16 && d % 8 == 0 && (dst.stride(0) * 2) % 16 == 0 && (ld_src * 2) % 16 == 0,
              "ep_pull_rows: bf16 16-byte aligned rows");
  TORCH_CHECK((int)table.size() == P && P >= 1 && P <= EP_MAXP, "ep_pull_rows: 1..8 peers");
  TORCH_CHECK(plan.scalar_type() == at::kInt && plan.is_contiguous(), "ep_pull_rows: int32 plan");
  PtrTable tab{};
  for (int i = 0; i < (int)P; ++i) tab.p[i] = reinterpret_cast<const void*>(table[i]);
  const int el = (int)((plan.numel() - 2) / (3 + 3 * P));      // total = 3*El + 2 + 3*P*El
  TORCH_CHECK(el >= 1 && PlanOff((int)P, el).total == plan.numel(), "ep_pull_rows: plan size");
  ep_pull_rows_kernel<<<4 * num_sms(), 256, 0, stream()>>>((__nv_bfloat16*)dst.data_ptr(), dst.stride(0), dst.size(0),
                                                           tab, ld_src, src_rows, plan.data_ptr<int>(), (int)P, el, d);
  MAMF_LAUNCH_CHECK();
}

int64_t ep_plan_size(int64_t P, int64_t El) { return PlanOff((int)P, (int)El).total; }

// ---- zero the pad rows of an expert-grouped buffer ------------------------------------------------
// Rows [seg[e] + counts[e], seg[e + 1]) of every expert segment: the grouped weight-gradient GEMM
// contracts over whole 64-row segments, so they must hold zeros; all other rows are written by
// the dispatch (so the buffer itself can start uninitialised).
__global__ void zero_pad_rows_kernel(__nv_bfloat16* __restrict__ buf, int64_t ld, int64_t rows,
                                     const int* __restrict__ seg, const int* __restrict__ counts, int64_t d) {
  const int e = blockIdx.x;
  const int64_t r0 = (int64_t)seg[e] + counts[e], r1 = seg[e + 1];
  const int64_t nv = d / 8;
  for (int64_t r = r0 + threadIdx.y; r < r1; r += blockDim.y) {
    if (!MAMF_BOUND(r >= 0 && r < rows, 1105)) continue;
    int4* o = reinterpret_cast<int4*>(buf + r * ld);
    for (int64_t v = threadIdx.x; v < nv; v += blockDim.x) o[v] = make_int4(0, 0, 0, 0);
  }
}

// buf (rows, d) bf16; seg (E+1) int32 64-aligned offsets; counts (E) int32 rows per expert.
void moe_zero_pad_rows(at::Tensor buf, at::Tensor seg, at::Tensor counts) {
  c10::cuda::CUDAGuard guard(buf.device());
  const int64_t E = counts.numel(), d = buf.size(1);
  if (E == 0) return;
  TORCH_CHECK(buf.scalar_type() == at::kBFloat16 && d % 8 == 0 && (buf.stride(0) * 2) % 16 == 0 &&
              aligned16(buf.data_ptr()), "zero_pad_rows: bf16 16-byte aligned rows");
  TORCH_CHECK(seg.scalar_type() == at::kInt && counts.scalar_type() == at::kInt && seg.numel() == E + 1,
              "zero_pad_rows: int32 seg (E+1) and counts (E)");
  zero_pad_rows_kernel<<<(unsigned)E, dim3(32, 8), 0, stream()>>>((__nv_bfloat16*)buf.data_ptr(), buf.stride(0),
                                                                  buf.size(0), seg.data_ptr<int>(),
                                                                  counts.data_ptr<int>(), d);
  MAMF_LAUNCH_CHECK();
}

MAMF_BOUNDS_READER(bounds_error_moe_rows)
bool bounds_check_built() { return MAMF_BOUNDS_BUILT != 0; }

}  // namespace mamf
