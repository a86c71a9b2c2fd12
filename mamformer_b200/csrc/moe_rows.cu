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
__global__ void scatter_rows_kernel(T* __restrict__ dst, int64_t ld_dst, const int64_t* __restrict__ dst_idx,
                                    const T* __restrict__ src, int64_t ld_src, int k, int64_t d) {
  const int64_t q = blockIdx.x;
  const int64_t t = q / k;
  const int4* s = reinterpret_cast<const int4*>(src + t * ld_src);
  int4* o = reinterpret_cast<int4*>(dst + dst_idx[q] * ld_dst);
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
        (scalar_t*)dst.data_ptr(), dst.stride(0), dst_idx.data_ptr<int64_t>(), (const scalar_t*)src.data_ptr(),
        src.stride(0), (int)k, d);
  });
  MAMF_LAUNCH_CHECK();
}

// ---- combine: out[t] = sum_j w[q] * row(q) ---------------------------------------------------------
template <typename S, typename O>
__global__ void combine_kernel(O* __restrict__ out, PtrTable tab, int64_t ld_src, const int32_t* __restrict__ owner,
                               const int64_t* __restrict__ pos, const float* __restrict__ w, int k, int64_t d,
                               S* __restrict__ rows_out) {
  const int64_t t = blockIdx.x;
  for (int64_t c = (int64_t)threadIdx.x * 8; c < d; c += (int64_t)blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const int64_t q = t * k + j;
      const S* base = static_cast<const S*>(tab.p[owner ? owner[q] : 0]);
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

// table: up to 8 base pointers (int64) of row arrays with row stride ld_src (elements) and dtype
// `src_dtype`; owner (Q,) int32 or None (all rows in table[0]); pos (Q,) int64; w (Q,) fp32 or None.
void moe_combine(at::Tensor out, std::vector<int64_t> table, int64_t ld_src, at::ScalarType src_dtype,
                 c10::optional<at::Tensor> owner, at::Tensor pos, c10::optional<at::Tensor> w, int64_t k,
                 c10::optional<at::Tensor> rows_out) {
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
        (O*)out.data_ptr(), tab, ld_src, owner ? owner->data_ptr<int32_t>() : nullptr, pos.data_ptr<int64_t>(),
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
                                   const float* __restrict__ gate, float* __restrict__ dgate, T* __restrict__ dy,
                                   const int64_t* __restrict__ dy_idx, int k, int64_t d) {
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
      float f[8];
      Chunk<T>::load(y + (y_idx ? y_idx[q] : q) * d + c, f);
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) s += f[i] * g[i];
      part[j] += s;
      const float gw = gate[q];
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = gw * g[i];
      Chunk<T>::store(dy + (dy_idx ? dy_idx[q] : q) * d + c, o);
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
    combine_bwd_kernel<scalar_t><<<(unsigned)T, thr, 0, stream()>>>(
        (const scalar_t*)dout.data_ptr(), (const scalar_t*)y.data_ptr(), y_idx ? y_idx->data_ptr<int64_t>() : nullptr,
        gate.data_ptr<float>(), dgate.data_ptr<float>(), (scalar_t*)dy.data_ptr(),
        dy_idx ? dy_idx->data_ptr<int64_t>() : nullptr, (int)k, d);
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

}  // namespace mamf
