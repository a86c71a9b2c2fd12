// MoE router: top-k selection, softmax over the selected scores and the expert histogram in one
// warp-per-token kernel, and the matching backward.
//
// Reference semantics (mamformer/layers/moe.py:163-183, st_moe.py:179-219):
//   vals, idx = topk(scores, k) (descending);  gates = softmax(vals)
// Ties are broken towards the lower expert index.  The histogram (counts per expert, used by the
// aux-loss-free bias update and load statistics) is accumulated with one atomic per selection,
// so no host synchronisation is needed (torch.bincount on CUDA reads the maximum back to the host).
// Backward: d scores[t, idx[t, j]] = g_j (dg_j - sum_i g_i dg_i); every other entry is 0.
#include "common.cuh"

namespace mamf {

constexpr int RT_MAXE = 8;    // experts per lane (E <= 256)
constexpr int RT_MAXK = 16;

__global__ void router_topk_kernel(const float* __restrict__ scores, int64_t T, int E, int k,
                                   float* __restrict__ gates, int64_t* __restrict__ idx, int* __restrict__ counts) {
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float v[RT_MAXE];
#pragma unroll
  for (int i = 0; i < RT_MAXE; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? scores[t * E + e] : -INFINITY;
  }
  float top_v[RT_MAXK];
  int top_i[RT_MAXK];
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < RT_MAXE; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (v[i] > bv || (v[i] == bv && e < bi))) { bv = v[i]; bi = e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    top_v[j] = bv;
    top_i[j] = bi;
    if ((bi & 31) == lane) {
#pragma unroll
      for (int i = 0; i < RT_MAXE; ++i)
        if (lane + 32 * i == bi) v[i] = -INFINITY;
    }
  }
  if (lane == 0) {
    const float m = top_v[0];
    float s = 0.f;
    for (int j = 0; j < k; ++j) s += __expf(top_v[j] - m);
    const float inv = 1.f / s;
    for (int j = 0; j < k; ++j) {
      gates[t * k + j] = __expf(top_v[j] - m) * inv;
      idx[t * k + j] = top_i[j];
      if (counts) atomicAdd(counts + top_i[j], 1);
    }
  }
}

__global__ void router_topk_bwd_kernel(const float* __restrict__ dg, const float* __restrict__ gates,
                                       const int64_t* __restrict__ idx, int64_t T, int E, int k,
                                       float* __restrict__ dscores) {
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float dot = 0.f;
  for (int j = 0; j < k; ++j) dot += gates[t * k + j] * dg[t * k + j];
  for (int e = lane; e < E; e += 32) {
    float val = 0.f;
    for (int j = 0; j < k; ++j)
      if (idx[t * k + j] == e) val = gates[t * k + j] * (dg[t * k + j] - dot);
    dscores[t * E + e] = val;
  }
}

// scores (T, E) fp32 -> (gates (T, k) fp32, idx (T, k) int64, counts (E,) int32)
std::vector<at::Tensor> router_topk(at::Tensor scores, int64_t k) {
  c10::cuda::CUDAGuard guard(scores.device());
  TORCH_CHECK(scores.is_cuda() && scores.scalar_type() == at::kFloat && scores.dim() == 2 && scores.is_contiguous(),
              "router_topk: contiguous fp32 (T, E) scores");
  const int64_t T = scores.size(0);
  const int E = scores.size(1);
  TORCH_CHECK(E <= 32 * RT_MAXE && k >= 1 && k <= RT_MAXK && k <= E, "router_topk: E <= 256, 1 <= k <= 16");
  auto gates = at::empty({T, k}, scores.options());
  auto idx = at::empty({T, k}, scores.options().dtype(at::kLong));
  auto counts = at::zeros({E}, scores.options().dtype(at::kInt));
  if (T > 0) {
    const int wpb = 8;
    router_topk_kernel<<<(unsigned)((T + wpb - 1) / wpb), wpb * 32, 0, stream()>>>(
        scores.data_ptr<float>(), T, E, (int)k, gates.data_ptr<float>(), idx.data_ptr<int64_t>(), counts.data_ptr<int>());
    MAMF_LAUNCH_CHECK();
  }
  return {gates, idx, counts};
}

at::Tensor router_topk_bwd(at::Tensor dg, at::Tensor gates, at::Tensor idx, int64_t E) {
  c10::cuda::CUDAGuard guard(dg.device());
  const int64_t T = gates.size(0), k = gates.size(1);
  auto dgc = dg.to(at::kFloat).contiguous();
  auto out = at::empty({T, E}, gates.options());
  if (T > 0) {
    const int wpb = 8;
    router_topk_bwd_kernel<<<(unsigned)((T + wpb - 1) / wpb), wpb * 32, 0, stream()>>>(
        dgc.data_ptr<float>(), gates.data_ptr<float>(), idx.data_ptr<int64_t>(), T, (int)E, (int)k, out.data_ptr<float>());
    MAMF_LAUNCH_CHECK();
  }
  return out;
}

__global__ void histogram_kernel(const int64_t* __restrict__ idx, int64_t n, int E, int* __restrict__ counts) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = idx[i];
    if (e >= 0 && e < E) atomicAdd(counts + e, 1);
  }
}

at::Tensor expert_histogram(at::Tensor idx, int64_t E) {
  c10::cuda::CUDAGuard guard(idx.device());
  auto ic = idx.to(at::kLong).contiguous();
  auto counts = at::zeros({E}, idx.options().dtype(at::kInt));
  const int64_t n = ic.numel();
  if (n > 0) {
    histogram_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 1184), 256, 0, stream()>>>(
        ic.data_ptr<int64_t>(), n, (int)E, counts.data_ptr<int>());
    MAMF_LAUNCH_CHECK();
  }
  return counts.to(at::kLong);
}


// ---- aux-loss-free expert-bias update ---------------------------------------------------------
// Reference moe.py:335-347 (and the DeepSeekMoE forward):  load = counts / (tokens * k + 1e-8),
// bias -= speed * sign(load - 1/E),  ema = 0.99 * ema + 0.01 * load.  Each product and sum is
// rounded separately (no FMA contraction) so the result matches the eager float32 ops bit for bit.
__global__ void bias_update_kernel(const int64_t* __restrict__ counts, int E, float denom, float inv_e, float speed,
                                   float* __restrict__ bias, float* __restrict__ ema) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= E) return;
  const float load = __fdiv_rn((float)counts[e], denom);
  const float dlt = __fsub_rn(load, inv_e);
  const float sg = dlt > 0.f ? 1.f : (dlt < 0.f ? -1.f : 0.f);
  bias[e] = __fsub_rn(bias[e], __fmul_rn(speed, sg));
  ema[e] = __fadd_rn(__fmul_rn(ema[e], 0.99f), __fmul_rn(0.01f, load));
}

void moe_bias_update(at::Tensor counts, double n_assign, int64_t E, double speed, at::Tensor bias, at::Tensor ema) {
  c10::cuda::CUDAGuard guard(counts.device());
  TORCH_CHECK(counts.scalar_type() == at::kLong && counts.numel() == E && counts.is_contiguous(), "bias_update: counts");
  TORCH_CHECK(bias.scalar_type() == at::kFloat && ema.scalar_type() == at::kFloat && bias.numel() == E &&
              ema.numel() == E && bias.is_contiguous() && ema.is_contiguous(), "bias_update: fp32 bias / ema");
  bias_update_kernel<<<(unsigned)((E + 127) / 128), 128, 0, stream()>>>(
      counts.data_ptr<int64_t>(), (int)E, (float)(n_assign + 1e-8), (float)(1.0 / (double)E), (float)speed,
      bias.data_ptr<float>(), ema.data_ptr<float>());
  MAMF_LAUNCH_CHECK();
}

}  // namespace mamf
