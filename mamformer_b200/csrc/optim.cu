// Fused optimizer kernels over flat fp32 buffers.
//
// adamw_step: one pass over (master, grad, m, v) -> (master, m, v, bf16 copy), PyTorch AdamW
// semantics (decoupled decay p *= 1 - lr*wd, bias-corrected moments, eps added to
// sqrt(v)/sqrt(bc2)).  The gradient multiplier (1/world for averaging x clip factor) is read
// from device memory, so gradient clipping needs no host synchronisation.
// sq_norm_accumulate: sum of g^2 for the global gradient norm.
#include "common.cuh"

namespace mamf {

__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ out16, int64_t n,
                             float lr, float b1, float b2, float eps, float wd, float bc1, float bc2_sqrt,
                             const float* __restrict__ gscale) {
  const float s = gscale ? *gscale : 1.f;
  const float decay = 1.f - lr * wd;
  const float step = lr / bc1;
  const int64_t n4 = n / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    float4 gg = reinterpret_cast<const float4*>(g)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* pa = &pp.x; float* ga = &gg.x; float* ma = &mm.x; float* va = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float gk = ga[k] * s;
      ma[k] = b1 * ma[k] + (1.f - b1) * gk;
      va[k] = b2 * va[k] + (1.f - b2) * gk * gk;
      pa[k] = pa[k] * decay - step * ma[k] / (sqrtf(va[k]) / bc2_sqrt + eps);
    }
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (out16) {
      __nv_bfloat162 lo = __floats2bfloat162_rn(pp.x, pp.y), hi = __floats2bfloat162_rn(pp.z, pp.w);
      reinterpret_cast<__nv_bfloat162*>(out16)[2 * i] = lo;
      reinterpret_cast<__nv_bfloat162*>(out16)[2 * i + 1] = hi;
    }
  }
  for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float gk = g[i] * s;
    m[i] = b1 * m[i] + (1.f - b1) * gk;
    v[i] = b2 * v[i] + (1.f - b2) * gk * gk;
    p[i] = p[i] * decay - step * m[i] / (sqrtf(v[i]) / bc2_sqrt + eps);
    if (out16) out16[i] = __float2bfloat16(p[i]);
  }
}

void adamw_step(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, c10::optional<at::Tensor> out16,
                double lr, double b1, double b2, double eps, double wd, int64_t step,
                c10::optional<at::Tensor> gscale) {
  c10::cuda::CUDAGuard guard(p.device());
  TORCH_CHECK(p.is_contiguous() && g.is_contiguous() && m.is_contiguous() && v.is_contiguous(), "adamw: contiguous");
  TORCH_CHECK(p.dtype() == at::kFloat && g.dtype() == at::kFloat, "adamw: fp32 master and grad");
  const int64_t n = p.numel();
  if (n == 0) return;
  TORCH_CHECK(aligned16(p.data_ptr()) && aligned16(g.data_ptr()) && aligned16(m.data_ptr()) && aligned16(v.data_ptr()),
              "adamw: 16-byte aligned buffers");
  __nv_bfloat16* o = nullptr;
  if (out16.has_value()) {
    TORCH_CHECK(out16->dtype() == at::kBFloat16 && out16->numel() == n && out16->is_contiguous(), "adamw: bf16 out");
    TORCH_CHECK((reinterpret_cast<uintptr_t>(out16->data_ptr()) & 7) == 0, "adamw: bf16 out 8-byte aligned");
    o = (__nv_bfloat16*)out16->data_ptr();
  }
  const float bc1 = 1.f - (float)std::pow(b1, (double)step);
  const float bc2 = 1.f - (float)std::pow(b2, (double)step);
  const int blocks = (int)std::min<int64_t>((n / 4 + 255) / 256 + 1, (int64_t)num_sms() * 8);
  adamw_kernel<<<blocks, 256, 0, stream()>>>(
      p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), o, n, (float)lr,
      (float)b1, (float)b2, (float)eps, (float)wd, bc1, std::sqrt(bc2),
      gscale.has_value() ? gscale->data_ptr<float>() : nullptr);
  MAMF_LAUNCH_CHECK();
}

// Deterministic sum of squares: every block writes its partial sum, and the last block to finish
// adds the partials in index order (fixed grid, fixed shuffle tree), so data-parallel replicas that
// hold bitwise-equal gradients compute bitwise-equal norms and clip factors.
constexpr int kSqMaxBlocks = 4096;
__device__ float g_sq_partial[kSqMaxBlocks];
__device__ unsigned int g_sq_ticket = 0;

__global__ void sq_norm_kernel(const float* __restrict__ g, int64_t n, float* __restrict__ out) {
  float acc = 0.f;
  const int64_t n4 = ((reinterpret_cast<uintptr_t>(g) & 15) == 0) ? n / 4 : 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 x = reinterpret_cast<const float4*>(g)[i];
    acc = fmaf(x.x, x.x, acc); acc = fmaf(x.y, x.y, acc); acc = fmaf(x.z, x.z, acc); acc = fmaf(x.w, x.w, acc);
  }
  for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) acc = fmaf(g[i], g[i], acc);
  __shared__ float sm[32];
  __shared__ bool last;
  acc = block_sum(acc, sm);
  if (threadIdx.x == 0) {
    g_sq_partial[blockIdx.x] = acc;
    __threadfence();
    last = atomicAdd(&g_sq_ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  float s = 0.f;
  for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) s += *reinterpret_cast<volatile float*>(&g_sq_partial[i]);
  s = block_sum(s, sm);
  if (threadIdx.x == 0) {
    *out += s;
    g_sq_ticket = 0;
  }
}

// out (fp32 scalar tensor) += sum(g^2)
void sq_norm_accumulate(at::Tensor g, at::Tensor out) {
  c10::cuda::CUDAGuard guard(g.device());
  TORCH_CHECK(g.is_contiguous() && g.scalar_type() == at::kFloat, "sq_norm_accumulate: contiguous fp32");
  const int64_t n = g.numel();
  if (n == 0) return;
  const int blocks = (int)std::min<int64_t>(std::min<int64_t>((n + 1023) / 1024, (int64_t)num_sms() * 4), kSqMaxBlocks);
  sq_norm_kernel<<<blocks, 256, 0, stream()>>>(g.data_ptr<float>(), n, out.data_ptr<float>());
  MAMF_LAUNCH_CHECK();
}

// scale[0] = inv_world * min(1, max_norm / (norm + 1e-6)),  norm = sqrt(sq[0]) * inv_world
__global__ void clip_scale_kernel(const float* sq, float* scale, float max_norm, float inv_world, float* norm_out) {
  const float nrm = sqrtf(*sq) * inv_world;   // norm of the averaged gradient
  float s = inv_world;
  if (max_norm > 0.f && nrm > max_norm) s *= max_norm / (nrm + 1e-6f);
  *scale = s;
  if (norm_out) *norm_out = nrm;
}

void clip_scale(at::Tensor sq, at::Tensor scale, double max_norm, double inv_world, at::Tensor norm_out) {
  c10::cuda::CUDAGuard guard(sq.device());
  clip_scale_kernel<<<1, 1, 0, stream()>>>(sq.data_ptr<float>(), scale.data_ptr<float>(), (float)max_norm,
                                           (float)inv_world, norm_out.data_ptr<float>());
  MAMF_LAUNCH_CHECK();
}

// dst(fp32) += src(bf16 or fp32)  -- gradient accumulation into the fp32 main-grad buffer
template <typename T>
__global__ void accum_kernel(float* __restrict__ dst, const T* __restrict__ src, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] += to_f(src[i]);
}

void grad_accumulate(at::Tensor dst, at::Tensor src) {
  c10::cuda::CUDAGuard guard(dst.device());
  TORCH_CHECK(dst.is_contiguous() && src.is_contiguous() && dst.numel() == src.numel(), "grad_accumulate");
  const int64_t n = dst.numel();
  if (n == 0) return;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 8);
  MAMF_DISPATCH_FLOAT_BF16(src.scalar_type(), "grad_accumulate", [&] {
    accum_kernel<scalar_t><<<blocks, 256, 0, stream()>>>(dst.data_ptr<float>(), (const scalar_t*)src.data_ptr(), n);
  });
  MAMF_LAUNCH_CHECK();
}

// Embedding weight gradient: mg (V, d) fp32 += dy rows (N, d) at rows ids (N,), with fp32
// reductions at L2 (a block per token row, consecutive lanes on consecutive columns), so no dense
// V x d gradient is materialised and no separate accumulation pass runs.  Ids outside [0, V) are
// skipped (the forward gather has already rejected them).
template <typename T>
__global__ void embedding_grad_kernel(float* __restrict__ mg, const int64_t* __restrict__ ids,
                                      const T* __restrict__ dy, int64_t N, int64_t V, int64_t d) {
  for (int64_t r = blockIdx.x; r < N; r += gridDim.x) {
    const int64_t v = ids[r];
    if (v < 0 || v >= V) continue;
    float* dst = mg + v * d;
    const T* src = dy + r * d;
    for (int64_t c = threadIdx.x; c < d; c += blockDim.x) atomicAdd(dst + c, to_f(src[c]));
  }
}

void embedding_grad_accumulate(at::Tensor mg, at::Tensor ids, at::Tensor dy) {
  c10::cuda::CUDAGuard guard(mg.device());
  TORCH_CHECK(mg.is_contiguous() && mg.dim() == 2 && mg.scalar_type() == at::kFloat, "embedding grad: fp32 (V, d)");
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous() && dy.is_contiguous() && dy.dim() == 2 &&
              dy.size(0) == ids.numel() && dy.size(1) == mg.size(1), "embedding grad: ids (N,), dy (N, d)");
  const int64_t N = ids.numel(), V = mg.size(0), d = mg.size(1);
  if (N == 0) return;
  const unsigned blocks = (unsigned)std::min<int64_t>(N, (int64_t)num_sms() * 16);
  MAMF_DISPATCH_FLOAT_BF16(dy.scalar_type(), "embedding_grad", [&] {
    embedding_grad_kernel<scalar_t><<<blocks, 256, 0, stream()>>>(mg.data_ptr<float>(), ids.data_ptr<int64_t>(),
                                                                  (const scalar_t*)dy.data_ptr(), N, V, d);
  });
  MAMF_LAUNCH_CHECK();
}

}  // namespace mamf
