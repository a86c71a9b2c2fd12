// Cross-entropy row kernels for the fused linear + cross-entropy path.
//
// Reference semantics: F.cross_entropy(logits, labels, ignore_index=-100), mean over the
// non-ignored rows (mamformer/model.py:551-562, layers/mtp.py:264-276).  The logits of a chunk of
// rows come from the tcgen05 GEMM (bf16); these kernels make one pass over each row:
//   ce_stats:        online max / sum-exp in fp32 -> lse[row], loss[row] = lse - logit[label]
//   ce_grad_inplace: logits[row, :] <- (exp(logit - lse) - onehot(label)) * scale / n_valid
// with `scale` and `n_valid` read from device memory (no host synchronisation).
#include "common.cuh"

namespace mamf {

constexpr int CE_THREADS = 512;

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  const float mx = fmaxf(m, m2);
  if (mx == -INFINITY) { m = mx; s = 0.f; return; }
  s = s * __expf(m - mx) + s2 * __expf(m2 - mx);
  m = mx;
}

template <typename T>
__global__ void __launch_bounds__(CE_THREADS) ce_stats_kernel(const T* __restrict__ logits, int64_t ld,
                                                              const int64_t* __restrict__ labels, int V,
                                                              int ignore_index, float* __restrict__ loss,
                                                              float* __restrict__ lse_out) {
  constexpr int VEC = 16 / sizeof(T);
  const int64_t row = blockIdx.x;
  const T* lr = logits + row * ld;
  float m = -INFINITY, s = 0.f;
  const int nv = V / VEC;
  for (int i = threadIdx.x; i < nv; i += CE_THREADS) {
    Vec16<T> v = ld16(lr + (int64_t)i * VEC);
    float lm = -INFINITY;
#pragma unroll
    for (int k = 0; k < VEC; ++k) lm = fmaxf(lm, to_f(v.v[k]));
    float ls = 0.f;
#pragma unroll
    for (int k = 0; k < VEC; ++k) ls += __expf(to_f(v.v[k]) - lm);
    online_merge(m, s, lm, ls);
  }
  for (int i = nv * VEC + threadIdx.x; i < V; i += CE_THREADS) online_merge(m, s, to_f(lr[i]), 1.f);
  // warp merge
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    online_merge(m, s, m2, s2);
  }
  __shared__ float sm_m[32], sm_s[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) { sm_m[wid] = m; sm_s[wid] = s; }
  __syncthreads();
  if (wid == 0) {
    m = lane < CE_THREADS / 32 ? sm_m[lane] : -INFINITY;
    s = lane < CE_THREADS / 32 ? sm_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
      online_merge(m, s, m2, s2);
    }
    if (lane == 0) {
      const float lse = m + __logf(s);
      lse_out[row] = lse;
      const int64_t lab = labels[row];
      const bool valid = lab >= 0 && lab < V;
      (void)MAMF_BOUND(valid || lab == ignore_index, 1201);    // a label outside the vocabulary
      loss[row] = (lab == ignore_index || !valid) ? 0.f : lse - to_f(lr[lab]);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(CE_THREADS) ce_grad_kernel(T* __restrict__ logits, int64_t ld,
                                                             const int64_t* __restrict__ labels, int V,
                                                             int ignore_index, const float* __restrict__ lse,
                                                             const float* __restrict__ scale,
                                                             const float* __restrict__ n_valid) {
  constexpr int VEC = 16 / sizeof(T);
  const int64_t row = blockIdx.x;
  T* lr = logits + row * ld;
  const int64_t lab = labels[row];
  const bool ignored = (lab == ignore_index || lab < 0 || lab >= V);
  const float g = ignored ? 0.f : (*scale) / fmaxf(*n_valid, 1.f);
  const float l = lse[row];
  const int nv = V / VEC;
  for (int i = threadIdx.x; i < nv; i += CE_THREADS) {
    Vec16<T> v = ld16(lr + (int64_t)i * VEC);
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
      const int col = i * VEC + k;
      const float p = __expf(to_f(v.v[k]) - l);
      v.v[k] = from_f<T>(g * (p - (col == lab ? 1.f : 0.f)));
    }
    st16(lr + (int64_t)i * VEC, v);
  }
  for (int col = nv * VEC + threadIdx.x; col < V; col += CE_THREADS) {
    const float p = __expf(to_f(lr[col]) - l);
    lr[col] = from_f<T>(g * (p - (col == lab ? 1.f : 0.f)));
  }
}

// logits (R, V) (row stride ld, 16-byte aligned rows); labels (R,) int64 -> loss (R,), lse (R,)
void ce_stats(at::Tensor logits, at::Tensor labels, int64_t ignore_index, at::Tensor loss, at::Tensor lse) {
  c10::cuda::CUDAGuard guard(logits.device());
  const int64_t R = logits.size(0);
  const int V = logits.size(1);
  if (R == 0) return;
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous(), "ce: int64 labels");
  MAMF_DISPATCH_FLOAT_BF16(logits.scalar_type(), "ce_stats", [&] {
    TORCH_CHECK((logits.stride(0) * sizeof(scalar_t)) % 16 == 0 && aligned16(logits.data_ptr()), "ce: aligned rows");
    ce_stats_kernel<scalar_t><<<(unsigned)R, CE_THREADS, 0, stream()>>>(
        (const scalar_t*)logits.data_ptr(), logits.stride(0), labels.data_ptr<int64_t>(), V, (int)ignore_index,
        loss.data_ptr<float>(), lse.data_ptr<float>());
  });
  MAMF_LAUNCH_CHECK();
}

void ce_grad_inplace(at::Tensor logits, at::Tensor labels, int64_t ignore_index, at::Tensor lse,
                     at::Tensor scale, at::Tensor n_valid) {
  c10::cuda::CUDAGuard guard(logits.device());
  const int64_t R = logits.size(0);
  const int V = logits.size(1);
  if (R == 0) return;
  MAMF_DISPATCH_FLOAT_BF16(logits.scalar_type(), "ce_grad", [&] {
    TORCH_CHECK((logits.stride(0) * sizeof(scalar_t)) % 16 == 0 && aligned16(logits.data_ptr()), "ce: aligned rows");
    ce_grad_kernel<scalar_t><<<(unsigned)R, CE_THREADS, 0, stream()>>>(
        (scalar_t*)logits.data_ptr(), logits.stride(0), labels.data_ptr<int64_t>(), V, (int)ignore_index,
        lse.data_ptr<float>(), scale.data_ptr<float>(), n_valid.data_ptr<float>());
  });
  MAMF_LAUNCH_CHECK();
}

MAMF_BOUNDS_READER(bounds_error_ce)

}  // namespace mamf
