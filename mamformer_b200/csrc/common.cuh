// Shared helpers for the mamformer_b200 sm_100a kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#define MAMF_CHECK(cond, ...) TORCH_CHECK(cond, __VA_ARGS__)
#define MAMF_CUDA_CHECK(expr)                                                        \
  do {                                                                               \
    cudaError_t _e = (expr);                                                         \
    TORCH_CHECK(_e == cudaSuccess, "CUDA error: ", cudaGetErrorString(_e), " at ",   \
                __FILE__, ":", __LINE__);                                            \
  } while (0)
#define MAMF_LAUNCH_CHECK() MAMF_CUDA_CHECK(cudaGetLastError())

namespace mamf {

inline cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

inline int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// ---- element conversions ----------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16(v); }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half(v); }

// ---- reductions ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum over a 1-D or 2-D block; `smem` must hold >= 32 floats.  All threads get
// the result.
__device__ __forceinline__ float block_sum(float v, float* smem) {
  const int tid = threadIdx.x + threadIdx.y * blockDim.x;
  const int lane = tid & 31, wid = tid >> 5;
  const int nw = (blockDim.x * blockDim.y + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) smem[wid] = v;
  __syncthreads();
  float t = (lane < nw) ? smem[lane] : 0.f;
  return warp_sum(t);
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.f + __expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + __expf(-x)); }
__device__ __forceinline__ float softplus_f(float x) {
  // matches torch.nn.functional.softplus(beta=1, threshold=20)
  return x > 20.f ? x : log1pf(__expf(x));
}

// 16-byte vector of 8 bf16 (or 4 floats) for coalesced I/O.
template <typename T> struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
  union { uint4 raw; T v[N]; };
};

template <typename T>
__device__ __forceinline__ Vec16<T> ld16(const T* p) {
  Vec16<T> r;
  r.raw = *reinterpret_cast<const uint4*>(p);
  return r;
}
template <typename T>
__device__ __forceinline__ void st16(T* p, const Vec16<T>& r) {
  *reinterpret_cast<uint4*>(p) = r.raw;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// ---- debug bounds checks ----------------------------------------------------------------------
// In a build with MAMF_BOUNDS_CHECK defined, MAMF_BOUND(cond, code) evaluates `cond`; when it is
// false it records `code` in this file's error word (the first failure wins) and returns false,
// and the caller skips the access.  Nothing traps, so a bad index leaves the context usable.
// Without the flag MAMF_BOUND is the constant `true` and compiles away.  A file that uses it
// defines its reader with MAMF_BOUNDS_READER(name) (read-and-clear of its own word).
static __device__ int g_mamf_bounds_err = 0;
#ifdef MAMF_BOUNDS_CHECK
__device__ __forceinline__ bool mamf_bound(bool ok, int code) {
  if (!ok) atomicCAS(&g_mamf_bounds_err, 0, code);
  return ok;
}
#define MAMF_BOUND(cond, code) ::mamf::mamf_bound((cond), (code))
#define MAMF_BOUNDS_BUILT 1
#else
#define MAMF_BOUND(cond, code) true
#define MAMF_BOUNDS_BUILT 0
#endif
#define MAMF_BOUNDS_READER(fn)                                                        \
  int64_t fn() {                                                                      \
    int v = 0;                                                                        \
    MAMF_CUDA_CHECK(cudaMemcpyFromSymbol(&v, g_mamf_bounds_err, sizeof(int)));        \
    if (v) {                                                                          \
      int z = 0;                                                                      \
      MAMF_CUDA_CHECK(cudaMemcpyToSymbol(g_mamf_bounds_err, &z, sizeof(int)));        \
    }                                                                                 \
    return v;                                                                         \
  }

}  // namespace mamf

#define MAMF_DISPATCH_FLOAT_BF16(dtype, NAME, ...)                                      \
  [&] {                                                                               \
    if ((dtype) == at::kFloat) {                                                      \
      using scalar_t = float;                                                         \
      return __VA_ARGS__();                                                           \
    } else if ((dtype) == at::kBFloat16) {                                            \
      using scalar_t = __nv_bfloat16;                                                 \
      return __VA_ARGS__();                                                           \
    } else if ((dtype) == at::kHalf) {                                                \
      using scalar_t = __half;                                                        \
      return __VA_ARGS__();                                                           \
    }                                                                                 \
    TORCH_CHECK(false, NAME, ": unsupported dtype ", dtype);                          \
  }()
