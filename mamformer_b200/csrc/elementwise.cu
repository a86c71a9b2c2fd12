// Memory-bound kernels: RMSNorm, SwiGLU, RoPE, causal depthwise conv + SiLU, per-head
// GroupNorm.  All are bandwidth-bound on B200 (HBM3e), so each does one pass over its data
// with 16-byte vector accesses and fp32 math.
//
// Reference semantics: RMSNorm mamformer/layers/norm.py:34-43; RoPE rope.py:283-339
// (half-split rotation); conv mamba2.py:370-405; GroupNorm kda_diff.py:345-348
// (nn.GroupNorm(H, H*hd) over (hd x S) per sample); SwiGLU ffn.py:71-80.
#include "common.cuh"

namespace mamf {

// ============================ RMSNorm ========================================================
// One warp per row, the row is held in registers (up to 32*8*NV elements).
template <typename T, int NV>
__global__ void rmsnorm_fwd_kernel(const T* __restrict__ x, const float* __restrict__ w,
                                   T* __restrict__ y, float* __restrict__ rstd_out, int64_t rows,
                                   int d, float eps) {
  constexpr int V = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + row * d;
  Vec16<T> buf[NV];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int col = (i * 32 + lane) * V;
    if (col < d) {
      buf[i] = ld16(xr + col);
#pragma unroll
      for (int k = 0; k < V; ++k) { float f = to_f(buf[i].v[k]); ss += f * f; }
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / d + eps);
  if (lane == 0 && rstd_out) rstd_out[row] = r;
  T* yr = y + row * d;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int col = (i * 32 + lane) * V;
    if (col < d) {
      Vec16<T> o;
#pragma unroll
      for (int k = 0; k < V; ++k) o.v[k] = from_f<T>(to_f(buf[i].v[k]) * r * w[col + k]);
      st16(yr + col, o);
    }
  }
}

// dx = r * (g - xhat * mean(g * xhat)),  g = dy * w,  xhat = x * r
template <typename T, int NV>
__global__ void rmsnorm_bwd_dx_kernel(const T* __restrict__ x, const float* __restrict__ w,
                                      const T* __restrict__ dy, const float* __restrict__ rstd,
                                      T* __restrict__ dx, int64_t rows, int d) {
  constexpr int V = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float r = rstd[row];
  Vec16<T> xb[NV], gb[NV];
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int col = (i * 32 + lane) * V;
    if (col < d) {
      xb[i] = ld16(x + row * d + col);
      gb[i] = ld16(dy + row * d + col);
#pragma unroll
      for (int k = 0; k < V; ++k) dot += to_f(gb[i].v[k]) * w[col + k] * to_f(xb[i].v[k]);
    }
  }
  dot = warp_sum(dot) * r / d;   // mean(g * xhat) = r * mean(g*x)
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int col = (i * 32 + lane) * V;
    if (col < d) {
      Vec16<T> o;
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const float g = to_f(gb[i].v[k]) * w[col + k];
        const float xh = to_f(xb[i].v[k]) * r;
        o.v[k] = from_f<T>(r * (g - xh * dot));
      }
      st16(dx + row * d + col, o);
    }
  }
}

// dw partial sums: block (32 x 8 threads) covers 32 columns and a slab of rows.
template <typename T>
__global__ void rmsnorm_bwd_dw_kernel(const T* __restrict__ x, const T* __restrict__ dy,
                                      const float* __restrict__ rstd, float* __restrict__ part,
                                      int64_t rows, int d, int rows_per_block) {
  const int col = blockIdx.x * 32 + threadIdx.x;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_block;
  const int64_t r1 = min(rows, r0 + rows_per_block);
  float acc = 0.f;
  if (col < d)
    for (int64_t r = r0 + threadIdx.y; r < r1; r += blockDim.y)
      acc += to_f(dy[r * d + col]) * to_f(x[r * d + col]) * rstd[r];
  __shared__ float sm[8][33];
  sm[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y == 0 && col < d) {
    float s = 0.f;
    for (int i = 0; i < blockDim.y; ++i) s += sm[i][threadIdx.x];
    part[(int64_t)blockIdx.y * d + col] = s;
  }
}

// dw partial sums, vector form: a thread owns V consecutive columns (16-byte loads) of a slab of
// rows (row lanes y = 0..7); block = 32 column vectors x 8 row lanes.
template <typename T>
__global__ void rmsnorm_bwd_dw_vec_kernel(const T* __restrict__ x, const T* __restrict__ dy,
                                          const float* __restrict__ rstd, float* __restrict__ part,
                                          int64_t rows, int d, int rows_per_block) {
  constexpr int V = 16 / sizeof(T);
  const int col = (blockIdx.x * 32 + threadIdx.x) * V;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_block;
  const int64_t r1 = min(rows, r0 + rows_per_block);
  float acc[V];
#pragma unroll
  for (int k = 0; k < V; ++k) acc[k] = 0.f;
  if (col < d)
    for (int64_t r = r0 + threadIdx.y; r < r1; r += blockDim.y) {
      const Vec16<T> a = ld16(x + r * d + col), g = ld16(dy + r * d + col);
      const float rs = rstd[r];
#pragma unroll
      for (int k = 0; k < V; ++k) acc[k] = fmaf(to_f(g.v[k]) * rs, to_f(a.v[k]), acc[k]);
    }
  __shared__ float sm[8][32 * V + 1];
#pragma unroll
  for (int k = 0; k < V; ++k) sm[threadIdx.y][threadIdx.x * V + k] = acc[k];
  __syncthreads();
  const int t = threadIdx.y * 32 + threadIdx.x;          // one output column per thread
  const int c = blockIdx.x * 32 * V + t;
  if (t < 32 * V && c < d) {
    float s = 0.f;
    for (int i = 0; i < 8; ++i) s += sm[i][t];
    part[(int64_t)blockIdx.y * d + c] = s;
  }
}

// Block-per-row variants (256 threads, NVT 16-byte vectors per thread): a row's data is spread
// over the whole block, so each thread holds at most 4 vectors and the SM keeps 8 rows in flight
// (the warp-per-row kernels above hold a 4096-wide row in one warp's registers, which limits
// occupancy to 8-16 warps per SM).  Used when d is a multiple of the vector width and d / V <= 1024.
constexpr int RMS_BT = 256;

// w[col .. col + V) as fp32 (col a multiple of V, w 16-byte aligned)
template <int V>
__device__ __forceinline__ void ld_w(const float* __restrict__ w, int col, float (&out)[V]) {
#pragma unroll
  for (int q = 0; q < V / 4; ++q) {
    const float4 f = *reinterpret_cast<const float4*>(w + col + 4 * q);
    out[4 * q] = f.x; out[4 * q + 1] = f.y; out[4 * q + 2] = f.z; out[4 * q + 3] = f.w;
  }
}

template <typename T, int NVT>
__global__ void __launch_bounds__(RMS_BT) rms_blk_fwd_kernel(const T* __restrict__ x, const float* __restrict__ w,
                                                            T* __restrict__ y, float* __restrict__ rstd_out, int d,
                                                            float eps) {
  constexpr int V = 16 / sizeof(T);
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * d;
  Vec16<T> buf[NVT];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NVT; ++i) {
    const int col = (i * RMS_BT + threadIdx.x) * V;
    if (col < d) {
      buf[i] = ld16(xr + col);
#pragma unroll
      for (int k = 0; k < V; ++k) { const float f = to_f(buf[i].v[k]); ss = fmaf(f, f, ss); }
    }
  }
  ss = block_sum(ss, red);
  const float r = rsqrtf(ss / d + eps);
  if (threadIdx.x == 0 && rstd_out) rstd_out[row] = r;
  T* yr = y + row * d;
#pragma unroll
  for (int i = 0; i < NVT; ++i) {
    const int col = (i * RMS_BT + threadIdx.x) * V;
    if (col < d) {
      float wv[V];
      ld_w<V>(w, col, wv);
      Vec16<T> o;
#pragma unroll
      for (int k = 0; k < V; ++k) o.v[k] = from_f<T>(to_f(buf[i].v[k]) * r * wv[k]);
      st16(yr + col, o);
    }
  }
}

template <typename T, int NVT>
__global__ void __launch_bounds__(RMS_BT) rms_blk_bwd_dx_kernel(const T* __restrict__ x, const float* __restrict__ w,
                                                               const T* __restrict__ dy, const float* __restrict__ rstd,
                                                               T* __restrict__ dx, int d) {
  constexpr int V = 16 / sizeof(T);
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const float r = rstd[row];
  Vec16<T> xb[NVT], gb[NVT];
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < NVT; ++i) {
    const int col = (i * RMS_BT + threadIdx.x) * V;
    if (col < d) {
      xb[i] = ld16(x + row * d + col);
      gb[i] = ld16(dy + row * d + col);
      float wv[V];
      ld_w<V>(w, col, wv);
#pragma unroll
      for (int k = 0; k < V; ++k) dot = fmaf(to_f(gb[i].v[k]) * wv[k], to_f(xb[i].v[k]), dot);
    }
  }
  dot = block_sum(dot, red) * r / d;   // mean(g * xhat) = r * mean(g * x)
#pragma unroll
  for (int i = 0; i < NVT; ++i) {
    const int col = (i * RMS_BT + threadIdx.x) * V;
    if (col < d) {
      float wv[V];
      ld_w<V>(w, col, wv);
      Vec16<T> o;
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const float g = to_f(gb[i].v[k]) * wv[k];
        const float xh = to_f(xb[i].v[k]) * r;
        o.v[k] = from_f<T>(r * (g - xh * dot));
      }
      st16(dx + row * d + col, o);
    }
  }
}

// Calls fn(std::integral_constant<int, NVT>) for the block-per-row kernels; false if d does not fit.
template <typename T, typename F>
static bool with_blk_nvt(int d, F&& fn) {
  constexpr int V = 16 / sizeof(T);
  if (d % V != 0) return false;
  const int nv = d / V;
  if (nv <= RMS_BT) fn(std::integral_constant<int, 1>{});
  else if (nv <= 2 * RMS_BT) fn(std::integral_constant<int, 2>{});
  else if (nv <= 4 * RMS_BT) fn(std::integral_constant<int, 4>{});
  else return false;
  return true;
}

template <typename T>
static int rms_nv(int d) {
  constexpr int V = 16 / sizeof(T);
  return (d + 32 * V - 1) / (32 * V);
}

// Calls fn(std::integral_constant<int, NV>) for the smallest supported NV >= nv.
template <typename F>
static void with_nv(int nv, F&& fn) {
  if (nv <= 1) fn(std::integral_constant<int, 1>{});
  else if (nv <= 2) fn(std::integral_constant<int, 2>{});
  else if (nv <= 4) fn(std::integral_constant<int, 4>{});
  else if (nv <= 8) fn(std::integral_constant<int, 8>{});
  else if (nv <= 16) fn(std::integral_constant<int, 16>{});
  else if (nv <= 32) fn(std::integral_constant<int, 32>{});
  else TORCH_CHECK(false, "rmsnorm: d too large");
}

std::vector<at::Tensor> rmsnorm_fwd(at::Tensor x, at::Tensor w, double eps) {
  c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.is_contiguous() && w.dtype() == at::kFloat, "rmsnorm: contiguous x, fp32 weight");
  const int d = x.size(-1);
  const int64_t rows = x.numel() / d;
  at::Tensor y = at::empty_like(x);
  at::Tensor rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  at::Tensor wc = w.contiguous();
  MAMF_DISPATCH_FLOAT_BF16(x.scalar_type(), "rmsnorm_fwd", [&] {
    TORCH_CHECK((d * sizeof(scalar_t)) % 16 == 0 && aligned16(x.data_ptr()), "rmsnorm: d*elt must be a multiple of 16 bytes");
    const bool blk = rows > 0 && rows <= INT32_MAX && aligned16(wc.data_ptr()) &&
                     with_blk_nvt<scalar_t>(d, [&](auto nc) {
                       constexpr int NVT = decltype(nc)::value;
                       rms_blk_fwd_kernel<scalar_t, NVT><<<(unsigned)rows, RMS_BT, 0, stream()>>>(
                           (const scalar_t*)x.data_ptr(), wc.data_ptr<float>(), (scalar_t*)y.data_ptr(),
                           rstd.data_ptr<float>(), d, (float)eps);
                     });
    if (!blk) {
      const int blocks = (int)((rows + 7) / 8);
      with_nv(rms_nv<scalar_t>(d), [&](auto nvc) {
        constexpr int NVV = decltype(nvc)::value;
        rmsnorm_fwd_kernel<scalar_t, NVV><<<blocks, 256, 0, stream()>>>(
            (const scalar_t*)x.data_ptr(), wc.data_ptr<float>(), (scalar_t*)y.data_ptr(),
            rstd.data_ptr<float>(), rows, d, (float)eps);
      });
    }
  });
  MAMF_LAUNCH_CHECK();
  return {y, rstd};
}

std::vector<at::Tensor> rmsnorm_bwd(at::Tensor x, at::Tensor w, at::Tensor dy, at::Tensor rstd) {
  c10::cuda::CUDAGuard g(x.device());
  dy = dy.contiguous();
  const int d = x.size(-1);
  const int64_t rows = x.numel() / d;
  at::Tensor dx = at::empty_like(x);
  at::Tensor wc = w.contiguous();
  const int rpb = 256;
  const int nrb = (int)((rows + rpb - 1) / rpb);
  at::Tensor part = at::empty({nrb, d}, x.options().dtype(at::kFloat));
  MAMF_DISPATCH_FLOAT_BF16(x.scalar_type(), "rmsnorm_bwd", [&] {
    const bool blk = rows > 0 && rows <= INT32_MAX && aligned16(wc.data_ptr()) && aligned16(x.data_ptr()) &&
                     aligned16(dy.data_ptr()) &&
                     with_blk_nvt<scalar_t>(d, [&](auto nc) {
                       constexpr int NVT = decltype(nc)::value;
                       rms_blk_bwd_dx_kernel<scalar_t, NVT><<<(unsigned)rows, RMS_BT, 0, stream()>>>(
                           (const scalar_t*)x.data_ptr(), wc.data_ptr<float>(), (const scalar_t*)dy.data_ptr(),
                           rstd.data_ptr<float>(), (scalar_t*)dx.data_ptr(), d);
                     });
    if (!blk) {
      const int blocks = (int)((rows + 7) / 8);
      with_nv(rms_nv<scalar_t>(d), [&](auto nvc) {
        constexpr int NVV = decltype(nvc)::value;
        rmsnorm_bwd_dx_kernel<scalar_t, NVV><<<blocks, 256, 0, stream()>>>(
            (const scalar_t*)x.data_ptr(), wc.data_ptr<float>(), (const scalar_t*)dy.data_ptr(),
            rstd.data_ptr<float>(), (scalar_t*)dx.data_ptr(), rows, d);
      });
    }
    constexpr int V = 16 / sizeof(scalar_t);
    if (d % V == 0 && aligned16(x.data_ptr()) && aligned16(dy.data_ptr())) {
      dim3 grid((d / V + 31) / 32, nrb);
      rmsnorm_bwd_dw_vec_kernel<scalar_t><<<grid, dim3(32, 8), 0, stream()>>>(
          (const scalar_t*)x.data_ptr(), (const scalar_t*)dy.data_ptr(), rstd.data_ptr<float>(),
          part.data_ptr<float>(), rows, d, rpb);
    } else {
      dim3 grid((d + 31) / 32, nrb);
      rmsnorm_bwd_dw_kernel<scalar_t><<<grid, dim3(32, 8), 0, stream()>>>(
          (const scalar_t*)x.data_ptr(), (const scalar_t*)dy.data_ptr(), rstd.data_ptr<float>(),
          part.data_ptr<float>(), rows, d, rpb);
    }
  });
  MAMF_LAUNCH_CHECK();
  return {dx, part.sum(0)};
}

// ============================ SwiGLU =========================================================
template <typename T>
__global__ void swiglu_fwd_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ y,
                                  int64_t rows, int cols, int64_t gs, int64_t us) {
  constexpr int V = 16 / sizeof(T);
  const int cv = cols / V;
  const int64_t total = rows * cv;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cv;
    const int c = (int)(i - r * cv) * V;
    Vec16<T> a = ld16(g + r * gs + c), b = ld16(u + r * us + c), o;
#pragma unroll
    for (int k = 0; k < V; ++k) o.v[k] = from_f<T>(silu_f(to_f(a.v[k])) * to_f(b.v[k]));
    st16(y + r * cols + c, o);
  }
}

template <typename T>
__global__ void swiglu_bwd_kernel(const T* __restrict__ g, const T* __restrict__ u, const T* __restrict__ dy,
                                  T* __restrict__ dg, T* __restrict__ du, int64_t rows, int cols,
                                  int64_t gs, int64_t us) {
  constexpr int V = 16 / sizeof(T);
  const int cv = cols / V;
  const int64_t total = rows * cv;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cv;
    const int c = (int)(i - r * cv) * V;
    Vec16<T> a = ld16(g + r * gs + c), b = ld16(u + r * us + c), d = ld16(dy + r * cols + c), og, ou;
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float gv = to_f(a.v[k]), uv = to_f(b.v[k]), dv = to_f(d.v[k]);
      const float s = sigmoid_f(gv);
      og.v[k] = from_f<T>(dv * uv * s * (1.f + gv * (1.f - s)));
      ou.v[k] = from_f<T>(dv * gv * s);
    }
    st16(dg + r * cols + c, og);
    st16(du + r * cols + c, ou);
  }
}

static int ew_blocks(int64_t n) { return (int)std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 16); }

at::Tensor swiglu_fwd(at::Tensor g, at::Tensor u) {
  c10::cuda::CUDAGuard guard(g.device());
  const int cols = g.size(-1);
  const int64_t rows = g.numel() / cols;
  TORCH_CHECK(g.stride(-1) == 1 && u.stride(-1) == 1, "swiglu: unit inner stride");
  auto g2 = g.reshape({rows, cols}), u2 = u.reshape({rows, cols});
  at::Tensor y = at::empty({rows, cols}, g.options());
  MAMF_DISPATCH_FLOAT_BF16(g.scalar_type(), "swiglu_fwd", [&] {
    TORCH_CHECK((cols * sizeof(scalar_t)) % 16 == 0, "swiglu: cols*elt % 16");
    const int64_t n = rows * cols / (16 / sizeof(scalar_t));
    swiglu_fwd_kernel<scalar_t><<<ew_blocks(n), 256, 0, stream()>>>(
        (const scalar_t*)g2.data_ptr(), (const scalar_t*)u2.data_ptr(), (scalar_t*)y.data_ptr(), rows, cols,
        g2.stride(0), u2.stride(0));
  });
  MAMF_LAUNCH_CHECK();
  auto shape = g.sizes().vec();
  return y.view(shape);
}

std::vector<at::Tensor> swiglu_bwd(at::Tensor g, at::Tensor u, at::Tensor dy) {
  c10::cuda::CUDAGuard guard(g.device());
  const int cols = g.size(-1);
  const int64_t rows = g.numel() / cols;
  auto g2 = g.reshape({rows, cols}), u2 = u.reshape({rows, cols});
  auto dy2 = dy.reshape({rows, cols}).contiguous();
  at::Tensor dg = at::empty({rows, cols}, g.options()), du = at::empty({rows, cols}, g.options());
  MAMF_DISPATCH_FLOAT_BF16(g.scalar_type(), "swiglu_bwd", [&] {
    const int64_t n = rows * cols / (16 / sizeof(scalar_t));
    swiglu_bwd_kernel<scalar_t><<<ew_blocks(n), 256, 0, stream()>>>(
        (const scalar_t*)g2.data_ptr(), (const scalar_t*)u2.data_ptr(), (const scalar_t*)dy2.data_ptr(),
        (scalar_t*)dg.data_ptr(), (scalar_t*)du.data_ptr(), rows, cols, g2.stride(0), u2.stride(0));
  });
  MAMF_LAUNCH_CHECK();
  auto shape = g.sizes().vec();
  return {dg.view(shape), du.view(shape)};
}

// ============================ RoPE ===========================================================
// x: (B, S, H, hd) with row stride xs between (b,s) rows (heads contiguous); cos/sin (S, hd/2).
// sign = +1 forward, -1 backward (rotation by -theta).
template <typename T>
__global__ void rope_kernel(const T* __restrict__ x, T* __restrict__ y, const float* __restrict__ cs,
                            const float* __restrict__ sn, int64_t BS, int S, int H, int hd,
                            int64_t xs, float sign) {
  const int half = hd / 2;
  const int64_t total = BS * H * half;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(i % half);
    const int64_t rh = i / half;
    const int h = (int)(rh % H);
    const int64_t bs = rh / H;
    const int s = (int)(bs % S);
    const T* xp = x + bs * xs + (int64_t)h * hd;
    T* yp = y + (bs * H + h) * hd;
    const float c = cs[(int64_t)s * half + j], sv = sign * sn[(int64_t)s * half + j];
    const float x1 = to_f(xp[j]), x2 = to_f(xp[j + half]);
    yp[j] = from_f<T>(x1 * c - x2 * sv);
    yp[j + half] = from_f<T>(x2 * c + x1 * sv);
  }
}

// Vectorised form: one block per token row (b, s); a thread rotates V consecutive pairs
// (j .. j+V-1, j+half .. j+half+V-1) of one head with 16-byte loads, the row's cos / sin read as
// float4.  Needs half % V == 0 and 16-byte aligned rows.
template <typename T>
__global__ void rope_vec_kernel(const T* __restrict__ x, T* __restrict__ y, const float* __restrict__ cs,
                                const float* __restrict__ sn, int S, int H, int hd, int64_t xs, float sign) {
  constexpr int V = 16 / sizeof(T);
  const int half = hd / 2, nv = half / V;
  const int64_t bs = blockIdx.x;
  const int s = (int)(bs % S);
  const T* xr = x + bs * xs;
  T* yr = y + bs * (int64_t)H * hd;
  const float* cr = cs + (int64_t)s * half;
  const float* sr = sn + (int64_t)s * half;
  for (int e = threadIdx.x; e < H * nv; e += blockDim.x) {
    const int h = e / nv, j = (e - h * nv) * V;
    const Vec16<T> a = ld16(xr + h * hd + j), b = ld16(xr + h * hd + half + j);
    float c[V], sv[V];
    ld_w<V>(cr, j, c);
    ld_w<V>(sr, j, sv);
    Vec16<T> oa, ob;
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float x1 = to_f(a.v[k]), x2 = to_f(b.v[k]), si = sign * sv[k];
      oa.v[k] = from_f<T>(x1 * c[k] - x2 * si);
      ob.v[k] = from_f<T>(x2 * c[k] + x1 * si);
    }
    st16(yr + h * hd + j, oa);
    st16(yr + h * hd + half + j, ob);
  }
}

at::Tensor rope_apply(at::Tensor x, at::Tensor cos, at::Tensor sin, bool inverse) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.dim() == 4, "rope: x must be (B, S, H, hd)");
  const int B = x.size(0), S = x.size(1), H = x.size(2), hd = x.size(3);
  TORCH_CHECK(x.stride(3) == 1 && x.stride(2) == hd && x.stride(0) == x.stride(1) * S,
              "rope: heads must be contiguous within a token row");
  at::Tensor cc = cos.to(at::kFloat).contiguous(), ss = sin.to(at::kFloat).contiguous();
  TORCH_CHECK(cc.size(0) == S && cc.size(1) == hd / 2, "rope: table shape");
  at::Tensor y = at::empty({B, S, H, hd}, x.options());
  MAMF_DISPATCH_FLOAT_BF16(x.scalar_type(), "rope", [&] {
    constexpr int V = 16 / sizeof(scalar_t);
    const int64_t rows = (int64_t)B * S;
    if ((hd / 2) % V == 0 && aligned16(x.data_ptr()) && (x.stride(1) * sizeof(scalar_t)) % 16 == 0 &&
        aligned16(cc.data_ptr()) && aligned16(ss.data_ptr()) && rows > 0 && rows <= INT32_MAX) {
      const int work = H * (hd / 2 / V);
      const int threads = std::min(256, (work + 31) / 32 * 32);
      rope_vec_kernel<scalar_t><<<(unsigned)rows, threads, 0, stream()>>>(
          (const scalar_t*)x.data_ptr(), (scalar_t*)y.data_ptr(), cc.data_ptr<float>(), ss.data_ptr<float>(), S, H,
          hd, x.stride(1), inverse ? -1.f : 1.f);
      return;
    }
    const int64_t n = (int64_t)B * S * H * (hd / 2);
    rope_kernel<scalar_t><<<ew_blocks(n), 256, 0, stream()>>>(
        (const scalar_t*)x.data_ptr(), (scalar_t*)y.data_ptr(), cc.data_ptr<float>(), ss.data_ptr<float>(),
        (int64_t)B * S, S, H, hd, x.stride(1), inverse ? -1.f : 1.f);
  });
  MAMF_LAUNCH_CHECK();
  return y;
}

// ============================ causal depthwise conv + SiLU ===================================
// x (B, S, C) with row stride xs; w (C, K).  Thread = one channel x a TT-step time tile.
constexpr int CONV_TT = 64;

template <typename T, int K>
__global__ void conv_silu_fwd_kernel(const T* __restrict__ x, const float* __restrict__ w,
                                     T* __restrict__ y, int B, int S, int C, int64_t xs) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int t0 = blockIdx.y * CONV_TT;
  const int b = blockIdx.z;
  if (c >= C) return;
  float wk[K];
#pragma unroll
  for (int k = 0; k < K; ++k) wk[k] = w[c * K + k];
  float hist[K];
#pragma unroll
  for (int k = 0; k < K - 1; ++k) {
    const int t = t0 - (K - 1) + k;
    hist[k] = t >= 0 ? to_f(x[((int64_t)b * S + t) * xs + c]) : 0.f;
  }
  const int t1 = min(S, t0 + CONV_TT);
  for (int t = t0; t < t1; ++t) {
    hist[K - 1] = to_f(x[((int64_t)b * S + t) * xs + c]);
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) acc = fmaf(wk[k], hist[k], acc);
    y[((int64_t)b * S + t) * C + c] = from_f<T>(silu_f(acc));
#pragma unroll
    for (int k = 0; k < K - 1; ++k) hist[k] = hist[k + 1];
  }
}

// dpre[t] = dy[t] * silu'(pre[t]);  dx[t] = sum_k w[k] dpre[t + K-1-k];  dw[k] += dpre[t] x[t-K+1+k]
template <typename T, int K>
__global__ void conv_silu_bwd_kernel(const T* __restrict__ x, const float* __restrict__ w,
                                     const T* __restrict__ dy, T* __restrict__ dx,
                                     float* __restrict__ dw_part, int B, int S, int C, int64_t xs) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int tile = blockIdx.y;
  const int t0 = tile * CONV_TT;
  const int b = blockIdx.z;
  if (c >= C) return;
  float wk[K];
#pragma unroll
  for (int k = 0; k < K; ++k) wk[k] = w[c * K + k];
  auto X = [&](int t) -> float { return (t >= 0 && t < S) ? to_f(x[((int64_t)b * S + t) * xs + c]) : 0.f; };
  auto DPRE = [&](int t) -> float {
    if (t < 0 || t >= S) return 0.f;
    float pre = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) pre = fmaf(wk[k], X(t - (K - 1) + k), pre);
    const float s = sigmoid_f(pre);
    return to_f(dy[((int64_t)b * S + t) * C + c]) * s * (1.f + pre * (1.f - s));
  };
  float dp[K];
#pragma unroll
  for (int k = 0; k < K; ++k) dp[k] = DPRE(t0 + k);
  float dwa[K];
#pragma unroll
  for (int k = 0; k < K; ++k) dwa[k] = 0.f;
  const int t1 = min(S, t0 + CONV_TT);
  for (int t = t0; t < t1; ++t) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) acc = fmaf(wk[k], dp[K - 1 - k], acc);
    dx[((int64_t)b * S + t) * C + c] = from_f<T>(acc);
    const float d0 = dp[0];
#pragma unroll
    for (int k = 0; k < K; ++k) dwa[k] = fmaf(d0, X(t - (K - 1) + k), dwa[k]);
#pragma unroll
    for (int k = 0; k < K - 1; ++k) dp[k] = dp[k + 1];
    dp[K - 1] = DPRE(t + K);
  }
  const int64_t pidx = ((int64_t)b * gridDim.y + tile);
#pragma unroll
  for (int k = 0; k < K; ++k) dw_part[(pidx * C + c) * K + k] = dwa[k];
}

// Vectorised forms: a thread owns CV = 4 consecutive channels (8-byte bf16 / 16-byte fp32 loads),
// so a warp moves 256 / 512 contiguous bytes per time step.  The backward keeps a register window
// of x[t - K + 1 .. t + K] per channel and the K pending d pre-activations, so each step loads one
// x row and one dy row (the scalar kernel above recomputes every x tap from global memory).
constexpr int CV = 4;

template <typename T>
__device__ __forceinline__ void ld_cv(const T* __restrict__ p, float (&o)[CV]) {
  if constexpr (sizeof(T) == 2) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < CV; ++i) o[i] = to_f(h[i]);
  } else {
    const float4 f = *reinterpret_cast<const float4*>(p);
    o[0] = to_f(f.x); o[1] = to_f(f.y); o[2] = to_f(f.z); o[3] = to_f(f.w);
  }
}
template <typename T>
__device__ __forceinline__ void st_cv(T* __restrict__ p, const float (&v)[CV]) {
  if constexpr (sizeof(T) == 2) {
    uint2 u;
    T* h = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int i = 0; i < CV; ++i) h[i] = from_f<T>(v[i]);
    *reinterpret_cast<uint2*>(p) = u;
  } else {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
}

template <typename T, int K>
__global__ void conv_silu_fwd_vec_kernel(const T* __restrict__ x, const float* __restrict__ w,
                                         T* __restrict__ y, int S, int C, int64_t xs) {
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * CV;
  const int t0 = blockIdx.y * CONV_TT;
  const int b = blockIdx.z;
  if (c0 >= C) return;
  float wk[CV][K], hist[K][CV];
#pragma unroll
  for (int i = 0; i < CV; ++i)
#pragma unroll
    for (int k = 0; k < K; ++k) wk[i][k] = w[(c0 + i) * K + k];
#pragma unroll
  for (int k = 0; k < K - 1; ++k) {
    const int t = t0 - (K - 1) + k;
    if (t >= 0) ld_cv(x + ((int64_t)b * S + t) * xs + c0, hist[k]);
    else {
#pragma unroll
      for (int i = 0; i < CV; ++i) hist[k][i] = 0.f;
    }
  }
  const int t1 = min(S, t0 + CONV_TT);
  float nxt[CV];                                          // x row of the next step, loaded one ahead
  ld_cv(x + ((int64_t)b * S + t0) * xs + c0, nxt);
  for (int t = t0; t < t1; ++t) {
#pragma unroll
    for (int i = 0; i < CV; ++i) hist[K - 1][i] = nxt[i];
    if (t + 1 < t1) ld_cv(x + ((int64_t)b * S + t + 1) * xs + c0, nxt);
    float o[CV];
#pragma unroll
    for (int i = 0; i < CV; ++i) {
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < K; ++k) acc = fmaf(wk[i][k], hist[k][i], acc);
      o[i] = silu_f(acc);
    }
    st_cv(y + ((int64_t)b * S + t) * C + c0, o);
#pragma unroll
    for (int k = 0; k < K - 1; ++k)
#pragma unroll
      for (int i = 0; i < CV; ++i) hist[k][i] = hist[k + 1][i];
  }
}

template <typename T, int K>
__global__ void conv_silu_bwd_vec_kernel(const T* __restrict__ x, const float* __restrict__ w,
                                         const T* __restrict__ dy, T* __restrict__ dx,
                                         float* __restrict__ dw_part, int S, int C, int64_t xs) {
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * CV;
  const int tile = blockIdx.y;
  const int t0 = tile * CONV_TT;
  const int b = blockIdx.z;
  if (c0 >= C) return;
  float wk[CV][K];
#pragma unroll
  for (int i = 0; i < CV; ++i)
#pragma unroll
    for (int k = 0; k < K; ++k) wk[i][k] = w[(c0 + i) * K + k];
  auto ldx = [&](int t, float (&o)[CV]) {
    if (t >= 0 && t < S) ld_cv(x + ((int64_t)b * S + t) * xs + c0, o);
    else {
#pragma unroll
      for (int i = 0; i < CV; ++i) o[i] = 0.f;
    }
  };
  // xw[j] = x[t - K + 1 + j], j < 2K, for the current step t
  float xw[2 * K][CV];
#pragma unroll
  for (int j = 0; j < 2 * K; ++j) ldx(t0 - K + 1 + j, xw[j]);
  // d pre-activation at time u, from the window: pre(u) = sum_k w_k x[u - K + 1 + k]
  auto ldg = [&](int u, float (&o)[CV]) {
    if (u < S) ld_cv(dy + ((int64_t)b * S + u) * C + c0, o);
    else {
#pragma unroll
      for (int i = 0; i < CV; ++i) o[i] = 0.f;
    }
  };
  // g = dy[u] (zero past the end gives dpre = 0)
  auto dpre = [&](int u, int j0, const float (&g)[CV], float (&o)[CV]) {   // x[u - K + 1] is xw[j0]
#pragma unroll
    for (int i = 0; i < CV; ++i) {
      float pre = 0.f;
#pragma unroll
      for (int k = 0; k < K; ++k) pre = fmaf(wk[i][k], xw[j0 + k][i], pre);
      const float sg = sigmoid_f(pre);
      o[i] = g[i] * sg * (1.f + pre * (1.f - sg));
    }
  };
  float dp[K][CV];                                        // dp[j] = dpre(t + j)
#pragma unroll
  for (int k = 0; k < K; ++k) {
    float g[CV];
    ldg(t0 + k, g);
    dpre(t0 + k, k, g, dp[k]);
  }
  float gn[CV];                                           // dy row of the next step's dpre, loaded one ahead
  ldg(t0 + K, gn);
  float dwa[CV][K];
#pragma unroll
  for (int i = 0; i < CV; ++i)
#pragma unroll
    for (int k = 0; k < K; ++k) dwa[i][k] = 0.f;
  const int t1 = min(S, t0 + CONV_TT);
  for (int t = t0; t < t1; ++t) {
    float o[CV];
#pragma unroll
    for (int i = 0; i < CV; ++i) {
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < K; ++k) acc = fmaf(wk[i][k], dp[K - 1 - k][i], acc);
      o[i] = acc;
#pragma unroll
      for (int k = 0; k < K; ++k) dwa[i][k] = fmaf(dp[0][i], xw[k][i], dwa[i][k]);
    }
    st_cv(dx + ((int64_t)b * S + t) * C + c0, o);
#pragma unroll
    for (int k = 0; k < K - 1; ++k)
#pragma unroll
      for (int i = 0; i < CV; ++i) dp[k][i] = dp[k + 1][i];
    float gc[CV];
#pragma unroll
    for (int i = 0; i < CV; ++i) gc[i] = gn[i];
    ldg(t + K + 1, gn);
    dpre(t + K, K, gc, dp[K - 1]);                        // x[t + 1 .. t + K] = xw[K .. 2K - 1]
#pragma unroll
    for (int j = 0; j < 2 * K - 1; ++j)
#pragma unroll
      for (int i = 0; i < CV; ++i) xw[j][i] = xw[j + 1][i];
    ldx(t + K + 1, xw[2 * K - 1]);
  }
  const int64_t pidx = ((int64_t)b * gridDim.y + tile);
#pragma unroll
  for (int i = 0; i < CV; ++i)
#pragma unroll
    for (int k = 0; k < K; ++k) dw_part[(pidx * C + c0 + i) * K + k] = dwa[i][k];
}

template <typename T>
static bool conv_vec_ok(int C, int64_t xs, const void* x, const void* other) {
  return C % CV == 0 && (xs * (int64_t)sizeof(T)) % (CV * sizeof(T)) == 0 &&
         (reinterpret_cast<uintptr_t>(x) % (CV * sizeof(T))) == 0 &&
         (reinterpret_cast<uintptr_t>(other) % (CV * sizeof(T))) == 0;
}

at::Tensor conv_silu_fwd(at::Tensor x, at::Tensor w) {
  c10::cuda::CUDAGuard guard(x.device());
  const int B = x.size(0), S = x.size(1), C = x.size(2), K = w.size(1);
  TORCH_CHECK(x.stride(2) == 1 && x.stride(0) == x.stride(1) * S, "conv: x rows must be uniformly strided");
  at::Tensor wc = w.to(at::kFloat).contiguous();
  at::Tensor y = at::empty({B, S, C}, x.options());
  dim3 grid((C + 127) / 128, (S + CONV_TT - 1) / CONV_TT, B);
  MAMF_DISPATCH_FLOAT_BF16(x.scalar_type(), "conv_silu_fwd", [&] {
    TORCH_CHECK(K == 4, "conv: kernel size 4 supported");
    if (conv_vec_ok<scalar_t>(C, x.stride(1), x.data_ptr(), y.data_ptr())) {
      dim3 gv((C / CV + 127) / 128, (S + CONV_TT - 1) / CONV_TT, B);
      conv_silu_fwd_vec_kernel<scalar_t, 4><<<gv, 128, 0, stream()>>>(
          (const scalar_t*)x.data_ptr(), wc.data_ptr<float>(), (scalar_t*)y.data_ptr(), S, C, x.stride(1));
    } else {
      conv_silu_fwd_kernel<scalar_t, 4><<<grid, 128, 0, stream()>>>(
          (const scalar_t*)x.data_ptr(), wc.data_ptr<float>(), (scalar_t*)y.data_ptr(), B, S, C, x.stride(1));
    }
  });
  MAMF_LAUNCH_CHECK();
  return y;
}

std::vector<at::Tensor> conv_silu_bwd(at::Tensor x, at::Tensor w, at::Tensor dy) {
  c10::cuda::CUDAGuard guard(x.device());
  const int B = x.size(0), S = x.size(1), C = x.size(2), K = w.size(1);
  dy = dy.contiguous();
  at::Tensor wc = w.to(at::kFloat).contiguous();
  at::Tensor dx = at::empty({B, S, C}, x.options());
  const int tiles = (S + CONV_TT - 1) / CONV_TT;
  at::Tensor part = at::empty({(int64_t)B * tiles, C, K}, x.options().dtype(at::kFloat));
  dim3 grid((C + 127) / 128, tiles, B);
  MAMF_DISPATCH_FLOAT_BF16(x.scalar_type(), "conv_silu_bwd", [&] {
    TORCH_CHECK(K == 4, "conv: kernel size 4 supported");
    if (conv_vec_ok<scalar_t>(C, x.stride(1), x.data_ptr(), dy.data_ptr())) {
      dim3 gv((C / CV + 127) / 128, tiles, B);
      conv_silu_bwd_vec_kernel<scalar_t, 4><<<gv, 128, 0, stream()>>>(
          (const scalar_t*)x.data_ptr(), wc.data_ptr<float>(), (const scalar_t*)dy.data_ptr(),
          (scalar_t*)dx.data_ptr(), part.data_ptr<float>(), S, C, x.stride(1));
    } else {
      conv_silu_bwd_kernel<scalar_t, 4><<<grid, 128, 0, stream()>>>(
          (const scalar_t*)x.data_ptr(), wc.data_ptr<float>(), (const scalar_t*)dy.data_ptr(),
          (scalar_t*)dx.data_ptr(), part.data_ptr<float>(), B, S, C, x.stride(1));
    }
  });
  MAMF_LAUNCH_CHECK();
  return {dx, part.sum(0)};
}

// ============================ per-head GroupNorm =============================================
// x (B, S, H*hd) contiguous.  Group (b, h) spans S x hd elements.  Pass 1: per (b, h, S-tile)
// partial (count, mean, M2); finalize combines them (Chan) in double; pass 2 normalises.
constexpr int GN_ROWS = 64;

// Stats / reduce block: x covers the head dimension (rounded up to 8 so that x * 4 threads
// fill whole warps - block_sum shuffles over all 32 lanes), y = 4 rows.  Threads with
// x >= hd contribute zeros.
static inline dim3 gn_block(int64_t hd) {
  const int64_t x = std::min<int64_t>(128, (hd + 7) / 8 * 8);
  return dim3((unsigned)x, 4);
}

template <typename T>
__global__ void gn_stats_kernel(const T* __restrict__ x, float* __restrict__ part, int S, int H, int hd) {
  const int b = blockIdx.z, h = blockIdx.y, tile = blockIdx.x;
  const int s0 = tile * GN_ROWS, s1 = min(S, s0 + GN_ROWS);
  const int C = H * hd;
  float sum = 0.f, sq = 0.f;
  for (int s = s0 + threadIdx.y; s < s1; s += blockDim.y)
    for (int j = threadIdx.x; j < hd; j += blockDim.x) {
      const float v = to_f(x[((int64_t)b * S + s) * C + (int64_t)h * hd + j]);
      sum += v; sq += v * v;
    }
  __shared__ float sm[64];
  const int lin = threadIdx.y * blockDim.x + threadIdx.x;
  sum = block_sum(sum, sm);
  sq = block_sum(sq, sm);
  if (lin == 0) {
    const int64_t o = (((int64_t)b * H + h) * gridDim.x + tile) * 3;
    const float n = (float)((s1 - s0) * hd);
    const float mean = sum / n;
    part[o] = n; part[o + 1] = mean; part[o + 2] = fmaxf(sq - sum * mean, 0.f);
  }
}

// Vector form of the stats pass: block = (hd / V) x (256 / (hd / V)) threads (hd / V a power of
// two <= 32), a thread reads V consecutive dims of a row with one 16-byte load.
template <typename T>
__global__ void __launch_bounds__(256) gn_stats_vec_kernel(const T* __restrict__ x, float* __restrict__ part, int S,
                                                          int H, int hd) {
  constexpr int V = 16 / sizeof(T);
  const int b = blockIdx.z, h = blockIdx.y, tile = blockIdx.x;
  const int s0 = tile * GN_ROWS, s1 = min(S, s0 + GN_ROWS);
  const int C = H * hd;
  float sum = 0.f, sq = 0.f;
  for (int s = s0 + threadIdx.y; s < s1; s += blockDim.y) {
    const Vec16<T> a = ld16(x + ((int64_t)b * S + s) * C + (int64_t)h * hd + threadIdx.x * V);
#pragma unroll
    for (int k = 0; k < V; ++k) { const float v = to_f(a.v[k]); sum += v; sq = fmaf(v, v, sq); }
  }
  __shared__ float sm[64];
  sum = block_sum(sum, sm);
  sq = block_sum(sq, sm);
  if (threadIdx.x == 0 && threadIdx.y == 0) {
    const int64_t o = (((int64_t)b * H + h) * gridDim.x + tile) * 3;
    const float n = (float)((s1 - s0) * hd);
    const float mean = sum / n;
    part[o] = n; part[o + 1] = mean; part[o + 2] = fmaxf(sq - sum * mean, 0.f);
  }
}

__global__ void gn_finalize_kernel(const float* __restrict__ part, float* __restrict__ mean_rstd,
                                   int groups, int tiles, float eps) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= groups) return;
  double n = 0, mean = 0, m2 = 0;
  for (int t = 0; t < tiles; ++t) {
    const float* q = part + ((int64_t)g * tiles + t) * 3;
    const double nb = q[0], mb = q[1], m2b = q[2];
    const double nt = n + nb;
    const double delta = mb - mean;
    mean += delta * nb / nt;
    m2 += m2b + delta * delta * n * nb / nt;
    n = nt;
  }
  mean_rstd[2 * g] = (float)mean;
  mean_rstd[2 * g + 1] = (float)(1.0 / sqrt(m2 / n + (double)eps));
}

template <typename T>
__global__ void gn_apply_kernel(const T* __restrict__ x, const float* __restrict__ mr,
                                const float* __restrict__ w, const float* __restrict__ bias,
                                T* __restrict__ y, int64_t rows, int S, int H, int hd) {
  const int C = H * hd;
  const int64_t total = rows * C;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const int64_t r = i / C;
    const int b = (int)(r / S), h = c / hd;
    const float m = mr[2 * (b * H + h)], rs = mr[2 * (b * H + h) + 1];
    y[i] = from_f<T>((to_f(x[i]) - m) * rs * w[c] + bias[c]);
  }
}

// backward pass 1: per (b, h, tile): sum(dy*w), sum(dy*w*xhat); per channel partial dw, db.
template <typename T>
__global__ void gn_bwd_reduce_kernel(const T* __restrict__ x, const T* __restrict__ dy,
                                     const float* __restrict__ mr, const float* __restrict__ w,
                                     float* __restrict__ gpart, float* __restrict__ wpart,
                                     int S, int H, int hd) {
  const int b = blockIdx.z, h = blockIdx.y, tile = blockIdx.x;
  const int s0 = tile * GN_ROWS, s1 = min(S, s0 + GN_ROWS);
  const int C = H * hd;
  const float m = mr[2 * (b * H + h)], rs = mr[2 * (b * H + h) + 1];
  float a1 = 0.f, a2 = 0.f;
  for (int j = threadIdx.x; j < hd; j += blockDim.x) {
    float dwj = 0.f, dbj = 0.f;
    for (int s = s0 + threadIdx.y; s < s1; s += blockDim.y) {
      const int64_t off = ((int64_t)b * S + s) * C + (int64_t)h * hd + j;
      const float xh = (to_f(x[off]) - m) * rs;
      const float d = to_f(dy[off]);
      const float g = d * w[h * hd + j];
      a1 += g; a2 += g * xh;
      dwj += d * xh; dbj += d;
    }
    const int64_t wo = ((((int64_t)b * gridDim.x + tile) * blockDim.y + threadIdx.y) * C + (int64_t)h * hd + j) * 2;
    wpart[wo] = dwj; wpart[wo + 1] = dbj;
  }
  __shared__ float sm[64];
  a1 = block_sum(a1, sm);
  a2 = block_sum(a2, sm);
  if (threadIdx.x == 0 && threadIdx.y == 0) {
    const int64_t o = (((int64_t)b * H + h) * gridDim.x + tile) * 2;
    gpart[o] = a1; gpart[o + 1] = a2;
  }
}

template <typename T>
__global__ void gn_bwd_dx_kernel(const T* __restrict__ x, const T* __restrict__ dy, const float* __restrict__ mr,
                                 const float* __restrict__ w, const float* __restrict__ gsum,
                                 T* __restrict__ dx, int64_t rows, int S, int H, int hd) {
  const int C = H * hd;
  const float inv_n = 1.f / ((float)S * hd);
  const int64_t total = rows * C;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const int64_t r = i / C;
    const int b = (int)(r / S), h = c / hd;
    const int g = b * H + h;
    const float m = mr[2 * g], rs = mr[2 * g + 1];
    const float xh = (to_f(x[i]) - m) * rs;
    const float gg = to_f(dy[i]) * w[c];
    dx[i] = from_f<T>(rs * (gg - gsum[2 * g] * inv_n - xh * gsum[2 * g + 1] * inv_n));
  }
}

// Vectorised forms of the apply / dx passes: one block per token row, a thread handles V
// consecutive channels (one head: hd % V == 0) with 16-byte loads and float4 weight reads.
template <typename T>
__global__ void gn_apply_vec_kernel(const T* __restrict__ x, const float* __restrict__ mr,
                                    const float* __restrict__ w, const float* __restrict__ bias,
                                    T* __restrict__ y, int S, int H, int hd) {
  constexpr int V = 16 / sizeof(T);
  const int C = H * hd;
  const int64_t r = blockIdx.x;
  const int b = (int)(r / S);
  for (int v = threadIdx.x; v < C / V; v += blockDim.x) {
    const int c = v * V, h = c / hd;
    const float m = mr[2 * (b * H + h)], rs = mr[2 * (b * H + h) + 1];
    const Vec16<T> a = ld16(x + r * C + c);
    float wv[V], bv[V];
    ld_w<V>(w, c, wv);
    ld_w<V>(bias, c, bv);
    Vec16<T> o;
#pragma unroll
    for (int k = 0; k < V; ++k) o.v[k] = from_f<T>(fmaf((to_f(a.v[k]) - m) * rs, wv[k], bv[k]));
    st16(y + r * C + c, o);
  }
}

template <typename T>
__global__ void gn_bwd_dx_vec_kernel(const T* __restrict__ x, const T* __restrict__ dy, const float* __restrict__ mr,
                                     const float* __restrict__ w, const float* __restrict__ gsum,
                                     T* __restrict__ dx, int S, int H, int hd) {
  constexpr int V = 16 / sizeof(T);
  const int C = H * hd;
  const float inv_n = 1.f / ((float)S * hd);
  const int64_t r = blockIdx.x;
  const int b = (int)(r / S);
  for (int v = threadIdx.x; v < C / V; v += blockDim.x) {
    const int c = v * V, g = b * H + c / hd;
    const float m = mr[2 * g], rs = mr[2 * g + 1];
    const float g1 = gsum[2 * g] * inv_n, g2 = gsum[2 * g + 1] * inv_n;
    const Vec16<T> a = ld16(x + r * C + c), d = ld16(dy + r * C + c);
    float wv[V];
    ld_w<V>(w, c, wv);
    Vec16<T> o;
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const float xh = (to_f(a.v[k]) - m) * rs;
      o.v[k] = from_f<T>(rs * (to_f(d.v[k]) * wv[k] - g1 - xh * g2));
    }
    st16(dx + r * C + c, o);
  }
}

template <typename T>
static bool gn_vec_ok(int hd, int64_t rows, const void* a, const void* b, const void* c) {
  constexpr int V = 16 / sizeof(T);
  return hd % V == 0 && rows > 0 && rows <= INT32_MAX && aligned16(a) && aligned16(b) && aligned16(c);
}

// Stats, finalize and apply passes of the forward.  Shared by head_groupnorm_fwd and the
// allocation-free entry point at the end of this file, so both pick the same kernels (16-byte
// forms when hd, the row count and the pointers allow) and give bitwise-equal results.
template <typename T>
static void gn_fwd_launch(const T* x, const float* w, const float* bias, T* y, float* part, float* mr, int B, int S,
                          int H, int hd, int tiles, float eps, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  const int nx = hd / V;
  const int64_t rows = (int64_t)B * S;
  if (hd % V == 0 && nx > 0 && nx <= 32 && (nx & (nx - 1)) == 0 && aligned16(x))
    gn_stats_vec_kernel<T><<<dim3(tiles, H, B), dim3(nx, 256 / nx), 0, st>>>(x, part, S, H, hd);
  else
    gn_stats_kernel<T><<<dim3(tiles, H, B), gn_block(hd), 0, st>>>(x, part, S, H, hd);
  gn_finalize_kernel<<<(B * H + 127) / 128, 128, 0, st>>>(part, mr, B * H, tiles, eps);
  if (gn_vec_ok<T>(hd, rows, x, w, bias) && aligned16(y))
    gn_apply_vec_kernel<T><<<(unsigned)rows, 256, 0, st>>>(x, mr, w, bias, y, S, H, hd);
  else
    gn_apply_kernel<T><<<ew_blocks(rows * H * hd), 256, 0, st>>>(x, mr, w, bias, y, rows, S, H, hd);
}

std::vector<at::Tensor> head_groupnorm_fwd(at::Tensor x, int64_t H, at::Tensor w, at::Tensor bias, double eps) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.is_contiguous() && x.dim() == 3, "groupnorm: contiguous (B, S, C)");
  const int B = x.size(0), S = x.size(1), C = x.size(2), hd = C / H;
  const int tiles = (S + GN_ROWS - 1) / GN_ROWS;
  auto f32 = x.options().dtype(at::kFloat);
  at::Tensor part = at::empty({(int64_t)B * H * tiles * 3}, f32);
  at::Tensor mr = at::empty({(int64_t)B * H, 2}, f32);
  at::Tensor y = at::empty_like(x);
  at::Tensor wc = w.to(at::kFloat).contiguous(), bc = bias.to(at::kFloat).contiguous();
  MAMF_DISPATCH_FLOAT_BF16(x.scalar_type(), "gn_fwd", [&] {
    gn_fwd_launch<scalar_t>((const scalar_t*)x.data_ptr(), wc.data_ptr<float>(), bc.data_ptr<float>(),
                            (scalar_t*)y.data_ptr(), part.data_ptr<float>(), mr.data_ptr<float>(), B, S, (int)H, hd,
                            tiles, (float)eps, stream());
  });
  MAMF_LAUNCH_CHECK();
  return {y, mr};
}

std::vector<at::Tensor> head_groupnorm_bwd(at::Tensor x, int64_t H, at::Tensor w, at::Tensor mr, at::Tensor dy) {
  c10::cuda::CUDAGuard guard(x.device());
  dy = dy.contiguous();
  const int B = x.size(0), S = x.size(1), C = x.size(2), hd = C / H;
  const int tiles = (S + GN_ROWS - 1) / GN_ROWS;
  auto f32 = x.options().dtype(at::kFloat);
  const int by = 4;
  at::Tensor gpart = at::empty({(int64_t)B * H, tiles, 2}, f32);
  at::Tensor wpart = at::empty({(int64_t)B * tiles * by, C, 2}, f32);
  at::Tensor dx = at::empty_like(x);
  at::Tensor wc = w.to(at::kFloat).contiguous();
  MAMF_DISPATCH_FLOAT_BF16(x.scalar_type(), "gn_bwd", [&] {
    gn_bwd_reduce_kernel<scalar_t><<<dim3(tiles, H, B), gn_block(hd), 0, stream()>>>(
        (const scalar_t*)x.data_ptr(), (const scalar_t*)dy.data_ptr(), mr.data_ptr<float>(), wc.data_ptr<float>(),
        gpart.data_ptr<float>(), wpart.data_ptr<float>(), S, H, hd);
    at::Tensor gsum = gpart.sum(1).contiguous();
    if (gn_vec_ok<scalar_t>(hd, (int64_t)B * S, x.data_ptr(), dy.data_ptr(), wc.data_ptr()))
      gn_bwd_dx_vec_kernel<scalar_t><<<(unsigned)((int64_t)B * S), 256, 0, stream()>>>(
          (const scalar_t*)x.data_ptr(), (const scalar_t*)dy.data_ptr(), mr.data_ptr<float>(), wc.data_ptr<float>(),
          gsum.data_ptr<float>(), (scalar_t*)dx.data_ptr(), S, H, hd);
    else
      gn_bwd_dx_kernel<scalar_t><<<ew_blocks(x.numel()), 256, 0, stream()>>>(
          (const scalar_t*)x.data_ptr(), (const scalar_t*)dy.data_ptr(), mr.data_ptr<float>(), wc.data_ptr<float>(),
          gsum.data_ptr<float>(), (scalar_t*)dx.data_ptr(), (int64_t)B * S, S, H, hd);
  });
  MAMF_LAUNCH_CHECK();
  at::Tensor wsum = wpart.sum(0);
  return {dx, wsum.select(1, 0), wsum.select(1, 1)};
}

}  // namespace mamf

// ============================ allocation-free GroupNorm forward ==============================
// See noalloc.h: same kernels as head_groupnorm_fwd, scratch in a fixed device array.
#include <mutex>
#include <stdio.h>

#include "noalloc.h"

namespace mamf {
namespace noalloc {

static __device__ __align__(256) float g_scratch[MAMF_NOALLOC_SCRATCH_FLOATS];

constexpr int kMaxDevices = 64;
static float* g_scratch_addr[kMaxDevices];    // device address of g_scratch, per device
static std::mutex g_setup_mutex;
static thread_local char g_msg[256] = "";

static int fail(int code, const char* msg) {
  snprintf(g_msg, sizeof(g_msg), "%s", msg);
  return code;
}

// Device address of the scratch array on the current device (looked up once per device).
static int scratch_address(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(3, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(1, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess) return fail(3, cudaGetErrorString(e));
    g_scratch_addr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_addr[dev];
  return 0;
}

// Drop the cached address of the current device; the next call looks it up again.  Used after
// a failed launch: if the failure came from a context that was reset, the old address is stale.
static void forget_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  g_scratch_addr[dev] = nullptr;
}

}  // namespace noalloc
}  // namespace mamf

extern "C" __attribute__((visibility("default")))
const char* mamf_noalloc_last_error(void) { return mamf::noalloc::g_msg; }

extern "C" __attribute__((visibility("default")))
int mamf_head_groupnorm_fwd_noalloc(const void* x, const float* w, const float* b, void* y,
                                    float* mean_rstd_out, int64_t B, int64_t S, int64_t H, int64_t hd,
                                    float eps, int dtype, void* stream_ptr) {
  using namespace mamf;
  if (!x || !w || !b || !y || B <= 0 || S <= 0 || H <= 0 || hd <= 0 || (dtype != 0 && dtype != 1))
    return noalloc::fail(1, "invalid arguments");
  // Index types of the kernels: grid y/z hold H and B; S, hd and C = H*hd are int; element
  // offsets are int64.  Check each factor before any product can overflow.
  if (B > 65535 || H > 65535) return noalloc::fail(1, "B and H must be <= 65535");
  if (S > INT32_MAX || hd > INT32_MAX || H * hd > INT32_MAX)
    return noalloc::fail(1, "S, hd and H*hd must fit in int32");
  if (B * S > INT64_MAX / (H * hd)) return noalloc::fail(1, "B*S*H*hd overflows int64");
  const int64_t tiles = (S + GN_ROWS - 1) / GN_ROWS;
  // B*H <= 2^32 and tiles <= 2^25, so this product fits easily in int64.
  const int64_t part_floats = B * H * tiles * 3;
  const int64_t mr_floats = mean_rstd_out ? 0 : 2 * B * H;
  if (part_floats + mr_floats > MAMF_NOALLOC_SCRATCH_FLOATS) {
    char buf[200];
    snprintf(buf, sizeof(buf), "problem needs %lld scratch floats, the fixed array holds %d",
             (long long)(part_floats + mr_floats), MAMF_NOALLOC_SCRATCH_FLOATS);
    return noalloc::fail(2, buf);
  }
  // A launch error left behind by earlier, unrelated work on this thread is reported as such
  // (and cleared) instead of being attributed to this call's kernels.
  const cudaError_t prior = cudaGetLastError();
  if (prior != cudaSuccess) {
    char buf[200];
    snprintf(buf, sizeof(buf), "a CUDA error was pending before this call (nothing launched): %s",
             cudaGetErrorString(prior));
    return noalloc::fail(3, buf);
  }
  float* scratch = nullptr;
  if (int rc = noalloc::scratch_address(&scratch)) return rc;
  float* part = scratch;
  float* mr = mean_rstd_out ? mean_rstd_out : scratch + part_floats;
  cudaStream_t st = static_cast<cudaStream_t>(stream_ptr);
  const int Bi = (int)B, Si = (int)S, Hi = (int)H, hdi = (int)hd;
  if (dtype == 1)
    gn_fwd_launch<__nv_bfloat16>((const __nv_bfloat16*)x, w, b, (__nv_bfloat16*)y, part, mr, Bi, Si, Hi, hdi,
                                 (int)tiles, eps, st);
  else
    gn_fwd_launch<float>((const float*)x, w, b, (float*)y, part, mr, Bi, Si, Hi, hdi, (int)tiles, eps, st);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    noalloc::forget_current_device();   // a reset context invalidates the cached address
    return noalloc::fail(3, cudaGetErrorString(e));
  }
  noalloc::g_msg[0] = '\0';
  return 0;
}
