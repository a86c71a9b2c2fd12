// Data-parallel gradient all-reduce over NVLink peer memory (no NCCL on this path).
//
// The fp32 gradient segments of a data-parallel group live in symmetric memory (every rank maps
// every peer's buffer).  A bucket [lo, hi) of a segment is reduced in place on every rank:
//
//   NVLS (NVSwitch multicast object available): rank r owns slice r of the bucket; for each
//     16-byte word it issues one multimem.ld_reduce on the multicast address (the switch returns
//     the sum over all GPUs), scales it, and one multimem.st that writes the result into every
//     GPU's copy.  Each word crosses NVLink once in and once out per GPU.
//   two-shot (plain P2P): phase 1 - rank r reads slice r from every peer (P2P loads, fixed rank
//     order, so the sum is the same bits whoever computes it), scales it and stores it into its
//     own slice; phase 2 - rank r copies slice q from its owner q for every q != r.
//
// The caller orders the phases with the bounded signal-pad barrier (before: every peer finished
// accumulating the bucket; between the phases; after: every peer finished reading this rank's
// slice), all on one side stream so the reduction overlaps the rest of the backward pass.
// The scale folds the 1/world averaging (and anything else the caller wants) into the pass.
// Optionally each owner writes the sum of squares of its reduced slice (per block, summed by the
// caller in index order) so the gradient norm needs no second pass over the gradients.
//
// Replaces the reference's FSDP gradient reduce-scatter (scripts/train.py:243-252, C10).
#include "common.cuh"

namespace mamf {
namespace dpg {

constexpr int MAXP = 8;
struct Ptrs { float* p[MAXP]; };

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

__device__ __forceinline__ void block_partial(float acc, float* sq, float* sm) {
  acc = block_sum(acc, sm);
  if (sq != nullptr && threadIdx.x == 0) sq[blockIdx.x] = acc;
}

// phase 1 of two-shot: dst[i] = scale * sum_r src_r[i] over my slice [s0, s1) (multiple of 4)
__global__ void rs_kernel(Ptrs src, int P, float* __restrict__ dst, int64_t s0, int64_t s1, float scale,
                          float* __restrict__ sq) {
  __shared__ float sm[32];
  float acc = 0.f;
  const int64_t n4 = (s1 - s0) / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = s0 + 4 * i;
    float4 a = ld4(src.p[0] + e);
#pragma unroll
    for (int r = 1; r < MAXP; ++r) {
      if (r < P) {
        const float4 b = ld4(src.p[r] + e);
        a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
      }
    }
    a.x *= scale; a.y *= scale; a.z *= scale; a.w *= scale;
    acc += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
    st4(dst + e, a);
  }
  block_partial(acc, sq, sm);
}

// phase 2 of two-shot: for every owner q != me copy slice q of q's buffer into mine
__global__ void ag_kernel(Ptrs src, int me, float* __restrict__ dst, int64_t lo, int64_t slice, int64_t hi) {
  const int q = blockIdx.y;
  if (q == me) return;
  const int64_t s0 = lo + q * slice, s1 = min(hi, s0 + slice);
  const int64_t n4 = s1 > s0 ? (s1 - s0) / 4 : 0;
  const float* s = src.p[q];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x)
    st4(dst + s0 + 4 * i, ld4(s + s0 + 4 * i));
}

// NVLS: switch-side reduction and multicast store of my slice
__global__ void nvls_kernel(float* mc, int64_t s0, int64_t s1, float scale, float* __restrict__ sq) {
  __shared__ float sm[32];
  float acc = 0.f;
  const int64_t n4 = (s1 - s0) / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float* a = mc + s0 + 4 * i;
    float x, y, z, w;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(x), "=f"(y), "=f"(z), "=f"(w) : "l"(a) : "memory");
    x *= scale; y *= scale; z *= scale; w *= scale;
    acc += x * x + y * y + z * z + w * w;
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};"
                 :: "l"(a), "f"(x), "f"(y), "f"(z), "f"(w) : "memory");
  }
  block_partial(acc, sq, sm);
}

int grid_for(int64_t n4) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((n4 + 255) / 256, (int64_t)num_sms() * 2));
}

}  // namespace dpg

// slice of rank r in a bucket [lo, hi): [lo + r * slice, min(hi, lo + (r + 1) * slice)), slice a
// multiple of 4 elements so every word is 16-byte aligned (lo is a multiple of 4).
int64_t dp_slice(int64_t lo, int64_t hi, int64_t P) {
  const int64_t n = hi - lo;
  return ((n + P - 1) / P + 3) / 4 * 4;
}

static void check_bucket(int64_t lo, int64_t hi) {
  TORCH_CHECK(lo >= 0 && hi >= lo && lo % 4 == 0 && hi % 4 == 0, "dp grad: bucket bounds must be multiples of 4");
}

// Phase 1 (two-shot).  bufs: every rank's buffer base (fp32 element 0), this rank's at index me.
// Returns per-block squared sums of the reduced slice when want_sq.
at::Tensor dp_reduce_scatter(std::vector<int64_t> bufs, int64_t me, int64_t lo, int64_t hi, double scale,
                             bool want_sq) {
  const int P = (int)bufs.size();
  TORCH_CHECK(P >= 1 && P <= dpg::MAXP && me >= 0 && me < P, "dp_reduce_scatter: 1..8 ranks");
  check_bucket(lo, hi);
  dpg::Ptrs src{};
  for (int i = 0; i < P; ++i) {
    src.p[i] = reinterpret_cast<float*>(bufs[i]);
    TORCH_CHECK((bufs[i] & 15) == 0, "dp_reduce_scatter: 16-byte aligned buffers");
  }
  const int64_t slice = dp_slice(lo, hi, P);
  const int64_t s0 = std::min(hi, lo + me * slice), s1 = std::min(hi, s0 + slice);
  const int grid = dpg::grid_for((s1 - s0) / 4);
  auto sq = at::zeros({want_sq ? grid : 0}, at::TensorOptions().device(at::kCUDA, c10::cuda::current_device()).dtype(at::kFloat));
  if (s1 > s0)
    dpg::rs_kernel<<<grid, 256, 0, stream()>>>(src, P, src.p[me], s0, s1, (float)scale,
                                              want_sq ? sq.data_ptr<float>() : nullptr);
  MAMF_LAUNCH_CHECK();
  return sq;
}

// Phase 2 (two-shot).
void dp_all_gather(std::vector<int64_t> bufs, int64_t me, int64_t lo, int64_t hi) {
  const int P = (int)bufs.size();
  TORCH_CHECK(P >= 1 && P <= dpg::MAXP && me >= 0 && me < P, "dp_all_gather: 1..8 ranks");
  check_bucket(lo, hi);
  dpg::Ptrs src{};
  for (int i = 0; i < P; ++i) src.p[i] = reinterpret_cast<float*>(bufs[i]);
  const int64_t slice = dp_slice(lo, hi, P);
  dim3 grid(dpg::grid_for(slice / 4) / P + 1, P);
  dpg::ag_kernel<<<grid, 256, 0, stream()>>>(src, (int)me, src.p[me], lo, slice, hi);
  MAMF_LAUNCH_CHECK();
}

// NVLS all-reduce of this rank's slice through the multicast address of the buffer.
at::Tensor dp_allreduce_nvls(int64_t mc_base, int64_t P, int64_t me, int64_t lo, int64_t hi, double scale,
                             bool want_sq) {
  TORCH_CHECK(P >= 1 && me >= 0 && me < P && mc_base != 0 && (mc_base & 15) == 0, "dp_allreduce_nvls: bad args");
  check_bucket(lo, hi);
  const int64_t slice = dp_slice(lo, hi, P);
  const int64_t s0 = std::min(hi, lo + me * slice), s1 = std::min(hi, s0 + slice);
  const int grid = dpg::grid_for((s1 - s0) / 4);
  auto sq = at::zeros({want_sq ? grid : 0}, at::TensorOptions().device(at::kCUDA, c10::cuda::current_device()).dtype(at::kFloat));
  if (s1 > s0)
    dpg::nvls_kernel<<<grid, 256, 0, stream()>>>(reinterpret_cast<float*>(mc_base), s0, s1, (float)scale,
                                                want_sq ? sq.data_ptr<float>() : nullptr);
  MAMF_LAUNCH_CHECK();
  return sq;
}

}  // namespace mamf
