// Muon element-wise passes around the batched Newton-Schulz GEMMs.
//
//   muon_momentum : M <- mu M + G  (in place), U = mu M + G, per-matrix sum of U^2
//   muon_normalize: Y = U / (||U||_F + eps) as bf16 (the Newton-Schulz input)
//   muon_apply    : W <- W (1 - lr wd) - (lr * scale) O
//   adamw_multi   : decoupled-weight-decay Adam over a table of tensors in one launch
//
// Tensors are flat views of one parameter holding `n / slice` matrices of `slice`
// elements each (a 2-D weight is one slice; stacked expert weights hold E slices).
#include <ATen/cuda/CUDAContext.h>
#include <cmath>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace sv4 {

template <typename T> __device__ __forceinline__ float ld(const T* p, int64_t i);
template <> __device__ __forceinline__ float ld<float>(const float* p, int64_t i) { return p[i]; }
template <> __device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}
template <typename T> __device__ __forceinline__ void st(T* p, int64_t i, float v);
template <> __device__ __forceinline__ void st<float>(float* p, int64_t i, float v) { p[i] = v; }
template <> __device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, int64_t i, float v) {
  p[i] = __float2bfloat16(v);
}

// Grid: (blocks_per_slice, n_slices).  Each block reduces its part of one slice.
template <typename TM>
__global__ void muon_momentum_kernel(TM* __restrict__ m, const float* __restrict__ g, float* __restrict__ sumsq,
                                     int64_t slice, float mu) {
  const int64_t base = static_cast<int64_t>(blockIdx.y) * slice;
  float acc = 0.f;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < slice;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float gi = g[base + i];
    const float mi = mu * ld(m, base + i) + gi;
    st(m, base + i, mi);
    const float ui = mu * mi + gi;
    acc += ui * ui;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) atomicAdd(&sumsq[blockIdx.y], v);
  }
}

template <typename TM>
__global__ void muon_normalize_kernel(const TM* __restrict__ m, const float* __restrict__ g,
                                      const float* __restrict__ sumsq, __nv_bfloat16* __restrict__ y, int64_t slice,
                                      float mu, float eps) {
  const int64_t base = static_cast<int64_t>(blockIdx.y) * slice;
  const float inv = 1.0f / (sqrtf(sumsq[blockIdx.y]) + eps);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < slice;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    y[base + i] = __float2bfloat16((mu * ld(m, base + i) + g[base + i]) * inv);
  }
}

template <typename TP>
__global__ void muon_apply_kernel(TP* __restrict__ p, const __nv_bfloat16* __restrict__ o, int64_t n, float decay,
                                  float step) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    st(p, i, ld(p, i) * decay - step * __bfloat162float(o[i]));
  }
}

static dim3 slice_grid(int64_t slice, int64_t n_slices) {
  const int64_t per = std::max<int64_t>(1, std::min<int64_t>((slice + 255) / 256, 4096 / std::max<int64_t>(1, n_slices) + 1));
  return dim3(static_cast<unsigned>(per), static_cast<unsigned>(n_slices));
}

void muon_momentum(torch::Tensor m, torch::Tensor g, torch::Tensor sumsq, int64_t slice, double mu) {
  c10::cuda::CUDAGuard guard(m.device());
  TORCH_CHECK(m.is_contiguous() && g.is_contiguous() && g.scalar_type() == at::kFloat, "muon_momentum layout");
  const int64_t n_slices = m.numel() / slice;
  sumsq.zero_();
  auto s = at::cuda::getCurrentCUDAStream();
  dim3 grid = slice_grid(slice, n_slices);
  if (m.scalar_type() == at::kBFloat16) {
    muon_momentum_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(m.data_ptr()), g.data_ptr<float>(),
                                              sumsq.data_ptr<float>(), slice, static_cast<float>(mu));
  } else {
    muon_momentum_kernel<<<grid, 256, 0, s>>>(m.data_ptr<float>(), g.data_ptr<float>(), sumsq.data_ptr<float>(),
                                              slice, static_cast<float>(mu));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void muon_normalize(torch::Tensor m, torch::Tensor g, torch::Tensor sumsq, torch::Tensor y, int64_t slice, double mu,
                    double eps) {
  c10::cuda::CUDAGuard guard(m.device());
  const int64_t n_slices = m.numel() / slice;
  auto s = at::cuda::getCurrentCUDAStream();
  dim3 grid = slice_grid(slice, n_slices);
  auto yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  if (m.scalar_type() == at::kBFloat16) {
    muon_normalize_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(m.data_ptr()),
                                               g.data_ptr<float>(), sumsq.data_ptr<float>(), yp, slice,
                                               static_cast<float>(mu), static_cast<float>(eps));
  } else {
    muon_normalize_kernel<<<grid, 256, 0, s>>>(m.data_ptr<float>(), g.data_ptr<float>(), sumsq.data_ptr<float>(), yp,
                                               slice, static_cast<float>(mu), static_cast<float>(eps));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void muon_apply(torch::Tensor p, torch::Tensor o, double decay, double step) {
  c10::cuda::CUDAGuard guard(p.device());
  TORCH_CHECK(p.is_contiguous() && o.is_contiguous() && o.scalar_type() == at::kBFloat16, "muon_apply layout");
  const int64_t n = p.numel();
  if (n == 0) return;
  auto s = at::cuda::getCurrentCUDAStream();
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 32));
  auto op = reinterpret_cast<const __nv_bfloat16*>(o.data_ptr());
  if (p.scalar_type() == at::kBFloat16) {
    muon_apply_kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(p.data_ptr()), op, n,
                                             static_cast<float>(decay), static_cast<float>(step));
  } else {
    muon_apply_kernel<<<blocks, 256, 0, s>>>(p.data_ptr<float>(), op, n, static_cast<float>(decay),
                                             static_cast<float>(step));
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------ AdamW, multi-tensor
// One entry per parameter: fp32 gradient (main_grad), the parameter (bf16 or fp32) and its
// fp32 moments.  The grid walks a chunk list (entry, first element) so one launch covers
// every AdamW parameter of the optimizer group:
//   m <- b1 m + (1 - b1) g;  v <- b2 v + (1 - b2) g^2
//   p <- p (1 - lr wd) - lr (m / bc1) / (sqrt(v / bc2) + eps)
struct AdamEntry {
  const float* g;
  void* p;
  float* m;
  float* v;
  int64_t n;
  int64_t bf16;
};

constexpr int64_t kAdamChunk = 1 << 16;

__global__ void __launch_bounds__(256) adamw_multi_kernel(const AdamEntry* __restrict__ entries,
                                                          const int64_t* __restrict__ chunks, float lr, float b1,
                                                          float b2, float eps, float wd, float inv_bc1,
                                                          float inv_bc2) {
  const int64_t c = chunks[blockIdx.x];
  const AdamEntry e = entries[c >> 32];
  const int64_t start = (c & 0xFFFFFFFFll) * kAdamChunk;
  const int64_t end = min(e.n, start + kAdamChunk);
  const float decay = 1.f - lr * wd;
  for (int64_t i = start + threadIdx.x; i < end; i += blockDim.x) {
    const float g = e.g[i];
    const float m = b1 * e.m[i] + (1.f - b1) * g;
    const float v = b2 * e.v[i] + (1.f - b2) * g * g;
    e.m[i] = m;
    e.v[i] = v;
    const float upd = (m * inv_bc1) / (sqrtf(v * inv_bc2) + eps);
    if (e.bf16) {
      __nv_bfloat16* p = static_cast<__nv_bfloat16*>(e.p);
      p[i] = __float2bfloat16(__bfloat162float(p[i]) * decay - lr * upd);
    } else {
      float* p = static_cast<float*>(e.p);
      p[i] = p[i] * decay - lr * upd;
    }
  }
}

// table: (n_entries, 6) int64 on the device (AdamEntry rows); chunks: (n_chunks) int64 on
// the device, entry << 32 | chunk index.
void adamw_multi(torch::Tensor table, torch::Tensor chunks, double lr, double beta1, double beta2, double eps,
                 double weight_decay, double step) {
  TORCH_CHECK(table.scalar_type() == at::kLong && table.is_cuda() && table.dim() == 2 && table.size(1) == 6,
              "table: (entries, 6) int64 on the device");
  TORCH_CHECK(chunks.scalar_type() == at::kLong && chunks.is_cuda() && chunks.dim() == 1, "chunks: int64");
  static_assert(sizeof(AdamEntry) == 6 * sizeof(int64_t), "AdamEntry layout");
  const int64_t n_chunks = chunks.numel();
  if (n_chunks == 0) return;
  c10::cuda::CUDAGuard guard(table.device());
  const float inv_bc1 = static_cast<float>(1.0 / (1.0 - std::pow(beta1, step)));
  const float inv_bc2 = static_cast<float>(1.0 / (1.0 - std::pow(beta2, step)));
  adamw_multi_kernel<<<static_cast<unsigned>(n_chunks), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const AdamEntry*>(table.data_ptr<int64_t>()), chunks.data_ptr<int64_t>(),
      static_cast<float>(lr), static_cast<float>(beta1), static_cast<float>(beta2), static_cast<float>(eps),
      static_cast<float>(weight_decay), inv_bc1, inv_bc2);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t adamw_chunk_elems() { return kAdamChunk; }

}  // namespace sv4
