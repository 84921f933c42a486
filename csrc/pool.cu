// Token-level compressor pooling of CSA / HCA (and of the lightning indexer's keys), forward
// and backward in one kernel each:
//
//   out[b, s, :] = sum_j p_j c[b, s*m + j, :],   p_j = softmax_j(z[b, s*m + j, :] + bias[j, :])
//
// (softmax over the m tokens of a block, per channel; reference core/attention/csa.py
// TokenLevelCompressor).  Backward, with g = dout[b, s, :]:
//
//   dc_j = p_j g,   dz_j = p_j g (c_j - out)   (bias gradient: the sum of dz_j over b and s)
//
// One thread per (b, s, channel) walks the m tokens twice (max, then exponentials); c and z
// are bf16 column slices of a wider projection output (row stride ld), out / dout fp32.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

namespace sv4 {
namespace {

template <typename TB>
__device__ __forceinline__ float bias_at(const TB* bias, int64_t i);
template <>
__device__ __forceinline__ float bias_at<float>(const float* bias, int64_t i) { return bias[i]; }
template <>
__device__ __forceinline__ float bias_at<__nv_bfloat16>(const __nv_bfloat16* bias, int64_t i) {
  return __bfloat162float(bias[i]);
}

template <typename TB>
__global__ void pool_fwd_kernel(const __nv_bfloat16* __restrict__ c, const __nv_bfloat16* __restrict__ z,
                                int64_t ld_c, int64_t ld_z, const TB* __restrict__ bias, int T, int n, int m, int C,
                                float* __restrict__ out, int64_t total) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int ch = static_cast<int>(i % C);
  const int64_t bs = i / C;
  const int s = static_cast<int>(bs % n);
  const int64_t b = bs / n;
  const int64_t row0 = b * T + static_cast<int64_t>(s) * m;
  float mx = -INFINITY;
  for (int j = 0; j < m; ++j)
    mx = fmaxf(mx, __bfloat162float(z[(row0 + j) * ld_z + ch]) + bias_at<TB>(bias, static_cast<int64_t>(j) * C + ch));
  float den = 0.f, num = 0.f;
  for (int j = 0; j < m; ++j) {
    const float e = __expf(__bfloat162float(z[(row0 + j) * ld_z + ch]) +
                           bias_at<TB>(bias, static_cast<int64_t>(j) * C + ch) - mx);
    den += e;
    num += e * __bfloat162float(c[(row0 + j) * ld_c + ch]);
  }
  out[i] = num / den;
}

template <typename TB>
__global__ void pool_bwd_kernel(const __nv_bfloat16* __restrict__ c, const __nv_bfloat16* __restrict__ z,
                                int64_t ld_c, int64_t ld_z, const TB* __restrict__ bias, int T, int n, int m, int C,
                                const float* __restrict__ out, const float* __restrict__ dout,
                                __nv_bfloat16* __restrict__ dc, __nv_bfloat16* __restrict__ dz,
                                float* __restrict__ dz_f32, int64_t total) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int ch = static_cast<int>(i % C);
  const int64_t bs = i / C;
  const int s = static_cast<int>(bs % n);
  const int64_t b = bs / n;
  const int64_t row0 = b * T + static_cast<int64_t>(s) * m;
  float mx = -INFINITY;
  for (int j = 0; j < m; ++j)
    mx = fmaxf(mx, __bfloat162float(z[(row0 + j) * ld_z + ch]) + bias_at<TB>(bias, static_cast<int64_t>(j) * C + ch));
  float den = 0.f;
  for (int j = 0; j < m; ++j)
    den += __expf(__bfloat162float(z[(row0 + j) * ld_z + ch]) + bias_at<TB>(bias, static_cast<int64_t>(j) * C + ch) -
                  mx);
  const float g = dout[i], o = out[i], inv = 1.f / den;
  for (int j = 0; j < m; ++j) {
    const int64_t r = row0 + j;
    const float p = __expf(__bfloat162float(z[r * ld_z + ch]) + bias_at<TB>(bias, static_cast<int64_t>(j) * C + ch) -
                           mx) * inv;
    const float cj = __bfloat162float(c[r * ld_c + ch]);
    const float dzj = p * g * (cj - o);
    dc[r * C + ch] = __float2bfloat16(p * g);
    dz[r * C + ch] = __float2bfloat16(dzj);
    dz_f32[(bs * m + j) * C + ch] = dzj;  // (b, s, j, ch): summed over (b, s) for the bias
  }
}

}  // namespace

// c, z: (B, T, C) bf16 views with unit channel stride (row stride may exceed C); bias (m, C)
// fp32 or bf16; out (B, n, C) fp32 with n = T / m.
void compress_pool_fwd(torch::Tensor c, torch::Tensor z, torch::Tensor bias, int64_t m, torch::Tensor out) {
  TORCH_CHECK(c.dim() == 3 && z.sizes() == c.sizes() && c.stride(2) == 1 && z.stride(2) == 1 &&
                  c.scalar_type() == at::kBFloat16 && z.scalar_type() == at::kBFloat16, "c / z: (B, T, C) bf16");
  TORCH_CHECK(c.stride(0) == c.size(1) * c.stride(1) && z.stride(0) == z.size(1) * z.stride(1),
              "c / z rows must be evenly strided across the batch");
  const int64_t B = c.size(0), T = c.size(1), C = c.size(2), n = T / m;
  TORCH_CHECK(bias.is_contiguous() && bias.size(0) == m && bias.size(1) == C, "bias (m, C)");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() == B * n * C, "out (B, n, C)");
  const int64_t total = B * n * C;
  if (total == 0) return;
  c10::cuda::CUDAGuard guard(c.device());
  const unsigned grid = static_cast<unsigned>((total + 255) / 256);
  auto st = at::cuda::getCurrentCUDAStream();
  auto cp = reinterpret_cast<const __nv_bfloat16*>(c.data_ptr());
  auto zp = reinterpret_cast<const __nv_bfloat16*>(z.data_ptr());
  if (bias.scalar_type() == at::kFloat) {
    pool_fwd_kernel<float><<<grid, 256, 0, st>>>(cp, zp, c.stride(1), z.stride(1), bias.data_ptr<float>(),
                                                 static_cast<int>(T), static_cast<int>(n), static_cast<int>(m),
                                                 static_cast<int>(C), out.data_ptr<float>(), total);
  } else {
    TORCH_CHECK(bias.scalar_type() == at::kBFloat16, "bias fp32 or bf16");
    pool_fwd_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        cp, zp, c.stride(1), z.stride(1), reinterpret_cast<const __nv_bfloat16*>(bias.data_ptr()),
        static_cast<int>(T), static_cast<int>(n), static_cast<int>(m), static_cast<int>(C), out.data_ptr<float>(),
        total);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// dc, dz: (B, T, C) bf16 contiguous (rows past n * m untouched by the kernel: the caller
// zeroes them); dz_f32: (B, n, m, C) fp32 scratch for the bias gradient.
void compress_pool_bwd(torch::Tensor c, torch::Tensor z, torch::Tensor bias, int64_t m, torch::Tensor out,
                       torch::Tensor dout, torch::Tensor dc, torch::Tensor dz, torch::Tensor dz_f32) {
  const int64_t B = c.size(0), T = c.size(1), C = c.size(2), n = T / m;
  TORCH_CHECK(dout.scalar_type() == at::kFloat && dout.is_contiguous() && dout.numel() == B * n * C, "dout");
  TORCH_CHECK(dc.is_contiguous() && dz.is_contiguous() && dc.sizes() == c.sizes() && dz.sizes() == c.sizes() &&
                  dz_f32.is_contiguous() && dz_f32.numel() == B * n * m * C, "dc / dz / dz_f32");
  TORCH_CHECK(c.stride(2) == 1 && z.stride(2) == 1 && bias.is_contiguous(), "layout");
  const int64_t total = B * n * C;
  if (total == 0) return;
  c10::cuda::CUDAGuard guard(c.device());
  const unsigned grid = static_cast<unsigned>((total + 255) / 256);
  auto st = at::cuda::getCurrentCUDAStream();
  auto cp = reinterpret_cast<const __nv_bfloat16*>(c.data_ptr());
  auto zp = reinterpret_cast<const __nv_bfloat16*>(z.data_ptr());
  auto dcp = reinterpret_cast<__nv_bfloat16*>(dc.data_ptr());
  auto dzp = reinterpret_cast<__nv_bfloat16*>(dz.data_ptr());
  if (bias.scalar_type() == at::kFloat) {
    pool_bwd_kernel<float><<<grid, 256, 0, st>>>(cp, zp, c.stride(1), z.stride(1), bias.data_ptr<float>(),
                                                 static_cast<int>(T), static_cast<int>(n), static_cast<int>(m),
                                                 static_cast<int>(C), out.data_ptr<float>(), dout.data_ptr<float>(),
                                                 dcp, dzp, dz_f32.data_ptr<float>(), total);
  } else {
    pool_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        cp, zp, c.stride(1), z.stride(1), reinterpret_cast<const __nv_bfloat16*>(bias.data_ptr()),
        static_cast<int>(T), static_cast<int>(n), static_cast<int>(m), static_cast<int>(C), out.data_ptr<float>(),
        dout.data_ptr<float>(), dcp, dzp, dz_f32.data_ptr<float>(), total);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sv4
