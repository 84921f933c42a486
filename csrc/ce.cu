// Cross-entropy over fp32 logit rows produced by the LM-head GEMM (chunked over rows):
//   ce_fwd:  lse[r] = logsumexp_v z[r, v],  nll[r] = lse[r] - z[r, target[r]]
//   ce_bwd:  dz[r, v] = scale * (exp(z - lse) - [v == target]) * cap'(raw)   (bf16 out)
// with the optional softcap z = c * tanh(raw / c) applied on the fly (cap' = 1 - tanh^2).
// One CTA per row, 16-byte loads, one online (max, sum) pass in the forward.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cuda_bf16.h>

namespace sv4 {

namespace {

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  const float mx = fmaxf(m, m2);
  if (mx == -INFINITY) return;
  s = s * __expf(m - mx) + s2 * __expf(m2 - mx);
  m = mx;
}

__global__ void ce_fwd_kernel(const float* __restrict__ z, const int64_t* __restrict__ target, int rows, int V,
                              int ld, float softcap, float* __restrict__ lse, float* __restrict__ nll) {
  const int r = blockIdx.x;
  if (r >= rows) return;
  const float* zr = z + static_cast<int64_t>(r) * ld;
  float m = -INFINITY, s = 0.f;
  auto add = [&](float raw) {
    const float t = softcap > 0.f ? softcap * tanhf(raw / softcap) : raw;
    if (t > m) {
      s = s * __expf(m - t) + 1.f;
      m = t;
    } else {
      s += __expf(t - m);
    }
  };
  const int vec_end = (ld % 4 == 0) ? (V & ~3) : 0;
  for (int v = threadIdx.x * 4; v < vec_end; v += blockDim.x * 4) {
    const float4 x = *reinterpret_cast<const float4*>(zr + v);
    add(x.x);
    add(x.y);
    add(x.z);
    add(x.w);
  }
  for (int v = vec_end + threadIdx.x; v < V; v += blockDim.x) add(zr[v]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, off);
    online_merge(m, s, m2, s2);
  }
  __shared__ float sm[32], ss[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    m = lane < nw ? sm[lane] : -INFINITY;
    s = lane < nw ? ss[lane] : 0.f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, off);
      online_merge(m, s, m2, s2);
    }
    if (lane == 0) {
      const float l = m + __logf(s);
      const int64_t t = target[r];
      float zt = (t >= 0 && t < V) ? zr[t] : 0.f;
      if (softcap > 0.f) zt = softcap * tanhf(zt / softcap);
      lse[r] = l;
      nll[r] = l - zt;
    }
  }
}

__global__ void ce_bwd_kernel(const float* __restrict__ z, const int64_t* __restrict__ target,
                              const float* __restrict__ lse, int rows, int rows_out, int V, int ld, float softcap,
                              const float* __restrict__ scale_ptr, int scale_per_row,
                              __nv_bfloat16* __restrict__ dz) {
  const int r = blockIdx.x;
  __nv_bfloat16* out = dz + static_cast<int64_t>(r) * V;
  if (r >= rows) {  // padding rows of the weight-gradient GEMM operand
    for (int v = threadIdx.x; v < V; v += blockDim.x) out[v] = __float2bfloat16(0.f);
    return;
  }
  const float* zr = z + static_cast<int64_t>(r) * ld;
  const float l = lse[r];
  const int64_t t = target[r];
  const float scale = scale_ptr[scale_per_row ? r : 0];
  auto grad = [&](int v) {
    float zz = zr[v], d = 1.f;
    if (softcap > 0.f) {
      const float th = tanhf(zz / softcap);
      zz = softcap * th;
      d = 1.f - th * th;
    }
    return (__expf(zz - l) - (v == t ? 1.f : 0.f)) * scale * d;
  };
  const int vec_end = (V % 8 == 0 && ld % 4 == 0) ? V : 0;
  for (int v = vec_end + threadIdx.x; v < V; v += blockDim.x) out[v] = __float2bfloat16(grad(v));
  for (int v = threadIdx.x * 8; v < vec_end; v += blockDim.x * 8) {
    const float4 a = *reinterpret_cast<const float4*>(zr + v);
    const float4 b = *reinterpret_cast<const float4*>(zr + v + 4);
    const float e[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float g2[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i = 2 * q + u;
        float zz = e[i], d = 1.f;
        if (softcap > 0.f) {
          const float th = tanhf(e[i] / softcap);
          zz = softcap * th;
          d = 1.f - th * th;
        }
        float g = __expf(zz - l) - (v + i == t ? 1.f : 0.f);
        g2[u] = g * scale * d;
      }
      __nv_bfloat162 h = __floats2bfloat162_rn(g2[0], g2[1]);
      w[q] = *reinterpret_cast<uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(out + v) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  (void)rows_out;
}

}  // namespace

void ce_fwd(torch::Tensor z, torch::Tensor target, double softcap, torch::Tensor lse, torch::Tensor nll) {
  c10::cuda::CUDAGuard guard(z.device());
  const int rows = z.size(0), V = z.size(1), ld = z.stride(0);
  TORCH_CHECK(z.scalar_type() == at::kFloat && z.stride(1) == 1, "ce_fwd: fp32 rows with unit stride");
  if (rows == 0) return;
  ce_fwd_kernel<<<rows, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      z.data_ptr<float>(), target.data_ptr<int64_t>(), rows, V, ld, static_cast<float>(softcap),
      lse.data_ptr<float>(), nll.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// dz: (rows_out >= rows, V) bf16; rows past `rows` are zero-filled.  scale: one device
// scalar for every row, or one value per row (per-token weights, e.g. policy gradients).
void ce_bwd(torch::Tensor z, torch::Tensor target, torch::Tensor lse, double softcap, torch::Tensor scale,
            torch::Tensor dz) {
  c10::cuda::CUDAGuard guard(z.device());
  const int rows = z.size(0), V = z.size(1), ld = z.stride(0), rows_out = dz.size(0);
  TORCH_CHECK(z.stride(1) == 1 && dz.is_contiguous() && dz.size(1) == V, "ce_bwd shapes");
  TORCH_CHECK(scale.numel() == 1 || scale.numel() == rows, "ce_bwd: scale must have 1 or `rows` values");
  if (rows_out == 0) return;
  ce_bwd_kernel<<<rows_out, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      z.data_ptr<float>(), target.data_ptr<int64_t>(), lse.data_ptr<float>(), rows, rows_out, V, ld,
      static_cast<float>(softcap), scale.data_ptr<float>(), scale.numel() == rows && rows > 1 ? 1 : 0,
      reinterpret_cast<__nv_bfloat16*>(dz.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sv4
