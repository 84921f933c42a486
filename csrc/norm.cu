// Normalisation-family kernels: RMSNorm, fused RoPE+RMSNorm on attention heads, and
// the mHC (manifold-constrained hyper-connection) split / combine passes.
//
// All kernels read bf16 activations, compute in fp32 and write bf16; statistics
// needed by the backward pass (1/rms) are saved in fp32.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace sv4 {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 t = __bfloat1622float2(h[q]);
    f[2 * q] = t.x;
    f[2 * q + 1] = t.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 v;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
  for (int q = 0; q < 4; ++q) h[q] = __floats2bfloat162_rn(f[2 * q], f[2 * q + 1]);
  *reinterpret_cast<uint4*>(p) = v;
}

// ------------------------------------------------------------------ RMSNorm
// y = w * x * rstd, rstd = 1/sqrt(mean(x^2) + eps).  One warp per row, D % 8 == 0.
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
                                   __nv_bfloat16* __restrict__ y, float* __restrict__ rstd, int rows, int D,
                                   float eps) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const __nv_bfloat16* xr = x + static_cast<int64_t>(row) * D;
  float ss = 0.f;
  for (int d = lane * 8; d < D; d += 256) {
    float f[8];
    load8(xr + d, f);
#pragma unroll
    for (int q = 0; q < 8; ++q) ss += f[q] * f[q];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / D + eps);
  if (lane == 0) rstd[row] = r;
  __nv_bfloat16* yr = y + static_cast<int64_t>(row) * D;
  for (int d = lane * 8; d < D; d += 256) {
    float f[8];
    load8(xr + d, f);
#pragma unroll
    for (int q = 0; q < 8; ++q) f[q] = w[d + q] * (f[q] * r);
    store8(yr + d, f);
  }
}

// dx = r * (w*dy - x * r^2 * mean(w*dy*x)); dw partials per CTA (rows_per_cta rows).
// Phase 1: one warp per row computes mean(w*dy*x).  Phase 2: thread t owns columns
// [8t, 8t+8) (+ 8*blockDim strides): coalesced 16-byte row reads, dx writes, and dw
// accumulated in registers (no shared-memory atomics).
constexpr int kNormRowsPerCta = 16;
__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                   const float* __restrict__ w, const float* __restrict__ rstd,
                                   __nv_bfloat16* __restrict__ dx, float* __restrict__ dw_part, int rows, int D) {
  __shared__ float sdot[kNormRowsPerCta];
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kNormRowsPerCta;
  const int nrows = min(kNormRowsPerCta, rows - row0);
  for (int rr = threadIdx.x >> 5; rr < nrows; rr += warps) {
    const int row = row0 + rr;
    const __nv_bfloat16* xr = x + static_cast<int64_t>(row) * D;
    const __nv_bfloat16* gr = dy + static_cast<int64_t>(row) * D;
    float dot = 0.f;
    for (int d = lane * 8; d < D; d += 256) {
      float fx[8], fg[8];
      load8(xr + d, fx);
      load8(gr + d, fg);
#pragma unroll
      for (int q = 0; q < 8; ++q) dot += w[d + q] * fg[q] * fx[q];
    }
    dot = warp_sum(dot);
    if (lane == 0) sdot[rr] = dot / D;
  }
  __syncthreads();
  for (int d0 = threadIdx.x * 8; d0 < D; d0 += blockDim.x * 8) {
    float wv[8], acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      wv[q] = w[d0 + q];
      acc[q] = 0.f;
    }
    for (int rr = 0; rr < nrows; rr += 4) {
      uint4 xv[4], gv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {  // issue all loads of four rows first
        const int64_t off = static_cast<int64_t>(row0 + min(rr + u, nrows - 1)) * D + d0;
        xv[u] = *reinterpret_cast<const uint4*>(x + off);
        gv[u] = *reinterpret_cast<const uint4*>(dy + off);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (rr + u >= nrows) break;
        const int64_t off = static_cast<int64_t>(row0 + rr + u) * D + d0;
        const float r = rstd[row0 + rr + u];
        const float c = r * r * sdot[rr + u];
        const __nv_bfloat162* xh = reinterpret_cast<const __nv_bfloat162*>(&xv[u]);
        const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&gv[u]);
        float o[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 fx = __bfloat1622float2(xh[q]), fg = __bfloat1622float2(gh[q]);
          acc[2 * q] += fg.x * fx.x * r;
          acc[2 * q + 1] += fg.y * fx.y * r;
          o[2 * q] = r * (wv[2 * q] * fg.x - fx.x * c);
          o[2 * q + 1] = r * (wv[2 * q + 1] * fg.y - fx.y * c);
        }
        store8(dx + off, o);
      }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) dw_part[static_cast<int64_t>(blockIdx.x) * D + d0 + q] = acc[q];
  }
}

__global__ void column_sum_kernel(const float* __restrict__ part, int n, int D, float* __restrict__ out) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= D) return;
  float s = 0.f;
  for (int i = 0; i < n; ++i) s += part[static_cast<int64_t>(i) * D + d];
  out[d] = s;
}

void rmsnorm_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor y, torch::Tensor rstd, double eps) {
  c10::cuda::CUDAGuard guard(x.device());
  const int D = x.size(-1);
  const int rows = x.numel() / D;
  TORCH_CHECK(D % 8 == 0 && w.scalar_type() == at::kFloat, "rmsnorm: D % 8 == 0, fp32 weight");
  if (rows == 0) return;
  rmsnorm_fwd_kernel<<<(rows * 32 + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), w.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), rstd.data_ptr<float>(), rows, D, static_cast<float>(eps));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// returns dw (fp32, D)
torch::Tensor rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd, torch::Tensor dx) {
  c10::cuda::CUDAGuard guard(x.device());
  const int D = x.size(-1);
  const int rows = x.numel() / D;
  TORCH_CHECK(D % 8 == 0, "rmsnorm_bwd: D % 8 == 0");
  const int ctas = std::max(1, (rows + kNormRowsPerCta - 1) / kNormRowsPerCta);
  auto part = torch::empty({ctas, D}, x.options().dtype(at::kFloat));
  auto dw = torch::empty({D}, x.options().dtype(at::kFloat));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (rows == 0) return dw.zero_();
  rmsnorm_bwd_kernel<<<ctas, 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
      w.data_ptr<float>(), rstd.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()),
      part.data_ptr<float>(), rows, D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  column_sum_kernel<<<(D + 255) / 256, 256, 0, stream>>>(part.data_ptr<float>(), ctas, D, dw.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dw;
}

// ------------------------------------------------------------ RoPE + RMSNorm
// Rows are (token, head) vectors of length HD (<= 256, % 8); the rotary part is the last RD
// channels with interleaved pairs.  norm_first: y = rope(norm(x)) else y = norm(rope(x)).
// Token of a row = row / heads.  One warp per row; lane l owns channels [8l, 8l+8).
__device__ __forceinline__ void rope8(float (&f)[8], int c0, int HD, int RD, const float* cs, const float* sn,
                                      bool inverse) {
#pragma unroll
  for (int q = 0; q < 8; q += 2) {
    const int c = c0 + q;
    if (c >= HD - RD) {
      const int p = (c - (HD - RD)) >> 1;
      const float co = cs[p], si = inverse ? -sn[p] : sn[p];
      const float e = f[q], o = f[q + 1];
      f[q] = e * co - o * si;
      f[q + 1] = e * si + o * co;
    }
  }
}

__global__ void rope_norm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
                                     const float* __restrict__ cosb, const float* __restrict__ sinb,
                                     __nv_bfloat16* __restrict__ y, float* __restrict__ rstd, int rows, int heads,
                                     int HD, int RD, bool norm_first, float eps) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int t = row / heads;
  const float* cs = cosb + static_cast<int64_t>(t) * (RD / 2);
  const float* sn = sinb + static_cast<int64_t>(t) * (RD / 2);
  const int c0 = lane * 8;
  const bool act = c0 < HD;
  float f[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (act) load8(x + static_cast<int64_t>(row) * HD + c0, f);
  if (!norm_first && act) rope8(f, c0, HD, RD, cs, sn, false);
  float ss = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) ss += f[q] * f[q];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / HD + eps);
  if (lane == 0) rstd[row] = r;
  if (!act) return;
#pragma unroll
  for (int q = 0; q < 8; ++q) f[q] = w[c0 + q] * (f[q] * r);
  if (norm_first) rope8(f, c0, HD, RD, cs, sn, false);
  store8(y + static_cast<int64_t>(row) * HD + c0, f);
}

__global__ void rope_norm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                     const float* __restrict__ w, const float* __restrict__ cosb,
                                     const float* __restrict__ sinb, const float* __restrict__ rstd,
                                     __nv_bfloat16* __restrict__ dx, float* __restrict__ dw_part, int rows,
                                     int heads, int HD, int RD, bool norm_first, int rows_per_cta) {
  __shared__ float sdw[256];
  for (int d = threadIdx.x; d < HD; d += blockDim.x) sdw[d] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int c0 = lane * 8;
  const bool act = c0 < HD;
  float wl[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) wl[q] = act ? w[c0 + q] : 0.f;
  float dwl[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const int row0 = blockIdx.x * rows_per_cta;
  for (int rr = threadIdx.x >> 5; rr < rows_per_cta; rr += blockDim.x >> 5) {
    const int row = row0 + rr;
    if (row >= rows) break;
    const int t = row / heads;
    const float* cs = cosb + static_cast<int64_t>(t) * (RD / 2);
    const float* sn = sinb + static_cast<int64_t>(t) * (RD / 2);
    const float r = rstd[row];
    float g[8] = {0, 0, 0, 0, 0, 0, 0, 0}, z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (act) {
      load8(dy + static_cast<int64_t>(row) * HD + c0, g);
      load8(x + static_cast<int64_t>(row) * HD + c0, z);
      if (norm_first) rope8(g, c0, HD, RD, cs, sn, true);  // undo the rotation on the gradient
      else rope8(z, c0, HD, RD, cs, sn, false);            // z = rope(x) is the norm input
    }
    float dot = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      dot += wl[q] * g[q] * z[q];
      dwl[q] += g[q] * z[q] * r;
    }
    dot = warp_sum(dot) / HD;
    if (!act) continue;
    float o[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) o[q] = r * (wl[q] * g[q] - z[q] * r * r * dot);
    if (!norm_first) rope8(o, c0, HD, RD, cs, sn, true);
    store8(dx + static_cast<int64_t>(row) * HD + c0, o);
  }
  if (act) {
#pragma unroll
    for (int q = 0; q < 8; ++q) atomicAdd(&sdw[c0 + q], dwl[q]);
  }
  __syncthreads();
  for (int d = threadIdx.x; d < HD; d += blockDim.x) dw_part[static_cast<int64_t>(blockIdx.x) * HD + d] = sdw[d];
}

void rope_norm_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor cosb, torch::Tensor sinb, torch::Tensor y,
                   torch::Tensor rstd, int64_t heads, int64_t rd, bool norm_first, double eps) {
  c10::cuda::CUDAGuard guard(x.device());
  const int HD = x.size(-1);
  const int rows = x.numel() / HD;
  TORCH_CHECK(HD % 8 == 0 && HD <= 256 && rd % 2 == 0 && rd <= HD, "rope_norm shape");
  if (rows == 0) return;
  rope_norm_fwd_kernel<<<(rows * 32 + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), w.data_ptr<float>(), cosb.data_ptr<float>(),
      sinb.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), rstd.data_ptr<float>(), rows, heads,
      HD, rd, norm_first, static_cast<float>(eps));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

torch::Tensor rope_norm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor cosb,
                            torch::Tensor sinb, torch::Tensor rstd, torch::Tensor dx, int64_t heads, int64_t rd,
                            bool norm_first) {
  c10::cuda::CUDAGuard guard(x.device());
  const int HD = x.size(-1);
  const int rows = x.numel() / HD;
  const int rpc = 128;
  const int ctas = std::max(1, (rows + rpc - 1) / rpc);
  auto part = torch::zeros({ctas, HD}, x.options().dtype(at::kFloat));
  if (rows > 0) {
    rope_norm_bwd_kernel<<<ctas, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
        w.data_ptr<float>(), cosb.data_ptr<float>(), sinb.data_ptr<float>(), rstd.data_ptr<float>(),
        reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), part.data_ptr<float>(), rows, heads, HD, rd, norm_first,
        rpc);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  return part.sum(0);
}

// ---------------------------------------------------------------------- mHC
// Stream X: (T, F) with F = n*D.  W: (P, F) gate projections with the RMSNorm weight folded
// in (P = 2n + n^2).  The raw dots q = X W^T come from the GEMM, the row sums of squares from
// row_sumsq; the gates kernel turns them into r = 1/rms and p = r q.
constexpr int kMhcTok = 32;    // tokens per CTA of the split backward
constexpr int kMhcStep = 8;    // tokens whose loads are in flight together (160 registers, 3 CTAs / SM)
// ssq[t] = sum_k X[t, k]^2 (bf16 rows, fp32 result): one warp per row, 16-byte loads.
// The mHC projection itself (X W^T, skinny N) runs on the tcgen05 GEMM with split-K.
__global__ void row_sumsq_kernel(const __nv_bfloat16* __restrict__ X, float* __restrict__ ssq, int T, int F) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= T) return;
  const __nv_bfloat16* xr = X + static_cast<int64_t>(row) * F;
  float s = 0.f;
  for (int k = lane * 8; k < F; k += 32 * 8) {
    float f[8];
    load8(xr + k, f);
#pragma unroll
    for (int q = 0; q < 8; ++q) s += f[q] * f[q];
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) ssq[row] = s;
}

void row_sumsq(torch::Tensor X, torch::Tensor ssq) {
  c10::cuda::CUDAGuard guard(X.device());
  const int T = X.size(0), F = X.size(1);
  TORCH_CHECK(X.is_contiguous() && F % 8 == 0, "row_sumsq: contiguous rows, F % 8 == 0");
  if (T == 0) return;
  row_sumsq_kernel<<<(T + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(X.data_ptr()), ssq.data_ptr<float>(), T, F);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Gates: z = alpha * p + s;  A = sigmoid(z_pre), B = Sinkhorn(z_res), C = 2 sigmoid(z_post).
// One thread per token; n <= 4, iters <= 32.  Layout of p/dz rows: [pre(n) | res(n*n) | post(n)].
template <int N>
__device__ __forceinline__ void sinkhorn_fwd(float (&m)[N][N], int iters, float (*hist)[N][N]) {
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) mx = fmaxf(mx, m[i][j]);
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) m[i][j] = __expf(m[i][j] - mx);
  for (int it = 0; it < iters; ++it) {
    if (hist) {
#pragma unroll
      for (int i = 0; i < N; ++i)
#pragma unroll
        for (int j = 0; j < N; ++j) hist[2 * it][i][j] = m[i][j];
    }
#pragma unroll
    for (int i = 0; i < N; ++i) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < N; ++j) s += m[i][j];
      const float inv = 1.0f / (s + 1e-12f);
#pragma unroll
      for (int j = 0; j < N; ++j) m[i][j] *= inv;
    }
    if (hist) {
#pragma unroll
      for (int i = 0; i < N; ++i)
#pragma unroll
        for (int j = 0; j < N; ++j) hist[2 * it + 1][i][j] = m[i][j];
    }
#pragma unroll
    for (int j = 0; j < N; ++j) {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < N; ++i) s += m[i][j];
      const float inv = 1.0f / (s + 1e-12f);
#pragma unroll
      for (int i = 0; i < N; ++i) m[i][j] *= inv;
    }
  }
}

template <int N>
__global__ void mhc_gates_fwd_kernel(float* __restrict__ p, const float* __restrict__ ssq, float* __restrict__ r_out,
                                     const float* __restrict__ alpha, const float* __restrict__ s_pre,
                                     const float* __restrict__ s_res, const float* __restrict__ s_post,
                                     float* __restrict__ a, float* __restrict__ b, float* __restrict__ c, int T,
                                     int iters, float inv_f, float eps) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  constexpr int P = 2 * N + N * N;
  float* pr = p + static_cast<int64_t>(t) * P;
  const float r = rsqrtf(ssq[t] * inv_f + eps);
  r_out[t] = r;
#pragma unroll
  for (int j = 0; j < P; ++j) pr[j] *= r;
  const float ap = alpha[0], ar = alpha[1], ac = alpha[2];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    a[t * N + i] = 1.0f / (1.0f + __expf(-(ap * pr[i] + s_pre[i])));
    c[t * N + i] = 2.0f / (1.0f + __expf(-(ac * pr[N + N * N + i] + s_post[i])));
  }
  float m[N][N];
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) m[i][j] = ar * pr[N + i * N + j] + s_res[i * N + j];
  sinkhorn_fwd<N>(m, iters, nullptr);
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) b[static_cast<int64_t>(t) * N * N + i * N + j] = m[i][j];
}

// dz (T, P): gradient w.r.t. z = alpha * p + s.
template <int N>
__global__ void mhc_gates_bwd_kernel(const float* __restrict__ p, const float* __restrict__ alpha,
                                     const float* __restrict__ s_pre, const float* __restrict__ s_res,
                                     const float* __restrict__ s_post, const float* __restrict__ da,
                                     const float* __restrict__ db, const float* __restrict__ dc,
                                     float* __restrict__ dz, int T, int iters) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  constexpr int P = 2 * N + N * N;
  const float* pr = p + static_cast<int64_t>(t) * P;
  float* dzr = dz + static_cast<int64_t>(t) * P;
  const float ap = alpha[0], ar = alpha[1], ac = alpha[2];
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const float sa = 1.0f / (1.0f + __expf(-(ap * pr[i] + s_pre[i])));
    dzr[i] = da[t * N + i] * sa * (1.0f - sa);
    const float sc = 1.0f / (1.0f + __expf(-(ac * pr[N + N * N + i] + s_post[i])));
    dzr[N + N * N + i] = dc[t * N + i] * 2.0f * sc * (1.0f - sc);
  }
  float m[N][N];
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) m[i][j] = ar * pr[N + i * N + j] + s_res[i * N + j];
  float hist[64][N][N];  // inputs of each normalisation (2 per iteration), iters <= 32
  sinkhorn_fwd<N>(m, iters, hist);
  float g[N][N];
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) g[i][j] = db[static_cast<int64_t>(t) * N * N + i * N + j];
  for (int it = iters - 1; it >= 0; --it) {
    {  // column normalisation: y_ij = x_ij / (S_j + eps), x = hist[2it+1]
      float (&x)[N][N] = hist[2 * it + 1];
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float s = 0.f, gd = 0.f;
#pragma unroll
        for (int i = 0; i < N; ++i) s += x[i][j];
        const float inv = 1.0f / (s + 1e-12f);
#pragma unroll
        for (int i = 0; i < N; ++i) gd += g[i][j] * x[i][j];
#pragma unroll
        for (int i = 0; i < N; ++i) g[i][j] = g[i][j] * inv - gd * inv * inv;
      }
    }
    {  // row normalisation, x = hist[2it]
      float (&x)[N][N] = hist[2 * it];
#pragma unroll
      for (int i = 0; i < N; ++i) {
        float s = 0.f, gd = 0.f;
#pragma unroll
        for (int j = 0; j < N; ++j) s += x[i][j];
        const float inv = 1.0f / (s + 1e-12f);
#pragma unroll
        for (int j = 0; j < N; ++j) gd += g[i][j] * x[i][j];
#pragma unroll
        for (int j = 0; j < N; ++j) g[i][j] = g[i][j] * inv - gd * inv * inv;
      }
    }
  }
  // through exp(z - max): dz = g * exp(z - max) (the max shift cancels in the output)
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) mx = fmaxf(mx, ar * pr[N + i * N + j] + s_res[i * N + j]);
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j)
      dzr[N + i * N + j] = g[i][j] * __expf(ar * pr[N + i * N + j] + s_res[i * N + j] - mx);
}

#define SV4_MHC_N(n, GRID, KERNEL, ...)                                                       \
  switch (n) {                                                                                \
    case 1: KERNEL<1><<<GRID, 128, 0, stream>>>(__VA_ARGS__); break;                          \
    case 2: KERNEL<2><<<GRID, 128, 0, stream>>>(__VA_ARGS__); break;                          \
    case 3: KERNEL<3><<<GRID, 128, 0, stream>>>(__VA_ARGS__); break;                          \
    case 4: KERNEL<4><<<GRID, 128, 0, stream>>>(__VA_ARGS__); break;                          \
    default: TORCH_CHECK(false, "mHC expansion factor must be 1..4");                          \
  }

// p: raw dots in, p = r * dots out (in place); ssq: row sums of squares; r: 1/rms out.
void mhc_gates_fwd(torch::Tensor p, torch::Tensor ssq, torch::Tensor r, int64_t F, double eps, torch::Tensor alpha,
                   torch::Tensor s_pre, torch::Tensor s_res, torch::Tensor s_post, torch::Tensor a, torch::Tensor b,
                   torch::Tensor c, int64_t n, int64_t iters) {
  c10::cuda::CUDAGuard guard(p.device());
  const int T = p.size(0);
  if (T == 0) return;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  SV4_MHC_N(n, (T + 127) / 128, mhc_gates_fwd_kernel, p.data_ptr<float>(), ssq.data_ptr<float>(),
            r.data_ptr<float>(), alpha.data_ptr<float>(), s_pre.data_ptr<float>(), s_res.data_ptr<float>(),
            s_post.data_ptr<float>(), a.data_ptr<float>(), b.data_ptr<float>(), c.data_ptr<float>(), T,
            static_cast<int>(iters), 1.0f / static_cast<float>(F), static_cast<float>(eps));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mhc_gates_bwd(torch::Tensor p, torch::Tensor alpha, torch::Tensor s_pre, torch::Tensor s_res,
                   torch::Tensor s_post, torch::Tensor da, torch::Tensor db, torch::Tensor dc, torch::Tensor dz,
                   int64_t n, int64_t iters) {
  c10::cuda::CUDAGuard guard(p.device());
  TORCH_CHECK(iters <= 32, "sinkhorn_iters <= 32 on the native path");
  const int T = p.size(0);
  if (T == 0) return;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  SV4_MHC_N(n, (T + 127) / 128, mhc_gates_bwd_kernel, p.data_ptr<float>(), alpha.data_ptr<float>(),
            s_pre.data_ptr<float>(), s_res.data_ptr<float>(), s_post.data_ptr<float>(), da.data_ptr<float>(),
            db.data_ptr<float>(), dc.data_ptr<float>(), dz.data_ptr<float>(), T, static_cast<int>(iters));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// inner[t, d] = sum_h a[t, h] X[t, h, d].  One CTA (128 threads) per token.
template <int N>
__global__ void mhc_premix_kernel(const __nv_bfloat16* __restrict__ X, const float* __restrict__ a,
                                  __nv_bfloat16* __restrict__ out, int D) {
  const int t = blockIdx.x;
  float av[N];
#pragma unroll
  for (int h = 0; h < N; ++h) av[h] = a[t * N + h];
  for (int d = threadIdx.x * 8; d < D; d += blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int h = 0; h < N; ++h) {
      float f[8];
      load8(X + (static_cast<int64_t>(t) * N + h) * D + d, f);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += av[h] * f[q];
    }
    store8(out + static_cast<int64_t>(t) * D + d, acc);
  }
}

// X'[t, h] = sum_k B[t,h,k] X[t,k] + C[t,h] out[t].  One CTA per token.
template <int N>
__global__ void mhc_combine_kernel(const __nv_bfloat16* __restrict__ X, const __nv_bfloat16* __restrict__ o,
                                   const float* __restrict__ B, const float* __restrict__ C,
                                   __nv_bfloat16* __restrict__ Y, int D) {
  const int t = blockIdx.x;
  float bm[N][N], cv[N];
#pragma unroll
  for (int h = 0; h < N; ++h) {
    cv[h] = C[t * N + h];
#pragma unroll
    for (int k = 0; k < N; ++k) bm[h][k] = B[(static_cast<int64_t>(t) * N + h) * N + k];
  }
  for (int d = threadIdx.x * 8; d < D; d += blockDim.x * 8) {
    float xs[N][8], of[8];
#pragma unroll
    for (int k = 0; k < N; ++k) load8(X + (static_cast<int64_t>(t) * N + k) * D + d, xs[k]);
    load8(o + static_cast<int64_t>(t) * D + d, of);
#pragma unroll
    for (int h = 0; h < N; ++h) {
      float y[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float s = cv[h] * of[q];
#pragma unroll
        for (int k = 0; k < N; ++k) s += bm[h][k] * xs[k][q];
        y[q] = s;
      }
      store8(Y + (static_cast<int64_t>(t) * N + h) * D + d, y);
    }
  }
}

// Backward of combine: dX[t,k] = sum_h B[t,h,k] dY[t,h];  dout[t] = sum_h C[t,h] dY[t,h];
// dB[t,h,k] = <dY[t,h], X[t,k]>;  dC[t,h] = <dY[t,h], out[t]>.  One CTA (128 threads) per token.
template <int N>
__global__ void mhc_combine_bwd_kernel(const __nv_bfloat16* __restrict__ dY, const __nv_bfloat16* __restrict__ X,
                                       const __nv_bfloat16* __restrict__ o, const float* __restrict__ B,
                                       const float* __restrict__ C, __nv_bfloat16* __restrict__ dX,
                                       __nv_bfloat16* __restrict__ dO, float* __restrict__ dB,
                                       float* __restrict__ dC, int D) {
  const int t = blockIdx.x;
  float bm[N][N], cv[N];
#pragma unroll
  for (int h = 0; h < N; ++h) {
    cv[h] = C[t * N + h];
#pragma unroll
    for (int k = 0; k < N; ++k) bm[h][k] = B[(static_cast<int64_t>(t) * N + h) * N + k];
  }
  float accB[N][N], accC[N];
#pragma unroll
  for (int h = 0; h < N; ++h) {
    accC[h] = 0.f;
#pragma unroll
    for (int k = 0; k < N; ++k) accB[h][k] = 0.f;
  }
  for (int d = threadIdx.x * 8; d < D; d += blockDim.x * 8) {
    float g[N][8], xs[N][8], of[8];
#pragma unroll
    for (int h = 0; h < N; ++h) {
      load8(dY + (static_cast<int64_t>(t) * N + h) * D + d, g[h]);
      load8(X + (static_cast<int64_t>(t) * N + h) * D + d, xs[h]);
    }
    load8(o + static_cast<int64_t>(t) * D + d, of);
    float dof[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float s = 0.f;
#pragma unroll
      for (int h = 0; h < N; ++h) s += cv[h] * g[h][q];
      dof[q] = s;
    }
    store8(dO + static_cast<int64_t>(t) * D + d, dof);
#pragma unroll
    for (int k = 0; k < N; ++k) {
      float dx[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float s = 0.f;
#pragma unroll
        for (int h = 0; h < N; ++h) s += bm[h][k] * g[h][q];
        dx[q] = s;
      }
      store8(dX + (static_cast<int64_t>(t) * N + k) * D + d, dx);
    }
#pragma unroll
    for (int h = 0; h < N; ++h) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        accC[h] += g[h][q] * of[q];
#pragma unroll
        for (int k = 0; k < N; ++k) accB[h][k] += g[h][q] * xs[k][q];
      }
    }
  }
  __shared__ float red[4][N * N + N];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int h = 0; h < N; ++h) {
    const float v = warp_sum(accC[h]);
    if (lane == 0) red[w][N * N + h] = v;
#pragma unroll
    for (int k = 0; k < N; ++k) {
      const float u = warp_sum(accB[h][k]);
      if (lane == 0) red[w][h * N + k] = u;
    }
  }
  __syncthreads();
  if (threadIdx.x < N * N + N) {
    float s = 0.f;
    for (int i = 0; i < (blockDim.x >> 5); ++i) s += red[i][threadIdx.x];
    if (threadIdx.x < N * N) dB[static_cast<int64_t>(t) * N * N + threadIdx.x] = s;
    else dC[t * N + threadIdx.x - N * N] = s;
  }
}

// da[t,h] = <X[t,h], dinner[t]>
template <int N>
__global__ void mhc_premix_da_kernel(const __nv_bfloat16* __restrict__ X, const __nv_bfloat16* __restrict__ din,
                                     float* __restrict__ da, int D) {
  const int t = blockIdx.x;
  float acc[N];
#pragma unroll
  for (int h = 0; h < N; ++h) acc[h] = 0.f;
  for (int d = threadIdx.x * 8; d < D; d += blockDim.x * 8) {
    float g[8];
    load8(din + static_cast<int64_t>(t) * D + d, g);
#pragma unroll
    for (int h = 0; h < N; ++h) {
      float f[8];
      load8(X + (static_cast<int64_t>(t) * N + h) * D + d, f);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[h] += f[q] * g[q];
    }
  }
  __shared__ float red[4][N];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int h = 0; h < N; ++h) {
    const float v = warp_sum(acc[h]);
    if (lane == 0) red[w][h] = v;
  }
  __syncthreads();
  if (threadIdx.x < N) {
    float s = 0.f;
    for (int i = 0; i < (blockDim.x >> 5); ++i) s += red[i][threadIdx.x];
    da[t * N + threadIdx.x] = s;
  }
}

// Backward of split (pre-mix + norm-projection), accumulated onto dX (which holds the carry grad):
//   dX[t,h] = a[t,h] * dinner[t]  +  r * (dp_t W)_h  -  (r^3 / F) * X[t,h] * sum_j dp_tj q_tj
// where q = p / r.  CTA per 32 tokens; each thread owns 4 features.
template <int N>
__global__ void mhc_split_bwd_kernel(__nv_bfloat16* __restrict__ dX, const __nv_bfloat16* __restrict__ X,
                                     const __nv_bfloat16* __restrict__ din, const float* __restrict__ a,
                                     const float* __restrict__ dp, const float* __restrict__ p,
                                     const float* __restrict__ r, const float* __restrict__ W, int T, int D) {
  constexpr int P = 2 * N + N * N;
  const int F = N * D;
  __shared__ float sdp[kMhcTok][P];
  __shared__ float scoef[kMhcTok][2];
  __shared__ float sa[kMhcTok][N];
  const int t0 = blockIdx.x * kMhcTok;
  for (int i = threadIdx.x; i < kMhcTok * P; i += blockDim.x) {
    const int tt = i / P, j = i % P;
    sdp[tt][j] = (t0 + tt < T) ? dp[static_cast<int64_t>(t0 + tt) * P + j] : 0.f;
  }
  for (int i = threadIdx.x; i < kMhcTok * N; i += blockDim.x) {
    const int tt = i / N;
    sa[tt][i % N] = (t0 + tt < T) ? a[static_cast<int64_t>(t0 + tt) * N + i % N] : 0.f;
  }
  __syncthreads();
  for (int tt0 = threadIdx.x; tt0 < kMhcTok; tt0 += blockDim.x) {
    const int t = t0 + tt0;
    float rr = 0.f, s = 0.f;
    if (t < T) {
      rr = r[t];
      for (int j = 0; j < P; ++j) s += sdp[tt0][j] * p[static_cast<int64_t>(t) * P + j] / rr;
    }
    scoef[tt0][0] = rr;
    scoef[tt0][1] = rr * rr * rr / F * s;
  }
  __syncthreads();
  for (int f0 = (blockIdx.y * blockDim.x + threadIdx.x) * 4; f0 < F; f0 += gridDim.y * blockDim.x * 4) {
    float wv[P][4];
#pragma unroll
    for (int j = 0; j < P; ++j) {
      const float4 w4 = *reinterpret_cast<const float4*>(W + static_cast<int64_t>(j) * F + f0);
      wv[j][0] = w4.x; wv[j][1] = w4.y; wv[j][2] = w4.z; wv[j][3] = w4.w;
    }
    const int h = f0 / D, d = f0 % D;
    const int n_tok = min(kMhcTok, T - t0);
    // kMhcStep tokens per step: all 2*kMhcStep loads are issued before any math (memory parallelism)
    for (int tt = 0; tt < n_tok; tt += kMhcStep) {
      uint2 xv[kMhcStep], gv[kMhcStep];
#pragma unroll
      for (int u = 0; u < kMhcStep; ++u) {
        const int t = t0 + min(tt + u, n_tok - 1);
        xv[u] = __ldcs(reinterpret_cast<const uint2*>(X + static_cast<int64_t>(t) * F + f0));
        gv[u] = *reinterpret_cast<const uint2*>(din + static_cast<int64_t>(t) * D + d);
      }
#pragma unroll
      for (int u = 0; u < kMhcStep; ++u) {
        if (tt + u >= n_tok) break;
        const int ti = tt + u;
        const __nv_bfloat162* xh = reinterpret_cast<const __nv_bfloat162*>(&xv[u]);
        const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&gv[u]);
        float x[4], g[4];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const float2 a2 = __bfloat1622float2(xh[q]);
          const float2 c2 = __bfloat1622float2(gh[q]);
          x[2 * q] = a2.x; x[2 * q + 1] = a2.y;
          g[2 * q] = c2.x; g[2 * q + 1] = c2.y;
        }
        const float ah = sa[ti][h];
        const float rr = scoef[ti][0], cc = scoef[ti][1];
        float acc[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float sum = 0.f;
#pragma unroll
          for (int j = 0; j < P; ++j) sum += sdp[ti][j] * wv[j][q];
          acc[q] = ah * g[q] + rr * sum - cc * x[q];
        }
        uint2 ov;
        __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&ov);
        oh[0] = __floats2bfloat162_rn(acc[0], acc[1]);
        oh[1] = __floats2bfloat162_rn(acc[2], acc[3]);
        __stcs(reinterpret_cast<uint2*>(dX + static_cast<int64_t>(t0 + ti) * F + f0), ov);
      }
    }
  }
}

void mhc_premix(torch::Tensor X, torch::Tensor a, torch::Tensor out, int64_t n) {
  c10::cuda::CUDAGuard guard(X.device());
  const int T = out.size(0), D = out.size(1);
  if (T == 0) return;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  SV4_MHC_N(n, T, mhc_premix_kernel, reinterpret_cast<const __nv_bfloat16*>(X.data_ptr()), a.data_ptr<float>(),
            reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mhc_combine(torch::Tensor X, torch::Tensor o, torch::Tensor B, torch::Tensor C, torch::Tensor Y, int64_t n) {
  c10::cuda::CUDAGuard guard(X.device());
  const int T = o.size(0), D = o.size(1);
  if (T == 0) return;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  SV4_MHC_N(n, T, mhc_combine_kernel, reinterpret_cast<const __nv_bfloat16*>(X.data_ptr()),
            reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), B.data_ptr<float>(), C.data_ptr<float>(),
            reinterpret_cast<__nv_bfloat16*>(Y.data_ptr()), D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mhc_combine_bwd(torch::Tensor dY, torch::Tensor X, torch::Tensor o, torch::Tensor B, torch::Tensor C,
                     torch::Tensor dX, torch::Tensor dO, torch::Tensor dB, torch::Tensor dC, int64_t n) {
  c10::cuda::CUDAGuard guard(X.device());
  const int T = o.size(0), D = o.size(1);
  if (T == 0) return;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  SV4_MHC_N(n, T, mhc_combine_bwd_kernel, reinterpret_cast<const __nv_bfloat16*>(dY.data_ptr()),
            reinterpret_cast<const __nv_bfloat16*>(X.data_ptr()),
            reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), B.data_ptr<float>(), C.data_ptr<float>(),
            reinterpret_cast<__nv_bfloat16*>(dX.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dO.data_ptr()),
            dB.data_ptr<float>(), dC.data_ptr<float>(), D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mhc_premix_da(torch::Tensor X, torch::Tensor din, torch::Tensor da, int64_t n) {
  c10::cuda::CUDAGuard guard(X.device());
  const int T = din.size(0), D = din.size(1);
  if (T == 0) return;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  SV4_MHC_N(n, T, mhc_premix_da_kernel, reinterpret_cast<const __nv_bfloat16*>(X.data_ptr()),
            reinterpret_cast<const __nv_bfloat16*>(din.data_ptr()), da.data_ptr<float>(), D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mhc_split_bwd(torch::Tensor dX, torch::Tensor X, torch::Tensor din, torch::Tensor a, torch::Tensor dp,
                   torch::Tensor p, torch::Tensor r, torch::Tensor W, int64_t n) {
  c10::cuda::CUDAGuard guard(X.device());
  const int T = din.size(0), D = din.size(1);
  TORCH_CHECK(D % 4 == 0, "mhc_split_bwd: D % 4 == 0");
  if (T == 0) return;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const dim3 grid((T + kMhcTok - 1) / kMhcTok, std::max(1, (static_cast<int>(n) * D) / 512));
  SV4_MHC_N(n, grid, mhc_split_bwd_kernel, reinterpret_cast<__nv_bfloat16*>(dX.data_ptr()),
            reinterpret_cast<const __nv_bfloat16*>(X.data_ptr()),
            reinterpret_cast<const __nv_bfloat16*>(din.data_ptr()), a.data_ptr<float>(), dp.data_ptr<float>(),
            p.data_ptr<float>(), r.data_ptr<float>(), W.data_ptr<float>(), T, D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sv4
