// MoE data-movement kernels around the grouped tcgen05 GEMMs.
//
// Layout: every expert owns a contiguous segment of the permuted row buffer, padded
// to a multiple of 128 rows (the GEMM M tile), so a GEMM tile never straddles two
// experts.  All routing bookkeeping stays on the device (no host sync):
//
//   moe_route_plan   : per-expert counts -> padded segment starts/rows, a
//                      deterministic slot position for every (token, k) pair
//                      (token order within an expert), and row -> token maps.
//   moe_gather       : x_perm[row] = h[token(row)] (zero for padding rows).
//   moe_combine      : out[t] = sum_j gate[t, j] * y[pos(t, j)], and the
//                      un-weighted variant used for dX in backward.
//   moe_combine_bwd  : dy[pos] = gate * dout[t];  dgate[t, j] = <dout[t], y[pos]>.
//   swiglu_bwd       : d[gate|up] pre-activations from d(act) and the saved pre-acts,
//                      honouring the V4 clamps (gate <= gmax, lo <= up <= hi).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace sv4 {

constexpr int kRowPad = 128;

// One CTA per expert: scans the flattened (T*k) expert ids in order and assigns
// consecutive slots to the matches (block-wide prefix sum per 1024-id chunk).
__global__ void route_positions_kernel(const int64_t* __restrict__ idx, int n_pairs,
                                       const int* __restrict__ seg_start, int* __restrict__ pos,
                                       int* __restrict__ row_token, int k, int* err, int n_experts) {
  const int e = blockIdx.x;
  __shared__ int warp_sums[32];
  __shared__ int running;
  if (threadIdx.x == 0) running = 0;
  __syncthreads();
  const int base = seg_start[e];
  for (int off = 0; off < n_pairs; off += blockDim.x) {
    const int i = off + threadIdx.x;
    int hit = 0;
    if (i < n_pairs) {
      const int64_t ex = idx[i];
      if (ex < 0 || ex >= n_experts) record_error(err, kErrBounds);
      hit = (ex == e) ? 1 : 0;
    }
    int v = hit;  // inclusive warp scan
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, v, d);
      if (lane >= d) v += n;
    }
    if (lane == 31) warp_sums[wid] = v;
    __syncthreads();
    if (wid == 0) {
      int w = lane < (blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, w, d);
        if (lane >= d) w += n;
      }
      warp_sums[lane] = w;
    }
    __syncthreads();
    const int prefix = (wid > 0 ? warp_sums[wid - 1] : 0) + v - hit;  // exclusive
    if (hit) {
      const int p = base + running + prefix;
      pos[i] = p;
      row_token[p] = i / k;
    }
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) running += prefix + hit;
    __syncthreads();
  }
}

__global__ void count_experts_kernel(const int64_t* __restrict__ idx, int n_pairs, int* __restrict__ counts,
                                     int n_experts) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_pairs; i += gridDim.x * blockDim.x) {
    const int64_t e = idx[i];
    if (e >= 0 && e < n_experts) atomicAdd(&counts[e], 1);
  }
}

__global__ void segments_kernel(const int* __restrict__ counts, int n_experts, int* __restrict__ seg_start,
                                int* __restrict__ seg_rows, int* __restrict__ total_rows) {
  if (threadIdx.x != 0) return;
  int acc = 0;
  for (int e = 0; e < n_experts; ++e) {
    const int rows = (counts[e] + kRowPad - 1) / kRowPad * kRowPad;
    seg_start[e] = acc;
    seg_rows[e] = rows;
    acc += rows;
  }
  *total_rows = acc;
}

// idx: (T*k) int64 expert ids.  Outputs: counts (E), seg_start (E), seg_rows (E), total (1),
// pos (T*k), row_token (M_cap) pre-filled with -1 by the caller.
void moe_route_plan(torch::Tensor idx, int64_t n_experts, int64_t k, torch::Tensor counts, torch::Tensor seg_start,
                    torch::Tensor seg_rows, torch::Tensor total, torch::Tensor pos, torch::Tensor row_token,
                    torch::Tensor err) {
  c10::cuda::CUDAGuard guard(idx.device());
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  const int n = idx.numel();
  counts.zero_();
  count_experts_kernel<<<std::min(1024, (n + 255) / 256 + 1), 256, 0, s>>>(idx.data_ptr<int64_t>(), n,
                                                                          counts.data_ptr<int>(), n_experts);
  segments_kernel<<<1, 32, 0, s>>>(counts.data_ptr<int>(), n_experts, seg_start.data_ptr<int>(),
                                   seg_rows.data_ptr<int>(), total.data_ptr<int>());
  route_positions_kernel<<<n_experts, 1024, 0, s>>>(idx.data_ptr<int64_t>(), n, seg_start.data_ptr<int>(),
                                                    pos.data_ptr<int>(), row_token.data_ptr<int>(), k,
                                                    err.data_ptr<int>(), n_experts);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// x_perm[r, :] = h[row_token[r], :] or 0.  One warp per row, 16-byte vectors.  A token id
// outside [-1, T) records kErrBounds and leaves the row zero.
__global__ void gather_rows_kernel(const uint4* __restrict__ h, const int* __restrict__ row_token,
                                   uint4* __restrict__ out, int rows, int vec_per_row, int T, int* err) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  int t = row_token[warp];
  if (!index_ok(t, -1, T, err)) t = -1;
  uint4* dst = out + static_cast<int64_t>(warp) * vec_per_row;
  if (t < 0) {
    for (int v = lane; v < vec_per_row; v += 32) dst[v] = make_uint4(0, 0, 0, 0);
  } else {
    const uint4* src = h + static_cast<int64_t>(t) * vec_per_row;
    for (int v = lane; v < vec_per_row; v += 32) dst[v] = src[v];
  }
}

void moe_gather(torch::Tensor h, torch::Tensor row_token, torch::Tensor out, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(h.device());
  TORCH_CHECK(h.is_contiguous() && out.is_contiguous() && h.scalar_type() == out.scalar_type(), "layout");
  TORCH_CHECK(h.size(1) * h.element_size() % 16 == 0, "row bytes must be a multiple of 16");
  const int rows = out.size(0);
  const int vpr = h.size(1) * h.element_size() / 16;
  if (rows == 0) return;
  gather_rows_kernel<<<(rows * 32 + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint4*>(h.data_ptr()), row_token.data_ptr<int>(),
      reinterpret_cast<uint4*>(out.data_ptr()), rows, vpr, static_cast<int>(h.size(0)), err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out[t, :] = sum_j w[t, j] * y[pos[t, j], :]   (w == nullptr -> weight 1).  One CTA per token.
// A slot position outside [0, rows_y) records kErrBounds and contributes nothing.
__global__ void combine_kernel(const __nv_bfloat16* __restrict__ y, const int* __restrict__ pos,
                               const float* __restrict__ w, __nv_bfloat16* __restrict__ out, int D, int kk,
                               int rows_y, int* err) {
  const int t = blockIdx.x;
  int p[16];
  float g[16];
  for (int j = 0; j < kk; ++j) {
    p[j] = pos[t * kk + j];
    g[j] = w ? w[t * kk + j] : 1.0f;
    const bool ok = threadIdx.x == 0 ? index_ok(p[j], 0, rows_y, err) : (p[j] >= 0 && p[j] < rows_y);
    if (!ok) {
      p[j] = 0;
      g[j] = 0.f;
    }
  }
  for (int d = threadIdx.x * 8; d < D; d += blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = 0; j < kk; ++j) {
      const uint4 v = *reinterpret_cast<const uint4*>(y + static_cast<int64_t>(p[j]) * D + d);
      const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(hv[q]);
        acc[2 * q] += g[j] * f.x;
        acc[2 * q + 1] += g[j] * f.y;
      }
    }
    uint4 o;
    __nv_bfloat162* ho = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int q = 0; q < 4; ++q) ho[q] = __floats2bfloat162_rn(acc[2 * q], acc[2 * q + 1]);
    *reinterpret_cast<uint4*>(out + static_cast<int64_t>(t) * D + d) = o;
  }
}

void moe_combine(torch::Tensor y, torch::Tensor pos, c10::optional<torch::Tensor> w, torch::Tensor out,
                 torch::Tensor err) {
  c10::cuda::CUDAGuard guard(y.device());
  const int T = out.size(0), D = out.size(1), k = pos.size(1);
  TORCH_CHECK(D % 8 == 0 && k <= 16, "combine: D % 8 == 0 and k <= 16");
  if (T == 0) return;
  const float* wp = w.has_value() ? w->data_ptr<float>() : nullptr;
  const int threads = std::min(256, std::max(32, D / 8));
  combine_kernel<<<T, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), pos.data_ptr<int>(), wp,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), D, k, static_cast<int>(y.size(0)), err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Backward of the weighted combine: dy[pos[t,j]] = w[t,j] * dout[t];  dw[t,j] = <dout[t], y[pos[t,j]]>.
// One warp per (t, j); padding rows of dy are zeroed separately (moe_zero_pad_rows).
__global__ void combine_bwd_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ y,
                                   const int* __restrict__ pos, const float* __restrict__ w,
                                   __nv_bfloat16* __restrict__ dy, float* __restrict__ dw, int n_pairs, int k,
                                   int D, int rows, int* err) {
  const int pair = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (pair >= n_pairs) return;
  const int t = pair / k;
  const int p = pos[pair];
  const bool ok = lane == 0 ? index_ok(p, 0, rows, err) : (p >= 0 && p < rows);
  if (!ok) {  // the pair's gradient row cannot be placed: no write, zero gate gradient
    if (lane == 0 && dw != nullptr) dw[pair] = 0.f;
    return;
  }
  const float g = w[pair];
  float dot = 0.f;
  for (int d = lane * 8; d < D; d += 32 * 8) {
    const uint4 a = *reinterpret_cast<const uint4*>(dout + static_cast<int64_t>(t) * D + d);
    const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&a);
    uint4 o;
    __nv_bfloat162* ho = reinterpret_cast<__nv_bfloat162*>(&o);
    if (y != nullptr) {
      const uint4 b = *reinterpret_cast<const uint4*>(y + static_cast<int64_t>(p) * D + d);
      const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 fa = __bfloat1622float2(ha[q]);
        const float2 fb = __bfloat1622float2(hb[q]);
        dot += fa.x * fb.x + fa.y * fb.y;
        ho[q] = __floats2bfloat162_rn(fa.x * g, fa.y * g);
      }
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 fa = __bfloat1622float2(ha[q]);
        ho[q] = __floats2bfloat162_rn(fa.x * g, fa.y * g);
      }
    }
    *reinterpret_cast<uint4*>(dy + static_cast<int64_t>(p) * D + d) = o;
  }
  if (y == nullptr || dw == nullptr) return;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  if (lane == 0) dw[pair] = dot;
}

// y / dw omitted: only the gate-scaled output gradient rows are written (the gate gradient
// then comes from swiglu_bwd_gate, which needs no saved expert outputs).
void moe_combine_bwd(torch::Tensor dout, c10::optional<torch::Tensor> y, torch::Tensor pos, torch::Tensor w,
                     torch::Tensor dy, c10::optional<torch::Tensor> dw, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(dout.device());
  const int n_pairs = pos.numel(), k = pos.size(1), D = dout.size(1);
  TORCH_CHECK(D % 8 == 0, "D % 8");
  TORCH_CHECK(y.has_value() == dw.has_value(), "y and dw come together");
  if (n_pairs == 0) return;
  const int64_t rows = y.has_value() ? std::min(y->size(0), dy.size(0)) : dy.size(0);
  combine_bwd_kernel<<<(n_pairs * 32 + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
      y.has_value() ? reinterpret_cast<const __nv_bfloat16*>(y->data_ptr()) : nullptr, pos.data_ptr<int>(),
      w.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dy.data_ptr()),
      dw.has_value() ? dw->data_ptr<float>() : nullptr, n_pairs, k, D, static_cast<int>(rows), err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Zero the rows of a (rows, D) buffer whose row_token is -1 (padding rows).
__global__ void zero_pad_rows_kernel(const int* __restrict__ row_token, uint4* __restrict__ buf, int rows,
                                     int vec_per_row) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows || row_token[warp] >= 0) return;
  uint4* dst = buf + static_cast<int64_t>(warp) * vec_per_row;
  for (int v = lane; v < vec_per_row; v += 32) dst[v] = make_uint4(0, 0, 0, 0);
}

void moe_zero_pad_rows(torch::Tensor row_token, torch::Tensor buf) {
  c10::cuda::CUDAGuard guard(buf.device());
  const int rows = buf.size(0);
  if (rows == 0) return;
  const int vpr = buf.size(1) * buf.element_size() / 16;
  zero_pad_rows_kernel<<<(rows * 32 + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      row_token.data_ptr<int>(), reinterpret_cast<uint4*>(buf.data_ptr()), rows, vpr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// d_pre = [d_gate | d_up] from d_act and pre = [gate | up] (rows x 2I).
//   act = silu(min(g, gmax)) * clamp(u, lo, hi)
// With act != nullptr the forward activation act = silu(min(g, gmax)) * clamp(u, lo, hi) is
// recomputed from the saved pre-activations and written too (the forward does not keep it).
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dact, int64_t ld_dact,
                                  const __nv_bfloat16* __restrict__ pre, __nv_bfloat16* __restrict__ dpre,
                                  int64_t rows, int I, float gmax, float lo, float hi,
                                  __nv_bfloat16* __restrict__ act) {
  const int64_t n = rows * I;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / I;
    const int c = static_cast<int>(i - r * I);
    const float da = __bfloat162float(dact[r * ld_dact + c]);
    const float g = __bfloat162float(pre[r * 2 * I + c]);
    const float u = __bfloat162float(pre[r * 2 * I + I + c]);
    const float gc = fminf(g, gmax);
    const float uc = fminf(fmaxf(u, lo), hi);
    const float sig = 1.0f / (1.0f + __expf(-gc));
    const float silu = gc * sig;
    const float dsilu = sig * (1.0f + gc * (1.0f - sig));
    const float dg = (g <= gmax) ? da * uc * dsilu : 0.0f;
    const float du = (u >= lo && u <= hi) ? da * silu : 0.0f;
    dpre[r * 2 * I + c] = __float2bfloat16(dg);
    dpre[r * 2 * I + I + c] = __float2bfloat16(du);
    if (act != nullptr) act[r * I + c] = __float2bfloat16(silu * uc);
  }
}

void swiglu_bwd(torch::Tensor dact, torch::Tensor pre, torch::Tensor dpre, double gmax, double lo, double hi,
                c10::optional<torch::Tensor> act) {
  c10::cuda::CUDAGuard guard(dact.device());
  const int64_t rows = dact.size(0);
  const int I = dact.size(1);
  TORCH_CHECK(dact.stride(1) == 1 && pre.is_contiguous() && dpre.is_contiguous(), "swiglu_bwd layout");
  TORCH_CHECK(!act.has_value() || (act->is_contiguous() && act->size(0) == rows && act->size(1) == I &&
                                   act->scalar_type() == at::kBFloat16), "act: contiguous (rows, I) bf16");
  if (rows == 0) return;
  const int64_t n = rows * I;
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 16));
  swiglu_bwd_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dact.data_ptr()), dact.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(pre.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dpre.data_ptr()),
      rows, I, static_cast<float>(gmax), static_cast<float>(lo), static_cast<float>(hi),
      act.has_value() ? reinterpret_cast<__nv_bfloat16*>(act->data_ptr()) : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// SwiGLU backward of the routed experts with the gate gradient folded in, one warp per row:
// dpre from d(act) and the saved pre-activations, act recomputed (for the down projection's
// weight gradient), and for the (token, slot) pair p that owns the row
//   dgate[p] = <dout_t, y_row> = <dout_t Wd, act_row> = <dact_row, act_row> / gate[p]
// because dact_row = (gate[p] dout_t) Wd.  The expert outputs y therefore need not be kept
// for the backward.  row_pair[r] = p, or -1 for padding rows (whose dgate is not written).
__global__ void swiglu_bwd_gate_kernel(const __nv_bfloat16* __restrict__ dact, const __nv_bfloat16* __restrict__ pre,
                                       __nv_bfloat16* __restrict__ dpre, __nv_bfloat16* __restrict__ act, int64_t rows,
                                       int I, float gmax, float lo, float hi, const int* __restrict__ row_pair,
                                       const float* __restrict__ gate, float* __restrict__ dgate, int n_pairs,
                                       int* err) {
  const int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const __nv_bfloat16* dr = dact + r * I;
  const __nv_bfloat16* pg = pre + r * 2 * I;
  float dot = 0.f;
  for (int c = lane * 8; c < I; c += 256) {
    const uint4 va = *reinterpret_cast<const uint4*>(dr + c);
    const uint4 vg = *reinterpret_cast<const uint4*>(pg + c);
    const uint4 vu = *reinterpret_cast<const uint4*>(pg + I + c);
    const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&va);
    const __nv_bfloat162* hg = reinterpret_cast<const __nv_bfloat162*>(&vg);
    const __nv_bfloat162* hu = reinterpret_cast<const __nv_bfloat162*>(&vu);
    uint4 og, ou, oa;
    __nv_bfloat162* pog = reinterpret_cast<__nv_bfloat162*>(&og);
    __nv_bfloat162* pou = reinterpret_cast<__nv_bfloat162*>(&ou);
    __nv_bfloat162* poa = reinterpret_cast<__nv_bfloat162*>(&oa);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 da = __bfloat1622float2(ha[q]);
      const float2 g2 = __bfloat1622float2(hg[q]);
      const float2 u2 = __bfloat1622float2(hu[q]);
      float dg[2], du[2], a[2];
      const float dav[2] = {da.x, da.y}, gv[2] = {g2.x, g2.y}, uv[2] = {u2.x, u2.y};
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float gc = fminf(gv[e], gmax);
        const float uc = fminf(fmaxf(uv[e], lo), hi);
        const float sig = 1.0f / (1.0f + __expf(-gc));
        const float silu = gc * sig;
        const float dsilu = sig * (1.0f + gc * (1.0f - sig));
        dg[e] = (gv[e] <= gmax) ? dav[e] * uc * dsilu : 0.0f;
        du[e] = (uv[e] >= lo && uv[e] <= hi) ? dav[e] * silu : 0.0f;
        a[e] = silu * uc;
      }
      pog[q] = __floats2bfloat162_rn(dg[0], dg[1]);
      pou[q] = __floats2bfloat162_rn(du[0], du[1]);
      poa[q] = __floats2bfloat162_rn(a[0], a[1]);
      const float2 ar = __bfloat1622float2(poa[q]);  // the act the weight gradient will read
      dot += dav[0] * ar.x + dav[1] * ar.y;
    }
    *reinterpret_cast<uint4*>(dpre + r * 2 * I + c) = og;
    *reinterpret_cast<uint4*>(dpre + r * 2 * I + I + c) = ou;
    *reinterpret_cast<uint4*>(act + r * I + c) = oa;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  if (lane == 0) {
    const int p = row_pair[r];
    if (p >= 0 && index_ok(p, 0, n_pairs, err)) {
      const float g = gate[p];
      dgate[p] = g != 0.f ? dot / g : 0.f;
    }
  }
}

void swiglu_bwd_gate(torch::Tensor dact, torch::Tensor pre, torch::Tensor dpre, double gmax, double lo, double hi,
                     torch::Tensor act, torch::Tensor row_pair, torch::Tensor gate, torch::Tensor dgate,
                     torch::Tensor err) {
  c10::cuda::CUDAGuard guard(dact.device());
  const int64_t rows = dact.size(0);
  const int I = dact.size(1);
  TORCH_CHECK(dact.is_contiguous() && pre.is_contiguous() && dpre.is_contiguous() && act.is_contiguous() &&
                  I % 8 == 0 && act.size(0) == rows && act.size(1) == I, "swiglu_bwd_gate layout (I % 8 == 0)");
  TORCH_CHECK(row_pair.scalar_type() == at::kInt && row_pair.numel() >= rows && gate.scalar_type() == at::kFloat &&
                  dgate.scalar_type() == at::kFloat && gate.numel() == dgate.numel(), "row_pair / gate / dgate");
  if (rows == 0) return;
  swiglu_bwd_gate_kernel<<<static_cast<unsigned>((rows * 32 + 255) / 256), 256, 0,
                           at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dact.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(pre.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(dpre.data_ptr()), reinterpret_cast<__nv_bfloat16*>(act.data_ptr()), rows, I,
      static_cast<float>(gmax), static_cast<float>(lo), static_cast<float>(hi), row_pair.data_ptr<int>(),
      gate.data_ptr<float>(), dgate.data_ptr<float>(), static_cast<int>(gate.numel()), err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sv4
