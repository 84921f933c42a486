// Fused MoE router forward: affinity, biased top-k selection and gate renormalisation in
// one pass over the router logits (one warp per token).
//
//   aff    = sqrt(softplus(z) + 1e-12)   (or sigmoid(z))
//   score  = aff + aux_free_bias (+ modality_bias[is_visual])
//   idx    = top-k of score (ties: the lower expert index first)
//   gate_j = aff[idx_j] / (sum_i aff[idx_i] + 1e-12)
//
// This is the reference's learned router (core/moe.py:54-111: affinity, bias-adjusted
// top-k, renormalised gates) without the ~10 separate element-wise / top-k launches.
//
// Backward (router_bwd, one warp per token): with s = sum_j aff[idx_j] and the incoming
// gate gradient dg, d aff[idx_j] += (dg_j - sum_i dg_i gate_i) / s on top of the affinity
// gradient (the sequence-balance loss), then dz = d aff * d aff / dz
// (sigmoid(z) / (2 aff) for sqrt-softplus, aff (1 - aff) for sigmoid).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

namespace sv4 {
namespace {

constexpr int kMaxPerLane = 8;  // up to 256 experts

__device__ __forceinline__ float softplus_f(float x) {
  // log(1 + e^x), written to stay finite for large |x|
  return x > 20.f ? x : log1pf(expf(x));
}

template <int MODE>
__global__ void router_fwd_kernel(const float* __restrict__ z, int T, int E, int k, const float* __restrict__ bias,
                                  const float* __restrict__ mbias, const uint8_t* __restrict__ visual,
                                  float* __restrict__ aff, int64_t* __restrict__ idx, float* __restrict__ gate) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const int64_t row = static_cast<int64_t>(warp) * E;
  const float* mb = (mbias != nullptr && visual != nullptr) ? mbias + (visual[warp] ? E : 0) : nullptr;
  float a[kMaxPerLane], s[kMaxPerLane];
#pragma unroll
  for (int q = 0; q < kMaxPerLane; ++q) {
    const int e = lane + 32 * q;
    if (e < E) {
      const float x = z[row + e];
      a[q] = MODE == 0 ? sqrtf(softplus_f(x) + 1.0e-12f) : 1.0f / (1.0f + expf(-x));
      aff[row + e] = a[q];
      s[q] = a[q] + (bias != nullptr ? bias[e] : 0.f) + (mb != nullptr ? mb[e] : 0.f);
    } else {
      a[q] = 0.f;
      s[q] = -INFINITY;
    }
  }
  float picked[16];
  int pidx[16];
  float sum = 0.f;
  for (int j = 0; j < k; ++j) {
    // lane-local best (lowest index on ties), then a warp argmax
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int q = 0; q < kMaxPerLane; ++q) {
      const int e = lane + 32 * q;
      if (e < E && (s[q] > bv || (s[q] == bv && e < bi))) {
        bv = s[q];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    // the owner lane removes the winner and broadcasts its affinity
    float av = 0.f;
    if ((bi & 31) == lane) {
#pragma unroll
      for (int q = 0; q < kMaxPerLane; ++q) {
        if (lane + 32 * q == bi) {
          av = a[q];
          s[q] = -INFINITY;
        }
      }
    }
    av = __shfl_sync(0xffffffffu, av, bi & 31);
    if (bi >= E) {  // only when every remaining score is NaN: pick expert 0 with no weight
      bi = 0;
      av = 0.f;
    }
    if (j < 16) {
      picked[j] = av;
      pidx[j] = bi;
    }
    sum += av;
  }
  if (lane == 0) {
    const float inv = 1.0f / (sum + 1.0e-12f);
    for (int j = 0; j < k; ++j) {
      idx[static_cast<int64_t>(warp) * k + j] = pidx[j];
      gate[static_cast<int64_t>(warp) * k + j] = picked[j] * inv;
    }
  }
}

}  // namespace

// z (T, E) fp32 logits -> aff (T, E), idx (T, k) int64, gate (T, k) fp32.
template <int MODE>
__global__ void router_bwd_kernel(const float* __restrict__ z, const float* __restrict__ aff,
                                  const int64_t* __restrict__ idx, const float* __restrict__ gate,
                                  const float* __restrict__ d_gate, const float* __restrict__ d_aff, int T, int E, int k,
                                  float* __restrict__ dz) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const int64_t row = static_cast<int64_t>(warp) * E;
  float da[kMaxPerLane];
#pragma unroll
  for (int q = 0; q < kMaxPerLane; ++q) {
    const int e = lane + 32 * q;
    da[q] = (e < E && d_aff != nullptr) ? d_aff[row + e] : 0.f;
  }
  if (d_gate != nullptr) {
    // every lane computes the k-term sums (k <= 16 loads, all from L1)
    float s = 0.f, dot = 0.f;
    for (int j = 0; j < k; ++j) {
      const int64_t e = idx[static_cast<int64_t>(warp) * k + j];
      s += aff[row + e];
      dot += d_gate[static_cast<int64_t>(warp) * k + j] * gate[static_cast<int64_t>(warp) * k + j];
    }
    const float inv = 1.f / (s + 1.0e-12f);
    for (int j = 0; j < k; ++j) {
      const int e = static_cast<int>(idx[static_cast<int64_t>(warp) * k + j]);
      if ((e & 31) != lane) continue;
      const float add = (d_gate[static_cast<int64_t>(warp) * k + j] - dot) * inv;
#pragma unroll
      for (int q = 0; q < kMaxPerLane; ++q)
        if (e == lane + 32 * q) da[q] += add;
    }
  }
#pragma unroll
  for (int q = 0; q < kMaxPerLane; ++q) {
    const int e = lane + 32 * q;
    if (e >= E) continue;
    const float a = aff[row + e];
    float d;
    if (MODE == 0) {
      const float sg = 1.0f / (1.0f + expf(-z[row + e]));
      d = da[q] * sg / (2.0f * a);
    } else {
      d = da[q] * a * (1.0f - a);
    }
    dz[row + e] = d;
  }
}

void router_bwd(torch::Tensor z, torch::Tensor aff, torch::Tensor idx, torch::Tensor gate,
                c10::optional<torch::Tensor> d_gate, c10::optional<torch::Tensor> d_aff, int64_t mode,
                torch::Tensor dz) {
  TORCH_CHECK(z.scalar_type() == at::kFloat && z.dim() == 2 && z.is_contiguous(), "z: contiguous (T, E) fp32");
  const int64_t T = z.size(0), E = z.size(1), k = idx.size(-1);
  TORCH_CHECK(E <= 32 * kMaxPerLane && k >= 1 && k <= 16, "router: E <= 256, 1 <= k <= 16");
  TORCH_CHECK(aff.is_contiguous() && aff.sizes() == z.sizes() && dz.is_contiguous() && dz.sizes() == z.sizes(),
              "aff / dz (T, E)");
  TORCH_CHECK(idx.is_contiguous() && idx.numel() == T * k && gate.is_contiguous() && gate.numel() == T * k,
              "idx / gate (T, k)");
  const float* dg = nullptr;
  if (d_gate.has_value()) {
    TORCH_CHECK(d_gate->scalar_type() == at::kFloat && d_gate->is_contiguous() && d_gate->numel() == T * k, "d_gate");
    dg = d_gate->data_ptr<float>();
  }
  const float* dap = nullptr;
  if (d_aff.has_value()) {
    TORCH_CHECK(d_aff->scalar_type() == at::kFloat && d_aff->is_contiguous() && d_aff->numel() == T * E, "d_aff");
    dap = d_aff->data_ptr<float>();
  }
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(z.device());
  const int threads = 256;
  const unsigned blocks = static_cast<unsigned>((T * 32 + threads - 1) / threads);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (mode == 0) {
    router_bwd_kernel<0><<<blocks, threads, 0, stream>>>(z.data_ptr<float>(), aff.data_ptr<float>(),
                                                         idx.data_ptr<int64_t>(), gate.data_ptr<float>(), dg, dap, T,
                                                         E, k, dz.data_ptr<float>());
  } else {
    router_bwd_kernel<1><<<blocks, threads, 0, stream>>>(z.data_ptr<float>(), aff.data_ptr<float>(),
                                                         idx.data_ptr<int64_t>(), gate.data_ptr<float>(), dg, dap, T,
                                                         E, k, dz.data_ptr<float>());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void router_fwd(torch::Tensor z, int64_t k, int64_t mode, c10::optional<torch::Tensor> bias,
                c10::optional<torch::Tensor> modality_bias, c10::optional<torch::Tensor> is_visual,
                torch::Tensor aff, torch::Tensor idx, torch::Tensor gate) {
  TORCH_CHECK(z.scalar_type() == at::kFloat && z.dim() == 2 && z.is_contiguous(), "z: contiguous (T, E) fp32");
  const int64_t T = z.size(0), E = z.size(1);
  TORCH_CHECK(E <= 32 * kMaxPerLane && k >= 1 && k <= 16 && k <= E, "router: E <= 256, 1 <= k <= min(16, E)");
  TORCH_CHECK(aff.is_contiguous() && aff.sizes() == z.sizes() && aff.scalar_type() == at::kFloat, "aff");
  TORCH_CHECK(idx.is_contiguous() && idx.scalar_type() == at::kLong && idx.numel() == T * k, "idx");
  TORCH_CHECK(gate.is_contiguous() && gate.scalar_type() == at::kFloat && gate.numel() == T * k, "gate");
  const float* bp = nullptr;
  if (bias.has_value()) {
    TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->is_contiguous() && bias->numel() == E, "bias");
    bp = bias->data_ptr<float>();
  }
  const float* mp = nullptr;
  const uint8_t* vp = nullptr;
  if (modality_bias.has_value() && is_visual.has_value()) {
    TORCH_CHECK(modality_bias->scalar_type() == at::kFloat && modality_bias->is_contiguous() &&
                    modality_bias->numel() == 2 * E, "modality bias (2, E) fp32");
    TORCH_CHECK(is_visual->scalar_type() == at::kBool && is_visual->is_contiguous() && is_visual->numel() == T,
                "is_visual (T) bool");
    mp = modality_bias->data_ptr<float>();
    vp = reinterpret_cast<const uint8_t*>(is_visual->data_ptr());
  }
  if (T == 0) return;
  c10::cuda::CUDAGuard guard(z.device());
  const int threads = 256;
  const unsigned blocks = static_cast<unsigned>((T * 32 + threads - 1) / threads);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (mode == 0) {
    router_fwd_kernel<0><<<blocks, threads, 0, stream>>>(z.data_ptr<float>(), T, E, k, bp, mp, vp,
                                                          aff.data_ptr<float>(), idx.data_ptr<int64_t>(),
                                                          gate.data_ptr<float>());
  } else {
    router_fwd_kernel<1><<<blocks, threads, 0, stream>>>(z.data_ptr<float>(), T, E, k, bp, mp, vp,
                                                          aff.data_ptr<float>(), idx.data_ptr<int64_t>(),
                                                          gate.data_ptr<float>());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sv4
