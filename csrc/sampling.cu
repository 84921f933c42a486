// Fused next-token sampling: bias, temperature, top-k, top-p (nucleus) and the draw in
// one kernel, one CTA per row of logits.  Semantics of the reference's decoders
// (inference/generate.py:271-323): top-k keeps every logit >= the k-th largest (ties
// kept); top-p keeps the smallest descending prefix whose mass before each kept token is
// <= p, always including the best token, with the mass normalised over what top-k kept;
// the draw picks a token with probability proportional to exp(logit / T) over the kept set.
//
// Thresholds are found by radix selection over the 32 bits of an order-preserving integer
// key of each scaled logit, 8 bits per pass: a 256-bin histogram of the keys that share the
// prefix fixed so far (counts for top-k, softmax mass for top-p), scanned from the top.  No
// sort and no (V)-sized temporary: the logits row is re-read from L2 on each pass.  The draw
// is an inverse-CDF in vocabulary order against a caller-supplied uniform u in [0, 1), so a
// seeded torch generator reproduces a run.  temperature < 1e-8 is greedy: the first index
// of the maximum (torch.argmax's tie rule).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

#include <cfloat>
#include <cstdint>

namespace sv4 {
namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;

// Order-preserving map float -> uint32 (larger float -> larger key; -inf lowest but one).
__device__ __forceinline__ uint32_t float_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <typename T>
__device__ __forceinline__ float load_logit(const T* row, int i);
template <>
__device__ __forceinline__ float load_logit<float>(const float* row, int i) { return row[i]; }
template <>
__device__ __forceinline__ float load_logit<__nv_bfloat16>(const __nv_bfloat16* row, int i) {
  return __bfloat162float(row[i]);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < kWarps; ++w) t += red[w];  // same order in every thread
  return t;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) sample_kernel(const T* __restrict__ logits, int64_t ld, int V,
                                                          const float* __restrict__ bias, float inv_temp, int greedy,
                                                          int top_k, float top_p, const float* __restrict__ u,
                                                          int64_t* __restrict__ out, uint32_t* __restrict__ thr_out) {
  __shared__ float red[kWarps];
  __shared__ int redi[kWarps];
  __shared__ float hist_mass[256];
  __shared__ unsigned hist_cnt[256];
  __shared__ uint32_t s_prefix;
  __shared__ float s_above;
  __shared__ unsigned s_above_cnt;
  __shared__ int s_pick;
  const T* row = logits + static_cast<int64_t>(blockIdx.x) * ld;
  auto x_at = [&](int i) -> float {
    float v = load_logit<T>(row, i);
    if (bias != nullptr) v += bias[i];
    return v * inv_temp;
  };

  // row maximum (and its first index for greedy)
  float m = -INFINITY;
  int arg = V;
  for (int i = threadIdx.x; i < V; i += kThreads) {
    const float v = x_at(i);
    if (v > m || (v == m && i < arg)) { m = v; arg = i; }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const int oa = __shfl_xor_sync(0xffffffffu, arg, o);
    if (om > m || (om == m && oa < arg)) { m = om; arg = oa; }
  }
  if ((threadIdx.x & 31) == 0) { red[threadIdx.x >> 5] = m; redi[threadIdx.x >> 5] = arg; }
  __syncthreads();
  m = red[0];
  arg = redi[0];
  for (int w = 1; w < kWarps; ++w) {
    if (red[w] > m || (red[w] == m && redi[w] < arg)) { m = red[w]; arg = redi[w]; }
  }
  if (greedy) {
    if (threadIdx.x == 0) {
      out[blockIdx.x] = arg;
      if (thr_out != nullptr) thr_out[blockIdx.x] = float_key(m);
    }
    return;
  }

  // ---- top-k threshold: the k-th largest key (radix select on counts)
  uint32_t tk = 0;  // keep keys >= tk
  if (top_k > 0 && top_k < V) {
    uint32_t prefix = 0, mask = 0;
    unsigned need = static_cast<unsigned>(top_k);
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = threadIdx.x; b < 256; b += kThreads) hist_cnt[b] = 0;
      __syncthreads();
      for (int i = threadIdx.x; i < V; i += kThreads) {
        const uint32_t key = float_key(x_at(i));
        if ((key & mask) == prefix) atomicAdd(&hist_cnt[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        unsigned acc = 0;
        int b = 255;
        for (; b > 0; --b) {
          if (acc + hist_cnt[b] >= need) break;
          acc += hist_cnt[b];
        }
        s_prefix = prefix | (static_cast<uint32_t>(b) << shift);
        s_above_cnt = need - acc;
      }
      __syncthreads();
      prefix = s_prefix;
      need = s_above_cnt;
      mask |= 255u << shift;
      __syncthreads();
    }
    tk = prefix;
  }

  // ---- softmax mass over the top-k set
  float z = 0.f;
  for (int i = threadIdx.x; i < V; i += kThreads) {
    const float v = x_at(i);
    if (float_key(v) >= tk) z += __expf(v - m);
  }
  z = block_sum(z, red);

  // ---- top-p threshold: the key of the token whose preceding (larger) mass first
  // exceeds p; every key >= it is kept (the best token always is)
  uint32_t tp = 0;
  if (top_p < 1.f) {
    const float target = top_p * z;
    uint32_t prefix = 0, mask = 0;
    float above = 0.f;  // mass of keys strictly above the current prefix range
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = threadIdx.x; b < 256; b += kThreads) hist_mass[b] = 0.f;
      __syncthreads();
      for (int i = threadIdx.x; i < V; i += kThreads) {
        const float v = x_at(i);
        const uint32_t key = float_key(v);
        if (key >= tk && (key & mask) == prefix) atomicAdd(&hist_mass[(key >> shift) & 255u], __expf(v - m));
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        // walk down: keep the bucket in which the mass above the token first exceeds target
        float acc = above;
        int b = 255;
        for (; b > 0; --b) {
          if (hist_mass[b] > 0.f && acc + hist_mass[b] > target) break;
          acc += hist_mass[b];
        }
        s_prefix = prefix | (static_cast<uint32_t>(b) << shift);
        s_above = acc;
      }
      __syncthreads();
      prefix = s_prefix;
      above = s_above;
      mask |= 255u << shift;
      __syncthreads();
    }
    tp = prefix;
  }
  const uint32_t thr = tk > tp ? tk : tp;
  if (thr_out != nullptr && threadIdx.x == 0) thr_out[blockIdx.x] = thr;

  // ---- inverse-CDF draw in vocabulary order over the kept set
  float zk = 0.f;
  const int per = (V + kThreads - 1) / kThreads;
  const int i0 = threadIdx.x * per, i1 = min(V, i0 + per);
  for (int i = i0; i < i1; ++i) {
    const float v = x_at(i);
    if (float_key(v) >= thr) zk += __expf(v - m);
  }
  // exclusive scan of the per-thread sums (contiguous ranges, so vocabulary order)
  __shared__ float part[kThreads];
  part[threadIdx.x] = zk;
  __syncthreads();
  for (int o = 1; o < kThreads; o <<= 1) {
    const float add = threadIdx.x >= o ? part[threadIdx.x - o] : 0.f;
    __syncthreads();
    part[threadIdx.x] += add;
    __syncthreads();
  }
  const float total = part[kThreads - 1];
  const float before = part[threadIdx.x] - zk;
  const float target = u[blockIdx.x] * total;
  if (threadIdx.x == 0) s_pick = -1;
  __syncthreads();
  if (zk > 0.f && target >= before && target < before + zk) {
    float acc = before;
    int pick = -1, last = -1;
    for (int i = i0; i < i1; ++i) {
      const float v = x_at(i);
      if (float_key(v) < thr) continue;
      last = i;
      acc += __expf(v - m);
      if (target < acc) { pick = i; break; }
    }
    atomicMax(&s_pick, pick >= 0 ? pick : last);
  }
  __syncthreads();
  if (threadIdx.x == 0) out[blockIdx.x] = s_pick >= 0 ? s_pick : arg;  // rounding edge: the best token
}

}  // namespace

// logits (B, V) fp32 or bf16 (unit inner stride); bias (V) fp32 or None; u (B) fp32 uniforms
// in [0, 1); out (B) int64 token ids; thr (B) int32: the kept-set threshold key (testing).
void sample_tokens(torch::Tensor logits, c10::optional<torch::Tensor> bias, double temperature, int64_t top_k,
                   double top_p, torch::Tensor u, torch::Tensor out, c10::optional<torch::Tensor> thr) {
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "logits: (B, V) with unit inner stride");
  TORCH_CHECK(logits.scalar_type() == at::kFloat || logits.scalar_type() == at::kBFloat16, "logits fp32 or bf16");
  const int64_t B = logits.size(0), V = logits.size(1);
  TORCH_CHECK(V > 0 && V < (1LL << 31), "vocabulary size");
  TORCH_CHECK(u.scalar_type() == at::kFloat && u.numel() >= B && u.is_contiguous(), "u: (B) fp32");
  TORCH_CHECK(out.scalar_type() == at::kLong && out.numel() >= B && out.is_contiguous(), "out: (B) int64");
  TORCH_CHECK(top_p > 0.0 && top_p <= 1.0, "top_p in (0, 1]");
  const float* bp = nullptr;
  if (bias.has_value()) {
    TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == V && bias->is_contiguous(), "bias: (V) fp32");
    bp = bias->data_ptr<float>();
  }
  uint32_t* tp = nullptr;
  if (thr.has_value()) {
    TORCH_CHECK(thr->scalar_type() == at::kInt && thr->numel() >= B, "thr: (B) int32");
    tp = reinterpret_cast<uint32_t*>(thr->data_ptr<int>());
  }
  if (B == 0) return;
  c10::cuda::CUDAGuard guard(logits.device());
  const bool greedy = temperature < 1e-8;
  const float inv_t = greedy ? 1.f : static_cast<float>(1.0 / temperature);
  auto stream = at::cuda::getCurrentCUDAStream();
  const int k = static_cast<int>(top_k > 0 ? std::min<int64_t>(top_k, V) : 0);
  if (logits.scalar_type() == at::kFloat) {
    sample_kernel<float><<<static_cast<unsigned>(B), kThreads, 0, stream>>>(
        logits.data_ptr<float>(), logits.stride(0), static_cast<int>(V), bp, inv_t, greedy ? 1 : 0, k,
        static_cast<float>(top_p), u.data_ptr<float>(), out.data_ptr<int64_t>(), tp);
  } else {
    sample_kernel<__nv_bfloat16><<<static_cast<unsigned>(B), kThreads, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0), static_cast<int>(V), bp, inv_t,
        greedy ? 1 : 0, k, static_cast<float>(top_p), u.data_ptr<float>(), out.data_ptr<int64_t>(), tp);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sv4
