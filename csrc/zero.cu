// Hybrid-ZeRO gradient reduction and parameter broadcast over NVLink peer memory (one process
// per GPU, one node).
//
// The replicated parameters of every rank live in one symmetric byte arena and their fp32
// gradients in one symmetric fp32 arena, with the same layout on every rank (CUDA IPC maps each
// rank's arenas into every peer).  Each parameter has one owner.  Per step (epoch e):
//
//   zero_signal        after a group's gradients are final on this rank: fence at system scope,
//                      then release flags[slot = group][rank] = e on every rank
//   zero_pull_reduce   on the owner: wait until every rank's flag for the group reached e, then
//                      grad[i] = scale * sum over ranks (rank order) of that rank's grad[i] for the
//                      owned chunks (peer loads; the sum is the same on every rank's copy)
//   zero_signal        after the optimizer: flags[slot = params][rank] = e ("my owned
//                      parameters of step e are updated")
//   zero_pull_params   on every rank: wait for each chunk owner's params flag, then copy the
//                      owner's bytes of the chunk into the local arena (peer loads)
//
// Why no buffer is overwritten while a peer still reads it: an owner updates a parameter only
// after pulling the step's gradients from every rank, which waited for each rank's group flag,
// which that rank set after pulling the previous step's parameters; a rank zeroes its gradients
// for the next step only after pulling every owner's parameters, which each owner published
// after its gradient pulls.  Flags carry the epoch and are never reset.  Every wait is bounded
// (iterations and %globaltimer) and records kErrPeerTimeout, leaving the context usable.  No TMA
// and no multicast: plain 16-byte loads.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "common.cuh"

namespace sv4 {
namespace {

constexpr int kZeroMaxRanks = 8;

struct ZeroPeers {
  unsigned long long p[kZeroMaxRanks];
};

ZeroPeers zero_table(const std::vector<int64_t>& v) {
  TORCH_CHECK(!v.empty() && v.size() <= kZeroMaxRanks, "1..8 ranks");
  ZeroPeers t{};
  for (size_t i = 0; i < v.size(); ++i) t.p[i] = static_cast<unsigned long long>(v[i]);
  return t;
}

__device__ __forceinline__ uint64_t zero_now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned zero_ld_acquire(const unsigned* a) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}

// Thread 0: wait until flags[slot][src] >= epoch for every src in `mask`.  Bounded.
__device__ bool zero_wait(const unsigned* flags, int slot, unsigned mask, unsigned epoch, uint64_t timeout_ns,
                          int* err) {
  const uint64_t t0 = zero_now_ns();
  for (int src = 0; src < kZeroMaxRanks; ++src) {
    if (!(mask >> src & 1u)) continue;
    const unsigned* f = flags + slot * kZeroMaxRanks + src;
    uint32_t it = 0;
    while (static_cast<int>(zero_ld_acquire(f) - epoch) < 0) {
      ++it;
      if (it > kSpinLimit || ((it & 63u) == 0 && zero_now_ns() - t0 > timeout_ns)) {
        record_error(err, kErrPeerTimeout);
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

__global__ void zero_signal_kernel(ZeroPeers flags, int slot, int rank, int ws, unsigned epoch) {
  __threadfence_system();
  if (threadIdx.x < ws)
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(reinterpret_cast<unsigned*>(flags.p[threadIdx.x]) +
                                                             slot * kZeroMaxRanks + rank),
                 "r"(epoch)
                 : "memory");
}

// chunks: int64 [n][2] = (first float, floats), both multiples of 4.
__global__ void zero_pull_reduce_kernel(const int64_t* __restrict__ chunks, int n_chunks, ZeroPeers grads, int ws,
                                        int rank, float scale, const unsigned* __restrict__ flags, int slot,
                                        unsigned epoch, uint64_t timeout_ns, int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = zero_wait(flags, slot, ((1u << ws) - 1u) & ~(1u << rank), epoch, timeout_ns, err);
  __syncthreads();
  if (!ok) return;
  float4* mine = reinterpret_cast<float4*>(grads.p[rank]);
  for (int c = blockIdx.x; c < n_chunks; c += gridDim.x) {
    const int64_t off4 = chunks[2 * c] / 4, n4 = chunks[2 * c + 1] / 4;
    for (int64_t i = threadIdx.x; i < n4; i += blockDim.x) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int s = 0; s < ws; ++s) {
        const float4 v = s == rank ? mine[off4 + i] : __ldcg(reinterpret_cast<const float4*>(grads.p[s]) + off4 + i);
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      acc.x *= scale; acc.y *= scale; acc.z *= scale; acc.w *= scale;
      mine[off4 + i] = acc;
    }
  }
}

// chunks: int64 [n][3] = (first byte, bytes, owner), byte counts multiples of 16.
__global__ void zero_pull_params_kernel(const int64_t* __restrict__ chunks, int n_chunks, ZeroPeers params, int ws,
                                        int rank, const unsigned* __restrict__ flags, int slot, unsigned epoch,
                                        uint64_t timeout_ns, int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = zero_wait(flags, slot, ((1u << ws) - 1u) & ~(1u << rank), epoch, timeout_ns, err);
  __syncthreads();
  if (!ok) return;
  uint4* mine = reinterpret_cast<uint4*>(params.p[rank]);
  for (int c = blockIdx.x; c < n_chunks; c += gridDim.x) {
    const int64_t off16 = chunks[3 * c] / 16, n16 = chunks[3 * c + 1] / 16;
    const int owner = static_cast<int>(chunks[3 * c + 2]);
    if (owner == rank || owner < 0 || owner >= ws) continue;
    const uint4* src = reinterpret_cast<const uint4*>(params.p[owner]) + off16;
    for (int64_t i = threadIdx.x; i < n16; i += blockDim.x) mine[off16 + i] = __ldcg(src + i);
  }
}

}  // namespace

void zero_signal(std::vector<int64_t> flag_ptrs, int64_t slot, int64_t rank, int64_t epoch) {
  TORCH_CHECK(slot >= 0 && rank >= 0 && rank < static_cast<int64_t>(flag_ptrs.size()), "slot / rank");
  zero_signal_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      zero_table(flag_ptrs), static_cast<int>(slot), static_cast<int>(rank), static_cast<int>(flag_ptrs.size()),
      static_cast<unsigned>(epoch));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void zero_pull_reduce(torch::Tensor chunks, std::vector<int64_t> grad_ptrs, int64_t rank, double scale,
                      torch::Tensor my_flags, int64_t slot, int64_t epoch, int64_t timeout_ns, int64_t blocks,
                      torch::Tensor err) {
  TORCH_CHECK(chunks.scalar_type() == at::kLong && chunks.is_contiguous() && chunks.dim() == 2 && chunks.size(1) == 2,
              "chunks: int64 (n, 2)");
  for (auto p : grad_ptrs) TORCH_CHECK((p & 15) == 0, "gradient arenas 16-byte aligned");
  const int n = static_cast<int>(chunks.size(0));
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(chunks.device());
  zero_pull_reduce_kernel<<<static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(blocks, n))), 256, 0,
                            at::cuda::getCurrentCUDAStream()>>>(
      chunks.data_ptr<int64_t>(), n, zero_table(grad_ptrs), static_cast<int>(grad_ptrs.size()),
      static_cast<int>(rank), static_cast<float>(scale), reinterpret_cast<const unsigned*>(my_flags.data_ptr()),
      static_cast<int>(slot), static_cast<unsigned>(epoch), static_cast<uint64_t>(timeout_ns), err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void zero_pull_params(torch::Tensor chunks, std::vector<int64_t> param_ptrs, int64_t rank, torch::Tensor my_flags,
                      int64_t slot, int64_t epoch, int64_t timeout_ns, int64_t blocks, torch::Tensor err) {
  TORCH_CHECK(chunks.scalar_type() == at::kLong && chunks.is_contiguous() && chunks.dim() == 2 && chunks.size(1) == 3,
              "chunks: int64 (n, 3)");
  for (auto p : param_ptrs) TORCH_CHECK((p & 15) == 0, "parameter arenas 16-byte aligned");
  const int n = static_cast<int>(chunks.size(0));
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(chunks.device());
  zero_pull_params_kernel<<<static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(blocks, n))), 256, 0,
                            at::cuda::getCurrentCUDAStream()>>>(
      chunks.data_ptr<int64_t>(), n, zero_table(param_ptrs), static_cast<int>(param_ptrs.size()),
      static_cast<int>(rank), reinterpret_cast<const unsigned*>(my_flags.data_ptr()), static_cast<int>(slot),
      static_cast<unsigned>(epoch), static_cast<uint64_t>(timeout_ns), err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sv4
