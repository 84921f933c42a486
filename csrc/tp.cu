// Tensor-parallel all-reduce over NVLink peer memory (one process per GPU, TP ranks on one node).
//
// Every TP rank owns a symmetric receive buffer  recv[2 parities][ws sources][slot elems]  (bf16)
// and an arrival counter per source, both mapped into every peer through CUDA IPC.  A reduction
// of call c (parity c % 2) has two halves:
//
//   producer   the row-parallel projection itself (gemm_peer_push: the tcgen05 GEMM's epilogue
//              stores each output tile into every peer's slot while later tiles are still being
//              multiplied, then each CTA release-adds 1 to every peer's counter), or tp_push for
//              a tensor that is not produced by one GEMM (the input gradient of a TP block);
//   tp_reduce  waits until every source's counter reaches the expected cumulative arrivals
//              (bounded; on timeout it records kErrPeerTimeout and leaves `x` unreduced), then
//              x = sum over ranks in rank order (fp32 sums, bf16 out), so every rank gets
//              bit-identical results.
//
// Two parities suffice: a peer can be at most one call ahead, because its reduce of call c + 1
// waits for this rank's producer of call c + 1, which runs after this rank's reduce of call c.
// Counters are never reset; the host advances the expected counts identically on every rank
// (the producer's grid depends only on the shape).  No TMA and no multicast touch peer memory:
// the peer traffic is plain 16-byte stores.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

#include <vector>

#include "common.cuh"

namespace sv4 {
namespace {

constexpr int kTpMaxRanks = 8;

struct TpPeers {
  unsigned long long p[kTpMaxRanks];
};

TpPeers tp_table(const std::vector<int64_t>& v) {
  TORCH_CHECK(v.size() <= kTpMaxRanks, "at most 8 TP ranks");
  TpPeers t{};
  for (size_t i = 0; i < v.size(); ++i) t.p[i] = static_cast<unsigned long long>(v[i]);
  return t;
}

__device__ __forceinline__ uint64_t tp_now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned tp_ld_acquire(const unsigned* a) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}

// x (n bf16, n % 8 == 0) -> every peer's slot; then one release-add per CTA per peer.  Each
// thread moves 4 independent 16-byte vectors per iteration (loads issued before the stores), so
// enough remote stores are in flight to fill the link.
constexpr int kTpUnroll = 4;

__global__ void tp_push_kernel(const uint4* __restrict__ x, int64_t n8, TpPeers slots, TpPeers cnts, int n_peers) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i0 < n8; i0 += stride * kTpUnroll) {
    uint4 v[kTpUnroll];
#pragma unroll
    for (int u = 0; u < kTpUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < n8) v[u] = x[i];
    }
    for (int p = 0; p < n_peers; ++p) {
      uint4* dst = reinterpret_cast<uint4*>(slots.p[p]);
#pragma unroll
      for (int u = 0; u < kTpUnroll; ++u) {
        const int64_t i = i0 + u * stride;
        if (i < n8) dst[i] = v[u];
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < n_peers)
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(cnts.p[threadIdx.x]), "r"(1u) : "memory");
}

// x (n bf16) += the other ranks' slots, summed in rank order.  recv: this parity's
// [ws][slot_elems] block of the local receive buffer; cnt: the local counters [ws].
__global__ void tp_reduce_kernel(uint4* __restrict__ x, int64_t n8, const __nv_bfloat16* __restrict__ recv,
                                 int64_t slot_elems, const unsigned* __restrict__ cnt, TpPeers expect, int rank,
                                 int ws, uint64_t timeout_ns, int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const uint64_t t0 = tp_now_ns();
    for (int s = 0; s < ws && ok; ++s) {
      if (s == rank) continue;
      const unsigned want = static_cast<unsigned>(expect.p[s]);
      uint32_t it = 0;
      while (static_cast<int>(tp_ld_acquire(cnt + s) - want) < 0) {
        ++it;
        if (it > kSpinLimit || ((it & 63u) == 0 && tp_now_ns() - t0 > timeout_ns)) {
          record_error(err, kErrPeerTimeout);
          ok = 0;
          break;
        }
        __nanosleep(64);
      }
    }
  }
  __syncthreads();
  if (!ok) return;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i0 < n8; i0 += stride * kTpUnroll) {
    float acc[kTpUnroll][8];
#pragma unroll
    for (int u = 0; u < kTpUnroll; ++u)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[u][j] = 0.f;
    for (int s = 0; s < ws; ++s) {
      uint4 v[kTpUnroll];
#pragma unroll
      for (int u = 0; u < kTpUnroll; ++u) {  // all loads of this source first
        const int64_t i = i0 + u * stride;
        if (i < n8) v[u] = s == rank ? x[i] : __ldcg(reinterpret_cast<const uint4*>(recv + s * slot_elems) + i);
      }
#pragma unroll
      for (int u = 0; u < kTpUnroll; ++u) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[u]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h[j]);
          acc[u][2 * j] += f.x;
          acc[u][2 * j + 1] += f.y;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kTpUnroll; ++u) {
      const int64_t i = i0 + u * stride;
      if (i >= n8) continue;
      uint4 o;
      __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) oh[j] = __floats2bfloat162_rn(acc[u][2 * j], acc[u][2 * j + 1]);
      x[i] = o;
    }
  }
}

int tp_grid(int64_t n8) {
  int dev = 0;
  cudaGetDevice(&dev);
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n8 + 255) / 256, 2 * sms)));
}

}  // namespace

// Push x (contiguous bf16, numel % 8 == 0) into every peer's slot; returns the grid (arrivals
// per peer).
int64_t tp_push(torch::Tensor x, std::vector<int64_t> peer_slots, std::vector<int64_t> peer_cnts) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.numel() % 8 == 0,
              "x: contiguous bf16 with numel % 8 == 0");
  TORCH_CHECK(peer_slots.size() == peer_cnts.size() && !peer_slots.empty(), "peer tables");
  for (auto a : peer_slots) TORCH_CHECK((a & 15) == 0, "peer slots 16-byte aligned");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t n8 = x.numel() / 8;
  const int grid = tp_grid(n8);
  tp_push_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint4*>(x.data_ptr()), n8, tp_table(peer_slots), tp_table(peer_cnts),
      static_cast<int>(peer_slots.size()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return grid;
}

// x += the other ranks' contributions (see the file comment).  recv_parity: uint8 view of this
// parity's [ws][slot_elems] bf16 block; counters: int32 [ws]; expect[s]: cumulative arrivals.
void tp_reduce(torch::Tensor x, torch::Tensor recv_parity, int64_t slot_elems, torch::Tensor counters,
               std::vector<int64_t> expect, int64_t rank, int64_t timeout_ns, torch::Tensor err) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.is_contiguous() && x.numel() % 8 == 0 &&
                  x.numel() <= slot_elems, "x: contiguous bf16, numel % 8 == 0, fits the slot");
  const int ws = static_cast<int>(expect.size());
  TORCH_CHECK(ws >= 1 && ws <= kTpMaxRanks && rank >= 0 && rank < ws, "rank / world");
  TORCH_CHECK(recv_parity.numel() >= ws * slot_elems * 2 && counters.numel() >= ws, "receive buffer / counters");
  TORCH_CHECK(slot_elems % 8 == 0, "slot_elems % 8 == 0");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t n8 = x.numel() / 8;
  tp_reduce_kernel<<<tp_grid(n8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<uint4*>(x.data_ptr()), n8, reinterpret_cast<const __nv_bfloat16*>(recv_parity.data_ptr()),
      slot_elems, reinterpret_cast<const unsigned*>(counters.data_ptr()), tp_table(expect), static_cast<int>(rank),
      ws, static_cast<uint64_t>(timeout_ns), err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sv4
