// Expert-parallel dispatch / combine over NVLink peer memory, one process per GPU.
//
// Every rank owns the same set of "symmetric" buffers (same sizes, allocated
// collectively, mapped into every peer through CUDA IPC), so a kernel on rank s can
// store into / load from rank d's buffer through a plain pointer.  Per MoE call:
//
//   ep_post_counts   push this rank's per-expert pair counts into every peer's count
//                    table, then release a flag per peer               (phase CNT)
//   ep_plan          wait for all counts; compute each destination's receive layout
//                    (local experts back to back, each padded to 128 rows, rows of a
//                    segment ordered by source rank then token) and the global row of
//                    every (token, slot) pair: gpos = dst * C + row; the owner's segment
//                    table holds both the row counts and the 128-padded counts (the
//                    grouped GEMMs run over whole padded segments, padding rows zero)
//   ep_dispatch      push each token row into the k destination buffers (P2P stores)
//   ep_signal        fence + release one flag per peer                 (phase X / Y / DY / DX)
//   ep_wait_zero     wait for every source's flag, zero the padding rows of the
//                    receive buffer (the grouped GEMMs then run on it locally)
//   ep_combine       wait for the expert outputs, pull the k rows of each token from
//                    the owners (P2P loads) and reduce them with the gate weights;
//                    keeps a local copy of the pulled rows for the backward
//   ep_combine_bwd   dgate = <dout, y>, push gate * dout to the owners (P2P stores)
//   ep_dispatch_bwd  pull the k input-gradient rows of each token and sum them
//
// Ordering: a producer fences at system scope and then writes the consumer's flag
// with st.release.sys; the consumer polls with ld.acquire.sys.  Flags carry a
// per-phase epoch that every rank advances identically, so they are never reset.
// Every wait is bounded (iterations and %globaltimer); on timeout the kernel records
// kErrPeerTimeout in the error word and returns, leaving the context usable.  Data
// written by peers is read with L1-bypassing loads.  No TMA multicast anywhere.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

#include <vector>

#include "common.cuh"

namespace sv4 {

constexpr int kEpMaxRanks = 8;
constexpr int kEpPhaseCnt = 0;

struct PeerTable {
  unsigned long long p[kEpMaxRanks];
};

static PeerTable make_table(const std::vector<int64_t>& ptrs) {
  TORCH_CHECK(!ptrs.empty() && ptrs.size() <= kEpMaxRanks, "peer table: 1..8 ranks");
  PeerTable t{};
  for (size_t i = 0; i < ptrs.size(); ++i) t.p[i] = static_cast<unsigned long long>(ptrs[i]);
  return t;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_release_sys(unsigned* addr, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* addr) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// Wait until flags[phase][src] has reached `epoch` for every src < ws.  Bounded.
__device__ bool wait_flags(const unsigned* flags, int phase, int ws, unsigned epoch, uint64_t timeout_ns, int* err) {
  const uint64_t t0 = global_ns();
  for (int src = 0; src < ws; ++src) {
    const unsigned* f = flags + phase * kEpMaxRanks + src;
    uint32_t it = 0;
    while (static_cast<int>(ld_acquire_sys(f) - epoch) < 0) {
      ++it;
      if (it > kSpinLimit || ((it & 63u) == 0 && global_ns() - t0 > timeout_ns)) {
        record_error(err, kErrPeerTimeout);
        return false;
      }
      __nanosleep(64);
    }
  }
  return true;
}

// ----------------------------------------------------------------------- signals
__global__ void ep_signal_kernel(PeerTable flags, int phase, int rank, int ws, unsigned epoch) {
  __threadfence_system();
  if (threadIdx.x < ws)
    st_release_sys(reinterpret_cast<unsigned*>(flags.p[threadIdx.x]) + phase * kEpMaxRanks + rank, epoch);
}

void ep_signal(std::vector<int64_t> flag_ptrs, int64_t phase, int64_t rank, int64_t epoch) {
  ep_signal_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(make_table(flag_ptrs), phase, rank,
                                                                   static_cast<int>(flag_ptrs.size()),
                                                                   static_cast<unsigned>(epoch));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------ count exchange
// Count table of every rank: int32 [2 slots][kEpMaxRanks sources][E].
__global__ void ep_post_counts_kernel(const int* __restrict__ counts, int E, PeerTable cnt, PeerTable flags, int rank,
                                      int ws, int slot, unsigned epoch) {
  for (int i = threadIdx.x; i < ws * E; i += blockDim.x) {
    const int dst = i / E, e = i - dst * E;
    int* remote = reinterpret_cast<int*>(cnt.p[dst]) + (slot * kEpMaxRanks + rank) * E + e;
    *remote = counts[e];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < ws)
    st_release_sys(reinterpret_cast<unsigned*>(flags.p[threadIdx.x]) + kEpPhaseCnt * kEpMaxRanks + rank, epoch);
}

void ep_post_counts(torch::Tensor counts, std::vector<int64_t> cnt_ptrs, std::vector<int64_t> flag_ptrs, int64_t rank,
                    int64_t slot, int64_t epoch) {
  c10::cuda::CUDAGuard guard(counts.device());
  TORCH_CHECK(counts.scalar_type() == torch::kInt32 && counts.is_contiguous(), "counts: int32 contiguous");
  TORCH_CHECK(cnt_ptrs.size() == flag_ptrs.size(), "peer tables differ in size");
  ep_post_counts_kernel<<<1, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(
      counts.data_ptr<int>(), counts.numel(), make_table(cnt_ptrs), make_table(flag_ptrs), rank,
      static_cast<int>(cnt_ptrs.size()), slot, static_cast<unsigned>(epoch));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// One CTA.  tot[e] = rows of expert e over all sources; a destination's layout puts
// its local experts back to back, each padded to 128 rows; within a segment the rows
// of source 0 come first.  pos_local / seg_start_local are this rank's own
// token-ordered ranking of its pairs per expert (moe_route_plan over all E experts).
__global__ void ep_plan_kernel(const int64_t* __restrict__ idx, const int* __restrict__ pos_local,
                               const int* __restrict__ seg_start_local, int n_pairs, const int* my_cnt,
                               const unsigned* my_flags, int slot, unsigned epoch, int rank, int ws, int E, int C,
                               int* __restrict__ gpos, int* __restrict__ seg_start_dst, int* __restrict__ seg_rows_dst,
                               int* __restrict__ seg_pad_dst, uint64_t timeout_ns, int* err) {
  extern __shared__ int sm[];
  int* tot = sm;
  int* segg = sm + E;
  int* base = sm + 2 * E;
  __shared__ int ok;
  __shared__ int over[kEpMaxRanks];
  const int El = E / ws;
  if (threadIdx.x == 0) ok = wait_flags(my_flags, kEpPhaseCnt, ws, epoch, timeout_ns, err) ? 1 : 0;
  __syncthreads();
  if (!ok) {
    for (int p = threadIdx.x; p < n_pairs; p += blockDim.x) gpos[p] = -1;
    for (int e = threadIdx.x; e < El; e += blockDim.x) seg_start_dst[e] = seg_rows_dst[e] = seg_pad_dst[e] = 0;
    return;
  }
  const int* cnt = my_cnt + slot * kEpMaxRanks * E;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int s = 0, before = 0;
    for (int src = 0; src < ws; ++src) {
      const int v = __ldcv(cnt + src * E + e);
      s += v;
      if (src < rank) before += v;
    }
    tot[e] = s;
    base[e] = before;
  }
  __syncthreads();
  if (threadIdx.x < ws) {
    const int d = threadIdx.x;
    int run = 0;
    for (int el = 0; el < El; ++el) {
      segg[d * El + el] = run;
      run += (tot[d * El + el] + 127) & ~127;
    }
    over[d] = run > C ? 1 : 0;
    if (run > C) record_error(err, kErrCapacity);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) base[e] += segg[e];
  for (int el = threadIdx.x; el < El; el += blockDim.x) {
    seg_start_dst[el] = over[rank] ? 0 : segg[rank * El + el];
    seg_rows_dst[el] = over[rank] ? 0 : tot[rank * El + el];
    seg_pad_dst[el] = over[rank] ? 0 : (tot[rank * El + el] + 127) & ~127;
  }
  __syncthreads();
  for (int p = threadIdx.x; p < n_pairs; p += blockDim.x) {
    const int64_t e = idx[p];
    if (e < 0 || e >= E) {
      gpos[p] = -1;
      record_error(err, kErrBounds);
      continue;
    }
    const int d = static_cast<int>(e) / El;
    const int r = base[e] + (pos_local[p] - seg_start_local[e]);
    gpos[p] = (over[d] || r >= C) ? -1 : d * C + r;
  }
}

void ep_plan(torch::Tensor idx, torch::Tensor pos_local, torch::Tensor seg_start_local, torch::Tensor my_cnt,
             torch::Tensor my_flags, int64_t slot, int64_t epoch, int64_t rank, int64_t ws, int64_t C,
             torch::Tensor gpos, torch::Tensor seg_start_dst, torch::Tensor seg_rows_dst, torch::Tensor seg_pad_dst,
             int64_t timeout_ns, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(idx.device());
  TORCH_CHECK(idx.scalar_type() == torch::kInt64 && idx.is_contiguous(), "idx int64");
  const int E = seg_start_local.numel();
  TORCH_CHECK(ws >= 1 && ws <= kEpMaxRanks && E % ws == 0, "ep_plan: ws in 1..8 dividing E");
  TORCH_CHECK(my_cnt.numel() >= 2 * kEpMaxRanks * E, "count table too small");
  ep_plan_kernel<<<1, 1024, 3 * E * sizeof(int), at::cuda::getCurrentCUDAStream()>>>(
      idx.data_ptr<int64_t>(), pos_local.data_ptr<int>(), seg_start_local.data_ptr<int>(), idx.numel(),
      my_cnt.data_ptr<int>(), reinterpret_cast<const unsigned*>(my_flags.data_ptr<int>()), slot,
      static_cast<unsigned>(epoch), rank, ws, E, C, gpos.data_ptr<int>(), seg_start_dst.data_ptr<int>(),
      seg_rows_dst.data_ptr<int>(), seg_pad_dst.data_ptr<int>(), static_cast<uint64_t>(timeout_ns),
      err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// A global receive row (destination rank * C + row) of a (token, slot) pair, or -1 for a
// dropped pair.  Anything outside [-1, ws * C) is a corrupt layout: thread 0 of the CTA
// records kErrBounds and every thread treats the pair as dropped (no peer access).
__device__ __forceinline__ int checked_gpos(int p, int ws, int C, int* err) {
  const bool ok = threadIdx.x == 0 ? index_ok(p, -1, static_cast<int64_t>(ws) * C, err)
                                   : (p >= -1 && p < ws * C);
  return ok ? p : -1;
}

// ----------------------------------------------------------------- dispatch (push)
// One CTA per token: the row is read once and stored into each of its k destinations.
__global__ void ep_dispatch_kernel(const uint4* __restrict__ h, const int* __restrict__ gpos, int k, int vpr, int C,
                                   PeerTable xbuf, int ws, int* err) {
  const int t = blockIdx.x;
  int p[16];
  for (int j = 0; j < k; ++j) p[j] = checked_gpos(gpos[t * k + j], ws, C, err);
  for (int v = threadIdx.x; v < vpr; v += blockDim.x) {
    const uint4 val = h[static_cast<int64_t>(t) * vpr + v];
    for (int j = 0; j < k; ++j) {
      if (p[j] < 0) continue;
      const int d = p[j] / C, r = p[j] - d * C;
      reinterpret_cast<uint4*>(xbuf.p[d])[static_cast<int64_t>(r) * vpr + v] = val;
    }
  }
  __threadfence_system();
}

void ep_dispatch(torch::Tensor h, torch::Tensor gpos, int64_t C, std::vector<int64_t> x_ptrs, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(h.device());
  const int T = h.size(0), k = gpos.size(1);
  TORCH_CHECK(h.is_contiguous() && h.size(1) * h.element_size() % 16 == 0 && k <= 16, "ep_dispatch layout");
  if (T == 0) return;
  const int vpr = h.size(1) * h.element_size() / 16;
  ep_dispatch_kernel<<<T, std::min(256, std::max(32, vpr)), 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint4*>(h.data_ptr()), gpos.data_ptr<int>(), k, vpr, C, make_table(x_ptrs),
      static_cast<int>(x_ptrs.size()), err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ---------------------------------------------------- wait + zero the padding rows
// Grid: one CTA per local expert.  Rows [start + rows, start + pad128(rows)) are zeroed.
__global__ void ep_wait_zero_kernel(const unsigned* my_flags, int phase, int ws, unsigned epoch, uint4* buf, int vpr,
                                    const int* __restrict__ seg_start, const int* __restrict__ seg_rows,
                                    uint64_t timeout_ns, int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = wait_flags(my_flags, phase, ws, epoch, timeout_ns, err) ? 1 : 0;
  __syncthreads();
  if (!ok) return;
  const int e = blockIdx.x;
  const int rows = seg_rows[e];
  const int64_t s = seg_start[e] + rows, end = seg_start[e] + ((rows + 127) & ~127);
  for (int64_t i = threadIdx.x; i < (end - s) * vpr; i += blockDim.x) buf[s * vpr + i] = make_uint4(0, 0, 0, 0);
}

void ep_wait_zero(torch::Tensor my_flags, int64_t phase, int64_t ws, int64_t epoch, torch::Tensor buf,
                  torch::Tensor seg_start, torch::Tensor seg_rows, int64_t timeout_ns, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(buf.device());
  const int El = seg_start.numel();
  const int vpr = buf.size(1) * buf.element_size() / 16;
  ep_wait_zero_kernel<<<El, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const unsigned*>(my_flags.data_ptr<int>()), phase, ws, static_cast<unsigned>(epoch),
      reinterpret_cast<uint4*>(buf.data_ptr()), vpr, seg_start.data_ptr<int>(), seg_rows.data_ptr<int>(),
      static_cast<uint64_t>(timeout_ns), err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------ combine (pull)
__device__ __forceinline__ void acc_bf16x8(float* acc, const uint4& v, float g) {
  const __nv_bfloat162* hv = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 f = __bfloat1622float2(hv[q]);
    acc[2 * q] += g * f.x;
    acc[2 * q + 1] += g * f.y;
  }
}

__device__ __forceinline__ uint4 pack_bf16x8(const float* acc) {
  uint4 o;
  __nv_bfloat162* ho = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
  for (int q = 0; q < 4; ++q) ho[q] = __floats2bfloat162_rn(acc[2 * q], acc[2 * q + 1]);
  return o;
}

// One CTA per token: out[t] = sum_j gate[t,j] * y_{owner}[row]; rows are also copied to
// ypair[t*k + j] (zero for a dropped pair) for the backward.
__global__ void ep_combine_kernel(PeerTable ybuf, const int* __restrict__ gpos, const float* __restrict__ gate, int k,
                                  int C, int vpr, uint4* __restrict__ out, uint4* __restrict__ ypair,
                                  const unsigned* my_flags, int phase, int ws, unsigned epoch, uint64_t timeout_ns,
                                  int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = wait_flags(my_flags, phase, ws, epoch, timeout_ns, err) ? 1 : 0;
  __syncthreads();
  const int t = blockIdx.x;
  int p[16];
  float g[16];
  for (int j = 0; j < k; ++j) {
    p[j] = ok ? checked_gpos(gpos[t * k + j], ws, C, err) : -1;
    g[j] = gate[t * k + j];
  }
  for (int v = threadIdx.x; v < vpr; v += blockDim.x) {
    uint4 val[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (j >= k) break;
      if (p[j] < 0) {
        val[j] = make_uint4(0, 0, 0, 0);
      } else {
        const int d = p[j] / C, r = p[j] - d * C;
        val[j] = __ldcg(reinterpret_cast<const uint4*>(ybuf.p[d]) + static_cast<int64_t>(r) * vpr + v);
      }
    }
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (j >= k) break;
      acc_bf16x8(acc, val[j], g[j]);
      if (ypair != nullptr) ypair[(static_cast<int64_t>(t) * k + j) * vpr + v] = val[j];
    }
    out[static_cast<int64_t>(t) * vpr + v] = pack_bf16x8(acc);
  }
}

void ep_combine(std::vector<int64_t> y_ptrs, torch::Tensor gpos, torch::Tensor gate, int64_t C, torch::Tensor out,
                c10::optional<torch::Tensor> ypair, torch::Tensor my_flags, int64_t phase, int64_t ws, int64_t epoch,
                int64_t timeout_ns, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(out.device());
  const int T = out.size(0), k = gpos.size(1);
  TORCH_CHECK(out.is_contiguous() && out.size(1) * out.element_size() % 16 == 0 && k <= 16, "ep_combine layout");
  TORCH_CHECK(gate.scalar_type() == torch::kFloat32 && gate.is_contiguous(), "gate fp32");
  if (T == 0) return;
  const int vpr = out.size(1) * out.element_size() / 16;
  ep_combine_kernel<<<T, std::min(256, std::max(32, vpr)), 0, at::cuda::getCurrentCUDAStream()>>>(
      make_table(y_ptrs), gpos.data_ptr<int>(), gate.data_ptr<float>(), k, C, vpr,
      reinterpret_cast<uint4*>(out.data_ptr()), ypair.has_value() ? reinterpret_cast<uint4*>(ypair->data_ptr()) : nullptr,
      reinterpret_cast<const unsigned*>(my_flags.data_ptr<int>()), phase, ws, static_cast<unsigned>(epoch),
      static_cast<uint64_t>(timeout_ns), err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------- combine backward (push dy)
// One CTA per token (<= 256 threads): dgate[t,j] = <dout[t], ypair[t,j]>; the owner's
// dy row = gate[t,j] * dout[t].
__global__ void ep_combine_bwd_kernel(const uint4* __restrict__ dout, const uint4* __restrict__ ypair,
                                      const float* __restrict__ gate, const int* __restrict__ gpos, int k, int C,
                                      int vpr, PeerTable dybuf, float* __restrict__ dgate, int ws, int* err) {
  // Loops over the k slots are unrolled to the maximum (16) with an early exit, so the
  // per-slot arrays stay in registers and the k row loads of a chunk are issued together.
  const int t = blockIdx.x;
  int p[16];
  float g[16], dot[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    p[j] = j < k ? checked_gpos(gpos[t * k + j], ws, C, err) : -1;
    g[j] = j < k ? gate[t * k + j] : 0.f;
    dot[j] = 0.f;
  }
  for (int v = threadIdx.x; v < vpr; v += blockDim.x) {
    const uint4 a = dout[static_cast<int64_t>(t) * vpr + v];
    const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&a);
    float fa[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __bfloat1622float2(ha[q]);
      fa[2 * q] = f.x;
      fa[2 * q + 1] = f.y;
    }
    uint4 yb[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (j >= k) break;
      yb[j] = ypair[(static_cast<int64_t>(t) * k + j) * vpr + v];
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (j >= k) break;
      const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&yb[j]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(hb[q]);
        dot[j] += fa[2 * q] * f.x + fa[2 * q + 1] * f.y;
      }
      if (p[j] >= 0) {
        float s8[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) s8[q] = fa[q] * g[j];
        const int d = p[j] / C, r = p[j] - d * C;
        reinterpret_cast<uint4*>(dybuf.p[d])[static_cast<int64_t>(r) * vpr + v] = pack_bf16x8(s8);
      }
    }
  }
  __shared__ float red[8][16];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (j >= k) break;
    float x = dot[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if (lane == 0) red[wid][j] = x;
  }
  __syncthreads();
  if (threadIdx.x < k) {
    float s = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s += red[w][threadIdx.x];
    dgate[t * k + threadIdx.x] = s;
  }
  __threadfence_system();
}

void ep_combine_bwd(torch::Tensor dout, torch::Tensor ypair, torch::Tensor gate, torch::Tensor gpos, int64_t C,
                    std::vector<int64_t> dy_ptrs, torch::Tensor dgate, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(dout.device());
  const int T = dout.size(0), k = gpos.size(1);
  TORCH_CHECK(dout.is_contiguous() && ypair.is_contiguous() && k <= 16, "ep_combine_bwd layout");
  if (T == 0) return;
  const int vpr = dout.size(1) * dout.element_size() / 16;
  const int threads = std::min(256, std::max(32, (vpr + 31) / 32 * 32));
  ep_combine_bwd_kernel<<<T, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const uint4*>(dout.data_ptr()), reinterpret_cast<const uint4*>(ypair.data_ptr()),
      gate.data_ptr<float>(), gpos.data_ptr<int>(), k, C, vpr, make_table(dy_ptrs), dgate.data_ptr<float>(),
      static_cast<int>(dy_ptrs.size()), err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ----------------------------------------------------- dispatch backward (pull dx)
__global__ void ep_dispatch_bwd_kernel(PeerTable dxbuf, const int* __restrict__ gpos, int k, int C, int vpr,
                                       uint4* __restrict__ dh, const unsigned* my_flags, int phase, int ws,
                                       unsigned epoch, uint64_t timeout_ns, int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = wait_flags(my_flags, phase, ws, epoch, timeout_ns, err) ? 1 : 0;
  __syncthreads();
  const int t = blockIdx.x;
  int p[16];
  for (int j = 0; j < k; ++j) p[j] = ok ? checked_gpos(gpos[t * k + j], ws, C, err) : -1;
  for (int v = threadIdx.x; v < vpr; v += blockDim.x) {
    uint4 val[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (j >= k) break;
      if (p[j] < 0) {
        val[j] = make_uint4(0, 0, 0, 0);
      } else {
        const int d = p[j] / C, r = p[j] - d * C;
        val[j] = __ldcg(reinterpret_cast<const uint4*>(dxbuf.p[d]) + static_cast<int64_t>(r) * vpr + v);
      }
    }
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (j >= k) break;
      acc_bf16x8(acc, val[j], 1.0f);
    }
    dh[static_cast<int64_t>(t) * vpr + v] = pack_bf16x8(acc);
  }
}

void ep_dispatch_bwd(std::vector<int64_t> dx_ptrs, torch::Tensor gpos, int64_t C, torch::Tensor dh,
                     torch::Tensor my_flags, int64_t phase, int64_t ws, int64_t epoch, int64_t timeout_ns,
                     torch::Tensor err) {
  c10::cuda::CUDAGuard guard(dh.device());
  const int T = dh.size(0), k = gpos.size(1);
  TORCH_CHECK(dh.is_contiguous() && k <= 16, "ep_dispatch_bwd layout");
  if (T == 0) return;
  const int vpr = dh.size(1) * dh.element_size() / 16;
  ep_dispatch_bwd_kernel<<<T, std::min(256, std::max(32, vpr)), 0, at::cuda::getCurrentCUDAStream()>>>(
      make_table(dx_ptrs), gpos.data_ptr<int>(), k, C, vpr, reinterpret_cast<uint4*>(dh.data_ptr()),
      reinterpret_cast<const unsigned*>(my_flags.data_ptr<int>()), phase, ws, static_cast<unsigned>(epoch),
      static_cast<uint64_t>(timeout_ns), err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------- symmetric buffers
// cudaMalloc'd (outside the caching allocator, so the IPC handle covers exactly this
// buffer) and zero-filled.  The returned tensor does NOT own the memory: peers map it,
// so it may only be released by symm_free once every peer has stopped using it (the
// Python heap does that behind a barrier); a buffer never released lives until the
// process exits.
std::tuple<torch::Tensor, std::string> symm_alloc(int64_t nbytes, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&ptr, nbytes));
  C10_CUDA_CHECK(cudaMemset(ptr, 0, nbytes));
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, ptr));
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device);
  torch::Tensor t = torch::from_blob(ptr, {nbytes}, [](void*) {}, opts);
  return {t, std::string(reinterpret_cast<const char*>(&h), sizeof(h))};
}

void symm_free(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  C10_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr)));
}

int64_t symm_open(const std::string& handle, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  TORCH_CHECK(handle.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data(), sizeof(h));
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(ptr);
}

void symm_close(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

}  // namespace sv4
