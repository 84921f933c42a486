// Allocation-free RMSNorm backward (see noalloc.h for the contract).
//
//   dx = r * (w * dy - x * r^2 * mean(w * dy * x))        per row, r = rstd[row]
//   dw = sum over rows of dy * x * r
//
// Pass 1: up to SV4_NOALLOC_MAX_BLOCKS blocks each take a contiguous range of rows,
// write dx, and store their partial dw row in the static scratch array.  Inside a block
// each of the four warps accumulates its rows' dw into its own shared-memory row (every
// lane owns its columns, so no atomics), and the four rows are summed in a fixed order.
// Pass 2: one thread per column sums the partial rows into the caller's dw, in block
// order.  The result is therefore bit-reproducible from call to call.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "noalloc.h"

namespace {

constexpr int kMaxDevices = 64;

// File-scope scratch: per-block partial dW rows.  In host code this name is only a
// stand-in for the symbol; kernels receive the device address looked up below.
static __device__ __align__(256) float g_rmsnorm_bwd_scratch[SV4_NOALLOC_MAX_BLOCKS * SV4_NOALLOC_MAX_DIM];

enum : int {
  kOk = 0,
  kBadDim = 1,
  kBadRows = 2,
  kTooManyBlocks = 3,
  kMisaligned = 4,
  kSetupFailed = 5,
  kLaunchFailed = 6,
  kNoDevice = 7,
  kPriorError = 8,
};

constexpr int kWarps = 4;  // shared memory: kWarps x dim floats (128 KiB at dim 8192)

float* g_scratch_addr[kMaxDevices] = {nullptr};
bool g_smem_ready[kMaxDevices] = {false};
std::mutex g_setup_mutex;

__device__ __forceinline__ float warp_sum32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void load8f(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 t = __bfloat1622float2(h[q]);
    f[2 * q] = t.x;
    f[2 * q + 1] = t.y;
  }
}

__global__ void noalloc_rmsnorm_bwd_partial(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                            const float* __restrict__ w, const float* __restrict__ rstd,
                                            __nv_bfloat16* __restrict__ dx, float* __restrict__ scratch, int rows,
                                            int D, int rows_per_block) {
  extern __shared__ float sdw[];  // kWarps rows of D floats: one partial dw row per warp
  for (int d = threadIdx.x; d < kWarps * D; d += blockDim.x) sdw[d] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  float* mine = sdw + static_cast<long long>(warp) * D;
  const int row0 = blockIdx.x * rows_per_block;
  const int row1 = min(rows, row0 + rows_per_block);
  for (int row = row0 + warp; row < row1; row += kWarps) {
    const float r = rstd[row];
    const __nv_bfloat16* xr = x + static_cast<long long>(row) * D;
    const __nv_bfloat16* gr = dy + static_cast<long long>(row) * D;
    float dot = 0.f;
    for (int d = lane * 8; d < D; d += 256) {
      float fx[8], fg[8];
      load8f(xr + d, fx);
      load8f(gr + d, fg);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        dot += w[d + q] * fg[q] * fx[q];
        mine[d + q] += fg[q] * fx[q] * r;  // this lane's own columns of this warp's row
      }
    }
    dot = warp_sum32(dot) / D;
    __nv_bfloat16* dr = dx + static_cast<long long>(row) * D;
    for (int d = lane * 8; d < D; d += 256) {
      float fx[8], fg[8];
      load8f(xr + d, fx);
      load8f(gr + d, fg);
      uint4 o;
      __nv_bfloat162* ho = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float a = r * (w[d + 2 * q] * fg[2 * q] - fx[2 * q] * r * r * dot);
        const float b = r * (w[d + 2 * q + 1] * fg[2 * q + 1] - fx[2 * q + 1] * r * r * dot);
        ho[q] = __floats2bfloat162_rn(a, b);
      }
      *reinterpret_cast<uint4*>(dr + d) = o;
    }
  }
  __syncthreads();
  // every block writes its full partial row (warps summed in order), so the scratch never
  // needs clearing
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) acc += sdw[static_cast<long long>(k) * D + d];
    scratch[static_cast<long long>(blockIdx.x) * D + d] = acc;
  }
}

__global__ void noalloc_rmsnorm_bwd_reduce(const float* __restrict__ scratch, float* __restrict__ dw, int D,
                                           int n_blocks) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= D) return;
  float s = 0.f;
  for (int b = 0; b < n_blocks; ++b) s += scratch[static_cast<long long>(b) * D + d];
  dw[d] = s;
}

// Device address of the scratch array for the current device (looked up once).
float* scratch_for_current_device(int* code) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *code = kNoDevice;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_rmsnorm_bwd_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *code = kSetupFailed;
      return nullptr;
    }
    g_scratch_addr[dev] = static_cast<float*>(p);
  }
  if (!g_smem_ready[dev]) {  // the per-warp partial rows need more than the default 48 KiB
    const int bytes = static_cast<int>(sizeof(float)) * kWarps * SV4_NOALLOC_MAX_DIM;
    if (cudaFuncSetAttribute(noalloc_rmsnorm_bwd_partial, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
        cudaSuccess) {
      *code = kSetupFailed;
      return nullptr;
    }
    g_smem_ready[dev] = true;
  }
  return g_scratch_addr[dev];
}

bool aligned16(const void* p) { return (reinterpret_cast<unsigned long long>(p) & 15ull) == 0; }

}  // namespace

extern "C" __attribute__((visibility("default"))) int sv4_rmsnorm_bwd_noalloc(
    const void* dy, const void* x, const float* w, const float* rstd, void* dx, float* dw, int rows, int dim,
    void* stream) {
  if (dim <= 0 || dim % 8 != 0 || dim > SV4_NOALLOC_MAX_DIM) return kBadDim;
  if (rows < 0) return kBadRows;
  if (!aligned16(dy) || !aligned16(x) || !aligned16(dx)) return kMisaligned;
  // an error left pending by earlier work on this thread is reported, not consumed: the
  // launch-error checks below would otherwise mistake it for this call's
  if (cudaPeekAtLastError() != cudaSuccess) return kPriorError;
  int code = kOk;
  float* scratch = scratch_for_current_device(&code);
  if (scratch == nullptr) return code;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    if (cudaMemsetAsync(dw, 0, sizeof(float) * dim, s) != cudaSuccess) return kLaunchFailed;
    return kOk;
  }
  const int rows_per_block = (rows + SV4_NOALLOC_MAX_BLOCKS - 1) / SV4_NOALLOC_MAX_BLOCKS;
  const int n_blocks = (rows + rows_per_block - 1) / rows_per_block;
  if (n_blocks > SV4_NOALLOC_MAX_BLOCKS) return kTooManyBlocks;
  noalloc_rmsnorm_bwd_partial<<<n_blocks, 32 * kWarps, sizeof(float) * kWarps * dim, s>>>(
      static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x), w, rstd,
      static_cast<__nv_bfloat16*>(dx), scratch, rows, dim, rows_per_block);
  if (cudaGetLastError() != cudaSuccess) return kLaunchFailed;
  noalloc_rmsnorm_bwd_reduce<<<(dim + 255) / 256, 256, 0, s>>>(scratch, dw, dim, n_blocks);
  if (cudaGetLastError() != cudaSuccess) return kLaunchFailed;
  return kOk;
}

extern "C" __attribute__((visibility("default"))) const char* sv4_noalloc_error_string(int code) {
  switch (code) {
    case kOk: return "ok";
    case kBadDim: return "dim must be a positive multiple of 8 and at most SV4_NOALLOC_MAX_DIM (8192)";
    case kBadRows: return "rows must be non-negative";
    case kTooManyBlocks: return "internal: block count exceeds SV4_NOALLOC_MAX_BLOCKS";
    case kMisaligned: return "dy, x and dx must be 16-byte aligned";
    case kSetupFailed: return "set-up failed on this device (scratch address lookup or shared-memory opt-in)";
    case kLaunchFailed: return "kernel launch failed";
    case kNoDevice: return "no current CUDA device (or device index too large)";
    case kPriorError: return "a CUDA error from earlier work is pending on this thread (left for its owner to read)";
    default: return "unknown error code";
  }
}
