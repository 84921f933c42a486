// Lightning-indexer scores on tcgen05 (reference: csa.py LightningIndexer, lines 91-156):
//
//   score[b, t, s] = sum_h w[b, t, h] * relu(q[b, t, h, :] . k[b, s, :])
//                    (+ 0.5 * vis[b, s] * sum_h w[b, t, h])
//   masked to -inf unless block s is complete strictly before t: s*m + m - 1 < t.
//
// One CTA per (128 queries x 128 blocks) tile; 6 warps: warp 4 issues TMA (the key
// tile once, then one query-head tile per head through a 3-stage ring), warp 5
// allocates TMEM and issues the MMAs (S_h = Q_h K^T, M = N = 128, K = c, into one of
// two TMEM buffers), warps 0-3 read S_h (thread = query row), apply ReLU and the head
// weight and accumulate in registers, so the (T, heads, blocks) tensor never exists.
// Tiles with no visible block only write -inf.  All waits are bounded.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>
#include <torch/extension.h>

#include "common.cuh"

namespace sv4 {

CUtensorMap make_map_nd(const void* base, CUtensorMapDataType dt, int rank, const uint64_t* dims,
                        const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz);

namespace {

constexpr uint32_t kIdxAtom = 16384;  // 128 rows x 128 B
constexpr int kIdxStages = 3;

struct IdxParams {
  const float* w;    // (B, T, nh) fp32
  const float* vis;  // (B, nb) or nullptr
  float* out;        // (B, T, nb) fp32
  int T, nb, nh, m, q_start;
  int* err;
};

__device__ __forceinline__ uint64_t idx_desc_k(uint32_t base, int s) {
  return make_smem_desc(base + (s >> 2) * kIdxAtom + (s & 3) * 32, 16, 1024, 2);
}

template <int A>
__global__ void __launch_bounds__(192, 1)
indexer_scores_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                      const IdxParams P) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bt = blockIdx.x, t0 = blockIdx.y * 128, b = blockIdx.z;
  const int n0 = bt * 128;
  // visible iff n*m + m - 1 < t for some query of the tile
  const int t_last = P.q_start + min(P.T, t0 + 128) - 1;
  const bool any_visible = static_cast<int64_t>(n0) * P.m + P.m - 1 < t_last;
  const int nb_tile = min(128, P.nb - n0);
  if (!any_visible) {
    for (int i = tid; i < 128 * nb_tile; i += blockDim.x) {
      const int r = i / nb_tile, c = i - r * nb_tile;
      if (t0 + r < P.T) P.out[(static_cast<int64_t>(b) * P.T + t0 + r) * P.nb + n0 + c] = -INFINITY;
    }
    return;
  }

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sQ = sK + A * kIdxAtom;
  float* sW = reinterpret_cast<float*>(sQ + kIdxStages * A * kIdxAtom);  // [nh][128]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sW + P.nh * 128);
  uint64_t* kfull = bar;
  uint64_t* qfull = bar + 1;
  uint64_t* qempty = qfull + kIdxStages;
  uint64_t* sfull = qempty + kIdxStages;
  uint64_t* sempty = sfull + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sempty + 2);

  if (tid == 0) {
    mbar_init(kfull, 1);
    for (int i = 0; i < kIdxStages; ++i) {
      mbar_init(&qfull[i], 1);
      mbar_init(&qempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sfull[i], 1);
      mbar_init(&sempty[i], 4);
    }
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  // head weights of the tile's rows, transposed so a thread reads its row per head
  for (int i = tid; i < 128 * P.nh; i += blockDim.x) {
    const int r = i / P.nh, hh = i - r * P.nh;
    sW[hh * 128 + r] = t0 + r < P.T ? P.w[(static_cast<int64_t>(b) * P.T + t0 + r) * P.nh + hh] : 0.f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const int nh = P.nh;

  if (warp == 4) {
    if (lane == 0) {
      mbar_arrive_expect_tx(kfull, A * kIdxAtom);
      for (int a = 0; a < A; ++a) tma_load_3d(sK + a * kIdxAtom, &mk, kfull, a * 64, n0, b);
      for (int h = 0; h < nh; ++h) {
        const int st = h % kIdxStages;
        if (h >= kIdxStages) mbar_wait(&qempty[st], ((h / kIdxStages) - 1) & 1, P.err, kErrTimeoutEmpty);
        uint8_t* dst = sQ + st * A * kIdxAtom;
        mbar_arrive_expect_tx(&qfull[st], A * kIdxAtom);
        for (int a = 0; a < A; ++a) tma_load_3d(dst + a * kIdxAtom, &mq, &qfull[st], (h * A + a) * 64, t0, b);
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t kId = make_idesc_f16(128, 128, 1, 1, false, false);
      mbar_wait(kfull, 0, P.err, kErrTimeoutFull);
      const uint32_t ak = smem_u32(sK);
      for (int h = 0; h < nh; ++h) {
        const int st = h % kIdxStages, buf = h & 1;
        mbar_wait(&qfull[st], (h / kIdxStages) & 1, P.err, kErrTimeoutFull);
        if (h >= 2) mbar_wait(&sempty[buf], ((h >> 1) - 1) & 1, P.err, kErrTimeoutAccum);
        tc_fence_after();
        const uint32_t aq = smem_u32(sQ + st * A * kIdxAtom);
#pragma unroll
        for (int s = 0; s < A * 4; ++s) mma_bf16(tbase + buf * 128, idx_desc_k(aq, s), idx_desc_k(ak, s), kId, s > 0);
        mma_commit(&qempty[st]);
        mma_commit(&sfull[buf]);
      }
    }
    __syncwarp();
  } else {
    float acc[128];
#pragma unroll
    for (int j = 0; j < 128; ++j) acc[j] = 0.f;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    for (int h = 0; h < nh; ++h) {
      const int buf = h & 1;
      mbar_wait(&sfull[buf], (h >> 1) & 1, P.err, kErrTimeoutAccum);
      __syncwarp();
      tc_fence_after();
      const float wv = sW[h * 128 + tid];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tbase + buf * 128 + c * 32 + lane_off, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[c * 32 + j] = fmaf(wv, fmaxf(__uint_as_float(r[j]), 0.f), acc[c * 32 + j]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sempty[buf]);
    }
    const int t = t0 + tid;
    if (t < P.T) {
      const int qpos = P.q_start + t;
      float wsum = 0.f;
      if (P.vis != nullptr)
        for (int h = 0; h < nh; ++h) wsum += sW[h * 128 + tid];
      float* row = P.out + (static_cast<int64_t>(b) * P.T + t) * P.nb + n0;
#pragma unroll
      for (int j = 0; j < 128; ++j) {
        const int n = n0 + j;
        float v = acc[j];
        if (P.vis != nullptr && j < nb_tile) v += 0.5f * P.vis[static_cast<int64_t>(b) * P.nb + n] * wsum;
        acc[j] = (static_cast<int64_t>(n) * P.m + P.m - 1 < qpos) ? v : -INFINITY;
      }
      if (nb_tile == 128 && (P.nb & 3) == 0) {
#pragma unroll
        for (int j = 0; j < 128; j += 4)
          *reinterpret_cast<float4*>(row + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 128; ++j)
          if (j < nb_tile) row[j] = acc[j];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) tmem_dealloc(tbase, 256);
}

CUtensorMap bf16_3d_map(const torch::Tensor& t, int64_t inner, int64_t rows, int64_t batch) {
  uint64_t dims[3] = {static_cast<uint64_t>(inner), static_cast<uint64_t>(rows), static_cast<uint64_t>(batch)};
  uint64_t strides[2] = {static_cast<uint64_t>(inner * 2), static_cast<uint64_t>(inner * rows * 2)};
  uint32_t box[3] = {64, 128, 1};
  return make_map_nd(t.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

void indexer_scores(torch::Tensor q, torch::Tensor keys, torch::Tensor w, c10::optional<torch::Tensor> vis,
                    int64_t m, int64_t q_start, torch::Tensor out, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && keys.scalar_type() == at::kBFloat16, "indexer: bf16 q / keys");
  TORCH_CHECK(w.scalar_type() == at::kFloat && out.scalar_type() == at::kFloat, "indexer: fp32 w / out");
  TORCH_CHECK(q.is_contiguous() && keys.is_contiguous() && w.is_contiguous() && out.is_contiguous(), "contiguous");
  const int64_t B = q.size(0), T = q.size(1), nb = keys.size(1), c = keys.size(2), nh = w.size(2);
  TORCH_CHECK(c == 64 || c == 128, "indexer head dim must be 64 or 128");
  TORCH_CHECK(q.size(2) == nh * c && keys.size(0) == B && w.size(0) == B && w.size(1) == T, "indexer shapes");
  TORCH_CHECK(nh >= 1 && nh <= 128, "indexer heads must be 1..128");
  TORCH_CHECK(out.size(0) == B && out.size(1) == T && out.size(2) == nb, "indexer out shape");
  if (B == 0 || T == 0 || nb == 0) return;
  if (vis.has_value()) TORCH_CHECK(vis->is_contiguous() && vis->scalar_type() == at::kFloat, "vis fp32");
  CUtensorMap mq = bf16_3d_map(q, nh * c, T, B), mk = bf16_3d_map(keys, c, nb, B);
  IdxParams P{w.data_ptr<float>(), vis.has_value() ? vis->data_ptr<float>() : nullptr, out.data_ptr<float>(),
              static_cast<int>(T), static_cast<int>(nb), static_cast<int>(nh), static_cast<int>(m),
              static_cast<int>(q_start), err.data_ptr<int>()};
  const int A = static_cast<int>(c / 64);
  const int smem = 1024 + (A + kIdxStages * A) * kIdxAtom + nh * 128 * 4 + 16 * 8 + 16;
  dim3 grid(static_cast<unsigned>((nb + 127) / 128), static_cast<unsigned>((T + 127) / 128),
            static_cast<unsigned>(B));
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  if (A == 2) {
    cudaFuncSetAttribute(indexer_scores_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    indexer_scores_kernel<2><<<grid, 192, smem, s>>>(mq, mk, P);
  } else {
    cudaFuncSetAttribute(indexer_scores_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    indexer_scores_kernel<1><<<grid, 192, smem, s>>>(mq, mk, P);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sv4
