// Block-scaled FP8 GEMM on the sm_100a tensor cores, and the quantisation kernels feeding it.
//
//   D[m, n] = sum_k (A[m, k] * sa[m, k / 128]) * (B[n, k] * sb[n / 128, k / 128])      (bf16 D)
//
// A (activations) is quantised in 1 x 128 blocks, B (weights, (N, K) row-major) in 128 x 128
// blocks; values are E4M3, scales powers of two stored as UE8M0 bytes (2^(byte - 127)).  The
// forward recipe follows the reference's FP8 linear (kernels/fp8_gemm.py:24-101 scales a
// rowwise activation and a per-channel weight through torch._scaled_mm); here the blocks are
// finer and the scaling is done by the MMA itself: tcgen05.mma kind::mxf8f6f4.block_scale reads
// one scale per row of A and per column of B for every 32-element K step from tensor memory, so
// no per-block promotion runs on the CUDA cores.
//
// Scale-factor layout (produced by the quantisation kernels, consumed by the GEMM): for an
// operand of R rows (padded to a multiple of 128) and K columns, chunk (rb, kg) covers rows
// [128 rb, 128 rb + 128) and the four 128-column K blocks 4 kg .. 4 kg + 3; it is 512
// contiguous bytes at ((rb * KG) + kg) * 512 with KG = ceil(K / 512).  Row r of the chunk owns
// the 32-bit word at byte 16 * (r % 32) + 4 * (r / 32), whose byte j is the scale of K block
// 4 kg + j.  That is the shape tcgen05.cp 32x128b.warpx4 copies into tensor memory: smem row
// r % 32 (16 bytes) lands in lane r % 32 of every lane quarter, word i in column i, which is
// where the MMA looks for the scales of row r % 32 + 32 i; the instruction descriptor's
// scale-factor id picks byte j for the MMAs of K block 4 kg + j.  One copy per 512 columns of
// K keeps tcgen05.cp off the MMA stream's critical path.
//
// GEMM roles (one CTA per SM, persistent over 128 x 128 output tiles):
//   warp 0     : producer -- TMA loads of the A and B k-blocks (128 x 128 bytes each, 128B
//                swizzle) into a 6-deep ring, plus bulk copies of the two 512-byte scale chunks
//                with the first k-block of every group of four;
//   warp 1     : MMA issuer -- tcgen05.cp of a group's scale chunks into tensor memory, then
//                four M=128, N=128, K=32 block-scaled MMAs per k-block into one of two
//                accumulators;
//   warps 2..5 : epilogue -- tcgen05.ld, bf16 pack, TMA stores through swizzled staging.
// Tensor memory: accumulators in columns [0, 256), scale factors in two alternating slots at
// columns 256 + 8 s (A) and 256 + 8 s + 4 (B).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_fp8.h>
#include <torch/extension.h>

#include "gemm.cuh"

namespace sv4 {

CUtensorMap make_map_3d(const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t d0, uint64_t d1,
                        uint64_t d2, uint64_t s1_bytes, uint64_t s2_bytes, uint32_t b0, uint32_t b1,
                        CUtensorMapSwizzle swz);

namespace {

constexpr float kE4M3Max = 448.0f;
constexpr int kF8BN = 128;
constexpr int kF8BK = 128;  // elements = bytes = one 128B swizzle row
constexpr int kF8Stages = 6;
constexpr int kF8ABytes = kBM * kF8BK;
constexpr int kF8BBytes = kF8BN * kF8BK;
constexpr int kF8StageBytes = kF8ABytes + kF8BBytes;
constexpr int kSfChunk = 512;
constexpr int kF8SfOffset = kF8Stages * kF8StageBytes;
constexpr int kF8EpiOffset = kF8SfOffset + kF8Stages * 2 * kSfChunk;
constexpr int kF8BarOffset = kF8EpiOffset + 4 * kEpiStageBytes;  // one staging buffer per epilogue warp
constexpr int kF8SmemTotal = kF8BarOffset + 256 + 1024;
constexpr int kF8SfTmemCol = 2 * kF8BN;
constexpr uint32_t kF8TmemCols = 512;
static_assert(kF8SfTmemCol + 16 <= static_cast<int>(kF8TmemCols), "tensor memory budget");
static_assert(kF8SmemTotal <= 232448, "shared memory budget");

// Exponent e of the smallest power of two with amax / 2^e <= 448 (amax == 0 -> 0): the
// exponent of r = amax / 448 rounded up, read from its bits (exact, no log2).
__device__ __forceinline__ int pow2_exponent(float amax) {
  if (!(amax > 0.f)) return 0;
  const uint32_t b = __float_as_uint(__fdiv_rn(amax, kE4M3Max));
  int e = static_cast<int>((b >> 23) & 0xFFu) - 127;
  if ((b & 0x7FFFFFu) != 0u) e += 1;
  return max(-126, min(126, e));
}

__device__ __forceinline__ float exp2_int(int e) {  // 2^e for e in [-126, 127]
  return __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
}

__device__ __forceinline__ uint2 quant8x(const float* v, float inv) {
  uint32_t w[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    const __nv_fp8x2_storage_t p =
        __nv_cvt_float2_to_fp8x2(make_float2(v[i] * inv, v[i + 1] * inv), __NV_SATFINITE, __NV_E4M3);
    w[i / 4] |= static_cast<uint32_t>(p) << (8 * (i % 4));
  }
  return make_uint2(w[0], w[1]);
}

__device__ __forceinline__ void unpack8(const uint4& u, float* v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__host__ __device__ __forceinline__ int64_t sf_groups(int64_t k) { return (k / 128 + 3) / 4; }

// Byte holding the scale of row r (of its 128-row block rb) for K block kb.
__device__ __forceinline__ int64_t sf_byte_offset(int64_t rb, int64_t kb, int64_t kgroups, int r) {
  return (rb * kgroups + kb / 4) * kSfChunk + 16 * (r & 31) + 4 * (r >> 5) + (kb & 3);
}

// 1 x 128 activation quantisation: one 16-lane group per block, 8 elements per lane.  Rows in
// [M, Mpad) get the neutral scale byte (their A rows are zero-filled by TMA).  With a row map
// (MoE gather fused into the quantisation) output row r takes source row row_map[r] (-1: a zero
// padding row); a source row outside [-1, src_rows) records kErrBounds and is zero.
__global__ void __launch_bounds__(256) quant_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int M,
                                                         int Mpad, int K, uint8_t* __restrict__ q, int64_t ldq,
                                                         uint8_t* __restrict__ sf, float* __restrict__ scale,
                                                         const int* __restrict__ row_map, int src_rows, int* err) {
  const int kblocks = K / 128;
  const int64_t g = static_cast<int64_t>(blockIdx.x) * 16 + threadIdx.x / 16;
  const int sub = threadIdx.x & 15;
  const bool active = g < static_cast<int64_t>(Mpad) * kblocks;
  const int row = active ? static_cast<int>(g / kblocks) : 0;
  const int kb = active ? static_cast<int>(g % kblocks) : 0;
  const bool in_rows = active && row < M;
  int64_t src = row;
  if (row_map != nullptr && in_rows) {
    const int t = row_map[row];
    src = (sub == 0 && kb == 0) ? (index_ok(t, -1, src_rows, err) ? t : -1) : ((t >= -1 && t < src_rows) ? t : -1);
  }
  const bool live = in_rows && src >= 0;
  float v[8];
  if (live) {
    unpack8(*reinterpret_cast<const uint4*>(x + src * ldx + kb * 128 + sub * 8), v);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const int e = pow2_exponent(amax);
  if (in_rows) *reinterpret_cast<uint2*>(q + row * ldq + kb * 128 + sub * 8) = quant8x(v, exp2_int(-e));
  if (active && sub == 0) {
    sf[sf_byte_offset(row / 128, kb, sf_groups(K), row & 127)] = static_cast<uint8_t>(e + 127);
    if (in_rows && scale != nullptr) scale[static_cast<int64_t>(row) * kblocks + kb] = exp2_int(e);
  }
}

// 128 x 128 weight quantisation: one CTA per block; lane group (warp w, half h) covers rows
// {16 i + 2 w + h}, 16 lanes x 8 columns.  With a second source (gate / up pair of a SwiGLU
// expert pool, each (E * I, K) with I % 64 == 0) the quantised matrix is the interleave the
// SwiGLU epilogue reads: block row nb of expert e = nb / (2I / 128) holds 64 gate rows then the
// matching 64 up rows (rows j * 64 .. j * 64 + 63 of that expert, j = nb mod (2I / 128)).
__global__ void __launch_bounds__(256) quant_blocks_kernel(const __nv_bfloat16* __restrict__ w,
                                                           const __nv_bfloat16* __restrict__ w_up, int I,
                                                           int64_t ldw, int K, uint8_t* __restrict__ q, int64_t ldq,
                                                           uint8_t* __restrict__ sf, float* __restrict__ scale) {
  __shared__ float red[8];
  const int nb = blockIdx.y, kb = blockIdx.x, kblocks = K / 128;
  const int r0 = threadIdx.x / 16, sub = threadIdx.x & 15;
  auto src_row = [&](int r) -> const __nv_bfloat16* {
    if (w_up == nullptr) return w + (static_cast<int64_t>(nb) * 128 + r) * ldw;
    const int per = 2 * I / 128;
    const int64_t e = nb / per, j = nb % per;
    const int64_t row = e * I + j * 64 + (r & 63);
    return (r < 64 ? w : w_up) + row * ldw;
  };
  float v[8][8];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    unpack8(*reinterpret_cast<const uint4*>(src_row(r0 + 16 * i) + kb * 128 + sub * 8), v[i]);
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) amax = fmaxf(amax, red[i]);
  const int e = pow2_exponent(amax);
  const float inv = exp2_int(-e);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t row = static_cast<int64_t>(nb) * 128 + r0 + 16 * i;
    *reinterpret_cast<uint2*>(q + row * ldq + kb * 128 + sub * 8) = quant8x(v[i], inv);
  }
  if (threadIdx.x < 128) sf[sf_byte_offset(nb, kb, sf_groups(K), threadIdx.x)] = static_cast<uint8_t>(e + 127);
  if (threadIdx.x == 0 && scale != nullptr) scale[static_cast<int64_t>(nb) * kblocks + kb] = exp2_int(e);
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// 32 rows x 16 bytes of shared memory -> 4 columns of every lane quarter of tensor memory.
__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// kind::mxf8f6f4 block-scaled instruction descriptor: E4M3 x E4M3, K-major A and B, UE8M0
// scales, scale-factor byte 0 of each word (the four bytes of a word are equal here).
__host__ __device__ constexpr uint32_t make_idesc_mxf8(int m, int n) {
  return (0u << 7)                                 // A format E4M3
         | (0u << 10)                              // B format E4M3
         | (static_cast<uint32_t>(n >> 3) << 17)   // N / 8
         | (1u << 23)                              // scale format UE8M0
         | (static_cast<uint32_t>(m >> 4) << 24);  // M / 16
}

struct F8Params {
  // single problem: D (m x n) = A (m x k) B (n x k)^T, tiles row-major over (m / 128, n / 128)
  int m, n, k;
  int tiles_n, total;
  // grouped (table) mode: per-expert problems of the MoE layer (rows of A in 128-aligned
  // segments, B = experts stacked along rows, b_rows rows each)
  const GemmProblem* probs;
  const int* total_tiles;
  int n_probs, b_rows;
  int write_pre;                   // SwiGLU: also store the gate / up pre-activations
  float gate_max, lin_lo, lin_hi;  // SwiGLU clamps
  const uint8_t* sfa;
  const uint8_t* sfb;
  int* err;
};

enum F8Epi : int { kF8EpiBF16 = 0, kF8EpiSwiGLU = 1 };

// Where one output tile reads and writes.
struct F8Tile {
  int a_row, b_row;   // first row of the A / B tile (multiples of 128)
  int k;              // reduction length
  int d_row, d_col;   // first output row / column
  int aux_row, n;     // SwiGLU: first pre-activation row; problem width (I)
  bool store;         // rows of this tile exist in D
};

template <int EPI, bool TABLE>
__device__ __forceinline__ bool f8_locate(const F8Params& P, int t, int& hint, F8Tile& tl) {
  constexpr int kOut = EPI == kF8EpiSwiGLU ? kF8BN / 2 : kF8BN;  // output columns per tile
  if (!TABLE) {
    const int mt = t / P.tiles_n, nt = t % P.tiles_n;
    tl.a_row = mt * kBM; tl.b_row = nt * kF8BN; tl.k = P.k;
    tl.d_row = mt * kBM; tl.d_col = nt * kOut; tl.aux_row = tl.d_row; tl.n = P.n;
    tl.store = true;
    return true;
  }
  while (hint + 1 < P.n_probs && P.probs[hint + 1].tile_begin <= t) ++hint;
  const GemmProblem& pr = P.probs[hint];
  const int tn = (pr.n + kOut - 1) / kOut;
  const int local = t - pr.tile_begin;
  if (local < 0 || tn == 0 || local >= ((pr.m + kBM - 1) / kBM) * tn) return false;
  const int mt = local / tn, nt = local % tn;
  tl.a_row = pr.a_m + mt * kBM;
  tl.b_row = pr.b_b * P.b_rows + nt * kF8BN;
  tl.k = pr.k;
  tl.d_row = static_cast<int>(pr.d_off / pr.d_ld) + mt * kBM;
  tl.d_col = nt * kOut;
  tl.aux_row = EPI == kF8EpiSwiGLU ? static_cast<int>(pr.aux_off / pr.aux_ld) + mt * kBM : tl.d_row;
  tl.n = pr.n;
  tl.store = true;  // whole 128-row tiles: segments are padded to 128 rows inside the buffers
  return true;
}

// Stage 32 rows x 128 bytes (row = lane) in this warp's buffer and TMA-store them.
template <typename Pack>
__device__ __forceinline__ void f8_store(uint8_t* stg, int lane, Pack pack, const CUtensorMap* map, int c0, int c1,
                                         bool issue) {
  if (lane == 0) bulk_wait_read<0>();  // one buffer per warp: the previous store has read it
  __syncwarp();
  uint8_t* myrow = stg + lane * 128;
#pragma unroll
  for (int q = 0; q < 8; ++q) *reinterpret_cast<uint4*>(myrow + ((q ^ (lane & 7)) << 4)) = pack(q);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0 && issue) {
    tma_store_3d(map, stg, c0, c1, 0);
    bulk_commit_group();
  }
}

template <int EPI, bool TABLE>
__global__ void __launch_bounds__(192, 1)
gemm_mxf8_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                 const __grid_constant__ CUtensorMap map_d, const __grid_constant__ CUtensorMap map_aux,
                 const F8Params P) {
  constexpr uint32_t kIdesc = make_idesc_mxf8(kBM, kF8BN);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kF8BarOffset);
  uint64_t* empty = full + kF8Stages;
  uint64_t* acc_full = empty + kF8Stages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kF8Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kF8TmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    tma_prefetch_desc(&map_d);
    if (EPI == kF8EpiSwiGLU) tma_prefetch_desc(&map_aux);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = TABLE ? *P.total_tiles : P.total;

  if (warp == 0) {
    if (elect_one()) {
      int stage = 0, hint = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        F8Tile tl;
        if (!f8_locate<EPI, TABLE>(P, t, hint, tl)) continue;
        const int kblocks = tl.k / kF8BK;
        const int64_t kgroups = sf_groups(tl.k);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, P.err, kErrTimeoutEmpty)) { ok = false; break; }
          uint8_t* sa = smem + stage * kF8StageBytes;
          uint8_t* sfs = smem + kF8SfOffset + stage * 2 * kSfChunk;
          const bool group_start = (kb & 3) == 0;
          mbar_arrive_expect_tx(&full[stage], kF8StageBytes + (group_start ? 2 * kSfChunk : 0));
          tma_load_3d(sa, &map_a, &full[stage], kb * kF8BK, tl.a_row, 0);
          tma_load_3d(sa + kF8ABytes, &map_b, &full[stage], kb * kF8BK, tl.b_row, 0);
          if (group_start) {
            bulk_load(sfs, P.sfa + (tl.a_row / kBM * kgroups + kb / 4) * kSfChunk, kSfChunk, &full[stage]);
            bulk_load(sfs + kSfChunk, P.sfb + (tl.b_row / kF8BN * kgroups + kb / 4) * kSfChunk, kSfChunk,
                      &full[stage]);
          }
          if (++stage == kF8Stages) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      int stage = 0, hint = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      uint32_t slot = 1;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        F8Tile tl;
        if (!f8_locate<EPI, TABLE>(P, t, hint, tl)) continue;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, P.err, kErrTimeoutAccum)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kF8BN;
        const int kblocks = tl.k / kF8BK;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, P.err, kErrTimeoutFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * kF8StageBytes);
          const uint32_t sb = sa + kF8ABytes;
          if ((kb & 3) == 0) {
            // a new group of four K blocks: its scales go to the other tensor-memory slot (the
            // MMAs still reading the previous slot were issued earlier and execute in order)
            slot ^= 1u;
            const uint32_t sfs = smem_u32(smem + kF8SfOffset + stage * 2 * kSfChunk);
            const uint32_t t_sf = tmem_base + kF8SfTmemCol + 8 * slot;
            // no-swizzle K-major core matrices of 8 rows x 16 bytes, 128 bytes apart
            tmem_cp_sf(t_sf, make_smem_desc(sfs, 128, 128, 0));
            tmem_cp_sf(t_sf + 4, make_smem_desc(sfs + kSfChunk, 128, 128, 0));
          }
          // scale-factor byte j of each word: in the descriptor ids and the address's top bits
          const uint32_t j = static_cast<uint32_t>(kb & 3);
          const uint32_t idesc = kIdesc | (j << 29) | (j << 4);
          const uint32_t t_sfa = (tmem_base + kF8SfTmemCol + 8 * slot) | (j << 30);
          const uint32_t t_sfb = (tmem_base + kF8SfTmemCol + 8 * slot + 4) | (j << 30);
#pragma unroll
          for (int kk = 0; kk < kF8BK / 32; ++kk) {
            const uint64_t da = make_smem_desc(sa + kk * 32, 16, 1024, 2);
            const uint64_t db = make_smem_desc(sb + kk * 32, 16, 1024, 2);
            mma_mxf8(d_tmem, da, db, idesc, t_sfa, t_sfb, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == kF8Stages) { stage = 0; phase ^= 1; }
        }
        mma_commit(&acc_full[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    }
  } else {
    const int quarter = warp & 3;
    uint8_t* stg = smem + kF8EpiOffset + quarter * kEpiStageBytes;
    int acc = 0, hint = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      F8Tile tl;
      if (!f8_locate<EPI, TABLE>(P, t, hint, tl)) continue;
      if (!mbar_wait(&acc_full[acc], acc_phase, P.err, kErrTimeoutAccum)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + acc * kF8BN + (static_cast<uint32_t>(quarter * 32) << 16);
      const int drow = tl.d_row + quarter * 32;
      const bool issue = tl.store && (TABLE || drow < P.m);
      if constexpr (EPI == kF8EpiSwiGLU) {
        // columns [0, 64): gate, [64, 128): up  ->  act, and the pre-activations for backward
        float g[64], u[64];
#pragma unroll
        for (int h = 0; h < 64; h += 32) {
          uint32_t r[32];
          tmem_ld32(t_row + h, r);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 32; ++q) g[h + q] = __uint_as_float(r[q]);
          tmem_ld32(t_row + 64 + h, r);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 32; ++q) u[h + q] = __uint_as_float(r[q]);
        }
        const float gmax = P.gate_max, lo = P.lin_lo, hi = P.lin_hi;
        const int arow = tl.aux_row + quarter * 32;
        f8_store(stg, lane, [&](int q) {
          float a8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            a8[e] = silu_f(fminf(g[8 * q + e], gmax)) * fminf(fmaxf(u[8 * q + e], lo), hi);
          return pack_bf16x8(a8);
        }, &map_d, tl.d_col, drow, issue);
        if (P.write_pre) {
          f8_store(stg, lane, [&](int q) { return pack_bf16x8(g + 8 * q); }, &map_aux, tl.d_col, arow, issue);
          f8_store(stg, lane, [&](int q) { return pack_bf16x8(u + 8 * q); }, &map_aux, tl.n + tl.d_col, arow, issue);
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < kF8BN; c += 64) {
          float v[64];
#pragma unroll
          for (int h = 0; h < 64; h += 32) {
            uint32_t r[32];
            tmem_ld32(t_row + c + h, r);
            tmem_ld_wait();
#pragma unroll
            for (int q = 0; q < 32; ++q) v[h + q] = __uint_as_float(r[q]);
          }
          f8_store(stg, lane, [&](int q) { return pack_bf16x8(v + 8 * q); }, &map_d, tl.d_col + c, drow, issue);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    if (lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kF8TmemCols);
  }
}

int sm_count(int dev) {
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

void check_fp8_operand(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.dim() == 2 && t.element_size() == 1, name, ": 2-D one-byte CUDA tensor required");
  TORCH_CHECK(t.stride(1) == 1 && t.stride(0) % 16 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              name, ": rows must be contiguous, 16-byte aligned");
}

}  // namespace

// x (M, K) bf16 -> q (M, K) e4m3 bytes, sf (ceil(M/128) * K/128 * 512) bytes, scale (M, K/128) fp32.
void fp8_quant_rows(torch::Tensor x, torch::Tensor q, torch::Tensor sf, c10::optional<torch::Tensor> scale) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "x: 2-D bf16, unit inner stride");
  const int64_t M = x.size(0), K = x.size(1);
  TORCH_CHECK(K % 128 == 0, "K must be a multiple of 128");
  TORCH_CHECK(x.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "x rows 16-byte aligned");
  check_fp8_operand(q, "q");
  TORCH_CHECK(q.size(0) == M && q.size(1) == K, "q shape");
  const int64_t Mpad = (M + 127) / 128 * 128;
  TORCH_CHECK(sf.numel() >= Mpad / 128 * sf_groups(K) * kSfChunk && sf.element_size() == 1, "sf size");
  float* sp = nullptr;
  if (scale.has_value()) {
    TORCH_CHECK(scale->scalar_type() == at::kFloat && scale->is_contiguous() && scale->numel() == M * (K / 128),
                "scale (M, K/128) fp32");
    sp = scale->data_ptr<float>();
  }
  if (M == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t groups = Mpad * (K / 128);
  quant_rows_kernel<<<static_cast<unsigned>((groups + 15) / 16), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), static_cast<int>(M), static_cast<int>(Mpad),
      static_cast<int>(K), reinterpret_cast<uint8_t*>(q.data_ptr()), q.stride(0),
      reinterpret_cast<uint8_t*>(sf.data_ptr()), sp, nullptr, 0, nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// MoE gather fused into the 1 x 128 quantisation: q[r] = quant(h[row_token[r]]) (zero rows
// for -1), sf in the GEMM's scale-factor layout.  h (T, K) bf16; q (M, K) bytes.
void fp8_gather_quant_rows(torch::Tensor h, torch::Tensor row_token, torch::Tensor q, torch::Tensor sf,
                           torch::Tensor err) {
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && h.dim() == 2 && h.stride(1) == 1, "h: 2-D bf16, unit inner stride");
  const int64_t K = h.size(1), M = q.size(0);
  TORCH_CHECK(K % 128 == 0 && h.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(h.data_ptr()) % 16 == 0,
              "h rows: K % 128 == 0, 16-byte aligned");
  check_fp8_operand(q, "q");
  TORCH_CHECK(q.size(1) == K && row_token.scalar_type() == at::kInt && row_token.numel() >= M, "q / row_token");
  const int64_t Mpad = (M + 127) / 128 * 128;
  TORCH_CHECK(sf.numel() >= Mpad / 128 * sf_groups(K) * kSfChunk && sf.element_size() == 1, "sf size");
  if (M == 0) return;
  c10::cuda::CUDAGuard guard(h.device());
  const int64_t groups = Mpad * (K / 128);
  quant_rows_kernel<<<static_cast<unsigned>((groups + 15) / 16), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()), h.stride(0), static_cast<int>(M), static_cast<int>(Mpad),
      static_cast<int>(K), reinterpret_cast<uint8_t*>(q.data_ptr()), q.stride(0),
      reinterpret_cast<uint8_t*>(sf.data_ptr()), nullptr, row_token.data_ptr<int>(), static_cast<int>(h.size(0)),
      err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// w (N, K) bf16 -> q (N, K) e4m3 bytes, sf (N/128 * K/128 * 512) bytes, scale (N/128, K/128) fp32.
void fp8_quant_blocks(torch::Tensor w, torch::Tensor q, torch::Tensor sf, c10::optional<torch::Tensor> scale) {
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.dim() == 2 && w.stride(1) == 1, "w: 2-D bf16, unit inner stride");
  const int64_t N = w.size(0), K = w.size(1);
  TORCH_CHECK(N % 128 == 0 && K % 128 == 0, "N and K must be multiples of 128");
  TORCH_CHECK(w.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0, "w rows 16-byte aligned");
  check_fp8_operand(q, "q");
  TORCH_CHECK(q.size(0) == N && q.size(1) == K, "q shape");
  TORCH_CHECK(sf.numel() >= N / 128 * sf_groups(K) * kSfChunk && sf.element_size() == 1, "sf size");
  float* sp = nullptr;
  if (scale.has_value()) {
    TORCH_CHECK(scale->scalar_type() == at::kFloat && scale->is_contiguous() &&
                    scale->numel() == (N / 128) * (K / 128), "scale (N/128, K/128) fp32");
    sp = scale->data_ptr<float>();
  }
  if (N == 0) return;
  c10::cuda::CUDAGuard guard(w.device());
  const dim3 grid(static_cast<unsigned>(K / 128), static_cast<unsigned>(N / 128));
  quant_blocks_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), nullptr, 0, w.stride(0), static_cast<int>(K),
      reinterpret_cast<uint8_t*>(q.data_ptr()), q.stride(0), reinterpret_cast<uint8_t*>(sf.data_ptr()), sp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// SwiGLU expert pool gate / up weights (each (E, I, K) bf16, contiguous) -> q (E * 2I, K) in
// the interleaved 64-row group layout of the FP8 SwiGLU epilogue, 128 x 128 block scales.
void fp8_quant_blocks_gu(torch::Tensor wg, torch::Tensor wu, torch::Tensor q, torch::Tensor sf) {
  TORCH_CHECK(wg.scalar_type() == at::kBFloat16 && wu.scalar_type() == at::kBFloat16 && wg.is_contiguous() &&
                  wu.is_contiguous() && wg.sizes() == wu.sizes() && wg.dim() == 3, "wg / wu: (E, I, K) bf16");
  const int64_t E = wg.size(0), I = wg.size(1), K = wg.size(2);
  TORCH_CHECK(I % 64 == 0 && K % 128 == 0, "I % 64 == 0 and K % 128 == 0");
  check_fp8_operand(q, "q");
  TORCH_CHECK(q.size(0) == E * 2 * I && q.size(1) == K, "q shape (E * 2I, K)");
  const int64_t N = E * 2 * I;
  TORCH_CHECK(sf.numel() >= N / 128 * sf_groups(K) * kSfChunk && sf.element_size() == 1, "sf size");
  if (N == 0) return;
  c10::cuda::CUDAGuard guard(wg.device());
  const dim3 grid(static_cast<unsigned>(K / 128), static_cast<unsigned>(N / 128));
  quant_blocks_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(wg.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(wu.data_ptr()),
      static_cast<int>(I), K, static_cast<int>(K), reinterpret_cast<uint8_t*>(q.data_ptr()), q.stride(0),
      reinterpret_cast<uint8_t*>(sf.data_ptr()), nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out (M, N) bf16 = block-scaled a (M, K) x b (N, K)^T.
void gemm_fp8(torch::Tensor a, torch::Tensor sfa, torch::Tensor b, torch::Tensor sfb, torch::Tensor out,
              torch::Tensor err) {
  check_fp8_operand(a, "a");
  check_fp8_operand(b, "b");
  const int64_t M = a.size(0), K = a.size(1), N = b.size(0);
  TORCH_CHECK(b.size(1) == K, "K mismatch");
  TORCH_CHECK(K % 128 == 0 && K > 0 && N % 128 == 0, "K and N must be multiples of 128");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.dim() == 2 && out.size(0) == M && out.size(1) == N &&
                  out.stride(1) == 1 && (out.stride(0) * 2) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
              "out: (M, N) bf16, 16-byte aligned rows");
  const int64_t mt = (M + 127) / 128;
  TORCH_CHECK(sfa.numel() >= mt * sf_groups(K) * kSfChunk && sfb.numel() >= N / 128 * sf_groups(K) * kSfChunk,
              "scale-factor buffers too small");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(sfa.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(sfb.data_ptr()) % 16 == 0, "scale-factor buffers 16-byte aligned");
  if (M == 0) return;
  c10::cuda::CUDAGuard guard(a.device());
  const CUtensorMap ma = make_map_3d(a.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, 1, a.stride(0),
                                     a.stride(0) * M, kF8BK, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap mb = make_map_3d(b.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, 1, b.stride(0),
                                     b.stride(0) * N, kF8BK, kF8BN, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap md = make_map_3d(out.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, 1, out.stride(0) * 2,
                                     out.stride(0) * 2 * M, 64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  F8Params p{};
  p.m = static_cast<int>(M);
  p.n = static_cast<int>(N);
  p.k = static_cast<int>(K);
  p.tiles_n = static_cast<int>(N / kF8BN);
  p.total = static_cast<int>(mt * p.tiles_n);
  p.sfa = reinterpret_cast<const uint8_t*>(sfa.data_ptr());
  p.sfb = reinterpret_cast<const uint8_t*>(sfb.data_ptr());
  p.err = err.data_ptr<int>();
  const int grid = std::min(p.total, sm_count(a.get_device()));
  auto kern = gemm_mxf8_kernel<kF8EpiBF16, false>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kF8SmemTotal);
  kern<<<grid, 192, kF8SmemTotal, at::cuda::getCurrentCUDAStream()>>>(ma, mb, md, md, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Grouped (MoE) block-scaled FP8 GEMM over a device problem table (build_moe_problems modes
// 6 / 7).  a: (rows, K) quantised rows, expert segments 128-aligned; b: (E * b_rows, K)
// quantised expert weights stacked along rows.
//   mode 0: out = act (rows, I) = SwiGLU of the tile's gate | up halves, pre (rows, 2 I) = gate | up;
//           b rows of expert e: 64-row groups alternating gate and up (b_rows = 2 I)
//   mode 1: out (rows, N) = a b_e^T (b_rows = N)
void grouped_gemm_fp8(int64_t mode, torch::Tensor a, torch::Tensor sfa, torch::Tensor b, torch::Tensor sfb,
                      torch::Tensor out, c10::optional<torch::Tensor> pre, torch::Tensor probs, torch::Tensor total,
                      int64_t n_probs, int64_t b_rows, double gmax, double lo, double hi, torch::Tensor err) {
  check_fp8_operand(a, "a");
  check_fp8_operand(b, "b");
  const int64_t M = a.size(0), K = a.size(1);
  TORCH_CHECK(b.size(1) == K && K % 128 == 0 && K > 0, "K mismatch or K % 128");
  TORCH_CHECK(b_rows % 128 == 0 && b.size(0) % b_rows == 0, "b_rows must be a multiple of 128 dividing b's rows");
  TORCH_CHECK(sfa.numel() >= (M + 127) / 128 * sf_groups(K) * kSfChunk &&
                  sfb.numel() >= b.size(0) / 128 * sf_groups(K) * kSfChunk, "scale-factor buffers too small");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.size(0) == M, "out: (rows, N) bf16");
  c10::cuda::CUDAGuard guard(a.device());
  const CUtensorMap ma = make_map_3d(a.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, 1, a.stride(0),
                                     a.stride(0) * M, kF8BK, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap mb = make_map_3d(b.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, b.size(0), 1, b.stride(0),
                                     b.stride(0) * b.size(0), kF8BK, kF8BN, CU_TENSOR_MAP_SWIZZLE_128B);
  const int64_t N = out.size(1);
  TORCH_CHECK((N * 2) % 16 == 0, "output rows must be 16-byte multiples");
  const CUtensorMap md = make_map_3d(out.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, 1, N * 2, N * 2 * M,
                                     64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap mx = md;
  if (mode == 0) {
    TORCH_CHECK(b_rows == 2 * N && N % 64 == 0, "SwiGLU: b_rows = 2 I, I % 64 == 0");
    if (pre.has_value()) {
      TORCH_CHECK(pre->scalar_type() == at::kBFloat16 && pre->is_contiguous() && pre->size(0) == M &&
                      pre->size(1) == 2 * N, "pre: (rows, 2 I) bf16");
      mx = make_map_3d(pre->data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 2 * N, M, 1, 4 * N, 4 * N * M, 64, 32,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    }
  } else {
    TORCH_CHECK(mode == 1 && b_rows == N, "mode 1: b_rows = N");
  }
  F8Params p{};
  p.probs = reinterpret_cast<const GemmProblem*>(probs.data_ptr());
  p.total_tiles = total.data_ptr<int>();
  p.n_probs = static_cast<int>(n_probs);
  p.b_rows = static_cast<int>(b_rows);
  p.write_pre = pre.has_value() ? 1 : 0;
  p.gate_max = static_cast<float>(gmax);
  p.lin_lo = static_cast<float>(lo);
  p.lin_hi = static_cast<float>(hi);
  p.sfa = reinterpret_cast<const uint8_t*>(sfa.data_ptr());
  p.sfb = reinterpret_cast<const uint8_t*>(sfb.data_ptr());
  p.err = err.data_ptr<int>();
  if (M == 0 || n_probs == 0) return;
  const int grid = sm_count(a.get_device());
  auto kern = mode == 0 ? gemm_mxf8_kernel<kF8EpiSwiGLU, true> : gemm_mxf8_kernel<kF8EpiBF16, true>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kF8SmemTotal);
  kern<<<grid, 192, kF8SmemTotal, at::cuda::getCurrentCUDAStream()>>>(ma, mb, md, mx, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ---------------------------------------------------------------- MXFP4 fake quantisation (QAT)
// The reference's MX FP4 straight-through quantiser (kernels/quant/fp4.py) over blocks of 32
// along the last axis, one warp per block: scale = 2^ceil(log2(max(amax / 6, 2^-126))) (an
// E8M0 value), each element rounded to the nearest E2M1 magnitude {0, .5, 1, 1.5, 2, 3, 4, 6}
// of |x| / scale clamped to 6 (an exact tie goes to the smaller magnitude), times the scale and
// the sign; the output is x + (q - x) evaluated in x's dtype, as the PyTorch expression does.
namespace {
__device__ __forceinline__ float e2m1_round(float mag) {
  const float lv[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  float best = lv[0], bd = fabsf(mag - lv[0]);
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    const float d = fabsf(mag - lv[i]);
    if (d < bd) { bd = d; best = lv[i]; }
  }
  return best;
}

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16(v); }

template <typename T>
__global__ void fake_quant_fp4_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t n_blocks) {
  const int64_t blk = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (blk >= n_blocks) return;
  const T xv = x[blk * 32 + lane];
  const float v = to_f<T>(xv);
  float amax = fabsf(v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float raw = fmaxf(amax / 6.0f, 1.17549435e-38f);
  const float scale = exp2f(ceilf(log2f(raw)));
  const float q = copysignf(e2m1_round(fminf(fabsf(v / scale), 6.0f)), v) * scale;
  const T qd = from_f<T>(q);
  const T diff = from_f<T>(to_f<T>(qd) - v);
  out[blk * 32 + lane] = from_f<T>(v + to_f<T>(diff));
}
}  // namespace

void fake_quant_fp4(torch::Tensor x, torch::Tensor out) {
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous() && x.sizes() == out.sizes() &&
                  x.scalar_type() == out.scalar_type(), "fake_quant_fp4: contiguous, same shape / dtype");
  TORCH_CHECK(x.size(-1) % 32 == 0, "last dimension must be a multiple of 32");
  const int64_t n_blocks = x.numel() / 32;
  if (n_blocks == 0) return;
  c10::cuda::CUDAGuard guard(x.device());
  const unsigned grid = static_cast<unsigned>((n_blocks * 32 + 255) / 256);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == at::kFloat) {
    fake_quant_fp4_kernel<float><<<grid, 256, 0, stream>>>(x.data_ptr<float>(), out.data_ptr<float>(), n_blocks);
  } else {
    TORCH_CHECK(x.scalar_type() == at::kBFloat16, "fake_quant_fp4: fp32 or bf16");
    fake_quant_fp4_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
        n_blocks);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t fp8_sf_bytes(int64_t rows, int64_t k) { return (rows + 127) / 128 * sf_groups(k) * kSfChunk; }

}  // namespace sv4
