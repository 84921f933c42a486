// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   D[m, n] = sum_k A[m, k] * B[n, k]        (fp32 accumulation in TMEM)
//
// One CTA per SM loops over output tiles of 128 x BN.  Roles (6 warps):
//   warp 0      : TMA producer -- one elected lane streams A/B k-blocks into a
//                 kStages-deep shared-memory ring (128B swizzle).
//   warp 1      : MMA issuer   -- one elected lane issues tcgen05.mma (M=128, N=BN,
//                 K=16 per instruction) into one of two TMEM accumulators, then
//                 tcgen05.commit releases the smem stage / publishes the accumulator.
//   warps 2..5  : epilogue     -- tcgen05.ld the accumulator (each warp owns its
//                 32-lane TMEM quarter), apply the fused epilogue, store to global.
// Two TMEM accumulators (2 x BN columns) let the epilogue of tile i overlap the
// MMAs of tile i+1.
//
// Work is described by GemmProblem records: a single problem (optionally repeated
// over a batch dimension, used by the batched Newton-Schulz GEMMs) or a device-side
// table (MoE grouped GEMMs, filled on the GPU from the routing counts, so no host
// sync).  A and B are read through 3-D TMA tensor maps (dims: inner, outer, batch)
// that may be K-major or MN-major; the B operand can be split across two tensor
// maps along N (fused SwiGLU gate|up) or along K (dgrad through [W_gate; W_up]).
#pragma once
#include "common.cuh"

namespace sv4 {

struct GemmProblem {
  int m, n, k;            // logical problem size (k % 64 == 0)
  int a_m, a_k, a_b;      // A tensor-map coordinates of element (0, 0) and batch index
  int b_n, b_k, b_b;      // B tensor-map coordinates of element (0, 0) and batch index
  int tile_begin;         // first global tile id of this problem (table mode)
  int batch;              // single mode: number of repeats along the batch dims
  long long d_off;        // element offset of D(0, 0)
  long long d_ld;         // row stride of D in elements
  long long d_bstride;    // single mode: D offset between batch repeats
  long long aux_off;      // SwiGLU: element offset of the pre-activation rows; rowscale: row index base
  long long aux_ld;       // SwiGLU: row stride of the pre-activation buffer
};

enum BMode : int { kBSingle = 0, kBSplitN = 1, kBSplitK = 2 };
// kEpiAxpbyBF16: D = alpha * acc + beta * C with C (bf16) laid out exactly like D (pointer `aux`).
// kEpiPeerBF16: D (bf16) as kEpiBF16, and the same tile values stored into every peer's receive
// slot (`peer_d`, D's layout, peer memory over NVLink) as the tile is written; when all of a CTA's
// tiles are out, one thread adds 1 to every peer's arrival counter (`peer_cnt`, release at system
// scope after a system fence), so a peer's consumer waits for gridDim.x arrivals per source.
enum Epi : int {
  kEpiBF16 = 0, kEpiF32 = 1, kEpiF32Acc = 2, kEpiSwiGLU = 3, kEpiRowScaleBF16 = 4, kEpiAxpbyBF16 = 5, kEpiPeerBF16 = 6
};
constexpr int kGemmMaxPeers = 7;

struct GemmParams {
  const GemmProblem* probs;   // device table or nullptr (single mode)
  const int* total_tiles;     // device scalar (table mode)
  int n_probs;
  GemmProblem single;
  void* d;
  void* aux;                  // SwiGLU pre-activations (bf16)
  const float* rowscale;      // kEpiRowScaleBF16
  float alpha, beta;
  float gate_max, lin_lo, lin_hi;
  int ksplit;                 // kBSplitK: K index where B switches from map 0 to map 1
  int tma_d;                  // 1: D is written through map_d (TMA store / reduce-add) where possible
  int splitk;                 // single mode: > 1 splits K into `splitk` slices of `kc` (reduce-add into D)
  int kc;
  int sym;                    // single mode: D is symmetric; tiles strictly below the diagonal are skipped
  int* err;
  int n_peers;                // kEpiPeerBF16
  unsigned long long peer_d[kGemmMaxPeers];
  unsigned long long peer_cnt[kGemmMaxPeers];
};

constexpr int kBM = 128;
constexpr int kBK = 64;  // bf16: 64 elements = 128 bytes = one swizzle row

// Epilogue staging: two 32-row x 128-byte buffers per epilogue warp (128B-swizzled, the
// layout of a D tensor-map box), written by the warp and drained by TMA stores/reduces;
// the warp fills one buffer while the previous store still reads the other.
constexpr int kEpiStageBytes = 32 * 128;
constexpr int kEpiBufs = 2;

template <int BN>
struct GemmSmem {
  static constexpr int kStages = BN >= 256 ? 4 : 6;
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiOffset = kStages * kStageBytes;          // 1024-aligned
  static constexpr int kBarOffset = kEpiOffset + 4 * kEpiBufs * kEpiStageBytes;
  static constexpr int kTotal = kBarOffset + 256 + 1024;  // + barriers + alignment slack
};

// Write this warp's 32 rows x 128 B (row = lane) into the next staging buffer, 128B-swizzled,
// then (lane 0, if `issue`) store or reduce-add it to `map` at (c0, c1, c2).  `pack(q)` returns
// the q-th 16-byte chunk of the calling lane's row.
template <typename Pack>
__device__ __forceinline__ void stage_store(uint8_t* stg_warp, int& buf, int lane, Pack pack, const CUtensorMap* map,
                                            bool reduce, int c0, int c1, int c2, bool issue) {
  uint8_t* b = stg_warp + buf * kEpiStageBytes;
  if (lane == 0) bulk_wait_read<kEpiBufs - 1>();  // the store that last used this buffer has read it
  __syncwarp();
  uint8_t* myrow = b + lane * 128;
#pragma unroll
  for (int q = 0; q < 8; ++q) *reinterpret_cast<uint4*>(myrow + ((q ^ (lane & 7)) << 4)) = pack(q);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0 && issue) {
    if (reduce) tma_reduce_add_3d(map, b, c0, c1, c2);
    else tma_store_3d(map, b, c0, c1, c2);
    bulk_commit_group();
  }
  // Only a buffer that a committed store reads moves the rotation: with an un-issued chunk the
  // next write may reuse this buffer, and wait_read<kEpiBufs - 1> keeps its meaning.
  if (issue) buf = (buf + 1) % kEpiBufs;
}

__device__ __forceinline__ uint4 pack_bf16x8(const float* v) {
  __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]);
  __nv_bfloat162 h1 = __floats2bfloat162_rn(v[2], v[3]);
  __nv_bfloat162 h2 = __floats2bfloat162_rn(v[4], v[5]);
  __nv_bfloat162 h3 = __floats2bfloat162_rn(v[6], v[7]);
  return make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                    *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
}

// kEpiPeerBF16: copy one staged 32-row x 64-column bf16 chunk (128B-swizzled, as stage_store
// wrote it) to every peer's slot.  Eight lanes per row, so each store instruction writes four
// whole 128-byte row segments (coalesced NVLink writes).  `off0`: element offset of the chunk's
// first row and column in D's layout; rows past `rows` / columns past `cols` are not written.
__device__ __forceinline__ void push_chunk_to_peers(const GemmParams& P, const uint8_t* b, int lane, long long off0,
                                                    long long ld, int rows, int cols) {
  const int q = lane & 7;
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int r = it * 4 + (lane >> 3);
    if (r >= rows || q * 8 >= cols) continue;
    const uint4 v = *reinterpret_cast<const uint4*>(b + r * 128 + ((q ^ (r & 7)) << 4));
    const long long off = off0 + r * ld + q * 8;
    for (int p = 0; p < P.n_peers; ++p) {
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(P.peer_d[p]) + off;
      if (q * 8 + 8 <= cols) {
        *reinterpret_cast<uint4*>(dst) = v;
      } else {
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
        for (int j = 0; j < cols - q * 8; ++j) dst[j] = e[j];
      }
    }
  }
}

// Symmetric outputs (P.sym): tiles entirely below the diagonal are skipped, and the tiles that
// are computed write the transposes of their values into those skipped tiles, so no separate
// mirror pass is needed.  For this lane's row r, the target (c, r) lies in a skipped tile exactly
// when c >= c_min = (floor(((r / BN) * BN + BN - 1) / 128) + 1) * 128 (tile (c / 128, r / BN)
// has all its columns left of its first row); those c are strictly above the diagonal.  Lanes
// hold consecutive rows, so each store instruction writes 32 consecutive elements of row c.
template <int BN, int W, bool F32>
__device__ __forceinline__ void sym_store_transposed(const GemmParams& P, const GemmProblem& pr, int bt, int row,
                                                     int col0, const float* v) {
  if (row >= pr.m) return;
  const int c_min = (((row / BN) * BN + BN - 1) / kBM + 1) * kBM;
  if (col0 + W <= c_min) return;
  const long long base = pr.d_off + static_cast<long long>(bt) * pr.d_bstride + row;
#pragma unroll
  for (int j = 0; j < W; ++j) {
    const int c = col0 + j;
    if (c >= c_min && c < pr.n) {
      if constexpr (F32) reinterpret_cast<float*>(P.d)[base + static_cast<long long>(c) * pr.d_ld] = v[j];
      else reinterpret_cast<__nv_bfloat16*>(P.d)[base + static_cast<long long>(c) * pr.d_ld] = __float2bfloat16(v[j]);
    }
  }
}

__device__ __forceinline__ void red_release_sys_add(unsigned long long addr, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ int tiles_m(const GemmProblem& p) { return (p.m + kBM - 1) / kBM; }

template <int BN, int BMODE>
__device__ __forceinline__ int tiles_n(const GemmProblem& p) {
  constexpr int kOutN = BMODE == kBSplitN ? BN / 2 : BN;
  return (p.n + kOutN - 1) / kOutN;
}

// Map a global tile id to (problem, m-tile, n-tile, batch).  `hint` carries the last
// problem index (tile ids only increase per CTA, so the scan is amortised O(1)).
template <int BN, int BMODE>
__device__ __forceinline__ bool locate_tile(const GemmParams& P, int t, int& hint, GemmProblem& pr, int& mt,
                                            int& nt, int& bt) {
  if (P.probs == nullptr) {
    pr = P.single;
    const int per = tiles_m(pr) * tiles_n<BN, BMODE>(pr);
    if (per == 0) return false;
    bt = t / per;  // batch index, or K-slice index when split-K is on
    if (bt >= (P.splitk > 1 ? P.splitk : pr.batch)) return false;
    const int local = t - bt * per;
    mt = local / tiles_n<BN, BMODE>(pr);
    nt = local % tiles_n<BN, BMODE>(pr);
    // symmetric output: a tile whose every column is left of its first row is skipped (the
    // epilogue of its transpose tile fills it)
    return !(P.sym && nt * BN + BN - 1 < mt * kBM);
  }
  while (hint + 1 < P.n_probs && P.probs[hint + 1].tile_begin <= t) ++hint;
  pr = P.probs[hint];
  const int tn = tiles_n<BN, BMODE>(pr);
  const int local = t - pr.tile_begin;
  if (local < 0 || tn == 0 || local >= tiles_m(pr) * tn) return false;
  mt = local / tn;
  nt = local % tn;
  bt = 0;
  return true;
}

template <int BN, bool A_MN, bool B_MN, int BMODE, int EPI>
__global__ void __launch_bounds__(192, 1)
gemm_bf16_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b0,
                 const __grid_constant__ CUtensorMap map_b1, const __grid_constant__ CUtensorMap map_d,
                 const __grid_constant__ CUtensorMap map_aux, const GemmParams P) {
  using S = GemmSmem<BN>;
  constexpr int kStages = S::kStages;
  constexpr uint32_t kIdesc = make_idesc_f16(kBM, BN, 1, 1, A_MN, B_MN);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOffset);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
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
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b0);
    if (BMODE != kBSingle) tma_prefetch_desc(&map_b1);
    if (P.tma_d) tma_prefetch_desc(&map_d);
    if (P.tma_d && EPI == kEpiSwiGLU) tma_prefetch_desc(&map_aux);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total = P.probs == nullptr
                        ? (P.splitk > 1 ? P.splitk : P.single.batch) * tiles_m(P.single) * tiles_n<BN, BMODE>(P.single)
                        : *P.total_tiles;
  const bool split = P.probs == nullptr && P.splitk > 1;

  if (warp == 0) {
    // ------------------------------------------------------------- TMA producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int hint = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        GemmProblem pr;
        int mt, nt, bt;
        if (!locate_tile<BN, BMODE>(P, t, hint, pr, mt, nt, bt)) continue;
        const int k_begin = split ? bt * P.kc : 0;
        const int nk = (split ? min(P.kc, pr.k - k_begin) : pr.k) / kBK;
        const int ab = pr.a_b + (split ? 0 : bt), bb = pr.b_b + (split ? 0 : bt);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, P.err, kErrTimeoutEmpty)) { ok = false; break; }
          uint8_t* sa = smem + stage * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
          const int ka = pr.a_k + k_begin + kb * kBK;
          const int m0 = pr.a_m + mt * kBM;
          if (!A_MN) {
            tma_load_3d(sa, &map_a, &full[stage], ka, m0, ab);
          } else {
            tma_load_3d(sa, &map_a, &full[stage], m0, ka, ab);
            tma_load_3d(sa + kBM / 2 * kBK * 2, &map_a, &full[stage], m0 + 64, ka, ab);
          }
          int kbk = pr.b_k + k_begin + kb * kBK;
          const CUtensorMap* mb = &map_b0;
          if (BMODE == kBSplitK && kbk >= P.ksplit) { mb = &map_b1; kbk -= P.ksplit; }
          if (BMODE == kBSplitN) {
            const int n0 = pr.b_n + nt * (BN / 2);
            if (!B_MN) {
              tma_load_3d(sb, &map_b0, &full[stage], kbk, n0, bb);
              tma_load_3d(sb + (BN / 2) * kBK * 2, &map_b1, &full[stage], kbk, n0, bb);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 128; ++j) {
                tma_load_3d(sb + j * 64 * kBK * 2, &map_b0, &full[stage], n0 + j * 64, kbk, bb);
                tma_load_3d(sb + (BN / 128 + j) * 64 * kBK * 2, &map_b1, &full[stage], n0 + j * 64, kbk, bb);
              }
            }
          } else {
            const int n0 = pr.b_n + nt * BN;
            if (!B_MN) {
              tma_load_3d(sb, mb, &full[stage], kbk, n0, bb);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j)
                tma_load_3d(sb + j * 64 * kBK * 2, mb, &full[stage], n0 + j * 64, kbk, bb);
            }
          }
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------------------------- MMA issuer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      int hint = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        GemmProblem pr;
        int mt, nt, bt;
        if (!locate_tile<BN, BMODE>(P, t, hint, pr, mt, nt, bt)) continue;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, P.err, kErrTimeoutAccum)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        const int nk = (split ? min(P.kc, pr.k - bt * P.kc) : pr.k) / kBK;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[stage], phase, P.err, kErrTimeoutFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * S::kStageBytes);
          const uint32_t sb = sa + S::kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            // K-major: advance 16 elements (32 B) inside the swizzle row.
            // MN-major: advance 16 K-rows (2 x 1024 B atoms); 64-wide MN blocks are 8 KB apart.
            const uint64_t da = A_MN ? make_smem_desc(sa + kk * 2048, kBK * 128, 1024, 2)
                                     : make_smem_desc(sa + kk * 32, 16, 1024, 2);
            const uint64_t db = B_MN ? make_smem_desc(sb + kk * 2048, kBK * 128, 1024, 2)
                                     : make_smem_desc(sb + kk * 32, 16, 1024, 2);
            mma_bf16(d_tmem, da, db, kIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
        mma_commit(&acc_full[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32)
    uint8_t* stg = smem + S::kEpiOffset + quarter * kEpiBufs * kEpiStageBytes;
    int sbuf = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    int hint = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      GemmProblem pr;
      int mt, nt, bt;
      if (!locate_tile<BN, BMODE>(P, t, hint, pr, mt, nt, bt)) continue;
      if (!mbar_wait(&acc_full[acc], acc_phase, P.err, kErrTimeoutAccum)) break;
      tc_fence_after();
      const int row = mt * kBM + quarter * 32 + lane;
      const bool row_ok = row < pr.m;
      const bool zero_k = pr.k == 0;
      const uint32_t t_row = tmem_base + acc * BN + (static_cast<uint32_t>(quarter * 32) << 16);
      if (split) bt = 0;  // every K-slice reduces into the same D
      const long long dbase = pr.d_off + static_cast<long long>(bt) * pr.d_bstride + row * pr.d_ld;
      if (EPI == kEpiSwiGLU && P.tma_d && (P.probs == nullptr || mt * kBM + kBM <= pr.m)) {
        // act -> map_d, gate / up pre-activations -> map_aux columns [0, n) / [n, 2n)
        const int half = BN / 2;
        const int drow = static_cast<int>(pr.d_off / pr.d_ld) + mt * kBM + quarter * 32;
        const int arow = static_cast<int>(pr.aux_off / pr.aux_ld) + mt * kBM + quarter * 32;
        const bool rows_in = mt * kBM + quarter * 32 < pr.m;
#pragma unroll 1
        for (int c = 0; c < half; c += 64) {
          uint32_t g[64], u[64];
          tmem_ld32(t_row + c, *reinterpret_cast<uint32_t(*)[32]>(g));
          tmem_ld32(t_row + c + 32, *reinterpret_cast<uint32_t(*)[32]>(g + 32));
          tmem_ld32(t_row + half + c, *reinterpret_cast<uint32_t(*)[32]>(u));
          tmem_ld32(t_row + half + c + 32, *reinterpret_cast<uint32_t(*)[32]>(u + 32));
          tmem_ld_wait();
          if (zero_k) {
#pragma unroll
            for (int j = 0; j < 64; ++j) g[j] = u[j] = 0u;
          }
          const int col0 = nt * half + c;
          const bool issue = rows_in && col0 < pr.n;
          const float gmax = P.gate_max, lo = P.lin_lo, hi = P.lin_hi;
          stage_store(stg, sbuf, lane, [&](int q) {
            float a8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float gv = __uint_as_float(g[8 * q + e]), uv = __uint_as_float(u[8 * q + e]);
              a8[e] = silu_f(fminf(gv, gmax)) * fminf(fmaxf(uv, lo), hi);
            }
            return pack_bf16x8(a8);
          }, &map_d, false, col0, drow, 0, issue);
          stage_store(stg, sbuf, lane, [&](int q) {
            float g8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) g8[e] = __uint_as_float(g[8 * q + e]);
            return pack_bf16x8(g8);
          }, &map_aux, false, col0, arow, 0, issue);
          stage_store(stg, sbuf, lane, [&](int q) {
            float u8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) u8[e] = __uint_as_float(u[8 * q + e]);
            return pack_bf16x8(u8);
          }, &map_aux, false, pr.n + col0, arow, 0, issue);
        }
      } else if constexpr (EPI == kEpiSwiGLU) {
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(P.d);
        __nv_bfloat16* pre = reinterpret_cast<__nv_bfloat16*>(P.aux);
        const int half = BN / 2;
#pragma unroll 1
        for (int c = 0; c < half; c += 32) {
          uint32_t g[32], u[32];
          tmem_ld32(t_row + c, g);
          tmem_ld32(t_row + half + c, u);
          tmem_ld_wait();
          const int col0 = nt * half + c;
          if (row_ok) {
            const long long pbase = pr.aux_off + row * pr.aux_ld;
            float av[32], gv[32], uv[32];
#pragma unroll
            for (int q = 0; q < 32; ++q) {
              gv[q] = zero_k ? 0.f : __uint_as_float(g[q]);
              uv[q] = zero_k ? 0.f : __uint_as_float(u[q]);
              av[q] = silu_f(fminf(gv[q], P.gate_max)) * fminf(fmaxf(uv[q], P.lin_lo), P.lin_hi);
            }
            __nv_bfloat16* o_act = out + dbase + col0;
            __nv_bfloat16* o_g = pre + pbase + col0;
            __nv_bfloat16* o_u = pre + pbase + pr.n + col0;
            const bool vec = col0 + 32 <= pr.n &&
                             ((reinterpret_cast<uintptr_t>(o_act) | reinterpret_cast<uintptr_t>(o_g) |
                               reinterpret_cast<uintptr_t>(o_u)) & 15) == 0;
            if (vec) {
#pragma unroll
              for (int q = 0; q < 32; q += 8) {
                uint4 pa, pg, pu;
                uint32_t* wa = reinterpret_cast<uint32_t*>(&pa);
                uint32_t* wg = reinterpret_cast<uint32_t*>(&pg);
                uint32_t* wu = reinterpret_cast<uint32_t*>(&pu);
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                  __nv_bfloat162 ta = __floats2bfloat162_rn(av[q + 2 * h], av[q + 2 * h + 1]);
                  __nv_bfloat162 tg = __floats2bfloat162_rn(gv[q + 2 * h], gv[q + 2 * h + 1]);
                  __nv_bfloat162 tu = __floats2bfloat162_rn(uv[q + 2 * h], uv[q + 2 * h + 1]);
                  wa[h] = *reinterpret_cast<uint32_t*>(&ta);
                  wg[h] = *reinterpret_cast<uint32_t*>(&tg);
                  wu[h] = *reinterpret_cast<uint32_t*>(&tu);
                }
                *reinterpret_cast<uint4*>(o_act + q) = pa;
                *reinterpret_cast<uint4*>(o_g + q) = pg;
                *reinterpret_cast<uint4*>(o_u + q) = pu;
              }
            } else {
              for (int q = 0; q < 32; ++q) {
                if (col0 + q < pr.n) {
                  o_act[q] = __float2bfloat16(av[q]);
                  o_g[q] = __float2bfloat16(gv[q]);
                  o_u[q] = __float2bfloat16(uv[q]);
                }
              }
            }
          }
        }
      } else if (P.tma_d && (P.probs == nullptr || mt * kBM + kBM <= pr.m)) {
        // Stage 32 rows x 128 B per warp in swizzled smem, then one TMA store (or
        // reduce-add for kEpiF32Acc) per chunk.  The tensor map clips the ragged edges
        // (single mode: per batch, 3-D map); table-mode tiles are whole 128-row tiles.
        constexpr bool kF32 = (EPI == kEpiF32 || EPI == kEpiF32Acc);
        constexpr int kCW = kF32 ? 32 : 64;  // columns per 128-byte row chunk
        const float rs = (EPI == kEpiRowScaleBF16 && row_ok) ? P.rowscale[pr.aux_off + row] : 1.0f;
        const int drow = static_cast<int>(pr.d_off / pr.d_ld) + mt * kBM + quarter * 32;
#pragma unroll 1
        for (int c = 0; c < BN; c += kCW) {
          float v[kCW];
#pragma unroll
          for (int h = 0; h < kCW; h += 32) {
            uint32_t r[32];
            tmem_ld32(t_row + c + h, r);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) v[h + j] = zero_k ? 0.f : __uint_as_float(r[j]) * P.alpha * rs;
          }
          const int col0 = nt * BN + c;
          if constexpr (EPI == kEpiAxpbyBF16) {
            if (row_ok) {
              const __nv_bfloat16* cin = reinterpret_cast<const __nv_bfloat16*>(P.aux) + dbase + col0;
              if (col0 + kCW <= pr.n && (reinterpret_cast<uintptr_t>(cin) & 15) == 0) {
#pragma unroll
                for (int j = 0; j < kCW; j += 8) {  // 16-byte loads of C
                  const uint4 cv = *reinterpret_cast<const uint4*>(cin + j);
                  const __nv_bfloat162* ch = reinterpret_cast<const __nv_bfloat162*>(&cv);
#pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    const float2 f = __bfloat1622float2(ch[q]);
                    v[j + 2 * q] += P.beta * f.x;
                    v[j + 2 * q + 1] += P.beta * f.y;
                  }
                }
              } else {
                for (int j = 0; j < kCW; ++j)
                  if (col0 + j < pr.n) v[j] += P.beta * __bfloat162float(cin[j]);
              }
            }
          }
          if (P.sym) sym_store_transposed<BN, kCW, kF32>(P, pr, bt, row, col0, v);
          // Boxes starting past the problem are skipped (never issue a fully clipped store).
          const bool issue = col0 < pr.n && mt * kBM + quarter * 32 < pr.m;
          const uint8_t* staged = stg + sbuf * kEpiStageBytes;
          stage_store(stg, sbuf, lane, [&](int q) {
            if constexpr (kF32) {
              return make_uint4(__float_as_uint(v[4 * q]), __float_as_uint(v[4 * q + 1]),
                                __float_as_uint(v[4 * q + 2]), __float_as_uint(v[4 * q + 3]));
            } else {
              return pack_bf16x8(v + 8 * q);
            }
          }, &map_d, EPI == kEpiF32Acc, col0, drow, bt, issue);
          if constexpr (EPI == kEpiPeerBF16) {
            if (issue) {
              const int r0 = mt * kBM + quarter * 32;
              push_chunk_to_peers(P, staged, lane, pr.d_off + static_cast<long long>(bt) * pr.d_bstride +
                                  r0 * pr.d_ld + col0, pr.d_ld, min(32, pr.m - r0), min(kCW, pr.n - col0));
            }
          }
        }
      } else {
        const float rs = (EPI == kEpiRowScaleBF16 && row_ok) ? P.rowscale[pr.aux_off + row] : 1.0f;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld32(t_row + c, r);
          tmem_ld_wait();
          const int col0 = nt * BN + c;
          if (!row_ok) continue;
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = zero_k ? 0.f : __uint_as_float(r[j]) * P.alpha * rs;
          const bool full_chunk = col0 + 32 <= pr.n;
          const bool sym_here = P.sym != 0;
          if constexpr (EPI == kEpiAxpbyBF16) {
            const __nv_bfloat16* cin = reinterpret_cast<const __nv_bfloat16*>(P.aux) + dbase + col0;
            if (full_chunk && ((reinterpret_cast<uintptr_t>(cin) & 15) == 0)) {
#pragma unroll
              for (int j = 0; j < 32; j += 8) {
                const uint4 cv = *reinterpret_cast<const uint4*>(cin + j);
                const __nv_bfloat162* ch = reinterpret_cast<const __nv_bfloat162*>(&cv);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const float2 f = __bfloat1622float2(ch[q]);
                  v[j + 2 * q] += P.beta * f.x;
                  v[j + 2 * q + 1] += P.beta * f.y;
                }
              }
            } else {
              for (int j = 0; j < 32; ++j)
                if (col0 + j < pr.n) v[j] += P.beta * __bfloat162float(cin[j]);
            }
          }
          if (sym_here) {
            constexpr bool kF32o = (EPI == kEpiF32 || EPI == kEpiF32Acc);
            sym_store_transposed<BN, 32, kF32o>(P, pr, bt, row, col0, v);
          }
          if constexpr (EPI == kEpiPeerBF16) {  // fallback path: per-lane row stores to the peers
            for (int p = 0; p < P.n_peers; ++p) {
              __nv_bfloat16* po = reinterpret_cast<__nv_bfloat16*>(P.peer_d[p]) + dbase + col0;
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (col0 + j < pr.n) po[j] = __float2bfloat16(v[j]);
            }
          }
          if constexpr (EPI == kEpiBF16 || EPI == kEpiRowScaleBF16 || EPI == kEpiAxpbyBF16 || EPI == kEpiPeerBF16) {
            __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(P.d) + dbase + col0;
            if (full_chunk && ((reinterpret_cast<uintptr_t>(out) & 15) == 0)) {
#pragma unroll
              for (int j = 0; j < 32; j += 8) {
                uint4 pk;
                __nv_bfloat162 h0 = __floats2bfloat162_rn(v[j], v[j + 1]);
                __nv_bfloat162 h1 = __floats2bfloat162_rn(v[j + 2], v[j + 3]);
                __nv_bfloat162 h2 = __floats2bfloat162_rn(v[j + 4], v[j + 5]);
                __nv_bfloat162 h3 = __floats2bfloat162_rn(v[j + 6], v[j + 7]);
                pk.x = *reinterpret_cast<uint32_t*>(&h0);
                pk.y = *reinterpret_cast<uint32_t*>(&h1);
                pk.z = *reinterpret_cast<uint32_t*>(&h2);
                pk.w = *reinterpret_cast<uint32_t*>(&h3);
                *reinterpret_cast<uint4*>(out + j) = pk;
              }
            } else {
              for (int j = 0; j < 32; ++j)
                if (col0 + j < pr.n) out[j] = __float2bfloat16(v[j]);
            }
          } else {
            float* out = reinterpret_cast<float*>(P.d) + dbase + col0;
            if (full_chunk && ((reinterpret_cast<uintptr_t>(out) & 15) == 0)) {
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                float4 o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                if (EPI == kEpiF32Acc) {
                  const float4 prev = *reinterpret_cast<const float4*>(out + j);
                  o.x += prev.x; o.y += prev.y; o.z += prev.z; o.w += prev.w;
                }
                *reinterpret_cast<float4*>(out + j) = o;
              }
            } else {
              for (int j = 0; j < 32; ++j)
                if (col0 + j < pr.n) out[j] = (EPI == kEpiF32Acc) ? out[j] + v[j] : v[j];
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    if (lane == 0) bulk_wait_all();  // TMA stores of this warp are complete before exit
    if constexpr (EPI == kEpiPeerBF16) {
      // every epilogue thread's peer stores are ordered before the arrival (system fence,
      // then a barrier over the four epilogue warps, then one release-add per peer)
      __threadfence_system();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (warp == 2 && lane == 0)
        for (int p = 0; p < P.n_peers; ++p) red_release_sys_add(P.peer_cnt[p], 1u);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

}  // namespace sv4
