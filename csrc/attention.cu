// Fused attention of the V4 attention layers on tcgen05 (sm_100a), forward and backward.
//
// One CTA per (128-query block, head, batch row); single KV head (MQA).  Two branches
// whose softmaxes are independent and whose outputs are summed:
//   branch 0: causal sliding window of `window` keys over the layer's own K/V, an optional
//             per-head sink logit (a virtual key with value 0), optional tanh softcap, and
//             the max-|logit| telemetry used by MuonClip;
//   branch 1: the compressed table (K = V = kv, n entries): HCA (entry i visible iff block i
//             ended before the query, plus the sink) or CSA (entries picked by the indexer,
//             a bitmask per query).
// Reference math: core/attention/swa.py, hca.py:126-169, csa.py:325-375 of the reference.
//
// Layout: every 128-row operand tile lives in shared memory as 64-column, 128B-swizzled
// atoms ([atom][row][128 B]) -- the image of a TMA box.  The same tile serves as a
// K-major operand (contraction over columns) and, with LBO = one atom (16 KB), as an
// MN-major operand (contraction over rows), so backward needs no transposed copies.
// Accumulators live in TMEM; thread t of the CTA owns TMEM lane t = query (or key) row t.
// Forward is the online-softmax loop over 128-key blocks; backward recomputes P from the
// saved log-sum-exp, accumulates dQ in TMEM and reduce-adds per-block dK/dV tiles into
// fp32 buffers with TMA (cp.reduce.async.bulk .add), since all heads share K/V.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace sv4 {


CUtensorMap make_map_nd(const void* base, CUtensorMapDataType dt, int rank, const uint64_t* dims,
                        const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz);

struct AttnParams {
  int B, T, H, n;           // n: compressed entries
  int window;               // sliding-window length
  int mode;                 // 0: window only, 1: + HCA compressed branch, 2: + CSA compressed branch
  int m;                    // compression rate (block-causal bound of branch 1)
  int mask_words;           // CSA: 32-bit words per query row of `sel`
  float scale;              // 1 / sqrt(head_dim)
  float softcap;            // <= 0: none (window branch only)
  const float* sink;        // (H) or nullptr
  const uint32_t* sel;      // (B, T, mask_words)
  __nv_bfloat16* o_sw;      // (B, T, H, HD) window-branch output
  __nv_bfloat16* o_c;       // (B, T, H, HD) compressed-branch output
  __nv_bfloat16* out;       // (B, T, H, HD) o_sw + o_c
  float* lse;               // (2, B, H, T)
  float* max_logit;         // (1) max |q.k| / sqrt(d) over visible window pairs
  const __nv_bfloat16* dout;  // backward: (B, T, H, HD)
  __nv_bfloat16* dq;        // (B, T, H, HD)
  float* dsink;             // (H)
  int* err;
};

constexpr uint32_t kAtom = 16384;  // 128 rows x 128 B

__device__ __forceinline__ uint64_t desc_k(uint32_t base, int s) {  // contraction over columns
  return make_smem_desc(base + (s >> 2) * kAtom + (s & 3) * 32, 16, 1024, 2);
}
__device__ __forceinline__ uint64_t desc_mn(uint32_t base, int s) {  // contraction over rows
  return make_smem_desc(base + s * 2048, kAtom, 1024, 2);
}

// 32 fp32 values of row r, columns [c0, c0 + 32), as bf16 into a canonical tile.
// e^x as one special-function-unit instruction: 2^(x log2 e) with ex2.approx.ftz
// (flush-to-zero: results below the normal range become 0, which the bf16 P tile could
// not represent anyway).
__device__ __forceinline__ float exp_sfu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.4426950408889634f));
  return y;
}

__device__ __forceinline__ void put_row32(uint8_t* tile, int r, int c0, const float (&v)[32]) {
  uint8_t* rowp = tile + (c0 >> 6) * kAtom + r * 128;
  const int q0 = (c0 & 63) >> 3;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    __nv_bfloat162 h0 = __floats2bfloat162_rn(v[8 * q], v[8 * q + 1]);
    __nv_bfloat162 h1 = __floats2bfloat162_rn(v[8 * q + 2], v[8 * q + 3]);
    __nv_bfloat162 h2 = __floats2bfloat162_rn(v[8 * q + 4], v[8 * q + 5]);
    __nv_bfloat162 h3 = __floats2bfloat162_rn(v[8 * q + 6], v[8 * q + 7]);
    uint4 pk = make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                          *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
    *reinterpret_cast<uint4*>(rowp + (((q0 + q) ^ (r & 7)) << 4)) = pk;
  }
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    __nv_bfloat162 h0 = __floats2bfloat162_rn(v[8 * q], v[8 * q + 1]);
    __nv_bfloat162 h1 = __floats2bfloat162_rn(v[8 * q + 2], v[8 * q + 3]);
    __nv_bfloat162 h2 = __floats2bfloat162_rn(v[8 * q + 4], v[8 * q + 5]);
    __nv_bfloat162 h3 = __floats2bfloat162_rn(v[8 * q + 6], v[8 * q + 7]);
    *reinterpret_cast<uint4*>(dst + 8 * q) =
        make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                   *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
  }
}

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* src, float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 pk = *reinterpret_cast<const uint4*>(src + 8 * q);
    const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&pk);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(hp[e]);
      v[8 * q + 2 * e] = f.x;
      v[8 * q + 2 * e + 1] = f.y;
    }
  }
}

// Key-block range [lo, hi) of branch `br` for the query block starting at t0.
__device__ __forceinline__ void key_blocks(const AttnParams& P, int br, int t0, int& lo, int& hi) {
  if (br == 0) {
    const int first = t0 - P.window + 1;
    lo = first <= 0 ? 0 : first / 128;
    hi = min(t0 + 127, P.T - 1) / 128 + 1;
  } else {
    // entry i can be visible to some query of the block iff i*m + m - 1 < t0 + 127
    int imax = t0 + 127 - P.m >= 0 ? (t0 + 127 - P.m) / P.m : -1;
    imax = min(imax, P.n - 1);
    lo = 0;
    hi = imax >= 0 ? imax / 128 + 1 : 0;
  }
}

__device__ __forceinline__ bool branch_has_sink(const AttnParams& P, int br) {
  return P.sink != nullptr && (br == 0 || P.mode == 1);
}

// ====================================================================== forward
template <int HD>
__global__ void __launch_bounds__(128, 2)
attn_fwd_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mkv,
                const AttnParams P) {
  constexpr int A = HD / 64;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // P aliases the K buffer: K is dead once S = Q K^T has completed, and the next K is
  // loaded only after P V has completed.  96 KB per CTA -> two CTAs per SM (d = 128).
  constexpr int KA = A > 2 ? A : 2;
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + A * kAtom;
  uint8_t* sV = sK + KA * kAtom;
  uint8_t* sP = sK;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sV + A * kAtom);  // 0 q, 1 kv, 2 s, 3 o
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 4);
  __shared__ float red[4];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = blockIdx.x * 128, h = blockIdx.y, b = blockIdx.z;
  const int qpos = t0 + tid;
  const bool row_ok = qpos < P.T;
  const bool leader = tid == 0;
  const float scale = P.scale, softcap = P.softcap;
  const int window = P.window, mode = P.mode, cm = P.m, cn = P.n;
  if (leader) {
    for (int i = 0; i < 4; ++i) mbar_init(&bar[i], 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t tS = tbase + lane_off, tO = tbase + 128 + lane_off;
  constexpr uint32_t kIdS = make_idesc_f16(128, 128, 1, 1, false, false);
  constexpr uint32_t kIdO = make_idesc_f16(128, HD, 1, 1, false, true);

  if (leader) {
    mbar_arrive_expect_tx(&bar[0], A * kAtom);
    for (int a = 0; a < A; ++a) tma_load_4d(sQ + a * kAtom, &mq, &bar[0], a * 64, h, t0, b);
  }
  int n_kv = 0, n_s = 0, n_o = 0;
  bool q_wait = true;
  float amax = 0.f;
  const int64_t row_base = (static_cast<int64_t>(b) * P.T + qpos) * P.H + h;  // (b, qpos, h) row index

  for (int br = 0; br < 2; ++br) {
    if (br == 1 && P.mode == 0) break;
    int lo, hi;
    key_blocks(P, br, t0, lo, hi);
    const bool sink_on = branch_has_sink(P, br);
    float m_run = sink_on ? P.sink[h] : -INFINITY;
    float l_run = sink_on ? 1.f : 0.f;
    const int o_before = n_o;
    for (int kb = lo; kb < hi; ++kb) {
      if (leader) {
        if (n_o > 0) mbar_wait(&bar[3], (n_o - 1) & 1, P.err, kErrTimeoutAccum);  // V free
        if (br == 0) {
          mbar_arrive_expect_tx(&bar[1], 2 * A * kAtom);
          for (int a = 0; a < A; ++a) {
            tma_load_3d(sK + a * kAtom, &mk, &bar[1], a * 64, kb * 128, b);
            tma_load_3d(sV + a * kAtom, &mv, &bar[1], a * 64, kb * 128, b);
          }
        } else {  // K = V = kv: kept in the V buffer (the K buffer holds P)
          mbar_arrive_expect_tx(&bar[1], A * kAtom);
          for (int a = 0; a < A; ++a) tma_load_3d(sV + a * kAtom, &mkv, &bar[1], a * 64, kb * 128, b);
        }
        mbar_wait(&bar[1], n_kv & 1, P.err, kErrTimeoutFull);
        if (q_wait) {
          mbar_wait(&bar[0], 0, P.err, kErrTimeoutFull);
          q_wait = false;
        }
        tc_fence_after();
        const uint32_t aq = smem_u32(sQ), ak = smem_u32(br == 0 ? sK : sV);
#pragma unroll
        for (int s = 0; s < HD / 16; ++s) mma_bf16(tbase, desc_k(aq, s), desc_k(ak, s), kIdS, s > 0 ? 1u : 0u);
        mma_commit(&bar[2]);
      }
      __syncwarp();
      ++n_kv;
      mbar_wait(&bar[2], n_s & 1, P.err, kErrTimeoutAccum);
      __syncwarp();  // reconverge before warp-collective tcgen05.ld
      ++n_s;
      tc_fence_after();
      uint32_t wmask[4] = {0u, 0u, 0u, 0u};
      if (br == 1 && P.mode == 2 && row_ok) {
        const uint32_t* srow = P.sel + (static_cast<int64_t>(b) * P.T + qpos) * P.mask_words;
#pragma unroll
        for (int c = 0; c < 4; ++c) wmask[c] = kb * 4 + c < P.mask_words ? srow[kb * 4 + c] : 0u;
      }
      // visible keys of this row: [klo, khi], and for CSA the indexer's bitmask
      int klo = 1, khi = 0;
      if (row_ok) {
        if (br == 0) {
          klo = qpos - window + 1;
          khi = qpos;
        } else if (mode == 1) {
          klo = 0;
          khi = qpos >= cm ? min(cn - 1, (qpos - cm) / cm) : -1;
        } else {
          klo = 0;
          khi = cn - 1;
        }
      }
      const bool bits = br == 1 && mode == 2;
      const bool cap = br == 0 && softcap > 0.f;
      // pass 1: row max of the visible logits (branch-free per element)
      float rmax = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tS + c * 32, r);
        const uint32_t word = !bits ? 0xffffffffu : (c == 0 ? wmask[0] : c == 1 ? wmask[1] : c == 2 ? wmask[2] : wmask[3]);
        const int base = kb * 128 + c * 32;
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int key = base + j;
          const bool vis = key >= klo && key <= khi && ((word >> j) & 1u);
          float sv = __uint_as_float(r[j]) * scale;
          if (br == 0) amax = fmaxf(amax, vis ? fabsf(sv) : 0.f);
          if (cap) sv = softcap * tanhf(sv / softcap);
          rmax = fmaxf(rmax, vis ? sv : -INFINITY);
        }
      }
      const float m_new = fmaxf(m_run, rmax);
      if (n_o > o_before) {  // previous PV of this branch must finish before P / O are touched
        mbar_wait(&bar[3], (n_o - 1) & 1, P.err, kErrTimeoutAccum);
        __syncwarp();  // reconverge before warp-collective tcgen05.ld
        tc_fence_after();
        // tcgen05.ld/st are warp-collective: rescale when any lane of the warp needs it
        const bool need = m_new > m_run;
        if (__any_sync(0xffffffffu, need)) {
          const float alpha = need ? __expf(m_run - m_new) : 1.f;
          l_run *= alpha;
#pragma unroll 1
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(tO + c * 32, r);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * alpha);
            tmem_st32(tO + c * 32, r);
          }
          tmem_st_wait();
        }
      } else if (m_new > m_run) {
        l_run *= __expf(m_run - m_new);  // only the sink contributed so far
      }
      m_run = m_new;
      // pass 2: probabilities -> bf16 P tile
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tS + c * 32, r);
        const uint32_t word = !bits ? 0xffffffffu : (c == 0 ? wmask[0] : c == 1 ? wmask[1] : c == 2 ? wmask[2] : wmask[3]);
        const int base = kb * 128 + c * 32;
        tmem_ld_wait();
        float pv[32];
        float lp[4] = {0.f, 0.f, 0.f, 0.f};  // independent partial sums (no 32-long add chain)
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int key = base + j;
          const bool vis = key >= klo && key <= khi && ((word >> j) & 1u);
          float sv = __uint_as_float(r[j]) * scale;
          if (cap) sv = softcap * tanhf(sv / softcap);
          const float pr = exp_sfu(vis ? sv - m_run : -INFINITY);  // masked lanes: e^-inf = 0
          lp[j & 3] += pr;
          pv[j] = pr;
        }
        l_run += (lp[0] + lp[1]) + (lp[2] + lp[3]);
        put_row32(sP, tid, c * 32, pv);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      if (leader) {
        tc_fence_after();
        const uint32_t ap = smem_u32(sP), av = smem_u32(sV);
#pragma unroll
        for (int s = 0; s < 8; ++s)
          mma_bf16(tbase + 128, desc_k(ap, s), desc_mn(av, s), kIdO, (n_o > o_before || s > 0) ? 1u : 0u);
        mma_commit(&bar[3]);
      }
      __syncwarp();
      ++n_o;
    }
    // ---- branch epilogue
    const bool any = n_o > o_before;
    if (any) {
      mbar_wait(&bar[3], (n_o - 1) & 1, P.err, kErrTimeoutAccum);
      __syncwarp();  // reconverge before warp-collective tcgen05.ld
      tc_fence_after();
    }
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    if (row_ok) P.lse[((static_cast<int64_t>(br) * P.B + b) * P.H + h) * P.T + qpos] =
        l_run > 0.f ? m_run + __logf(l_run) : INFINITY;
    __nv_bfloat16* dst = (br == 0 ? P.o_sw : P.o_c) + row_base * HD;
#pragma unroll 1
    for (int c = 0; c < HD / 32; ++c) {
      float v[32];
      if (any) {
        uint32_t r[32];
        tmem_ld32(tO + c * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * inv;
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
      }
      if (row_ok) {
        store_bf16x32(dst + c * 32, v);
        if (br == 1) {
          float w[32];
          load_bf16x32(P.o_sw + row_base * HD + c * 32, w);
#pragma unroll
          for (int j = 0; j < 32; ++j) w[j] += v[j];
          store_bf16x32(P.out + row_base * HD + c * 32, w);
        }
      }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }

  if (P.max_logit != nullptr) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    if (lane == 0) red[warp] = amax;
    __syncthreads();
    if (tid == 0) {
      const float mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
      atomicMax(reinterpret_cast<int*>(P.max_logit), __float_as_int(mx));  // non-negative floats order as ints
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 256);
  }
}

// ===================================================================== backward
template <int HD>
__global__ void __launch_bounds__(128, 1)
attn_bwd_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mdo,
                const __grid_constant__ CUtensorMap mk, const __grid_constant__ CUtensorMap mv,
                const __grid_constant__ CUtensorMap mkv, const __grid_constant__ CUtensorMap rdk,
                const __grid_constant__ CUtensorMap rdv, const __grid_constant__ CUtensorMap rdkv,
                const AttnParams P) {
  constexpr int A = HD / 64;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sdO = sQ + A * kAtom;
  uint8_t* sK = sdO + A * kAtom;
  uint8_t* sV = sK + A * kAtom;
  uint8_t* sP = sV + A * kAtom;
  uint8_t* sdS = sP + 2 * kAtom;
  uint8_t* stg = sdS + 2 * kAtom;  // 4 x 4 KB reduce staging
  uint64_t* bar = reinterpret_cast<uint64_t*>(stg + 4 * 4096);  // 0 q/dO, 1 kv, 2 s/dp, 3 grads
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 4);
  __shared__ float red[4];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = blockIdx.x * 128, h = blockIdx.y, b = blockIdx.z;
  const int qpos = t0 + tid;
  const bool row_ok = qpos < P.T;
  const bool leader = tid == 0;
  if (leader) {
    for (int i = 0; i < 4; ++i) mbar_init(&bar[i], 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t tS = tbase, tdP = tbase + 128, tdQ = tbase + 256;
  constexpr uint32_t kIdSS = make_idesc_f16(128, 128, 1, 1, false, false);
  constexpr uint32_t kIdQ = make_idesc_f16(128, HD, 1, 1, false, true);
  constexpr uint32_t kIdKV = make_idesc_f16(128, HD, 1, 1, true, true);

  if (leader) {
    mbar_arrive_expect_tx(&bar[0], 2 * A * kAtom);
    for (int a = 0; a < A; ++a) {
      tma_load_4d(sQ + a * kAtom, &mq, &bar[0], a * 64, h, t0, b);
      tma_load_4d(sdO + a * kAtom, &mdo, &bar[0], a * 64, h, t0, b);
    }
  }
  // per-row softmax statistics and D = rowsum(dO * O) of each branch
  const int64_t row_base = (static_cast<int64_t>(b) * P.T + qpos) * P.H + h;
  float lse[2] = {INFINITY, INFINITY}, Dv[2] = {0.f, 0.f};
  if (row_ok) {
    for (int br = 0; br < (P.mode ? 2 : 1); ++br) {
      lse[br] = P.lse[((static_cast<int64_t>(br) * P.B + b) * P.H + h) * P.T + qpos];
      const __nv_bfloat16* o = (br == 0 ? P.o_sw : P.o_c) + row_base * HD;
      float acc = 0.f;
      for (int c = 0; c < HD; c += 32) {
        float x[32], y[32];
        load_bf16x32(P.dout + row_base * HD + c, x);
        load_bf16x32(o + c, y);
#pragma unroll
        for (int j = 0; j < 32; ++j) acc += x[j] * y[j];
      }
      Dv[br] = acc;
    }
  }
  int n_kv = 0, n_s = 0, n_g = 0;
  bool q_wait = true, dq_any = false;
  float dsink = 0.f;

  for (int br = 0; br < 2; ++br) {
    if (br == 1 && P.mode == 0) break;
    int lo, hi;
    key_blocks(P, br, t0, lo, hi);
    if (branch_has_sink(P, br) && row_ok) dsink -= __expf(P.sink[h] - lse[br]) * Dv[br];
    const int limit = br == 0 ? P.T : P.n;
    for (int kb = lo; kb < hi; ++kb) {
      if (leader) {
        if (n_g > 0) mbar_wait(&bar[3], (n_g - 1) & 1, P.err, kErrTimeoutAccum);
        if (br == 0) {
          mbar_arrive_expect_tx(&bar[1], 2 * A * kAtom);
          for (int a = 0; a < A; ++a) {
            tma_load_3d(sK + a * kAtom, &mk, &bar[1], a * 64, kb * 128, b);
            tma_load_3d(sV + a * kAtom, &mv, &bar[1], a * 64, kb * 128, b);
          }
        } else {
          mbar_arrive_expect_tx(&bar[1], A * kAtom);
          for (int a = 0; a < A; ++a) tma_load_3d(sK + a * kAtom, &mkv, &bar[1], a * 64, kb * 128, b);
        }
        mbar_wait(&bar[1], n_kv & 1, P.err, kErrTimeoutFull);
        if (q_wait) {
          mbar_wait(&bar[0], 0, P.err, kErrTimeoutFull);
          q_wait = false;
        }
        tc_fence_after();
        const uint32_t aq = smem_u32(sQ), ado = smem_u32(sdO), ak = smem_u32(sK);
        const uint32_t av = smem_u32(br == 0 ? sV : sK);
#pragma unroll
        for (int s = 0; s < HD / 16; ++s) mma_bf16(tS, desc_k(aq, s), desc_k(ak, s), kIdSS, s > 0 ? 1u : 0u);
#pragma unroll
        for (int s = 0; s < HD / 16; ++s) mma_bf16(tdP, desc_k(ado, s), desc_k(av, s), kIdSS, s > 0 ? 1u : 0u);
        mma_commit(&bar[2]);
      }
      __syncwarp();
      ++n_kv;
      mbar_wait(&bar[2], n_s & 1, P.err, kErrTimeoutAccum);
      __syncwarp();  // reconverge before warp-collective tcgen05.ld
      ++n_s;
      tc_fence_after();
      uint32_t wmask[4] = {0u, 0u, 0u, 0u};
      if (br == 1 && P.mode == 2 && row_ok) {
        const uint32_t* srow = P.sel + (static_cast<int64_t>(b) * P.T + qpos) * P.mask_words;
#pragma unroll
        for (int c = 0; c < 4; ++c) wmask[c] = kb * 4 + c < P.mask_words ? srow[kb * 4 + c] : 0u;
      }
      int klo = 1, khi = 0;
      if (row_ok) {
        if (br == 0) {
          klo = qpos - P.window + 1;
          khi = qpos;
        } else if (P.mode == 1) {
          klo = 0;
          khi = qpos >= P.m ? min(P.n - 1, (qpos - P.m) / P.m) : -1;
        } else {
          klo = 0;
          khi = P.n - 1;
        }
      }
      const bool bits = br == 1 && P.mode == 2;
      const bool cap = br == 0 && P.softcap > 0.f;
      const float scale = P.scale, softcap = P.softcap, lse_b = lse[br], dv_b = Dv[br];
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t rs[32], rp[32];
        tmem_ld32(tS + lane_off + c * 32, rs);
        tmem_ld32(tdP + lane_off + c * 32, rp);
        const uint32_t word = !bits ? 0xffffffffu : (c == 0 ? wmask[0] : c == 1 ? wmask[1] : c == 2 ? wmask[2] : wmask[3]);
        const int base = kb * 128 + c * 32;
        tmem_ld_wait();
        float pv[32], dv[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int key = base + j;
          const bool vis = key >= klo && key <= khi && ((word >> j) & 1u);
          const float raw = __uint_as_float(rs[j]) * scale;
          float sv = raw, dcap = 1.f;
          if (cap) {
            const float th = tanhf(raw / softcap);
            sv = softcap * th;
            dcap = 1.f - th * th;
          }
          const float pr = exp_sfu(vis ? sv - lse_b : -INFINITY);
          pv[j] = pr;
          dv[j] = pr * (__uint_as_float(rp[j]) - dv_b) * dcap * scale;
        }
        put_row32(sP, tid, c * 32, pv);
        put_row32(sdS, tid, c * 32, dv);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      if (leader) {
        tc_fence_after();
        const uint32_t ads = smem_u32(sdS), ap = smem_u32(sP), ak = smem_u32(sK), aq = smem_u32(sQ);
        const uint32_t ado = smem_u32(sdO);
#pragma unroll
        for (int s = 0; s < 8; ++s)  // dQ += dS K
          mma_bf16(tdQ, desc_k(ads, s), desc_mn(ak, s), kIdQ, (dq_any || s > 0) ? 1u : 0u);
#pragma unroll
        for (int s = 0; s < 8; ++s)  // dK_blk = dS^T Q
          mma_bf16(tS, desc_mn(ads, s), desc_mn(aq, s), kIdKV, s > 0 ? 1u : 0u);
        // dV_blk = P^T dO (window branch) or added to dKV (compressed branch, K = V)
        const uint32_t tv = br == 0 ? tdP : tS;
#pragma unroll
        for (int s = 0; s < 8; ++s)
          mma_bf16(tv, desc_mn(ap, s), desc_mn(ado, s), kIdKV, (br == 1 || s > 0) ? 1u : 0u);
        mma_commit(&bar[3]);
      }
      __syncwarp();
      dq_any = true;
      mbar_wait(&bar[3], n_g & 1, P.err, kErrTimeoutAccum);
      __syncwarp();  // reconverge before warp-collective tcgen05.ld
      ++n_g;
      tc_fence_after();
      // reduce the per-block key gradients into the fp32 buffers (TMA .add); thread = key row
      const int krow = kb * 128 + warp * 32;
      uint8_t* wst = stg + warp * 4096;
      for (int part = 0; part < (br == 0 ? 2 : 1); ++part) {
        const uint32_t tp = (part == 0 ? tS : tdP) + lane_off;
        const CUtensorMap* map = br == 1 ? &rdkv : (part == 0 ? &rdk : &rdv);
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tp + c * 32, r);
          tmem_ld_wait();
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
          uint8_t* myrow = wst + lane * 128;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<uint4*>(myrow + ((q ^ (lane & 7)) << 4)) =
                make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && krow < limit) {
            tma_reduce_add_3d(map, wst, c * 32, krow, b);
            bulk_commit_group();
          }
        }
      }
      tc_fence_before();
      __syncthreads();
    }
  }
  // dQ
  if (dq_any) tc_fence_after();
#pragma unroll 1
  for (int c = 0; c < HD / 32; ++c) {
    float v[32];
    if (dq_any) {
      uint32_t r[32];
      tmem_ld32(tdQ + lane_off + c * 32, r);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = 0.f;
    }
    if (row_ok) store_bf16x32(P.dq + row_base * HD + c * 32, v);
  }
  if (P.sink != nullptr && P.dsink != nullptr) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) dsink += __shfl_xor_sync(0xffffffffu, dsink, off);
    if (lane == 0) red[warp] = dsink;
    __syncthreads();
    if (tid == 0) atomicAdd(P.dsink + h, red[0] + red[1] + red[2] + red[3]);
  }
  if (lane == 0) bulk_wait_all();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ========================================================================= host
static CUtensorMap bf16_rows_map(const torch::Tensor& t, int64_t rows, int64_t batch) {
  // t: (batch, rows, HD) contiguous -> 3-D (HD, rows, batch), box 64 x 128, 128B swizzle
  const int64_t hd = t.size(-1);
  uint64_t dims[3] = {static_cast<uint64_t>(hd), static_cast<uint64_t>(rows), static_cast<uint64_t>(batch)};
  uint64_t strides[2] = {static_cast<uint64_t>(hd * 2), static_cast<uint64_t>(rows * hd * 2)};
  uint32_t box[3] = {64, 128, 1};
  return make_map_nd(t.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

static CUtensorMap bf16_heads_map(const torch::Tensor& t) {
  // t: (B, T, H, HD) contiguous -> 4-D (HD, H, T, B), box 64 x 1 x 128 x 1
  const int64_t B = t.size(0), T = t.size(1), H = t.size(2), hd = t.size(3);
  uint64_t dims[4] = {static_cast<uint64_t>(hd), static_cast<uint64_t>(H), static_cast<uint64_t>(T),
                      static_cast<uint64_t>(B)};
  uint64_t strides[3] = {static_cast<uint64_t>(hd * 2), static_cast<uint64_t>(H * hd * 2),
                         static_cast<uint64_t>(T * H * hd * 2)};
  uint32_t box[4] = {64, 1, 128, 1};
  return make_map_nd(t.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

static CUtensorMap f32_rows_map(const torch::Tensor& t, int64_t rows, int64_t batch) {
  // fp32 (batch, rows, HD) -> reduce-add destination, box 32 x 32
  const int64_t hd = t.size(-1);
  uint64_t dims[3] = {static_cast<uint64_t>(hd), static_cast<uint64_t>(rows), static_cast<uint64_t>(batch)};
  uint64_t strides[2] = {static_cast<uint64_t>(hd * 4), static_cast<uint64_t>(rows * hd * 4)};
  uint32_t box[3] = {32, 32, 1};
  return make_map_nd(t.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

static AttnParams make_params(const torch::Tensor& q, const torch::Tensor& kv, int64_t mode, int64_t m,
                              int64_t window, const torch::Tensor& sink, const torch::Tensor& sel, double softcap,
                              double scale, torch::Tensor err) {
  AttnParams p{};
  p.B = q.size(0); p.T = q.size(1); p.H = q.size(2);
  p.n = mode ? static_cast<int>(kv.size(1)) : 0;
  p.window = static_cast<int>(window);
  p.mode = static_cast<int>(mode);
  p.m = static_cast<int>(std::max<int64_t>(m, 1));
  p.mask_words = mode == 2 ? static_cast<int>(sel.size(-1)) : 0;
  p.scale = static_cast<float>(scale);
  p.softcap = static_cast<float>(softcap);
  p.sink = sink.numel() ? sink.data_ptr<float>() : nullptr;
  p.sel = mode == 2 ? reinterpret_cast<const uint32_t*>(sel.data_ptr<int32_t>()) : nullptr;
  p.err = err.data_ptr<int>();
  return p;
}

static void check_inputs(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                         const torch::Tensor& kv, int64_t mode) {
  TORCH_CHECK(q.dim() == 4 && q.is_contiguous() && q.scalar_type() == at::kBFloat16, "q: (B, T, H, HD) bf16");
  const int64_t hd = q.size(3);
  TORCH_CHECK(hd == 64 || hd == 128, "head_dim must be 64 or 128 (pad smaller heads)");
  TORCH_CHECK(k.sizes() == v.sizes() && k.dim() == 3 && k.size(0) == q.size(0) && k.size(1) == q.size(1) &&
                  k.size(2) == hd && k.is_contiguous() && v.is_contiguous(), "k/v: (B, T, HD)");
  if (mode) TORCH_CHECK(kv.dim() == 3 && kv.size(0) == q.size(0) && kv.size(2) == hd && kv.is_contiguous(),
                        "kv: (B, n, HD)");
}

static int fwd_smem(int hd) { return 2 * (hd / 64) * kAtom + std::max(hd / 64, 2) * kAtom + 64 + 1024; }
static int bwd_smem(int hd) { return 4 * (hd / 64) * kAtom + 4 * kAtom + 4 * 4096 + 64 + 1024; }


void attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor kv, torch::Tensor sel, int64_t mode,
              int64_t m, int64_t window, torch::Tensor sink, double softcap, double scale, torch::Tensor o_sw,
              torch::Tensor o_c, torch::Tensor out, torch::Tensor lse, torch::Tensor max_logit, torch::Tensor err) {
  check_inputs(q, k, v, kv, mode);
  c10::cuda::CUDAGuard guard(q.device());
  AttnParams p = make_params(q, kv, mode, m, window, sink, sel, softcap, scale, err);
  if (mode && p.n == 0) p.mode = 0;
  p.o_sw = reinterpret_cast<__nv_bfloat16*>(o_sw.data_ptr());
  p.o_c = p.mode ? reinterpret_cast<__nv_bfloat16*>(o_c.data_ptr()) : nullptr;
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.lse = lse.data_ptr<float>();
  p.max_logit = max_logit.numel() ? max_logit.data_ptr<float>() : nullptr;
  const int64_t B = q.size(0), T = q.size(1), H = q.size(2), hd = q.size(3);
  if (B * T == 0) return;
  CUtensorMap mq = bf16_heads_map(q), mk = bf16_rows_map(k, T, B), mv = bf16_rows_map(v, T, B);
  CUtensorMap mkv = p.mode ? bf16_rows_map(kv, kv.size(1), B) : mk;
  const dim3 grid((T + 127) / 128, H, B);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int smem = fwd_smem(hd);
  if (hd == 128) {
    cudaFuncSetAttribute(attn_fwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attn_fwd_kernel<128><<<grid, 128, smem, stream>>>(mq, mk, mv, mkv, p);
  } else {
    cudaFuncSetAttribute(attn_fwd_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attn_fwd_kernel<64><<<grid, 128, smem, stream>>>(mq, mk, mv, mkv, p);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// dk/dv/dkv/dsink must be zero-initialised fp32 buffers.
void attn_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor kv, torch::Tensor sel, int64_t mode,
              int64_t m, int64_t window, torch::Tensor sink, double softcap, double scale, torch::Tensor o_sw,
              torch::Tensor o_c, torch::Tensor lse, torch::Tensor dout, torch::Tensor dq, torch::Tensor dk,
              torch::Tensor dv, torch::Tensor dkv, torch::Tensor dsink, torch::Tensor err) {
  check_inputs(q, k, v, kv, mode);
  TORCH_CHECK(dout.sizes() == q.sizes() && dout.is_contiguous(), "dout like q");
  c10::cuda::CUDAGuard guard(q.device());
  AttnParams p = make_params(q, kv, mode, m, window, sink, sel, softcap, scale, err);
  if (mode && p.n == 0) p.mode = 0;
  p.o_sw = reinterpret_cast<__nv_bfloat16*>(o_sw.data_ptr());
  p.o_c = p.mode ? reinterpret_cast<__nv_bfloat16*>(o_c.data_ptr()) : nullptr;
  p.lse = lse.data_ptr<float>();
  p.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  p.dq = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr());
  p.dsink = dsink.numel() ? dsink.data_ptr<float>() : nullptr;
  const int64_t B = q.size(0), T = q.size(1), H = q.size(2), hd = q.size(3);
  if (B * T == 0) return;
  CUtensorMap mq = bf16_heads_map(q), mdo = bf16_heads_map(dout);
  CUtensorMap mk = bf16_rows_map(k, T, B), mv = bf16_rows_map(v, T, B);
  CUtensorMap mkv = p.mode ? bf16_rows_map(kv, kv.size(1), B) : mk;
  CUtensorMap rdk = f32_rows_map(dk, T, B), rdv = f32_rows_map(dv, T, B);
  CUtensorMap rdkv = p.mode ? f32_rows_map(dkv, dkv.size(1), B) : rdk;
  const dim3 grid((T + 127) / 128, H, B);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const int smem = bwd_smem(hd);
  if (hd == 128) {
    cudaFuncSetAttribute(attn_bwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attn_bwd_kernel<128><<<grid, 128, smem, stream>>>(mq, mdo, mk, mv, mkv, rdk, rdv, rdkv, p);
  } else {
    cudaFuncSetAttribute(attn_bwd_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attn_bwd_kernel<64><<<grid, 128, smem, stream>>>(mq, mdo, mk, mv, mkv, rdk, rdv, rdkv, p);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// CSA selection bitmask from the indexer's top-k ids (-1 = none): sel[b, t, i / 32] |= 1 << (i % 32).
// An id outside [-1, n) records kErrBounds and selects nothing.
__global__ void csa_select_mask_kernel(const int64_t* __restrict__ top, int rows, int k, int n, int words,
                                       uint32_t* __restrict__ sel, int* err) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  for (int i = lane; i < k; i += 32) {
    const int64_t id = top[static_cast<int64_t>(row) * k + i];
    if (index_ok(id, -1, n, err) && id >= 0)
      atomicOr(sel + static_cast<int64_t>(row) * words + id / 32, 1u << (id % 32));
  }
}

void csa_select_mask(torch::Tensor top, int64_t n, torch::Tensor sel, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(top.device());
  TORCH_CHECK(top.scalar_type() == at::kLong && top.is_contiguous(), "top: int64 contiguous");
  TORCH_CHECK(sel.size(-1) * 32 >= n, "sel has fewer bits per row than blocks");
  const int k = top.size(-1);
  const int rows = top.numel() / std::max(k, 1);
  sel.zero_();
  if (rows == 0 || k == 0) return;
  csa_select_mask_kernel<<<(rows + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      top.data_ptr<int64_t>(), rows, k, static_cast<int>(n), static_cast<int>(sel.size(-1)),
      reinterpret_cast<uint32_t*>(sel.data_ptr<int32_t>()), err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Indexer top-k straight to the CSA selection bitmask: per query row, the k highest finite
// scores among n blocks (masked blocks are -inf and never picked; ties at the k-th score are
// taken lowest block index first), written as bits of sel (B*T rows of `words` uint32).  The
// k-th largest score is found by radix selection over an order-preserving integer key, 8 bits
// per pass, reading the row from L2; no (rows, k) index tensor and no sort.
namespace {
__device__ __forceinline__ uint32_t score_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
}  // namespace

__global__ void __launch_bounds__(256) indexer_select_kernel(const float* __restrict__ scores, int n, int k,
                                                            int words, uint32_t* __restrict__ sel) {
  __shared__ unsigned hist[256];
  __shared__ unsigned s_cnt[8];
  __shared__ uint32_t s_prefix;
  __shared__ unsigned s_need;
  __shared__ unsigned wsum[512 + 1];
  const int row = blockIdx.x;
  const float* sr = scores + static_cast<int64_t>(row) * n;
  uint32_t* out = sel + static_cast<int64_t>(row) * words;
  // finite scores only
  unsigned fin = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) fin += isfinite(sr[i]) ? 1u : 0u;
  for (int o = 16; o > 0; o >>= 1) fin += __shfl_xor_sync(0xffffffffu, fin, o);
  if ((threadIdx.x & 31) == 0) s_cnt[threadIdx.x >> 5] = fin;
  __syncthreads();
  fin = 0;
  for (int w = 0; w < 8; ++w) fin += s_cnt[w];
  const bool all = static_cast<unsigned>(k) >= fin;
  uint32_t tau = 0;  // keep keys > tau, plus `need` ties at tau (lowest index first)
  unsigned need = 0;
  if (!all) {
    uint32_t prefix = 0, mask = 0;
    unsigned want = static_cast<unsigned>(k);
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0;
      __syncthreads();
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = sr[i];
        if (!isfinite(v)) continue;
        const uint32_t key = score_key(v);
        if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        unsigned acc = 0;
        int b = 255;
        for (; b > 0; --b) {
          if (acc + hist[b] >= want) break;
          acc += hist[b];
        }
        s_prefix = prefix | (static_cast<uint32_t>(b) << shift);
        s_need = want - acc;
      }
      __syncthreads();
      prefix = s_prefix;
      want = s_need;
      mask |= 255u << shift;
      __syncthreads();
    }
    tau = prefix;
    need = want;  // how many of the keys equal to tau are kept
  }
  // per-word tie counts, exclusive scan in word order, then the bits
  for (int w = threadIdx.x; w < words; w += blockDim.x) {
    unsigned ties = 0;
    if (!all) {
      for (int j = 0; j < 32; ++j) {
        const int i = w * 32 + j;
        if (i < n && isfinite(sr[i]) && score_key(sr[i]) == tau) ++ties;
      }
    }
    wsum[w] = ties;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned acc = 0;
    for (int w = 0; w < words; ++w) {
      const unsigned t = wsum[w];
      wsum[w] = acc;
      acc += t;
    }
  }
  __syncthreads();
  for (int w = threadIdx.x; w < words; w += blockDim.x) {
    uint32_t bits = 0;
    unsigned rank = wsum[w];
    for (int j = 0; j < 32; ++j) {
      const int i = w * 32 + j;
      if (i >= n) break;
      const float v = sr[i];
      if (!isfinite(v)) continue;
      if (all) {
        bits |= 1u << j;
        continue;
      }
      const uint32_t key = score_key(v);
      if (key > tau || (key == tau && rank++ < need)) bits |= 1u << j;
    }
    out[w] = bits;
  }
}

// scores (B, T, n) fp32 (block-causally masked with -inf) -> sel (B, T, words) int32 bitmask of
// the top-k finite blocks per row.
void indexer_select_mask(torch::Tensor scores, int64_t k, torch::Tensor sel) {
  c10::cuda::CUDAGuard guard(scores.device());
  TORCH_CHECK(scores.scalar_type() == at::kFloat && scores.is_contiguous(), "scores: contiguous fp32");
  const int64_t n = scores.size(-1);
  const int64_t rows = scores.numel() / std::max<int64_t>(n, 1);
  const int64_t words = sel.size(-1);
  TORCH_CHECK(sel.scalar_type() == at::kInt && sel.is_contiguous() && sel.numel() == rows * words &&
                  words * 32 >= n && words <= 512, "sel: (rows, words) int32, n <= 16384");
  if (rows == 0) return;
  indexer_select_kernel<<<static_cast<unsigned>(rows), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      scores.data_ptr<float>(), static_cast<int>(n), static_cast<int>(k), static_cast<int>(words),
      reinterpret_cast<uint32_t*>(sel.data_ptr<int32_t>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sv4
