// Single-token decode attention over the heterogeneous cache, one kernel per layer.
//
// For every sequence b and query head h (one query token, MQA: one K/V head):
//
//   out[b, h] = SW(b, h) + C(b, h)
//   SW : softmax over the sliding-window ring (W slots; slot j is live iff its age
//        (pos % W - j) mod W is <= pos), scores softcapped, plus an optional per-head sink
//        logit in the denominator;
//   C  : softmax over compressed entries with K = V = RMSNorm(entry) (weight w, eps):
//        mode 1 (HCA): entries 0..n-1, entry s visible iff s*m + m - 1 < pos, optional sink;
//        mode 2 (CSA): the entries listed in top[b, :] (-1 = none), no sink.
//   A branch with no visible key and no sink contributes zero.
//
// This is the decode step of the reference's cached attention (core/attention/swa.py,
// hca.py and csa.py with kv_cache; the scores follow common.py's scaled_dot_product and
// softmax_with_sink) with every mask, gather, normalisation and both softmaxes in one
// pass: the eager composition is ~40 small launches per layer, which made a CUDA-graph
// decode step launch-bound.
//
// Layout: one CTA per (b, group of 4 heads), 128 threads.  Scores: thread t owns keys
// t, t + 128, ... and computes the 4 heads' dot products from its own key row (the
// queries, pre-multiplied by the norm weight for C, are broadcast from shared memory).
// Softmax: warp h reduces head h.  Output: thread t owns dimension t and streams the value
// rows (coalesced 256-byte rows) against the 4 heads' probabilities.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cuda_bf16.h>

#include "common.cuh"

namespace sv4 {
namespace {

constexpr int kD = 128;
constexpr int kHeads = 4;  // heads per CTA
constexpr int kThreads = 128;

struct DecodeArgs {
  const __nv_bfloat16* q;      // (B, H, kD)
  const __nv_bfloat16* kw;     // (B, W, kD)
  const __nv_bfloat16* vw;     // (B, W, kD)
  const int64_t* pos;          // device scalar
  const float* sink_sw;        // (H) or null
  const __nv_bfloat16* comp;   // (B, n, kD) raw entries or null
  const float* norm_w;         // (kD)
  const int64_t* top;          // (B, ktop) or null
  const float* sink_c;         // (H) or null
  __nv_bfloat16* out;          // (B, H, kD)
  int H, W, n, m, ktop, mode;
  float scale, softcap, eps;
};

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// One attention branch over L keys whose key and value are the same normalised row
// (K = V = w * x * rsqrt(mean(x^2) + eps), w folded into the queries by the caller); adds
// (p @ x * rsqrt) / denominator into acc[4] for dimension t.  key_row(j) returns the raw
// row or null when key j is not visible.
template <bool NORM, typename RowFn, typename ValFn>
__device__ void branch_kv(const float (*qs)[kD], float4* s, float* rs, float* red, int L, RowFn key_row,
                          ValFn val_row, const float* sink, int h0, float scale, float softcap, float eps,
                          float* acc) {
  const int t = threadIdx.x, warp = t / 32, lane = t % 32;
  // scores
  for (int j = t; j < L; j += kThreads) {
    const __nv_bfloat16* row = key_row(j);
    float4 sc = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    if (row != nullptr) {
      float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f, ss = 0.f;
#pragma unroll 4
      for (int c = 0; c < kD; c += 8) {
        float x[8];
        load8(row + c, x);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          d0 = fmaf(qs[0][c + e], x[e], d0);
          d1 = fmaf(qs[1][c + e], x[e], d1);
          d2 = fmaf(qs[2][c + e], x[e], d2);
          d3 = fmaf(qs[3][c + e], x[e], d3);
          if (NORM) ss = fmaf(x[e], x[e], ss);
        }
      }
      float r = scale;
      if (NORM) {
        const float rn = rsqrtf(ss / kD + eps);
        rs[j] = rn;
        r *= rn;
      }
      sc = make_float4(d0 * r, d1 * r, d2 * r, d3 * r);
      if (softcap > 0.f) {
        sc.x = softcap * tanhf(sc.x / softcap);
        sc.y = softcap * tanhf(sc.y / softcap);
        sc.z = softcap * tanhf(sc.z / softcap);
        sc.w = softcap * tanhf(sc.w / softcap);
      }
    } else if (NORM) {
      rs[j] = 0.f;
    }
    s[j] = sc;
  }
  __syncthreads();
  // softmax of head h0 + warp; probabilities overwrite the scores, 1 / denominator in red[warp]
  {
    float* sh = reinterpret_cast<float*>(s) + warp;
    const float sk = sink != nullptr ? sink[h0 + warp] : -INFINITY;
    float mx = sk;
    for (int j = lane; j < L; j += 32) mx = fmaxf(mx, sh[4 * j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    if (mx == -INFINITY) {
      for (int j = lane; j < L; j += 32) sh[4 * j] = 0.f;
    } else {
      for (int j = lane; j < L; j += 32) {
        const float p = __expf(sh[4 * j] - mx);
        sh[4 * j] = p;
        sum += p;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
      const float den = sum + (sink != nullptr && mx != -INFINITY ? __expf(sk - mx) : 0.f);
      red[warp] = den > 0.f ? 1.0f / den : 0.f;
    }
  }
  __syncthreads();
  // p @ V for dimension t
  float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
#pragma unroll 4
  for (int j = 0; j < L; ++j) {
    float4 p = s[j];
    if (NORM) {
      const float rn = rs[j];
      p.x *= rn; p.y *= rn; p.z *= rn; p.w *= rn;
    }
    if (p.x == 0.f && p.y == 0.f && p.z == 0.f && p.w == 0.f) continue;  // also skips invisible rows
    const __nv_bfloat16* row = val_row(j);
    const float v = __bfloat162float(row[t]);
    o0 = fmaf(p.x, v, o0);
    o1 = fmaf(p.y, v, o1);
    o2 = fmaf(p.z, v, o2);
    o3 = fmaf(p.w, v, o3);
  }
  // (for NORM the value rows still lack the norm weight: the caller applies it)
  acc[0] += o0 * red[0];
  acc[1] += o1 * red[1];
  acc[2] += o2 * red[2];
  acc[3] += o3 * red[3];
  __syncthreads();  // scores / probabilities are reused by the next branch
}

template <bool NORM, typename RowFn>
__device__ void branch(const float (*qs)[kD], float4* s, float* rs, float* red, int L, RowFn key_row,
                       const float* sink, int h0, float scale, float softcap, float eps, float* acc) {
  branch_kv<NORM>(qs, s, rs, red, L, key_row, key_row, sink, h0, scale, softcap, eps, acc);
}

__global__ void __launch_bounds__(kThreads) decode_attn_kernel(const DecodeArgs a) {
  extern __shared__ __align__(16) float dsm[];
  __shared__ float qs[kHeads][kD];
  __shared__ float red[kHeads];
  float4* s = reinterpret_cast<float4*>(dsm);
  const int lmax = max(a.W, a.mode == 2 ? a.ktop : a.n);
  float* rs = dsm + 4 * lmax;
  const int b = blockIdx.x, h0 = blockIdx.y * kHeads, t = threadIdx.x;
  const int64_t pos = *a.pos;
#pragma unroll
  for (int h = 0; h < kHeads; ++h) qs[h][t] = __bfloat162float(a.q[(static_cast<int64_t>(b) * a.H + h0 + h) * kD + t]);
  __syncthreads();
  float acc[kHeads] = {0.f, 0.f, 0.f, 0.f};

  // sliding-window ring
  const int slot = static_cast<int>(pos % a.W);
  const __nv_bfloat16* kb = a.kw + static_cast<int64_t>(b) * a.W * kD;
  const __nv_bfloat16* vb = a.vw + static_cast<int64_t>(b) * a.W * kD;
  {
    // keys and values are different rows: score with K, then accumulate with V
    const int W = a.W;
    auto krow = [&](int j) -> const __nv_bfloat16* {
      const int age = ((slot - j) % W + W) % W;
      return age <= pos ? kb + static_cast<int64_t>(j) * kD : nullptr;
    };
    // scores over K
    for (int j = t; j < W; j += kThreads) {
      const __nv_bfloat16* row = krow(j);
      float4 sc = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      if (row != nullptr) {
        float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll 4
        for (int c = 0; c < kD; c += 8) {
          float x[8];
          load8(row + c, x);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            d0 = fmaf(qs[0][c + e], x[e], d0);
            d1 = fmaf(qs[1][c + e], x[e], d1);
            d2 = fmaf(qs[2][c + e], x[e], d2);
            d3 = fmaf(qs[3][c + e], x[e], d3);
          }
        }
        sc = make_float4(d0 * a.scale, d1 * a.scale, d2 * a.scale, d3 * a.scale);
        if (a.softcap > 0.f) {
          sc.x = a.softcap * tanhf(sc.x / a.softcap);
          sc.y = a.softcap * tanhf(sc.y / a.softcap);
          sc.z = a.softcap * tanhf(sc.z / a.softcap);
          sc.w = a.softcap * tanhf(sc.w / a.softcap);
        }
      }
      s[j] = sc;
    }
  }
  __syncthreads();
  {
    const int warp = t / 32, lane = t % 32;
    float* sh = reinterpret_cast<float*>(s) + warp;
    const float sk = a.sink_sw != nullptr ? a.sink_sw[h0 + warp] : -INFINITY;
    float mx = sk;
    for (int j = lane; j < a.W; j += 32) mx = fmaxf(mx, sh[4 * j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int j = lane; j < a.W; j += 32) {
      const float p = mx == -INFINITY ? 0.f : __expf(sh[4 * j] - mx);
      sh[4 * j] = p;
      sum += p;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
      const float den = sum + (a.sink_sw != nullptr && mx != -INFINITY ? __expf(sk - mx) : 0.f);
      red[warp] = den > 0.f ? 1.0f / den : 0.f;
    }
  }
  __syncthreads();
  {
    float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
#pragma unroll 4
    for (int j = 0; j < a.W; ++j) {
      const float4 p = s[j];
      if (p.x == 0.f && p.y == 0.f && p.z == 0.f && p.w == 0.f) continue;
      const float v = __bfloat162float(vb[static_cast<int64_t>(j) * kD + t]);
      o0 = fmaf(p.x, v, o0);
      o1 = fmaf(p.y, v, o1);
      o2 = fmaf(p.z, v, o2);
      o3 = fmaf(p.w, v, o3);
    }
    acc[0] = o0 * red[0];
    acc[1] = o1 * red[1];
    acc[2] = o2 * red[2];
    acc[3] = o3 * red[3];
  }
  __syncthreads();

  if (a.mode != 0) {
    // compressed branch: queries pre-multiplied by the norm weight (K = V = w * x * rsqrt)
    const float w_t = a.norm_w[t];
#pragma unroll
    for (int h = 0; h < kHeads; ++h) qs[h][t] *= w_t;
    __syncthreads();
    const __nv_bfloat16* cb = a.comp + static_cast<int64_t>(b) * a.n * kD;
    float cacc[kHeads] = {0.f, 0.f, 0.f, 0.f};
    if (a.mode == 1) {
      const int64_t m = a.m;
      auto row = [&](int j) -> const __nv_bfloat16* {
        return static_cast<int64_t>(j) * m + m - 1 < pos ? cb + static_cast<int64_t>(j) * kD : nullptr;
      };
      branch<true>(qs, s, rs, red, a.n, row, a.sink_c, h0, a.scale, 0.f, a.eps, cacc);
    } else {
      const int64_t* tb = a.top + static_cast<int64_t>(b) * a.ktop;
      const int n = a.n;
      auto row = [&](int j) -> const __nv_bfloat16* {
        const int64_t e = tb[j];
        return (e >= 0 && e < n) ? cb + e * kD : nullptr;
      };
      branch<true>(qs, s, rs, red, a.ktop, row, nullptr, h0, a.scale, 0.f, a.eps, cacc);
    }
#pragma unroll
    for (int h = 0; h < kHeads; ++h) acc[h] += cacc[h] * w_t;
  }
#pragma unroll
  for (int h = 0; h < kHeads; ++h)
    a.out[(static_cast<int64_t>(b) * a.H + h0 + h) * kD + t] = __float2bfloat16(acc[h]);
}

// ------------------------------------------------------------------ paged variant
// Sequences of different lengths decode together; every cache stream lives in pages of a
// shared pool (page_rows rows of 128) addressed through per-sequence block tables.
//   K / V stream (B tables into kpool / vpool): len[b] rows including the current token; the
//        window branch attends to the last min(window, len) rows (window 0: all of them).
//   entries stream (mode 1 / 2, tables into epool): elen[b] compressed entries; mode 1 sees
//        entry s iff s*m + m - 1 < len - 1 (the contiguous kernel's rule at pos = len - 1);
//        mode 2 sees the entries listed in top[b, :] that are < elen[b].
struct PagedArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* kpool;
  const __nv_bfloat16* vpool;
  const int* ktab;             // (B, kmaxp)
  const int* klen;             // (B)
  const __nv_bfloat16* epool;  // or null
  const int* etab;             // (B, emaxp)
  const int* elen;             // (B)
  const float* norm_w;
  const int64_t* top;          // (B, ktop) or null
  const float* sink_sw;
  const float* sink_c;
  __nv_bfloat16* out;
  int H, page_rows, kmaxp, emaxp, n_pages_k, n_pages_e, window, m, ktop, mode, lmax;
  float scale, softcap, eps;
  int* err;
};

__device__ __forceinline__ const __nv_bfloat16* paged_row(const __nv_bfloat16* pool, const int* tab, int maxp,
                                                           int n_pages, int page_rows, int64_t r, int* err) {
  const int slot = static_cast<int>(r / page_rows);
  if (slot < 0 || slot >= maxp) { record_error(err, kErrBounds); return nullptr; }
  const int page = tab[slot];
  if (page < 0 || page >= n_pages) { record_error(err, kErrBounds); return nullptr; }
  return pool + (static_cast<int64_t>(page) * page_rows + r % page_rows) * kD;
}

__global__ void __launch_bounds__(kThreads) decode_attn_paged_kernel(const PagedArgs a) {
  extern __shared__ __align__(16) float dsm[];
  __shared__ float qs[kHeads][kD];
  __shared__ float red[kHeads];
  float4* s = reinterpret_cast<float4*>(dsm);
  float* rs = dsm + 4 * a.lmax;
  const int b = blockIdx.x, h0 = blockIdx.y * kHeads, t = threadIdx.x;
  const int len = a.klen[b];
#pragma unroll
  for (int h = 0; h < kHeads; ++h) qs[h][t] = __bfloat162float(a.q[(static_cast<int64_t>(b) * a.H + h0 + h) * kD + t]);
  __syncthreads();
  float acc[kHeads] = {0.f, 0.f, 0.f, 0.f};
  {
    int L = a.window < 0 ? 0 : (a.window > 0 ? min(a.window, len) : len);  // window < 0: compressed only
    L = max(0, min(L, a.lmax));
    const int64_t first = static_cast<int64_t>(len) - L;
    const int* kt = a.ktab + static_cast<int64_t>(b) * a.kmaxp;
    auto krow = [&](int j) { return paged_row(a.kpool, kt, a.kmaxp, a.n_pages_k, a.page_rows, first + j, a.err); };
    auto vrow = [&](int j) { return paged_row(a.vpool, kt, a.kmaxp, a.n_pages_k, a.page_rows, first + j, a.err); };
    branch_kv<false>(qs, s, rs, red, L, krow, vrow, a.sink_sw, h0, a.scale, a.softcap, a.eps, acc);
  }
  if (a.mode != 0) {
    const float w_t = a.norm_w[t];
#pragma unroll
    for (int h = 0; h < kHeads; ++h) qs[h][t] *= w_t;
    __syncthreads();
    const int ne = a.elen[b];
    const int* et = a.etab + static_cast<int64_t>(b) * a.emaxp;
    float cacc[kHeads] = {0.f, 0.f, 0.f, 0.f};
    if (a.mode == 1) {
      const int64_t pos = static_cast<int64_t>(len) - 1, m = a.m;
      const int L = max(0, min(ne, a.lmax));
      auto row = [&](int j) -> const __nv_bfloat16* {
        return static_cast<int64_t>(j) * m + m - 1 < pos
                   ? paged_row(a.epool, et, a.emaxp, a.n_pages_e, a.page_rows, j, a.err) : nullptr;
      };
      branch<true>(qs, s, rs, red, L, row, a.sink_c, h0, a.scale, 0.f, a.eps, cacc);
    } else {
      const int64_t* tb = a.top + static_cast<int64_t>(b) * a.ktop;
      auto row = [&](int j) -> const __nv_bfloat16* {
        const int64_t e = tb[j];
        return (e >= 0 && e < ne) ? paged_row(a.epool, et, a.emaxp, a.n_pages_e, a.page_rows, e, a.err) : nullptr;
      };
      branch<true>(qs, s, rs, red, a.ktop, row, nullptr, h0, a.scale, 0.f, a.eps, cacc);
    }
#pragma unroll
    for (int h = 0; h < kHeads; ++h) acc[h] += cacc[h] * w_t;
  }
#pragma unroll
  for (int h = 0; h < kHeads; ++h)
    a.out[(static_cast<int64_t>(b) * a.H + h0 + h) * kD + t] = __float2bfloat16(acc[h]);
}

// ------------------------------------------------------ split-K window + LSE merge
// Long windows (or window 0 = the whole stream) at small batch leave most SMs idle with one CTA
// per (sequence, 4 heads); the split variant gives each of S CTAs a contiguous slice of the
// window rows and writes the partial (m, l, o): row max of the scores, sum of exp(s - m) and the
// normalised output, which lse_merge combines (the associative merge of tree attention).
__global__ void __launch_bounds__(kThreads) decode_window_split_kernel(const PagedArgs a, int splits, float* pm,
                                                                       float* pl, float* po) {
  extern __shared__ __align__(16) float dsm[];
  __shared__ float qs[kHeads][kD];
  const int b = blockIdx.x, h0 = blockIdx.y * kHeads, z = blockIdx.z, t = threadIdx.x;
  const int warp = t / 32, lane = t % 32;
  const int len = a.klen[b];
  int L = a.window > 0 ? min(a.window, len) : len;
  const int64_t first = static_cast<int64_t>(len) - L;
  const int chunk = (L + splits - 1) / splits;
  const int lo = min(L, z * chunk), n = min(L, lo + chunk) - lo;
  float4* sc = reinterpret_cast<float4*>(dsm);
#pragma unroll
  for (int h = 0; h < kHeads; ++h) qs[h][t] = __bfloat162float(a.q[(static_cast<int64_t>(b) * a.H + h0 + h) * kD + t]);
  __syncthreads();
  const int* kt = a.ktab + static_cast<int64_t>(b) * a.kmaxp;
  for (int j = t; j < n; j += kThreads) {
    const __nv_bfloat16* row = paged_row(a.kpool, kt, a.kmaxp, a.n_pages_k, a.page_rows, first + lo + j, a.err);
    float4 v = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    if (row != nullptr) {
      float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll 4
      for (int c = 0; c < kD; c += 8) {
        float x[8];
        load8(row + c, x);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          d0 = fmaf(qs[0][c + e], x[e], d0);
          d1 = fmaf(qs[1][c + e], x[e], d1);
          d2 = fmaf(qs[2][c + e], x[e], d2);
          d3 = fmaf(qs[3][c + e], x[e], d3);
        }
      }
      v = make_float4(d0 * a.scale, d1 * a.scale, d2 * a.scale, d3 * a.scale);
      if (a.softcap > 0.f) {
        v.x = a.softcap * tanhf(v.x / a.softcap);
        v.y = a.softcap * tanhf(v.y / a.softcap);
        v.z = a.softcap * tanhf(v.z / a.softcap);
        v.w = a.softcap * tanhf(v.w / a.softcap);
      }
    }
    sc[j] = v;
  }
  __syncthreads();
  __shared__ float sm[kHeads], sl[kHeads];
  {  // warp h: max and sum of exponentials of head h0 + h
    float* sh = reinterpret_cast<float*>(sc) + warp;
    float mx = -INFINITY;
    for (int j = lane; j < n; j += 32) mx = fmaxf(mx, sh[4 * j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int j = lane; j < n; j += 32) {
      const float p = mx == -INFINITY ? 0.f : __expf(sh[4 * j] - mx);
      sh[4 * j] = p;
      sum += p;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
      sm[warp] = mx;
      sl[warp] = sum;
    }
  }
  __syncthreads();
  float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
  for (int j = 0; j < n; ++j) {
    const float4 p = sc[j];
    if (p.x == 0.f && p.y == 0.f && p.z == 0.f && p.w == 0.f) continue;
    const __nv_bfloat16* row = paged_row(a.vpool, kt, a.kmaxp, a.n_pages_k, a.page_rows, first + lo + j, nullptr);
    if (row == nullptr) continue;
    const float v = __bfloat162float(row[t]);
    o0 = fmaf(p.x, v, o0);
    o1 = fmaf(p.y, v, o1);
    o2 = fmaf(p.z, v, o2);
    o3 = fmaf(p.w, v, o3);
  }
  const float acc[kHeads] = {o0, o1, o2, o3};
#pragma unroll
  for (int h = 0; h < kHeads; ++h) {
    const int64_t row = (static_cast<int64_t>(z) * gridDim.x + b) * a.H + h0 + h;  // (split, b, head)
    po[row * kD + t] = sl[h] > 0.f ? acc[h] / sl[h] : 0.f;
    if (t == 0) {
      pm[row] = sm[h];
      pl[row] = sl[h];
    }
  }
}

// out[r] = merge over s of (m[s, r], l[s, r], o[s, r, :]); an optional extra logit per row (a
// sink) joins the denominator only.  Rows whose every partial is empty (and no sink) give 0.
__global__ void lse_merge_kernel(const float* __restrict__ m, const float* __restrict__ l,
                                 const float* __restrict__ o, int S, int64_t rows, int D,
                                 const float* __restrict__ extra, int64_t extra_mod, float* __restrict__ out,
                                 float* __restrict__ out_m, float* __restrict__ out_l) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * D) return;
  const int64_t r = i / D;
  const int d = static_cast<int>(i % D);
  float mx = extra != nullptr ? extra[r % extra_mod] : -INFINITY;
  for (int s = 0; s < S; ++s)
    if (l[s * rows + r] > 0.f) mx = fmaxf(mx, m[s * rows + r]);
  float den = 0.f, num = 0.f;
  if (mx != -INFINITY) {
    for (int s = 0; s < S; ++s) {
      const float ls = l[s * rows + r];
      if (ls <= 0.f) continue;
      const float w = __expf(m[s * rows + r] - mx) * ls;
      den += w;
      num += w * o[(s * rows + r) * D + d];
    }
    if (extra != nullptr) den += __expf(extra[r % extra_mod] - mx);
  }
  out[i] = den > 0.f ? num / den : 0.f;
  if (d == 0 && out_m != nullptr) {
    out_m[r] = mx;
    out_l[r] = den;
  }
}

const __nv_bfloat16* bf16_ptr(const torch::Tensor& t) {
  return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr());
}

}  // namespace

// q (B, H, 128); k_win / v_win (B, W, 128); pos int64 scalar; out (B, H, 128).
// mode 0: window only; 1: + prefix-visible compressed entries (HCA); 2: + listed entries (CSA).
void decode_attention(torch::Tensor q, torch::Tensor k_win, torch::Tensor v_win, torch::Tensor pos,
                      c10::optional<torch::Tensor> sink_sw, double softcap, int64_t mode,
                      c10::optional<torch::Tensor> comp, c10::optional<torch::Tensor> norm_w, double eps, int64_t m,
                      c10::optional<torch::Tensor> top, c10::optional<torch::Tensor> sink_c, double scale,
                      torch::Tensor out) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.dim() == 3 && q.size(2) == kD,
              "q: contiguous (B, H, 128) bf16");
  const int64_t B = q.size(0), H = q.size(1);
  TORCH_CHECK(H % kHeads == 0, "heads must be a multiple of 4");
  TORCH_CHECK(k_win.is_contiguous() && v_win.is_contiguous() && k_win.scalar_type() == at::kBFloat16 &&
                  v_win.scalar_type() == at::kBFloat16 && k_win.size(0) == B && k_win.size(2) == kD &&
                  v_win.sizes() == k_win.sizes(), "window K/V: contiguous (B, W, 128) bf16");
  TORCH_CHECK(pos.scalar_type() == at::kLong && pos.numel() == 1, "pos: int64 scalar");
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == at::kBFloat16 && out.numel() == q.numel(), "out");
  DecodeArgs a{};
  a.q = bf16_ptr(q);
  a.kw = bf16_ptr(k_win);
  a.vw = bf16_ptr(v_win);
  a.pos = pos.data_ptr<int64_t>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.H = static_cast<int>(H);
  a.W = static_cast<int>(k_win.size(1));
  a.scale = static_cast<float>(scale);
  a.softcap = static_cast<float>(softcap);
  a.eps = static_cast<float>(eps);
  a.mode = static_cast<int>(mode);
  if (sink_sw.has_value()) {
    TORCH_CHECK(sink_sw->scalar_type() == at::kFloat && sink_sw->numel() == H && sink_sw->is_contiguous(), "sink");
    a.sink_sw = sink_sw->data_ptr<float>();
  }
  if (mode != 0) {
    TORCH_CHECK(comp.has_value() && norm_w.has_value(), "compressed entries and norm weight required");
    TORCH_CHECK(comp->is_contiguous() && comp->scalar_type() == at::kBFloat16 && comp->size(0) == B &&
                    comp->size(2) == kD, "entries: contiguous (B, n, 128) bf16");
    TORCH_CHECK(norm_w->scalar_type() == at::kFloat && norm_w->numel() == kD && norm_w->is_contiguous(), "norm w");
    a.comp = bf16_ptr(*comp);
    a.n = static_cast<int>(comp->size(1));
    a.norm_w = norm_w->data_ptr<float>();
    a.m = static_cast<int>(m);
    if (sink_c.has_value()) {
      TORCH_CHECK(sink_c->scalar_type() == at::kFloat && sink_c->numel() == H && sink_c->is_contiguous(), "sink");
      a.sink_c = sink_c->data_ptr<float>();
    }
    if (mode == 2) {
      TORCH_CHECK(top.has_value() && top->scalar_type() == at::kLong && top->is_contiguous() && top->size(0) == B,
                  "top: contiguous (B, k) int64");
      a.top = top->data_ptr<int64_t>();
      a.ktop = static_cast<int>(top->numel() / B);
    } else {
      TORCH_CHECK(m > 0, "compression rate");
    }
  }
  if (B == 0) return;
  const int lmax = std::max(a.W, mode == 2 ? a.ktop : a.n);
  const size_t smem = static_cast<size_t>(lmax) * 5 * sizeof(float);
  TORCH_CHECK(smem <= 200 * 1024, "too many keys for one CTA");
  c10::cuda::CUDAGuard guard(q.device());
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(decode_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  decode_attn_kernel<<<dim3(static_cast<unsigned>(B), static_cast<unsigned>(H / kHeads)), kThreads, smem,
                       at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Paged decode attention (see PagedArgs).  q (B, H, 128); k_pool / v_pool (pages, page_rows, 128);
// k_table (B, kmaxp) int32; k_len (B) int32; max_rows: the longest branch any sequence may
// attend to (sizes shared memory; longer branches are cut to it, which the caller avoids).
void decode_attention_paged(torch::Tensor q, torch::Tensor k_pool, torch::Tensor v_pool, torch::Tensor k_table,
                            torch::Tensor k_len, int64_t window, c10::optional<torch::Tensor> sink_sw, double softcap,
                            int64_t mode, c10::optional<torch::Tensor> e_pool, c10::optional<torch::Tensor> e_table,
                            c10::optional<torch::Tensor> e_len, c10::optional<torch::Tensor> norm_w, double eps,
                            int64_t m, c10::optional<torch::Tensor> top, c10::optional<torch::Tensor> sink_c,
                            double scale, int64_t max_rows, torch::Tensor out, torch::Tensor err) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.dim() == 3 && q.size(2) == kD,
              "q: contiguous (B, H, 128) bf16");
  const int64_t B = q.size(0), H = q.size(1);
  TORCH_CHECK(H % kHeads == 0, "heads must be a multiple of 4");
  TORCH_CHECK(k_pool.is_contiguous() && v_pool.sizes() == k_pool.sizes() && v_pool.is_contiguous() &&
                  k_pool.dim() == 3 && k_pool.size(2) == kD && k_pool.scalar_type() == at::kBFloat16 &&
                  v_pool.scalar_type() == at::kBFloat16, "K / V pools: contiguous (pages, rows, 128) bf16");
  TORCH_CHECK(k_table.scalar_type() == at::kInt && k_table.is_contiguous() && k_table.dim() == 2 &&
                  k_table.size(0) == B, "k_table: (B, pages) int32");
  TORCH_CHECK(k_len.scalar_type() == at::kInt && k_len.numel() == B, "k_len: (B) int32");
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == at::kBFloat16 && out.numel() == q.numel(), "out");
  TORCH_CHECK(max_rows > 0, "max_rows");
  PagedArgs a{};
  a.q = bf16_ptr(q);
  a.kpool = bf16_ptr(k_pool);
  a.vpool = bf16_ptr(v_pool);
  a.ktab = k_table.data_ptr<int>();
  a.klen = k_len.data_ptr<int>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.H = static_cast<int>(H);
  a.page_rows = static_cast<int>(k_pool.size(1));
  a.kmaxp = static_cast<int>(k_table.size(1));
  a.n_pages_k = static_cast<int>(k_pool.size(0));
  a.window = static_cast<int>(window);
  a.scale = static_cast<float>(scale);
  a.softcap = static_cast<float>(softcap);
  a.eps = static_cast<float>(eps);
  a.mode = static_cast<int>(mode);
  a.err = err.data_ptr<int>();
  if (sink_sw.has_value()) {
    TORCH_CHECK(sink_sw->scalar_type() == at::kFloat && sink_sw->numel() == H && sink_sw->is_contiguous(), "sink");
    a.sink_sw = sink_sw->data_ptr<float>();
  }
  int lmax = static_cast<int>(max_rows);
  if (mode != 0) {
    TORCH_CHECK(e_pool.has_value() && e_table.has_value() && e_len.has_value() && norm_w.has_value(),
                "entry pool, table, lengths and norm weight required");
    TORCH_CHECK(e_pool->is_contiguous() && e_pool->scalar_type() == at::kBFloat16 && e_pool->dim() == 3 &&
                    e_pool->size(1) == k_pool.size(1) && e_pool->size(2) == kD, "entry pool: (pages, rows, 128) bf16");
    TORCH_CHECK(e_table->scalar_type() == at::kInt && e_table->is_contiguous() && e_table->size(0) == B, "e_table");
    TORCH_CHECK(e_len->scalar_type() == at::kInt && e_len->numel() == B, "e_len");
    TORCH_CHECK(norm_w->scalar_type() == at::kFloat && norm_w->numel() == kD && norm_w->is_contiguous(), "norm w");
    a.epool = bf16_ptr(*e_pool);
    a.etab = e_table->data_ptr<int>();
    a.elen = e_len->data_ptr<int>();
    a.emaxp = static_cast<int>(e_table->size(1));
    a.n_pages_e = static_cast<int>(e_pool->size(0));
    a.norm_w = norm_w->data_ptr<float>();
    a.m = static_cast<int>(m);
    if (sink_c.has_value()) {
      TORCH_CHECK(sink_c->scalar_type() == at::kFloat && sink_c->numel() == H && sink_c->is_contiguous(), "sink");
      a.sink_c = sink_c->data_ptr<float>();
    }
    if (mode == 2) {
      TORCH_CHECK(top.has_value() && top->scalar_type() == at::kLong && top->is_contiguous() && top->size(0) == B,
                  "top: contiguous (B, k) int64");
      a.top = top->data_ptr<int64_t>();
      a.ktop = static_cast<int>(top->numel() / std::max<int64_t>(B, 1));
      lmax = std::max(lmax, a.ktop);
    } else {
      TORCH_CHECK(m > 0, "compression rate");
    }
  }
  a.lmax = lmax;
  if (B == 0) return;
  const size_t smem = static_cast<size_t>(lmax) * 5 * sizeof(float);
  TORCH_CHECK(smem <= 200 * 1024, "too many keys for one CTA");
  c10::cuda::CUDAGuard guard(q.device());
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(decode_attn_paged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
  decode_attn_paged_kernel<<<dim3(static_cast<unsigned>(B), static_cast<unsigned>(H / kHeads)), kThreads, smem,
                             at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Window branch of paged decode split over `splits` CTAs per (sequence, 4 heads): partial
// (m, l, o) into pm / pl (splits, B, H) and po (splits, B, H, 128), fp32.
void decode_window_split(torch::Tensor q, torch::Tensor k_pool, torch::Tensor v_pool, torch::Tensor k_table,
                         torch::Tensor k_len, int64_t window, double softcap, double scale, int64_t splits,
                         int64_t max_rows, torch::Tensor pm, torch::Tensor pl, torch::Tensor po, torch::Tensor err) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.dim() == 3 && q.size(2) == kD, "q");
  const int64_t B = q.size(0), H = q.size(1);
  TORCH_CHECK(H % kHeads == 0 && splits >= 1 && max_rows > 0, "heads % 4, splits >= 1, max_rows > 0");
  TORCH_CHECK(k_pool.is_contiguous() && v_pool.sizes() == k_pool.sizes() && v_pool.is_contiguous() &&
                  k_pool.dim() == 3 && k_pool.size(2) == kD, "pools");
  TORCH_CHECK(k_table.scalar_type() == at::kInt && k_table.is_contiguous() && k_table.size(0) == B, "k_table");
  TORCH_CHECK(k_len.scalar_type() == at::kInt && k_len.numel() == B, "k_len");
  TORCH_CHECK(pm.numel() == splits * B * H && pl.numel() == pm.numel() && po.numel() == pm.numel() * kD &&
                  pm.scalar_type() == at::kFloat && po.is_contiguous(), "partials");
  PagedArgs a{};
  a.q = bf16_ptr(q);
  a.kpool = bf16_ptr(k_pool);
  a.vpool = bf16_ptr(v_pool);
  a.ktab = k_table.data_ptr<int>();
  a.klen = k_len.data_ptr<int>();
  a.H = static_cast<int>(H);
  a.page_rows = static_cast<int>(k_pool.size(1));
  a.kmaxp = static_cast<int>(k_table.size(1));
  a.n_pages_k = static_cast<int>(k_pool.size(0));
  a.window = static_cast<int>(window);
  a.scale = static_cast<float>(scale);
  a.softcap = static_cast<float>(softcap);
  a.err = err.data_ptr<int>();
  if (B == 0) return;
  const int chunk = static_cast<int>((max_rows + splits - 1) / splits);
  const size_t smem = static_cast<size_t>(std::max(chunk, 1)) * 4 * sizeof(float);
  TORCH_CHECK(smem <= 200 * 1024, "too many rows per split");
  c10::cuda::CUDAGuard guard(q.device());
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(decode_window_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
  decode_window_split_kernel<<<dim3(static_cast<unsigned>(B), static_cast<unsigned>(H / kHeads),
                                    static_cast<unsigned>(splits)),
                               kThreads, smem, at::cuda::getCurrentCUDAStream()>>>(a, static_cast<int>(splits),
                                                                                   pm.data_ptr<float>(),
                                                                                   pl.data_ptr<float>(),
                                                                                   po.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Log-sum-exp merge of S partials: m, l (S, R), o (S, R, D) fp32 -> out (R, D) fp32 (and the
// merged m, l when given).  extra: optional logit per row (row r uses extra[r % extra.numel()]).
void lse_merge(torch::Tensor m, torch::Tensor l, torch::Tensor o, c10::optional<torch::Tensor> extra,
               torch::Tensor out, c10::optional<torch::Tensor> out_m, c10::optional<torch::Tensor> out_l) {
  TORCH_CHECK(m.scalar_type() == at::kFloat && l.scalar_type() == at::kFloat && o.scalar_type() == at::kFloat &&
                  out.scalar_type() == at::kFloat, "fp32 partials and output");
  TORCH_CHECK(m.is_contiguous() && l.is_contiguous() && o.is_contiguous() && out.is_contiguous() && m.dim() == 2 &&
                  l.sizes() == m.sizes() && o.dim() == 3 && o.size(0) == m.size(0) && o.size(1) == m.size(1),
              "m, l (S, R); o (S, R, D)");
  const int64_t S = m.size(0), R = m.size(1), D = o.size(2);
  TORCH_CHECK(out.numel() == R * D, "out (R, D)");
  const float* ex = nullptr;
  int64_t ex_mod = 1;
  if (extra.has_value()) {
    TORCH_CHECK(extra->scalar_type() == at::kFloat && extra->is_contiguous() && extra->numel() > 0, "extra");
    ex = extra->data_ptr<float>();
    ex_mod = extra->numel();
  }
  float* om = nullptr;
  float* ol = nullptr;
  if (out_m.has_value()) {
    TORCH_CHECK(out_l.has_value() && out_m->numel() == R && out_l->numel() == R, "out_m / out_l (R)");
    om = out_m->data_ptr<float>();
    ol = out_l->data_ptr<float>();
  }
  const int64_t total = R * D;
  if (total == 0) return;
  c10::cuda::CUDAGuard guard(m.device());
  lse_merge_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      m.data_ptr<float>(), l.data_ptr<float>(), o.data_ptr<float>(), static_cast<int>(S), R, static_cast<int>(D),
      ex, ex_mod, out.data_ptr<float>(), om, ol);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sv4
