// Host side of the tcgen05 GEMM: TMA tensor-map construction, kernel instantiations,
// launch helpers and the device-side builder of grouped (MoE) problem tables.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "gemm.cuh"

namespace sv4 {

static bool host_trace() {
  static const bool on = [] {
    const char* e = getenv("SV4_TRACE_HOST");
    return e != nullptr && e[0] == '1';
  }();
  return on;
}
#define SV4_TRACE(...)                      \
  do {                                      \
    if (host_trace()) {                     \
      fprintf(stderr, "[sv4] " __VA_ARGS__); \
      fprintf(stderr, "\n");                \
      fflush(stderr);                       \
    }                                       \
  } while (0)

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p != nullptr,
                "cuTensorMapEncodeTiled is unavailable");
    fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

// cuTensorMapEncodeTiled is a driver call that needs a current context in the calling
// thread.  Autograd runs backward passes on its own device threads, where no runtime call
// may have made the primary context current yet (a device guard does not), so every
// encode first makes the current device's primary context current in this thread.
static void ensure_context() {
  static thread_local int ready = -1;
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev != ready) {
    C10_CUDA_CHECK(cudaSetDevice(dev));
    ready = dev;
  }
}

static CUtensorMap* encode_scratch() {
  ensure_context();
  alignas(128) static thread_local CUtensorMap scratch;
  return &scratch;
}

// 3-D tiled map: dims/strides given inner-first; strides in bytes for dims 1 and 2.
CUtensorMap make_map_3d(const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t d0, uint64_t d1,
                        uint64_t d2, uint64_t s1_bytes, uint64_t s2_bytes, uint32_t b0, uint32_t b1,
                        CUtensorMapSwizzle swz) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base address must be 16-byte aligned");
  TORCH_CHECK(s1_bytes % 16 == 0 && s2_bytes % 16 == 0, "TMA strides must be multiples of 16 bytes");
  TORCH_CHECK((b0 * elem_bytes) % 16 == 0, "TMA inner box must span a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1_bytes, s2_bytes};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMap* tmp = encode_scratch();
  SV4_TRACE("map3d base=%p d=%llu,%llu,%llu s=%llu,%llu box=%u,%u local=%p scratch=%p", base,
            (unsigned long long)d0, (unsigned long long)d1, (unsigned long long)d2, (unsigned long long)s1_bytes,
            (unsigned long long)s2_bytes, b0, b1, (void*)&m, (void*)tmp);
  CUresult r = encode_fn()(tmp, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", int(r));
  memcpy(&m, tmp, sizeof(CUtensorMap));
  return m;
}

// Generic tiled map (rank 2..5): dims inner-first, strides in bytes for dims 1..rank-1.
CUtensorMap make_map_nd(const void* base, CUtensorMapDataType dt, int rank, const uint64_t* dims,
                        const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swz) {
  TORCH_CHECK(rank >= 2 && rank <= 5, "tensor map rank");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base address must be 16-byte aligned");
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) {
    TORCH_CHECK(strides_bytes[i] % 16 == 0, "TMA strides must be multiples of 16 bytes");
    st[i] = strides_bytes[i];
  }
  CUtensorMap m;
  CUtensorMap* tmp = encode_scratch();
  CUresult r = encode_fn()(tmp, dt, rank, const_cast<void*>(base), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", int(r));
  memcpy(&m, tmp, sizeof(CUtensorMap));
  return m;
}

// An operand view as (batch, outer, inner) with unit inner stride.
struct OperandView {
  const void* ptr;
  int64_t inner, outer, batch;
  int64_t outer_stride, batch_stride;  // elements
};

static OperandView view_of(const torch::Tensor& t) {
  TORCH_CHECK(t.dim() == 2 || t.dim() == 3, "operand must be 2-D or 3-D");
  TORCH_CHECK(t.stride(-1) == 1, "operand needs a unit-stride innermost dimension");
  OperandView v;
  v.ptr = t.data_ptr();
  v.inner = t.size(-1);
  v.outer = t.size(-2);
  v.outer_stride = t.stride(-2);
  // A single row's stride is never used to step; give TMA a legal (16-byte multiple) value.
  if (v.outer == 1) v.outer_stride = v.inner + (8 - v.inner % 8) % 8;
  if (t.dim() == 3 && t.size(0) > 1) {
    v.batch = t.size(0);
    v.batch_stride = t.stride(0);
  } else {
    v.batch = 1;
    v.batch_stride = v.outer * v.outer_stride;
  }
  return v;
}

// Box for an operand: K-major rows -> (64 x rows); MN-major -> (64 x 64).
static CUtensorMap map_for(const OperandView& v, uint32_t box_outer) {
  return make_map_3d(v.ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, v.inner, v.outer, v.batch, v.outer_stride * 2,
                     v.batch_stride * 2, 64, box_outer, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Map for writing D with TMA: 3-D (cols, rows, batch), box = 128 bytes x 32 rows, 128B swizzle.
// Returns false (and leaves `m` unset) when the layout cannot be a TMA destination.
static bool map_d_for(const void* base, bool f32, int64_t cols, int64_t rows, int64_t batch, int64_t ld,
                      int64_t bstride, CUtensorMap& m) {
  const int eb = f32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld * eb) % 16 != 0 || cols <= 0 || rows <= 0) return false;
  if (batch > 1 && (bstride * eb) % 16 != 0) return false;
  const int64_t bs = batch > 1 ? bstride : rows * ld;
  m = make_map_3d(base, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, eb, cols, rows,
                  batch, ld * eb, bs * eb, 128 / eb, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  return true;
}

static int num_sms(int dev) {
  static int cached[64] = {0};
  if (cached[dev] == 0) {
    cudaDeviceGetAttribute(&cached[dev], cudaDevAttrMultiProcessorCount, dev);
  }
  return cached[dev];
}

// Kernel instantiations live in gemm_inst_*.cu (compiled in parallel).
void gemm_launch_variant(int variant, const CUtensorMap& ma, const CUtensorMap& mb0, const CUtensorMap& mb1,
                         const CUtensorMap& md, const CUtensorMap& mx, const GemmParams& p, int grid,
                         cudaStream_t stream);

static void dispatch(bool a_mn, bool b_mn, int bmode, int epi, const CUtensorMap& ma, const CUtensorMap& mb0,
                     const CUtensorMap& mb1, const CUtensorMap& md, const GemmParams& p, int grid,
                     cudaStream_t stream, const CUtensorMap* mx = nullptr) {
  struct V { bool a, b; int bm, ep; };
  static const V table[] = {
      {false, false, kBSingle, kEpiBF16},
      {false, false, kBSingle, kEpiF32},
      {false, false, kBSingle, kEpiF32Acc},
      {false, true, kBSingle, kEpiBF16},
      {false, true, kBSingle, kEpiF32},
      {true, true, kBSingle, kEpiF32Acc},
      {true, true, kBSingle, kEpiF32},
      {true, true, kBSingle, kEpiBF16},
      {false, false, kBSplitN, kEpiSwiGLU},
      {false, false, kBSingle, kEpiRowScaleBF16},
      {false, true, kBSplitK, kEpiBF16},
      {true, false, kBSingle, kEpiBF16},
      {true, false, kBSingle, kEpiF32},
      {true, false, kBSingle, kEpiF32Acc},
      {false, true, kBSingle, kEpiF32Acc},
      {false, false, kBSingle, kEpiAxpbyBF16},
      {false, true, kBSingle, kEpiAxpbyBF16},
      {false, false, kBSingle, kEpiPeerBF16},
  };
  for (int i = 0; i < int(sizeof(table) / sizeof(table[0])); ++i) {
    const V& v = table[i];
    if (v.a == a_mn && v.b == b_mn && v.bm == bmode && v.ep == epi) {
      SV4_TRACE("launch variant %d grid %d m=%d n=%d k=%d tma_d=%d", i, grid, p.single.m, p.single.n, p.single.k,
                p.tma_d);
      gemm_launch_variant(i, ma, mb0, mb1, md, mx ? *mx : md, p, grid, stream);
      SV4_TRACE("launched variant %d", i);
      return;
    }
  }
  TORCH_CHECK(false, "unsupported GEMM variant a_mn=", a_mn, " b_mn=", b_mn, " bmode=", bmode, " epi=", epi);
}

// out (M, N) (+)= sum_s part[s] in slice order (fp32 sums; bf16 or fp32 out, any row stride).
__global__ void sum_partials_kernel(const float4* __restrict__ part, int S, int64_t mn4, int64_t n4, void* out,
                                    int64_t ld, int bf16_out, int accumulate) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= mn4) return;
  float4 acc = part[i];
  for (int s = 1; s < S; ++s) {
    const float4 v = part[s * mn4 + i];
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  const int64_t row = i / n4, col = (i % n4) * 4;
  if (bf16_out) {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out) + row * ld + col;
    *reinterpret_cast<__nv_bfloat162*>(o) = __floats2bfloat162_rn(acc.x, acc.y);
    *reinterpret_cast<__nv_bfloat162*>(o + 2) = __floats2bfloat162_rn(acc.z, acc.w);
  } else {
    float* o = reinterpret_cast<float*>(out) + row * ld + col;
    if (accumulate) {
      o[0] += acc.x; o[1] += acc.y; o[2] += acc.z; o[3] += acc.w;
    } else {
      o[0] = acc.x; o[1] = acc.y; o[2] = acc.z; o[3] = acc.w;
    }
  }
}

static void sum_partials(const torch::Tensor& part, torch::Tensor& out, bool accumulate) {
  const int64_t S = part.size(0), M = part.size(1), N = part.size(2);
  const bool bf16 = out.scalar_type() == at::kBFloat16;
  if (N % 4 != 0 || out.stride(1) != 1 || (bf16 && (reinterpret_cast<uintptr_t>(out.data_ptr()) & 3) != 0) ||
      (out.stride(0) % 2 != 0 && bf16)) {
    if (accumulate) out.add_(part.sum(0)); else out.copy_(part.sum(0));
    return;
  }
  const int64_t mn4 = M * N / 4;
  const int threads = 256;
  sum_partials_kernel<<<static_cast<unsigned>((mn4 + threads - 1) / threads), threads, 0,
                        at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const float4*>(part.data_ptr()), static_cast<int>(S), mn4, N / 4, out.data_ptr(),
      out.stride(0), bf16 ? 1 : 0, accumulate ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------ entry points
// Dense / batched:  out[b, m, n] (+)= alpha * sum_k A[b, m, k] B[b, n, k]
//   a: (.., M, K) if !a_mn  else (.., K, M)      (unit inner stride, bf16)
//   b: (.., N, K) if !b_mn  else (.., K, N)
//   out: (.., M, N) bf16 or fp32 with unit inner stride.
void gemm(torch::Tensor a, torch::Tensor b, torch::Tensor out, bool a_mn, bool b_mn, bool accumulate,
          double alpha, torch::Tensor err, bool symmetric) {
  SV4_TRACE("gemm a=%p b=%p out=%p a_mn=%d b_mn=%d", a.data_ptr(), b.data_ptr(), out.data_ptr(), a_mn, b_mn);
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "bf16 operands required");
  TORCH_CHECK(out.stride(-1) == 1, "output needs unit inner stride");
  c10::cuda::CUDAGuard guard(a.device());
  OperandView va = view_of(a), vb = view_of(b);
  const int64_t M = a_mn ? va.inner : va.outer;
  const int64_t K = a_mn ? va.outer : va.inner;
  const int64_t N = b_mn ? vb.inner : vb.outer;
  TORCH_CHECK((b_mn ? vb.outer : vb.inner) == K, "K mismatch");
  TORCH_CHECK(K % 64 == 0, "K must be a multiple of 64");
  const int64_t batch = std::max(va.batch, vb.batch);
  TORCH_CHECK(va.batch == vb.batch, "batch mismatch");
  TORCH_CHECK(out.size(-1) == N && out.size(-2) == M, "output shape mismatch");
  CUtensorMap ma = map_for(va, a_mn ? 64 : 128);
  CUtensorMap mb = map_for(vb, b_mn ? 64 : 256);
  GemmParams p{};
  p.probs = nullptr;
  p.total_tiles = nullptr;
  p.n_probs = 1;
  GemmProblem& s = p.single;
  s.m = M; s.n = N; s.k = K;
  s.a_m = 0; s.a_k = 0; s.a_b = 0;
  s.b_n = 0; s.b_k = 0; s.b_b = 0;
  s.tile_begin = 0;
  s.batch = batch;
  s.d_off = 0;
  s.d_ld = out.stride(-2);
  s.d_bstride = out.dim() == 3 ? out.stride(0) : 0;
  s.aux_off = 0; s.aux_ld = 0;
  p.d = out.data_ptr();
  p.aux = nullptr;
  p.rowscale = nullptr;
  p.alpha = static_cast<float>(alpha);
  p.err = err.data_ptr<int>();
  p.sym = symmetric ? 1 : 0;
  TORCH_CHECK(!symmetric || M == N, "symmetric output must be square");
  int epi;
  if (out.scalar_type() == at::kBFloat16) {
    TORCH_CHECK(!accumulate, "accumulate needs an fp32 output");
    epi = kEpiBF16;
  } else {
    TORCH_CHECK(out.scalar_type() == at::kFloat, "output must be bf16 or fp32");
    epi = accumulate ? kEpiF32Acc : kEpiF32;
  }
  int tiles = batch * ((M + 127) / 128) * ((N + 255) / 256);
  if (tiles == 0) return;
  const int sms = num_sms(a.get_device());
  // Skinny bf16 products (decode: a few dozen token rows against a whole weight matrix) are
  // weight-bandwidth bound but cover only N / 256 tiles: split K over the idle SMs.  The
  // slices run as a batch (A and B viewed as (S, rows, K / S)) into separate fp32 partials
  // that are summed in a fixed order, so the result is deterministic (no reduce-add races).
  if (!symmetric && batch == 1 && !a_mn && !b_mn && M <= 256 && tiles * 4 <= sms && K >= 512 && K % 128 == 0) {
    const int64_t kb = K / 128;
    int64_t S = 1;
    for (int64_t d = std::min<int64_t>(kb, sms / tiles); d >= 2; --d) {
      if (kb % d == 0) { S = d; break; }
    }
    if (S > 1) {
      const int64_t kc = K / S;
      // row strides are stride(-2): a batch-1 operand may arrive as (1, rows, K), whose
      // stride(0) is the batch stride
      auto a3 = a.as_strided({S, M, kc}, {kc, a.stride(-2), 1});
      auto b3 = b.as_strided({S, N, kc}, {kc, b.stride(-2), 1});
      auto part = at::empty({S, M, N}, out.options().dtype(at::kFloat));
      gemm(a3, b3, part, false, false, false, alpha, err, false);
      sum_partials(part, out, epi == kEpiF32Acc);
      return;
    }
  }
  CUtensorMap md = ma;
  p.tma_d = map_d_for(out.data_ptr(), epi != kEpiBF16, N, M, batch, s.d_ld, s.d_bstride, md) ? 1 : 0;
  p.splitk = 1;
  p.kc = static_cast<int>(K);
  // Few output tiles and a long K (weight gradients of small layers, skinny projections):
  // split K across SMs; every slice reduce-adds its partial tile into the fp32 output.
  if (!symmetric && batch == 1 && epi != kEpiBF16 && p.tma_d && tiles * 2 <= sms && K >= 1024) {
    int S = static_cast<int>(std::min<int64_t>(sms / tiles, K / 512));
    if (S > 1) {
      const int64_t kc = ((K + S - 1) / S + 63) / 64 * 64;
      S = static_cast<int>((K + kc - 1) / kc);
      if (S > 1) {
        if (epi == kEpiF32) {
          out.zero_();
          epi = kEpiF32Acc;
        }
        p.splitk = S;
        p.kc = static_cast<int>(kc);
        tiles *= S;
      }
    }
  }
  const int grid = std::min<int>(tiles, sms);
  dispatch(a_mn, b_mn, kBSingle, epi, ma, mb, mb, md, p, grid, at::cuda::getCurrentCUDAStream());
}

// Row-parallel projection whose output tiles also go to the tensor-parallel peers while the
// GEMM runs: out = x w^T (bf16, contiguous (M, N)), and every tile's bf16 values are stored into
// each peer's receive slot (`peer_slots[i]`: the address of this rank's slot on peer i, laid out
// like out) from the epilogue; each CTA then adds 1 to `peer_cnts[i]` (this rank's arrival
// counter on peer i).  Returns the grid, i.e. the arrivals each peer waits for.
int64_t gemm_peer_push(torch::Tensor x, torch::Tensor w, torch::Tensor out, std::vector<int64_t> peer_slots,
                       std::vector<int64_t> peer_cnts, torch::Tensor err) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16, "bf16 operands and output");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && out.dim() == 2 && out.is_contiguous(), "x (M, K), w (N, K), out (M, N)");
  TORCH_CHECK(peer_slots.size() == peer_cnts.size() && peer_slots.size() <= kGemmMaxPeers, "1..7 peers");
  c10::cuda::CUDAGuard guard(x.device());
  OperandView va = view_of(x), vb = view_of(w);
  const int64_t M = va.outer, K = va.inner, N = vb.outer;
  TORCH_CHECK(vb.inner == K && K % 64 == 0, "K mismatch or not a multiple of 64");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N && N % 8 == 0, "out (M, N), N % 8 == 0");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0, "out 16-byte aligned");
  for (auto a : peer_slots) TORCH_CHECK((a & 15) == 0, "peer slots 16-byte aligned");
  GemmParams p{};
  p.n_probs = 1;
  GemmProblem& s = p.single;
  s.m = M; s.n = N; s.k = K;
  s.batch = 1;
  s.d_ld = N;
  p.d = out.data_ptr();
  p.alpha = 1.0f;
  p.err = err.data_ptr<int>();
  p.splitk = 1;
  p.kc = static_cast<int>(K);
  p.n_peers = static_cast<int>(peer_slots.size());
  for (size_t i = 0; i < peer_slots.size(); ++i) {
    p.peer_d[i] = static_cast<unsigned long long>(peer_slots[i]);
    p.peer_cnt[i] = static_cast<unsigned long long>(peer_cnts[i]);
  }
  const int tiles = static_cast<int>(((M + 127) / 128) * ((N + 255) / 256));
  if (tiles == 0) return 0;
  CUtensorMap ma = map_for(va, 128);
  CUtensorMap mb = map_for(vb, 256);
  CUtensorMap md = ma;
  p.tma_d = map_d_for(out.data_ptr(), false, N, M, 1, N, 0, md) ? 1 : 0;
  const int grid = std::min<int>(tiles, num_sms(x.get_device()));
  dispatch(false, false, kBSingle, kEpiPeerBF16, ma, mb, mb, md, p, grid, at::cuda::getCurrentCUDAStream());
  return grid;
}

// out = alpha * (A B^T) + beta * C, bf16 out and bf16 C with identical layout to out
// (batched Newton-Schulz: P = c G G + b G and Y' = P Y + a Y in one pass each).
void gemm_axpby(torch::Tensor a, torch::Tensor b, torch::Tensor c, torch::Tensor out, bool a_mn, bool b_mn,
                double alpha, double beta, torch::Tensor err, bool symmetric) {
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "bf16 operands required");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && c.scalar_type() == at::kBFloat16, "bf16 out / C required");
  TORCH_CHECK(c.sizes() == out.sizes() && c.strides() == out.strides(), "C must be laid out like out");
  c10::cuda::CUDAGuard guard(a.device());
  OperandView va = view_of(a), vb = view_of(b);
  const int64_t M = a_mn ? va.inner : va.outer;
  const int64_t K = a_mn ? va.outer : va.inner;
  const int64_t N = b_mn ? vb.inner : vb.outer;
  TORCH_CHECK((b_mn ? vb.outer : vb.inner) == K && K % 64 == 0, "K mismatch or K % 64");
  TORCH_CHECK(va.batch == vb.batch, "batch mismatch");
  TORCH_CHECK(out.size(-1) == N && out.size(-2) == M, "output shape mismatch");
  CUtensorMap ma = map_for(va, a_mn ? 64 : 128);
  CUtensorMap mb = map_for(vb, b_mn ? 64 : 256);
  GemmParams p{};
  GemmProblem& s = p.single;
  s.m = M; s.n = N; s.k = K; s.batch = va.batch;
  s.d_ld = out.stride(-2);
  s.d_bstride = out.dim() == 3 ? out.stride(0) : 0;
  p.d = out.data_ptr();
  p.aux = c.data_ptr();
  p.alpha = static_cast<float>(alpha);
  p.beta = static_cast<float>(beta);
  p.err = err.data_ptr<int>();
  p.sym = symmetric ? 1 : 0;
  TORCH_CHECK(!symmetric || M == N, "symmetric output must be square");
  const int tiles = va.batch * ((M + 127) / 128) * ((N + 255) / 256);
  if (tiles == 0) return;
  CUtensorMap md = ma;
  p.tma_d = map_d_for(out.data_ptr(), false, N, M, va.batch, s.d_ld, s.d_bstride, md) ? 1 : 0;
  dispatch(a_mn, b_mn, kBSingle, kEpiAxpbyBF16, ma, mb, mb, md, p, std::min<int>(tiles, num_sms(a.get_device())),
           at::cuda::getCurrentCUDAStream());
}

// Grouped GEMM driven by a device-side problem table (MoE).
//   mode 0: SwiGLU fprop    A = x_perm (M_pad, D),    B0/B1 = W_gate/W_up (E, I, D)   -> out act (M_pad, I),
//                                                                                       aux pre (M_pad, 2I)
//   mode 1: down fprop      A = act (M_pad, I),       B = W_down (E, D, I)            -> out (M_pad, D) * rowscale
//   mode 2: down dgrad      A = d_out (M_pad, D),     B = W_down (E, D, I) MN-major   -> out d_act (M_pad, I) bf16
//   mode 3: gate/up dgrad   A = d_pre (M_pad, 2I),    B = [W_gate; W_up] split-K      -> out d_x (M_pad, D) bf16
//   mode 4: wgrad           A = g (M_pad, *) MN-major, B = x (M_pad, *) MN-major      -> out fp32 (+=)
void grouped_gemm(int64_t mode, torch::Tensor a, torch::Tensor b0, torch::Tensor b1, torch::Tensor out,
                  torch::Tensor aux, torch::Tensor rowscale, torch::Tensor probs, torch::Tensor total_tiles,
                  int64_t n_probs, double gate_max, double lin_lo, double lin_hi, int64_t ksplit,
                  bool accumulate, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(a.device());
  OperandView va = view_of(a), vb0 = view_of(b0), vb1 = view_of(b1);
  GemmParams p{};
  p.probs = reinterpret_cast<const GemmProblem*>(probs.data_ptr());
  p.total_tiles = total_tiles.data_ptr<int>();
  p.n_probs = static_cast<int>(n_probs);
  p.single = GemmProblem{};
  p.d = out.data_ptr();
  p.aux = aux.numel() ? aux.data_ptr() : nullptr;
  p.rowscale = rowscale.numel() ? rowscale.data_ptr<float>() : nullptr;
  p.alpha = 1.0f;
  p.gate_max = static_cast<float>(gate_max);
  p.lin_lo = static_cast<float>(lin_lo);
  p.lin_hi = static_cast<float>(lin_hi);
  p.ksplit = static_cast<int>(ksplit);
  p.err = err.data_ptr<int>();
  const int grid = num_sms(a.get_device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  // D as one (rows, cols) row-major buffer; problems address it by row (d_off is a multiple of d_ld).
  CUtensorMap md = map_for(va, 128);  // placeholder when D is not TMA-addressable
  CUtensorMap mx = md;
  if (out.is_contiguous() && out.numel() > 0) {
    const int64_t cols = out.size(-1);
    bool ok = map_d_for(out.data_ptr(), out.scalar_type() == at::kFloat, cols, out.numel() / cols, 1, cols, 0, md);
    if (mode == 0) {  // SwiGLU: pre-activations (rows, 2I) through a second map
      const int64_t ac = aux.size(-1);
      ok = ok && aux.is_contiguous() && map_d_for(aux.data_ptr(), false, ac, aux.numel() / ac, 1, ac, 0, mx);
    }
    p.tma_d = ok ? 1 : 0;
  }
  switch (mode) {
    case 0: {
      CUtensorMap ma = map_for(va, 128), m0 = map_for(vb0, 128), m1 = map_for(vb1, 128);
      dispatch(false, false, kBSplitN, kEpiSwiGLU, ma, m0, m1, md, p, grid, stream, &mx);
      break;
    }
    case 1: {
      CUtensorMap ma = map_for(va, 128), m0 = map_for(vb0, 256);
      dispatch(false, false, kBSingle, p.rowscale ? kEpiRowScaleBF16 : kEpiBF16, ma, m0, m0, md, p, grid, stream);
      break;
    }
    case 2: {
      CUtensorMap ma = map_for(va, 128), m0 = map_for(vb0, 64);
      dispatch(false, true, kBSingle, kEpiBF16, ma, m0, m0, md, p, grid, stream);
      break;
    }
    case 3: {
      CUtensorMap ma = map_for(va, 128), m0 = map_for(vb0, 64), m1 = map_for(vb1, 64);
      dispatch(false, true, kBSplitK, kEpiBF16, ma, m0, m1, md, p, grid, stream);
      break;
    }
    case 4: {
      CUtensorMap ma = map_for(va, 64), m0 = map_for(vb0, 64);
      dispatch(true, true, kBSingle, accumulate ? kEpiF32Acc : kEpiF32, ma, m0, m0, md, p, grid, stream);
      break;
    }
    default:
      TORCH_CHECK(false, "unknown grouped GEMM mode");
  }
}

// Dense fused SwiGLU (shared experts):  pre = [x Wg^T | x Wu^T],  act = silu(min(g,gmax)) * clamp(u)
void swiglu_dense(torch::Tensor x, torch::Tensor wg, torch::Tensor wu, torch::Tensor act, torch::Tensor pre,
                  double gmax, double lo, double hi, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(x.device());
  OperandView vx = view_of(x), vg = view_of(wg), vu = view_of(wu);
  const int64_t M = vx.outer, K = vx.inner, I = vg.outer;
  TORCH_CHECK(K % 64 == 0 && vg.inner == K && vu.inner == K && vu.outer == I, "swiglu_dense shapes");
  CUtensorMap ma = map_for(vx, 128), m0 = map_for(vg, 128), m1 = map_for(vu, 128);
  GemmParams p{};
  p.probs = nullptr;
  GemmProblem& s = p.single;
  s.m = M; s.n = I; s.k = K; s.batch = 1;
  s.d_ld = act.stride(0); s.aux_ld = pre.stride(0);
  p.d = act.data_ptr(); p.aux = pre.data_ptr();
  p.alpha = 1.f; p.gate_max = gmax; p.lin_lo = lo; p.lin_hi = hi;
  p.err = err.data_ptr<int>();
  const int tiles = ((M + 127) / 128) * ((I + 127) / 128);
  if (tiles == 0) return;
  CUtensorMap md = ma, mx = ma;
  p.tma_d = (map_d_for(act.data_ptr(), false, I, M, 1, s.d_ld, 0, md) &&
             map_d_for(pre.data_ptr(), false, 2 * I, M, 1, s.aux_ld, 0, mx)) ? 1 : 0;
  dispatch(false, false, kBSplitN, kEpiSwiGLU, ma, m0, m1, md, p, std::min<int>(tiles, num_sms(x.get_device())),
           at::cuda::getCurrentCUDAStream(), &mx);
}

// dx = dpre[:, :I] Wg + dpre[:, I:] Wu   (B split along K between the two weights)
void swiglu_dense_dgrad(torch::Tensor dpre, torch::Tensor wg, torch::Tensor wu, torch::Tensor dx, torch::Tensor err) {
  c10::cuda::CUDAGuard guard(dpre.device());
  OperandView va = view_of(dpre), vg = view_of(wg), vu = view_of(wu);
  const int64_t M = va.outer, K2 = va.inner, D = vg.inner, I = vg.outer;
  TORCH_CHECK(K2 == 2 * I && I % 64 == 0, "swiglu_dense_dgrad shapes");
  CUtensorMap ma = map_for(va, 128), m0 = map_for(vg, 64), m1 = map_for(vu, 64);
  GemmParams p{};
  p.probs = nullptr;
  GemmProblem& s = p.single;
  s.m = M; s.n = D; s.k = K2; s.batch = 1; s.d_ld = dx.stride(0);
  p.d = dx.data_ptr(); p.alpha = 1.f; p.ksplit = I; p.err = err.data_ptr<int>();
  const int tiles = ((M + 127) / 128) * ((D + 255) / 256);
  if (tiles == 0) return;
  CUtensorMap md = ma;
  p.tma_d = map_d_for(dx.data_ptr(), false, D, M, 1, s.d_ld, 0, md) ? 1 : 0;
  dispatch(false, true, kBSplitK, kEpiBF16, ma, m0, m1, md, p, std::min<int>(tiles, num_sms(dpre.get_device())),
           at::cuda::getCurrentCUDAStream());
}

// ------------------------------------------------------------------------------
// Device-side problem-table builders for the MoE grouped GEMMs.  `seg_start`/`seg_rows`
// (int32, E) describe each expert's row segment in the padded permuted buffer.
__global__ void build_moe_problems_kernel(const int* seg_start, const int* seg_rows, int n_experts, int mode,
                                          int D, int I, int bn_out, GemmProblem* probs, int* total) {
  // one warp: lane l builds the problems of experts l, l + 32, ...; tile ids by a warp scan
  const int lane = threadIdx.x;
  const int reps = (mode == 4) ? 2 : 1;  // wgrad of gate/up: two problems per expert
  const int base_mode = mode >= 6 ? mode - 6 : mode;  // 6 / 7: the FP8 kernel's tiles of modes 0 / 1
  int base = 0;
  for (int e0 = 0; e0 < n_experts; e0 += 32) {
    const int e = e0 + lane;
    GemmProblem pr[2];
    int cnt[2] = {0, 0};
    if (e < n_experts) {
      const int rows = seg_rows[e];
      const int start = seg_start[e];
      for (int r = 0; r < reps; ++r) {
        GemmProblem& q = pr[r];
        q = GemmProblem{};
        q.batch = 1;
        if (base_mode == 0) {         // SwiGLU fprop: m = rows, n = I, k = D
          q.m = rows; q.n = I; q.k = D;
          q.a_m = start; q.b_b = e;
          q.d_off = static_cast<long long>(start) * I; q.d_ld = I;
          q.aux_off = static_cast<long long>(start) * 2 * I; q.aux_ld = 2 * I;
        } else if (base_mode == 1) {  // down fprop: m = rows, n = D, k = I
          q.m = rows; q.n = D; q.k = I;
          q.a_m = start; q.b_b = e;
          q.d_off = static_cast<long long>(start) * D; q.d_ld = D;
          q.aux_off = start;
        } else if (base_mode == 2) {  // down dgrad: m = rows, n = I, k = D
          q.m = rows; q.n = I; q.k = D;
          q.a_m = start; q.b_b = e;
          q.d_off = static_cast<long long>(start) * I; q.d_ld = I;
        } else if (base_mode == 3) {  // gate/up dgrad: m = rows, n = D, k = 2I
          q.m = rows; q.n = D; q.k = 2 * I;
          q.a_m = start; q.b_b = e;
          q.d_off = static_cast<long long>(start) * D; q.d_ld = D;
        } else if (base_mode == 4) {  // gate/up wgrad: dW_{g|u}[e] (I x D) = dpre[:, r*I:(r+1)*I]^T x
          q.m = I; q.n = D; q.k = rows;
          q.a_m = r * I; q.a_k = start; q.b_k = start;
          q.d_off = (static_cast<long long>(r) * n_experts + e) * static_cast<long long>(I) * D; q.d_ld = D;
        } else {                      // mode 5: down wgrad: dWd[e] (D x I) = d_out^T act
          q.m = D; q.n = I; q.k = rows;
          q.a_k = start; q.b_k = start;
          q.d_off = static_cast<long long>(e) * D * I; q.d_ld = I;
        }
        const int tn = (q.n + bn_out - 1) / bn_out;
        const int tm = (q.m + 127) / 128;
        cnt[r] = (q.k == 0 && base_mode < 4) ? 0 : tm * tn;
      }
    }
    const int mine = cnt[0] + cnt[1];
    int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (e < n_experts) {
      int tb = base + incl - mine;
      for (int r = 0; r < reps; ++r) {
        pr[r].tile_begin = tb;
        tb += cnt[r];
        probs[e * reps + r] = pr[r];
      }
    }
    base += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) *total = base;
}

void build_moe_problems(torch::Tensor seg_start, torch::Tensor seg_rows, int64_t mode, int64_t D, int64_t I,
                        torch::Tensor probs, torch::Tensor total) {
  c10::cuda::CUDAGuard guard(seg_start.device());
  const int E = seg_start.numel();
  TORCH_CHECK(mode >= 0 && mode <= 7, "problem-table mode");
  // output columns per tile of the kernel that consumes the table
  const int bn_out = mode == 0 ? 128 : mode == 6 ? 64 : mode == 7 ? 128 : 256;
  build_moe_problems_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      seg_start.data_ptr<int>(), seg_rows.data_ptr<int>(), E, static_cast<int>(mode), static_cast<int>(D),
      static_cast<int>(I), bn_out, reinterpret_cast<GemmProblem*>(probs.data_ptr()), total.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t problem_bytes() { return sizeof(GemmProblem); }

bool gemm_launch_group0(int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                        const CUtensorMap&, const GemmParams&, int, cudaStream_t);
bool gemm_launch_group1(int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                        const CUtensorMap&, const GemmParams&, int, cudaStream_t);
bool gemm_launch_group2(int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                        const CUtensorMap&, const GemmParams&, int, cudaStream_t);
bool gemm_launch_group3(int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                        const CUtensorMap&, const GemmParams&, int, cudaStream_t);
bool gemm_launch_group4(int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                        const CUtensorMap&, const GemmParams&, int, cudaStream_t);
bool gemm_launch_group5(int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                        const CUtensorMap&, const GemmParams&, int, cudaStream_t);
bool gemm_launch_group6(int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                        const CUtensorMap&, const GemmParams&, int, cudaStream_t);
bool gemm_launch_group7(int, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&,
                        const CUtensorMap&, const GemmParams&, int, cudaStream_t);

void gemm_launch_variant(int variant, const CUtensorMap& ma, const CUtensorMap& mb0, const CUtensorMap& mb1,
                         const CUtensorMap& md, const CUtensorMap& mx, const GemmParams& p, int grid,
                         cudaStream_t stream) {
  const bool ok = gemm_launch_group0(variant, ma, mb0, mb1, md, mx, p, grid, stream) ||
                  gemm_launch_group1(variant, ma, mb0, mb1, md, mx, p, grid, stream) ||
                  gemm_launch_group2(variant, ma, mb0, mb1, md, mx, p, grid, stream) ||
                  gemm_launch_group3(variant, ma, mb0, mb1, md, mx, p, grid, stream) ||
                  gemm_launch_group4(variant, ma, mb0, mb1, md, mx, p, grid, stream) ||
                  gemm_launch_group5(variant, ma, mb0, mb1, md, mx, p, grid, stream) ||
                  gemm_launch_group6(variant, ma, mb0, mb1, md, mx, p, grid, stream) ||
                  gemm_launch_group7(variant, ma, mb0, mb1, md, mx, p, grid, stream);
  TORCH_CHECK(ok, "GEMM variant not instantiated");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace sv4
