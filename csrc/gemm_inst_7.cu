// Explicit instantiations of the tcgen05 GEMM kernel (split across files for parallel builds).
#include "gemm.cuh"

namespace sv4 {

template <int BN, bool A_MN, bool B_MN, int BMODE, int EPI>
static void launch_one(const CUtensorMap& ma, const CUtensorMap& mb0, const CUtensorMap& mb1, const CUtensorMap& md,
                       const CUtensorMap& mx, const GemmParams& p, int grid, cudaStream_t stream) {
  auto kern = gemm_bf16_kernel<BN, A_MN, B_MN, BMODE, EPI>;
  constexpr int smem = GemmSmem<BN>::kTotal;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  kern<<<grid, 192, smem, stream>>>(ma, mb0, mb1, md, mx, p);
}

bool gemm_launch_group7(int variant, const CUtensorMap& ma, const CUtensorMap& mb0, const CUtensorMap& mb1,
                         const CUtensorMap& md, const CUtensorMap& mx, const GemmParams& p, int grid,
                         cudaStream_t stream) {
  switch (variant) {
    case 15: launch_one<256, false, false, kBSingle, kEpiAxpbyBF16>(ma, mb0, mb1, md, mx, p, grid, stream); return true;
    case 16: launch_one<256, false, true, kBSingle, kEpiAxpbyBF16>(ma, mb0, mb1, md, mx, p, grid, stream); return true;
    case 17: launch_one<256, false, false, kBSingle, kEpiPeerBF16>(ma, mb0, mb1, md, mx, p, grid, stream); return true;
    default: return false;
  }
}

}  // namespace sv4
