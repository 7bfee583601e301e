// GEMM dispatch between the kernels of this library.
#include "gemm.h"
#include "kernels.h"

namespace le {

cudaError_t launch_gemm(const GemmW& W, const __half* A, long lda, const EpiParams& ep, DevStatus* status,
                        cudaStream_t s) {
  // The tensor-core kernels write through TMA: output rows 16-byte aligned.
  const bool tma_ok = ep.mode == EPI_F32 ? ep.ldo % 4 == 0 : ep.ldo % 8 == 0;
  // F32 weights exist only as fp16 operands: the TMA kernel at every M.
  if (W.qf == QF_F16) {
    if (!W.w16 || W.n_virtual % (2 * TILE_N) || !tma_ok) return cudaErrorInvalidValue;
    return launch_gemm_f16(W.w16, W.n_virtual, W.K, A, lda, ep, status, s);
  }
  if (ep.M >= TC_MIN_M && W.n_virtual % (2 * TILE_N) == 0 && tma_ok) {
    if (ep.M >= TC_F16_MIN_M && W.w16) return launch_gemm_f16(W.w16, W.n_virtual, W.K, A, lda, ep, status, s);
    return launch_gemm_tc2(W.qf, W.t128, W.n_virtual, W.K, A, lda, ep, status, s);
  }
  if (W.r16) return launch_gemm_r16(W.qf, W.r16, W.r16_tiles, W.K, A, lda, ep, s);
  return cudaErrorInvalidValue;
}

const char* gemm_variant_name() {
  return "tcgen05 cta_group::2 kind::f16 256x256 CTA-pair tiles: fp16 weights via TMA (M>=256), in-smem dequant "
         "(64<=M<256); mma.sync m16n8k16 row16 tiles on the quantised bytes (M<64)";
}

}  // namespace le
