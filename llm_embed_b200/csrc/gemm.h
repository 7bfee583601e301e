// GEMM dispatch: y = A . W^T with a fused epilogue (epilogue.cuh).
#pragma once
#include "common.cuh"
#include "epilogue.cuh"

namespace le {

// W: tile-blocked quantised weight (format qf) with n_virtual rows and K
// columns; A: fp16 activations [ep.M][K] with leading dimension lda.
// Token counts below TC_MIN_M stream the weights on CUDA cores
// (gemm_simt.cu); larger ones use the tcgen05 CTA-pair kernel (gemm_tc2.cu).
constexpr int TC_MIN_M = 64;
cudaError_t launch_gemm(int qf, const uint8_t* W, int n_virtual, int K, const __half* A, long lda, const EpiParams& ep,
                        DevStatus* status, cudaStream_t s);

// Name of the kernel family used for large token counts.
const char* gemm_variant_name();

}  // namespace le
