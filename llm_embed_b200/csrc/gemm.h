// GEMM dispatch: y = A . W^T with a fused epilogue (epilogue.cuh).
#pragma once
#include "common.cuh"
#include "epilogue.cuh"

namespace le {

// W: tile-blocked quantised weight (format qf) with n_virtual rows and K
// columns; W16: the same weight's fp16 operand values [n_virtual][K] (or
// null); A: fp16 activations [ep.M][K] with leading dimension lda.
// Token counts below TC_MIN_M stream the quantised weights on CUDA cores
// (gemm_simt.cu); up to TC_F16_MIN_M the tcgen05 CTA-pair kernel dequantises
// them in shared memory (gemm_tc2.cu), where weight bytes still matter;
// larger ones run the tcgen05 CTA-pair kernel on W16 (gemm_f16.cu).  The two
// tensor-core kernels compute bit-identical results.
constexpr int TC_MIN_M = 64;
constexpr int TC_F16_MIN_M = 256;
cudaError_t launch_gemm(int qf, const uint8_t* W, const __half* W16, int n_virtual, int K, const __half* A, long lda,
                        const EpiParams& ep, DevStatus* status, cudaStream_t s);

// Name of the kernel family used for large token counts.
const char* gemm_variant_name();

}  // namespace le
