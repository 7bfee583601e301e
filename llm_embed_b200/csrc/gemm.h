// GEMM dispatch: y = A . W^T with a fused epilogue (epilogue.cuh).
#pragma once
#include "common.cuh"
#include "epilogue.cuh"

namespace le {

// One projection weight in the layouts the GEMM kernels read (any may be
// null when the format has no such copy):
//   t128  tile-blocked quantised weight (common.cuh), n_virtual rows
//   r16   the row16 layout of it (gemm_r16.cuh), r16_tiles tiles
//   w16   fp16 operand values [n_virtual][K]
struct GemmW {
  int qf;
  const uint8_t* t128;
  const uint8_t* r16;
  const __half* w16;
  int n_virtual, r16_tiles, K;
};

// A: fp16 activations [ep.M][K] with leading dimension lda.  Token counts
// below TC_MIN_M run the row16 tensor-core kernel on the quantised bytes
// (gemm_r16.cu); up to TC_F16_MIN_M the tcgen05 CTA-pair kernel dequantises
// the 128-row tiles in shared memory (gemm_tc2.cu), where weight bytes still
// matter; larger ones run the tcgen05 CTA-pair kernel on w16 (gemm_f16.cu).
// The two tcgen05 kernels compute bit-identical results.  F32 weights
// (qf == QF_F16) have only w16 and always take the last kernel.
constexpr int TC_MIN_M = 64;
constexpr int TC_F16_MIN_M = 256;
cudaError_t launch_gemm(const GemmW& W, const __half* A, long lda, const EpiParams& ep, DevStatus* status,
                        cudaStream_t s);

// Name of the kernel family used for large token counts.
const char* gemm_variant_name();

}  // namespace le
