// Host-side launchers of the device kernels (all asynchronous on `s`).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "epilogue.cuh"

namespace le {

// weights.cu
cudaError_t launch_repack(int type, const uint8_t* src0, const uint8_t* src1, long src_row_bytes, int N_src, int K,
                          int n_tiles, int interleave, uint8_t* dst, cudaStream_t s);
cudaError_t launch_dequant_tiles(int qf, const uint8_t* w, int n_rows, int K, int mode, float* out, cudaStream_t s);
cudaError_t launch_gguf_rows(int type, const uint8_t* src, long row_bytes, int n_rows, int K, float* out, cudaStream_t s);
cudaError_t launch_expand_f16(int qf, const uint8_t* w, int n_rows, int K, __half* out, cudaStream_t s);

// elementwise.cu
cudaError_t launch_embed_ln(const int32_t* ids, int emb_type, const uint8_t* emb, long emb_row_bytes, int vocab,
                            const float* type0, const float* w, const float* b, float eps, int T, int H, float* out32,
                            __half* out16, DevStatus* status, cudaStream_t s);
cudaError_t launch_ln_add(const float* in, const float* add, const float* w, const float* b, float eps, int T, int H,
                          float* out32, __half* out16, cudaStream_t s);
cudaError_t launch_pool(const float* h, const int32_t* offsets, int nseq, int H, int out_dim, float* out,
                        cudaStream_t s);
cudaError_t launch_f32_to_f16(const float* in, long n, __half* out, cudaStream_t s);
cudaError_t launch_positions(const int32_t* offsets, int nseq, int32_t* pos, cudaStream_t s);

// attention.cu
cudaError_t launch_attention(const __half* qkv, const int32_t* offsets, int nseq, int max_len, int H, int heads,
                             int head_dim, __half* out, cudaStream_t s);

// gemm_simt.cu
cudaError_t launch_gemm_simt(int qf, const uint8_t* W, int n_virtual, int K, const __half* A, long lda,
                             const EpiParams& ep, cudaStream_t s);

// gemm_tc2.cu
cudaError_t launch_gemm_tc2(int qf, const uint8_t* W, int n_virtual, int K, const __half* A, long lda,
                            const EpiParams& ep, DevStatus* status, cudaStream_t s);

// gemm_f16.cu
cudaError_t launch_gemm_f16(const __half* W16, int n_virtual, int K, const __half* A, long lda, const EpiParams& ep,
                            DevStatus* status, cudaStream_t s);

}  // namespace le
