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
cudaError_t launch_repack_r16(int qf, const uint8_t* t128, int K, int geglu, int tiles, uint8_t* out,
                              cudaStream_t s);
cudaError_t launch_f32_rows_to_f16(const float* src0, const float* src1, int N_src, int K, int n_virt, int interleave,
                                   __half* out, cudaStream_t s);

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

// attention.cu: sequences of at most ATTN_SHORT_MAX tokens (mma.sync tiles)
constexpr int ATTN_SHORT_MAX = 128;
cudaError_t launch_attention(const __half* qkv, const int32_t* offsets, int nseq, int max_len, int H, int heads,
                             int head_dim, __half* out, cudaStream_t s);
// attention_stc.cu: sequences of at most ATTN_SHORT_MAX tokens in large
// batches (persistent tcgen05 kernel over (sequences, head) units).  The
// unit list (attention_units_bytes(cap) bytes, cap >= nseq) is built once
// per forward by launch_attention_units, before the layers.
size_t attention_units_bytes(int cap);
cudaError_t launch_attention_units(const int32_t* offsets, int nseq, int cap, void* buf, cudaStream_t s);
cudaError_t launch_attention_stc(const __half* qkv, const void* units, int cap, int nseq, int T, int H, int heads,
                                 __half* out, DevStatus* status, cudaStream_t s);
// attention_tc.cu: sequences of at least min_len tokens (tcgen05), T = rows of qkv
cudaError_t launch_attention_tc(const __half* qkv, const int32_t* offsets, int nseq, int T, int max_len, int min_len,
                                int H, int heads, __half* out, DevStatus* status, cudaStream_t s);

// gemm_r16.cu: fewer than 64 tokens (row16 weight layout, gemm_r16.cuh)
cudaError_t launch_gemm_r16(int qf, const uint8_t* W, int n_tiles, int K, const __half* A, long lda,
                            const EpiParams& ep, cudaStream_t s);

// gemm_tc2.cu
cudaError_t launch_gemm_tc2(int qf, const uint8_t* W, int n_virtual, int K, const __half* A, long lda,
                            const EpiParams& ep, DevStatus* status, cudaStream_t s);

// forward_small.cu: the whole forward for at most SMALL_MAX_TOKENS tokens in
// one cooperative kernel (nomic-bert shape, quantised weights only).
constexpr int SMALL_HIDDEN = 768;
constexpr int SMALL_FFN = 3072;
constexpr int SMALL_HEADS = 12;
constexpr int SMALL_MAX_TOKENS = 16;
constexpr int SMALL_MAX_LAYERS = 24;

struct SmallGemm {
  const uint8_t* w;  // row16 layout of the weight (gemm_r16.cuh)
  int qf;            // its QFmt
  int K;
  int tiles;         // row16 tiles
  int mode;          // EpiMode of the step
};
struct SmallLayer {
  SmallGemm g[4];  // qkv, attn_output, merged up/gate, down
  const float *attn_w, *attn_b, *out_w, *out_b;
};
struct SmallParams {
  int T, nseq, n_layers;
  const int32_t* ids;
  const int32_t* offsets;
  int emb_type;
  const uint8_t* emb;
  long emb_row_bytes;
  int vocab;
  const float *type0, *embd_w, *embd_b;
  float eps;
  const float *rope_cos, *rope_sin;
  int32_t* pos;   // [T] positions (written)
  __half* qkv;    // [T][3H]
  __half* att;    // [T][H]
  float* y1;      // [T][H] attention-output projection
  __half* ff;     // [T][F]
  float* y2;      // [T][H] down projection
  float* out;     // [nseq][out_dim] pooled, normalised embeddings
  int out_dim;
  unsigned* sync; // small_sync_bytes() of hand-off counters, zeroed by the launch
  DevStatus* status;
  SmallLayer layers[SMALL_MAX_LAYERS];
};
bool small_forward_supported(const SmallParams& p, int hidden, int ffn, int heads, int sms);
size_t small_sync_bytes();
cudaError_t launch_forward_small(const SmallParams& p, cudaStream_t s);

// gemm_ln.cu: projection to 768 columns with the residual add and
// LayerNorm fused: h = LN(h + A . W16^T), h in place, out16 = fp16(h).
// part (gemm_ln_part_bytes, sized for part_rows = gemm_ln_part_rows(M) or
// more) holds the rows' chunk statistics and ctl two counters (16 bytes);
// before the first launch and after any device error part must be all
// 0xFF bytes and ctl zero.
bool gemm_ln_supported(int N, int K);
int gemm_ln_part_rows(int M);
size_t gemm_ln_part_bytes(int M);
cudaError_t launch_gemm_ln(const __half* W16, int K, const __half* A, long lda, int M, float* h, __half* out16,
                           const float* ln_w, const float* ln_b, float eps, unsigned long long* part, int part_rows,
                           unsigned* ctl, DevStatus* status, cudaStream_t s);

// gemm_f16.cu
cudaError_t launch_gemm_f16(const __half* W16, int n_virtual, int K, const __half* A, long lda, const EpiParams& ep,
                            DevStatus* status, cudaStream_t s);

}  // namespace le
