/*
 * TEST INFRASTRUCTURE — NOT PART OF THE PRODUCT.
 *
 * CPU restatement of dbrushchenko/llm-embed's encoder forward path (pure Go +
 * amd64 asm upstream), written from the reference's behaviour.  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference arm
 * may load it, and only as the checker or the timed CPU baseline.  The CUDA
 * product path (llm_embed_b200/) never links or calls anything here.
 *
 * Parity status: dequantisation is pinned bit-exactly by the reference's own
 * known-answer tests (internal/ggml/dot_test.go, dot_q5k_test.go,
 * dot_q6k_test.go), restated in tests/test_oracle_known_answers.py.  The
 * end-to-end forward is "parity unpinned": the reference ships no golden
 * embeddings and no Go toolchain exists here to run it, so the forward pass is
 * pinned only by this restatement of internal/embed/bert.go.
 *
 * All citations are path:line inside the reference project.
 */
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML tensor type ids (internal/gguf/reader.go:46-65). */
enum { OR_F32 = 0, OR_Q8_0 = 8, OR_Q4_K = 12, OR_Q5_K = 13, OR_Q6_K = 14 };

/* GEMM operand-rounding emulation, used to choose the tensor-core precision. */
enum { OR_EMUL_FP32 = 0, OR_EMUL_FP16 = 1, OR_EMUL_BF16 = 2, OR_EMUL_TF32 = 3 };

float or_f16_to_f32(uint16_t h);                                  /* tensor.go:162 */
long  or_row_bytes(int type, long n);                             /* quant_q*.go RowSize */
int   or_dequant(int type, const uint8_t* data, long n, float* out);           /* tensor.go:51 */
int   or_dequant_matrix(int type, const uint8_t* data, int K, int N, float* out); /* gemm.go:221 */

/* ops_simd.go primitives, exposed for unit tests. */
void  or_layernorm(float* x, const float* w, const float* b, float eps, int n); /* ops_simd.go:7 */
void  or_gelu(float* x, int n);                                                /* ops_simd.go:27 */
void  or_softmax(float* x, int n);                                             /* ops_simd.go:46 */
float or_dot_f32(const float* a, const float* b, int n);                       /* ops_simd.go:85 */
void  or_rope_table(int max_seq, int head_dim, float base, float* cos_out, float* sin_out); /* ops_simd.go:107 */

/* GEMM: C[M][N] = A[M][K] . B[N][K]^T with the reference's blocking
 * (gemm_avx512.go:67, KC=128, 6x32 micro-tiles, scalar M edge). */
void or_prepack32(const float* B, int K, int N, float* packed);                 /* gemm_avx512.go:47 */
void or_gemm_prepacked32(const float* A, int M, const float* packed, float* C,
                         int N, int K, int nthreads);
/* Fused dequant.dot batch (ops.go:418 MatMulBatch). */
int  or_matmul_batch(int type, const uint8_t* w, int K, int N, const float* X, int M,
                     float* Y, int nthreads);

/* Whole model. */
typedef struct or_model or_model;
or_model* or_model_load(const char* gguf_path, int emul, char* err, int errlen); /* bert.go:91 + PreDequant */
void  or_model_free(or_model* m);
int   or_model_hparams(const or_model* m, int* out7, float* eps, float* rope_base);
/* Forward (bert.go:216) for one sequence with mask; writes hiddens[L][H]. */
int   or_forward(const or_model* m, const int32_t* ids, const int32_t* mask, int L,
                 float* hiddens, int nthreads);
/* Embed packed sequences: Forward + MeanPool + L2Normalize (+Matryoshka
 * truncation), embedder.go:46-70.  Sequence s is ids[offsets[s]:offsets[s+1]]
 * with an all-ones mask.  out is [nseq][out_dim]. */
int   or_embed_ids(const or_model* m, const int32_t* ids, const int32_t* offsets, int nseq,
                   int out_dim, float* out, int nthreads);
/* Dequantised weight [N][K] of layer `layer`, matrix `which`
 * (0 qkv, 1 attn_output, 2 ffn_up, 3 ffn_gate, 4 ffn_down). */
int   or_model_weight(const or_model* m, int layer, int which, float* out);

#ifdef __cplusplus
}
#endif
