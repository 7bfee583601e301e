// Weight-streaming quantised GEMM on CUDA cores, for few tokens.
//
// out[m][n] = sum_k A[m][k] * W[n][k] with W in the tile-blocked quantised
// layout, dequantised in registers to the same fp16 operand values the
// tensor-core GEMM uses, A in fp16, float32 accumulation.  One warp owns one
// pair of output rows (see epilogue.cuh), holds their quant bytes in
// registers, runs over the tokens in chunks of 8 and applies the epilogue.  Each output's accumulation order
// depends only on K, never on M, so a sequence's result does not depend on
// the other sequences in the call.
#include "dequant.cuh"
#include "epilogue.cuh"
#include "kernels.h"

namespace le {

namespace {

constexpr int MT = 8;  // tokens per pass

__device__ __forceinline__ void h8_to_f32(uint4 h, float* f) {
  const __half2* p = reinterpret_cast<const __half2*>(&h);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float2 v = __half22float2(p[i]);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace

// Each lane owns 16-weight chunks c = lane + 32 i of both rows (chunk c is
// bytes (c % 4) * 16 .. +15 of the row's 64 bytes in k-step c / 4) and
// issues all of their loads before any use, so a warp has its rows' whole
// weight stream in flight at once (the latency of one DRAM round trip, not
// one per k-step).  K <= 32 * 16 * MAXCH.
constexpr int MAXCH = 6;  // K <= 3072

template <int QF>
__global__ void __launch_bounds__(128) gemm_simt_kernel(const uint8_t* __restrict__ W, int n_pairs, int K,
                                                        const __half* __restrict__ A, long lda, EpiParams ep) {
  const int pair = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (pair >= n_pairs) return;
  int ra, rb;
  pair_rows(ep.mode, pair, &ra, &rb);
  const int ksteps = K / TILE_K;
  const long cb = chunk_bytes(QF);
  const uint8_t* ta = W + (long)(ra / TILE_N) * ksteps * cb;
  const uint8_t* tb = W + (long)(rb / TILE_N) * ksteps * cb;
  const int ia = ra % TILE_N, ib = rb % TILE_N;
  const int nch = K / 16;
  uint4 qa[MAXCH], qb[MAXCH];
#pragma unroll
  for (int i = 0; i < MAXCH; i++) {
    const int c = lane + 32 * i;
    if (c < nch) {
      const long off = (long)(c >> 2) * cb;
      qa[i] = __ldg(reinterpret_cast<const uint4*>(ta + off + ia * TILE_K + (c & 3) * 16));
      qb[i] = __ldg(reinterpret_cast<const uint4*>(tb + off + ib * TILE_K + (c & 3) * 16));
    }
  }
  // fp16 operand values of the lane's chunks: [chunk][8-weight half].
  uint4 wha[MAXCH][2], whb[MAXCH][2];
#pragma unroll
  for (int i = 0; i < MAXCH; i++) {
    const int c = lane + 32 * i;
    if (c < nch) {
      const uint8_t* ma = ta + (long)(c >> 2) * cb + TILE_Q_BYTES;
      const uint8_t* mb = tb + (long)(c >> 2) * cb + TILE_Q_BYTES;
      const int g = (c & 3) * 2;
      wha[i][0] = dq8_f16<QF>(make_uint2(qa[i].x, qa[i].y), ma, ia, g);
      wha[i][1] = dq8_f16<QF>(make_uint2(qa[i].z, qa[i].w), ma, ia, g + 1);
      whb[i][0] = dq8_f16<QF>(make_uint2(qb[i].x, qb[i].y), mb, ib, g);
      whb[i][1] = dq8_f16<QF>(make_uint2(qb[i].z, qb[i].w), mb, ib, g + 1);
    }
  }
  for (int m0 = 0; m0 < ep.M; m0 += MT) {
    float acca[MT], accb[MT];
#pragma unroll
    for (int i = 0; i < MT; i++) acca[i] = accb[i] = 0.f;
#pragma unroll
    for (int i = 0; i < MAXCH; i++) {
      const int c = lane + 32 * i;
      if (c < nch) {
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
          float wa[8], wb[8];
          h8_to_f32(wha[i][hh], wa);
          h8_to_f32(whb[i][hh], wb);
#pragma unroll
          for (int mm = 0; mm < MT; mm++) {
            if (m0 + mm < ep.M) {
              float x[8];
              h8_to_f32(*reinterpret_cast<const uint4*>(A + (long)(m0 + mm) * lda + c * 16 + hh * 8), x);
#pragma unroll
              for (int e = 0; e < 8; e++) {
                acca[mm] = fmaf(wa[e], x[e], acca[mm]);
                accb[mm] = fmaf(wb[e], x[e], accb[mm]);
              }
            }
          }
        }
      }
    }
#pragma unroll
    for (int mm = 0; mm < MT; mm++) {
      const float va = warp_allsum(acca[mm]);
      const float vb = warp_allsum(accb[mm]);
      if (lane == mm && m0 + mm < ep.M) epi_pair(ep, m0 + mm, ra, va, vb);
    }
  }
}

cudaError_t launch_gemm_simt(int qf, const uint8_t* W, int n_virtual, int K, const __half* A, long lda,
                             const EpiParams& ep, cudaStream_t s) {
  if (ep.M == 0) return cudaSuccess;
  if (K % TILE_K || K > 32 * 16 * MAXCH || (lda * 2) % 16 || (reinterpret_cast<uintptr_t>(A) & 15))
    return cudaErrorInvalidValue;
  const int n_pairs = n_virtual / 2;
  const unsigned grid = (unsigned)((n_pairs + 3) / 4);
  switch (qf) {
    case QF_Q8_0: gemm_simt_kernel<QF_Q8_0><<<grid, 128, 0, s>>>(W, n_pairs, K, A, lda, ep); break;
    case QF_KMIN: gemm_simt_kernel<QF_KMIN><<<grid, 128, 0, s>>>(W, n_pairs, K, A, lda, ep); break;
    case QF_Q6K: gemm_simt_kernel<QF_Q6K><<<grid, 128, 0, s>>>(W, n_pairs, K, A, lda, ep); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace le
