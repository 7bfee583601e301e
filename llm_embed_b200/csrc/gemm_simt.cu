// Weight-streaming quantised GEMM on CUDA cores, for few tokens.
//
// out[m][n] = sum_k A[m][k] * W[n][k] with W in the tile-blocked quantised
// layout, dequantised in registers to the same fp16 operand values the
// tensor-core GEMM uses, A in fp16, float32 accumulation.  One warp owns one
// pair of output rows (see epilogue.cuh), streams their quant bytes once per
// 8-token chunk, and applies the epilogue.  Each output's accumulation order
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

template <int QF>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const uint8_t* __restrict__ W, int n_pairs, int K,
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
  const int ngroups = K / 8;
  for (int m0 = 0; m0 < ep.M; m0 += MT) {
    float acca[MT], accb[MT];
#pragma unroll
    for (int i = 0; i < MT; i++) acca[i] = accb[i] = 0.f;
    for (int j = lane; j < ngroups; j += 32) {
      const int ks = j >> 3, g = j & 7;
      const uint8_t* ca = ta + ks * cb;
      const uint8_t* cbp = tb + ks * cb;
      float wa[8], wb[8];
      h8_to_f32(dq8_f16<QF>(*reinterpret_cast<const uint2*>(ca + ia * TILE_K + g * 8), ca + TILE_Q_BYTES, ia, g), wa);
      h8_to_f32(dq8_f16<QF>(*reinterpret_cast<const uint2*>(cbp + ib * TILE_K + g * 8), cbp + TILE_Q_BYTES, ib, g), wb);
#pragma unroll
      for (int mm = 0; mm < MT; mm++) {
        if (m0 + mm < ep.M) {
          float x[8];
          h8_to_f32(*reinterpret_cast<const uint4*>(A + (long)(m0 + mm) * lda + j * 8), x);
#pragma unroll
          for (int i = 0; i < 8; i++) {
            acca[mm] = fmaf(wa[i], x[i], acca[mm]);
            accb[mm] = fmaf(wb[i], x[i], accb[mm]);
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
  const int n_pairs = n_virtual / 2;
  const unsigned grid = (unsigned)((n_pairs + 7) / 8);
  switch (qf) {
    case QF_Q8_0: gemm_simt_kernel<QF_Q8_0><<<grid, 256, 0, s>>>(W, n_pairs, K, A, lda, ep); break;
    case QF_KMIN: gemm_simt_kernel<QF_KMIN><<<grid, 256, 0, s>>>(W, n_pairs, K, A, lda, ep); break;
    case QF_Q6K: gemm_simt_kernel<QF_Q6K><<<grid, 256, 0, s>>>(W, n_pairs, K, A, lda, ep); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace le
