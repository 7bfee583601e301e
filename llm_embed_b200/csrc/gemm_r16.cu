// Quantised GEMM for calls of fewer than 64 tokens: one CTA per 16-row
// weight tile, the tile's K split over 8 warps, tokens in groups of 8 as the
// N of mma.sync m16n8k16 (gemm_r16.cuh).  The weight bytes are the call's
// whole DRAM traffic, read once; each thread streams 8 bytes per weight row
// per unit straight from global memory into its fragment, dequantised in
// registers to the fp16 operand values every GEMM path uses.
#include <mutex>

#include "gemm_r16.cuh"
#include "kernels.h"

namespace le {
namespace {

template <int QF, int NT>
__global__ void __launch_bounds__(256) gemm_r16_kernel(const uint8_t* __restrict__ W, int n_tiles, int K,
                                                       const __half* __restrict__ A, long lda, EpiParams ep) {
  extern __shared__ float4 red[];  // [slices][8 warps][NT][32 lanes]
  const int j = blockIdx.x;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2;
  pdl_wait();
  const int M = ep.M, ns = r16::n_slices(K);
  auto bload = [&](int nt, int k) -> uint4 {
    const int m = 8 * nt + g;
    if (m >= M) return make_uint4(0, 0, 0, 0);
    return __ldg(reinterpret_cast<const uint4*>(A + (long)m * lda + k));
  };
  const uint8_t* tile = W + (long)j * r16::tile_bytes(QF, K);
  auto chunk_at = [&](int c) { return tile + (long)c * r16::chunk_bytes(QF); };
  for (int s = 0; s < ns; s++) {
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
    int u0, u1;
    r16::slice_units(K, s, w, &u0, &u1);
    r16::tile_units<QF, NT>(chunk_at, u0, u1, acc, bload);
    r16::store_partials<NT>(red + s * r16::WARPS * NT * 32, acc);
  }
  __syncthreads();
  pdl_trigger();
  for (int i = threadIdx.x; i < 64 * NT; i += blockDim.x) {
    int q, m;
    float va, vb;
    r16::reduce_item<NT>(red, i, &q, &m, &va, &vb, ns);
    if (m < M) epi_pair(ep, m, r16::pair_virtual_row(ep.mode, j, q), va, vb);
  }
}

// One launch with the partials of all K slices in dynamic shared memory
// (the attribute for MAX_SLICES slices set once per device).
template <int QF, int NT>
cudaError_t launch_nt(const cudaLaunchConfig_t& cfg0, const uint8_t* W, int n_tiles, int K, const __half* A, long lda,
                      const EpiParams& ep) {
  cudaLaunchConfig_t cfg = cfg0;
  cfg.dynamicSmemBytes = (size_t)r16::n_slices(K) * r16::WARPS * NT * 32 * sizeof(float4);
  static std::mutex mu;
  static bool done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (!done[dev]) {
      const cudaError_t e = cudaFuncSetAttribute(gemm_r16_kernel<QF, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)(r16::MAX_SLICES * r16::WARPS * NT * 32 * sizeof(float4)));
      if (e != cudaSuccess) return e;
      done[dev] = true;
    }
  }
  return cudaLaunchKernelEx(&cfg, gemm_r16_kernel<QF, NT>, W, n_tiles, K, A, lda, ep);
}

template <int QF>
cudaError_t launch_qf(const uint8_t* W, int n_tiles, int K, const __half* A, long lda, const EpiParams& ep,
                      cudaStream_t s) {
  const int nt = (ep.M + 7) / 8;
  cudaLaunchAttribute attr[1];
  const cudaLaunchConfig_t cfg = pdl_config(dim3(n_tiles), dim3(256), 0, s, attr);
  switch (nt) {
    case 1: return launch_nt<QF, 1>(cfg, W, n_tiles, K, A, lda, ep);
    case 2: return launch_nt<QF, 2>(cfg, W, n_tiles, K, A, lda, ep);
    case 3: return launch_nt<QF, 3>(cfg, W, n_tiles, K, A, lda, ep);
    case 4: return launch_nt<QF, 4>(cfg, W, n_tiles, K, A, lda, ep);
    case 5: return launch_nt<QF, 5>(cfg, W, n_tiles, K, A, lda, ep);
    case 6: return launch_nt<QF, 6>(cfg, W, n_tiles, K, A, lda, ep);
    case 7: return launch_nt<QF, 7>(cfg, W, n_tiles, K, A, lda, ep);
    case 8: return launch_nt<QF, 8>(cfg, W, n_tiles, K, A, lda, ep);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

// Calls of more than 64 tokens (only weights the tensor-core kernels cannot
// take) run as launches of up to 64 tokens each; a token's result does not
// depend on the others.
cudaError_t launch_gemm_r16(int qf, const uint8_t* W, int n_tiles, int K, const __half* A, long lda,
                            const EpiParams& ep, cudaStream_t s) {
  if (ep.M == 0) return cudaSuccess;
  if (K % TILE_K || K > r16::MAX_SLICES * r16::KSLICE || (lda * 2) % 16 || (reinterpret_cast<uintptr_t>(A) & 15) ||
      n_tiles <= 0)
    return cudaErrorInvalidValue;
  for (int m0 = 0; m0 < ep.M; m0 += 64) {
    EpiParams e = ep;
    e.M = ep.M - m0 < 64 ? ep.M - m0 : 64;
    if (e.out32) e.out32 += (long)m0 * ep.ldo;
    if (e.out16) e.out16 += (long)m0 * ep.ldo;
    if (e.pos) e.pos += m0;
    const __half* a = A + (long)m0 * lda;
    cudaError_t r;
    switch (qf) {
      case QF_Q8_0: r = launch_qf<QF_Q8_0>(W, n_tiles, K, a, lda, e, s); break;
      case QF_KMIN: r = launch_qf<QF_KMIN>(W, n_tiles, K, a, lda, e, s); break;
      case QF_Q6K: r = launch_qf<QF_Q6K>(W, n_tiles, K, a, lda, e, s); break;
      default: return cudaErrorInvalidValue;
    }
    if (r != cudaSuccess) return r;
  }
  return cudaSuccess;
}

}  // namespace le
