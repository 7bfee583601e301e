// Fused masked attention over packed variable-length sequences
// (bert.go:356-402): scores = (Q.K^T) * 0.125 per head, softmax with the
// reference's exp rule (ops_simd.go:70-82: weights whose score is more than
// 10 below the row maximum are exactly 0), weighted sum of V.
//
// Q, K, V come RoPE-rotated in fp16 from the QKV GEMM epilogue, laid out as
// rows of qkv[T][3H]; the output is att[T][H] fp16.  The cutoff is relative
// to the row's final maximum, so every kernel finds the exact maximum before
// exponentiating (an online-softmax rescale would not reproduce it).
// Tensor-core math: mma.sync m16n8k16 (fp16 in, fp32 accumulate), operand
// fragments loaded with ldmatrix.
//
//   attention_short_kernel  L <= 128: one CTA of 8 warps per (sequence,
//       head) stages Q and K, then V, of the whole sequence in shared memory
//       (cp.async, two groups); each warp takes 16 query rows, finds their
//       maxima while V lands, then recomputes the scores chunk by chunk for
//       the exponentials and P.V (no score kept: 80 registers, 3 CTAs per
//       SM).
//   Longer sequences run the tcgen05 kernel of attention_tc.cu.
#include <math.h>

#include <mutex>

#include "attention_tile.cuh"
#include "common.cuh"
#include "kernels.h"

namespace le {

namespace {

using namespace attn;

constexpr int SH_MAXL = 128;
static_assert(ATTN_SHORT_MAX <= SH_MAXL, "short-kernel length class");
constexpr int SH_QROWS = 128;
constexpr int SH_WARPS = SH_QROWS / 16;
constexpr int SH_SMEM = (SH_QROWS + 2 * SH_MAXL) * LDS * 2;

// Rows [r0, r0 + n) of one head's 64 columns into dst (zero rows past
// `valid`) with cp.async (16-byte, L2 only); the caller waits and syncs.
__device__ __forceinline__ void load_rows_async(__half (*dst)[LDS], const __half* src, long ld, int r0, int n,
                                                int valid) {
  for (int i = threadIdx.x; i < n * 8; i += blockDim.x) {
    const int r = i >> 3, c = (i & 7) * 8;
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(&dst[r][c]);
    if (r0 + r < valid)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src + (long)(r0 + r) * ld + c) : "memory");
    else
      *reinterpret_cast<uint4*>(&dst[r][c]) = make_uint4(0, 0, 0, 0);
  }
}

}  // namespace

__global__ void __launch_bounds__(SH_WARPS * 32, 3) attention_short_kernel(const __half* __restrict__ qkv,
                                                                       const int32_t* __restrict__ offsets, int H,
                                                                       __half* __restrict__ out) {
  const int head = blockIdx.y, s = blockIdx.x;
  const int t0 = offsets[s];
  const int L = offsets[s + 1] - t0;
  if (L == 0 || L > ATTN_SHORT_MAX) return;
  extern __shared__ __align__(16) uint8_t smem_attn[];
  __half(*sQ)[LDS] = reinterpret_cast<__half(*)[LDS]>(smem_attn);
  __half(*sK)[LDS] = sQ + SH_QROWS;
  __half(*sV)[LDS] = sK + SH_MAXL;
  const long ld = 3L * H;
  const __half* base = qkv + (long)t0 * ld + head * HD;
  const int Lp = (L + 15) & ~15;
  // Q and K first, V second: the maxima pass runs while V lands.
  load_rows_async(sQ, base, ld, 0, Lp, L);
  load_rows_async(sK, base + H, ld, 0, Lp, L);
  asm volatile("cp.async.commit_group;" ::: "memory");
  load_rows_async(sV, base + 2 * H, ld, 0, Lp, L);
  asm volatile("cp.async.commit_group;" ::: "memory");
  asm volatile("cp.async.wait_group 1;" ::: "memory");
  __syncthreads();
  const int warp = threadIdx.x >> 5;
  const int qrow0 = warp * 16;
  AttnRows r;
  if (qrow0 < L) attn_max(r, sQ, warp * 16, sK, L);
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  if (qrow0 >= L) return;
  attn_pv(r, sK, sV, L, out + (long)t0 * H + head * HD, H, qrow0);
}

cudaError_t launch_attention(const __half* qkv, const int32_t* offsets, int nseq, int max_len, int H, int heads,
                             int head_dim, __half* out, cudaStream_t s) {
  if (head_dim != HD) return cudaErrorInvalidValue;
  if (nseq == 0 || max_len == 0) return cudaSuccess;
  static std::mutex mu;
  static uint64_t attr_set = 0;  // per-device bit: the attribute is a per-device setting
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 64 || !(attr_set >> dev & 1)) {
      cudaError_t e =
          cudaFuncSetAttribute(attention_short_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SH_SMEM);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attention_short_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
      if (e != cudaSuccess) return e;
      if (dev < 64) attr_set |= 1ull << dev;
    }
  }
  attention_short_kernel<<<dim3(nseq, heads), SH_WARPS * 32, SH_SMEM, s>>>(qkv, offsets, H, out);
  return cudaGetLastError();
}

}  // namespace le
