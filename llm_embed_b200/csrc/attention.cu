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
//   attention_short_kernel  L <= 128: one CTA of 4 warps per (64 queries,
//       head, sequence) keeps K, V of the whole sequence and its Q rows in
//       shared memory (cp.async); each warp holds its 16 query rows' scores
//       for all keys in registers (one pass).
//   attention_long_kernel   L > 128: one CTA of 8 warps per (128 queries,
//       head, sequence), keys in 64-row blocks double-buffered with
//       cp.async, a max pass then an exp + P.V pass.
#include <math.h>

#include <mutex>

#include "attention_tile.cuh"
#include "common.cuh"
#include "kernels.h"

namespace le {

namespace {

using namespace attn;

constexpr int SH_MAXL = 128;
constexpr int SH_QROWS = 64;
constexpr int SH_WARPS = SH_QROWS / 16;
constexpr int SH_SMEM = (SH_QROWS + 2 * SH_MAXL) * LDS * 2;
constexpr int KB = 64;  // long kernel key block

// Rows [r0, r0 + n) of one head's 64 columns into dst (zero rows past
// `valid`), by all threads of the block.
__device__ __forceinline__ void load_rows(__half (*dst)[LDS], const __half* src, long ld, int r0, int n, int valid) {
  for (int i = threadIdx.x; i < n * 8; i += blockDim.x) {
    const int r = i >> 3, c = (i & 7) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r0 + r < valid) v = *reinterpret_cast<const uint4*>(src + (long)(r0 + r) * ld + c);
    *reinterpret_cast<uint4*>(&dst[r][c]) = v;
  }
}

// Same with cp.async (16-byte, L2 only); the caller waits and syncs.
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

__global__ void __launch_bounds__(SH_WARPS * 32, 4) attention_short_kernel(const __half* __restrict__ qkv,
                                                                       const int32_t* __restrict__ offsets, int H,
                                                                       __half* __restrict__ out) {
  const int qb = blockIdx.x, head = blockIdx.y, s = blockIdx.z;
  const int t0 = offsets[s];
  const int L = offsets[s + 1] - t0;
  if (L == 0 || L > SH_MAXL || qb * SH_QROWS >= L) return;
  extern __shared__ __align__(16) uint8_t smem_attn[];
  __half(*sQ)[LDS] = reinterpret_cast<__half(*)[LDS]>(smem_attn);
  __half(*sK)[LDS] = sQ + SH_QROWS;
  __half(*sV)[LDS] = sK + SH_MAXL;
  const long ld = 3L * H;
  const __half* base = qkv + (long)t0 * ld + head * HD;
  const int Lp = (L + 15) & ~15;
  load_rows_async(sQ, base, ld, qb * SH_QROWS, SH_QROWS, L);
  load_rows_async(sK, base + H, ld, 0, Lp, L);
  load_rows_async(sV, base + 2 * H, ld, 0, Lp, L);
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  const int warp = threadIdx.x >> 5;
  const int qrow0 = qb * SH_QROWS + warp * 16;
  if (qrow0 >= L) return;
  attn_rows16<SH_MAXL>(sQ, warp * 16, sK, sV, L, out + (long)t0 * H + head * HD, H, qrow0);
}

// Long sequences: one CTA of 8 warps per (128 queries, head, sequence);
// 64-key blocks of K (pass 1) and K, V (pass 2) stream through a double
// buffer with cp.async, so block kb+1 loads while block kb is multiplied.
constexpr int LQ = 128;  // query rows per CTA
constexpr int LWARPS = LQ / 16;
constexpr int LONG_SMEM = (LQ + 4 * KB) * LDS * 2;  // Q, K[2], V[2]

__global__ void __launch_bounds__(LWARPS * 32) attention_long_kernel(const __half* __restrict__ qkv,
                                                                    const int32_t* __restrict__ offsets, int H,
                                                                    __half* __restrict__ out) {
  const int qb = blockIdx.x, head = blockIdx.y, s = blockIdx.z;
  const int t0 = offsets[s];
  const int L = offsets[s + 1] - t0;
  if (L <= SH_MAXL || qb * LQ >= L) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tq = lane & 3;
  extern __shared__ __align__(16) uint8_t smem_long[];
  __half(*sQ)[LDS] = reinterpret_cast<__half(*)[LDS]>(smem_long);
  __half(*sK)[LDS] = sQ + LQ;       // [2][KB]
  __half(*sV)[LDS] = sK + 2 * KB;   // [2][KB]
  const long ld = 3L * H;
  const __half* base = qkv + (long)t0 * ld + head * HD;
  const int qrow0 = qb * LQ + warp * 16;
  const bool active = qrow0 < L;  // warp-uniform; idle warps still load and sync
  const int nkb = (L + KB - 1) / KB;
  load_rows_async(sQ, base, ld, qb * LQ, LQ, L);
  load_rows_async(sK, base + H, ld, 0, KB, L);
  asm volatile("cp.async.commit_group;" ::: "memory");

  // Pass 1: row maxima of the scaled scores.
  uint32_t qa[4][4];
  float mx0 = -INFINITY, mx1 = -INFINITY;
  for (int i = 0; i < nkb; i++) {
    if (i + 1 < nkb) load_rows_async(sK + ((i + 1) & 1) * KB, base + H, ld, (i + 1) * KB, KB, L);
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncthreads();
    if (i == 0 && active) load_q_frags(qa, sQ, warp * 16);
    if (active) {
      __half(*k)[LDS] = sK + (i & 1) * KB;
      const int kb = i * KB;
#pragma unroll
      for (int nt = 0; nt < KB / 8; nt++) {
        float c[4] = {0.f, 0.f, 0.f, 0.f};
        qk_tile(c, qa, k, nt * 8);
        const int key = kb + nt * 8 + tq * 2;
        if (key < L) {
          mx0 = fmaxf(mx0, c[0] * 0.125f);
          mx1 = fmaxf(mx1, c[2] * 0.125f);
        }
        if (key + 1 < L) {
          mx0 = fmaxf(mx0, c[1] * 0.125f);
          mx1 = fmaxf(mx1, c[3] * 0.125f);
        }
      }
    }
    __syncthreads();  // buffer i & 1 is refilled next iteration
  }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
  }

  // Pass 2: p = exp(s - max) (0 below -10), l = sum p, O = P.V.
  float l0 = 0.f, l1 = 0.f;
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  load_rows_async(sK, base + H, ld, 0, KB, L);
  load_rows_async(sV, base + 2 * H, ld, 0, KB, L);
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int i = 0; i < nkb; i++) {
    if (i + 1 < nkb) {
      load_rows_async(sK + ((i + 1) & 1) * KB, base + H, ld, (i + 1) * KB, KB, L);
      load_rows_async(sV + ((i + 1) & 1) * KB, base + 2 * H, ld, (i + 1) * KB, KB, L);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncthreads();
    if (active) {
      __half(*k)[LDS] = sK + (i & 1) * KB;
      __half(*v)[LDS] = sV + (i & 1) * KB;
      const int kb = i * KB;
#pragma unroll
      for (int kc2 = 0; kc2 < KB / 16; kc2++) {
        float p[2][4];
#pragma unroll
        for (int h2 = 0; h2 < 2; h2++) {
          const int nt = kc2 * 2 + h2;
          float c[4] = {0.f, 0.f, 0.f, 0.f};
          qk_tile(c, qa, k, nt * 8);
          const int key = kb + nt * 8 + tq * 2;
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const bool valid = key + (j & 1) < L;
            p[h2][j] = valid ? ref_exp(__fsub_rn(c[j] * 0.125f, (j < 2) ? mx0 : mx1)) : 0.f;
          }
          l0 += p[h2][0] + p[h2][1];
          l1 += p[h2][2] + p[h2][3];
        }
        const uint32_t pa[4] = {pack_half2(p[0][0], p[0][1]), pack_half2(p[0][2], p[0][3]),
                                pack_half2(p[1][0], p[1][1]), pack_half2(p[1][2], p[1][3])};
        pv_chunk(acc, pa, v, kc2 * 16);
      }
    }
    __syncthreads();
  }
  if (!active) return;
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  store_rows(out + (long)t0 * H + head * HD, H, L, qrow0 + (lane >> 2), acc, l0, l1);
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
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attention_long_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attention_long_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, LONG_SMEM);
      if (e != cudaSuccess) return e;
      if (dev < 64) attr_set |= 1ull << dev;
    }
  }
  for (int s0 = 0; s0 < nseq; s0 += 65535) {  // grid.y/z limit
    const int n = nseq - s0 < 65535 ? nseq - s0 : 65535;
    const int sq = (max_len < SH_MAXL ? max_len : SH_MAXL);
    attention_short_kernel<<<dim3((sq + SH_QROWS - 1) / SH_QROWS, heads, n), SH_WARPS * 32, SH_SMEM, s>>>(
        qkv, offsets + s0, H, out);
    if (max_len > SH_MAXL)
      attention_long_kernel<<<dim3((max_len + LQ - 1) / LQ, heads, n), LWARPS * 32, LONG_SMEM, s>>>(qkv, offsets + s0,
                                                                                                H, out);
  }
  return cudaGetLastError();
}

}  // namespace le
