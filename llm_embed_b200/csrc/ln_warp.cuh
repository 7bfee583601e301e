// LayerNorm of a row (ops_simd.go:7-24), shared by the row kernels
// (elementwise.cu), the single-kernel small forward (forward_small.cu) and
// the fused projection + LayerNorm kernel (gemm_ln.cu) so all give the same
// bits: every add and multiply is explicitly rounded (no contraction), sums
// reduce in one fixed order (ln_row_stats).
#pragma once
#include "common.cuh"

namespace le {

// Accumulate sum and sum of squares of four values.
__device__ __forceinline__ void ln_accum(const float4 a, float& s, float& ss) {
  s = __fadd_rn(s, __fadd_rn(__fadd_rn(__fadd_rn(a.x, a.y), a.z), a.w));
  ss = __fadd_rn(ss, __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(a.x, a.x), __fmul_rn(a.y, a.y)), __fmul_rn(a.z, a.z)),
                               __fmul_rn(a.w, a.w)));
}

// float32(1 / sqrt(float64(var + eps))) of the row totals, with
// var = sumSq / n - mean^2 (single pass, float32).
__device__ __forceinline__ void ln_stats(float s, float ss, int n, float eps, float* mean, float* inv) {
  const float nf = (float)n;
  *mean = __fdiv_rn(s, nf);
  const float var = __fsub_rn(__fdiv_rn(ss, nf), __fmul_rn(*mean, *mean));
  *inv = (float)(1.0 / sqrt((double)__fadd_rn(var, eps)));
}

// Row statistics of one warp's row.  Lane l holds float4 chunk i at columns
// (32 i + l) * 4, i < nv.  Each 128-column chunk reduces on its own: the
// lane's four values (ln_accum from zero), then a fixed butterfly over the
// lanes (xor 16, 8, 4, 2, 1); the chunk totals add in column order.  The
// fused projection + LayerNorm kernel (gemm_ln.cu), whose warps each own one
// chunk of a row, repeats exactly these operations, so every path gives the
// same bits.
template <int MAXV>
__device__ __forceinline__ void ln_row_stats(const float4 (&x)[MAXV], int nv, int n, float eps, float* mean,
                                             float* inv) {
  float ts = 0.f, tss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; i++) {
    if (i < nv) {
      float s = 0.f, ss = 0.f;
      ln_accum(x[i], s, ss);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
        ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      }
      ts = __fadd_rn(ts, s);
      tss = __fadd_rn(tss, ss);
    }
  }
  ln_stats(ts, tss, n, eps, mean, inv);
}

// (x - mean) * inv * w + b.
__device__ __forceinline__ float4 ln_apply(const float4 x, float mean, float inv, const float4 w, const float4 b) {
  float4 y;
  y.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x.x, mean), inv), w.x), b.x);
  y.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x.y, mean), inv), w.y), b.y);
  y.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x.z, mean), inv), w.z), b.z);
  y.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x.w, mean), inv), w.w), b.w);
  return y;
}

}  // namespace le
