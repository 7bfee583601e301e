// One warp's LayerNorm of a row (ops_simd.go:7-24), shared by the row
// kernels (elementwise.cu) and the single-kernel small forward
// (forward_small.cu) so both give the same bits: every add and multiply is
// explicitly rounded (no contraction), sums reduce in a fixed butterfly.
#pragma once
#include "common.cuh"

namespace le {

// Accumulate sum and sum of squares of four values.
__device__ __forceinline__ void ln_accum(const float4 a, float& s, float& ss) {
  s = __fadd_rn(s, __fadd_rn(__fadd_rn(__fadd_rn(a.x, a.y), a.z), a.w));
  ss = __fadd_rn(ss, __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(a.x, a.x), __fmul_rn(a.y, a.y)), __fmul_rn(a.z, a.z)),
                               __fmul_rn(a.w, a.w)));
}

// Warp totals -> mean and float32(1 / sqrt(float64(var + eps))), with
// var = sumSq / n - mean^2 (single pass, float32).
__device__ __forceinline__ void ln_finish(float s, float ss, int n, float eps, float* mean, float* inv) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  }
  const float nf = (float)n;
  *mean = __fdiv_rn(s, nf);
  const float var = __fsub_rn(__fdiv_rn(ss, nf), __fmul_rn(*mean, *mean));
  *inv = (float)(1.0 / sqrt((double)__fadd_rn(var, eps)));
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
