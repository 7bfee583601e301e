// Row softmax pieces shared by the tensor-core attention kernels
// (attention_stc.cu, attention_tc.cu): a thread owns one query row and
// reads its raw scores S from TMEM as 32-bit words.  bert.go:381-398 with
// the weight rule of ops_simd.go:70-82 (exp(0.125 S - max), 0 when more
// than 10 below the maximum), in base 2 with packed f32x2 arithmetic.
#pragma once
#include "gemm_epi_tc.cuh"

namespace le {
namespace tcx {

// Maximum of the NK raw scores in r (keys k0 ..) that are below k0 + kmax,
// in two interleaved chains.
template <int NK>
__device__ __forceinline__ void chunk_max(float& m0, float& m1, const uint32_t* r, int kmax) {
  if (kmax >= NK) {
#pragma unroll
    for (int k = 0; k < NK; k += 4) {
      m0 = max3(m0, __uint_as_float(r[k]), __uint_as_float(r[k + 1]));
      m1 = max3(m1, __uint_as_float(r[k + 2]), __uint_as_float(r[k + 3]));
    }
  } else {  // the step holding key L - 1 (columns past it are not this unit's)
#pragma unroll
    for (int k = 0; k < NK; k += 2) {
      m0 = fmaxf(m0, k < kmax ? __uint_as_float(r[k]) : -INFINITY);
      m1 = fmaxf(m1, k + 1 < kmax ? __uint_as_float(r[k + 1]) : -INFINITY);
    }
  }
}

// 2^x (the MUFU exponential, ex2.approx).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// exp(0.125 S - max) = 2^x with x = S * (0.125 log2 e) - max * (0.125 log2 e),
// one fused multiply-add for two keys; the reference's cutoff (weight 0
// when 0.125 S - max < -10, ops_simd.go:70-82) in the same base-2 units.
constexpr float SCALE2 = 0.125f * 1.4426950408889634f;
constexpr float CUT2 = -10.0f * 1.4426950408889634f;

// P of the NK scores in r as NK/2 fp16 pairs (0 at and past kmax), their
// sum added to two two-lane accumulators.  r is overwritten.
template <int NK>
__device__ __forceinline__ void chunk_p(uint32_t* r, int kmax, unsigned long long scale, unsigned long long off,
                                        unsigned long long& s0, unsigned long long& s1, uint32_t* w) {
#pragma unroll
  for (int e = 0; e < NK / 2; e++) {
    float x0, x1;
    f2_unpack(f2_fma(f2_pack(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1])), scale, off), x0, x1);
    r[2 * e] = __float_as_uint(x0 < CUT2 ? 0.f : ex2(x0));
    r[2 * e + 1] = __float_as_uint(x1 < CUT2 ? 0.f : ex2(x1));
  }
  if (kmax < NK) {  // the step holding key L - 1
#pragma unroll
    for (int e = 0; e < NK; e++) r[e] = e < kmax ? r[e] : 0u;
  }
#pragma unroll
  for (int e = 0; e < NK / 2; e++) {
    const float p0 = __uint_as_float(r[2 * e]), p1 = __uint_as_float(r[2 * e + 1]);
    if (e & 1)
      s1 = f2_add(s1, f2_pack(p0, p1));
    else
      s0 = f2_add(s0, f2_pack(p0, p1));
    w[e] = pack_half2(p0, p1);
  }
}

}  // namespace tcx
}  // namespace le
