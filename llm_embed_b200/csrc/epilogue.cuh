// GEMM epilogues shared by every GEMM kernel.  They receive output values in
// pairs (va, vb) of the GEMM's "virtual" output rows a, b:
//   EPI_F32    plain float32 store (attention-output and FFN-down
//              projections, whose residual add h += y is fused into the
//              following LayerNorm kernel, and the standalone qgemm op)
//   EPI_QKV    QKV projection: RoPE on the Q and K columns (adjacent pairs
//              2i, 2i+1 of each head, ops_simd.go:127-137), fp16 store
//   EPI_GEGLU  merged up/gate: gelu(gate) * up (bert.go:431-436), fp16 store
#pragma once
#include "common.cuh"

namespace le {

enum EpiMode : int { EPI_F32 = 0, EPI_QKV = 1, EPI_GEGLU = 3 };

struct EpiParams {
  int mode;
  int M;           // valid output rows (tokens)
  int N;           // output columns of the real result
  float* out32;    // EPI_F32
  __half* out16;   // EPI_QKV, EPI_GEGLU
  long ldo;        // leading dimension of out (elements)
  const int32_t* pos;  // EPI_QKV: position of each token in its sequence
  const float* rope_cos;  // [max_pos][head_dim/2]
  const float* rope_sin;
  int head_dim;
  int rope_cols;   // columns [0, rope_cols) get RoPE (= 2 * hidden)
};

// ops_simd.go:27-43: 0.5 v (1 + tanh_r(t)), t = 0.7978845608 v (1 + 0.044715
// v^2), tanh_r(t) = t (27 + t^2) / (27 + 9 t^2) clamped to +-1 for |t| > 4.97.
// The quotient uses the fast reciprocal: the result is rounded to fp16 (the
// next GEMM's operand), far coarser than the few-ulp difference.
__device__ __forceinline__ float gelu_tanh_rational(float v) {
  const float t = 0.7978845608f * v * (1.0f + 0.044715f * v * v);
  const float t2 = t * t;
  float th = __fdividef(t * (27.0f + t2), 27.0f + 9.0f * t2);
  th = t > 4.97f ? 1.0f : (t < -4.97f ? -1.0f : th);
  return 0.5f * v * (1.0f + th);
}

// Map GEMM output pair index p to virtual rows (a, b) and output columns.
// EPI_GEGLU: weight tile t = p/64 holds up rows t*128 + c (c < 64) and gate
// rows t*128 + 64 + c, for output column t*64 + c.  Others: a = 2p, b = 2p+1.
constexpr int GEGLU_HALF = TILE_N / 2;
__device__ __forceinline__ void pair_rows(int mode, int p, int* a, int* b) {
  if (mode == EPI_GEGLU) {
    const int t = p / GEGLU_HALF, c = p % GEGLU_HALF;
    *a = t * TILE_N + c;
    *b = *a + GEGLU_HALF;
  } else {
    *a = 2 * p;
    *b = 2 * p + 1;
  }
}

// Apply the epilogue to one pair.  For EPI_GEGLU, `a` is the up row (its
// output column is t*128 + c) and va/vb are (up, gate).
__device__ __forceinline__ void epi_pair(const EpiParams& ep, int m, int a, float va, float vb) {
  switch (ep.mode) {
    case EPI_F32: {
      float* o = ep.out32 + (long)m * ep.ldo;
      if (a < ep.N) o[a] = va;
      if (a + 1 < ep.N) o[a + 1] = vb;
      break;
    }
    case EPI_QKV: {
      if (a >= ep.N) return;
      float x0 = va, x1 = vb;
      if (a < ep.rope_cols) {
        const int i = (a % ep.head_dim) >> 1;
        const long r = (long)ep.pos[m] * (ep.head_dim >> 1) + i;
        const float c = ep.rope_cos[r], s = ep.rope_sin[r];
        x0 = __fsub_rn(__fmul_rn(va, c), __fmul_rn(vb, s));
        x1 = __fadd_rn(__fmul_rn(va, s), __fmul_rn(vb, c));
      }
      *reinterpret_cast<uint32_t*>(ep.out16 + (long)m * ep.ldo + a) = pack_half2(x0, x1);
      break;
    }
    case EPI_GEGLU: {
      const int col = (a / TILE_N) * GEGLU_HALF + (a % TILE_N);
      if (col >= ep.N) return;
      ep.out16[(long)m * ep.ldo + col] = __float2half_rn(gelu_tanh_rational(vb) * va);
      break;
    }
  }
}

}  // namespace le
