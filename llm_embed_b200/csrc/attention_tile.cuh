// Tensor-core attention tile of one warp (mma.sync m16n8k16, fp16 in, fp32
// accumulate, ldmatrix fragments), shared by the attention kernels
// (attention.cu) and the single-kernel small forward (forward_small.cu), so
// a sequence gets bit-identical attention whichever path runs it.
//
// Scores = (Q.K^T) * 0.125 per head (bert.go:362-378); softmax with the
// reference's exp rule (ops_simd.go:70-82: weights whose score is more than
// 10 below the row maximum are exactly 0), weighted sum of V, normalised by
// the weight sum.
#pragma once
#include <math.h>

#include "common.cuh"

namespace le {
namespace attn {

constexpr int HD = 64;   // head dim
constexpr int LDS = 72;  // smem row stride (halves): 144 B keeps ldmatrix rows on distinct banks

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t* r, const __half* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, const __half* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
}

// A fragments of 16 query rows (row0..row0+15) x 64 dims.
__device__ __forceinline__ void load_q_frags(uint32_t (*qa)[4], __half (*sQ)[LDS], int row0) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int kc = 0; kc < 4; kc++) ldsm_x4(qa[kc], &sQ[row0 + (lane & 15)][kc * 16 + (lane >> 4) * 8]);
}

// s += Q(16 x 64) . K(8 keys x 64)^T for keys key0..key0+7.
__device__ __forceinline__ void qk_tile(float* s, uint32_t (*qa)[4], __half (*sK)[LDS], int key0) {
  const int lane = threadIdx.x & 31;
  uint32_t b[8];
  ldsm_x4(b, &sK[key0 + (lane & 7)][(lane >> 3) * 8]);
  ldsm_x4(b + 4, &sK[key0 + (lane & 7)][32 + (lane >> 3) * 8]);
  mma16816(s, qa[0], b[0], b[1]);
  mma16816(s, qa[1], b[2], b[3]);
  mma16816(s, qa[2], b[4], b[5]);
  mma16816(s, qa[3], b[6], b[7]);
}

// o[8][4] += P(16 x 16 keys) . V(16 keys x 64) for keys key0..key0+15.
__device__ __forceinline__ void pv_chunk(float (*o)[4], const uint32_t* pa, __half (*sV)[LDS], int key0) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int dt = 0; dt < 8; dt += 2) {
    uint32_t b[4];
    ldsm_x4_t(b, &sV[key0 + (lane & 7) + ((lane >> 3) & 1) * 8][8 * dt + (lane >> 4) * 8]);
    mma16816(o[dt], pa, b[0], b[1]);
    mma16816(o[dt + 1], pa, b[2], b[3]);
  }
}

// exp rule of ops_simd.go:70-82 on a score x already reduced by the max
// (__expf, the hardware exponential: a few ulp from expf, far inside the
// fp16 rounding of P that follows).
__device__ __forceinline__ float ref_exp(float x) { return x < -10.f ? 0.f : __expf(x); }

// Normalise and store 16 rows x 64 dims (rows q0 and q0+8 of this lane).
__device__ __forceinline__ void store_rows(__half* out, long ldo, int L, int q0, float (*o)[4], float l0, float l1) {
  const int tq = threadIdx.x & 3;
  const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
#pragma unroll
  for (int dt = 0; dt < 8; dt++) {
    const int d = dt * 8 + tq * 2;
    if (q0 < L) *reinterpret_cast<uint32_t*>(out + (long)q0 * ldo + d) = pack_half2(o[dt][0] * inv0, o[dt][1] * inv0);
    if (q0 + 8 < L)
      *reinterpret_cast<uint32_t*>(out + (long)(q0 + 8) * ldo + d) = pack_half2(o[dt][2] * inv1, o[dt][3] * inv1);
  }
}

// One warp's 16 query rows, in two passes over the keys so that no score
// is kept: pass 1 (attn_max) finds each row's maximum tile by tile; pass 2
// (attn_pv) recomputes each 16-key chunk's scores, exponentiates them and
// multiplies by V.  Rows qrow_local .. +15 of sQ are query indices
// qrow0 .. qrow0+15 of a sequence of L tokens; sK and sV hold rows
// 0 .. round_up(L, 16) - 1 (zero past L).  Tiles at or past round_up(L, 16)
// hold only masked keys (weight exactly 0) and are skipped, so the result
// depends only on L.  pass 2 needs sV; pass 1 does not.
struct AttnRows {
  uint32_t qa[4][4];  // Q fragments (16 rows x 64 dims)
  float mx0, mx1;     // maxima of rows g and g + 8 of this lane
};

// Scores of keys n*8 .. n*8+7 for the warp's rows, scaled by 0.125, -inf
// past L.
__device__ __forceinline__ void attn_scores(float* s, const AttnRows& r, __half (*sK)[LDS], int n, int L) {
  s[0] = s[1] = s[2] = s[3] = 0.f;
  qk_tile(s, const_cast<uint32_t(*)[4]>(r.qa), sK, n * 8);
  if (n * 8 + 8 <= L) {  // warp-uniform: no masked key in this tile
#pragma unroll
    for (int j = 0; j < 4; j++) s[j] *= 0.125f;
  } else {
    const int key = n * 8 + (threadIdx.x & 3) * 2;
#pragma unroll
    for (int j = 0; j < 4; j++) s[j] = (key + (j & 1) < L) ? s[j] * 0.125f : -INFINITY;
  }
}

__device__ __forceinline__ void attn_max(AttnRows& r, __half (*sQ)[LDS], int qrow_local, __half (*sK)[LDS], int L) {
  load_q_frags(r.qa, sQ, qrow_local);
  const int Lp = (L + 15) & ~15;
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll 2
  for (int n = 0; n < Lp / 8; n++) {
    float s[4];
    attn_scores(s, r, sK, n, L);
    mx0 = fmaxf(mx0, fmaxf(s[0], s[1]));
    mx1 = fmaxf(mx1, fmaxf(s[2], s[3]));
  }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
  }
  r.mx0 = mx0;
  r.mx1 = mx1;
}

// Writes rows q < L of the head's output block `out` (row stride ldo).
__device__ __forceinline__ void attn_pv(const AttnRows& r, __half (*sK)[LDS], __half (*sV)[LDS], int L, __half* out,
                                        long ldo, int qrow0) {
  const int Lp = (L + 15) & ~15;
  float l0 = 0.f, l1 = 0.f;
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll 1
  for (int c = 0; c < Lp / 16; c++) {
    float s[2][4];
#pragma unroll
    for (int h = 0; h < 2; h++) {
      attn_scores(s[h], r, sK, 2 * c + h, L);
      s[h][0] = ref_exp(__fsub_rn(s[h][0], r.mx0));
      s[h][1] = ref_exp(__fsub_rn(s[h][1], r.mx0));
      s[h][2] = ref_exp(__fsub_rn(s[h][2], r.mx1));
      s[h][3] = ref_exp(__fsub_rn(s[h][3], r.mx1));
      l0 += s[h][0] + s[h][1];
      l1 += s[h][2] + s[h][3];
    }
    const uint32_t pa[4] = {pack_half2(s[0][0], s[0][1]), pack_half2(s[0][2], s[0][3]), pack_half2(s[1][0], s[1][1]),
                            pack_half2(s[1][2], s[1][3])};
    pv_chunk(acc, pa, sV, c * 16);
  }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  store_rows(out, ldo, L, qrow0 + ((threadIdx.x & 31) >> 2), acc, l0, l1);
}

// Both passes for at most 16 keys (one 16-key chunk): the chunk's scores
// are computed once and kept for the second pass; every operation and its
// order are those of attn_max + attn_pv, so the bits are the same.
__device__ __forceinline__ void attn_rows16_short(__half (*sQ)[LDS], int qrow_local, __half (*sK)[LDS],
                                                  __half (*sV)[LDS], int L, __half* out, long ldo, int qrow0) {
  AttnRows r;
  load_q_frags(r.qa, sQ, qrow_local);
  float s[2][4];
  attn_scores(s[0], r, sK, 0, L);
  attn_scores(s[1], r, sK, 1, L);
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int h = 0; h < 2; h++) {
    mx0 = fmaxf(mx0, fmaxf(s[h][0], s[h][1]));
    mx1 = fmaxf(mx1, fmaxf(s[h][2], s[h][3]));
  }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
  }
  float l0 = 0.f, l1 = 0.f;
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; i++) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
  for (int h = 0; h < 2; h++) {
    s[h][0] = ref_exp(__fsub_rn(s[h][0], mx0));
    s[h][1] = ref_exp(__fsub_rn(s[h][1], mx0));
    s[h][2] = ref_exp(__fsub_rn(s[h][2], mx1));
    s[h][3] = ref_exp(__fsub_rn(s[h][3], mx1));
    l0 += s[h][0] + s[h][1];
    l1 += s[h][2] + s[h][3];
  }
  const uint32_t pa[4] = {pack_half2(s[0][0], s[0][1]), pack_half2(s[0][2], s[0][3]), pack_half2(s[1][0], s[1][1]),
                          pack_half2(s[1][2], s[1][3])};
  pv_chunk(acc, pa, sV, 0);
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  store_rows(out, ldo, L, qrow0 + ((threadIdx.x & 31) >> 2), acc, l0, l1);
}

// Both passes, for callers that have K and V in shared memory already.
__device__ __forceinline__ void attn_rows16(__half (*sQ)[LDS], int qrow_local, __half (*sK)[LDS], __half (*sV)[LDS],
                                            int L, __half* out, long ldo, int qrow0) {
  if (L <= 16) {
    attn_rows16_short(sQ, qrow_local, sK, sV, L, out, ldo, qrow0);
    return;
  }
  AttnRows r;
  attn_max(r, sQ, qrow_local, sK, L);
  attn_pv(r, sK, sV, L, out, ldo, qrow0);
}

}  // namespace attn
}  // namespace le
