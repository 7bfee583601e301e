// Epilogue of the tensor-core GEMM kernels (gemm_tc2.cu, gemm_f16.cu): one
// warp drains 32 accumulator rows (TMEM lanes 32*(warp%4) ..) of a
// 256-column tile, applies the fused epilogue and writes 32-row x 128-byte
// output blocks with TMA stores from 128B-swizzled staging buffers.
#pragma once
#include <cudaTypedefs.h>

#include "epilogue.cuh"
#include "tcgen05.cuh"

namespace le {
namespace tcx {

// TMA store of a 32-row block from shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// One warp stages its 32 rows x 128 bytes (words[32] per lane = its row) in
// buffer `buf` of its two 4 KB buffers at `stage` and stores it with one TMA
// store at (col0, row0).  Before a buffer is rewritten the store that last
// read it must be done (at most one store group left in flight).
__device__ __forceinline__ void emit_block(const CUtensorMap* map, uint32_t stage, int& buf, const uint32_t* words,
                                           int col0, int row0) {
  const int lane = threadIdx.x & 31;
  if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
  __syncwarp();
  const uint32_t base = stage + buf * 4096 + lane * 128;
#pragma unroll
  for (int q = 0; q < 8; q++)
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(base + ((q ^ (lane & 7)) << 4)), "r"(words[4 * q]),
                 "r"(words[4 * q + 1]), "r"(words[4 * q + 2]), "r"(words[4 * q + 3])
                 : "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  if (lane == 0) tma_store_2d(map, stage + buf * 4096, col0, row0);
  buf ^= 1;
}

// gelu(v) * u with the GeLU of ops_simd.go:27-43:
//   t = 0.7978845608 v (1 + 0.044715 v^2)
//   tanh_r(t) = t (27 + t^2) / (27 + 9 t^2), +-1 where |t| > 4.97
//   gelu = 0.5 v (1 + tanh_r(t))
// evaluated as t = v (0.7978845608 + 0.0356774081 v^2), tanh_r = t ((27 +
// t^2) / (27 + 9 t^2)) with the fast reciprocal, and 0.5 v u + 0.5 v u
// tanh_r; the product is rounded to fp16 (the next GEMM's operand), far
// coarser than these few-ulp changes of the evaluation order.
__device__ __forceinline__ float geglu(float v, float u) {
  const float t = v * fmaf(0.0356774081f, v * v, 0.7978845608f);
  const float t2 = t * t;
  float th = t * __fdividef(27.0f + t2, fmaf(9.0f, t2, 27.0f));
  th = t > 4.97f ? 1.0f : (t < -4.97f ? -1.0f : th);
  const float hv = (0.5f * v) * u;
  return fmaf(hv, th, hv);
}

// Two-lane fp32 arithmetic (sm_100 packed f32x2: one instruction, two IEEE
// round-to-nearest results, the same as the scalar operations).
__device__ __forceinline__ unsigned long long f2_pack(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(unsigned long long r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b, unsigned long long c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// max(a, b, c) in one instruction (sm_100 three-input max; exact).
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// geglu() of two (gate, up) pairs, as fp16x2: the same operations in the
// same order, two lanes per instruction (the reciprocal stays per element).
__device__ __forceinline__ uint32_t geglu2(float v0, float v1, float u0, float u1) {
  const unsigned long long v = f2_pack(v0, v1);
  const unsigned long long t = f2_mul(v, f2_fma(f2_pack(0.0356774081f, 0.0356774081f), f2_mul(v, v),
                                                f2_pack(0.7978845608f, 0.7978845608f)));
  const unsigned long long t2 = f2_mul(t, t);
  const unsigned long long num = f2_add(f2_pack(27.0f, 27.0f), t2);
  const unsigned long long den = f2_fma(f2_pack(9.0f, 9.0f), t2, f2_pack(27.0f, 27.0f));
  float n0, n1, d0, d1, t0, t1;
  f2_unpack(num, n0, n1);
  f2_unpack(den, d0, d1);
  f2_unpack(t, t0, t1);
  float th0, th1;
  f2_unpack(f2_mul(t, f2_pack(__fdividef(n0, d0), __fdividef(n1, d1))), th0, th1);
  th0 = fabsf(t0) > 4.97f ? copysignf(1.0f, t0) : th0;
  th1 = fabsf(t1) > 4.97f ? copysignf(1.0f, t1) : th1;
  const unsigned long long hv = f2_mul(f2_mul(f2_pack(0.5f, 0.5f), v), f2_pack(u0, u1));
  float o0, o1;
  f2_unpack(f2_fma(hv, f2_pack(th0, th1), hv), o0, o1);
  return pack_half2(o0, o1);
}

// Epilogue of one 256-column pair tile for the calling warp: accumulator
// columns [c_begin, c_end) of TMEM address `tbase` (its lane quarter already
// added), output rows row0 .. row0+31, tile column origin n0 (virtual rows of
// the weight).  Rows at or beyond ep.M are clipped by the TMA store.
// RoPE of this lane's row: cos and sin of rotation pairs 0..31, loaded before
// the accumulator is ready (rope_prefetch) so their latency overlaps the MMA.
struct RopeRow {
  float4 c[8], s[8];
};

__device__ __forceinline__ bool rope_tile(const EpiParams& ep, int n0) { return ep.mode == EPI_QKV && n0 < ep.rope_cols; }

__device__ __forceinline__ void rope_prefetch(const EpiParams& ep, int row0, RopeRow& rr) {
  const int lane = threadIdx.x & 31;
  const long prow = (long)ep.pos[min(row0 + lane, ep.M - 1)] * 32;
  const float4* cp = reinterpret_cast<const float4*>(ep.rope_cos + prow);
  const float4* sp = reinterpret_cast<const float4*>(ep.rope_sin + prow);
#pragma unroll
  for (int q = 0; q < 8; q++) {
    rr.c[q] = __ldg(cp + q);
    rr.s[q] = __ldg(sp + q);
  }
}

// PRE: the caller passes the row's RoPE values (rope_prefetch) in `pre`;
// otherwise they are loaded here, per 16 columns.
template <bool PRE = false>
__device__ __forceinline__ void epilogue_tile(const EpiParams& ep, const CUtensorMap* tmap_out, uint32_t tbase,
                                              int row0, int n0, int c_begin, int c_end, uint32_t stage, int& buf,
                                              const RopeRow* pre = nullptr) {
  const int lane = threadIdx.x & 31;
  uint32_t words[32];
  if (ep.mode == EPI_GEGLU) {
    // Each 128-column half is one weight tile: up columns c, gate c + 64;
    // its 64 outputs form one fp16 block.
#pragma unroll 1
    for (int c = c_begin; c < c_end; c += TILE_N) {
#pragma unroll
      for (int h = 0; h < 4; h++) {
        float up[16], gt[16];
        tmem_ld16(tbase + c + 16 * h, up);
        tmem_ld16(tbase + c + 16 * h + GEGLU_HALF, gt);
#pragma unroll
        for (int i = 0; i < 8; i++)
          words[8 * h + i] = geglu2(gt[2 * i], gt[2 * i + 1], up[2 * i], up[2 * i + 1]);
      }
      emit_block(tmap_out, stage, buf, words, (n0 + c) / TILE_N * GEGLU_HALF, row0);
    }
  } else if (ep.mode == EPI_QKV) {
    // One head (64 columns) per fp16 block; RoPE on the Q and K heads
    // (ops_simd.go:127-137), pairs (2i, 2i+1) rotated by the row's position.
    const bool rope = n0 < ep.rope_cols;
    const long prow = PRE ? 0 : (long)ep.pos[min(row0 + lane, ep.M - 1)] * 32;
#pragma unroll 1
    for (int c = c_begin; c < c_end; c += 64) {
#pragma unroll
      for (int h = 0; h < 4; h++) {  // 16 columns = rotation pairs 8h .. 8h+7
        float4 cq[2], sq[2];
        if constexpr (PRE) {
          cq[0] = pre->c[2 * h];
          cq[1] = pre->c[2 * h + 1];
          sq[0] = pre->s[2 * h];
          sq[1] = pre->s[2 * h + 1];
        } else if (rope) {
          const float4* cp = reinterpret_cast<const float4*>(ep.rope_cos + prow + 8 * h);
          const float4* sp = reinterpret_cast<const float4*>(ep.rope_sin + prow + 8 * h);
          cq[0] = __ldg(cp);
          cq[1] = __ldg(cp + 1);
          sq[0] = __ldg(sp);
          sq[1] = __ldg(sp + 1);
        }
        float v[16];
        tmem_ld16(tbase + c + 16 * h, v);
        if (rope) {
          const float cc[8] = {cq[0].x, cq[0].y, cq[0].z, cq[0].w, cq[1].x, cq[1].y, cq[1].z, cq[1].w};
          const float ss[8] = {sq[0].x, sq[0].y, sq[0].z, sq[0].w, sq[1].x, sq[1].y, sq[1].z, sq[1].w};
#pragma unroll
          for (int i = 0; i < 8; i++) {
            const float x0 = v[2 * i], x1 = v[2 * i + 1];
            v[2 * i] = __fsub_rn(__fmul_rn(x0, cc[i]), __fmul_rn(x1, ss[i]));
            v[2 * i + 1] = __fadd_rn(__fmul_rn(x0, ss[i]), __fmul_rn(x1, cc[i]));
          }
        }
#pragma unroll
        for (int i = 0; i < 8; i++) words[8 * h + i] = pack_half2(v[2 * i], v[2 * i + 1]);
      }
      emit_block(tmap_out, stage, buf, words, n0 + c, row0);
    }
  } else {
#pragma unroll 1
    for (int c = c_begin; c < c_end; c += 32) {
      float v[32];
      tmem_ld32(tbase + c, v);
#pragma unroll
      for (int i = 0; i < 32; i++) words[i] = __float_as_uint(v[i]);
      emit_block(tmap_out, stage, buf, words, n0 + c, row0);
    }
  }
}

}  // namespace tcx
}  // namespace le
