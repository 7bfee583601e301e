// Row-tile GEMM for few tokens on tensor cores (mma.sync m16n8k16), shared by
// the small-batch GEMM kernel (gemm_r16.cu) and the single-kernel small
// forward (forward_small.cu) so that a token gets the same bits from both.
//
// out[token][row] = sum_k x[token][k] * W[row][k] for a tile of 16 weight
// rows (the MMA's M) and the tokens in groups of 8 (its N).  The weight is
// held in the "row16" layout built at load (weights.cu):
//
//   tile j (16 rows) = K/64 chunks; chunk = u8 q+128 [16][64] (1024 B), then
//   the rows' metadata [16][MRB] in the per-row format of the 128-row tile
//   layout (common.cuh), so dq8_f16 decodes it unchanged.
//
// Row r < 8 and row r + 8 of a tile form the output pair that one MMA
// thread holds (C fragment rows g, g+8): for QKV / output / down tiles they
// are features 16j + 2r and 16j + 2r + 1 (the RoPE pair), for the merged
// up/gate tile up[8j + r] and gate[8j + r] (the GEGLU pair).
//
// K order.  MMA thread (g, t) (g = lane/4, t = lane%4) feeds the k indices
// {2t, 2t+1, 2t+8, 2t+9} of each k16 step; here they are the bytes
// 16t + 8h + 4s + {0, 1, 2, 3} of a 64-column chunk (h = unit half, s = step
// of the unit), for the weight rows and for the activation row alike.  The
// k permutation is the same on both operands, so the products are those of
// x . W^T; a thread reads its 8 weight bytes per row and 8 fp16 activations
// per token with one load each.
//
// K split.  K is cut into slices of KSLICE = 1024 columns (the last may be
// shorter: K = 768 is one slice, K = 3072 three).  In each slice the K/32
// units (chunk u/2, half u%2) are divided evenly over the 8 warps of a CTA in
// order; each warp accumulates its units in order into its own fragments,
// the eight partial fragments are summed warp 0..7 in float32, and the
// slices' sums are added slice 0, 1, ... in float32.  Both kernels use
// exactly this split and order, for every token count (the batch-1 kernel
// computes the slices of a tile on different CTAs and adds them where they
// are read), so a token's output never depends on the other tokens in the
// call.
#pragma once
#include "dequant.cuh"
#include "epilogue.cuh"

namespace le {
namespace r16 {

constexpr int ROWS = 16;
constexpr int WARPS = 8;
constexpr int CHUNK_Q = ROWS * TILE_K;  // 1024

__host__ __device__ constexpr int meta_row_bytes(int qf) { return qf == QF_Q8_0 ? 4 : 16; }
__host__ __device__ constexpr int chunk_bytes(int qf) { return CHUNK_Q + ROWS * meta_row_bytes(qf); }
__host__ __device__ constexpr long tile_bytes(int qf, int K) { return (long)(K / TILE_K) * chunk_bytes(qf); }

constexpr int KSLICE = 1024;
constexpr int MAX_SLICES = 4;  // K <= 4096
__host__ __device__ constexpr int n_slices(int K) { return (K + KSLICE - 1) / KSLICE; }

// Units [u0, u1) (absolute unit indices) of warp w in slice s of a K-column
// tile.
__device__ __forceinline__ void slice_units(int K, int s, int w, int* u0, int* u1) {
  const int k0 = s * KSLICE, ks = K - k0 < KSLICE ? K - k0 : KSLICE;
  const int U = ks / 32, base = k0 / 32;
  *u0 = base + w * U / WARPS;
  *u1 = base + (w + 1) * U / WARPS;
}

__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Accumulate units [u0, u1) of one tile into acc[nt][4] (token group nt).
// chunk_at(c) returns the address of the tile's chunk c (shared or global
// memory); bload(nt, k) returns the 8 fp16 activations of token 8 nt + g at
// (physical) columns k .. k+7 as a uint4.
template <int QF, int NT, class ChunkAt, class BLoad>
__device__ __forceinline__ void tile_units(ChunkAt chunk_at, int u0, int u1, float (&acc)[NT][4], BLoad bload) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll 2
  for (int u = u0; u < u1; u++) {
    const int c = u >> 1, h = u & 1;
    const uint8_t* chunk = chunk_at(c);
    const uint2 qa = *reinterpret_cast<const uint2*>(chunk + g * TILE_K + 16 * t + 8 * h);
    const uint2 qb = *reinterpret_cast<const uint2*>(chunk + (g + 8) * TILE_K + 16 * t + 8 * h);
    const uint4 ha = dq8_f16<QF>(qa, chunk + CHUNK_Q, g, 2 * t + h);
    const uint4 hb = dq8_f16<QF>(qb, chunk + CHUNK_Q, g + 8, 2 * t + h);
    const int k = c * TILE_K + 16 * t + 8 * h;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
      const uint4 b = bload(nt, k);
      mma16816(acc[nt], ha.x, hb.x, ha.y, hb.y, b.x, b.y);
      mma16816(acc[nt], ha.z, hb.z, ha.w, hb.w, b.z, b.w);
    }
  }
}

// Shared-memory partials of the 8 warps: red[w][nt][lane] float4.
template <int NT>
__device__ __forceinline__ void store_partials(float4* red, const float (&acc)[NT][4]) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
    red[(w * NT + nt) * 32 + lane] = make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
}

// Output item i (< 64 * NT) of a tile after store_partials of its `ns`
// slices (slice s at red + s * WARPS * NT * 32): the pair index q (0..7, the
// tile's row pair), the token and the two sums: over the warps in order
// 0..7 per slice, then the slices in order.
template <int NT>
__device__ __forceinline__ void reduce_item(const float4* red, int i, int* q, int* token, float* va, float* vb,
                                            int ns = 1) {
  const int nt = i >> 6, j = i & 63, lane = j >> 1, which = j & 1;
  *q = lane >> 2;
  *token = 8 * nt + 2 * (lane & 3) + which;
  float A = 0.f, B = 0.f;
  for (int s = 0; s < ns; s++) {
    const float4* rs = red + s * WARPS * NT * 32;
    const float* r0 = reinterpret_cast<const float*>(&rs[nt * 32 + lane]);
    float a = r0[which], b = r0[which + 2];
#pragma unroll
    for (int w = 1; w < WARPS; w++) {
      const float* r = reinterpret_cast<const float*>(&rs[(w * NT + nt) * 32 + lane]);
      a = __fadd_rn(a, r[which]);
      b = __fadd_rn(b, r[which + 2]);
    }
    A = s == 0 ? a : __fadd_rn(A, a);
    B = s == 0 ? b : __fadd_rn(B, b);
  }
  *va = A;
  *vb = B;
}

// Virtual row `a` of epi_pair (epilogue.cuh) for pair q of tile j.
__device__ __forceinline__ int pair_virtual_row(int mode, int j, int q) {
  if (mode == EPI_GEGLU) {
    const int f = 8 * j + q;
    return (f / GEGLU_HALF) * TILE_N + (f % GEGLU_HALF);
  }
  return 16 * j + 2 * q;
}

// Number of row16 tiles of a weight with n_out real outputs.
__host__ __device__ inline int n_tiles(int mode_geglu, int n_out) {
  return mode_geglu ? (n_out + 7) / 8 : (n_out + 15) / 16;
}

}  // namespace r16
}  // namespace le
