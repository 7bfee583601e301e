// Mean pool + L2 normalisation + Matryoshka truncation of one sequence
// (pool.go:8-53, embedder.go:59-68), shared by the pool kernel
// (elementwise.cu) and the single-kernel small forward (forward_small.cu)
// so both give the same bits.
#pragma once
#include "common.cuh"

namespace le {

__device__ __forceinline__ double pool_warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Rows t0 .. t1-1 of h (row stride H; global or shared memory) -> out_row
// [out_dim]: masked mean (f32 sum in token order, x (1/count)), L2
// normalise (float64 sum of squares: per warp, then the warps in order;
// float32 multiply by float32(1/norm)), then truncation to out_dim and
// renormalisation.  Called by threads 0 .. H/4-1 (whole warps), thread i
// owning columns 4i..4i+3; `sync` is their barrier, `red` 32 doubles of
// shared memory.  U rows' loads are in flight at once (their sum is still
// formed in token order).  An empty sequence gives a zero vector.
template <int U, class Sync>
__device__ __forceinline__ void pool_seq(const float* h, int t0, int t1, int H, int out_dim, float* out_row,
                                         double* red, Sync sync) {
  const int c = threadIdx.x * 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (c < H) {
    for (int t = t0; t < t1; t += U) {
      float4 v[U];
#pragma unroll
      for (int u = 0; u < U; u++)
        if (t + u < t1) v[u] = *reinterpret_cast<const float4*>(h + (long)(t + u) * H + c);
#pragma unroll
      for (int u = 0; u < U; u++)
        if (t + u < t1) {
          acc.x += v[u].x;
          acc.y += v[u].y;
          acc.z += v[u].z;
          acc.w += v[u].w;
        }
    }
    if (t1 > t0) {
      const float inv = __fdiv_rn(1.0f, (float)(t1 - t0));
      acc.x = __fmul_rn(acc.x, inv);
      acc.y = __fmul_rn(acc.y, inv);
      acc.z = __fmul_rn(acc.z, inv);
      acc.w = __fmul_rn(acc.w, inv);
    }
  }
  float v[4] = {acc.x, acc.y, acc.z, acc.w};
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = (H / 4 + 31) >> 5;
  for (int pass = 0; pass < 2; pass++) {
    const int lim = pass == 0 ? H : out_dim;
    if (pass == 1 && out_dim >= H) break;
    double sq = 0.0;
    for (int i = 0; i < 4; i++)
      if (c + i < lim) sq += (double)v[i] * (double)v[i];
    sq = pool_warp_sum_d(sq);
    sync();
    if (lane == 0) red[warp] = sq;
    sync();
    double tot = 0.0;
    for (int i = 0; i < nw; i++) tot += red[i];
    const double norm = sqrt(tot);
    if (norm != 0.0) {
      const float inv = (float)(1.0 / norm);
      for (int i = 0; i < 4; i++) v[i] = __fmul_rn(v[i], inv);
    }
  }
  for (int i = 0; i < 4; i++)
    if (c + i < out_dim) out_row[c + i] = v[i];
}

}  // namespace le
