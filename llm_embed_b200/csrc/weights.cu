// Weight upload support: GGUF block decode, repack into the tile-blocked
// layout (common.cuh), and exact dequantisation back to [N][K] float32.
#include "dequant.cuh"
#include "gemm_r16.cuh"
#include "gguf_decode.cuh"
#include "kernels.h"

namespace le {

// One thread per (virtual row, 64-column k-step).  Virtual row v maps to a
// source row: identity (src0), or for the merged FFN up/gate matrix, tile
// t = v/128 holds up rows 64t..64t+63 (src0) then gate rows 64t..64t+63
// (src1).
template <int TYPE>
__global__ void repack_kernel(const uint8_t* __restrict__ src0, const uint8_t* __restrict__ src1, long src_row_bytes,
                              int N_src, int K, int n_tiles, int interleave, uint8_t* __restrict__ dst) {
  constexpr int QF = qfmt_of(TYPE);
  const int ksteps = K / TILE_K;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)n_tiles * TILE_N * ksteps) return;
  const int ks = (int)(idx % ksteps);
  const int v = (int)(idx / ksteps);
  const int t = v / TILE_N, r = v % TILE_N;
  const uint8_t* row = nullptr;
  if (interleave) {
    const int srow = t * (TILE_N / 2) + (r % (TILE_N / 2));
    if (srow < N_src) row = (r < TILE_N / 2 ? src0 : src1) + (long)srow * src_row_bytes;
  } else if (v < N_src) {
    row = src0 + (long)v * src_row_bytes;
  }
  uint8_t* chunk = dst + ((long)t * ksteps + ks) * chunk_bytes(QF);
  uint8_t* q = chunk + r * TILE_K;
  uint8_t* meta = chunk + TILE_Q_BYTES;
  const int k0 = ks * TILE_K;
  if (!row) {
    for (int c = 0; c < TILE_K; c++) q[c] = 128;
    for (int i = 0; i < meta_bytes(QF) / TILE_N; i++) meta[r * (meta_bytes(QF) / TILE_N) + i] = 0;
    return;
  }
  if constexpr (TYPE == T_Q8_0) {
    uint16_t* dm = reinterpret_cast<uint16_t*>(meta) + r * 2;
    for (int blk = 0; blk < 2; blk++) {
      const uint8_t* b = row + ((k0 >> 5) + blk) * 34;
      dm[blk] = rd16(b);
      for (int i = 0; i < 32; i++) q[blk * 32 + i] = (uint8_t)((int)(int8_t)b[2 + i] + 128);
    }
  } else if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
    constexpr int bs = TYPE == T_Q4_K ? 144 : 176;
    const uint8_t* b = row + (k0 >> 8) * bs;
    const int j = (k0 & 255) >> 6;  // 64-element group inside the super-block
    float2* sm = reinterpret_cast<float2*>(meta) + r * 2;
    const float d = f16_bits_to_f32(rd16(b)), dmin = f16_bits_to_f32(rd16(b + 2));
    for (int hi = 0; hi < 2; hi++) {
      int sc, m;
      scale_min_k4(2 * j + hi, b + 4, &sc, &m);
      sm[hi] = make_float2(__fmul_rn(d, (float)sc), __fmul_rn(dmin, (float)m));
      for (int l = 0; l < 32; l++) {
        int qq;
        if (TYPE == T_Q4_K)
          qq = (b[16 + 32 * j + l] >> (4 * hi)) & 0xF;
        else
          qq = ((b[48 + 32 * j + l] >> (4 * hi)) & 0xF) | (((b[16 + l] >> (2 * j + hi)) & 1) << 4);
        q[hi * 32 + l] = (uint8_t)(qq + 128);
      }
    }
  } else {  // Q6_K
    const uint8_t* b = row + (k0 >> 8) * 210;
    const float d = f16_bits_to_f32(rd16(b + 208));
    const int w0 = k0 & 255;
    float* ds = reinterpret_cast<float*>(meta) + r * 4;
    for (int i = 0; i < 4; i++) ds[i] = __fmul_rn(d, (float)(int8_t)b[192 + ((w0 >> 4) + i)]);
    for (int c = 0; c < 64; c++) {
      const int w = w0 + c, nn = w >> 7, rr = w & 127, gq = rr >> 5, l = rr & 31;
      const uint8_t* ql = b + nn * 64;
      const uint8_t* qh = b + 128 + nn * 32;
      const int lo = (gq & 1) ? ql[l + 32] : ql[l];
      const int nib = (gq >> 1) ? (lo >> 4) : (lo & 0xF);
      q[c] = (uint8_t)((nib | (((qh[l] >> (2 * gq)) & 3) << 4)) - 32 + 128);
    }
  }
}

// Exact (mode 0) or fp16-operand (mode 1) dequant of the tile layout into
// [n_rows][K] float32, virtual row order.
template <int QF>
__global__ void dequant_tiles_kernel(const uint8_t* __restrict__ w, int n_rows, int K, int mode, float* __restrict__ out) {
  const int ksteps = K / TILE_K;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;  // (row, k-step, group)
  if (idx >= (long)n_rows * ksteps * 8) return;
  const int g = (int)(idx & 7);
  const int ks = (int)((idx >> 3) % ksteps);
  const int v = (int)((idx >> 3) / ksteps);
  const int t = v / TILE_N, r = v % TILE_N;
  const uint8_t* chunk = w + ((long)t * ksteps + ks) * chunk_bytes(QF);
  const uint2 u = *reinterpret_cast<const uint2*>(chunk + r * TILE_K + g * 8);
  float* o = out + (long)v * K + ks * TILE_K + g * 8;
  if (mode == 0) {
    dq8_f32<QF>(u, chunk + TILE_Q_BYTES, r, g, o);
  } else {
    uint4 h = dq8_f16<QF>(u, chunk + TILE_Q_BYTES, r, g);
    const __half2* hh = reinterpret_cast<const __half2*>(&h);
    for (int i = 0; i < 4; i++) {
      float2 f = __half22float2(hh[i]);
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  }
}

// fp16 tensor-core operands of the tile layout as a row-major [n_rows][K]
// fp16 matrix (virtual row order), the B operand of the large-batch GEMM:
// the same dq8_f16 values the in-shared-memory dequant produces.
template <int QF>
__global__ void expand_f16_kernel(const uint8_t* __restrict__ w, int n_rows, int K, __half* __restrict__ out) {
  const int ksteps = K / TILE_K;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;  // (row, k-step, group)
  if (idx >= (long)n_rows * ksteps * 8) return;
  const int g = (int)(idx & 7);
  const int ks = (int)((idx >> 3) % ksteps);
  const int v = (int)((idx >> 3) / ksteps);
  const int t = v / TILE_N, r = v % TILE_N;
  const uint8_t* chunk = w + ((long)t * ksteps + ks) * chunk_bytes(QF);
  const uint2 u = *reinterpret_cast<const uint2*>(chunk + r * TILE_K + g * 8);
  *reinterpret_cast<uint4*>(out + (long)v * K + ks * TILE_K + g * 8) = dq8_f16<QF>(u, chunk + TILE_Q_BYTES, r, g);
}

// F32 weight rows (DequantWeightMatrix case 0, gemm.go:257-263: the values
// themselves) to the fp16 operand matrix [n_virt][K] in virtual row order
// (the merged up/gate order of repack_kernel when interleave), rows past the
// source zero.  One thread per 8 consecutive elements.
__global__ void f32_rows_to_f16_kernel(const float* __restrict__ src0, const float* __restrict__ src1, int N_src, int K,
                                       int n_virt, int interleave, __half* __restrict__ out) {
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int groups = K / 8;
  if (idx >= (long)n_virt * groups) return;
  const int v = (int)(idx / groups), c = (int)(idx % groups) * 8;
  const float* row = nullptr;
  if (interleave) {
    const int t = v / TILE_N, r = v % TILE_N, srow = t * (TILE_N / 2) + (r % (TILE_N / 2));
    if (srow < N_src) row = (r < TILE_N / 2 ? src0 : src1) + (long)srow * K;
  } else if (v < N_src) {
    row = src0 + (long)v * K;
  }
  uint4 h = make_uint4(0, 0, 0, 0);
  if (row) {
    const float4 a = *reinterpret_cast<const float4*>(row + c);
    const float4 b = *reinterpret_cast<const float4*>(row + c + 4);
    h = make_uint4(pack_half2(a.x, a.y), pack_half2(a.z, a.w), pack_half2(b.x, b.y), pack_half2(b.z, b.w));
  }
  *reinterpret_cast<uint4*>(out + (long)v * K + c) = h;
}

// The row16 layout (gemm_r16.cuh) from the 128-row tile layout: one thread
// per (tile, 64-column chunk, row) copies the row's 64 quant bytes and its
// metadata.  Tile j row r takes virtual row v: for the merged up/gate matrix
// (geglu) up[8j + r] (r < 8) or gate[8j + r - 8] in the 128-row tiles' order
// (64 up rows then 64 gate rows per tile), otherwise feature 16j + 2r
// (r < 8) or 16j + 2(r - 8) + 1.
template <int QF>
__global__ void repack_r16_kernel(const uint8_t* __restrict__ t128, int K, int geglu, int tiles,
                                  uint8_t* __restrict__ out) {
  const int ksteps = K / TILE_K;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)tiles * ksteps * r16::ROWS) return;
  const int r = (int)(idx % r16::ROWS);
  const int c = (int)((idx / r16::ROWS) % ksteps);
  const int j = (int)(idx / r16::ROWS / ksteps);
  int v;
  if (geglu) {
    const int f = 8 * j + (r & 7);
    v = (f / (TILE_N / 2)) * TILE_N + (r < 8 ? 0 : TILE_N / 2) + f % (TILE_N / 2);
  } else {
    v = 16 * j + (r < 8 ? 2 * r : 2 * (r - 8) + 1);
  }
  constexpr int MRB = r16::meta_row_bytes(QF);
  const uint8_t* src = t128 + ((long)(v / TILE_N) * ksteps + c) * chunk_bytes(QF);
  const int sr = v % TILE_N;
  uint8_t* dst = out + ((long)j * ksteps + c) * r16::chunk_bytes(QF);
  const uint4* q = reinterpret_cast<const uint4*>(src + sr * TILE_K);
  uint4* d = reinterpret_cast<uint4*>(dst + r * TILE_K);
#pragma unroll
  for (int i = 0; i < 4; i++) d[i] = q[i];
  const uint8_t* ms = src + TILE_Q_BYTES + sr * MRB;
  uint8_t* md = dst + r16::CHUNK_Q + r * MRB;
  if constexpr (MRB == 16) {
    *reinterpret_cast<uint4*>(md) = *reinterpret_cast<const uint4*>(ms);
  } else {
    *reinterpret_cast<uint32_t*>(md) = *reinterpret_cast<const uint32_t*>(ms);
  }
}

// Dequantise whole GGUF rows (used for the embedding table check).
__global__ void gguf_rows_kernel(int type, const uint8_t* __restrict__ src, long row_bytes, int n_rows, int K,
                                 float* __restrict__ out) {
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)n_rows * K) return;
  const int e = (int)(idx % K);
  const long rr = idx / K;
  out[idx] = gguf_elem(type, src + rr * row_bytes, e);
}

cudaError_t launch_repack(int type, const uint8_t* src0, const uint8_t* src1, long src_row_bytes, int N_src, int K,
                          int n_tiles, int interleave, uint8_t* dst, cudaStream_t s) {
  const long n = (long)n_tiles * TILE_N * (K / TILE_K);
  const int bs = 128;
  const unsigned grid = (unsigned)((n + bs - 1) / bs);
  switch (type) {
    case T_Q8_0: repack_kernel<T_Q8_0><<<grid, bs, 0, s>>>(src0, src1, src_row_bytes, N_src, K, n_tiles, interleave, dst); break;
    case T_Q4_K: repack_kernel<T_Q4_K><<<grid, bs, 0, s>>>(src0, src1, src_row_bytes, N_src, K, n_tiles, interleave, dst); break;
    case T_Q5_K: repack_kernel<T_Q5_K><<<grid, bs, 0, s>>>(src0, src1, src_row_bytes, N_src, K, n_tiles, interleave, dst); break;
    case T_Q6_K: repack_kernel<T_Q6_K><<<grid, bs, 0, s>>>(src0, src1, src_row_bytes, N_src, K, n_tiles, interleave, dst); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_dequant_tiles(int qf, const uint8_t* w, int n_rows, int K, int mode, float* out, cudaStream_t s) {
  const long n = (long)n_rows * (K / TILE_K) * 8;
  const int bs = 256;
  const unsigned grid = (unsigned)((n + bs - 1) / bs);
  switch (qf) {
    case QF_Q8_0: dequant_tiles_kernel<QF_Q8_0><<<grid, bs, 0, s>>>(w, n_rows, K, mode, out); break;
    case QF_KMIN: dequant_tiles_kernel<QF_KMIN><<<grid, bs, 0, s>>>(w, n_rows, K, mode, out); break;
    case QF_Q6K: dequant_tiles_kernel<QF_Q6K><<<grid, bs, 0, s>>>(w, n_rows, K, mode, out); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_gguf_rows(int type, const uint8_t* src, long row_bytes, int n_rows, int K, float* out, cudaStream_t s) {
  const long n = (long)n_rows * K;
  gguf_rows_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(type, src, row_bytes, n_rows, K, out);
  return cudaGetLastError();
}

cudaError_t launch_repack_r16(int qf, const uint8_t* t128, int K, int geglu, int tiles, uint8_t* out,
                              cudaStream_t s) {
  const long n = (long)tiles * (K / TILE_K) * r16::ROWS;
  const unsigned grid = (unsigned)((n + 255) / 256);
  switch (qf) {
    case QF_Q8_0: repack_r16_kernel<QF_Q8_0><<<grid, 256, 0, s>>>(t128, K, geglu, tiles, out); break;
    case QF_KMIN: repack_r16_kernel<QF_KMIN><<<grid, 256, 0, s>>>(t128, K, geglu, tiles, out); break;
    case QF_Q6K: repack_r16_kernel<QF_Q6K><<<grid, 256, 0, s>>>(t128, K, geglu, tiles, out); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_f32_rows_to_f16(const float* src0, const float* src1, int N_src, int K, int n_virt, int interleave,
                                   __half* out, cudaStream_t s) {
  if (K % 8) return cudaErrorInvalidValue;
  const long n = (long)n_virt * (K / 8);
  f32_rows_to_f16_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(src0, src1, N_src, K, n_virt, interleave, out);
  return cudaGetLastError();
}

cudaError_t launch_expand_f16(int qf, const uint8_t* w, int n_rows, int K, __half* out, cudaStream_t s) {
  const long n = (long)n_rows * (K / TILE_K) * 8;
  const int bs = 256;
  const unsigned grid = (unsigned)((n + bs - 1) / bs);
  switch (qf) {
    case QF_Q8_0: expand_f16_kernel<QF_Q8_0><<<grid, bs, 0, s>>>(w, n_rows, K, out); break;
    case QF_KMIN: expand_f16_kernel<QF_KMIN><<<grid, bs, 0, s>>>(w, n_rows, K, out); break;
    case QF_Q6K: expand_f16_kernel<QF_Q6K><<<grid, bs, 0, s>>>(w, n_rows, K, out); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace le
