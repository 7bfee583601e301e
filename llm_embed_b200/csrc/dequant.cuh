// Dequantisation of the tile-blocked weight format (see common.cuh).
//
// Two forms are provided for every format:
//   * dq8_f32:  the exact float32 values the reference computes
//               (tensor.go:291, quant_q4k.go:64-68, quant_q5k.go:216-226,
//               quant_q6k.go:362-365); used by le_dequant's bit-exact check
//               and as the definition of the fp16 operands below.
//   * dq8_f16:  the tensor-core operand, round-to-nearest fp16 of the exact
//               float32 value.  For Q8_0 it is computed in fp16 arithmetic:
//               int8 q and the fp16 scale d are exact in fp16 and q*d needs
//               at most 19 significant bits, so one fp16 multiply rounds the
//               exact product once -- the same value as rounding the exact
//               float32 product.  The K-quant formats go through float32.
#pragma once
#include "common.cuh"

namespace le {

// Eight consecutive elements (columns 8g..8g+7 of a 64-column tile) of one
// tile row: the 8 biased quant bytes and that row's metadata pointer.
struct Q8 {
  uint2 u;  // bytes q+128, little-endian element order
};

// fp16 magic: bits 0x6400|u is 1024+u exactly; subtract 1152 -> u-128.
__device__ __forceinline__ uint32_t bias_bytes_to_h2(uint32_t w, uint32_t sel) {
  return __byte_perm(w, 0x64646464u, sel);
}

__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t h2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// float32 magic: bits 0x4B000000|u is 8388608+u exactly.
__device__ __forceinline__ float byte_to_q(uint32_t w, int i) {
  uint32_t bits = __byte_perm(w, 0x4B000000u, 0x7440u | (uint32_t)i);
  return __fsub_rn(__uint_as_float(bits), 8388736.0f);  // (8388608 + u) - (8388608 + 128)
}

// Metadata accessors.  `meta` points at the tile's metadata block; `r` is
// the tile row; `g` the 8-column group (0..7) inside the 64-column tile.
template <int QF>
struct Meta;

template <>
struct Meta<QF_Q8_0> {
  // half d[256][2]
  __device__ __forceinline__ static uint32_t d_h2(const uint8_t* meta, int r, int g) {
    uint16_t d = reinterpret_cast<const uint16_t*>(meta)[r * 2 + (g >> 2)];
    return (uint32_t)d | ((uint32_t)d << 16);
  }
  __device__ __forceinline__ static float d_f32(const uint8_t* meta, int r, int g) {
    uint16_t d = reinterpret_cast<const uint16_t*>(meta)[r * 2 + (g >> 2)];
    return __half2float(__ushort_as_half(d));
  }
};

// Exact float32 dequant of 8 elements.
template <int QF>
__device__ __forceinline__ void dq8_f32(uint2 u, const uint8_t* meta, int r, int g, float* out) {
  if constexpr (QF == QF_Q8_0) {
    float d = Meta<QF_Q8_0>::d_f32(meta, r, g);
#pragma unroll
    for (int i = 0; i < 4; i++) out[i] = __fmul_rn(byte_to_q(u.x, i), d);
#pragma unroll
    for (int i = 0; i < 4; i++) out[4 + i] = __fmul_rn(byte_to_q(u.y, i), d);
  } else if constexpr (QF == QF_KMIN) {
    const float2 sm = reinterpret_cast<const float2*>(meta)[r * 2 + (g >> 2)];  // {d*sc, dmin*m}
#pragma unroll
    for (int i = 0; i < 4; i++) out[i] = __fsub_rn(__fmul_rn(sm.x, byte_to_q(u.x, i)), sm.y);
#pragma unroll
    for (int i = 0; i < 4; i++) out[4 + i] = __fsub_rn(__fmul_rn(sm.x, byte_to_q(u.y, i)), sm.y);
  } else {
    const float ds = reinterpret_cast<const float*>(meta)[r * 4 + (g >> 1)];  // d*sc per 16
#pragma unroll
    for (int i = 0; i < 4; i++) out[i] = __fmul_rn(ds, byte_to_q(u.x, i));
#pragma unroll
    for (int i = 0; i < 4; i++) out[4 + i] = __fmul_rn(ds, byte_to_q(u.y, i));
  }
}

// fp16 operand form of 8 elements, packed as 4 x half2 (element order).
template <int QF>
__device__ __forceinline__ uint4 dq8_f16(uint2 u, const uint8_t* meta, int r, int g) {
  uint4 o;
  if constexpr (QF == QF_Q8_0) {
    const uint32_t d2 = Meta<QF_Q8_0>::d_h2(meta, r, g);
    const uint32_t k1152 = 0x64806480u;  // half2(1152, 1152)
    o.x = h2_mul(h2_sub(bias_bytes_to_h2(u.x, 0x5140u), k1152), d2);
    o.y = h2_mul(h2_sub(bias_bytes_to_h2(u.x, 0x5342u), k1152), d2);
    o.z = h2_mul(h2_sub(bias_bytes_to_h2(u.y, 0x5140u), k1152), d2);
    o.w = h2_mul(h2_sub(bias_bytes_to_h2(u.y, 0x5342u), k1152), d2);
  } else {
    float f[8];
    dq8_f32<QF>(u, meta, r, g, f);
    o.x = pack_half2(f[0], f[1]);
    o.y = pack_half2(f[2], f[3]);
    o.z = pack_half2(f[4], f[5]);
    o.w = pack_half2(f[6], f[7]);
  }
  return o;
}

}  // namespace le
