// Exact float32 decode of GGUF rows, as the reference's getEmbedding /
// Dequantize compute them.
#pragma once
#include "common.cuh"

namespace le {

__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// quant_q4k.go:133-140 (getScaleMinK4).
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* s, int* sc, int* m) {
  if (j < 4) {
    *sc = s[j] & 63;
    *m = s[j + 4] & 63;
  } else {
    *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
    *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

// Exact float32 value of element e of a GGUF row (bert.go:290 getEmbedding
// semantics for F32 / Q8_0 / Q4_K / Q5_K / Q6_K).
__device__ __forceinline__ float gguf_elem(int type, const uint8_t* row, int e) {
  switch (type) {
    case T_F32: {
      float v;
      memcpy(&v, row + 4 * (size_t)e, 4);
      return v;
    }
    case T_Q8_0: {  // tensor.go:279-293
      const uint8_t* b = row + (e >> 5) * 34;
      return __fmul_rn((float)(int8_t)b[2 + (e & 31)], f16_bits_to_f32(rd16(b)));
    }
    case T_Q4_K:
    case T_Q5_K: {  // quant_q4k.go:36-74, quant_q5k.go:183-233
      const int bs = type == T_Q4_K ? 144 : 176;
      const uint8_t* b = row + (e >> 8) * bs;
      const int w = e & 255, j = w >> 6, hi = (w >> 5) & 1, l = w & 31;
      int sc, m;
      scale_min_k4(2 * j + hi, b + 4, &sc, &m);
      const float d1 = __fmul_rn(f16_bits_to_f32(rd16(b)), (float)sc);
      const float dm1 = __fmul_rn(f16_bits_to_f32(rd16(b + 2)), (float)m);
      int q;
      if (type == T_Q4_K) {
        q = (b[16 + 32 * j + l] >> (4 * hi)) & 0xF;
      } else {
        q = ((b[48 + 32 * j + l] >> (4 * hi)) & 0xF) | (((b[16 + l] >> (2 * j + hi)) & 1) << 4);
      }
      return __fsub_rn(__fmul_rn(d1, (float)q), dm1);
    }
    case T_Q6_K: {  // quant_q6k.go:331-371
      const uint8_t* b = row + (e >> 8) * 210;
      const int w = e & 255, nn = w >> 7, r = w & 127, gq = r >> 5, l = r & 31;
      const uint8_t* ql = b + nn * 64;
      const uint8_t* qh = b + 128 + nn * 32;
      const int lo = (gq & 1) ? ql[l + 32] : ql[l];
      const int nib = (gq >> 1) ? (lo >> 4) : (lo & 0xF);
      const int q = (nib | (((qh[l] >> (2 * gq)) & 3) << 4)) - 32;
      const int sc = (int8_t)b[192 + nn * 8 + (l >> 4) + 2 * gq];
      const float d = f16_bits_to_f32(rd16(b + 208));
      return __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
    }
  }
  return 0.f;
}

// Elements e .. e+3 (e a multiple of 4: one quant block, one sub-block of
// 32) with gguf_elem's arithmetic per element, the block's scales decoded
// once.
__device__ __forceinline__ float4 gguf_elem4(int type, const uint8_t* row, int e) {
  switch (type) {
    case T_Q8_0: {
      const uint8_t* b = row + (e >> 5) * 34;
      const float d = f16_bits_to_f32(rd16(b));
      const uint8_t* q = b + 2 + (e & 31);
      return make_float4(__fmul_rn((float)(int8_t)q[0], d), __fmul_rn((float)(int8_t)q[1], d),
                         __fmul_rn((float)(int8_t)q[2], d), __fmul_rn((float)(int8_t)q[3], d));
    }
    case T_Q4_K:
    case T_Q5_K: {
      const int bs = type == T_Q4_K ? 144 : 176;
      const uint8_t* b = row + (e >> 8) * bs;
      const int w = e & 255, j = w >> 6, hi = (w >> 5) & 1, l = w & 31;
      int sc, m;
      scale_min_k4(2 * j + hi, b + 4, &sc, &m);
      const float d1 = __fmul_rn(f16_bits_to_f32(rd16(b)), (float)sc);
      const float dm1 = __fmul_rn(f16_bits_to_f32(rd16(b + 2)), (float)m);
      float r[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        int q;
        if (type == T_Q4_K) {
          q = (b[16 + 32 * j + l + i] >> (4 * hi)) & 0xF;
        } else {
          q = ((b[48 + 32 * j + l + i] >> (4 * hi)) & 0xF) | (((b[16 + l + i] >> (2 * j + hi)) & 1) << 4);
        }
        r[i] = __fsub_rn(__fmul_rn(d1, (float)q), dm1);
      }
      return make_float4(r[0], r[1], r[2], r[3]);
    }
    case T_Q6_K: {
      const uint8_t* b = row + (e >> 8) * 210;
      const int w = e & 255, nn = w >> 7, r0 = w & 127, gq = r0 >> 5, l = r0 & 31;
      const uint8_t* ql = b + nn * 64;
      const uint8_t* qh = b + 128 + nn * 32;
      const int sc = (int8_t)b[192 + nn * 8 + (l >> 4) + 2 * gq];
      const float ds = __fmul_rn(f16_bits_to_f32(rd16(b + 208)), (float)sc);
      float r[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int lo = (gq & 1) ? ql[l + i + 32] : ql[l + i];
        const int nib = (gq >> 1) ? (lo >> 4) : (lo & 0xF);
        const int q = (nib | (((qh[l + i] >> (2 * gq)) & 3) << 4)) - 32;
        r[i] = __fmul_rn(ds, (float)q);
      }
      return make_float4(r[0], r[1], r[2], r[3]);
    }
  }
  return make_float4(gguf_elem(type, row, e), gguf_elem(type, row, e + 1), gguf_elem(type, row, e + 2),
                     gguf_elem(type, row, e + 3));
}

}  // namespace le
