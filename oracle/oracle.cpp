/*
 * TEST INFRASTRUCTURE — NOT PART OF THE PRODUCT.  See oracle.h for the rules
 * on who may load this file and for its parity status.
 *
 * CPU restatement of dbrushchenko/llm-embed's encoder path.  Every function
 * names the reference file:line it follows.  Floating-point expressions keep
 * the reference's evaluation order; the build uses -ffp-contract=off so that
 * only the explicit fmaf() calls (which stand for the asm micro-kernel's
 * VFMADD231PS) are fused, as Go on amd64 (GOAMD64=v1) emits no FMA itself.
 */
#include "oracle.h"

#include <immintrin.h>
#include <omp.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

/* ---------------------------------------------------------------- f16 ---- */

/* internal/ggml/tensor.go:162-191 (f16ToF32; subnormals are normalised).
 * f16ToF32Fast (ops_fast.go:229) computes the same values. */
float f16_to_f32(uint16_t h) {
  uint32_t sign = (h >> 15) & 1u;
  int32_t exp = (h >> 10) & 0x1f;
  uint32_t mant = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (mant == 0) {
      bits = sign << 31;
    } else {
      while ((mant & 0x400u) == 0) {
        mant <<= 1;
        exp--;
      }
      exp++;
      mant &= 0x3ffu;
      bits = (sign << 31) | ((uint32_t)(exp + 127 - 15) << 23) | (mant << 13);
    }
  } else if (exp < 31) {
    bits = (sign << 31) | ((uint32_t)(exp + 127 - 15) << 23) | (mant << 13);
  } else {
    bits = (sign << 31) | (0xffu << 23) | (mant << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* ------------------------------------------------------------ dequant ---- */

/* tensor.go:267-296 (dequantQ8_0) and gemm.go:270-282 (dequantQ8_0Row):
 * value = float32(int8 q) * f16(d). */
void dequant_q8_0(const uint8_t* data, long n, float* out) {
  long nb = n / 32;
  for (long b = 0; b < nb; b++) {
    const uint8_t* blk = data + b * 34;
    float scale = f16_to_f32(rd16(blk));
    for (int i = 0; i < 32; i++) out[b * 32 + i] = (float)(int8_t)blk[2 + i] * scale;
  }
}

/* quant_q4k.go:133-140 (getScaleMinK4). */
inline void scale_min_k4(int j, const uint8_t* s, uint8_t* sc, uint8_t* m) {
  if (j < 4) {
    *sc = s[j] & 63;
    *m = s[j + 4] & 63;
  } else {
    *sc = (uint8_t)((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
    *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
  }
}

/* quant_q4k.go:27-77 (DequantQ4_K): d1 = d*sc, dm1 = dmin*m, v = d1*q - dm1. */
void dequant_q4_k(const uint8_t* data, long n, float* out) {
  long nb = n / 256;
  for (long b = 0; b < nb; b++) {
    const uint8_t* blk = data + b * 144;
    float d = f16_to_f32(rd16(blk));
    float dmin = f16_to_f32(rd16(blk + 2));
    const uint8_t* scales = blk + 4;
    const uint8_t* qs = blk + 16;
    float* o = out + b * 256;
    int is = 0, qoff = 0;
    for (int j = 0; j < 256; j += 64) {
      uint8_t sc1, m1, sc2, m2;
      scale_min_k4(is, scales, &sc1, &m1);
      scale_min_k4(is + 1, scales, &sc2, &m2);
      float d1 = d * (float)sc1, dm1 = dmin * (float)m1;
      float d2 = d * (float)sc2, dm2 = dmin * (float)m2;
      for (int l = 0; l < 32; l++) o[j + l] = d1 * (float)(qs[qoff + l] & 0xF) - dm1;
      for (int l = 0; l < 32; l++) o[j + 32 + l] = d2 * (float)(qs[qoff + l] >> 4) - dm2;
      qoff += 32;
      is += 2;
    }
  }
}

/* quant_q5k.go:29-236 (DequantQ5_K): as Q4_K plus bit `qhBit` of qh[l]. */
void dequant_q5_k(const uint8_t* data, long n, float* out) {
  long nb = n / 256;
  for (long b = 0; b < nb; b++) {
    const uint8_t* blk = data + b * 176;
    float d = f16_to_f32(rd16(blk));
    float dmin = f16_to_f32(rd16(blk + 2));
    const uint8_t* scales = blk + 4;
    const uint8_t* qh = blk + 16;
    const uint8_t* qs = blk + 48;
    float* o = out + b * 256;
    int is = 0, qoff = 0;
    unsigned qhbit = 0;
    for (int j = 0; j < 256; j += 64) {
      uint8_t sc1, m1, sc2, m2;
      scale_min_k4(is, scales, &sc1, &m1);
      scale_min_k4(is + 1, scales, &sc2, &m2);
      float d1 = d * (float)sc1, dm1 = dmin * (float)m1;
      float d2 = d * (float)sc2, dm2 = dmin * (float)m2;
      for (int l = 0; l < 32; l++) {
        uint8_t q = (uint8_t)((qs[qoff + l] & 0xF) | (((qh[l] >> qhbit) & 1) << 4));
        o[j + l] = d1 * (float)q - dm1;
      }
      qhbit++;
      for (int l = 0; l < 32; l++) {
        uint8_t q = (uint8_t)((qs[qoff + l] >> 4) | (((qh[l] >> qhbit) & 1) << 4));
        o[j + 32 + l] = d2 * (float)q - dm2;
      }
      qhbit++;
      qoff += 32;
      is += 2;
    }
  }
}

/* quant_q6k.go:23-84 (DequantQ6_K): v = (d * float32(sc)) * float32(q - 32). */
void dequant_q6_k(const uint8_t* data, long n, float* out) {
  long nb = n / 256;
  for (long b = 0; b < nb; b++) {
    const uint8_t* blk = data + b * 210;
    const uint8_t* ql = blk;
    const uint8_t* qh = blk + 128;
    const int8_t* sc = (const int8_t*)(blk + 192);
    float d = f16_to_f32(rd16(blk + 208));
    float* o = out + b * 256;
    for (int nn = 0; nn < 256; nn += 128) {
      int qloff = nn / 2, qhoff = nn / 4, scoff = nn / 16;
      for (int l = 0; l < 32; l++) {
        int is = l / 16;
        int8_t q1 = (int8_t)((ql[qloff + l] & 0xF) | (((qh[qhoff + l] >> 0) & 3) << 4)) - 32;
        int8_t q2 = (int8_t)((ql[qloff + l + 32] & 0xF) | (((qh[qhoff + l] >> 2) & 3) << 4)) - 32;
        int8_t q3 = (int8_t)((ql[qloff + l] >> 4) | (((qh[qhoff + l] >> 4) & 3) << 4)) - 32;
        int8_t q4 = (int8_t)((ql[qloff + l + 32] >> 4) | (((qh[qhoff + l] >> 6) & 3) << 4)) - 32;
        o[nn + l] = d * (float)sc[scoff + is + 0] * (float)q1;
        o[nn + l + 32] = d * (float)sc[scoff + is + 2] * (float)q2;
        o[nn + l + 64] = d * (float)sc[scoff + is + 4] * (float)q3;
        o[nn + l + 96] = d * (float)sc[scoff + is + 6] * (float)q4;
      }
    }
  }
}

long row_bytes(int type, long n) {
  switch (type) {
    case OR_F32: return n * 4;
    case OR_Q8_0: return n / 32 * 34;
    case OR_Q4_K: return n / 256 * 144;
    case OR_Q5_K: return n / 256 * 176;
    case OR_Q6_K: return n / 256 * 210;
    default: return -1;
  }
}

/* tensor.go:51-68 (Dequantize). */
int dequant(int type, const uint8_t* data, long n, float* out) {
  switch (type) {
    case OR_F32: std::memcpy(out, data, n * 4); return 0;
    case OR_Q8_0: dequant_q8_0(data, n, out); return 0;
    case OR_Q4_K: dequant_q4_k(data, n, out); return 0;
    case OR_Q5_K: dequant_q5_k(data, n, out); return 0;
    case OR_Q6_K: dequant_q6_k(data, n, out); return 0;
    default: return -1;
  }
}

/* --------------------------------------------------- operand emulation ---- */

inline float round_fp16(float x) { return (float)(_Float16)x; }
inline float round_bits(float x, int drop) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) return x;
  uint32_t half = 1u << (drop - 1);
  uint32_t lsb = (u >> drop) & 1u;
  u = (u + half - 1 + lsb) & ~((1u << drop) - 1);
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}
inline float round_emul(float x, int emul) {
  switch (emul) {
    case OR_EMUL_FP16: return round_fp16(x);
    case OR_EMUL_BF16: return round_bits(x, 16);
    case OR_EMUL_TF32: return round_bits(x, 13);
    default: return x;
  }
}

/* ------------------------------------------------------------ ops_simd ---- */

/* ops_simd.go:7-24: single pass sum/sumSq in f32, var = E[x^2]-mean^2. */
void layernorm(float* x, const float* w, const float* b, float eps, int n) {
  float nf = (float)n;
  float sum = 0.f, sumsq = 0.f;
  for (int i = 0; i < n; i++) {
    sum += x[i];
    sumsq += x[i] * x[i];
  }
  float mean = sum / nf;
  float var = sumsq / nf - mean * mean;
  float inv = (float)(1.0 / std::sqrt((double)(var + eps)));
  for (int i = 0; i < n; i++) x[i] = (x[i] - mean) * inv * w[i] + b[i];
}

/* ops_simd.go:27-43: rational tanh GeLU, clamped at |t| > 4.97. */
void gelu(float* x, int n) {
  for (int i = 0; i < n; i++) {
    float v = x[i];
    float t = 0.7978845608f * v * (1.0f + 0.044715f * v * v);
    float t2 = t * t;
    float th = t * (27.0f + t2) / (27.0f + 9.0f * t2);
    if (t > 4.97f) th = 1.0f;
    else if (t < -4.97f) th = -1.0f;
    x[i] = 0.5f * v * (1.0f + th);
  }
}

/* ops_simd.go:70-82 (fastExp): 0 below -10, otherwise float32(exp(float64)). */
inline float fast_exp(float x) {
  if (x < -10.f) return 0.f;
  return (float)std::exp((double)x);
}

/* ops_simd.go:46-66. */
void softmax(float* x, int n) {
  float mx = x[0];
  for (int i = 1; i < n; i++)
    if (x[i] > mx) mx = x[i];
  float sum = 0.f;
  for (int i = 0; i < n; i++) {
    x[i] = fast_exp(x[i] - mx);
    sum += x[i];
  }
  float inv = 1.0f / sum;
  for (int i = 0; i < n; i++) x[i] *= inv;
}

/* ops_simd.go:85-97: 4-way unrolled, each group summed left to right. */
float dot_f32(const float* a, const float* b, int n) {
  float sum = 0.f;
  int i = 0;
  for (; i <= n - 4; i += 4) sum += a[i] * b[i] + a[i + 1] * b[i + 1] + a[i + 2] * b[i + 2] + a[i + 3] * b[i + 3];
  for (; i < n; i++) sum += a[i] * b[i];
  return sum;
}

/* ops_simd.go:107-124 (NewRoPETable). */
void rope_table(int max_seq, int head_dim, float base, float* cs, float* sn) {
  int nrot = head_dim / 2;
  for (int pos = 0; pos < max_seq; pos++)
    for (int i = 0; i < nrot; i++) {
      float freq = 1.0f / (float)std::pow((double)base, (double)(2 * i) / (double)head_dim);
      float theta = freq * (float)pos;
      cs[(long)pos * nrot + i] = (float)std::cos((double)theta);
      sn[(long)pos * nrot + i] = (float)std::sin((double)theta);
    }
}

/* ops_simd.go:127-137: rotate adjacent pairs (2i, 2i+1). */
inline void rope_apply(float* x, const float* c, const float* s, int nrot) {
  for (int i = 0; i < nrot; i++) {
    float x0 = x[2 * i], x1 = x[2 * i + 1];
    x[2 * i] = x0 * c[i] - x1 * s[i];
    x[2 * i + 1] = x0 * s[i] + x1 * c[i];
  }
}

/* ---------------------------------------------------------------- GEMM ---- */

constexpr int MR = 6, NR = 32, KC = 128;

/* gemm_avx512.go:47-64 (PrePackBPanel32): [N][K] -> [N/32][K][32]. */
void prepack32(const float* B, int K, int N, float* packed) {
  int panels = (N + NR - 1) / NR;
  std::memset(packed, 0, sizeof(float) * (size_t)panels * K * NR);
  for (int p = 0; p < panels; p++)
    for (int k = 0; k < K; k++)
      for (int n = 0; n < NR; n++) {
        int col = p * NR + n;
        if (col < N) packed[((size_t)p * K + k) * NR + n] = B[(size_t)col * K + k];
      }
}

/* gemm_avx512_amd64.s:22-195: C[6x32] += sum_k A[6][k]*B[k][32], one FMA
 * chain per accumulator from zero, added into C at the end. */
__attribute__((target("avx512f"))) void micro_avx512(const float* A, int lda, const float* Bp, float* C,
                                                     int ldc, int kc) {
  __m512 acc[MR][2];
  for (int m = 0; m < MR; m++) acc[m][0] = acc[m][1] = _mm512_setzero_ps();
  for (int k = 0; k < kc; k++) {
    __m512 b0 = _mm512_loadu_ps(Bp + k * NR), b1 = _mm512_loadu_ps(Bp + k * NR + 16);
    for (int m = 0; m < MR; m++) {
      __m512 a = _mm512_set1_ps(A[m * lda + k]);
      acc[m][0] = _mm512_fmadd_ps(a, b0, acc[m][0]);
      acc[m][1] = _mm512_fmadd_ps(a, b1, acc[m][1]);
    }
  }
  for (int m = 0; m < MR; m++) {
    float* c = C + (size_t)m * ldc;
    _mm512_storeu_ps(c, _mm512_add_ps(_mm512_loadu_ps(c), acc[m][0]));
    _mm512_storeu_ps(c + 16, _mm512_add_ps(_mm512_loadu_ps(c + 16), acc[m][1]));
  }
}

/* Same arithmetic on AVX2+FMA hosts (two 6x16 halves; gemm_amd64.s:197). */
__attribute__((target("avx2,fma"))) void micro_avx2(const float* A, int lda, const float* Bp, float* C, int ldc,
                                                    int kc) {
  for (int half = 0; half < 2; half++) {
    __m256 acc[MR][2];
    for (int m = 0; m < MR; m++) acc[m][0] = acc[m][1] = _mm256_setzero_ps();
    for (int k = 0; k < kc; k++) {
      __m256 b0 = _mm256_loadu_ps(Bp + k * NR + half * 16), b1 = _mm256_loadu_ps(Bp + k * NR + half * 16 + 8);
      for (int m = 0; m < MR; m++) {
        __m256 a = _mm256_set1_ps(A[m * lda + k]);
        acc[m][0] = _mm256_fmadd_ps(a, b0, acc[m][0]);
        acc[m][1] = _mm256_fmadd_ps(a, b1, acc[m][1]);
      }
    }
    for (int m = 0; m < MR; m++) {
      float* c = C + (size_t)m * ldc + half * 16;
      _mm256_storeu_ps(c, _mm256_add_ps(_mm256_loadu_ps(c), acc[m][0]));
      _mm256_storeu_ps(c + 8, _mm256_add_ps(_mm256_loadu_ps(c + 8), acc[m][1]));
    }
  }
}

void micro_scalar(const float* A, int lda, const float* Bp, float* C, int ldc, int kc) {
  float acc[MR][NR] = {};
  for (int k = 0; k < kc; k++)
    for (int m = 0; m < MR; m++)
      for (int j = 0; j < NR; j++) acc[m][j] = std::fmaf(A[m * lda + k], Bp[k * NR + j], acc[m][j]);
  for (int m = 0; m < MR; m++)
    for (int j = 0; j < NR; j++) C[(size_t)m * ldc + j] += acc[m][j];
}

using micro_fn = void (*)(const float*, int, const float*, float*, int, int);
micro_fn pick_micro() {
  __builtin_cpu_init();
  if (__builtin_cpu_supports("avx512f")) return micro_avx512;
  if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) return micro_avx2;
  return micro_scalar;
}
const micro_fn g_micro = pick_micro();

/* gemm_avx512.go:67-147 (GemmPrePacked32).  C is zeroed first (the caller's
 * make() in bert.go:603).  N panels are split over workers; K runs in KC=128
 * chunks; full 6-row tiles use the micro-kernel, the M%6 edge rows a plain
 * (unfused) dot per chunk added into C. */
void gemm_prepacked32(const float* A, int M, const float* packed, float* C, int N, int K, int nthreads) {
  std::memset(C, 0, sizeof(float) * (size_t)M * N);
  int panels = (N + NR - 1) / NR;
#pragma omp parallel for schedule(static) num_threads(nthreads) if (nthreads > 1 && !omp_in_parallel())
  for (int p = 0; p < panels; p++) {
    int j = p * NR;
    int nr = (j + NR > N) ? N - j : NR;
    for (int kc = 0; kc < K; kc += KC) {
      int kl = (kc + KC > K) ? K - kc : KC;
      const float* bp = packed + ((size_t)p * K + kc) * NR;
      for (int i = 0; i < M; i += MR) {
        int mr = (i + MR > M) ? M - i : MR;
        if (mr == MR && nr == NR) {
          g_micro(A + (size_t)i * K + kc, K, bp, C + (size_t)i * N + j, N, kl);
        } else {
          for (int ii = i; ii < i + mr; ii++)
            for (int jj = 0; jj < nr; jj++) {
              float sum = 0.f;
              for (int k = kc; k < kc + kl; k++) sum += A[(size_t)ii * K + k] * packed[((size_t)p * K + k) * NR + jj];
              C[(size_t)ii * N + j + jj] += sum;
            }
        }
      }
    }
  }
}

/* ------------------------------------------------ fused dequant.dot (a18) - */

/* ops_fast.go:52-90 (DotQ8_0x4): per block sum(float32(q)*x) then *scale. */
float dot_q8_0_row(const uint8_t* row, const float* x, int K) {
  float total = 0.f;
  for (int b = 0; b < K / 32; b++) {
    const uint8_t* blk = row + b * 34;
    float s = f16_to_f32(rd16(blk));
    float sum = 0.f;
    for (int i = 0; i < 32; i++) sum += (float)(int8_t)blk[2 + i] * x[b * 32 + i];
    total += sum * s;
  }
  return total;
}

/* quant_q4k.go:87-128, quant_q5k.go:245-299, quant_q6k.go:387-429 (the
 * scalar DotQ*_K; the AVX2 *Fast variants of ops_fast.go:269-454 agree with
 * them to relErr 1e-5 per dot_q5k_test.go / dot_q6k_test.go). */
float dot_kquant_row(int type, const uint8_t* row, const float* x, int K) {
  float w[256];
  float total = 0.f;
  long bs = row_bytes(type, 256);
  for (int b = 0; b < K / 256; b++) {
    dequant(type, row + b * bs, 256, w);
    if (type == OR_Q6_K) {
      /* quant_q6k.go:420-423: total += d*sc*q*x, element by element in the
       * (n, l, +0/+32/+64/+96) order. */
      for (int nn = 0; nn < 256; nn += 128)
        for (int l = 0; l < 32; l++)
          for (int g = 0; g < 4; g++) total += w[nn + l + 32 * g] * x[b * 256 + nn + l + 32 * g];
    } else {
      for (int i = 0; i < 256; i++) total += w[i] * x[b * 256 + i];
    }
  }
  return total;
}

/* ------------------------------------------------------------- GGUF ---- */

struct TensorInfo {
  std::string name;
  std::vector<uint64_t> dims;
  uint32_t type = 0;
  uint64_t offset = 0;
  uint64_t nelem() const {
    uint64_t n = 1;
    for (auto d : dims) n *= d;
    return n;
  }
};

struct GGUF {
  std::vector<uint8_t> bytes;
  std::map<std::string, uint32_t> u32;
  std::map<std::string, float> f32;
  std::vector<TensorInfo> tensors;
  uint64_t data_offset = 0;
  const TensorInfo* get(const std::string& n) const {
    for (auto& t : tensors)
      if (t.name == n) return &t;
    return nullptr;
  }
  const uint8_t* data(const TensorInfo& t) const { return bytes.data() + data_offset + t.offset; }
};

struct Cursor {
  const uint8_t* p;
  size_t n, pos = 0;
  template <class T>
  T get() {
    if (pos + sizeof(T) > n) throw std::runtime_error("gguf: unexpected EOF");
    T v;
    std::memcpy(&v, p + pos, sizeof(T));
    pos += sizeof(T);
    return v;
  }
  std::string str() {
    uint64_t len = get<uint64_t>();
    if (pos + len > n) throw std::runtime_error("gguf: unexpected EOF in string");
    std::string s((const char*)p + pos, len);
    pos += len;
    return s;
  }
};

/* reader.go:390-433 (readValue); only uint32/float32 scalars are kept, as
 * GetUint32/GetFloat32 (reader.go:293-332) accept exactly those types. */
void skip_or_keep(Cursor& c, uint32_t vt, GGUF& g, const std::string* key) {
  switch (vt) {
    case 0: case 1: case 7: c.get<uint8_t>(); break;
    case 2: case 3: c.get<uint16_t>(); break;
    case 4: { uint32_t v = c.get<uint32_t>(); if (key) g.u32[*key] = v; break; }
    case 5: c.get<int32_t>(); break;
    case 6: { float v = c.get<float>(); if (key) g.f32[*key] = v; break; }
    case 8: c.str(); break;
    case 9: {
      uint32_t et = c.get<uint32_t>();
      uint64_t len = c.get<uint64_t>();
      for (uint64_t i = 0; i < len; i++) skip_or_keep(c, et, g, nullptr);
      break;
    }
    case 10: case 11: case 12: c.get<uint64_t>(); break;
    default: throw std::runtime_error("gguf: unknown value type " + std::to_string(vt));
  }
}

/* reader.go:219-280 (Open): magic, version 2..3, KVs, tensor infos, data at
 * the next 32-byte boundary. */
void gguf_open(const char* path, GGUF& g) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error(std::string("gguf: open ") + path);
  f.seekg(0, std::ios::end);
  size_t sz = (size_t)f.tellg();
  f.seekg(0);
  g.bytes.resize(sz);
  f.read((char*)g.bytes.data(), sz);
  Cursor c{g.bytes.data(), sz};
  if (c.get<uint32_t>() != 0x46554747u) throw std::runtime_error("gguf: invalid magic");
  uint32_t ver = c.get<uint32_t>();
  if (ver < 2 || ver > 3) throw std::runtime_error("gguf: unsupported version");
  uint64_t nt = c.get<uint64_t>(), nkv = c.get<uint64_t>();
  for (uint64_t i = 0; i < nkv; i++) {
    std::string key = c.str();
    uint32_t vt = c.get<uint32_t>();
    skip_or_keep(c, vt, g, &key);
  }
  for (uint64_t i = 0; i < nt; i++) {
    TensorInfo t;
    t.name = c.str();
    uint32_t nd = c.get<uint32_t>();
    for (uint32_t d = 0; d < nd; d++) t.dims.push_back(c.get<uint64_t>());
    t.type = c.get<uint32_t>();
    t.offset = c.get<uint64_t>();
    g.tensors.push_back(t);
  }
  g.data_offset = (c.pos + 31) & ~(uint64_t)31;
}

}  // namespace

/* ------------------------------------------------------------- model ---- */

struct Layer {
  std::vector<float> pp[5];  // prepacked [N/32][K][32]: qkv, out, up, gate, down
  int N[5], K[5];
  std::vector<float> attn_w, attn_b, out_w, out_b;
};

struct or_model {
  int layers, hidden, heads, head_dim, ffn, max_seq;
  float eps, rope_base;
  int emul;
  GGUF g;
  const TensorInfo* tok_embd;
  const TensorInfo* tok_types;
  std::vector<float> embd_w, embd_b;
  std::vector<Layer> L;
  std::vector<float> rope_cos, rope_sin;
};

namespace {

std::vector<float> load_vec(const GGUF& g, const std::string& name) {
  const TensorInfo* t = g.get(name);
  if (!t) throw std::runtime_error("tensor \"" + name + "\" not found");
  std::vector<float> v(t->nelem());
  if (dequant(t->type, g.data(*t), (long)t->nelem(), v.data()) != 0) throw std::runtime_error("bad type " + name);
  return v;
}

/* bert.go:290-316 (getEmbedding): row idx of a [dim, rows] tensor. */
void get_embedding(const GGUF& g, const TensorInfo& t, int idx, int dim, float* out) {
  long rb = row_bytes(t.type, dim);
  if (rb < 0) throw std::runtime_error("unsupported embedding type");
  dequant(t.type, g.data(t) + (long)idx * rb, dim, out);
}

void gemm_emul(const or_model* m, const float* A, int M, int which, const Layer& l, float* C, int nthreads) {
  int K = l.K[which], N = l.N[which];
  if (m->emul == OR_EMUL_FP32) {
    gemm_prepacked32(A, M, l.pp[which].data(), C, N, K, nthreads);
    return;
  }
  std::vector<float> Ar((size_t)M * K);
  for (size_t i = 0; i < Ar.size(); i++) Ar[i] = round_emul(A[i], m->emul);
  gemm_prepacked32(Ar.data(), M, l.pp[which].data(), C, N, K, nthreads);
}

/* bert.go:319-411 (multiHeadAttention) for one sequence. */
void attention(const or_model* m, const Layer& l, std::vector<float>& h, const int32_t* mask, int L,
               std::vector<float>& out, int nthreads) {
  int H = m->hidden, hd = m->head_dim, nh = m->heads, nrot = hd / 2;
  std::vector<float> qkv((size_t)L * 3 * H);
  gemm_emul(m, h.data(), L, 0, l, qkv.data(), nthreads);
  std::vector<float> Q((size_t)L * H), K((size_t)L * H), V((size_t)L * H);
  for (int i = 0; i < L; i++) {
    std::memcpy(&Q[(size_t)i * H], &qkv[(size_t)i * 3 * H], H * 4);
    std::memcpy(&K[(size_t)i * H], &qkv[(size_t)i * 3 * H + H], H * 4);
    std::memcpy(&V[(size_t)i * H], &qkv[(size_t)i * 3 * H + 2 * H], H * 4);
    for (int hh = 0; hh < nh; hh++) {
      rope_apply(&Q[(size_t)i * H + hh * hd], &m->rope_cos[(size_t)i * nrot], &m->rope_sin[(size_t)i * nrot], nrot);
      rope_apply(&K[(size_t)i * H + hh * hd], &m->rope_cos[(size_t)i * nrot], &m->rope_sin[(size_t)i * nrot], nrot);
    }
  }
  if (m->emul != OR_EMUL_FP32) {
    for (auto* v : {&Q, &K, &V})
      for (auto& x : *v) x = round_emul(x, m->emul);
  }
  std::vector<float> att((size_t)L * H);
  float scale = (float)(1.0 / std::sqrt((double)hd));
#pragma omp parallel for num_threads(nthreads) if (nthreads > 1 && !omp_in_parallel())
  for (int hh = 0; hh < nh; hh++) {
    int off = hh * hd;
    std::vector<float> sc(L);
    for (int qi = 0; qi < L; qi++) {
      for (int ki = 0; ki < L; ki++) sc[ki] = dot_f32(&Q[(size_t)qi * H + off], &K[(size_t)ki * H + off], hd) * scale;
      for (int ki = 0; ki < L; ki++)
        if (mask[ki] == 0) sc[ki] = -1e9f;
      softmax(sc.data(), L);
      for (int d = 0; d < hd; d++) {
        float sum = 0.f;
        for (int vi = 0; vi < L; vi++) sum += sc[vi] * V[(size_t)vi * H + off + d];
        att[(size_t)qi * H + off + d] = sum;
      }
    }
  }
  out.assign((size_t)L * H, 0.f);
  gemm_emul(m, att.data(), L, 1, l, out.data(), nthreads);
}

/* bert.go:216-285 (Forward). */
void forward(const or_model* m, const int32_t* ids, const int32_t* mask, int L, float* hid, int nthreads) {
  int H = m->hidden, F = m->ffn;
  std::vector<float> type_e(H), tok(H);
  get_embedding(m->g, *m->tok_types, 0, H, type_e.data());
  std::vector<float> h((size_t)L * H);
  for (int i = 0; i < L; i++) {
    get_embedding(m->g, *m->tok_embd, ids[i], H, tok.data());
    float* r = &h[(size_t)i * H];
    for (int j = 0; j < H; j++) r[j] = tok[j] + type_e[j];
    layernorm(r, m->embd_w.data(), m->embd_b.data(), m->eps, H);
  }
  std::vector<float> att, up((size_t)L * F), gate((size_t)L * F), down((size_t)L * H);
  for (int li = 0; li < m->layers; li++) {
    const Layer& l = m->L[li];
    attention(m, l, h, mask, L, att, nthreads);
    for (int i = 0; i < L; i++) {
      for (int j = 0; j < H; j++) h[(size_t)i * H + j] += att[(size_t)i * H + j];
      layernorm(&h[(size_t)i * H], l.attn_w.data(), l.attn_b.data(), m->eps, H);
    }
    /* bert.go:415-445 (ffnForward): down(gelu(gate(x)) * up(x)). */
    gemm_emul(m, h.data(), L, 2, l, up.data(), nthreads);
    gemm_emul(m, h.data(), L, 3, l, gate.data(), nthreads);
    for (int i = 0; i < L; i++) {
      gelu(&gate[(size_t)i * F], F);
      for (int j = 0; j < F; j++) gate[(size_t)i * F + j] *= up[(size_t)i * F + j];
    }
    gemm_emul(m, gate.data(), L, 4, l, down.data(), nthreads);
    for (int i = 0; i < L; i++) {
      for (int j = 0; j < H; j++) h[(size_t)i * H + j] += down[(size_t)i * H + j];
      layernorm(&h[(size_t)i * H], l.out_w.data(), l.out_b.data(), m->eps, H);
    }
  }
  std::memcpy(hid, h.data(), sizeof(float) * (size_t)L * H);
}

/* pool.go:8-31 (MeanPool). */
void mean_pool(const float* hid, const int32_t* mask, int L, int H, float* out) {
  for (int j = 0; j < H; j++) out[j] = 0.f;
  float count = 0.f;
  for (int i = 0; i < L; i++)
    if (mask[i] == 1) {
      for (int j = 0; j < H; j++) out[j] += hid[(size_t)i * H + j];
      count++;
    }
  if (count == 0.f) return;
  float inv = 1.0f / count;
  for (int j = 0; j < H; j++) out[j] *= inv;
}

/* pool.go:37-53 (L2Normalize): float64 sum of squares, f32 multiply. */
void l2_normalize(float* v, int n) {
  double norm = 0.0;
  for (int i = 0; i < n; i++) norm += (double)v[i] * (double)v[i];
  norm = std::sqrt(norm);
  if (norm == 0.0) return;
  float inv = (float)(1.0 / norm);
  for (int i = 0; i < n; i++) v[i] = v[i] * inv;
}

thread_local std::string g_err;

}  // namespace

/* ------------------------------------------------------------ C API ---- */

extern "C" {

float or_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
long or_row_bytes(int type, long n) { return row_bytes(type, n); }
int or_dequant(int type, const uint8_t* data, long n, float* out) { return dequant(type, data, n, out); }

/* gemm.go:221-267 (DequantWeightMatrix): N rows of K, each row dequantised. */
int or_dequant_matrix(int type, const uint8_t* data, int K, int N, float* out) {
  long rb = row_bytes(type, K);
  if (rb < 0) return -1;
  for (int n = 0; n < N; n++) dequant(type, data + (long)n * rb, K, out + (size_t)n * K);
  return 0;
}

void or_layernorm(float* x, const float* w, const float* b, float eps, int n) { layernorm(x, w, b, eps, n); }
void or_gelu(float* x, int n) { gelu(x, n); }
void or_softmax(float* x, int n) { softmax(x, n); }
float or_dot_f32(const float* a, const float* b, int n) { return dot_f32(a, b, n); }
void or_rope_table(int max_seq, int head_dim, float base, float* c, float* s) { rope_table(max_seq, head_dim, base, c, s); }
void or_prepack32(const float* B, int K, int N, float* packed) { prepack32(B, K, N, packed); }
void or_gemm_prepacked32(const float* A, int M, const float* packed, float* C, int N, int K, int nthreads) {
  gemm_prepacked32(A, M, packed, C, N, K, nthreads);
}

/* ops.go:418-517 (MatMulBatch): Q8_0 via DotQ8_0x4 rows, K-quants via the
 * fused per-row dot, F32 via a plain dot. */
int or_matmul_batch(int type, const uint8_t* w, int K, int N, const float* X, int M, float* Y, int nthreads) {
  long rb = row_bytes(type, K);
  if (rb < 0) return -1;
#pragma omp parallel for schedule(static) num_threads(nthreads) if (nthreads > 1)
  for (int n = 0; n < N; n++) {
    const uint8_t* row = w + (long)n * rb;
    for (int s = 0; s < M; s++) {
      const float* x = X + (size_t)s * K;
      float v;
      if (type == OR_Q8_0) v = dot_q8_0_row(row, x, K);
      else if (type == OR_F32) {
        float sum = 0.f;
        const float* r = (const float*)row;
        for (int k = 0; k < K; k++) sum += r[k] * x[k];
        v = sum;
      } else v = dot_kquant_row(type, row, x, K);
      Y[(size_t)s * N + n] = v;
    }
  }
  return 0;
}

/* bert.go:91-211 (LoadBertModel) + bert.go:542-576 (PreDequant) +
 * embedder.go:29 (NewRoPETable). */
or_model* or_model_load(const char* path, int emul, char* err, int errlen) {
  try {
    auto m = std::make_unique<or_model>();
    gguf_open(path, m->g);
    auto u = [&](const char* k) { auto it = m->g.u32.find(k); return it == m->g.u32.end() ? 0u : it->second; };
    auto f = [&](const char* k) { auto it = m->g.f32.find(k); return it == m->g.f32.end() ? 0.f : it->second; };
    m->layers = (int)u("nomic-bert.block_count");
    m->hidden = (int)u("nomic-bert.embedding_length");
    m->ffn = (int)u("nomic-bert.feed_forward_length");
    m->heads = (int)u("nomic-bert.attention.head_count");
    m->max_seq = (int)u("nomic-bert.context_length");
    m->eps = f("nomic-bert.attention.layer_norm_epsilon");
    m->rope_base = f("nomic-bert.rope.freq_base");
    if (m->layers == 0 || m->hidden == 0) throw std::runtime_error("embed: missing model params in GGUF metadata");
    m->head_dim = m->hidden / m->heads;
    m->emul = emul;
    m->tok_embd = m->g.get("token_embd.weight");
    m->tok_types = m->g.get("token_types.weight");
    if (!m->tok_embd || !m->tok_types) throw std::runtime_error("embedding tensors not found");
    m->embd_w = load_vec(m->g, "token_embd_norm.weight");
    m->embd_b = load_vec(m->g, "token_embd_norm.bias");
    static const char* names[5] = {"attn_qkv", "attn_output", "ffn_up", "ffn_gate", "ffn_down"};
    m->L.resize(m->layers);
    for (int i = 0; i < m->layers; i++) {
      std::string p = "blk." + std::to_string(i) + ".";
      Layer& l = m->L[i];
      for (int w = 0; w < 5; w++) {
        const TensorInfo* t = m->g.get(p + names[w] + ".weight");
        if (!t) throw std::runtime_error("tensor \"" + p + names[w] + ".weight\" not found");
        int K = (w == 4) ? m->ffn : m->hidden;
        int N = 1;
        for (size_t d = 1; d < t->dims.size(); d++) N *= (int)t->dims[d];
        std::vector<float> dq((size_t)N * K);
        if (or_dequant_matrix((int)t->type, m->g.data(*t), K, N, dq.data()) != 0) throw std::runtime_error("bad weight type");
        if (emul != OR_EMUL_FP32)
          for (auto& x : dq) x = round_emul(x, emul);
        l.N[w] = N;
        l.K[w] = K;
        l.pp[w].resize((size_t)((N + NR - 1) / NR) * K * NR);
        prepack32(dq.data(), K, N, l.pp[w].data());
      }
      l.attn_w = load_vec(m->g, p + "attn_output_norm.weight");
      l.attn_b = load_vec(m->g, p + "attn_output_norm.bias");
      l.out_w = load_vec(m->g, p + "layer_output_norm.weight");
      l.out_b = load_vec(m->g, p + "layer_output_norm.bias");
    }
    int nrot = m->head_dim / 2;
    m->rope_cos.resize((size_t)m->max_seq * nrot);
    m->rope_sin.resize((size_t)m->max_seq * nrot);
    rope_table(m->max_seq, m->head_dim, m->rope_base, m->rope_cos.data(), m->rope_sin.data());
    return m.release();
  } catch (std::exception& e) {
    if (err && errlen > 0) std::snprintf(err, errlen, "%s", e.what());
    return nullptr;
  }
}

void or_model_free(or_model* m) { delete m; }

int or_model_hparams(const or_model* m, int* o, float* eps, float* rope_base) {
  o[0] = m->layers; o[1] = m->hidden; o[2] = m->heads; o[3] = m->head_dim;
  o[4] = m->ffn; o[5] = m->max_seq; o[6] = (int)m->tok_embd->dims.back();
  *eps = m->eps;
  *rope_base = m->rope_base;
  return 0;
}

int or_forward(const or_model* m, const int32_t* ids, const int32_t* mask, int L, float* hiddens, int nthreads) {
  if (L > m->max_seq) return -1;
  forward(m, ids, mask, L, hiddens, nthreads);
  return 0;
}

/* embedder.go:46-70 (Embed) over each packed sequence; sequences run in
 * parallel like EmbedBatch's workers (embedder.go:75-133). */
int or_embed_ids(const or_model* m, const int32_t* ids, const int32_t* offsets, int nseq, int out_dim, float* out,
                 int nthreads) {
  int H = m->hidden;
  if (out_dim < 1 || out_dim > H) return -1;
  for (int s = 0; s < nseq; s++)
    if (offsets[s + 1] - offsets[s] > m->max_seq || offsets[s + 1] < offsets[s]) return -1;
  int inner = nseq == 1 ? nthreads : 1;
#pragma omp parallel for schedule(dynamic) num_threads(nthreads) if (nseq > 1 && nthreads > 1)
  for (int s = 0; s < nseq; s++) {
    int L = offsets[s + 1] - offsets[s];
    std::vector<float> pooled(H, 0.f);
    if (L > 0) {
      std::vector<int32_t> mask(L, 1);
      std::vector<float> hid((size_t)L * H);
      forward(m, ids + offsets[s], mask.data(), L, hid.data(), inner);
      mean_pool(hid.data(), mask.data(), L, H, pooled.data());
    }
    l2_normalize(pooled.data(), H);
    if (out_dim < H) l2_normalize(pooled.data(), out_dim);
    std::memcpy(out + (size_t)s * out_dim, pooled.data(), sizeof(float) * out_dim);
  }
  return 0;
}

int or_model_weight(const or_model* m, int layer, int which, float* out) {
  if (layer < 0 || layer >= m->layers || which < 0 || which > 4) return -1;
  const Layer& l = m->L[layer];
  int K = l.K[which], N = l.N[which];
  for (int n = 0; n < N; n++)
    for (int k = 0; k < K; k++) out[(size_t)n * K + k] = l.pp[which][((size_t)(n / NR) * K + k) * NR + n % NR];
  return 0;
}

}  // extern "C"
