// Memory-bound kernels of the forward pass: embedding gather + LayerNorm,
// residual LayerNorm, masked mean-pool + L2 normalise, f32 -> f16.
//
// The residual LayerNorm reads h and the projection output y and writes
// LN(h + y) back to h (float32) and to the fp16 GEMM operand copy.
// Row kernels use one warp per 768-wide row: 24 floats per lane in float4s,
// warp-shuffle reductions, no shared memory.
#include "common.cuh"
#include "gguf_decode.cuh"
#include "kernels.h"
#include "ln_warp.cuh"
#include "pool_seq.cuh"

namespace le {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ops_simd.go:7-24: mean = sum/n, var = sumSq/n - mean^2 (single pass, f32),
// invStd = float32(1 / sqrt(float64(var + eps))), y = (x-mean)*invStd*w + b.
// H is a multiple of 128 and at most 128 * LN_MAXV.
constexpr int LN_MAXV = 8;  // float4 per lane -> H <= 1024
// Staged bytes of one embedding row per warp: an F32 row of 1,024 values
// plus the 16 bytes before its boundary, in 16-byte loads (32 lanes x 9).
constexpr int EMB_STAGE = 32 * 16 * 9;
static_assert(EMB_STAGE >= 4 * 128 * LN_MAXV + 16, "the widest row fits");

template <bool GATHER>
__global__ void __launch_bounds__(256) ln_rows_kernel(const float* in, const float* __restrict__ add,
                                                      const int32_t* __restrict__ ids,
                                                      int emb_type, const uint8_t* __restrict__ emb, long emb_row_bytes,
                                                      const float* __restrict__ type0, const float* __restrict__ w,
                                                      const float* __restrict__ b, float eps, int T, int H,
                                                      int vocab, DevStatus* status, float* out32,
                                                      __half* __restrict__ out16) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const int nv = H / 128;
  float4 x[LN_MAXV];
  if constexpr (GATHER) {
    // bert.go:227-247: token_embd row + token_types row 0, then LayerNorm.
    // The row's bytes come first into the warp's shared-memory slot with
    // 16-byte loads from the 16-byte boundary at or below the row (the
    // embedding buffer carries 16 spare bytes), all in flight at once; the
    // values are then decoded from there.
    __shared__ __align__(16) uint8_t stage[8][EMB_STAGE];
    int id = ids[warp];
    if (id < 0 || id >= vocab) {  // device-resident ids are not checked on the host
      if (lane == 0) report(status, DE_BOUNDS, 1, id);
      id = 0;
    }
    const uintptr_t ra = reinterpret_cast<uintptr_t>(emb + (long)id * emb_row_bytes);
    const uint4* src = reinterpret_cast<const uint4*>(ra & ~(uintptr_t)15);
    const int n16 = (int)(((ra & 15) + emb_row_bytes + 15) >> 4);
    uint8_t* st = stage[(threadIdx.x >> 5) & 7];
    uint4 q[EMB_STAGE / 16 / 32];
#pragma unroll
    for (int k = 0; k < EMB_STAGE / 16 / 32; k++)
      if (lane + 32 * k < n16) q[k] = __ldg(src + lane + 32 * k);
#pragma unroll
    for (int k = 0; k < EMB_STAGE / 16 / 32; k++)
      if (lane + 32 * k < n16) *reinterpret_cast<uint4*>(st + 16 * (lane + 32 * k)) = q[k];
    __syncwarp();
    const uint8_t* row = st + (ra & 15);
#pragma unroll
    for (int i = 0; i < LN_MAXV; i++) {
      if (i < nv) {
        const int c = (i * 32 + lane) * 4;
        const float4 t = *reinterpret_cast<const float4*>(type0 + c);
        const float4 g = gguf_elem4(emb_type, row, c);
        x[i] = make_float4(__fadd_rn(g.x, t.x), __fadd_rn(g.y, t.y), __fadd_rn(g.z, t.z), __fadd_rn(g.w, t.w));
      }
    }
  } else {
    // bert.go:262-266 / 276-280: h += y, then LayerNorm.
    const float* r = in + (long)warp * H;
    const float* y = add + (long)warp * H;
#pragma unroll
    for (int i = 0; i < LN_MAXV; i++)
      if (i < nv) {
        const float4 a = *reinterpret_cast<const float4*>(r + (i * 32 + lane) * 4);
        const float4 b = *reinterpret_cast<const float4*>(y + (i * 32 + lane) * 4);
        x[i] = make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
      }
  }
  float mean, inv;
  ln_row_stats(x, nv, H, eps, &mean, &inv);
  float* o32 = out32 + (long)warp * H;
  __half* o16 = out16 + (long)warp * H;
#pragma unroll
  for (int i = 0; i < LN_MAXV; i++)
    if (i < nv) {
      const int c = (i * 32 + lane) * 4;
      const float4 y = ln_apply(x[i], mean, inv, *reinterpret_cast<const float4*>(w + c),
                                *reinterpret_cast<const float4*>(b + c));
      *reinterpret_cast<float4*>(o32 + c) = y;
      uint2 h;
      h.x = pack_half2(y.x, y.y);
      h.y = pack_half2(y.z, y.w);
      *reinterpret_cast<uint2*>(o16 + c) = h;
    }
}

// pool.go:8-53 + embedder.go:59-68 (pool_seq.cuh): one CTA of H/4 threads
// per sequence, 32 rows' loads in flight per thread (a 128-token sequence
// is four DRAM round trips).
__global__ void pool_kernel(const float* __restrict__ h, const int32_t* __restrict__ offsets, int H, int out_dim,
                            float* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int s = blockIdx.x;
  __shared__ double red[32];
  pool_seq<32>(h, offsets[s], offsets[s + 1], H, out_dim, out + (long)s * out_dim, red, [] { __syncthreads(); });
}

__global__ void f32_to_f16_kernel(const float* __restrict__ in, long n, __half* __restrict__ out) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = __float2half_rn(in[i]);
}

// The same, 8 values per thread (two 16-byte loads, one 16-byte store) over
// n8 groups of 8; both pointers 16-byte aligned.
__global__ void f32_to_f16_x8_kernel(const float4* __restrict__ in, long n8, uint4* __restrict__ out) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const float4 a = __ldcs(in + 2 * i), b = __ldcs(in + 2 * i + 1);
  __stcs(out + i, make_uint4(pack_half2(a.x, a.y), pack_half2(a.z, a.w), pack_half2(b.x, b.y), pack_half2(b.z, b.w)));
}

// Per-token position inside its sequence (RoPE row index, bert.go:351).
__global__ void positions_kernel(const int32_t* __restrict__ offsets, int nseq, int32_t* __restrict__ pos) {
  const int s = blockIdx.x;
  if (s >= nseq) return;
  const int t0 = offsets[s], t1 = offsets[s + 1];
  for (int t = t0 + threadIdx.x; t < t1; t += blockDim.x) pos[t] = t - t0;
}

cudaError_t launch_embed_ln(const int32_t* ids, int emb_type, const uint8_t* emb, long emb_row_bytes, int vocab,
                            const float* type0, const float* w, const float* b, float eps, int T, int H, float* out32,
                            __half* out16, DevStatus* status, cudaStream_t s) {
  if (H % 128 || H > 128 * LN_MAXV || emb_row_bytes + 16 > EMB_STAGE) return cudaErrorInvalidValue;
  if (T == 0) return cudaSuccess;
  cudaLaunchAttribute attr[1];
  const cudaLaunchConfig_t cfg = pdl_config(dim3((T + 7) / 8), dim3(256), 0, s, attr);
  return cudaLaunchKernelEx(&cfg, ln_rows_kernel<true>, (const float*)nullptr, (const float*)nullptr, ids, emb_type, emb,
                            emb_row_bytes, type0, w, b, eps, T, H, vocab, status, out32, out16);
}

cudaError_t launch_ln_add(const float* in, const float* add, const float* w, const float* b, float eps, int T, int H,
                          float* out32, __half* out16, cudaStream_t s) {
  if (H % 128 || H > 128 * LN_MAXV) return cudaErrorInvalidValue;
  if (T == 0) return cudaSuccess;
  cudaLaunchAttribute attr[1];
  const cudaLaunchConfig_t cfg = pdl_config(dim3((T + 7) / 8), dim3(256), 0, s, attr);
  return cudaLaunchKernelEx(&cfg, ln_rows_kernel<false>, in, add, (const int32_t*)nullptr, 0, (const uint8_t*)nullptr, 0L,
                            (const float*)nullptr, w, b, eps, T, H, 0, (DevStatus*)nullptr, out32, out16);
}

cudaError_t launch_pool(const float* h, const int32_t* offsets, int nseq, int H, int out_dim, float* out,
                        cudaStream_t s) {
  if (nseq == 0) return cudaSuccess;
  cudaLaunchAttribute attr[1];
  const cudaLaunchConfig_t cfg = pdl_config(dim3(nseq), dim3(H / 4), 0, s, attr);
  return cudaLaunchKernelEx(&cfg, pool_kernel, h, offsets, H, out_dim, out);
}

cudaError_t launch_f32_to_f16(const float* in, long n, __half* out, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  long done = 0;
  if (((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) == 0) {
    const long n8 = n / 8;
    if (n8 > 0)
      f32_to_f16_x8_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, s>>>(reinterpret_cast<const float4*>(in), n8,
                                                                          reinterpret_cast<uint4*>(out));
    done = n8 * 8;
  }
  if (done < n)  // unaligned pointers, or the last n % 8 values
    f32_to_f16_kernel<<<(unsigned)((n - done + 255) / 256), 256, 0, s>>>(in + done, n - done, out + done);
  return cudaGetLastError();
}

cudaError_t launch_positions(const int32_t* offsets, int nseq, int32_t* pos, cudaStream_t s) {
  if (nseq == 0) return cudaSuccess;
  positions_kernel<<<nseq, 128, 0, s>>>(offsets, nseq, pos);
  return cudaGetLastError();
}

}  // namespace le
