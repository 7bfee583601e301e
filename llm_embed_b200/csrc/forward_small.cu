// The whole encoder forward for a few tokens in one persistent kernel.
//
// At batch 1 the forward pass is ~85 dependent steps whose work is tiny
// (8 tokens) next to the weights they stream (120 MB for Q8_0), so separate
// kernels leave the GPU idle between launches.  Here one CTA per SM runs all
// layers (cooperative launch, so every CTA is resident), with a grid barrier
// where a step needs another CTA's results:
//
//   per layer:  [LN + QKV GEMM + RoPE] | [attention] | [out GEMM] |
//               [LN + up/gate GEMM + GEGLU] | [down GEMM] |
//
// * The residual stream h (T x 768 float32) lives in every CTA's shared
//   memory: each CTA applies the residual LayerNorms (bert.go:262-280)
//   itself, in the same order, so all copies hold the same values and a
//   LayerNorm needs no barrier.
// * Each GEMM's output row pairs are split evenly over the CTAs.  A CTA's
//   slice of the next GEMM's tile-blocked quantised weight (quant bytes +
//   scales, up to ~41 KB) is prefetched into shared memory with cp.async
//   while the current step and its barrier run, and dequantised there to the
//   same fp16 operand values as every other GEMM path.
// * Attention runs one warp per (sequence, head) with the same tensor-core
//   tile code as the attention kernels (attention_tile.cuh), so a sequence
//   gets the same bits here as in a larger batch through the separate
//   kernels.
//
// Barriers are a global arrival counter (zeroed before the launch) polled
// with acquire loads; every wait is bounded by WAIT_LIMIT_NS and reports
// DE_TIMEOUT through the status word, after which all CTAs leave.
#include "attention_tile.cuh"
#include "dequant.cuh"
#include "epilogue.cuh"
#include "gguf_decode.cuh"
#include "kernels.h"
#include "ln_warp.cuh"

#include <mutex>

namespace le {
namespace fs {

constexpr int H = SMALL_HIDDEN;
constexpr int F = SMALL_FFN;
constexpr int HEADS = SMALL_HEADS;
constexpr int HD = H / HEADS;
constexpr int TS = SMALL_MAX_TOKENS;
constexpr int NTHREADS = 256;
constexpr int NWARPS = NTHREADS / 32;

// Weight slice of one GEMM step in shared memory: for each local pair j,
// k-step ks and row (a, b): 64 quant bytes, then (after all of them) MB
// bytes of scales per (j, ks, row).
__host__ __device__ constexpr int meta_row_bytes(int qf) { return qf == QF_Q8_0 ? 4 : 16; }
constexpr int WBUF_BYTES = 41472;  // 40.5 KB: the largest slice (K-quant up/gate, 21 pairs) is 40,320 B

// Shared memory: two weight slice buffers; the residual stream h; and one
// region U used by one step at a time: the LN output x [T][H] fp16 (QKV,
// up/gate), the attention staging, the attention output [T][H] (out
// projection) or the GEGLU output [T][F] (down projection), staged once per
// step so the GEMM reads its input from shared memory.
struct SmemLayout {
  static constexpr int OFF_W = 0;
  static constexpr int OFF_H = OFF_W + 2 * WBUF_BYTES;                 // float h[TS][H]
  static constexpr int ATT_WARP_BYTES = 3 * 16 * attn::LDS * 2;       // half Q, K, V [16][LDS] per warp
  static constexpr int U_BYTES = (TS * F * 2 > NWARPS * ATT_WARP_BYTES) ? TS * F * 2 : NWARPS * ATT_WARP_BYTES;
  static constexpr int OFF_U = OFF_H + TS * H * 4;
  static constexpr int OFF_TOK = OFF_U + U_BYTES;                      // int pos[TS] (and spare)
  static constexpr int OFF_MISC = OFF_TOK + 4 * TS * 4;                // int flag
  static constexpr int BYTES = OFF_MISC + 16;
};
static_assert(SmemLayout::BYTES <= 232448, "shared memory budget");

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid barrier number `k` (0, 1, ...): returns false in every thread of the
// CTA if the wait timed out or another CTA reported a failure.
__device__ bool grid_sync(unsigned* counter, unsigned k, DevStatus* st, int* flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    *flag = 1;
    // The release orders the CTA's writes (made visible to this thread by
    // the barrier above) before the arrival; the acquire loads below order
    // every later read after the other CTAs' arrivals.
    red_release_add(counter, 1u);
    const unsigned target = (k + 1) * gridDim.x;
    if (ld_acquire(counter) < target) {
      const uint64_t t0 = globaltimer_ns();
      for (uint32_t i = 1;; i++) {
        if (ld_acquire(counter) >= target) break;
        if ((i & 63) == 0) {
          if (ld_acquire(reinterpret_cast<const unsigned*>(&st->code)) != 0) {
            *flag = 0;
            break;
          }
          if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) {
            report(st, DE_TIMEOUT, 40 + (int)(k % 10), (int)blockIdx.x);
            *flag = 0;
            break;
          }
        }
      }
    }
  }
  __syncthreads();
  return *reinterpret_cast<volatile int*>(flag) != 0;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Output pairs [p0, p1) of a GEMM with `n_pairs` pairs for this CTA.
__device__ __forceinline__ void pair_range(int n_pairs, int* p0, int* p1) {
  *p0 = (int)((long)n_pairs * blockIdx.x / gridDim.x);
  *p1 = (int)((long)n_pairs * (blockIdx.x + 1) / gridDim.x);
}

// Issue (no wait) the cp.async copies of this CTA's slice of GEMM `g`.
__device__ void prefetch_slice(const SmallGemm& g, uint32_t buf) {
  const int ksteps = g.K / TILE_K;
  const int cb = chunk_bytes(g.qf), mb = meta_row_bytes(g.qf);
  int p0, p1;
  pair_range(g.n_pairs, &p0, &p1);
  const int units = (p1 - p0) * ksteps * 2;  // (pair, k-step, row)
  const uint32_t meta0 = buf + units * 64;
  for (int u = threadIdx.x; u < units * 5; u += NTHREADS) {
    const int unit = u / 5, part = u % 5;
    const int which = unit & 1, ks = (unit >> 1) % ksteps, j = (unit >> 1) / ksteps;
    int ra, rb;
    pair_rows(g.mode, p0 + j, &ra, &rb);
    const int row = which ? rb : ra;
    const uint8_t* chunk = g.w + ((long)(row / TILE_N) * ksteps + ks) * cb;
    const int r = row % TILE_N;
    if (part < 4) {
      cp_async16(buf + unit * 64 + part * 16, chunk + r * TILE_K + part * 16);
    } else if (mb == 16) {
      cp_async16(meta0 + unit * 16, chunk + TILE_Q_BYTES + r * 16);
    } else {
      cp_async4(meta0 + unit * 4, chunk + TILE_Q_BYTES + r * 4);
    }
  }
}

__device__ __forceinline__ void h8_to_f32(uint4 h, float* f) {
  const __half2* p = reinterpret_cast<const __half2*>(&h);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float2 v = __half22float2(p[i]);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}

// LayerNorm (ops_simd.go:7-24) of h[t] (+ y[t] when y) into h[t] and its fp16
// copy x[t]; one warp per token row, single-pass sum/sumSq in float32.
__device__ void ln_rows(float* h, __half* x, const float* y, const float* w, const float* b, float eps, int T) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t = warp; t < T; t += NWARPS) {
    float4 v[H / 128];
#pragma unroll
    for (int i = 0; i < H / 128; i++) {
      const int c = (i * 32 + lane) * 4;
      float4 a = *reinterpret_cast<const float4*>(h + t * H + c);
      if (y) {
        const float4 d = __ldcg(reinterpret_cast<const float4*>(y + (long)t * H + c));
        a = make_float4(__fadd_rn(a.x, d.x), __fadd_rn(a.y, d.y), __fadd_rn(a.z, d.z), __fadd_rn(a.w, d.w));
      }
      v[i] = a;
    }
    float mean, inv;
    ln_row_stats(v, H / 128, H, eps, &mean, &inv);
#pragma unroll
    for (int i = 0; i < H / 128; i++) {
      const int c = (i * 32 + lane) * 4;
      const float4 o = ln_apply(v[i], mean, inv, *reinterpret_cast<const float4*>(w + c),
                                *reinterpret_cast<const float4*>(b + c));
      *reinterpret_cast<float4*>(h + t * H + c) = o;
      uint2 hh;
      hh.x = pack_half2(o.x, o.y);
      hh.y = pack_half2(o.z, o.w);
      *reinterpret_cast<uint2*>(x + t * H + c) = hh;
    }
  }
}

// Embedding rows (bert.go:227-247): token_embd row + token_types row 0.
__device__ void embed_rows(const SmallParams& p, float* h, int T) {
  for (int i = threadIdx.x; i < T * H; i += NTHREADS) {
    const int t = i / H, c = i % H;
    int id = p.ids[t];
    if (id < 0 || id >= p.vocab) {
      if (c == 0) report(p.status, DE_BOUNDS, 2, id);
      id = 0;
    }
    h[i] = __fadd_rn(gguf_elem(p.emb_type, p.emb + (long)id * p.emb_row_bytes, c), p.type0[c]);
  }
}

// Copy rows [0, T) x K of an fp16 activation written by other CTAs into
// shared memory (cp.async through L2; the caller commits and waits).
__device__ void stage_rows(uint32_t dst, const __half* src, int T, int K) {
  const int n = T * K / 8;
  for (int i = threadIdx.x; i < n; i += NTHREADS) cp_async16(dst + i * 16, src + (long)i * 8);
}

// Butterfly reduce-scatter of NV (16 or 32) per-lane partial sums: lane l
// ends with the warp total of value l (NV = 32) or l / 2 (NV = 16).  Each
// total is formed by the same pairings, own partial first, as a xor-butterfly
// all-reduce of that value, so the bits equal warp_sum's.
template <int NV>
__device__ __forceinline__ float reduce_scatter(float (&v)[NV]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16, n = NV; n > 1; o >>= 1, n >>= 1) {
    const bool hi = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; i++) {
      const float keep = hi ? v[i + n / 2] : v[i];
      const float send = hi ? v[i] : v[i + n / 2];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  if constexpr (NV == 16) v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
  return v[0];
}

// One GEMM step over this CTA's pairs: y = x . W^T for T <= TT tokens, x
// fp16 [T][K] in shared memory, weights from the prefetched slice.  Lanes own
// 16-column chunks (the accumulation order of gemm_simt.cu); the sums reduce
// across the warp onto one lane per (row, token) and the epilogue runs for
// all tokens at once.
template <int QF, int TT>
__device__ void gemm_step(const SmallGemm& g, const uint8_t* wbuf, const __half* x, int T, const EpiParams& ep) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ksteps = g.K / TILE_K, nch = g.K / 16;
  constexpr int MB = meta_row_bytes(QF);
  int p0, p1;
  pair_range(g.n_pairs, &p0, &p1);
  const int units = (p1 - p0) * ksteps * 2;
  const uint8_t* meta0 = wbuf + units * 64;
  for (int j = warp; j < p1 - p0; j += NWARPS) {
    float acc[2 * TT];  // [row][token]
#pragma unroll
    for (int i = 0; i < 2 * TT; i++) acc[i] = 0.f;
    for (int c = lane; c < nch; c += 32) {
      const int ks = c >> 2, part = c & 3;
      const int ua = (j * ksteps + ks) * 2;
      const uint4 qa = *reinterpret_cast<const uint4*>(wbuf + ua * 64 + part * 16);
      const uint4 qb = *reinterpret_cast<const uint4*>(wbuf + (ua + 1) * 64 + part * 16);
      float wa[16], wb[16];
      h8_to_f32(dq8_f16<QF>(make_uint2(qa.x, qa.y), meta0 + ua * MB, 0, part * 2), wa);
      h8_to_f32(dq8_f16<QF>(make_uint2(qa.z, qa.w), meta0 + ua * MB, 0, part * 2 + 1), wa + 8);
      h8_to_f32(dq8_f16<QF>(make_uint2(qb.x, qb.y), meta0 + (ua + 1) * MB, 0, part * 2), wb);
      h8_to_f32(dq8_f16<QF>(make_uint2(qb.z, qb.w), meta0 + (ua + 1) * MB, 0, part * 2 + 1), wb + 8);
#pragma unroll
      for (int t = 0; t < TT; t++) {
        // Rows t >= T hold stale data; their sums are discarded.
        const uint4* xp = reinterpret_cast<const uint4*>(x + (long)t * g.K + c * 16);
        float xv[16];
        h8_to_f32(xp[0], xv);
        h8_to_f32(xp[1], xv + 8);
#pragma unroll
        for (int e = 0; e < 16; e++) {
          acc[t] = fmaf(wa[e], xv[e], acc[t]);
          acc[TT + t] = fmaf(wb[e], xv[e], acc[TT + t]);
        }
      }
    }
    const float v = reduce_scatter<2 * TT>(acc);
    // Row a of token t sits on lane t (TT = 16) or 2t (TT = 8), row b 16 lanes up.
    const float vb = __shfl_down_sync(0xffffffffu, v, 16);
    const int t = TT == 16 ? lane : lane >> 1;
    const bool mine = TT == 16 ? lane < 16 : (lane < 16 && (lane & 1) == 0);
    if (mine && t < T) {
      int ra, rb;
      pair_rows(g.mode, p0 + j, &ra, &rb);
      epi_pair(ep, t, ra, v, vb);
    }
  }
}

template <int TT>
__device__ void gemm_tt(const SmallGemm& g, const uint8_t* wbuf, const __half* x, int T, const EpiParams& ep) {
  switch (g.qf) {
    case QF_Q8_0: gemm_step<QF_Q8_0, TT>(g, wbuf, x, T, ep); break;
    case QF_KMIN: gemm_step<QF_KMIN, TT>(g, wbuf, x, T, ep); break;
    default: gemm_step<QF_Q6K, TT>(g, wbuf, x, T, ep); break;
  }
}
__device__ void gemm_any(const SmallGemm& g, const uint8_t* wbuf, const __half* x, int T, const EpiParams& ep) {
  if (T <= 8) gemm_tt<8>(g, wbuf, x, T, ep);
  else gemm_tt<16>(g, wbuf, x, T, ep);
}

// Attention (bert.go:356-402) for (sequence, head) units, one warp each:
// the unit's Q, K, V rows (written by other CTAs, read through L2) into the
// warp's staging area, zero past the sequence, then the shared warp tile.
__device__ void attention_step(const SmallParams& p, uint8_t* att_smem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * NWARPS + warp, nw = gridDim.x * NWARPS;
  __half(*sQ)[attn::LDS] = reinterpret_cast<__half(*)[attn::LDS]>(att_smem + warp * SmemLayout::ATT_WARP_BYTES);
  __half(*sK)[attn::LDS] = sQ + 16;
  __half(*sV)[attn::LDS] = sK + 16;
  for (int u = gw; u < p.nseq * HEADS; u += nw) {
    const int s = u / HEADS, head = u % HEADS;
    const int t0 = p.offsets[s], L = p.offsets[s + 1] - t0;
    if (L == 0) continue;
    for (int i = lane; i < 3 * 16 * 8; i += 32) {
      const int which = i >> 7, r = (i >> 3) & 15, c = (i & 7) * 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r < L)
        v = __ldcg(reinterpret_cast<const uint4*>(p.qkv + (long)(t0 + r) * 3 * H + which * H + head * HD + c));
      *reinterpret_cast<uint4*>(&sQ[which * 16 + r][c]) = v;
    }
    __syncwarp();
    attn::attn_rows16(sQ, 0, sK, sV, L, p.att + (long)t0 * H + head * HD, H, 0);
    __syncwarp();
  }
}

__global__ void __launch_bounds__(NTHREADS, 1) forward_small_kernel(const __grid_constant__ SmallParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem);
  float* h = reinterpret_cast<float*>(smem + SmemLayout::OFF_H);
  uint8_t* U = smem + SmemLayout::OFF_U;
  __half* x = reinterpret_cast<__half*>(U);
  const uint32_t u_addr = sbase + SmemLayout::OFF_U;
  int* flag = reinterpret_cast<int*>(smem + SmemLayout::OFF_MISC);
  const int T = p.T;

  // Token positions inside their sequences (offsets[nseq+1], packed; empty
  // sequences are skipped).  Every CTA writes the same values.
  if (threadIdx.x < T) {
    const int t = threadIdx.x;
    int s = 0;
    while (s + 1 < p.nseq && p.offsets[s + 1] <= t) s++;
    p.pos[t] = t - p.offsets[s];
  }
  // Weight step w = 4 * layer + m (m: 0 qkv, 1 out, 2 upgate, 3 down).
  const int nsteps = 4 * p.n_layers;
  prefetch_slice(p.layers[0].g[0], sbase + SmemLayout::OFF_W);
  cp_async_commit();
  embed_rows(p, h, T);
  __syncthreads();
  ln_rows(h, x, nullptr, p.embd_w, p.embd_b, p.eps, T);

  unsigned bar = 0;
  for (int w = 0; w < nsteps; w++) {
    const int l = w >> 2, m = w & 3;
    const SmallLayer& L = p.layers[l];
    const SmallGemm& g = L.g[m];
    // This step's input, if other CTAs produced it (one group), then the
    // next step's weight slice into the other buffer (the newest group);
    // wait for everything but the newest.
    if (m == 1) stage_rows(u_addr, p.att, T, H);
    if (m == 3) stage_rows(u_addr, p.ff, T, F);
    cp_async_commit();
    if (w + 1 < nsteps)
      prefetch_slice(p.layers[(w + 1) >> 2].g[(w + 1) & 3], sbase + SmemLayout::OFF_W + ((w + 1) & 1) * WBUF_BYTES);
    cp_async_commit();
    cp_async_wait1();
    __syncthreads();
    const uint8_t* wbuf = smem + SmemLayout::OFF_W + (w & 1) * WBUF_BYTES;
    EpiParams ep{};
    ep.M = T;
    if (m == 0) {
      // Residual LayerNorm after the previous layer's FFN (the embedding
      // LayerNorm for layer 0 ran above), then QKV with RoPE.
      if (l > 0) ln_rows(h, x, p.y, p.layers[l - 1].out_w, p.layers[l - 1].out_b, p.eps, T);
      __syncthreads();
      ep.mode = EPI_QKV;
      ep.N = 3 * H;
      ep.out16 = p.qkv;
      ep.ldo = 3 * H;
      ep.pos = p.pos;
      ep.rope_cos = p.rope_cos;
      ep.rope_sin = p.rope_sin;
      ep.head_dim = HD;
      ep.rope_cols = 2 * H;
      gemm_any(g, wbuf, x, T, ep);
      if (!grid_sync(p.barrier, bar++, p.status, flag)) return;
      attention_step(p, U);  // U (x) is free again
      if (!grid_sync(p.barrier, bar++, p.status, flag)) return;
    } else if (m == 1) {
      ep.mode = EPI_F32;
      ep.N = H;
      ep.out32 = p.y;
      ep.ldo = H;
      gemm_any(g, wbuf, x, T, ep);  // x = staged attention output
      if (!grid_sync(p.barrier, bar++, p.status, flag)) return;
    } else if (m == 2) {
      ln_rows(h, x, p.y, L.attn_w, L.attn_b, p.eps, T);
      __syncthreads();
      ep.mode = EPI_GEGLU;
      ep.N = F;
      ep.out16 = p.ff;
      ep.ldo = F;
      gemm_any(g, wbuf, x, T, ep);
      if (!grid_sync(p.barrier, bar++, p.status, flag)) return;
    } else {
      ep.mode = EPI_F32;
      ep.N = H;
      ep.out32 = p.y;
      ep.ldo = H;
      gemm_any(g, wbuf, x, T, ep);  // x = staged GEGLU output [T][F]
      if (!grid_sync(p.barrier, bar++, p.status, flag)) return;
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  // Final residual LayerNorm; one CTA writes h for the pooling kernel.
  if (blockIdx.x == 0) {
    ln_rows(h, x, p.y, p.layers[p.n_layers - 1].out_w, p.layers[p.n_layers - 1].out_b, p.eps, T);
    __syncthreads();
    for (int i = threadIdx.x; i < T * H; i += NTHREADS) p.h_out[i] = h[i];
  }
}

}  // namespace fs

bool small_forward_supported(const SmallParams& p, int hidden, int ffn, int heads, int sms) {
  if (hidden != SMALL_HIDDEN || ffn != SMALL_FFN || heads != SMALL_HEADS || p.T < 1 || p.T > SMALL_MAX_TOKENS ||
      p.n_layers < 1 || p.n_layers > SMALL_MAX_LAYERS || sms < 1)
    return false;
  // Every step's slice must fit a weight buffer with one CTA per SM.
  for (int l = 0; l < p.n_layers; l++)
    for (const SmallGemm& g : p.layers[l].g) {
      if (!g.w || g.K % TILE_K || g.K > 32 * 16 * 8) return false;
      const long pairs = (g.n_pairs + sms - 1) / sms;
      if (pairs * (g.K / TILE_K) * 2 * (64 + fs::meta_row_bytes(g.qf)) > fs::WBUF_BYTES) return false;
    }
  return true;
}

cudaError_t launch_forward_small(const SmallParams& p, cudaStream_t s) {
  static std::mutex mu;
  static int grid[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (grid[dev] == 0) {
      cudaError_t e = cudaFuncSetAttribute(fs::forward_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           fs::SmemLayout::BYTES);
      if (e != cudaSuccess) return e;
      int sms = 0, per_sm = 0;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fs::forward_small_kernel, fs::NTHREADS,
                                                        fs::SmemLayout::BYTES);
      if (e != cudaSuccess) return e;
      if (per_sm < 1) return cudaErrorNotSupported;
      grid[dev] = sms;  // one CTA per SM
    }
  }
  cudaError_t e = cudaMemsetAsync(p.barrier, 0, sizeof(unsigned), s);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid[dev]);
  cfg.blockDim = dim3(fs::NTHREADS);
  cfg.dynamicSmemBytes = fs::SmemLayout::BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fs::forward_small_kernel, p);
}

}  // namespace le
