// The whole encoder forward for a few tokens (at most SMALL_MAX_TOKENS) in
// one persistent kernel: one CTA per SM, all resident (cooperative launch).
//
// At batch 1 the forward is a chain of small dependent steps over 120 MB of
// weights (Q8_0).  Weights never depend on activations, so each CTA streams
// the weight pages of its share of every step into a shared-memory ring
// ahead of use (TMA bulk copies, mbarrier-tracked: one thread issues page k + R
// as soon as the warps are done with page k), and the chain itself only
// waits for the activations other CTAs produce.
//
// Per layer, CTA c:
//   QKV     LayerNorm of its own copy of the residual stream (every CTA holds
//           h and applies each LayerNorm itself, in one fixed order, so all
//           copies are equal), then its 16-row QKV tile(s) with RoPE
//   ATT     (12 CTAs, one per head) once the head's 12 QKV tiles are done:
//           attention of every sequence for that head
//   OUT     (48 CTAs) once all heads are done: an output-projection tile
//           (one sequence of at most 8 tokens: no ATT step; each OUT CTA
//           computes every head's attention into shared memory itself once
//           all QKV tiles are done)
//   UG      every CTA, once all output tiles are done: LayerNorm, then its
//           2-3 up/gate tiles with GEGLU
//   DOWN    (144 CTAs) once every CTA finished UG: one K slice of a
//           down-projection tile (48 tiles x 3 slices of 1,024 columns); the
//           slices' partial sums are added by the LayerNorm that reads them
// and at the end CTA s (s < number of sequences) applies the final LayerNorm
// and mean-pools, normalises and truncates sequence s into the output.
// Each hand-off is a release-add on a counter after the producing tile's
// stores and an acquire poll by the consumers (bounded: WAIT_LIMIT_NS, then
// DE_TIMEOUT and every CTA leaves); there is no grid-wide barrier.
//
// The GEMM tiles run the row16 mma.sync primitive of gemm_r16.cuh with the
// same K split and reduction order as the small-batch GEMM kernel, and
// attention the warp tile of attention_tile.cuh as the attention kernels do,
// so a sequence gets the same bits here as in a batch of up to 63 tokens.
#include "attention_tile.cuh"
#include "gemm_r16.cuh"
#include "gguf_decode.cuh"
#include "kernels.h"
#include "ln_warp.cuh"
#include "pool_seq.cuh"
#include "tcgen05.cuh"

#include <mutex>

namespace le {
namespace fs {

using tcx::bulk_load;
using tcx::mbar_expect_tx;
using tcx::mbar_init;
using tcx::mbar_wait;

constexpr int H = SMALL_HIDDEN;
constexpr int F = SMALL_FFN;
constexpr int HEADS = SMALL_HEADS;
constexpr int HD = H / HEADS;
constexpr int NCW = r16::WARPS;            // warps (the K split of gemm_r16.cuh)
constexpr int NTHREADS = NCW * 32;
constexpr int NCT = NTHREADS;
// The thread that issues the weight pages' bulk copies: the CTA's last,
// which has no output item of a step's reduction at 8 tokens (thread 0 also
// polls the hand-off counters), so the issue is off the step's critical path.
constexpr int ISSUER = NCT - 1;
constexpr int LDX = H + 8;                 // padded fp16 row stride of x
// A page is one work item: a 16-row tile's K slice (gemm_r16.cuh: K = 768 is
// one slice of 12 chunks, K = 3072 three of 16), contiguous in the row16
// layout.
constexpr int MAX_PAGE_CHUNKS = r16::KSLICE / TILE_K;
constexpr int SLOT = MAX_PAGE_CHUNKS * r16::chunk_bytes(QF_KMIN);  // 20,480 B: the largest page
constexpr int N_Y2 = 3;                    // K slices of a down-projection tile
constexpr int ATT_WARP_BYTES = 3 * 16 * attn::LDS * 2;
constexpr int SMEM_MAX = 232448;
constexpr int MAX_SLOTS = 16;
constexpr int MAX_TILES = 3;               // tiles of one step per CTA (up/gate: 384 over 148 CTAs)

// Hand-off counters (zeroed before each launch), one 128-byte line each.
constexpr int CNT_STRIDE = 32;
constexpr int CNT_QKV = 0;  // + head: QKV tiles done
constexpr int CNT_ATT = HEADS;
constexpr int CNT_Y1 = HEADS + 1;
constexpr int CNT_FF = HEADS + 2;
constexpr int CNT_Y2 = HEADS + 3;
constexpr int CNT_QKV_ALL = HEADS + 4;  // QKV tiles done, every head (calls of one sequence)
constexpr int N_CNT = HEADS + 5;
// Calls of one sequence of at most 8 tokens: every output-projection CTA
// computes all the heads' attention itself (AW warps, two rounds) into its
// shared memory after the per-warp staging, instead of 12 attention CTAs
// and two more hand-offs.
constexpr int AW = 6;

template <int NT>
struct Lay {
  static constexpr int TS = 8 * NT;
  static constexpr int H_BYTES = TS * H * 4;
  static constexpr int X_BYTES = TS * LDX * 2;
  static constexpr int U_BYTES = X_BYTES > NCW * ATT_WARP_BYTES ? X_BYTES : NCW * ATT_WARP_BYTES;
  static constexpr int RED_BYTES = MAX_TILES * NCW * NT * 32 * 16;
  static constexpr int STEP_BYTES = SMALL_MAX_LAYERS * 4 * 8;  // the page walk's per-step cache
  static constexpr int FIXED = H_BYTES + U_BYTES + RED_BYTES + STEP_BYTES + MAX_SLOTS * 8 + 64;
  static constexpr int R = (SMEM_MAX - FIXED) / SLOT < MAX_SLOTS ? (SMEM_MAX - FIXED) / SLOT : MAX_SLOTS;
  static constexpr int OFF_RING = 0;
  static constexpr int OFF_H = R * SLOT;
  static constexpr int OFF_U = OFF_H + H_BYTES;
  static constexpr int OFF_RED = OFF_U + U_BYTES;
  static constexpr int OFF_STEP = OFF_RED + RED_BYTES;  // int2 info[l][m]
  static constexpr int OFF_BAR = OFF_STEP + STEP_BYTES;  // full[R]
  static constexpr int OFF_MISC = OFF_BAR + R * 8;
  static constexpr int BYTES = OFF_MISC + 64;
  static_assert(R >= MAX_TILES + 1, "the ring must hold a step's pages and the next one");
  static_assert(OFF_STEP % 16 == 0, "step cache alignment");
  static_assert(NT != 1 || AW * ATT_WARP_BYTES + 8 * LDX * 2 <= U_BYTES, "one-sequence attention output");
  static_assert((AW * ATT_WARP_BYTES) % 16 == 0, "attention output alignment");
  static_assert(BYTES <= SMEM_MAX, "shared memory budget");
};

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Barrier of the CTA's warps (named barrier 1).
__device__ __forceinline__ void bar_compute() { asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory"); }

// Tiles [t0, t1) of step m for CTA c: an even split, the down projection's
// shifted by half the grid so its CTAs are not the output projection's.
__device__ __forceinline__ void tile_range(int m, int n_tiles, int* t0, int* t1) {
  const int G = gridDim.x;
  const int c = m == 3 ? (int)((blockIdx.x + G / 2) % G) : (int)blockIdx.x;
  *t0 = (int)((long)n_tiles * c / G);
  *t1 = (int)((long)n_tiles * (c + 1) / G);
}
__device__ __forceinline__ int att_cta(int head) { return (int)((long)head * gridDim.x / HEADS); }
// Work items (pages) of step g: its tiles times its K slices; item i is tile
// i / slices, slice i % slices.
__device__ __forceinline__ int items_of(const SmallGemm& g) { return g.tiles * r16::n_slices(g.K); }
__device__ __forceinline__ int page_chunks(const SmallGemm& g, int slice) {
  const int k0 = slice * r16::KSLICE;
  return (g.K - k0 < r16::KSLICE ? g.K - k0 : r16::KSLICE) / TILE_K;
}

template <int R_>
struct SharedT {
  static constexpr int R = R_;
  uint8_t* ring;
  float* h;
  __half* x;
  uint8_t* U;
  float4* red;
  const int2* step_info;  // per (layer, step): {K | qf << 16, first item | end item << 16} of this CTA
  uint32_t bar0;
  volatile int* abort;
  volatile int* flag;
};

// Compute threads: wait until *c >= target (thread 0 polls with acquire
// loads; the others learn the outcome at the barrier).  False if the wait
// timed out or another CTA reported a failure.
template <class SH>
__device__ bool wait_cnt(const SmallParams& p, const SH& S, int idx, unsigned target, int site) {
  if (threadIdx.x == 0) {
    const unsigned* c = p.sync + idx * CNT_STRIDE;
    int ok = !*S.abort;
    if (ok && ld_acquire(c) < target) {
      const uint64_t t0 = globaltimer_ns();
      for (uint32_t i = 1;; i++) {
        if (ld_acquire(c) >= target) break;
        if ((i & 63) == 0) {
          if (ld_acquire(reinterpret_cast<const unsigned*>(&p.status->code)) != 0) {
            ok = 0;
            break;
          }
          if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) {
            report(p.status, DE_TIMEOUT, site, (int)blockIdx.x);
            ok = 0;
            break;
          }
        }
      }
    }
    if (!ok) *S.abort = 1;
    *S.flag = ok;
  }
  bar_compute();
  return *S.flag != 0;
}

// Compute threads: after this CTA's stores of a hand-off, add 1 to counter idx.
__device__ __forceinline__ void signal(const SmallParams& p, int idx) {
  bar_compute();
  if (threadIdx.x == 0) red_release_add(p.sync + idx * CNT_STRIDE, 1u);
}

// LayerNorm (ops_simd.go:7-24) of h[t] (+ y[t] when y) into h[t] and its fp16
// copy x[t]; one warp per token row (ln_row_stats order).  y holds `nparts`
// partial sums (the K slices of the projection, SMALL_MAX_TOKENS rows apart),
// added in slice order and then to the residual.  Every global load (y,
// gamma, beta) is issued before the statistics, so the row waits for one
// memory round trip.
__device__ void ln_rows(float* h, __half* x, const float* y, const float* w, const float* b, float eps, int T,
                        int nparts = 1) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t = warp; t < T; t += NCW) {
    float4 v[H / 128], wv[H / 128], bv[H / 128], yv[N_Y2][H / 128];
#pragma unroll
    for (int i = 0; i < H / 128; i++) {
      const int c = (i * 32 + lane) * 4;
      wv[i] = __ldg(reinterpret_cast<const float4*>(w + c));
      bv[i] = __ldg(reinterpret_cast<const float4*>(b + c));
      v[i] = *reinterpret_cast<const float4*>(h + t * H + c);
#pragma unroll
      for (int q = 0; q < N_Y2; q++)
        if (y && q < nparts)
          yv[q][i] = __ldcg(reinterpret_cast<const float4*>(y + (long)q * SMALL_MAX_TOKENS * H + (long)t * H + c));
    }
    if (y) {
#pragma unroll
      for (int i = 0; i < H / 128; i++) {
        float4 d = yv[0][i];
#pragma unroll
        for (int q = 1; q < N_Y2; q++)
          if (q < nparts)
            d = make_float4(__fadd_rn(d.x, yv[q][i].x), __fadd_rn(d.y, yv[q][i].y), __fadd_rn(d.z, yv[q][i].z),
                            __fadd_rn(d.w, yv[q][i].w));
        v[i] = make_float4(__fadd_rn(v[i].x, d.x), __fadd_rn(v[i].y, d.y), __fadd_rn(v[i].z, d.z),
                           __fadd_rn(v[i].w, d.w));
      }
    }
    float mean, inv;
    ln_row_stats(v, H / 128, H, eps, &mean, &inv);
#pragma unroll
    for (int i = 0; i < H / 128; i++) {
      const int c = (i * 32 + lane) * 4;
      const float4 o = ln_apply(v[i], mean, inv, wv[i], bv[i]);
      *reinterpret_cast<float4*>(h + t * H + c) = o;
      uint2 hh;
      hh.x = pack_half2(o.x, o.y);
      hh.y = pack_half2(o.z, o.w);
      *reinterpret_cast<uint2*>(x + t * LDX + c) = hh;
    }
  }
}

// Embedding rows (bert.go:227-247): token_embd row + token_types row 0.  The
// rows' bytes are first staged into `stage` with 16-byte loads from the
// 16-byte boundary at or below each row (all issued at once; the embedding
// buffer carries 16 spare bytes), then decoded from shared memory.
__device__ void embed_rows(const SmallParams& p, float* h, uint8_t* stage, int T) {
  const int rb = (int)p.emb_row_bytes;
  const int stride = (rb + 31) & ~15;  // staged bytes per row (multiple of 16)
  const int n16 = stride / 16;
  constexpr int PER = 8;  // loads in flight per thread before their stores
  for (int i0 = threadIdx.x; i0 < T * n16; i0 += NCT * PER) {
    uint4 v[PER];
#pragma unroll
    for (int q = 0; q < PER; q++) {
      const int i = i0 + q * NCT;
      if (i < T * n16) {
        const int t = i / n16, j = i % n16;
        int id = p.ids[t];
        if (id < 0 || id >= p.vocab) id = 0;
        const uintptr_t a = reinterpret_cast<uintptr_t>(p.emb + (long)id * rb) & ~(uintptr_t)15;
        v[q] = __ldg(reinterpret_cast<const uint4*>(a) + j);
      }
    }
#pragma unroll
    for (int q = 0; q < PER; q++) {
      const int i = i0 + q * NCT;
      if (i < T * n16) *reinterpret_cast<uint4*>(stage + (i / n16) * stride + (i % n16) * 16) = v[q];
    }
  }
  bar_compute();
  for (int i = threadIdx.x; i < T * H; i += NCT) {
    const int t = i / H, c = i % H;
    const int id = p.ids[t];
    if (id < 0 || id >= p.vocab) {
      if (c == 0) report(p.status, DE_BOUNDS, 2, id);
    }
    const int sid = (id < 0 || id >= p.vocab) ? 0 : id;
    const int mis = (int)(reinterpret_cast<uintptr_t>(p.emb + (long)sid * rb) & 15);
    h[i] = __fadd_rn(gguf_elem(p.emb_type, stage + t * stride + mis, c), p.type0[c]);
  }
}

// L2 prefetch of the small per-layer tensors the chain reads after waits (the
// LayerNorm vectors, the RoPE rows of the call's positions), spread over the
// CTAs, so those reads hit L2 instead of DRAM.
__device__ void prefetch_small(const SmallParams& p) {
  const int G = gridDim.x;
  const int per_layer = 4 * (H * 4 / 128);  // 128-byte lines of the four vectors
  for (int i = blockIdx.x * NCT + threadIdx.x; i < p.n_layers * per_layer; i += G * NCT) {
    const int l = i / per_layer, r = i % per_layer, v = r / (H * 4 / 128), line = r % (H * 4 / 128);
    const SmallLayer& L = p.layers[l];
    const float* base = v == 0 ? L.attn_w : v == 1 ? L.attn_b : v == 2 ? L.out_w : L.out_b;
    asm volatile("prefetch.global.L2 [%0];" ::"l"(base + line * 32));
  }
  if (blockIdx.x == 0 && threadIdx.x < p.T) {
    const int t = threadIdx.x;
    int s = 0;
    while (s + 1 < p.nseq && p.offsets[s + 1] <= t) s++;
    const int pos = t - p.offsets[s];
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p.rope_cos + pos * (HD / 2)));
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p.rope_sin + pos * (HD / 2)));
  }
}

// Attention (bert.go:356-402) of head `head` for every sequence, one warp per
// sequence: its Q, K, V rows (from other CTAs, read through L2) into the
// warp's staging area, zero past the sequence, then the shared warp tile.
__device__ void attention_head(const SmallParams& p, uint8_t* U, int head) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __half(*sQ)[attn::LDS] = reinterpret_cast<__half(*)[attn::LDS]>(U + warp * ATT_WARP_BYTES);
  __half(*sK)[attn::LDS] = sQ + 16;
  __half(*sV)[attn::LDS] = sK + 16;
  for (int s = warp; s < p.nseq; s += NCW) {
    const int t0 = p.offsets[s], L = p.offsets[s + 1] - t0;
    if (L == 0) continue;
    // All twelve 16-byte loads of the lane first, then the stores (the
    // shared-memory stores go through generic pointers, which the compiler
    // cannot separate from the global loads).
    uint4 v[12];
#pragma unroll
    for (int j = 0; j < 12; j++) {
      const int i = lane + 32 * j, which = i >> 7, r = (i >> 3) & 15, c = (i & 7) * 8;
      v[j] = r < L ? __ldcg(reinterpret_cast<const uint4*>(p.qkv + (long)(t0 + r) * 3 * H + which * H + head * HD + c))
                   : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < 12; j++) {
      const int i = lane + 32 * j, which = i >> 7, r = (i >> 3) & 15, c = (i & 7) * 8;
      *reinterpret_cast<uint4*>(&sQ[which * 16 + r][c]) = v[j];
    }
    __syncwarp();
    attn::attn_rows16(sQ, 0, sK, sV, L, p.att + (long)t0 * H + head * HD, H, 0);
    __syncwarp();
  }
}

// Attention of every head for a call of one sequence (t0 = 0, L = T), on
// an output-projection CTA: heads over warps 0..AW-1, each staged and
// computed exactly as attention_head stages and computes a sequence, the
// output into `att` (row stride LDX, shared memory).
__device__ void attention_all_heads(const SmallParams& p, uint8_t* U, __half* att) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp >= AW) return;
  __half(*sQ)[attn::LDS] = reinterpret_cast<__half(*)[attn::LDS]>(U + warp * ATT_WARP_BYTES);
  __half(*sK)[attn::LDS] = sQ + 16;
  __half(*sV)[attn::LDS] = sK + 16;
  const int L = p.T;
  for (int head = warp; head < HEADS; head += AW) {
    uint4 v[12];
#pragma unroll
    for (int j = 0; j < 12; j++) {
      const int i = lane + 32 * j, which = i >> 7, r = (i >> 3) & 15, c = (i & 7) * 8;
      v[j] = r < L ? __ldcg(reinterpret_cast<const uint4*>(p.qkv + (long)r * 3 * H + which * H + head * HD + c))
                   : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < 12; j++) {
      const int i = lane + 32 * j, which = i >> 7, r = (i >> 3) & 15, c = (i & 7) * 8;
      *reinterpret_cast<uint4*>(&sQ[which * 16 + r][c]) = v[j];
    }
    __syncwarp();
    attn::attn_rows16(sQ, 0, sK, sV, L, att + head * HD, LDX, 0);
    __syncwarp();
  }
}

// The CTA's page sequence (every step's work items in consumption order),
// walked by the ISSUER thread as it issues the pages' bulk copies: page k goes to ring
// slot k % R once page k - R has been consumed.
struct PageIter {
  int l = 0, m = 0, it = 0, t1 = -1;
  uint32_t issued = 0;        // pages issued so far
  const uint8_t* w = nullptr;  // the current step's row16 weight
};

// Issue the next page of the sequence into its slot (ISSUER); false when
// the sequence is exhausted.
template <class SH>
__device__ bool issue_next(const SmallParams& p, const SH& S, PageIter& pi) {
  while (pi.l < p.n_layers) {
    const int sx = pi.l * 4 + pi.m;
    const int2 inf = S.step_info[sx];
    if (pi.t1 < 0) {
      pi.it = inf.y & 0xFFFF;
      pi.t1 = inf.y >> 16;
      pi.w = p.layers[pi.l].g[pi.m].w;
    }
    if (pi.it < pi.t1) {
      const int K = inf.x & 0xFFFF, cb = r16::chunk_bytes(inf.x >> 16), nch = K / TILE_K;
      const int ns = r16::n_slices(K), tile = pi.it / ns, slice = pi.it % ns;
      const int c0 = slice * (r16::KSLICE / TILE_K);
      const uint32_t slot = pi.issued % SH::R;
      const uint32_t bytes = (uint32_t)((nch - c0 < r16::KSLICE / TILE_K ? nch - c0 : r16::KSLICE / TILE_K) * cb);
      const uint8_t* src = pi.w + ((long)tile * nch + c0) * cb;
      mbar_expect_tx(S.bar0 + 8 * slot, bytes);
      bulk_load(tcx::smem_u32(S.ring + slot * SLOT), src, bytes, S.bar0 + 8 * slot);
      pi.it++;
      pi.issued++;
      return true;
    }
    pi.t1 = -1;
    if (++pi.m == 4) {
      pi.m = 0;
      pi.l++;
    }
  }
  return false;
}

// ISSUER before the CTA exits: every issued copy has landed (a CTA must not
// exit with bulk copies into its shared memory in flight).
template <class SH>
__device__ void drain(const SH& S, const PageIter& pi) {
  const uint32_t first = pi.issued > (uint32_t)SH::R ? pi.issued - SH::R : 0;
  volatile int no_abort = 0;
  for (uint32_t sq = first; sq < pi.issued; sq++)
    mbar_wait(S.bar0 + 8 * (sq % SH::R), (sq / SH::R) & 1, &no_abort, nullptr, 62);
}

// Work items it0 .. it0+n-1 (n <= MAX_TILES) of step g, one page each at
// ring positions seq0.. of the page sequence (the items of one call are K
// slices of equal size): every warp runs its units of every item (the B
// operand fragments loaded once per unit and shared by the items), then the
// partials, the reduction and the epilogue of all items.  An item of a
// sliced step (K > 1024) writes its slice's partial sums to
// ep.out32 + slice * SMALL_MAX_TOKENS * ldo; the reader adds the slices.
// B operand: x in shared memory (xs, stride LDX) or a global fp16 matrix
// (xg, stride ldg; all of the warp's fragments are loaded before the first
// MMA, one memory round trip).  For EPI_QKV the RoPE cos/sin of each output
// item come preloaded in rc/rs (item i < 64 NT of the first tile).  Returns
// false if a page wait failed.
template <int QF, int NT, int UMAX, bool GB, class SH>
__device__ bool gemm_tiles(const SmallParams& p, const SH& S, PageIter& pi, const SmallGemm& g, int it0, int n,
                           uint32_t seq0, const __half* xs, const __half* xg, int ldg, const EpiParams& ep, float rc,
                           float rs) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, gi = lane >> 2, ti = lane & 3;
  const int ns = r16::n_slices(g.K);
  const int slice0 = it0 % ns;
  int u0, u1;
  r16::slice_units(g.K, slice0, w, &u0, &u1);  // the same count in every item of the call
  const int ubase = slice0 * (r16::KSLICE / 32);
  // B fragments from global memory first: their latency overlaps the page waits.
  uint4 bq[GB ? UMAX : 1][NT];
  if constexpr (GB) {
#pragma unroll
    for (int i = 0; i < UMAX; i++)
#pragma unroll
      for (int nn = 0; nn < NT; nn++) {
        const int u = u0 + i, m = 8 * nn + gi;
        const int k = (u >> 1) * TILE_K + 16 * ti + 8 * (u & 1);
        bq[i][nn] = (u < u1 && m < p.T) ? __ldcg(reinterpret_cast<const uint4*>(xg + (long)m * ldg + k))
                                        : make_uint4(0, 0, 0, 0);
      }
  }
  bool ok = true;
  for (int i = 0; i < n && ok; i++) {
    const uint32_t sq = seq0 + i;
    ok = mbar_wait(S.bar0 + 8 * (sq % SH::R), (sq / SH::R) & 1, S.abort, p.status, 60);
  }
  float acc[MAX_TILES][NT][4];
#pragma unroll
  for (int i = 0; i < MAX_TILES; i++)
#pragma unroll
    for (int nn = 0; nn < NT; nn++) acc[i][nn][0] = acc[i][nn][1] = acc[i][nn][2] = acc[i][nn][3] = 0.f;
  if (ok) {
#pragma unroll
    for (int i = 0; i < UMAX; i++) {
      const int u = u0 + i;
      if (u >= u1) break;
      const int c = u >> 1, hf = u & 1;
      const int k = c * TILE_K + 16 * ti + 8 * hf;
      const int cl = (u - ubase) >> 1;  // chunk within the item's page
      uint4 b[NT];
#pragma unroll
      for (int nn = 0; nn < NT; nn++)
        b[nn] = GB ? bq[GB ? i : 0][nn] : *reinterpret_cast<const uint4*>(xs + (8 * nn + gi) * LDX + k);
#pragma unroll
      for (int tt = 0; tt < MAX_TILES; tt++) {
        if (tt >= n) break;
        const uint32_t sq = seq0 + tt;
        const uint8_t* chunk = S.ring + (sq % SH::R) * SLOT + cl * r16::chunk_bytes(QF);
        const uint2 qa = *reinterpret_cast<const uint2*>(chunk + gi * TILE_K + 16 * ti + 8 * hf);
        const uint2 qb = *reinterpret_cast<const uint2*>(chunk + (gi + 8) * TILE_K + 16 * ti + 8 * hf);
        const uint4 ha = dq8_f16<QF>(qa, chunk + r16::CHUNK_Q, gi, 2 * ti + hf);
        const uint4 hb = dq8_f16<QF>(qb, chunk + r16::CHUNK_Q, gi + 8, 2 * ti + hf);
#pragma unroll
        for (int nn = 0; nn < NT; nn++) {
          r16::mma16816(acc[tt][nn], ha.x, hb.x, ha.y, hb.y, b[nn].x, b[nn].y);
          r16::mma16816(acc[tt][nn], ha.z, hb.z, ha.w, hb.w, b[nn].z, b[nn].w);
        }
      }
    }
  }
#pragma unroll
  for (int tt = 0; tt < MAX_TILES; tt++)
    if (tt < n) r16::store_partials<NT>(S.red + tt * NCW * NT * 32, acc[tt]);
  bar_compute();
  // The items' pages are consumed: their slots take the next pages (the
  // proxy fence orders the warps' reads before the copies' writes).
  if (threadIdx.x == ISSUER) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    for (int q = 0; q < n; q++) issue_next(p, S, pi);
  }
  if (*S.abort) return false;
  for (int i = threadIdx.x; i < 64 * NT * n; i += NCT) {
    const int tt = i / (64 * NT), it = i % (64 * NT);
    const int item = it0 + tt, tile = item / ns, slice = item % ns;
    int q, m;
    float va, vb;
    r16::reduce_item<NT>(S.red + tt * NCW * NT * 32, it, &q, &m, &va, &vb);
    if (m >= p.T) continue;
    const int a = r16::pair_virtual_row(g.mode, tile, q);
    if (ep.mode == EPI_QKV && a < ep.rope_cols) {
      // epi_pair's RoPE with the preloaded table values.
      const float x0 = __fsub_rn(__fmul_rn(va, rc), __fmul_rn(vb, rs));
      const float x1 = __fadd_rn(__fmul_rn(va, rs), __fmul_rn(vb, rc));
      *reinterpret_cast<uint32_t*>(ep.out16 + (long)m * ep.ldo + a) = pack_half2(x0, x1);
    } else if (ns > 1) {
      float* o = ep.out32 + (long)slice * SMALL_MAX_TOKENS * ep.ldo + (long)m * ep.ldo;
      *reinterpret_cast<float2*>(o + a) = make_float2(va, vb);
    } else {
      epi_pair(ep, m, a, va, vb);
    }
  }
  bar_compute();  // the partials buffer is free for the next items
  return true;
}

template <int NT, int UMAX, bool GB, class SH>
__device__ bool gemm_tiles_any(const SmallParams& p, const SH& S, PageIter& pi, const SmallGemm& g, int t0, int nt,
                               uint32_t seq0, const __half* xs, const __half* xg, int ldg, const EpiParams& ep,
                               float rc = 0.f, float rs = 0.f) {
  switch (g.qf) {
    case QF_Q8_0: return gemm_tiles<QF_Q8_0, NT, UMAX, GB, SH>(p, S, pi, g, t0, nt, seq0, xs, xg, ldg, ep, rc, rs);
    case QF_KMIN: return gemm_tiles<QF_KMIN, NT, UMAX, GB, SH>(p, S, pi, g, t0, nt, seq0, xs, xg, ldg, ep, rc, rs);
    default: return gemm_tiles<QF_Q6K, NT, UMAX, GB, SH>(p, S, pi, g, t0, nt, seq0, xs, xg, ldg, ep, rc, rs);
  }
}

template <int NT>
__global__ void __launch_bounds__(NTHREADS, 1) forward_small_kernel(const __grid_constant__ SmallParams p) {
  using L = Lay<NT>;
  extern __shared__ __align__(128) uint8_t smem[];
  SharedT<L::R> S;
  S.ring = smem + L::OFF_RING;
  S.h = reinterpret_cast<float*>(smem + L::OFF_H);
  S.U = smem + L::OFF_U;
  S.x = reinterpret_cast<__half*>(S.U);
  // One sequence of at most 8 tokens: the attention output goes after the
  // AW warps' staging areas (past x, which the output phase does not read).
  const bool one_seq = NT == 1 && p.nseq == 1;
  __half* att_s = reinterpret_cast<__half*>(S.U + AW * ATT_WARP_BYTES);
  S.red = reinterpret_cast<float4*>(smem + L::OFF_RED);
  S.step_info = reinterpret_cast<const int2*>(smem + L::OFF_STEP);
  S.bar0 = tcx::smem_u32(smem + L::OFF_BAR);
  S.abort = reinterpret_cast<volatile int*>(smem + L::OFF_MISC);
  S.flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC + 4);
  const int T = p.T;

  // The page walk's per-step cache: K, format and this CTA's items of step
  // (l, m), one thread per step (the walk then needs no division of the
  // grid and no parameter loads per page).
  if (threadIdx.x < p.n_layers * 4) {
    const int l = threadIdx.x >> 2, m = threadIdx.x & 3;
    const SmallGemm& g = p.layers[l].g[m];
    int t0, t1;
    tile_range(m, items_of(g), &t0, &t1);
    reinterpret_cast<int2*>(smem + L::OFF_STEP)[threadIdx.x] = make_int2(g.K | (g.qf << 16), t0 | (t1 << 16));
  }
  __syncthreads();
  PageIter pi;  // (meaningful in the ISSUER thread)
  if (threadIdx.x == ISSUER) {
    for (int i = 0; i < L::R; i++) mbar_init(S.bar0 + 8 * i, 1);
    *S.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int i = 0; i < L::R; i++)
      if (!issue_next(p, S, pi)) break;
  }
  __syncthreads();

  // Token positions inside their sequences (every CTA writes the same values).
  prefetch_small(p);
  if (threadIdx.x < T) {
    const int t = threadIdx.x;
    int s = 0;
    while (s + 1 < p.nseq && p.offsets[s + 1] <= t) s++;
    p.pos[t] = t - p.offsets[s];
  }
  embed_rows(p, S.h, S.U, T);
  bar_compute();
  ln_rows(S.h, S.x, nullptr, p.embd_w, p.embd_b, p.eps, T);
  bar_compute();

  uint32_t seq = 0;  // next page of this CTA's sequence
  const int G = gridDim.x;
  for (int l = 0; l < p.n_layers; l++) {
    const SmallLayer& Ly = p.layers[l];
    // ---- QKV: residual LayerNorm of the previous layer's FFN, QKV + RoPE.
    {
      const SmallGemm& g = Ly.g[0];
      int t0, t1;
      tile_range(0, g.tiles, &t0, &t1);
      // The RoPE table values of this thread's first-tile output item, loaded
      // before the wait.
      float rc = 0.f, rs = 0.f;
      if (t1 > t0 && threadIdx.x < 64 * NT) {
        const int q = (threadIdx.x & 63) >> 3;
        const int m = 8 * (threadIdx.x >> 6) + 2 * ((threadIdx.x >> 1) & 3) + (threadIdx.x & 1);
        const int a = 16 * t0 + 2 * q;
        if (m < T && a < 2 * H) {
          const long r = (long)p.pos[m] * (HD / 2) + ((a % HD) >> 1);
          rc = __ldg(p.rope_cos + r);
          rs = __ldg(p.rope_sin + r);
        }
      }
      if (l > 0) {
        const SmallGemm& prev = p.layers[l - 1].g[3];
        if (!wait_cnt(p, S, CNT_Y2, (unsigned)(items_of(prev) * l), 70)) goto out;
        ln_rows(S.h, S.x, p.y2, p.layers[l - 1].out_w, p.layers[l - 1].out_b, p.eps, T, r16::n_slices(prev.K));
        bar_compute();
      }
      EpiParams ep{};
      ep.M = T;
      ep.mode = EPI_QKV;
      ep.N = 3 * H;
      ep.out16 = p.qkv;
      ep.ldo = 3 * H;
      ep.pos = p.pos;
      ep.rope_cos = p.rope_cos;
      ep.rope_sin = p.rope_sin;
      ep.head_dim = HD;
      ep.rope_cols = 2 * H;
      for (int t = t0; t < t1; t++) {
        // RoPE values preloaded for the first tile only.
        if (t == t0) {
          if (!gemm_tiles_any<NT, 3, false>(p, S, pi, g, t, 1, seq, S.x, nullptr, 0, ep, rc, rs)) goto out;
        } else {
          if (!gemm_tiles_any<NT, 3, false>(p, S, pi, g, t, 1, seq, S.x, nullptr, 0, ep)) goto out;
        }
        seq += 1;
        signal(p, one_seq ? CNT_QKV_ALL : CNT_QKV + ((16 * t) % H) / HD);
      }
    }
    // ---- Attention of one head, once its 12 QKV tiles are in.
    for (int hd = 0; hd < HEADS && !one_seq; hd++) {
      if (att_cta(hd) != (int)blockIdx.x) continue;
      if (!wait_cnt(p, S, CNT_QKV + hd, (unsigned)(3 * HD / 16 * (l + 1)), 71)) goto out;
      attention_head(p, S.U, hd);
      signal(p, CNT_ATT);
    }
    // ---- Output projection tiles, once every head is in.
    {
      const SmallGemm& g = Ly.g[1];
      int t0, t1;
      tile_range(1, items_of(g), &t0, &t1);
      EpiParams ep{};
      ep.M = T;
      ep.mode = EPI_F32;
      ep.N = H;
      ep.out32 = p.y1;
      ep.ldo = H;
      if (one_seq) {
        if (t1 > t0) {
          if (!wait_cnt(p, S, CNT_QKV_ALL, (unsigned)(items_of(Ly.g[0]) * (l + 1)), 72)) goto out;
          attention_all_heads(p, S.U, att_s);
          bar_compute();
        }
        for (int t = t0; t < t1; t++) {
          if (!gemm_tiles_any<NT, 3, false>(p, S, pi, g, t, 1, seq, att_s, nullptr, 0, ep)) goto out;
          seq += 1;
          signal(p, CNT_Y1);
        }
      } else {
        if (t1 > t0 && !wait_cnt(p, S, CNT_ATT, (unsigned)(HEADS * (l + 1)), 72)) goto out;
        for (int t = t0; t < t1; t++) {
          if (!gemm_tiles_any<NT, 3, true>(p, S, pi, g, t, 1, seq, nullptr, p.att, H, ep)) goto out;
          seq += 1;
          signal(p, CNT_Y1);
        }
      }
    }
    // ---- Up/gate: residual LayerNorm after attention, GEGLU tiles.
    {
      if (!wait_cnt(p, S, CNT_Y1, (unsigned)(items_of(Ly.g[1]) * (l + 1)), 73)) goto out;
      ln_rows(S.h, S.x, p.y1, Ly.attn_w, Ly.attn_b, p.eps, T);
      bar_compute();
      EpiParams ep{};
      ep.M = T;
      ep.mode = EPI_GEGLU;
      ep.N = F;
      ep.out16 = p.ff;
      ep.ldo = F;
      const SmallGemm& g = Ly.g[2];
      int t0, t1;
      tile_range(2, items_of(g), &t0, &t1);
      for (int t = t0; t < t1; t += MAX_TILES) {
        const int n = t1 - t < MAX_TILES ? t1 - t : MAX_TILES;
        if (!gemm_tiles_any<NT, 3, false>(p, S, pi, g, t, n, seq, S.x, nullptr, 0, ep)) goto out;
        seq += n;
      }
      signal(p, CNT_FF);
    }
    // ---- Down projection: (tile, K slice) items, one page each, once every
    // CTA finished up/gate; the next LayerNorm adds the slices' partial sums.
    {
      const SmallGemm& g = Ly.g[3];
      int t0, t1;
      tile_range(3, items_of(g), &t0, &t1);
      if (t1 > t0 && !wait_cnt(p, S, CNT_FF, (unsigned)(G * (l + 1)), 74)) goto out;
      EpiParams ep{};
      ep.M = T;
      ep.mode = EPI_F32;
      ep.N = H;
      ep.out32 = p.y2;
      ep.ldo = H;
      for (int t = t0; t < t1; t++) {
        if (!gemm_tiles_any<NT, 4, true>(p, S, pi, g, t, 1, seq, nullptr, p.ff, F, ep)) goto out;
        seq += 1;
        signal(p, CNT_Y2);
      }
    }
  }
  // Final residual LayerNorm, then CTA s pools sequence s straight from its
  // shared-memory rows (the pool kernel's thread layout and summation order).
  if (blockIdx.x < p.nseq) {
    const SmallGemm& last = p.layers[p.n_layers - 1].g[3];
    if (!wait_cnt(p, S, CNT_Y2, (unsigned)(items_of(last) * p.n_layers), 75)) goto out;
    ln_rows(S.h, S.x, p.y2, p.layers[p.n_layers - 1].out_w, p.layers[p.n_layers - 1].out_b, p.eps, T,
            r16::n_slices(last.K));
    bar_compute();
    if (threadIdx.x < H / 4) {
      const int s = blockIdx.x;
      pool_seq<8>(S.h, p.offsets[s], p.offsets[s + 1], H, p.out_dim, p.out + (long)s * p.out_dim,
               reinterpret_cast<double*>(S.red), [] { asm volatile("bar.sync 2, %0;" ::"n"(H / 4) : "memory"); });
    }
  }
out:
  if (threadIdx.x == ISSUER) drain(S, pi);
}

}  // namespace fs

bool small_forward_supported(const SmallParams& p, int hidden, int ffn, int heads, int sms) {
  if (hidden != SMALL_HIDDEN || ffn != SMALL_FFN || heads != SMALL_HEADS || p.T < 1 || p.T > SMALL_MAX_TOKENS ||
      p.n_layers < 1 || p.n_layers > SMALL_MAX_LAYERS || sms < fs::HEADS || p.nseq < 1 || p.nseq > sms ||
      p.out_dim < 1 || p.out_dim > hidden)
    return false;
  for (int l = 0; l < p.n_layers; l++)
    for (int m = 0; m < 4; m++) {
      const SmallGemm& g = p.layers[l].g[m];
      if (!g.w || g.K % TILE_K || r16::n_slices(g.K) > (m == 3 ? fs::N_Y2 : 1) ||
          (g.qf != QF_Q8_0 && g.qf != QF_KMIN && g.qf != QF_Q6K))
        return false;
      const int want = m == 0 ? 3 * SMALL_HIDDEN / 16 : m == 2 ? SMALL_FFN / 8 : SMALL_HIDDEN / 16;
      if (g.tiles != want) return false;
    }
  return true;
}

size_t small_sync_bytes() { return (size_t)fs::N_CNT * fs::CNT_STRIDE * 4; }

cudaError_t launch_forward_small(const SmallParams& p, cudaStream_t s) {
  static std::mutex mu;
  static int grid[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  const bool two = p.T > 8;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (grid[dev] == 0) {
      cudaError_t e = cudaFuncSetAttribute(fs::forward_small_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           fs::Lay<1>::BYTES);
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(fs::forward_small_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 fs::Lay<2>::BYTES);
      if (e != cudaSuccess) return e;
      int sms = 0, per_sm1 = 0, per_sm2 = 0;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm1, fs::forward_small_kernel<1>, fs::NTHREADS,
                                                        fs::Lay<1>::BYTES);
      if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm2, fs::forward_small_kernel<2>, fs::NTHREADS,
                                                          fs::Lay<2>::BYTES);
      if (e != cudaSuccess) return e;
      if (per_sm1 < 1 || per_sm2 < 1) return cudaErrorNotSupported;
      grid[dev] = sms;  // one CTA per SM
    }
  }
  cudaError_t e = cudaMemsetAsync(p.sync, 0, small_sync_bytes(), s);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid[dev]);
  cfg.blockDim = dim3(fs::NTHREADS);
  cfg.dynamicSmemBytes = two ? fs::Lay<2>::BYTES : fs::Lay<1>::BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return two ? cudaLaunchKernelEx(&cfg, fs::forward_small_kernel<2>, p)
             : cudaLaunchKernelEx(&cfg, fs::forward_small_kernel<1>, p);
}

}  // namespace le
