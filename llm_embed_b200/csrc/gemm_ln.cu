// Projection GEMM with the residual add and LayerNorm fused into its
// epilogue, for the attention-output and FFN-down projections (768 output
// columns): h = LN(h + x . W^T) (bert.go:262-266, 276-280).  It writes the
// new residual stream h (float32, in place) and its fp16 copy, the next
// GEMM's operand, and replaces "GEMM -> y (float32) -> residual LayerNorm
// kernel", whose y written and read back is 40% of that pair's traffic.
//
// Persistent kernel on CTA pairs (tcgen05.mma cta_group::2, kind::f16,
// M=256, N=256, K=16), the same main loop as the large-batch GEMM
// (gemm_f16.cu): TMA A and B tiles in a 4-stage ring, fp32 accumulators
// double-buffered in TMEM.  A row of the output (768 columns) is split over
// three 256-column tiles computed by different pairs, so the row's
// LayerNorm statistics are exchanged through global memory:
//
//   pass 1   each epilogue warp owns 32 rows x one 128-column chunk of a
//            tile: x = h + acc, with h brought in by TMA (32 x 32 float
//            blocks, two in flight); x goes back into the accumulator
//            columns of TMEM; the chunk's sum and sum of squares per row are
//            formed exactly as ln_row_stats forms a chunk total;
//   exchange each lane stores its row's chunk totals as one 64-bit word
//            part[row][chunk] and polls (bounded) the row's six words until
//            none holds the empty marker; every warp adds the six totals in
//            column order, so all agree bit for bit with the row kernels.
//            The word is its own flag: no fence or counter.  part has two
//            halves used by alternate launches (a launch counter in ctl[1]);
//            each launch returns the other half to the marker, so a word is
//            never stale;
//   pass 2   y = (x - mean) inv w + b from TMEM, written as float32 h and
//            fp16 through a swizzled shared-memory transpose (whole
//            128-byte row segments per store instruction).
//
// A warp waits only for tiles of the same 256-row block, which the tile
// order places on neighbouring pairs in the same or the next round; the
// cooperative launch keeps every pair resident, so those tiles always make
// progress.  The last CTA to finish (ctl[0] counts them) advances the
// launch counter.  Every wait is bounded (WAIT_LIMIT_NS) and reports
// DE_TIMEOUT; after any device error the host returns part to the marker.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>

#include "gemm_epi_tc.cuh"
#include "kernels.h"
#include "ln_warp.cuh"

namespace le {
namespace tcl {

using namespace tcx;

constexpr int UM = 128;            // token rows per CTA
constexpr int PM = 2 * UM;         // token rows per pair tile
constexpr int UN = 128;            // output columns per CTA's B tile
constexpr int PN = 2 * UN;         // output columns per pair tile (MMA N)
constexpr int NT = 3;              // column tiles per row block
constexpr int HID = NT * PN;       // 768
constexpr int NCHUNK = HID / 128;  // 128-column chunks per row
constexpr int BK = 64;
constexpr int EPI_WARP0 = 2, EPI_WARPS = 8;
constexpr int NTHREADS = (EPI_WARP0 + EPI_WARPS) * 32;
constexpr int A_BYTES = UM * BK * 2;  // 16 KB
constexpr int B_BYTES = UN * BK * 2;  // 16 KB
constexpr int BLK = 4096;             // one 32-row x 128-byte block
constexpr int TMEM_COLS = 512;
constexpr uint32_t IDESC = idesc_f16(PM, PN);

// Shared memory: S operand stages, and per epilogue warp NHIN residual
// blocks (TMA loads, NHIN in flight) and NSTG store staging blocks (TMA
// stores, NSTG in flight).  Short K (the attention-output projection) is
// epilogue bound: more epilogue buffers; long K (FFN down) is bound by the
// operand feed: more stages.
template <int S_, int NHIN_, int NSTG_>
struct Lay {
  static constexpr int S = S_, NHIN = NHIN_, NSTG = NSTG_;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + S * A_BYTES;
  static constexpr int OFF_HIN = OFF_B + S * B_BYTES;
  static constexpr int OFF_STG = OFF_HIN + EPI_WARPS * NHIN * BLK;
  static constexpr int OFF_BAR = OFF_STG + EPI_WARPS * NSTG * BLK;
  // full[S], empty[S], tfull[2], tempty[2], hfull[EPI_WARPS][NHIN]
  static constexpr int NBAR = 2 * S + 4 + NHIN * EPI_WARPS;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int ALLOC = BYTES + 1024;
  static_assert(ALLOC <= 232448, "shared memory budget");
};
using LayShortK = Lay<3, 2, 2>;
using LayLongK = Lay<5, 1, 1>;
constexpr int SHORT_K_MAX = 1024;

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])),
      "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
      "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])),
      "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
      "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])),
      "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

constexpr unsigned long long PART_EMPTY = ~0ull;  // never a (sum, sum of squares >= 0) pair

__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Bounded wait for a TMA load before the CTA exits (no abort shortcut).
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try(bar, parity))
    if (globaltimer_ns() - t0 > 10000000ull) break;  // 10 ms
}

// One warp's 32 rows x 128 bytes (words[32] per lane = its row) to
// (col0, row0) of `map`: staged 128B-swizzled in the next of its NSTG
// buffers, then one TMA store (rows past the map's extent are clipped).  A
// buffer is rewritten only after the store that last read it has done so.
template <int NSTG>
__device__ __forceinline__ void emit(const CUtensorMap* map, uint32_t stage, int& buf, const uint32_t* words, int col0,
                                     int row0) {
  const int lane = threadIdx.x & 31;
  if (lane == 0) asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(NSTG - 1) : "memory");
  __syncwarp();
  const uint32_t base = stage + buf * BLK + lane * 128;
#pragma unroll
  for (int q = 0; q < 8; q++)
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(base + ((q ^ (lane & 7)) << 4)), "r"(words[4 * q]),
                 "r"(words[4 * q + 1]), "r"(words[4 * q + 2]), "r"(words[4 * q + 3])
                 : "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  if (lane == 0) tma_store_2d(map, stage + buf * BLK, col0, row0);
  buf = buf + 1 == NSTG ? 0 : buf + 1;
}

template <class L>
__global__ void __launch_bounds__(NTHREADS, 1)
    gemm_ln_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   const __grid_constant__ CUtensorMap tmap_h, const __grid_constant__ CUtensorMap tmap_o, int K, int M,
                   int m_tiles, float* __restrict__ h, const float* __restrict__ lw, const float* __restrict__ lb,
                   float eps, unsigned long long* __restrict__ part, int part_rows, unsigned* __restrict__ ctl,
                   DevStatus* status) {
  constexpr int S = L::S, NHIN = L::NHIN, NSTG = L::NSTG;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::OFF_BAR;
  auto full = [&](int s) { return bar0 + 8 * s; };
  auto empty = [&](int s) { return bar0 + 8 * (S + s); };
  auto tfull = [&](int a) { return bar0 + 8 * (2 * S + a); };
  auto tempty = [&](int a) { return bar0 + 8 * (2 * S + 2 + a); };
  auto hfull = [&](int e, int b) { return bar0 + 8 * (2 * S + 4 + NHIN * e + b); };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::OFF_MISC);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int ksteps = K / BK;
  const int total = m_tiles * NT;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < S; s++) {
      mbar_init(full(s), 1);   // even CTA: its producer's expect_tx; both CTAs' bytes
      mbar_init(empty(s), 1);  // MMA commit
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(tfull(a), 1);               // MMA commit
      mbar_init(tempty(a), 2 * EPI_WARPS);  // even CTA: epilogue warps of both CTAs
    }
    for (int e = 0; e < EPI_WARPS; e++)
      for (int b = 0; b < NHIN; b++) mbar_init(hfull(e, b), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // (a no-op: this cooperative launch waits for its predecessor)
  pdl_trigger();  // the next kernel may take the SMs this one leaves
  // This launch's half of part; the idle lanes of warps 0 and 1 return the
  // other half (the next launch's) to the marker.
  const unsigned epoch = *reinterpret_cast<volatile unsigned*>(ctl + 1);
  const long half_words = (long)part_rows * NCHUNK;
  unsigned long long* cur = part + (epoch & 1) * half_words;
  if (warp < 2 && lane > 0) {
    unsigned long long* other = part + ((epoch + 1) & 1) * half_words;
    for (long i = (long)blockIdx.x * 62 + warp * 31 + lane - 1; i < half_words; i += (long)gridDim.x * 62)
      other[i] = PART_EMPTY;
  }

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_b)) : "memory");
      uint32_t it = 0;
      bool ok = true;
      for (int tile = pair; tile < total && ok; tile += npairs) {
        const int mt = tile / NT, nt = tile % NT;
        for (int ks = 0; ks < ksteps; ks++, it++) {
          const int s = it % S;
          if (!mbar_wait(empty(s), ((it / S) & 1) ^ 1, abort_flag, status, 71)) {
            ok = false;
            break;
          }
          if (leader) mbar_expect_tx(full(s), 2 * (A_BYTES + B_BYTES));
          const uint32_t bar = map_to_rank(full(s), 0);
          tma_load_2d_pair(sbase + L::OFF_A + s * A_BYTES, &tmap_a, ks * BK, mt * PM + rank * UM, bar);
          tma_load_2d_pair(sbase + L::OFF_B + s * B_BYTES, &tmap_b, ks * BK, nt * PN + rank * UN, bar);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA (even CTA)
    if (leader && lane == 0) {
      uint32_t it = 0;
      int tcount = 0;
      for (int tile = pair; tile < total && !*abort_flag; tile += npairs, tcount++) {
        const int acc = tcount & 1;
        if (!mbar_wait(tempty(acc), ((tcount >> 1) & 1) ^ 1, abort_flag, status, 72)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * PN;
        bool ok = true;
        for (int ks = 0; ks < ksteps; ks++, it++) {
          const int s = it % S;
          if (!mbar_wait(full(s), (it / S) & 1, abort_flag, status, 73)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = sbase + L::OFF_A + s * A_BYTES;
          const uint32_t b_addr = sbase + L::OFF_B + s * B_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; kk++)
            mma_f16_pair(d, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), IDESC, (ks | kk) != 0);
          mma_commit_pair(empty(s), 0x3);
        }
        if (!ok) break;
        mma_commit_pair(tfull(acc), 0x3);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int e = warp - EPI_WARP0;
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. of this warp
    const int half = e >> 2;       // 128-column half of the 256-column tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t hin = sbase + L::OFF_HIN + e * NHIN * BLK;
    const uint32_t stage = sbase + L::OFF_STG + e * NSTG * BLK;
    const uint32_t tempty_leader0 = map_to_rank(tempty(0), 0);
    // Residual block q of this warp is block q % 4 of its (q / 4)-th tile,
    // loaded into buffer q % NHIN; hk blocks issued, hc consumed.
    int hk = 0, hc = 0;
    int obuf = 0;
    int tcount = 0;
    bool ok = true;
    // Rows and columns of this warp's part of a tile.
    auto row_of = [&](int tile) { return (tile / NT) * PM + rank * UM + quarter * 32; };
    auto col_of = [&](int tile) { return ((tile % NT) * 2 + half) * 128; };
    auto issue = [&](int q) {  // warp-uniform call; lane 0 issues
      const int tile = pair + (q >> 2) * npairs;
      if (tile >= total) return;
      if (lane == 0) {
        const int b = q % NHIN;
        mbar_expect_tx(hfull(e, b), BLK);  // the warp's reads of buffer b are complete
        tma_load_2d(hin + b * BLK, &tmap_h, col_of(tile) + (q & 3) * 32, row_of(tile), hfull(e, b));
      }
      hk = q + 1;
    };
#pragma unroll
    for (int q = 0; q < NHIN; q++) issue(q);
    for (int tile = pair; tile < total && ok; tile += npairs, tcount++) {
      const int acc = tcount & 1;
      const int row0 = row_of(tile), col = col_of(tile);
      const int chunk = col / 128;
      const uint32_t tacc = tmem + lane_off + acc * PN + half * 128;
      // LayerNorm weight and bias of columns col + 4 lane .. +3 (pass 2
      // takes each group of four from its lane by shuffle).
      const float4 wl = __ldg(reinterpret_cast<const float4*>(lw + col) + lane);
      const float4 bl = __ldg(reinterpret_cast<const float4*>(lb + col) + lane);
      ok = __all_sync(0xffffffffu, mbar_wait(tfull(acc), (tcount >> 1) & 1, abort_flag, status, 74));
      if (!ok) break;
      tc_fence_after();
      // Pass 1.  Chunk column 4l + i belongs to lane l of ln_row_stats;
      // q*[l] are those lanes' values.
      float qs[32], qss[32];
#pragma unroll
      for (int blk = 0; blk < 4; blk++) {
        const int q = tcount * 4 + blk;
        const int b = q % NHIN;
        ok = __all_sync(0xffffffffu, mbar_wait(hfull(e, b), (q / NHIN) & 1, abort_flag, status, 75));
        if (!ok) break;
        hc = q + 1;
        float v[32];
        tmem_ld32(tacc + blk * 32, v);
        const uint8_t* hrow = smem + L::OFF_HIN + (e * NHIN + b) * BLK + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const float4 r = *reinterpret_cast<const float4*>(hrow + ((j ^ (lane & 7)) << 4));
          v[4 * j] = __fadd_rn(r.x, v[4 * j]);
          v[4 * j + 1] = __fadd_rn(r.y, v[4 * j + 1]);
          v[4 * j + 2] = __fadd_rn(r.z, v[4 * j + 2]);
          v[4 * j + 3] = __fadd_rn(r.w, v[4 * j + 3]);
          const int l = blk * 8 + j;
          qs[l] = 0.f;
          qss[l] = 0.f;
          ln_accum(make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]), qs[l], qss[l]);
        }
        tmem_st32(tacc + blk * 32, v);
        __syncwarp();
        // Refill the buffer NHIN blocks ahead (into the next tile's first
        // blocks, which then load during the rest of this tile).
        issue(q + NHIN);
      }
      if (!ok) break;
      // The butterfly of ln_row_stats, unrolled in one thread.
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int l = 0; l < o; l++) {
          qs[l] = __fadd_rn(qs[l], qs[l + o]);
          qss[l] = __fadd_rn(qss[l], qss[l + o]);
        }
      // Exchange the chunk totals: this lane's row, all six chunks.
      const long row = row0 + lane;
      st_relaxed_u64(cur + row * NCHUNK + chunk,
                     (unsigned long long)__float_as_uint(qs[0]) | ((unsigned long long)__float_as_uint(qss[0]) << 32));
      unsigned long long pw[NCHUNK];
      {
        const uint64_t t0 = globaltimer_ns();
        for (uint32_t i = 0;; i++) {
          bool have = true;
#pragma unroll
          for (int g = 0; g < NCHUNK; g++) {
            pw[g] = ld_relaxed_u64(cur + row * NCHUNK + g);
            have = have && pw[g] != PART_EMPTY;
          }
          if (__all_sync(0xffffffffu, have)) break;
          if ((i & 15) == 15) {
            if (*abort_flag) {
              ok = false;
              break;
            }
            if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) {
              if (lane == 0) {
                *abort_flag = 1;
                report(status, DE_TIMEOUT, 76, (int)blockIdx.x);
              }
              ok = false;
              break;
            }
          }
        }
      }
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      float ts = 0.f, tss = 0.f;
#pragma unroll
      for (int g = 0; g < NCHUNK; g++) {
        ts = __fadd_rn(ts, __uint_as_float((unsigned)pw[g]));
        tss = __fadd_rn(tss, __uint_as_float((unsigned)(pw[g] >> 32)));
      }
      float mean, inv;
      ln_stats(ts, tss, HID, eps, &mean, &inv);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      // Pass 2: 64 columns at a time -> two float32 blocks, one fp16 block.
      // A block wholly past the last token is not stored.
#pragma unroll 1
      for (int c = 0; c < 128 && row0 < M; c += 64) {
        float a[32], b[32];
        tmem_ld32(tacc + c, a);
        tmem_ld32(tacc + c + 32, b);
        uint32_t w16[32];
#pragma unroll
        for (int j = 0; j < 16; j++) {
          float* src = j < 8 ? a + 4 * j : b + 4 * (j - 8);
          const int from = c / 4 + j;  // the lane holding columns col + c + 4j ..
          const float4 w = make_float4(__shfl_sync(0xffffffffu, wl.x, from), __shfl_sync(0xffffffffu, wl.y, from),
                                       __shfl_sync(0xffffffffu, wl.z, from), __shfl_sync(0xffffffffu, wl.w, from));
          const float4 bb = make_float4(__shfl_sync(0xffffffffu, bl.x, from), __shfl_sync(0xffffffffu, bl.y, from),
                                        __shfl_sync(0xffffffffu, bl.z, from), __shfl_sync(0xffffffffu, bl.w, from));
          const float4 y = ln_apply(make_float4(src[0], src[1], src[2], src[3]), mean, inv, w, bb);
          src[0] = y.x;
          src[1] = y.y;
          src[2] = y.z;
          src[3] = y.w;
          w16[2 * j] = pack_half2(y.x, y.y);
          w16[2 * j + 1] = pack_half2(y.z, y.w);
        }
        emit<NSTG>(&tmap_h, stage, obuf, reinterpret_cast<const uint32_t*>(a), col + c, row0);
        emit<NSTG>(&tmap_h, stage, obuf, reinterpret_cast<const uint32_t*>(b), col + c + 32, row0);
        emit<NSTG>(&tmap_o, stage, obuf, w16, col + c, row0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader0 + 8 * acc);
    }
    // Loads still in flight land before the CTA exits; stores have read
    // their staging buffers.
    for (; hc < hk; hc++) drain_wait(hfull(e, hc % NHIN), (hc / NHIN) & 1);
    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer is done with this CTA's shared memory and TMEM
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
  // The last CTA to finish advances the launch counter (every CTA has read
  // it at its start).
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(ctl, 1u) == gridDim.x - 1) {
      ctl[0] = 0;
      ctl[1] = epoch + 1;
    }
  }
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D row-major map: rows x cols of `type`, row pitch ld elements, boxes of
// box_rows x 128 bytes, 128B swizzle.
static bool encode_2d(PFN_cuTensorMapEncodeTiled_v12000 enc, CUtensorMap* map, CUtensorMapDataType type, int esize,
                      const void* p, long rows, long cols, long ld, int box_rows) {
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(ld * esize)};
  const cuuint32_t box[2] = {(cuuint32_t)(128 / esize), (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, type, 2, const_cast<void*>(p), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


}  // namespace tcl

bool gemm_ln_supported(int N, int K) { return N == tcl::HID && K % tcl::BK == 0 && K > 0; }

int gemm_ln_part_rows(int M) { return (M + tcl::PM - 1) / tcl::PM * tcl::PM; }
size_t gemm_ln_part_bytes(int M) { return (size_t)2 * gemm_ln_part_rows(M) * tcl::NCHUNK * 8; }

namespace tcl {

// Per device and layout: the shared-memory attribute and the number of CTA
// pairs that can be resident at once (the cooperative grid's size).
template <class L>
static cudaError_t launch_layout(const CUtensorMap& amap, const CUtensorMap& bmap, const CUtensorMap& hmap,
                                 const CUtensorMap& omap, int K, int M, float* h, const float* ln_w, const float* ln_b,
                                 float eps, unsigned long long* part, int part_rows, unsigned* ctl, DevStatus* status,
                                 cudaStream_t s) {
  static std::mutex mu;
  static int max_pairs[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  int npairs;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (max_pairs[dev] == 0) {
      cudaError_t e = cudaFuncSetAttribute(gemm_ln_kernel<L>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC);
      if (e != cudaSuccess) return e;
      int sms = 0;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(sms & ~1);
      cfg.blockDim = dim3(NTHREADS);
      cfg.dynamicSmemBytes = L::ALLOC;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      e = cudaOccupancyMaxActiveClusters(&n, gemm_ln_kernel<L>, &cfg);
      if (e != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return e != cudaSuccess ? e : cudaErrorNotSupported;
      }
      max_pairs[dev] = n;
    }
    npairs = max_pairs[dev];
  }
  const int m_tiles = (M + PM - 1) / PM;
  const int total = m_tiles * NT;
  const int pairs = total < npairs ? total : npairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(NTHREADS);
  cfg.dynamicSmemBytes = L::ALLOC;
  cfg.stream = s;
  cfg.attrs = attr;
#ifdef LE_LN_NONCOOPERATIVE
  // Profiling builds only (nvcc -DLE_LN_NONCOOPERATIVE): Nsight Compute
  // cannot replay cooperative cluster launches, so this build launches
  // without the cooperative attribute.  The grid still fits an otherwise
  // idle GPU, but co-residency of the CTAs (which wait on each other's
  // statistics) is then not guaranteed; release builds never take it.
  cfg.numAttrs = 1;
#else
  cfg.numAttrs = 2;
#endif
  return cudaLaunchKernelEx(&cfg, gemm_ln_kernel<L>, amap, bmap, hmap, omap, K, M, m_tiles, h, ln_w, ln_b, eps, part,
                            part_rows, ctl, status);
}

}  // namespace tcl

cudaError_t launch_gemm_ln(const __half* W16, int K, const __half* A, long lda, int M, float* h, __half* out16,
                           const float* ln_w, const float* ln_b, float eps, unsigned long long* part, int part_rows,
                           unsigned* ctl, DevStatus* status, cudaStream_t s) {
  using namespace tcl;
  if (M <= 0) return cudaSuccess;
  auto enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  const auto misaligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; };
  if (!gemm_ln_supported(HID, K) || (lda * 2) % 16 || misaligned(A) || misaligned(W16) || misaligned(h) ||
      misaligned(out16) || misaligned(ln_w) || misaligned(ln_b) || misaligned(part) || !ctl ||
      part_rows < gemm_ln_part_rows(M))
    return cudaErrorInvalidValue;
  CUtensorMap amap, bmap, hmap, omap;
  if (!encode_2d(enc, &amap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, A, M, K, lda, UM) ||
      !encode_2d(enc, &bmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, W16, HID, K, K, UN) ||
      !encode_2d(enc, &hmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, h, M, HID, HID, 32) ||
      !encode_2d(enc, &omap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, out16, M, HID, HID, 32))
    return cudaErrorInvalidValue;
  if (K <= SHORT_K_MAX)
    return launch_layout<LayShortK>(amap, bmap, hmap, omap, K, M, h, ln_w, ln_b, eps, part, part_rows, ctl, status, s);
  return launch_layout<LayLongK>(amap, bmap, hmap, omap, K, M, h, ln_w, ln_b, eps, part, part_rows, ctl, status, s);
}


}  // namespace le
