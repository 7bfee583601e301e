// Quantised GEMM on CTA pairs (tcgen05 cta_group::2, sm_100a).
//
// out = A . W^T with A fp16 [M][K] (tokens) and W the tile-blocked quantised
// weight (common.cuh).  Persistent kernel launched as clusters of two CTAs on
// two SMs.  A pair computes 256-token x 256-weight-row output tiles with one
// tcgen05.mma (kind::f16, M=256, N=256, K=16) per 16-column K sub-step,
// issued by the even CTA: each CTA supplies 128 token rows of A and 128
// weight rows of B from its own shared memory and receives its 128 x 256
// accumulator in its own TMEM.  So every dequantised weight feeds 256 tokens
// and each SM dequantises only the 128 weight rows it owns.
//
//   warp 0     A producer: TMA 2-D load of this CTA's A tile (128 x 64
//              fp16, 128B swizzle; completes on the even CTA's barrier).
//   warp 2     raw producer: 1-D bulk copy of this CTA's raw quant chunk
//              (128 x 64 bytes + scales).  Raw stages are freed as soon as
//              they are dequantised, A stages when the MMA has read them,
//              so each pipeline runs at its own depth.
//   warp 1     TMEM allocation (512 columns: two 128x256 fp32 accumulators);
//              in the even CTA one lane issues the MMAs and the commits,
//              which arrive on the barriers of both CTAs.
//   dequant    raw chunk -> fp16 B operand (exact reference value rounded to
//              fp16, dequant.cuh) in the 128B-swizzled K-major layout, each
//              warp for its own rows; the odd CTA's warps arrive on the even
//              CTA's barrier.
//   epilogue   tcgen05.ld of the local accumulator, fused epilogue math
//              (epilogue.cuh), TMA stores of 32-row x 128-byte blocks from
//              swizzled staging buffers; frees the accumulator on the even
//              CTA's barrier.
//
// Every mbarrier wait is bounded (WAIT_LIMIT_NS); on expiry the kernel
// records DE_TIMEOUT and all roles leave their loops.  A cluster barrier
// before the first remote access and before exit keeps both CTAs' shared
// memory valid while the other may touch it.
#include <cudaTypedefs.h>

#include <mutex>

#include "gemm_epi_tc.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace le {
namespace tc2 {

using namespace tcx;

#ifndef LE_TC2_S_A
#define LE_TC2_S_A 6
#endif
#ifndef LE_TC2_S_R
#define LE_TC2_S_R 4
#endif
#ifndef LE_TC2_S_B
#define LE_TC2_S_B 3
#endif
#ifndef LE_TC2_DQ_WARPS
#define LE_TC2_DQ_WARPS 8
#endif
#ifndef LE_TC2_EPI_WARPS
#define LE_TC2_EPI_WARPS 4
#endif

constexpr int UM = 128;       // token rows per CTA
constexpr int PM = 2 * UM;    // token rows per pair tile
constexpr int PN = 2 * TILE_N;  // weight rows per pair tile (MMA N)
constexpr int BK = TILE_K;
constexpr int S_A = LE_TC2_S_A;  // A stages (freed by the MMA)
constexpr int S_R = LE_TC2_S_R;  // raw quant stages (freed by the dequant group)
constexpr int S_B = LE_TC2_S_B;  // fp16 B stages (freed by the MMA)
constexpr int DQ_WARPS = LE_TC2_DQ_WARPS;
constexpr int DQ_THREADS = DQ_WARPS * 32;
constexpr int DQ_WARP0 = 3;
constexpr int EPI_WARP0 = DQ_WARP0 + DQ_WARPS;
constexpr int EPI_WARPS = LE_TC2_EPI_WARPS;  // 4: all 256 columns each; 8: 128 columns each
static_assert(EPI_WARPS == 4 || EPI_WARPS == 8, "epilogue warps");
constexpr int NTHREADS = (EPI_WARP0 + EPI_WARPS) * 32;
constexpr int A_BYTES = UM * BK * 2;        // 16384
constexpr int B16_BYTES = TILE_N * BK * 2;  // 16384
constexpr int TMEM_COLS = 512;
constexpr uint32_t IDESC = idesc_f16(PM, PN);

template <int QF>
struct Layout {
  static constexpr int RAW = chunk_bytes(QF);
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B16 = OFF_A + S_A * A_BYTES;
  static constexpr int OFF_RAW = OFF_B16 + S_B * B16_BYTES;
  // Epilogue staging: per epilogue warp two 32-row x 128-byte buffers in the
  // 128B-swizzled layout of the output tensor map (TMA stores read them).
  static constexpr int OFF_STAGE = ((OFF_RAW + S_R * RAW + 1023) / 1024) * 1024;
  static constexpr int OFF_BAR = OFF_STAGE + EPI_WARPS * 2 * 4096;
  // full_a empty_a [S_A], full_raw empty_raw [S_R], full_b empty_b [S_B], tfull tempty [2]
  static constexpr int NBAR = 2 * S_A + 2 * S_R + 2 * S_B + 4;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int ALLOC = BYTES + 1024;
  static_assert(ALLOC <= 232448, "shared memory budget of one CTA exceeded");
};

template <int QF>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NTHREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_out,
                     const uint8_t* __restrict__ W, int K, int m_tiles, int n_tiles, EpiParams ep, DevStatus* status) {
  using Lay = Layout<QF>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + Lay::OFF_BAR;
  auto full_a = [&](int s) { return bar0 + 8 * s; };
  auto empty_a = [&](int s) { return bar0 + 8 * (S_A + s); };
  auto full_raw = [&](int r) { return bar0 + 8 * (2 * S_A + r); };
  auto empty_raw = [&](int r) { return bar0 + 8 * (2 * S_A + S_R + r); };
  auto full_b = [&](int j) { return bar0 + 8 * (2 * S_A + 2 * S_R + j); };
  auto empty_b = [&](int j) { return bar0 + 8 * (2 * S_A + 2 * S_R + S_B + j); };
  auto tfull = [&](int a) { return bar0 + 8 * (2 * S_A + 2 * S_R + 2 * S_B + a); };
  auto tempty = [&](int a) { return bar0 + 8 * (2 * S_A + 2 * S_R + 2 * S_B + 2 + a); };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Lay::OFF_MISC);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Lay::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int ksteps = K / BK;
  const int total = m_tiles * n_tiles;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < S_A; s++) {
      mbar_init(full_a(s), 1);   // even CTA: its producer's expect_tx; both CTAs' A bytes
      mbar_init(empty_a(s), 1);  // MMA commit
    }
    for (int r = 0; r < S_R; r++) {
      mbar_init(full_raw(r), 1);          // local producer's expect_tx; local raw bytes
      mbar_init(empty_raw(r), DQ_WARPS);  // every local dequant warp
    }
    for (int j = 0; j < S_B; j++) {
      mbar_init(full_b(j), 2 * DQ_WARPS);  // even CTA: the dequant warps of both CTAs
      mbar_init(empty_b(j), 1);            // MMA commit
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(tfull(a), 1);                 // MMA commit
      mbar_init(tempty(a), 2 * EPI_WARPS);    // even CTA: epilogue warps of both CTAs
    }
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

  if (warp == 0) {
    // ------------------------------------------------------------ A producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
      uint32_t it = 0;
      bool ok = true;
      for (int tile = cluster; tile < total && ok; tile += nclusters) {
        const int mt = tile / n_tiles;
        for (int ks = 0; ks < ksteps; ks++, it++) {
          const int s = it % S_A;
          if (!mbar_wait(empty_a(s), ((it / S_A) & 1) ^ 1, abort_flag, status, 11)) {
            ok = false;
            break;
          }
          if (leader) mbar_expect_tx(full_a(s), 2 * A_BYTES);
          tma_load_2d_pair(sbase + Lay::OFF_A + s * A_BYTES, &tmap_a, ks * BK, mt * PM + rank * UM,
                           map_to_rank(full_a(s), 0));
        }
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ raw producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int tile = cluster; tile < total && ok; tile += nclusters) {
        const int nt = tile % n_tiles;
        const uint8_t* wt = W + (long)(2 * nt + rank) * ksteps * Lay::RAW;
        for (int ks = 0; ks < ksteps; ks++, it++) {
          const int r = it % S_R;
          if (!mbar_wait(empty_raw(r), ((it / S_R) & 1) ^ 1, abort_flag, status, 19)) {
            ok = false;
            break;
          }
          mbar_expect_tx(full_raw(r), Lay::RAW);
          bulk_load(sbase + Lay::OFF_RAW + r * Lay::RAW, wt + (long)ks * Lay::RAW, Lay::RAW, full_raw(r));
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA (even CTA)
    if (leader && lane == 0) {
      uint32_t it = 0, jt = 0;
      int tcount = 0;
      for (int tile = cluster; tile < total && !*abort_flag; tile += nclusters, tcount++) {
        const int acc = tcount & 1;
        if (!mbar_wait(tempty(acc), ((tcount >> 1) & 1) ^ 1, abort_flag, status, 12)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * PN;
        bool ok = true;
        for (int ks = 0; ks < ksteps; ks++, it++, jt++) {
          const int s = it % S_A, j = jt % S_B;
          if (!mbar_wait(full_a(s), (it / S_A) & 1, abort_flag, status, 13) ||
              !mbar_wait(full_b(j), (jt / S_B) & 1, abort_flag, status, 14)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = sbase + Lay::OFF_A + s * A_BYTES;
          const uint32_t b_addr = sbase + Lay::OFF_B16 + j * B16_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; kk++)
            mma_f16_pair(d, sw128_desc(a_addr + kk * 32), sw128_desc(b_addr + kk * 32), IDESC, (ks | kk) != 0);
          mma_commit_pair(empty_a(s), 0x3);
          mma_commit_pair(empty_b(j), 0x3);
        }
        if (!ok) break;
        mma_commit_pair(tfull(acc), 0x3);
      }
    }
  } else if (warp >= DQ_WARP0 && warp < EPI_WARP0) {
    // ------------------------------------------------------------ dequant
    // Each warp owns TILE_N / DQ_WARPS weight rows of the stage and signals
    // completion itself: no barrier across the dequant warps.
    constexpr int ROWS_PER_WARP = TILE_N / DQ_WARPS;
    const int dw = warp - DQ_WARP0;
    const int c16 = lane & 3;
    const uint32_t full_b_leader0 = map_to_rank(full_b(0), 0);
    uint32_t it = 0, jt = 0;
    bool ok = true;
    for (int tile = cluster; tile < total && ok; tile += nclusters) {
      for (int ks = 0; ks < ksteps; ks++, it++, jt++) {
        const int s = it % S_R, j = jt % S_B;
        const bool w = mbar_wait(full_raw(s), (it / S_R) & 1, abort_flag, status, 15) &&
                       mbar_wait(empty_b(j), ((jt / S_B) & 1) ^ 1, abort_flag, status, 16);
        if (!__all_sync(0xffffffffu, w)) {
          ok = false;
          break;
        }
        const uint8_t* raw = smem + Lay::OFF_RAW + s * Lay::RAW;
        uint8_t* b16 = smem + Lay::OFF_B16 + j * B16_BYTES;
#pragma unroll
        for (int q = 0; q < ROWS_PER_WARP / 8; q++) {
          const int n = dw * ROWS_PER_WARP + 8 * q + (lane >> 2);
          const uint4 u = *reinterpret_cast<const uint4*>(raw + n * BK + c16 * 16);
          const int g0 = 2 * c16, sw = n & 7;
          *reinterpret_cast<uint4*>(b16 + n * 128 + ((g0 ^ sw) << 4)) =
              dq8_f16<QF>(make_uint2(u.x, u.y), raw + TILE_Q_BYTES, n, g0);
          *reinterpret_cast<uint4*>(b16 + n * 128 + (((g0 + 1) ^ sw) << 4)) =
              dq8_f16<QF>(make_uint2(u.z, u.w), raw + TILE_Q_BYTES, n, g0 + 1);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(empty_raw(s));
          if (leader) mbar_arrive(full_b(j));
          else mbar_arrive_cluster(full_b_leader0 + 8 * j);
        }
      }
    }
  } else if (warp >= EPI_WARP0) {
    // ------------------------------------------------------------ epilogue
    // Accumulator rows -> registers (tcgen05.ld, one row per lane), fused
    // epilogue math, then 128-byte row blocks through a swizzled staging
    // buffer and a TMA store of the warp's 32 x 128-byte block.
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    const int ew = warp - EPI_WARP0;
    const int c_begin = EPI_WARPS == 8 ? (ew >> 2) * TILE_N : 0;
    const int c_end = EPI_WARPS == 8 ? c_begin + TILE_N : PN;
    const uint32_t stage = sbase + Lay::OFF_STAGE + ew * 2 * 4096;
    int buf = 0;
    const uint32_t tempty_leader0 = map_to_rank(tempty(0), 0);
    int tcount = 0;
    for (int tile = cluster; tile < total; tile += nclusters, tcount++) {
      const int acc = tcount & 1;
      const bool w = mbar_wait(tfull(acc), (tcount >> 1) & 1, abort_flag, status, 17);
      if (!__all_sync(0xffffffffu, w)) break;  // warp-uniform: tcgen05.ld is .sync.aligned
      tc_fence_after();
      const int mt = tile / n_tiles, nt = tile % n_tiles;
      const int row0 = mt * PM + rank * UM + quarter * 32;
      const uint32_t tbase = tmem + acc * PN + ((uint32_t)(quarter * 32) << 16);
      if (row0 < ep.M)  // warp-uniform
        epilogue_tile(ep, &tmap_out, tbase, row0, nt * PN, c_begin, c_end, stage, buf);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader0 + 8 * acc);
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // all stores done
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer is done with this CTA's shared memory and TMEM
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

// ---------------------------------------------------------------- host ----

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

template <int QF>
cudaError_t launch(const uint8_t* W, int n_virtual, int K, const __half* A, long lda, const EpiParams& ep,
                   DevStatus* status, cudaStream_t s) {
  auto enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  if (K % BK || (lda * 2) % 16 || (reinterpret_cast<uintptr_t>(A) & 15) || n_virtual % PN)
    return cudaErrorInvalidValue;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)ep.M};
  const cuuint64_t strides[1] = {(cuuint64_t)lda * 2};
  const cuuint32_t box[2] = {BK, UM};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(A), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  // Output map: 32-row x 128-byte boxes (32 float32 or 64 fp16 columns),
  // 128B swizzle as the epilogue stages them.
  CUtensorMap omap;
  {
    const bool f32 = ep.mode == EPI_F32;
    void* out = f32 ? static_cast<void*>(ep.out32) : static_cast<void*>(ep.out16);
    const int esz = f32 ? 4 : 2;
    if ((ep.ldo * esz) % 16 || (reinterpret_cast<uintptr_t>(out) & 15)) return cudaErrorInvalidValue;
    const cuuint64_t odims[2] = {(cuuint64_t)ep.N, (cuuint64_t)ep.M};
    const cuuint64_t ostrides[1] = {(cuuint64_t)ep.ldo * esz};
    const cuuint32_t obox[2] = {(cuuint32_t)(128 / esz), 32};
    if (enc(&omap, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, out, odims, ostrides,
            obox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  // Per device: the shared-memory attribute and the number of CTA pairs
  // that can be resident at once (the persistent grid's size).
  static std::mutex mu;
  static int max_pairs[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (max_pairs[dev] == 0) {
      cudaError_t e = cudaFuncSetAttribute(gemm_pair_kernel<QF>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           Layout<QF>::ALLOC);
      if (e != cudaSuccess) return e;
      int sms = 0;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(sms & ~1);
      cfg.blockDim = dim3(NTHREADS);
      cfg.dynamicSmemBytes = Layout<QF>::ALLOC;
      int n = 0;
      e = cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<QF>, &cfg);
      if (e != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = sms / 2;
      }
      max_pairs[dev] = n;
    }
  }
  const int m_tiles = (ep.M + PM - 1) / PM;
  const int n_tiles = n_virtual / PN;
  const int total = m_tiles * n_tiles;
  const int pairs = total < max_pairs[dev] ? total : max_pairs[dev];
  gemm_pair_kernel<QF><<<2 * pairs, NTHREADS, Layout<QF>::ALLOC, s>>>(map, omap, W, K, m_tiles, n_tiles, ep, status);
  return cudaGetLastError();
}

}  // namespace tc2


cudaError_t launch_gemm_tc2(int qf, const uint8_t* W, int n_virtual, int K, const __half* A, long lda,
                            const EpiParams& ep, DevStatus* status, cudaStream_t s) {
  if (ep.M == 0) return cudaSuccess;
  switch (qf) {
    case QF_Q8_0: return tc2::launch<QF_Q8_0>(W, n_virtual, K, A, lda, ep, status, s);
    case QF_KMIN: return tc2::launch<QF_KMIN>(W, n_virtual, K, A, lda, ep, status, s);
    case QF_Q6K: return tc2::launch<QF_Q6K>(W, n_virtual, K, A, lda, ep, status, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace le
