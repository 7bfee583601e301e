// Large-batch GEMM on CTA pairs with load-time fp16 weights (tcgen05
// cta_group::2, sm_100a).
//
// out = A . W16^T with A fp16 [M][K] (tokens) and W16 fp16 [n_virtual][K],
// the weight's tensor-core operand values expanded once at load from the
// tile-blocked quantised copy (the same round-to-nearest fp16 of the exact
// dequantised value that the in-shared-memory dequant of gemm_tc2.cu
// produces, so both kernels compute identical products in the same order).
// Above a few hundred tokens the GEMM is compute bound and dequantising each
// weight tile once per 256-token tile costs issue slots and shared-memory
// bandwidth the tensor pipe needs; below it the quantised kernels, which
// read fewer weight bytes, run instead (gemm.cu).
//
// Persistent kernel on clusters of two CTAs; a pair computes 256-token x
// 256-weight-row tiles with tcgen05.mma (kind::f16, M=256, N=256, K=16)
// issued by the even CTA, each CTA holding 128 token rows of A and 128
// weight rows of B and receiving its 128 x 256 fp32 accumulator in TMEM.
//
//   warp 0     producer: TMA 2-D loads of this CTA's A tile and B tile
//              (128 x 64 fp16 each, 128B swizzle) into one stage; both
//              CTAs' loads complete on the even CTA's stage barrier.
//   warp 1     TMEM allocation (512 columns: two 128x256 accumulators);
//              in the even CTA one lane issues the MMAs and commits, which
//              arrive on the barriers of both CTAs.
//   epilogue   EPI_WARPS warps: tcgen05.ld, fused epilogue, TMA stores
//              (gemm_epi_tc.cuh); they free the accumulator on the even
//              CTA's barrier.
//
// Every mbarrier wait is bounded (WAIT_LIMIT_NS); on expiry the kernel
// records DE_TIMEOUT and all roles leave their loops.
#include <cudaTypedefs.h>

#include <mutex>

#include "gemm_epi_tc.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace le {
namespace tcf {

using namespace tcx;

#ifndef LE_TCF_STAGES
#define LE_TCF_STAGES 5
#endif
#ifndef LE_TCF_EPI_WARPS
#define LE_TCF_EPI_WARPS 8
#endif

constexpr int UM = 128;         // token rows per CTA
constexpr int PM = 2 * UM;      // token rows per pair tile
constexpr int UN = TILE_N;      // weight rows per CTA
constexpr int PN = 2 * UN;      // weight rows per pair tile (MMA N)
constexpr int BK = 64;
constexpr int S = LE_TCF_STAGES;
constexpr int EPI_WARPS = LE_TCF_EPI_WARPS;  // 4: all 256 columns each; 8: 128 columns each
static_assert(EPI_WARPS == 4 || EPI_WARPS == 8, "epilogue warps");
constexpr int EPI_WARP0 = 2;
constexpr int NTHREADS = (EPI_WARP0 + EPI_WARPS) * 32;
constexpr int A_BYTES = UM * BK * 2;  // 16384
constexpr int B_BYTES = UN * BK * 2;  // 16384
constexpr int TMEM_COLS = 512;
constexpr uint32_t IDESC = idesc_f16(PM, PN);

struct Lay {
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + S * A_BYTES;
  static constexpr int OFF_STAGE = OFF_B + S * B_BYTES;  // 1024-aligned (16 KB multiples)
  static constexpr int OFF_BAR = OFF_STAGE + EPI_WARPS * 2 * 4096;
  // full empty [S], tfull tempty [2]
  static constexpr int NBAR = 2 * S + 4;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int ALLOC = BYTES + 1024;
  static_assert(ALLOC <= 232448, "shared memory budget of one CTA exceeded");
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NTHREADS, 1)
    gemm_f16_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                         const __grid_constant__ CUtensorMap tmap_out, int K, int m_tiles, int n_tiles, EpiParams ep,
                         DevStatus* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + Lay::OFF_BAR;
  auto full = [&](int s) { return bar0 + 8 * s; };
  auto empty = [&](int s) { return bar0 + 8 * (S + s); };
  auto tfull = [&](int a) { return bar0 + 8 * (2 * S + a); };
  auto tempty = [&](int a) { return bar0 + 8 * (2 * S + 2 + a); };
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
    for (int s = 0; s < S; s++) {
      mbar_init(full(s), 1);   // even CTA: its producer's expect_tx; both CTAs' A and B bytes
      mbar_init(empty(s), 1);  // MMA commit
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(tfull(a), 1);               // MMA commit
      mbar_init(tempty(a), 2 * EPI_WARPS);  // even CTA: epilogue warps of both CTAs
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
  pdl_wait();  // the operands and the output buffer are the previous kernels'
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_b)) : "memory");
      uint32_t it = 0;
      bool ok = true;
      for (int tile = cluster; tile < total && ok; tile += nclusters) {
        const int mt = tile / n_tiles, nt = tile % n_tiles;
        for (int ks = 0; ks < ksteps; ks++, it++) {
          const int s = it % S;
          if (!mbar_wait(empty(s), ((it / S) & 1) ^ 1, abort_flag, status, 21)) {
            ok = false;
            break;
          }
          if (leader) mbar_expect_tx(full(s), 2 * (A_BYTES + B_BYTES));
          const uint32_t bar = map_to_rank(full(s), 0);
          tma_load_2d_pair(sbase + Lay::OFF_A + s * A_BYTES, &tmap_a, ks * BK, mt * PM + rank * UM, bar);
          tma_load_2d_pair(sbase + Lay::OFF_B + s * B_BYTES, &tmap_b, ks * BK, nt * PN + rank * UN, bar);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA (even CTA)
    if (leader && lane == 0) {
      uint32_t it = 0;
      int tcount = 0;
      for (int tile = cluster; tile < total && !*abort_flag; tile += nclusters, tcount++) {
        const int acc = tcount & 1;
        if (!mbar_wait(tempty(acc), ((tcount >> 1) & 1) ^ 1, abort_flag, status, 22)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * PN;
        bool ok = true;
        for (int ks = 0; ks < ksteps; ks++, it++) {
          const int s = it % S;
          if (!mbar_wait(full(s), (it / S) & 1, abort_flag, status, 23)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = sbase + Lay::OFF_A + s * A_BYTES;
          const uint32_t b_addr = sbase + Lay::OFF_B + s * B_BYTES;
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
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    const int ew = warp - EPI_WARP0;
    const int c_begin = EPI_WARPS == 8 ? (ew >> 2) * UN : 0;
    const int c_end = EPI_WARPS == 8 ? c_begin + UN : PN;
    const uint32_t stage = sbase + Lay::OFF_STAGE + ew * 2 * 4096;
    int buf = 0;
    const uint32_t tempty_leader0 = map_to_rank(tempty(0), 0);
    int tcount = 0;
    for (int tile = cluster; tile < total; tile += nclusters, tcount++) {
      const int acc = tcount & 1;
      const int mt = tile / n_tiles, nt = tile % n_tiles;
      const int row0 = mt * PM + rank * UM + quarter * 32;
      RopeRow rr;
      const bool rope = row0 < ep.M && rope_tile(ep, nt * PN);
      if (rope) rope_prefetch(ep, row0, rr);
      const bool w = mbar_wait(tfull(acc), (tcount >> 1) & 1, abort_flag, status, 24);
      if (!__all_sync(0xffffffffu, w)) break;  // warp-uniform: tcgen05.ld is .sync.aligned
      tc_fence_after();
      const uint32_t tbase = tmem + acc * PN + ((uint32_t)(quarter * 32) << 16);
      if (row0 < ep.M)  // warp-uniform
        epilogue_tile<true>(ep, &tmap_out, tbase, row0, nt * PN, c_begin, c_end, stage, buf, &rr);
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

// 2-D fp16 K-major operand map: rows x K, 64 x 128 boxes, 128B swizzle.
static bool encode_operand(PFN_cuTensorMapEncodeTiled_v12000 enc, CUtensorMap* map, const __half* p, long rows, int K,
                           long ld) {
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {BK, 128};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(p), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static cudaError_t launch(const __half* W16, int n_virtual, int K, const __half* A, long lda, const EpiParams& ep,
                          DevStatus* status, cudaStream_t s) {
  auto enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  if (K % BK || (lda * 2) % 16 || (reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(W16) & 15) ||
      n_virtual % PN)
    return cudaErrorInvalidValue;
  CUtensorMap amap, bmap, omap;
  if (!encode_operand(enc, &amap, A, ep.M, K, lda) || !encode_operand(enc, &bmap, W16, n_virtual, K, K))
    return cudaErrorInvalidValue;
  {
    // Output map: 32-row x 128-byte boxes (32 float32 or 64 fp16 columns),
    // 128B swizzle as the epilogue stages them.
    const bool f32 = ep.mode == EPI_F32;
    void* out = f32 ? static_cast<void*>(ep.out32) : static_cast<void*>(ep.out16);
    const int esz = f32 ? 4 : 2;
    if ((ep.ldo * esz) % 16 || (reinterpret_cast<uintptr_t>(out) & 15)) return cudaErrorInvalidValue;
    const cuuint64_t odims[2] = {(cuuint64_t)ep.N, (cuuint64_t)ep.M};
    const cuuint64_t ostrides[1] = {(cuuint64_t)ep.ldo * esz};
    const cuuint32_t obox[2] = {(cuuint32_t)(128 / esz), 32};
    const cuuint32_t estr[2] = {1, 1};
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
      cudaError_t e =
          cudaFuncSetAttribute(gemm_f16_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::ALLOC);
      if (e != cudaSuccess) return e;
      int sms = 0;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(sms & ~1);
      cfg.blockDim = dim3(NTHREADS);
      cfg.dynamicSmemBytes = Lay::ALLOC;
      int n = 0;
      e = cudaOccupancyMaxActiveClusters(&n, gemm_f16_pair_kernel, &cfg);
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
  cudaLaunchAttribute attr[1];
  const cudaLaunchConfig_t cfg = pdl_config(dim3(2 * pairs), dim3(NTHREADS), Lay::ALLOC, s, attr);
  return cudaLaunchKernelEx(&cfg, gemm_f16_pair_kernel, amap, bmap, omap, K, m_tiles, n_tiles, ep, status);
}

}  // namespace tcf


cudaError_t launch_gemm_f16(const __half* W16, int n_virtual, int K, const __half* A, long lda, const EpiParams& ep,
                            DevStatus* status, cudaStream_t s) {
  if (ep.M == 0) return cudaSuccess;
  return tcf::launch(W16, n_virtual, K, A, lda, ep, status, s);
}

}  // namespace le
