// Quantised GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// out = A . W^T with A fp16 [M][K] (tokens) and W the tile-blocked quantised
// weight (common.cuh).  Persistent kernel, one CTA per SM, 256x128 output
// tiles (256 tokens x 128 weight rows), K in 64-column steps:
//
//   warp 0     producer: TMA 2-D load of the A tile (256 x 64 fp16, 128B
//              swizzle) and a 1-D bulk copy of the raw quant chunk (128 x 64
//              bytes + scales) into a load stage, both completing on one
//              mbarrier.
//   warp 1     allocates 512 TMEM columns and one lane issues tcgen05.mma
//              (kind::f16, M=128, N=128, K=16): per 16-column sub-step one
//              MMA for each 128-token half, both reading the same B tile, so
//              each dequantised weight feeds 256 tokens.
//   warps 2-5  dequantise the raw chunk into the fp16 B operand (the exact
//              reference value rounded to fp16, dequant.cuh), written in the
//              128B-swizzled K-major layout tcgen05 reads.
//   warps 6-9  epilogue: tcgen05.ld the accumulators (each thread one row of
//              each half), apply the fused epilogue (epilogue.cuh), store.
//
// A tile's two accumulators take 256 TMEM columns; two tiles' worth are
// allocated so the epilogue of tile i overlaps the main loop of tile i+1.  Every mbarrier wait is bounded (WAIT_LIMIT_NS); on
// expiry the kernel records DE_TIMEOUT in the status word and every role
// leaves its loop, so a fault in the pipeline ends the launch instead of
// hanging the GPU.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "dequant.cuh"
#include "epilogue.cuh"
#include "kernels.h"

namespace le {

namespace tc {

constexpr int BM = 256, UM = 128, BN = TILE_N, BK = TILE_K;  // UM: rows per MMA
constexpr int S_LD = 4;  // load stages (A + raw)
constexpr int S_B = 2;   // fp16 B stages
constexpr int A_BYTES = BM * BK * 2;    // 32768
constexpr int B16_BYTES = BN * BK * 2;  // 16384
constexpr int NTHREADS = 320;
constexpr int TMEM_COLS = 512;
constexpr int ACC_COLS = 2 * BN;  // one tile: two 128x128 fp32 accumulators
constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(UM >> 4) << 24);

template <int QF>
struct Layout {
  static constexpr int RAW = chunk_bytes(QF);
  static constexpr int OFF_A = 0;
  static constexpr int OFF_RAW = OFF_A + S_LD * A_BYTES;
  static constexpr int OFF_B16 = ((OFF_RAW + S_LD * RAW + 1023) / 1024) * 1024;
  static constexpr int OFF_STAGE = OFF_B16 + S_B * B16_BYTES;  // 4 epilogue warps x 32x33 floats
  static constexpr int OFF_BAR = OFF_STAGE + 4 * 32 * 33 * 4;
  // barriers: full_ld[S_LD], empty_ld[S_LD], full_b[S_B], empty_b[S_B], tfull[2], tempty[2]
  static constexpr int NBAR = 2 * S_LD + 2 * S_B + 4;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int ALLOC = BYTES + 1024;  // slack to align the base to 1024
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false (and the abort flag set, DE_TIMEOUT recorded) if the
// phase does not complete within WAIT_LIMIT_NS or another role aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, DevStatus* st,
                                          int site) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; i++) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 255) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) {
        *abort_flag = 1;
        report(st, DE_TIMEOUT, site, (int)blockIdx.x);
        return false;
      }
    }
  }
}

// AND of `ok` over the 128 dequant threads (named barrier 1): every thread
// of the group takes the same branch, so no thread is left at a barrier.
__device__ __forceinline__ bool dequant_group_all(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n.reg .pred p, q;\nsetp.ne.u32 q, %1, 0;\nbar.red.and.pred p, 1, 128, q;\nselp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)ok)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// Shared-memory matrix descriptor: K-major, 128B swizzle, 8-row atoms of
// 1024 bytes (SBO), version 1 (sm_100).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
         ((uint64_t)2 << 61);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accumulate));
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%"
      "20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// Epilogue of one 32-row x 32-column block, run by one warp.  Lane l holds
// row row0 + l of the block in v[] (for EPI_GEGLU: up values in v, gate
// values of the same output columns in g).  Row-wise math (RoPE pairs,
// gelu(gate)*up) happens in registers; the block then goes through the
// warp's shared staging area (32 x 33 floats, conflict-free both ways) so
// that global loads and stores cover whole 128-byte (f32) or 64-byte (fp16)
// row segments instead of one row per lane.
__device__ __forceinline__ void epi_block(const EpiParams& ep, int row0, int n0, float* v, const float* g,
                                          float* stg) {
  const int lane = threadIdx.x & 31;
  const int m = row0 + lane;
  int col0 = n0;  // first output column of the block
  switch (ep.mode) {
    case EPI_QKV:
      if (n0 < ep.rope_cols && m < ep.M) {
        const int i0 = (n0 % ep.head_dim) >> 1;
        const float4* cs = reinterpret_cast<const float4*>(ep.rope_cos + (long)ep.pos[m] * (ep.head_dim >> 1) + i0);
        const float4* sn = reinterpret_cast<const float4*>(ep.rope_sin + (long)ep.pos[m] * (ep.head_dim >> 1) + i0);
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const float4 c = cs[q], s = sn[q];
          const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const float x0 = v[8 * q + 2 * i], x1 = v[8 * q + 2 * i + 1];
            v[8 * q + 2 * i] = __fsub_rn(__fmul_rn(x0, cc[i]), __fmul_rn(x1, ss[i]));
            v[8 * q + 2 * i + 1] = __fadd_rn(__fmul_rn(x0, ss[i]), __fmul_rn(x1, cc[i]));
          }
        }
      }
      break;
    case EPI_GEGLU:
#pragma unroll
      for (int i = 0; i < 32; i++) v[i] = gelu_tanh_rational(g[i]) * v[i];
      col0 = (n0 / TILE_N) * GEGLU_HALF + (n0 % TILE_N);
      break;
    default:
      break;
  }
#pragma unroll
  for (int j = 0; j < 32; j++) stg[lane * 33 + j] = v[j];
  __syncwarp();
  if (ep.mode == EPI_QKV || ep.mode == EPI_GEGLU) {
    // fp16 out: two rows per instruction, lane pairs of columns.
    const int hr = lane >> 4, c = 2 * (lane & 15);
    if (col0 + c < ep.N) {
#pragma unroll 4
      for (int i = 0; i < 32; i += 2) {
        const int r = i + hr;
        if (row0 + r < ep.M)
          *reinterpret_cast<uint32_t*>(ep.out16 + (long)(row0 + r) * ep.ldo + col0 + c) =
              pack_half2(stg[r * 33 + c], stg[r * 33 + c + 1]);
      }
    }
  } else {
    const int col = col0 + lane;
    if (col < ep.N) {
      const int nrow = min(32, ep.M - row0);
      float* out = ep.out32 + (long)row0 * ep.ldo + col;
      if (ep.mode == EPI_RESID) {
        // resid may alias out: read the whole block before the first store.
        const float* rp = ep.resid + (long)row0 * ep.ldo + col;
        float r[32];
#pragma unroll
        for (int i = 0; i < 32; i++) r[i] = i < nrow ? rp[(long)i * ep.ldo] : 0.f;
#pragma unroll
        for (int i = 0; i < 32; i++)
          if (i < nrow) out[(long)i * ep.ldo] = __fadd_rn(r[i], stg[i * 33 + lane]);
      } else {
#pragma unroll 8
        for (int i = 0; i < 32; i++)
          if (i < nrow) out[(long)i * ep.ldo] = stg[i * 33 + lane];
      }
    }
  }
  __syncwarp();
}

template <int QF>
__global__ void __launch_bounds__(NTHREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const uint8_t* __restrict__ W, int K, int m_tiles,
                   int n_tiles, EpiParams ep, DevStatus* status) {
  using Lay = Layout<QF>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + Lay::OFF_BAR;
  auto full_ld = [&](int s) { return bar0 + 8 * s; };
  auto empty_ld = [&](int s) { return bar0 + 8 * (S_LD + s); };
  auto full_b = [&](int j) { return bar0 + 8 * (2 * S_LD + j); };
  auto empty_b = [&](int j) { return bar0 + 8 * (2 * S_LD + S_B + j); };
  auto tfull = [&](int a) { return bar0 + 8 * (2 * S_LD + 2 * S_B + a); };
  auto tempty = [&](int a) { return bar0 + 8 * (2 * S_LD + 2 * S_B + 2 + a); };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Lay::OFF_MISC);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Lay::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ksteps = K / BK;
  const int total = m_tiles * n_tiles;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    for (int s = 0; s < S_LD; s++) {
      mbar_init(full_ld(s), 1);
      mbar_init(empty_ld(s), 2);  // MMA commit + dequant group
    }
    for (int j = 0; j < S_B; j++) {
      mbar_init(full_b(j), 1);
      mbar_init(empty_b(j), 1);
    }
    for (int a = 0; a < 2; a++) {
      mbar_init(tfull(a), 1);
      mbar_init(tempty(a), 4);  // one arrival per epilogue warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < total && !*abort_flag; tile += gridDim.x) {
        const int mt = tile / n_tiles, nt = tile % n_tiles;
        const uint8_t* wt = W + (long)nt * ksteps * Lay::RAW;
        for (int ks = 0; ks < ksteps; ks++, it++) {
          const int s = it % S_LD;
          const uint32_t r = it / S_LD;
          if (!mbar_wait(empty_ld(s), (r & 1) ^ 1, abort_flag, status, 1)) break;
          mbar_expect_tx(full_ld(s), A_BYTES + Lay::RAW);
          tma_load_2d(sbase + Lay::OFF_A + s * A_BYTES, &tmap_a, ks * BK, mt * BM, full_ld(s));
          bulk_load(sbase + Lay::OFF_RAW + s * Lay::RAW, wt + (long)ks * Lay::RAW, Lay::RAW, full_ld(s));
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t it = 0, jt = 0;
      int tcount = 0;
      for (int tile = blockIdx.x; tile < total && !*abort_flag; tile += gridDim.x, tcount++) {
        const int acc = tcount & 1;
        const uint32_t ar = tcount >> 1;
        if (!mbar_wait(tempty(acc), (ar & 1) ^ 1, abort_flag, status, 2)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * ACC_COLS;
        bool ok = true;
        for (int ks = 0; ks < ksteps; ks++, it++, jt++) {
          const int s = it % S_LD, j = jt % S_B;
          if (!mbar_wait(full_ld(s), (it / S_LD) & 1, abort_flag, status, 3) ||
              !mbar_wait(full_b(j), (jt / S_B) & 1, abort_flag, status, 4)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = sbase + Lay::OFF_A + s * A_BYTES;
          const uint32_t b_addr = sbase + Lay::OFF_B16 + j * B16_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; kk++) {
            const uint64_t bdesc = sw128_desc(b_addr + kk * 32);
            mma_f16(d, sw128_desc(a_addr + kk * 32), bdesc, (ks | kk) != 0);
            mma_f16(d + BN, sw128_desc(a_addr + UM * 128 + kk * 32), bdesc, (ks | kk) != 0);
          }
          mma_commit(empty_ld(s));
          mma_commit(empty_b(j));
        }
        if (!ok) break;
        mma_commit(tfull(acc));
      }
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ dequant
    const int t = threadIdx.x - 64;  // 0..127
    const int c16 = t & 3, r0 = t >> 2;  // 16-byte column chunk, first row
    uint32_t it = 0, jt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
      for (int ks = 0; ks < ksteps; ks++, it++, jt++) {
        const int s = it % S_LD, j = jt % S_B;
        const bool w = mbar_wait(full_ld(s), (it / S_LD) & 1, abort_flag, status, 5) &&
                       mbar_wait(empty_b(j), ((jt / S_B) & 1) ^ 1, abort_flag, status, 6);
        if (!dequant_group_all(w)) {
          ok = false;
          break;
        }
        const uint8_t* raw = smem + Lay::OFF_RAW + s * Lay::RAW;
        uint8_t* b16 = smem + Lay::OFF_B16 + j * B16_BYTES;
#pragma unroll
        for (int q = 0; q < BN / 32; q++) {
          const int n = r0 + 32 * q;
          const uint4 u = *reinterpret_cast<const uint4*>(raw + n * BK + c16 * 16);
          const int g0 = 2 * c16, sw = n & 7;
          *reinterpret_cast<uint4*>(b16 + n * 128 + ((g0 ^ sw) << 4)) =
              dq8_f16<QF>(make_uint2(u.x, u.y), raw + TILE_Q_BYTES, n, g0);
          *reinterpret_cast<uint4*>(b16 + n * 128 + (((g0 + 1) ^ sw) << 4)) =
              dq8_f16<QF>(make_uint2(u.z, u.w), raw + TILE_Q_BYTES, n, g0 + 1);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (t == 0) {
          mbar_arrive(full_b(j));
          mbar_arrive(empty_ld(s));
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    int tcount = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, tcount++) {
      const int acc = tcount & 1;
      const bool w = mbar_wait(tfull(acc), (tcount >> 1) & 1, abort_flag, status, 7);
      if (!__all_sync(0xffffffffu, w)) break;  // warp-uniform: tcgen05.ld is .sync.aligned
      tc_fence_after();
      const int mt = tile / n_tiles, nt = tile % n_tiles;
      float* stg = reinterpret_cast<float*>(smem + Lay::OFF_STAGE) + (warp - 6) * 32 * 33;
      for (int h = 0; h < BM / UM; h++) {
        const int row0 = mt * BM + h * UM + quarter * 32;
        const uint32_t tbase = tmem + acc * ACC_COLS + h * BN + ((uint32_t)(quarter * 32) << 16);
        if (row0 >= ep.M) continue;  // warp-uniform
        if (ep.mode == EPI_GEGLU) {
          for (int c = 0; c < BN / 2; c += 32) {
            float v[32], gt[32];
            tmem_ld32(tbase + c, v);
            tmem_ld32(tbase + BN / 2 + c, gt);
            epi_block(ep, row0, nt * BN + c, v, gt, stg);
          }
        } else {
          for (int c = 0; c < BN; c += 32) {
            float v[32];
            tmem_ld32(tbase + c, v);
            epi_block(ep, row0, nt * BN + c, v, nullptr, stg);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty(acc));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
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

int num_sms() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

template <int QF>
cudaError_t launch_tc(const uint8_t* W, int n_virtual, int K, const __half* A, long lda, const EpiParams& ep,
                      DevStatus* status, cudaStream_t s) {
  auto enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  if (K % BK || (lda * 2) % 16 || (reinterpret_cast<uintptr_t>(A) & 15)) return cudaErrorInvalidValue;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)ep.M};
  const cuuint64_t strides[1] = {(cuuint64_t)lda * 2};
  const cuuint32_t box[2] = {BK, BM};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(A), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  static std::mutex mu;
  static uint64_t attr_set = 0;  // per-device bit: the attribute is a per-device setting
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 64 || !(attr_set >> dev & 1)) {
      cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<QF>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           Layout<QF>::ALLOC);
      if (e != cudaSuccess) return e;
      if (dev < 64) attr_set |= 1ull << dev;
    }
  }
  const int m_tiles = (ep.M + BM - 1) / BM;
  const int n_tiles = n_virtual / BN;
  const int total = m_tiles * n_tiles;
  const int grid = total < num_sms() ? total : num_sms();
  gemm_tc_kernel<QF><<<grid, NTHREADS, Layout<QF>::ALLOC, s>>>(map, W, K, m_tiles, n_tiles, ep, status);
  return cudaGetLastError();
}

}  // namespace tc

cudaError_t launch_gemm_tc(int qf, const uint8_t* W, int n_virtual, int K, const __half* A, long lda,
                           const EpiParams& ep, DevStatus* status, cudaStream_t s) {
  if (ep.M == 0) return cudaSuccess;
  if (n_virtual % TILE_N) return cudaErrorInvalidValue;
  switch (qf) {
    case QF_Q8_0: return tc::launch_tc<QF_Q8_0>(W, n_virtual, K, A, lda, ep, status, s);
    case QF_KMIN: return tc::launch_tc<QF_KMIN>(W, n_virtual, K, A, lda, ep, status, s);
    case QF_Q6K: return tc::launch_tc<QF_Q6K>(W, n_virtual, K, A, lda, ep, status, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace le
