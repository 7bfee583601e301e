// PTX helpers for the tcgen05 GEMM kernels (sm_100a): mbarriers with
// bounded waits, TMA / bulk copies, UMMA descriptors, tcgen05.mma / commit /
// ld, and the shared epilogue block.
#pragma once
#include <cuda.h>

#include "dequant.cuh"
#include "epilogue.cuh"

namespace le {
namespace tcx {

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
// Cluster-scope acquire: pairs with releases from the other CTA of a pair.
__device__ __forceinline__ bool mbar_try_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, "
      "0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
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

// try_wait with a suspend-time hint: the thread may sleep (up to `ns`)
// until the phase completes instead of returning at once, so waiting warps
// take no issue slots from working ones.
__device__ __forceinline__ bool mbar_try_sleep(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\nselp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
// mbar_wait with sleeping tries (bounded the same way; each try sleeps at
// most 20 us).
__device__ __forceinline__ bool mbar_wait_sleep(uint32_t bar, uint32_t parity, volatile int* abort_flag, DevStatus* st,
                                                int site) {
  if (mbar_try_sleep(bar, parity, 20000)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; i++) {
    if (mbar_try_sleep(bar, parity, 20000)) return true;
    if ((i & 15) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > WAIT_LIMIT_NS) {
        *abort_flag = 1;
        report(st, DE_TIMEOUT, site, (int)blockIdx.x);
        return false;
      }
    }
  }
}


// Bounded wait: false (and the abort flag set, DE_TIMEOUT recorded) if the
// phase does not complete within WAIT_LIMIT_NS or another role aborted.
template <bool CLUSTER = false>
__device__ __forceinline__ bool mbar_wait_impl(uint32_t bar, uint32_t parity, volatile int* abort_flag, DevStatus* st,
                                               int site);
template <bool CLUSTER = false>
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, DevStatus* st,
                                          int site) {
  return mbar_wait_impl<CLUSTER>(bar, parity, abort_flag, st, site);
}
template <bool CLUSTER>
__device__ __forceinline__ bool mbar_wait_impl(uint32_t bar, uint32_t parity, volatile int* abort_flag, DevStatus* st,
                                               int site) {
  auto try_once = [&] { return CLUSTER ? mbar_try_cluster(bar, parity) : mbar_try(bar, parity); };
  if (try_once()) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; i++) {
    if (try_once()) return true;
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

// AND of `ok` over the dequant threads (named barrier 1): every thread of
// the group takes the same branch, so no thread is left at a barrier.
__device__ __forceinline__ bool dequant_group_all(bool ok, int nthreads) {
  uint32_t r;
  asm volatile(
      "{\n.reg .pred p, q;\nsetp.ne.u32 q, %1, 0;\nbar.red.and.pred p, 1, %2, q;\nselp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)ok), "r"(nthreads)
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

// Instruction descriptor of kind::f16: fp16 A and B (K-major), fp32 D.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// CTA-pair MMA (issued by the pair's even CTA): A and B operands are read
// from the same shared-memory offsets in both CTAs, D is written to both
// CTAs' TMEM (each its own 128 rows).
__device__ __forceinline__ void mma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// Arrive on the barrier at this shared offset in every CTA of `mask` once
// all prior tcgen05.mma of the pair have completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar, uint16_t mask) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                   bar),
               "h"(mask)
               : "memory");
}
// Address of the same shared variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Arrive on a barrier of another CTA of the cluster (address from mapa).
// Default semantics, as CUTLASS's cluster pipelines use: a cluster-scope
// release here costs thousands of cycles per arrive.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA 2-D load of a CTA-pair kernel: data to this CTA's shared memory, the
// transaction bytes to the barrier at `bar_cluster` (the even CTA's).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
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
// values of the same output columns in g; for EPI_QKV with RoPE: the row's
// cos/sin for the block's 16 rotation pairs in cs/sn).  Row-wise math
// happens in registers; the block then goes through the warp's shared
// staging area (32 x 33 floats, conflict-free both ways) so that global
// stores cover whole 128-byte (f32) or 64-byte (fp16) row segments.
__device__ __forceinline__ void epi_block(const EpiParams& ep, int row0, int n0, float* v, const float* g,
                                          const float* cs, const float* sn, float* stg) {
  const int lane = threadIdx.x & 31;
  int col0 = n0;  // first output column of the block
  if (ep.mode == EPI_QKV && cs) {
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const float x0 = v[2 * i], x1 = v[2 * i + 1];
      v[2 * i] = __fsub_rn(__fmul_rn(x0, cs[i]), __fmul_rn(x1, sn[i]));
      v[2 * i + 1] = __fadd_rn(__fmul_rn(x0, sn[i]), __fmul_rn(x1, cs[i]));
    }
  } else if (ep.mode == EPI_GEGLU) {
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = gelu_tanh_rational(g[i]) * v[i];
    col0 = (n0 / TILE_N) * GEGLU_HALF + (n0 % TILE_N);
  }
#pragma unroll
  for (int j = 0; j < 32; j++) stg[lane * 33 + j] = v[j];
  __syncwarp();
  const int nrow = min(32, ep.M - row0);
  if (ep.mode == EPI_F32) {
    const int col = col0 + lane;
    if (col < ep.N) {
      float* out = ep.out32 + (long)row0 * ep.ldo + col;
#pragma unroll 8
      for (int i = 0; i < 32; i++)
        if (i < nrow) out[(long)i * ep.ldo] = stg[i * 33 + lane];
    }
  } else {
    // fp16 out: two rows per instruction, lane pairs of columns.
    const int hr = lane >> 4, c = 2 * (lane & 15);
    if (col0 + c < ep.N) {
#pragma unroll 4
      for (int i = 0; i < 32; i += 2) {
        const int r = i + hr;
        if (r < nrow)
          *reinterpret_cast<uint32_t*>(ep.out16 + (long)(row0 + r) * ep.ldo + col0 + c) =
              pack_half2(stg[r * 33 + c], stg[r * 33 + c + 1]);
      }
    }
  }
  __syncwarp();
}


}  // namespace tcx
}  // namespace le
