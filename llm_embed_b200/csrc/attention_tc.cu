// Tensor-core (tcgen05) attention for long sequences (bert.go:356-402).
//
// One CTA per (128 queries, head, sequence), three CTAs per SM.  Scores
// S = Q.K^T of a 64-key block are one tcgen05.mma chain (M=128 queries, N=64
// keys, K=64) into TMEM; the softmax warps read S from TMEM, and in the
// second pass write P = exp(0.125 S - max) (the reference's rule: 0 when
// more than 10 below the row maximum, ops_simd.go:70-82) as fp16 into shared
// memory, from where O += P.V runs on the tensor cores (M=128, N=64, K=64)
// into TMEM (128 columns per CTA: S and O).
// Two passes over the keys, as in the mma.sync kernels: the exact row maximum
// must be known before any weight is exponentiated.  P = 2^(S * 0.125 log2 e
// - max * 0.125 log2 e), one fused multiply-add per two keys, with the
// cutoff in the same base-2 units (softmax_tc.cuh, shared with the short
// kernel).
//
//   warp 0      producer: TMA loads of Q (once), of each key block's K
//               (both passes) into a 2-stage ring freed as soon as S has
//               read it, and of its V (pass 2) into a second 2-stage ring
//               freed by P.V, so the next K never waits behind a P.V.
//   warp 1      TMEM allocation; one lane issues the MMAs: S(j+1) is issued
//               before P(j).V (the softmax releases S as soon as it holds
//               it in registers), so the softmax of block j overlaps it.
//   warps 2-5   softmax and epilogue: thread = query row (TMEM lane), all
//               64 columns of a block.
//
// Operand layouts: Q, K, V tiles come from one TMA map over qkv [T][3H]
// (128-byte swizzle, 64 columns = one head); Q and K are K-major operands as
// in the GEMMs, V [keys][64] is the MN-major B operand of P.V (16 keys = two
// 8-row swizzle atoms = 2048 bytes per MMA).  P [128][64] is one K-major
// block written by the softmax warps in the swizzled layout.
// Rows of Q and K/V past the sequence belong to the next sequence (or are
// zero past T): their scores are masked, their weights exactly 0.
// Every wait is bounded (WAIT_LIMIT_NS) and reports DE_TIMEOUT.
#include <cudaTypedefs.h>

#include <mutex>

#include "kernels.h"
#include "softmax_tc.cuh"
#include "tcgen05.cuh"

namespace le {
namespace atc {

using namespace tcx;

constexpr int BQ = 128;   // query rows per CTA (TMEM lanes)
constexpr int BKEY = 64;  // keys per block
constexpr int HD = 64;
constexpr int NSOFT = 4;  // softmax warps: one query row per thread
constexpr int SOFT_WARP0 = 2;
constexpr int NTHREADS = (SOFT_WARP0 + NSOFT) * 32;
constexpr int Q_BYTES = BQ * HD * 2;     // 16 KB
constexpr int KV_BYTES = BKEY * HD * 2;  // 8 KB: one K or V block
constexpr int P_BYTES = BQ * BKEY * 2;   // 16 KB: P [128][64], one K-major swizzled block
constexpr int TMEM_COLS = 128;           // S at 0, O at 64
constexpr uint32_t IDESC_S = idesc_f16(BQ, BKEY);
constexpr uint32_t IDESC_O = idesc_f16(BQ, HD) | (1u << 16);  // B (V) MN-major

struct Lay {
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;       // [2 stages]
  static constexpr int OFF_V = OFF_K + 2 * KV_BYTES;  // [2 stages]
  static constexpr int OFF_P = OFF_V + 2 * KV_BYTES;
  static constexpr int OFF_BAR = OFF_P + P_BYTES;
  // q_full, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full, s_empty,
  // p_full, p_empty, o_full
  static constexpr int NBAR = 14;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_MISC + 16;
  static constexpr int ALLOC = BYTES + 1024;
  static_assert(ALLOC <= 232448 / 3, "three CTAs per SM");
};

__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%"
      "20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__global__ void __launch_bounds__(NTHREADS, 3)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmap, const int32_t* __restrict__ offsets, int H,
                        int min_len, __half* __restrict__ out, DevStatus* status) {
  const int qb = blockIdx.x, head = blockIdx.y, seq = blockIdx.z;
  const int t0 = offsets[seq];
  const int L = offsets[seq + 1] - t0;
  if (L <= 0 || L < min_len || qb * BQ >= L) return;
  const int nkb = (L + BKEY - 1) / BKEY;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + Lay::OFF_BAR;
  const uint32_t q_full = bar0;
  auto k_full = [&](int s) { return bar0 + 8 * (1 + s); };
  auto k_empty = [&](int s) { return bar0 + 8 * (3 + s); };
  auto v_full = [&](int s) { return bar0 + 8 * (5 + s); };
  auto v_empty = [&](int s) { return bar0 + 8 * (7 + s); };
  const uint32_t s_full = bar0 + 8 * 9, s_empty = bar0 + 8 * 10;
  const uint32_t p_full = bar0 + 8 * 11, p_empty = bar0 + 8 * 12, o_full = bar0 + 8 * 13;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Lay::OFF_MISC);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Lay::OFF_MISC + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; i++) {
      mbar_init(k_full(i), 1);
      mbar_init(k_empty(i), 1);
      mbar_init(v_full(i), 1);
      mbar_init(v_empty(i), 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, NSOFT);
    mbar_init(p_full, NSOFT);
    mbar_init(p_empty, 1);
    mbar_init(o_full, 1);
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
  const int colq = head * HD, colk = H + head * HD, colv = 2 * H + head * HD;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap)) : "memory");
      mbar_expect_tx(q_full, Q_BYTES);
      // Q as two 64-row boxes: stacked, they form the 128-row swizzled tile.
      tma_load_2d(sbase + Lay::OFF_Q, &tmap, colq, t0 + qb * BQ, q_full);
      tma_load_2d(sbase + Lay::OFF_Q + KV_BYTES, &tmap, colq, t0 + qb * BQ + BKEY, q_full);
      uint32_t ik = 0, iv = 0;  // K and V ring counters
      bool ok = true;
      for (int pass = 0; pass < 2 && ok; pass++)
        for (int j = 0; j < nkb; j++, ik++) {
          const int s = ik & 1;
          if (!mbar_wait(k_empty(s), ((ik >> 1) & 1) ^ 1, abort_flag, status, 31)) {
            ok = false;
            break;
          }
          mbar_expect_tx(k_full(s), KV_BYTES);
          tma_load_2d(sbase + Lay::OFF_K + s * KV_BYTES, &tmap, colk, t0 + j * BKEY, k_full(s));
          if (pass == 1) {
            const int v = iv & 1;
            if (!mbar_wait(v_empty(v), ((iv >> 1) & 1) ^ 1, abort_flag, status, 30)) {
              ok = false;
              break;
            }
            mbar_expect_tx(v_full(v), KV_BYTES);
            tma_load_2d(sbase + Lay::OFF_V + v * KV_BYTES, &tmap, colv, t0 + j * BKEY, v_full(v));
            iv++;
          }
        }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, abort_flag, status, 32);
      tc_fence_after();
      const uint32_t qaddr = sbase + Lay::OFF_Q;
      uint32_t ik = 0, sn = 0;  // K ring counter, S use counter
      // S(j) = Q . K(j)^T into the S columns, once the softmax has read the
      // last S; the K stage is free once S is computed.
      auto issue_s = [&]() -> bool {
        const int s = ik & 1;
        if (!mbar_wait(k_full(s), (ik >> 1) & 1, abort_flag, status, 33) ||
            !mbar_wait(s_empty, (sn & 1) ^ 1, abort_flag, status, 34))
          return false;
        tc_fence_after();
        const uint32_t kaddr = sbase + Lay::OFF_K + s * KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++)
          mma_f16(tmem, sw128_desc(qaddr + kk * 32), sw128_desc(kaddr + kk * 32), IDESC_S, kk != 0);
        mma_commit(s_full);
        mma_commit(k_empty(s));
        sn++;
        ik++;
        return true;
      };
      // Pass 1: scores only.
      for (int j = 0; j < nkb && ok; j++) ok = issue_s();
      // Pass 2: S(j), then P(j-1).V(j-1), which frees V's stage and P.
      uint32_t pn = 0, iv = 0;
      auto issue_pv = [&](bool first) -> bool {
        const int v = iv & 1;
        if (!mbar_wait(p_full, pn & 1, abort_flag, status, 35) ||
            !mbar_wait(v_full(v), (iv >> 1) & 1, abort_flag, status, 37))
          return false;
        tc_fence_after();
        const uint32_t vaddr = sbase + Lay::OFF_V + v * KV_BYTES;
        const uint32_t paddr = sbase + Lay::OFF_P;
#pragma unroll
        for (int kk = 0; kk < BKEY / 16; kk++)
          mma_f16(tmem + BKEY, sw128_desc(paddr + kk * 32), sw128_desc(vaddr + kk * 2048), IDESC_O,
                  !(first && kk == 0));
        mma_commit(v_empty(v));
        mma_commit(p_empty);
        pn++;
        iv++;
        return true;
      };
      for (int j = 0; j < nkb && ok; j++) {
        ok = issue_s();
        if (ok && j > 0) ok = issue_pv(j == 1);
      }
      if (ok) ok = issue_pv(nkb == 1);
      if (ok) mma_commit(o_full);
    }
  } else {
    // ---------------------------------------------------------------- softmax
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // query row in the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint8_t* prow = smem + Lay::OFF_P + row * 128;
    bool ok = true;
    uint32_t sn = 0, pn = 0;
    float m0 = -INFINITY, m1 = -INFINITY;
    for (int j = 0; j < nkb; j++, sn++) {
      ok = ok && __all_sync(0xffffffffu, mbar_wait(s_full, sn & 1, abort_flag, status, 36));
      uint32_t r[64];
      if (ok) {
        tc_fence_after();
        tmem_ld32_nowait(tmem + lane_off, r);
        tmem_ld32_nowait(tmem + lane_off + 32, r + 32);
        tmem_wait_ld();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_empty);
      if (ok) {
        // Maximum of the raw scores of keys < L.
        const int kmax = L - j * BKEY;
#pragma unroll
        for (int c = 0; c < BKEY / 16; c++)
          if (16 * c < kmax) chunk_max<16>(m0, m1, r + 16 * c, kmax - 16 * c);
      }
    }
    const float mx = fmaxf(m0, m1);
    const unsigned long long scale = f2_pack(SCALE2, SCALE2), off = f2_pack(-mx * SCALE2, -mx * SCALE2);
    unsigned long long s0 = f2_pack(0.f, 0.f), s1 = s0;
    for (int j = 0; j < nkb; j++, sn++, pn++) {
      ok = ok && __all_sync(0xffffffffu, mbar_wait(s_full, sn & 1, abort_flag, status, 38));
      uint32_t r[64];
      if (ok) {
        tc_fence_after();
        tmem_ld32_nowait(tmem + lane_off, r);
        tmem_ld32_nowait(tmem + lane_off + 32, r + 32);
        tmem_wait_ld();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_empty);
      ok = ok && __all_sync(0xffffffffu, mbar_wait(p_empty, (pn & 1) ^ 1, abort_flag, status, 39));
      if (ok) {
        // P row `row` = 8 chunks of 8 fp16 keys in the 128-byte-swizzled
        // K-major layout, 16 keys per step; keys past the sequence get
        // weight 0.
        const int kmax = L - j * BKEY;
#pragma unroll
        for (int c = 0; c < BKEY / 16; c++) {
          uint32_t w[8];
          chunk_p<16>(r + 16 * c, kmax - 16 * c, scale, off, s0, s1, w);
          *reinterpret_cast<uint4*>(prow + (((2 * c) ^ (row & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint4*>(prow + (((2 * c + 1) ^ (row & 7)) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    ok = ok && __all_sync(0xffffffffu, mbar_wait(o_full, 0, abort_flag, status, 41));
    if (ok) {
      tc_fence_after();
      float l0, l1;
      f2_unpack(f2_add(s0, s1), l0, l1);
      const float inv = 1.0f / (l0 + l1);
      uint32_t r[64];
      tmem_ld32_nowait(tmem + lane_off + BKEY, r);
      tmem_ld32_nowait(tmem + lane_off + BKEY + 32, r + 32);
      tmem_wait_ld();
      const int q = qb * BQ + row;
      if (q < L) {
        uint4* o = reinterpret_cast<uint4*>(out + (long)(t0 + q) * H + head * HD);
#pragma unroll
        for (int c = 0; c < 8; c++)
          o[c] = make_uint4(pack_half2(__uint_as_float(r[8 * c]) * inv, __uint_as_float(r[8 * c + 1]) * inv),
                            pack_half2(__uint_as_float(r[8 * c + 2]) * inv, __uint_as_float(r[8 * c + 3]) * inv),
                            pack_half2(__uint_as_float(r[8 * c + 4]) * inv, __uint_as_float(r[8 * c + 5]) * inv),
                            pack_half2(__uint_as_float(r[8 * c + 6]) * inv, __uint_as_float(r[8 * c + 7]) * inv));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
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

}  // namespace atc

cudaError_t launch_attention_tc(const __half* qkv, const int32_t* offsets, int nseq, int T, int max_len, int min_len,
                                int H, int heads, __half* out, DevStatus* status, cudaStream_t s) {
  if (nseq == 0 || max_len == 0 || T == 0) return cudaSuccess;
  auto enc = atc::encode_fn();
  if (!enc) return cudaErrorNotSupported;
  if ((3L * H * 2) % 16 || (reinterpret_cast<uintptr_t>(qkv) & 15)) return cudaErrorInvalidValue;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)(3 * H), (cuuint64_t)T};
  const cuuint64_t strides[1] = {(cuuint64_t)(3 * H) * 2};
  const cuuint32_t box[2] = {atc::HD, atc::BKEY};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(qkv), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  static std::mutex mu;
  static uint64_t attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 64 || !(attr_set >> dev & 1)) {
      cudaError_t e = cudaFuncSetAttribute(atc::attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           atc::Lay::ALLOC);
      if (e != cudaSuccess) return e;
      if (dev < 64) attr_set |= 1ull << dev;
    }
  }
  for (int s0 = 0; s0 < nseq; s0 += 65535) {  // grid.z limit
    const int n = nseq - s0 < 65535 ? nseq - s0 : 65535;
    atc::attention_tc_kernel<<<dim3((max_len + atc::BQ - 1) / atc::BQ, heads, n), atc::NTHREADS, atc::Lay::ALLOC,
                                 s>>>(map, offsets + s0, H, min_len, out, status);
  }
  return cudaGetLastError();
}

}  // namespace le
