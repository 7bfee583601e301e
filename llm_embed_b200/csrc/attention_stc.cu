// Tensor-core (tcgen05) attention for sequences of at most 128 tokens in
// large batches (bert.go:356-402): the workload of the batched configs,
// where every (sequence, head) is one small unit of work.
//
// Persistent kernel, one CTA per SM, four independent groups of four warps
// (thread = query row = TMEM lane), each with a unit in flight in its own
// 128-column TMEM slot.  A unit is one head of one sequence of 65..128
// tokens, or of two sequences of at most 64 tokens packed into query rows
// 0..63 (A) and 64..127 (B); the work list comes from attention_units_kernel
// (below), once per forward.  A unit's whole key range fits one MMA: S =
// Q.K^T (M=128 query rows, N = the keys rounded up to 16: 128 when packed,
// A's keys in columns 0..63 and B's in 64..127, K=64) into the slot; each
// row reads its own sequence's scores, finds the exact maximum and writes P
// = exp(0.125 S - max) (0 when more than 10 below the maximum, the
// reference's rule, ops_simd.go:70-82) as fp16 pairs back into the slot
// over the scores it has read, and zeros over the other sequence's keys;
// O = P.V (A = P from TMEM, B = V from shared memory; N=64, K = the keys)
// lands in the slot's upper 64 columns, and the group normalises and stores
// it.  A row's scores, P and O are those of the same row in a unit of its
// sequence alone (the other sequence's keys add exact zeros), so packing
// does not change any bit.  Warps whose 32 rows all lie past their sequence
// skip the unit's arithmetic.
//
// One elected thread per group (lane 0 of its first warp) takes the CTA's
// next unit from a shared counter (unit u = descriptor u / heads, head u %
// heads; CTA c takes c, c + grid, ... in turn) and issues everything
// asynchronous of the group: the TMA loads of the next unit's Q|K (as soon
// as S has read the current ones), S of the next unit and its V (once the
// group has read O out of the slot, P.V having read V), and P.V.  The four
// warps meet at two named barriers per unit (P written; O read), then store
// their rows' outputs straight from registers as whole 32-byte sectors.  No
// group ever waits for another, so a long unit holds back only its own
// group.
//
// Operands: one TMA map over qkv [T][3H] (64-column boxes of 64 rows,
// 128-byte swizzle); Q and K K-major; V [keys][64] the MN-major B operand of
// P.V (16 keys = 2048 bytes).  Rows past the sequence belong to the next one
// (or are zero past T): their scores are masked and their outputs not
// stored.  Every mbarrier wait is bounded (WAIT_LIMIT_NS) and reports
// DE_TIMEOUT; a group leaves its loop only on a decision all its threads
// share (an OR-reduction at its named barrier), after its elected thread
// has drained the copies and MMAs it still has in flight.
#include <cudaTypedefs.h>

#include <mutex>

#include "gemm_epi_tc.cuh"
#include "kernels.h"
#include "softmax_tc.cuh"

namespace le {
namespace stc {

using namespace tcx;

constexpr int BQ = 128;  // query rows per unit (TMEM lanes)
constexpr int MAXL = 128;
static_assert(MAXL == ATTN_SHORT_MAX, "this kernel covers the short-sequence class");
constexpr int HD = 64;
constexpr int BOX = 64;         // rows per TMA box
constexpr int G = 4;            // groups = units in flight = TMEM slots
constexpr int GROUP_WARPS = 4;  // one query row per thread
constexpr int NTHREADS = G * GROUP_WARPS * 32;
constexpr int QKV_BYTES = MAXL * HD * 2;  // 16 KB: 128 rows of one of Q, K, V
constexpr int TMEM_COLS = 512;            // G slots of 128 columns
// Within a slot: S at columns [0, 128); P (fp16 pairs) written over S at
// [0, L/2); O at [64, 128) once S is consumed.
constexpr int TM_O = 64;

struct Lay {
  static constexpr int GSTRIDE = 3 * QKV_BYTES;  // per group: Q, K, V
  static constexpr int OFF_BAR = G * GSTRIDE;
  // per group: qk_full, v_full, s_full, o_full
  static constexpr int NBAR = 4 * G;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;  // abort flag, TMEM base, unit counter
  static constexpr int OFF_UNITS = OFF_MISC + 16;      // next unit [G][2] (int4)
  static constexpr int OFF_GS = OFF_UNITS + 16 * 2 * G;  // GroupState [G]
  static constexpr int BYTES = OFF_GS + 80 * G;
  static constexpr int ALLOC = BYTES + 1024;
  static_assert(ALLOC <= 232448, "shared memory budget");
};

// The elected thread's bookkeeping, kept in shared memory so that the
// registers go to the rows' scores: the unit whose Q|K are loading, the
// unit fetch in flight, and the phases issued / waited (for the drain on
// exit).
struct GroupState {
  int4 un;
  int4 desc;     // the fetched unit's descriptor (cp.async target)
  long long pu;  // counter value taken (-1: none in flight)
  uint32_t nq, nqw, nv, nvw, ns, no, sw, ow;
};
static_assert(sizeof(GroupState) <= 80, "group state slot");

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
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

constexpr int PK = 16;  // keys per step of the P pass (one TMEM load each; 32 spills registers)

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
template <int N>
__device__ __forceinline__ void tmem_ld_nowait(uint32_t taddr, uint32_t* r) {
  static_assert(N == 16 || N == 32, "16 or 32 columns");
  if constexpr (N == 16)
    tmem_ld16_nowait(taddr, r);
  else
    tmem_ld32_nowait(taddr, r);
}
// N/2 columns: the fp16 pairs of N keys.
template <int N>
__device__ __forceinline__ void tmem_st_half(uint32_t taddr, const uint32_t* v) {
  if constexpr (N == 16)
    tmem_st8(taddr, v);
  else
    tmem_st16(taddr, v);
}
// D (TMEM) (+)= A (TMEM: lane = row, two fp16 of K per 32-bit column) . B
// (shared memory descriptor).
__device__ __forceinline__ void mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// ---------------------------------------------------------------- unit list
//
// The kernel's work list, built once per forward: descriptors {t0A, LA,
// t0B, LB} (LB = 0: one sequence), each taken by `heads` units.  A sequence
// of PACK_MAX + 1 .. MAXL tokens is one descriptor; sequences of at most
// PACK_MAX tokens go two to a descriptor (a lone last one alone).
// Descriptors are ordered longest first (sequences sorted by length; the
// short ones paired in that order), so the units every CTA takes in turn
// are of about the same length and the CTAs finish together.  Empty
// sequences and those longer than MAXL (attention_tc.cu) are left out.
//
// Buffer: descriptors [cap] int4, sorted sequence indices [cap] int32, then
// the descriptor count (int32, 16-byte aligned).
constexpr int PACK_MAX = 64;
__host__ __device__ inline size_t units_sorted_off(int cap) { return (size_t)cap * 16; }
__host__ __device__ inline size_t units_count_off(int cap) { return ((size_t)cap * 20 + 15) & ~(size_t)15; }

// One CTA: a counting sort of the sequences by length (descending), then
// the descriptors.  The order of equal lengths follows the atomics; a row's
// result does not depend on the sequence it is packed with.
__global__ void __launch_bounds__(1024) attention_units_kernel(const int32_t* __restrict__ offsets, int nseq, int cap,
                                                               uint8_t* __restrict__ buf) {
  int4* desc = reinterpret_cast<int4*>(buf);
  int32_t* sorted = reinterpret_cast<int32_t*>(buf + units_sorted_off(cap));
  int32_t* count = reinterpret_cast<int32_t*>(buf + units_count_off(cap));
  __shared__ int hist[MAXL + 1], next[MAXL + 1], totals[2];
  for (int i = threadIdx.x; i <= MAXL; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  for (int q = threadIdx.x; q < nseq; q += blockDim.x) {
    const int L = offsets[q + 1] - offsets[q];
    if (L >= 1 && L <= MAXL) atomicAdd(&hist[L], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int L = MAXL; L >= 1; L--) {
      next[L] = acc;
      acc += hist[L];
      if (L == PACK_MAX + 1) totals[0] = acc;
    }
    totals[1] = acc;
    *count = totals[0] + (acc - totals[0] + 1) / 2;
  }
  __syncthreads();
  for (int q = threadIdx.x; q < nseq; q += blockDim.x) {
    const int L = offsets[q + 1] - offsets[q];
    if (L >= 1 && L <= MAXL) sorted[atomicAdd(&next[L], 1)] = q;
  }
  __syncthreads();
  const int nlong = totals[0], nall = totals[1];
  const int ndesc = nlong + (nall - nlong + 1) / 2;
  for (int d = threadIdx.x; d < ndesc; d += blockDim.x) {
    const int j = d < nlong ? d : nlong + 2 * (d - nlong);
    const int a = sorted[j];
    int4 v = make_int4(offsets[a], offsets[a + 1] - offsets[a], 0, 0);
    if (d >= nlong && j + 1 < nall) {
      const int b = sorted[j + 1];
      v.z = offsets[b];
      v.w = offsets[b + 1] - offsets[b];
    }
    desc[d] = v;
  }
}

// A unit in flight as {t0A, LA | head << 8, t0B, LB} (LA = 0: none).
__device__ __forceinline__ int unit_la(int4 u) { return u.y & 0xFF; }
__device__ __forceinline__ int unit_head(int4 u) { return u.y >> 8; }
// S's N and P.V's K: every key column of the unit, rounded up to 16.
__device__ __forceinline__ int unit_np(int4 u) { return u.w > 0 ? 2 * PACK_MAX : (unit_la(u) + 15) & ~15; }

// OR of `v` over the 128 threads of named barrier `id` (all of them get
// the same answer), with the barrier's memory ordering.
__device__ __forceinline__ bool group_any(int id, bool v) {
  uint32_t r;
  asm volatile(
      "{\n.reg .pred p, q;\nsetp.ne.u32 q, %1, 0;\nbarrier.cta.red.or.pred p, %2, 128, q;\nselp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id)
      : "memory");
  return r != 0;
}

// Bounded wait for a phase without the abort check: the elected thread
// draining its own copies and MMAs before the CTA exits.
__device__ __forceinline__ void drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try(bar, parity))
    if (globaltimer_ns() - t0 > 10000000ull) break;  // 10 ms
}

// 128 registers per thread: 16 warps of 32 threads share the SM's 64K.
__global__ void __launch_bounds__(NTHREADS, 1)
    attention_stc_kernel(const __grid_constant__ CUtensorMap tmap, const int4* __restrict__ desc,
                         const int32_t* __restrict__ desc_count, int heads, int H, __half* __restrict__ out,
                         DevStatus* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = smem_u32(smem);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Lay::OFF_MISC);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Lay::OFF_MISC + 4);
  int* unit_ctr = reinterpret_cast<int*>(smem + Lay::OFF_MISC + 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = warp / GROUP_WARPS;
  // Next unit of the group, double-buffered by unit parity: written by the
  // elected thread while the group may still read the other entry.
  int4* unit_next = reinterpret_cast<int4*>(smem + Lay::OFF_UNITS) + 2 * grp;
  const uint32_t qk_full = sbase + Lay::OFF_BAR + 8 * (4 * grp), v_full = qk_full + 8, s_full = qk_full + 16,
                 o_full = qk_full + 24;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    *unit_ctr = 0;
    for (int b = 0; b < Lay::NBAR; b++) mbar_init(sbase + Lay::OFF_BAR + 8 * b, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int quarter = warp & 3;         // TMEM lanes 32*quarter .. +31
  const int row = quarter * 32 + lane;  // query row of the unit
  const bool elect = quarter == 0 && lane == 0;
  const int bar_id = 1 + grp;
  const uint32_t sq = sbase + grp * Lay::GSTRIDE, sk = sq + QKV_BYTES, sv = sk + QKV_BYTES;
  const uint32_t col = tmem + grp * MAXL;  // the group's slot
  const uint32_t slot = col + ((uint32_t)(quarter * 32) << 16);

  // The descriptor list was written before the previous kernel started (a
  // forward builds it before its first layer), so it is read before the
  // wait on the previous kernel.
  const long long nunits = (long long)__ldg(desc_count) * heads;
  auto unit_of = [&](long long u, int4 d) { return make_int4(d.x, d.y | ((int)(u % heads) << 8), d.z, d.w); };
  // Elected thread: the CTA's next unit.
  auto fetch = [&]() -> int4 {
    const long long u = blockIdx.x + (long long)atomicAdd(unit_ctr, 1) * gridDim.x;
    if (u >= nunits) return make_int4(0, 0, 0, 0);
    return unit_of(u, __ldg(desc + u / heads));
  };
  // The same in two steps, so that the descriptor load is in flight while
  // the group works: fetch_issue takes the counter and copies the
  // descriptor to shared memory (cp.async), fetch_resolve (a phase later)
  // waits for the copy.
  GroupState& gs = *reinterpret_cast<GroupState*>(smem + Lay::OFF_GS + 80 * grp);
  auto fetch_issue = [&]() {
    const long long u = blockIdx.x + (long long)atomicAdd(unit_ctr, 1) * gridDim.x;
    gs.pu = u;
    if (u < nunits)
      asm volatile("cp.async.ca.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(&gs.desc)), "l"(desc + u / heads)
                   : "memory");
  };
  auto fetch_resolve = [&]() -> int4 {
    const long long u = gs.pu;
    gs.pu = -1;
    if (u < 0 || u >= nunits) return make_int4(0, 0, 0, 0);
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    return unit_of(u, gs.desc);
  };
  // Rows 0..63 of Q, K and V from A's first token, rows 64..127 from B's
  // (packed) or A's 65th (K and V only when A has more than 64 tokens).
  auto nbox_of = [&](int4 un) { return un.w > 0 ? 2 : (unit_la(un) + BOX - 1) / BOX; };
  auto box1_of = [&](int4 un) { return un.w > 0 ? un.z : un.x + BOX; };
  auto load_qk = [&](int4 un) {
    const int nbox = nbox_of(un), c = unit_head(un) * HD, r1 = box1_of(un);
    mbar_expect_tx(qk_full, QKV_BYTES + nbox * BOX * HD * 2);
    tma_load_2d(sq, &tmap, c, un.x, qk_full);
    tma_load_2d(sq + BOX * 128, &tmap, c, r1, qk_full);
    tma_load_2d(sk, &tmap, H + c, un.x, qk_full);
    if (nbox > 1) tma_load_2d(sk + BOX * 128, &tmap, H + c, r1, qk_full);
  };
  auto load_v = [&](int4 un) {
    const int nbox = nbox_of(un), c = 2 * H + unit_head(un) * HD;
    mbar_expect_tx(v_full, nbox * BOX * HD * 2);
    tma_load_2d(sv, &tmap, c, un.x, v_full);
    if (nbox > 1) tma_load_2d(sv + BOX * 128, &tmap, c, box1_of(un), v_full);
  };
  // S = Q . K^T into the slot (N = the unit's keys rounded up to 16).
  auto issue_s = [&](int np) {
    const uint32_t idesc = idesc_f16(BQ, np);
#pragma unroll
    for (int kk = 0; kk < HD / 16; kk++)
      mma_f16(col, sw128_desc(sq + kk * 32), sw128_desc(sk + kk * 32), idesc, kk != 0);
    mma_commit(s_full);
  };
  // O = P.V, P read from the slot's TMEM (K = the unit's keys).
  auto issue_pv = [&](int np) {
    const uint32_t idesc = idesc_f16(BQ, HD) | (1u << 16);  // B (V) MN-major
    for (int kk = 0; kk < np / 16; kk++)
      mma_f16_ts(col + TM_O, col + kk * 8, sw128_desc(sv + kk * 2048), idesc, kk != 0);
    mma_commit(o_full);
  };

  bool bad = false;
  // The first units are taken before the wait on the previous kernel (which
  // wrote qkv).
  int4 u0 = make_int4(0, 0, 0, 0);
  if (elect) {
    gs.un = make_int4(0, 0, 0, 0);
    gs.pu = -1;
    gs.nq = gs.nqw = gs.nv = gs.nvw = gs.ns = gs.no = gs.sw = gs.ow = 0;
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap)) : "memory");
    u0 = fetch();
    unit_next[0] = u0;
    if (unit_la(u0) > 0) fetch_issue();
  }
  pdl_wait();  // qkv and the output buffer are the previous kernels'
  pdl_trigger();
  if (elect) {
    if (unit_la(u0) > 0) {
      load_qk(u0), gs.nq++;
      load_v(u0), gs.nv++;
      bad = !mbar_wait_sleep(qk_full, 0, abort_flag, status, 81);
      if (!bad) gs.nqw++, issue_s(unit_np(u0)), gs.ns++;
    }
  }
  bad = group_any(bar_id, bad);
  int4 cur = bad ? make_int4(0, 0, 0, 0) : unit_next[0];
  for (int k = 0; unit_la(cur) > 0; k++) {
    const int head = unit_head(cur), np = unit_np(cur);
    const bool packed = cur.w > 0;
    // This warp's rows: of B (rows 64..127 of a packed unit) or of A.
    const int rbase = packed && quarter >= 2 ? PACK_MAX : 0;
    const int t0 = rbase ? cur.z : cur.x, L = rbase ? cur.w : unit_la(cur);
    const uint32_t srow = slot + rbase;      // the row's keys in S
    const uint32_t prow = slot + rbase / 2;  // and their P pairs
    // A warp whose 32 rows are all past its sequence has nothing to do:
    // its rows of P and O are never stored (rows are independent in both
    // MMAs).
    const bool live = quarter * 32 - rbase < L;
    // (Only the elected thread can come here with `bad` set: a failed wait
    // after the last barrier.  Its warp then fails as a whole.)
    if (live || elect) {
      const bool w = !bad && mbar_wait(s_full, k & 1, abort_flag, status, 87);
      bad = !__all_sync(0xffffffffu, w);
      if (elect && !bad) gs.sw++;
    }
    tc_fence_after();
    if (elect && !bad) {
      // Q and K are read: the next unit's go to the same buffers.
      const int4 un = fetch_resolve();
      gs.un = un;
      unit_next[(k + 1) & 1] = un;
      if (unit_la(un) > 0) load_qk(un), gs.nq++;
    }
    float l = 0.f;
    if (live && !bad) {
      // Maximum of the raw scores of keys < L, 16 keys per TMEM load, the
      // next load in flight while one is reduced.
      const int n16 = (L + 15) >> 4;
      float m0 = -INFINITY, m1 = -INFINITY;
      {
        uint32_t ra[16], rb[16];
        tmem_ld16_nowait(srow, ra);
#pragma unroll
        for (int c = 0; c < MAXL / 16; c += 2) {
          if (c < n16) {
            tmem_wait_ld();
            if (c + 1 < n16) tmem_ld16_nowait(srow + (c + 1) * 16, rb);
            chunk_max<16>(m0, m1, ra, L - c * 16);
          }
          if (c + 1 < n16) {
            tmem_wait_ld();
            if (c + 2 < n16) tmem_ld16_nowait(srow + (c + 2) * 16, ra);
            chunk_max<16>(m0, m1, rb, L - (c + 1) * 16);
          }
        }
      }
      const float mx = fmaxf(m0, m1);
      // P, PK keys per TMEM load, over the scores already read: keys PK c ..
      // to columns PK/2 c .. (columns past the unit's N hold no scores of
      // it: masked, and P.V reads only the first N/2).
      const unsigned long long scale = f2_pack(SCALE2, SCALE2), off = f2_pack(-mx * SCALE2, -mx * SCALE2);
      unsigned long long s0 = f2_pack(0.f, 0.f), s1 = s0;
      const int nst = (L + PK - 1) / PK;
#pragma unroll 1
      for (int c = 0; c < nst; c++) {
        uint32_t r[PK], w[PK / 2];
        tmem_ld_nowait<PK>(srow + c * PK, r);
        tmem_wait_ld();
        chunk_p<PK>(r, L - c * PK, scale, off, s0, s1, w);
        tmem_st_half<PK>(prow + c * (PK / 2), w);
      }
      if (packed) {
        // P.V reads all 64 pair columns: zeros over the other sequence's
        // keys and over this one's past its last 16-key step (written after
        // the scores there have been read).
        const uint32_t z[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
#pragma unroll 1
        for (int c = 0; c < 2 * PACK_MAX / 16; c++) {
          const int c8 = c * 8;
          if (c8 < rbase / 2 || c8 >= rbase / 2 + nst * (PK / 2)) tmem_st8(slot + c8, z);
        }
      }
      float l0, l1;
      f2_unpack(f2_add(s0, s1), l0, l1);
      l = l0 + l1;
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    if (group_any(bar_id, bad)) break;  // P is written
    if (elect) {
      tc_fence_after();
      bad = !mbar_wait_sleep(v_full, k & 1, abort_flag, status, 84);
      if (!bad) gs.nvw++, issue_pv(np), gs.no++;
      if (unit_la(gs.un) > 0) fetch_issue();
    }
    if (live || elect) {
      const bool w = !bad && mbar_wait(o_full, k & 1, abort_flag, status, 88);
      bad = !__all_sync(0xffffffffu, w);
      if (elect && !bad) gs.ow++;
    }
    tc_fence_after();
    uint32_t o[64];
    if (live && !bad) {
      tmem_ld32_nowait(slot + TM_O, o);
      tmem_ld32_nowait(slot + TM_O + 32, o + 32);
      tmem_wait_ld();
    }
    tc_fence_before();
    if (group_any(bar_id, bad)) break;  // O is read: the slot is free
    cur = unit_next[(k + 1) & 1];
    if (elect && unit_la(cur) > 0) {
      // S of the next unit, overlapping this unit's stores, and its V (P.V
      // has read the V buffer: o_full).
      tc_fence_after();
      bad = !mbar_wait_sleep(qk_full, (k + 1) & 1, abort_flag, status, 81);
      if (!bad) gs.nqw++, issue_s(unit_np(cur)), gs.ns++;
      if (!bad) load_v(cur), gs.nv++;
    }
    if (live && !bad) {
      // O / l as fp16, straight from registers: each row's 128 bytes as
      // four 32-byte stores (whole sectors).  Rows past the sequence (l may
      // be 0 there) are not stored.
      const int rr = row - rbase;  // the row in its sequence
      if (rr < L) {
        const float inv = 1.0f / l;
        const unsigned long long inv2 = f2_pack(inv, inv);
        uint32_t* dst = reinterpret_cast<uint32_t*>(out + (long)(t0 + rr) * H + head * HD);
#pragma unroll
        for (int c = 0; c < 4; c++) {
          uint32_t h[8];
#pragma unroll
          for (int j = 0; j < 8; j++) {
            float a, b;
            f2_unpack(f2_mul(f2_pack(__uint_as_float(o[16 * c + 2 * j]), __uint_as_float(o[16 * c + 2 * j + 1])),
                             inv2),
                      a, b);
            h[j] = pack_half2(a, b);
          }
          asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst + 8 * c), "r"(h[0]),
                       "r"(h[1]), "r"(h[2]), "r"(h[3]), "r"(h[4]), "r"(h[5]), "r"(h[6]), "r"(h[7])
                       : "memory");
        }
      }
    }
  }
  // Copies and MMAs this group's elected thread issued but nobody waited
  // for (only after a failure) land before the CTA exits.
  if (elect) {
    if (gs.nq > gs.nqw) drain(qk_full, (gs.nq - 1) & 1);
    if (gs.nv > gs.nvw) drain(v_full, (gs.nv - 1) & 1);
    if (gs.ns > gs.sw) drain(s_full, (gs.ns - 1) & 1);
    if (gs.no > gs.ow) drain(o_full, (gs.no - 1) & 1);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
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

}  // namespace stc

size_t attention_units_bytes(int cap) { return stc::units_count_off(cap) + 16; }

cudaError_t launch_attention_units(const int32_t* offsets, int nseq, int cap, void* buf, cudaStream_t s) {
  if (nseq <= 0) return cudaSuccess;
  if (nseq > cap || !buf || (reinterpret_cast<uintptr_t>(buf) & 15)) return cudaErrorInvalidValue;
  stc::attention_units_kernel<<<1, 1024, 0, s>>>(offsets, nseq, cap, static_cast<uint8_t*>(buf));
  return cudaGetLastError();
}

cudaError_t launch_attention_stc(const __half* qkv, const void* units, int cap, int nseq, int T, int H, int heads,
                                 __half* out, DevStatus* status, cudaStream_t s) {
  if (nseq == 0 || T == 0) return cudaSuccess;
  if (H != heads * stc::HD || heads >= (1 << 22) || nseq > cap) return cudaErrorInvalidValue;
  auto enc = stc::encode_fn();
  if (!enc) return cudaErrorNotSupported;
  if ((3L * H * 2) % 16 || (reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(units) & 15))
    return cudaErrorInvalidValue;
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)(3 * H), (cuuint64_t)T};
  const cuuint64_t strides[1] = {(cuuint64_t)(3 * H) * 2};
  const cuuint32_t box[2] = {stc::HD, stc::BOX};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(qkv), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  static std::mutex mu;
  static int sms[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64) return cudaErrorInvalidDevice;
  {
    std::lock_guard<std::mutex> lk(mu);
    if (sms[dev] == 0) {
      cudaError_t e = cudaFuncSetAttribute(stc::attention_stc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           stc::Lay::ALLOC);
      if (e != cudaSuccess) return e;
      cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    }
  }
  // At most nseq * heads units (fewer when sequences are packed).
  const long nunits = (long)nseq * heads;
  const int grid = nunits < sms[dev] ? (int)nunits : sms[dev];
  const uint8_t* ub = static_cast<const uint8_t*>(units);
  cudaLaunchAttribute attr[1];
  const cudaLaunchConfig_t cfg = pdl_config(dim3(grid), dim3(stc::NTHREADS), stc::Lay::ALLOC, s, attr);
  return cudaLaunchKernelEx(&cfg, stc::attention_stc_kernel, map, reinterpret_cast<const int4*>(ub),
                            reinterpret_cast<const int32_t*>(ub + stc::units_count_off(cap)), heads, H, out, status);
}

}  // namespace le
