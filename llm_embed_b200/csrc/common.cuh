// Shared device-side definitions for libllmembed_cuda (sm_100a only).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libllmembed_cuda targets sm_100a only"
#endif

namespace le {

// Programmatic dependent launch.  Kernels of the forward pass are launched
// with programmatic stream serialization (pdl_config) so that a kernel's
// CTAs can be placed on SMs its predecessor has left while the predecessor
// finishes.  Every such kernel calls pdl_wait() in every thread before its
// first global memory access (it returns once the preceding kernel has
// completed and its writes are visible; without the launch attribute it
// returns at once), then pdl_trigger(), which lets the next kernel be
// scheduled once all CTAs of this one have issued it.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch configuration with the programmatic stream serialization attribute
// (attr must outlive the launch call).
inline cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, size_t smem, cudaStream_t s, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// GGML tensor type ids (reference internal/gguf/reader.go:46-65).
enum GgmlType : int { T_F32 = 0, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14 };

// ---------------------------------------------------------------------------
// Repacked ("tile-blocked") weight format, built on the device at load time.
//
// A weight W[N][K] (GGUF dims [K, N], row n = output feature n) is cut into
// tiles of TILE_N=128 rows x TILE_K=64 columns.  Each tile is one contiguous,
// 16-byte aligned chunk, chunks ordered [n_tile][k_step]:
//   [0, 8192)             u8  q[128][64]   q + 128 of the signed integer
//                                          multiplier of every element
//   [8192, +META_BYTES)   per-row dequant metadata for the 64 columns:
//       Q8_0:       half  d[128][2]                   (one per 32-block)
//       Q4_K, Q5_K: float {d*sc, dmin*m}[128][2]      (one pair per 32-block)
//       Q6_K:       float d*sc[128][4]                (one per 16-block)
// The float products are formed exactly as the reference does
// (quant_q4k.go:54-60, quant_q5k.go:202-208, quant_q6k.go:362-365), so a
// device dequant from this layout is bit-identical to the reference's.
// Rows past N are zero (q=0, scales 0).
// ---------------------------------------------------------------------------
constexpr int TILE_N = 128;
constexpr int TILE_K = 64;
constexpr int TILE_Q_BYTES = TILE_N * TILE_K;  // 8192

enum QFmt : int { QF_Q8_0 = 0, QF_KMIN = 1, QF_Q6K = 2 };
// F32 GGUF weights have no tile-blocked copy: they are held only as the fp16
// operand matrix (and their exact float32 rows for le_dequant), and every
// GEMM on them runs the fp16-operand tensor-core kernel.
constexpr int QF_F16 = 3;

__host__ __device__ constexpr int qfmt_of(int ggml_type) {
  return ggml_type == T_Q8_0 ? QF_Q8_0 : (ggml_type == T_Q6_K ? QF_Q6K : QF_KMIN);
}
__host__ __device__ constexpr int meta_bytes(int qfmt) { return qfmt == QF_Q8_0 ? TILE_N * 4 : TILE_N * 16; }
__host__ __device__ constexpr int chunk_bytes(int qfmt) { return TILE_Q_BYTES + meta_bytes(qfmt); }

// ---------------------------------------------------------------------------
// Error reporting from kernels: the first failing kernel writes a code and a
// location into a per-device status word that the host reads after each call.
// ---------------------------------------------------------------------------
enum DevErr : int { DE_OK = 0, DE_TIMEOUT = 1, DE_BOUNDS = 2, DE_TMEM = 3 };

struct DevStatus {
  int code;
  int where;
  int info;
  int pad;
};

__device__ __forceinline__ void report(DevStatus* st, int code, int where, int info) {
  if (st && atomicCAS(&st->code, 0, code) == 0) {
    st->where = where;
    st->info = info;
  }
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait limit for every spin in this library (mbarrier waits).
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;  // 2 s

// ---------------------------------------------------------------------------
// fp16 helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace le
