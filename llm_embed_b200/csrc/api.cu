// Host implementation of the C ABI declared in include/llmembed.h.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/llmembed.h"
#include "common.cuh"
#include "gemm.h"
#include "kernels.h"

using namespace le;

// ------------------------------------------------------------- errors -----

static thread_local std::string g_err;

static int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

// The same for the library's other host sources (tokenizer.cpp).
int le_fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

#define CK(call)                                                                                 \
  do {                                                                                           \
    cudaError_t e_ = (call);                                                                     \
    if (e_ != cudaSuccess) return fail(LE_ECUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                                       __FILE__, __LINE__);                                      \
  } while (0)

#define TRY(call)              \
  do {                         \
    int r_ = (call);           \
    if (r_ != LE_OK) return r_; \
  } while (0)

// ------------------------------------------------------------ helpers -----

static long row_bytes_of(int type, long k) {
  switch (type) {
    case T_F32: return k * 4;
    case T_Q8_0: return k % 32 ? -1 : k / 32 * 34;
    case T_Q4_K: return k % 256 ? -1 : k / 256 * 144;
    case T_Q5_K: return k % 256 ? -1 : k / 256 * 176;
    case T_Q6_K: return k % 256 ? -1 : k / 256 * 210;
    default: return -1;
  }
}

// Projection weight types as DequantWeightMatrix reads them (gemm.go:224-263):
// ids 15 and 16 share the Q5_K case there, so they decode as Q5_K here.
static int weight_type(int type) { return (type == 15 || type == 16) ? T_Q5_K : type; }

static bool is_quant(int type) { return type == T_Q8_0 || type == T_Q4_K || type == T_Q5_K || type == T_Q6_K; }

namespace {

struct DevBuf {
  void* p = nullptr;
  size_t n = 0;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
  int ensure(size_t bytes) {
    if (bytes <= n) return LE_OK;
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
      cudaGetLastError();
      return fail(LE_ENOMEM, "cudaMalloc(%zu) failed", bytes);
    }
    n = bytes;
    return LE_OK;
  }
  template <class T>
  T* as() const {
    return reinterpret_cast<T*>(p);
  }
};

struct HostBuf {
  void* p = nullptr;
  size_t n = 0;
  ~HostBuf() {
    if (p) cudaFreeHost(p);
  }
  int ensure(size_t bytes) {
    if (bytes <= n) return LE_OK;
    if (p) cudaFreeHost(p);
    p = nullptr;
    n = 0;
    if (cudaMallocHost(&p, bytes) != cudaSuccess) {
      cudaGetLastError();
      return fail(LE_ENOMEM, "cudaMallocHost(%zu) failed", bytes);
    }
    n = bytes;
    return LE_OK;
  }
  template <class T>
  T* as() const {
    return reinterpret_cast<T*>(p);
  }
};

// A repacked projection weight.
struct QMat {
  DevBuf buf;      // tile-blocked quantised weight (common.cuh)
  DevBuf r16;      // the same bytes in 16-row tiles (gemm_r16.cuh) for few tokens
  int r16_tiles = 0;
  DevBuf w16;      // its fp16 operand values [n_virt][K] for the large-batch GEMM
  int type = 0;   // GGML type
  int qf = 0;     // QFmt
  int n_real = 0;  // real output rows
  int n_virt = 0;  // rows in tile layout (multiple of TILE_N)
  int K = 0;
  bool interleaved = false;  // merged ffn_up / ffn_gate
};

struct Layer {
  QMat qkv, out, upgate, down;
  DevBuf attn_w, attn_b, out_w, out_b;
};

struct Workspace {
  int cap_tokens = 0, cap_seqs = 0;
  DevBuf ids, offsets, pos, h32, y32, hA, qkv, att, ff, out;
  DevBuf att_units;  // the short-sequence attention's work list
  DevBuf ln_part, ln_ctl;  // row statistics of the fused projection + LayerNorm
  HostBuf h_ids, h_offsets, h_out;
};

constexpr int CHUNK_TOKENS = LE_MAX_DEVICE_TOKENS;

// Wall-clock phases of one model load (le_model_load_stats).
struct LoadTimes {
  double upload_ms = 0, repack_ms = 0, expand_ms = 0;
  int64_t h2d_bytes = 0;
};
static double now_ms() {
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

}  // namespace

// CUDA-event timing of each kernel launch, by kernel class.
struct Profiler {
  bool on = false;
  int64_t launches = 0;
  std::vector<cudaEvent_t> pool;
  size_t used = 0;
  std::vector<std::pair<int, size_t>> pending;  // (class, index of start event)
  int64_t count[LE_NCLASS] = {};
  double ms[LE_NCLASS] = {};
  ~Profiler() {
    for (auto e : pool) cudaEventDestroy(e);
  }
  cudaEvent_t next() {
    if (used == pool.size()) {
      cudaEvent_t e = nullptr;
      cudaEventCreate(&e);
      pool.push_back(e);
    }
    return pool[used++];
  }
  void begin(int cls, cudaStream_t s) {
    launches++;
    if (!on) return;
    pending.push_back({cls, used});
    cudaEventRecord(next(), s);
  }
  void end(cudaStream_t s) {
    if (on) cudaEventRecord(next(), s);
  }
  int collect() {
    for (auto& p : pending) {
      float t = 0.f;
      if (cudaEventElapsedTime(&t, pool[p.second], pool[p.second + 1]) != cudaSuccess)
        return fail(LE_ECUDA, "cudaEventElapsedTime failed");
      ms[p.first] += t;
      count[p.first]++;
    }
    pending.clear();
    used = 0;
    return LE_OK;
  }
};

// An instantiated CUDA graph of forward() for one call shape.  Kernel
// parameters hold the caller's id/offset/output pointers and the workspace
// buffers, so those are part of the key; workspace growth drops all graphs.
struct GraphEntry {
  int T = 0, nseq = 0, max_len = 0, out_dim = 0;
  const void* ids = nullptr;
  const void* offsets = nullptr;
  void* out = nullptr;
  cudaGraphExec_t exec = nullptr;
  uint64_t last_use = 0;
};

// Calls of at most this many tokens replay a cached graph of the forward
// pass (launch overhead dominates them); larger ones launch directly.
constexpr int GRAPH_MAX_TOKENS = 4096;
constexpr size_t GRAPH_CACHE = 32;

struct le_model {
  int dev = 0;
  Profiler prof;
  le_hparams hp{};
  int head_dim = 0;
  int emb_type = 0;
  long emb_row_bytes = 0;
  int vocab = 0;
  DevBuf emb, type0, embd_w, embd_b, rope_cos, rope_sin, status;
  DevBuf barrier;  // hand-off counters of the single-kernel small forward
  int sms = 0;
  std::vector<Layer> layers;
  cudaStream_t stream = nullptr;
  cudaStream_t capture_stream = nullptr;  // graphs are captured here, replayed on the caller's stream
  std::vector<GraphEntry> graphs;
  uint64_t graph_clock = 0;
  std::mutex mu;
  Workspace ws;
  // Completion of the last forward enqueued on the workspace (any stream).
  cudaEvent_t ws_done = nullptr;
  bool ws_used = false;
  LoadTimes load;
  double parse_ms = 0, load_ms = 0;
  void drop_graphs() {
    for (auto& g : graphs)
      if (g.exec) cudaGraphExecDestroy(g.exec);
    graphs.clear();
  }
  ~le_model() {
    drop_graphs();
    if (ws_done) cudaEventDestroy(ws_done);
    if (capture_stream) cudaStreamDestroy(capture_stream);
    if (stream) cudaStreamDestroy(stream);
  }
};

struct le_qweight {
  int dev = 0;
  QMat w;
  DevBuf x16, status;
  cudaStream_t stream = nullptr;
  std::mutex mu;
  ~le_qweight() {
    if (stream) cudaStreamDestroy(stream);
  }
};

// --------------------------------------------------------- device status --

static int check_status(DevBuf& status, cudaStream_t s) {
  DevStatus st{};
  CK(cudaMemcpyAsync(&st, status.p, sizeof st, cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  if (st.code != DE_OK) {
    cudaMemsetAsync(status.p, 0, sizeof(DevStatus), s);
    return fail(LE_EDEVICE, "kernel failure code %d at site %d (info %d)", st.code, st.where, st.info);
  }
  return LE_OK;
}

// ---------------------------------------------------------- weights -------

// Upload raw GGUF rows of one or two source tensors and repack them into the
// tile layout (interleave: merged ffn_up/ffn_gate).  F32 weights (accepted
// when allow_f32) keep their exact rows in `buf` and get only the fp16
// operand matrix.
static int make_qmat(QMat& q, int type, const void* src0, const void* src1, int N, int K, bool interleave,
                     cudaStream_t s, bool allow_f32 = false, LoadTimes* lt = nullptr) {
  LoadTimes scratch;
  if (!lt) lt = &scratch;
  const bool f32 = type == T_F32 && allow_f32;
  if (!is_quant(type) && !f32)
    return fail(LE_EINVAL, "unsupported weight type %d (F32/Q8_0/Q4_K/Q5_K/Q6_K only)", type);
  const long rb = row_bytes_of(type, K);
  if (rb < 0 || K % TILE_K) return fail(LE_EINVAL, "K=%d is not a multiple of the block size of type %d", K, type);
  if (N <= 0 || N % 2) return fail(LE_EINVAL, "N=%d must be positive and even", N);
  q.type = type;
  q.qf = f32 ? QF_F16 : qfmt_of(type);
  q.K = K;
  q.n_real = interleave ? 2 * N : N;
  int n_tiles = interleave ? (N + TILE_N / 2 - 1) / (TILE_N / 2) : (N + TILE_N - 1) / TILE_N;
  n_tiles += n_tiles & 1;  // even: the CTA-pair GEMM takes weight tiles two at a time
  q.n_virt = n_tiles * TILE_N;
  q.interleaved = interleave;
  const size_t nb = (size_t)N * rb;
  double t0 = now_ms();
  lt->h2d_bytes += (int64_t)(nb * (interleave ? 2 : 1));
  if (f32) {
    TRY(q.buf.ensure(nb * (interleave ? 2 : 1)));
    CK(cudaMemcpyAsync(q.buf.p, src0, nb, cudaMemcpyHostToDevice, s));
    if (interleave) CK(cudaMemcpyAsync(q.buf.as<uint8_t>() + nb, src1, nb, cudaMemcpyHostToDevice, s));
    CK(cudaStreamSynchronize(s));
    lt->upload_ms += now_ms() - t0;
    t0 = now_ms();
    TRY(q.w16.ensure((size_t)q.n_virt * K * 2));
    CK(launch_f32_rows_to_f16(q.buf.as<float>(), interleave ? q.buf.as<float>() + (size_t)N * K : nullptr, N, K,
                              q.n_virt, interleave ? 1 : 0, q.w16.as<__half>(), s));
    CK(cudaStreamSynchronize(s));
    lt->expand_ms += now_ms() - t0;
    return LE_OK;
  }
  TRY(q.buf.ensure((size_t)n_tiles * (K / TILE_K) * chunk_bytes(q.qf)));
  DevBuf raw;
  TRY(raw.ensure(nb * (interleave ? 2 : 1)));
  CK(cudaMemcpyAsync(raw.p, src0, nb, cudaMemcpyHostToDevice, s));
  if (interleave) CK(cudaMemcpyAsync(raw.as<uint8_t>() + nb, src1, nb, cudaMemcpyHostToDevice, s));
  CK(cudaStreamSynchronize(s));
  lt->upload_ms += now_ms() - t0;
  t0 = now_ms();
  CK(launch_repack(type, raw.as<uint8_t>(), interleave ? raw.as<uint8_t>() + nb : nullptr, rb, N, K, n_tiles,
                   interleave ? 1 : 0, q.buf.as<uint8_t>(), s));
  CK(cudaStreamSynchronize(s));
  lt->repack_ms += now_ms() - t0;
  t0 = now_ms();
  TRY(q.w16.ensure((size_t)q.n_virt * K * 2));
  CK(launch_expand_f16(q.qf, q.buf.as<uint8_t>(), q.n_virt, K, q.w16.as<__half>(), s));
  CK(cudaStreamSynchronize(s));
  lt->expand_ms += now_ms() - t0;
  t0 = now_ms();
  q.r16_tiles = interleave ? (N + 7) / 8 : (N + 15) / 16;
  TRY(q.r16.ensure((size_t)q.r16_tiles * (K / TILE_K) * (1024 + 16 * (q.qf == QF_Q8_0 ? 4 : 16))));
  CK(launch_repack_r16(q.qf, q.buf.as<uint8_t>(), K, interleave ? 1 : 0, q.r16_tiles, q.r16.as<uint8_t>(), s));
  CK(cudaStreamSynchronize(s));
  lt->repack_ms += now_ms() - t0;
  return LE_OK;
}

// The layouts of a weight as the GEMM dispatch takes them (n_rows: the rows
// the GEMM covers).
static GemmW gemm_w(const QMat& q, int n_rows) {
  return GemmW{q.qf, q.buf.as<uint8_t>(), q.r16.as<uint8_t>(), q.w16.as<__half>(), n_rows, q.r16_tiles, q.K};
}

static int upload_f32(DevBuf& b, const le_tensor_desc* t, int n, cudaStream_t s) {
  if (t->type != T_F32) return fail(LE_EINVAL, "tensor %s must be F32 (type %d)", t->name, t->type);
  if (t->n_bytes < (int64_t)n * 4) return fail(LE_EINVAL, "tensor %s too short", t->name);
  TRY(b.ensure((size_t)n * 4));
  CK(cudaMemcpyAsync(b.p, t->data, (size_t)n * 4, cudaMemcpyHostToDevice, s));
  return LE_OK;
}

// ---------------------------------------------------------- workspace -----

static int ensure_ws(le_model* m, int tokens, int seqs) {
  Workspace& w = m->ws;
  const int H = m->hp.hidden, F = m->hp.ffn;
  if (tokens > w.cap_tokens || seqs > w.cap_seqs) {
    m->drop_graphs();  // they point at the old buffers
    // A forward still running on another stream may use the old buffers.
    if (m->ws_used) CK(cudaEventSynchronize(m->ws_done));
  }
  if (tokens > w.cap_tokens) {
    const size_t T = (size_t)std::max(tokens, 256);
    TRY(w.ids.ensure(T * 4));
    TRY(w.pos.ensure(T * 4));
    TRY(w.h32.ensure(T * H * 4));
    TRY(w.y32.ensure(T * H * 4));
    TRY(w.hA.ensure(T * H * 2));
    TRY(w.qkv.ensure(T * 3 * H * 2));
    TRY(w.att.ensure(T * H * 2));
    TRY(w.ff.ensure(T * F * 2));
    TRY(w.h_ids.ensure(T * 4));
    TRY(w.ln_part.ensure(gemm_ln_part_bytes((int)T)));
    TRY(w.ln_ctl.ensure(16));
    CK(cudaMemsetAsync(w.ln_part.p, 0xFF, gemm_ln_part_bytes((int)T), m->stream));
    CK(cudaMemsetAsync(w.ln_ctl.p, 0, 16, m->stream));
    CK(cudaStreamSynchronize(m->stream));  // before forward() on any stream
    w.cap_tokens = (int)T;
  }
  if (seqs > w.cap_seqs) {
    const size_t S = (size_t)std::max(seqs, 64);
    TRY(w.offsets.ensure((S + 1) * 4));
    TRY(w.att_units.ensure(attention_units_bytes((int)S)));
    TRY(w.out.ensure(S * H * 4));
    TRY(w.h_offsets.ensure((S + 1) * 4));
    TRY(w.h_out.ensure(S * H * 4));
    w.cap_seqs = (int)S;
  }
  return LE_OK;
}

// check_status of a model; after a device error the fused LayerNorm's
// statistics words may be left filled, so they return to the empty marker.
static int model_status(le_model* m, cudaStream_t s) {
  const int rc = check_status(m->status, s);
  if (rc != LE_OK && m->ws.cap_tokens > 0) {
    cudaMemsetAsync(m->ws.ln_part.p, 0xFF, gemm_ln_part_bytes(m->ws.cap_tokens), s);
    cudaMemsetAsync(m->ws.ln_ctl.p, 0, 16, s);
    cudaStreamSynchronize(s);
  }
  return rc;
}

// ---------------------------------------------------------- forward -------

// Every forward of a model uses its one workspace (activations, the fused
// LayerNorm's statistics words), so forwards enqueued on different streams
// must not overlap on the GPU: each waits for the completion event of the
// previous one before its first kernel and records its own after its last.
// Under stream capture (the caller's graph) the caller orders the replays.
static int ws_order_begin(le_model* m, cudaStream_t s, bool* capturing) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  CK(cudaStreamIsCapturing(s, &cs));
  *capturing = cs != cudaStreamCaptureStatusNone;
  if (!*capturing && m->ws_used) CK(cudaStreamWaitEvent(s, m->ws_done, 0));
  return LE_OK;
}
static int ws_order_end(le_model* m, cudaStream_t s, bool capturing) {
  if (capturing) return LE_OK;
  CK(cudaEventRecord(m->ws_done, s));
  m->ws_used = true;
  return LE_OK;
}

static int gemm(le_model* m, int cls, const QMat& W, const __half* A, int lda, const EpiParams& ep, cudaStream_t s) {
  m->prof.begin(cls, s);
  CK(launch_gemm(gemm_w(W, W.n_virt), A, lda, ep, m->status.as<DevStatus>(), s));
  m->prof.end(s);
  return LE_OK;
}

// Launch one non-GEMM kernel under the profiler.
#define PLAUNCH(cls, call)  \
  do {                      \
    m->prof.begin(cls, s);  \
    CK(call);               \
    m->prof.end(s);         \
  } while (0)

// bert.go:216-285 (Forward) for packed sequences + pool.go (MeanPool,
// L2Normalize) + embedder.go:66-68 (truncation), all enqueued on `s`.
static int forward(le_model* m, const int32_t* d_ids, const int32_t* d_offsets, int nseq, int T, int max_len,
                   int out_dim, float* d_out, cudaStream_t s) {
  const int H = m->hp.hidden, F = m->hp.ffn;
  Workspace& w = m->ws;
  float* h32 = w.h32.as<float>();
  float* y32 = w.y32.as<float>();
  __half* hA = w.hA.as<__half>();
  __half* qkv = w.qkv.as<__half>();
  __half* att = w.att.as<__half>();
  __half* ff = w.ff.as<__half>();
  int32_t* pos = w.pos.as<int32_t>();
  unsigned long long* ln_part = w.ln_part.as<unsigned long long>();
  unsigned* ln_ctl = w.ln_ctl.as<unsigned>();
  const int ln_rows = gemm_ln_part_rows(w.cap_tokens);
  if (T > 0 && T <= SMALL_MAX_TOKENS && (int)m->layers.size() <= SMALL_MAX_LAYERS) {
    // A few tokens: the whole encoder and the pool in one cooperative kernel.
    SmallParams sp{};
    sp.T = T;
    sp.nseq = nseq;
    sp.n_layers = (int)m->layers.size();
    sp.ids = d_ids;
    sp.offsets = d_offsets;
    sp.emb_type = m->emb_type;
    sp.emb = m->emb.as<uint8_t>();
    sp.emb_row_bytes = m->emb_row_bytes;
    sp.vocab = m->vocab;
    sp.type0 = m->type0.as<float>();
    sp.embd_w = m->embd_w.as<float>();
    sp.embd_b = m->embd_b.as<float>();
    sp.eps = m->hp.ln_eps;
    sp.rope_cos = m->rope_cos.as<float>();
    sp.rope_sin = m->rope_sin.as<float>();
    sp.pos = pos;
    sp.qkv = qkv;
    sp.att = att;
    sp.y1 = y32;
    sp.y2 = y32 + (size_t)SMALL_MAX_TOKENS * H;
    sp.ff = ff;
    sp.out = d_out;
    sp.out_dim = out_dim;
    sp.sync = m->barrier.as<unsigned>();
    sp.status = m->status.as<DevStatus>();
    for (int l = 0; l < sp.n_layers; l++) {
      const Layer& L = m->layers[l];
      const QMat* q[4] = {&L.qkv, &L.out, &L.upgate, &L.down};
      const int modes[4] = {EPI_QKV, EPI_F32, EPI_GEGLU, EPI_F32};
      for (int i = 0; i < 4; i++)
        sp.layers[l].g[i] = SmallGemm{q[i]->qf == QF_F16 ? nullptr : q[i]->r16.as<uint8_t>(), q[i]->qf, q[i]->K,
                                      q[i]->r16_tiles, modes[i]};
      sp.layers[l].attn_w = L.attn_w.as<float>();
      sp.layers[l].attn_b = L.attn_b.as<float>();
      sp.layers[l].out_w = L.out_w.as<float>();
      sp.layers[l].out_b = L.out_b.as<float>();
    }
    if (small_forward_supported(sp, H, F, m->hp.heads, m->sms)) {
      PLAUNCH(8, launch_forward_small(sp, s));
      return LE_OK;
    }
  }
  if (T > 0) {
    PLAUNCH(7, launch_positions(d_offsets, nseq, pos, s));
    PLAUNCH(6, launch_embed_ln(d_ids, m->emb_type, m->emb.as<uint8_t>(), m->emb_row_bytes, m->vocab,
                               m->type0.as<float>(), m->embd_w.as<float>(), m->embd_b.as<float>(), m->hp.ln_eps, T,
                               H, h32, hA, m->status.as<DevStatus>(), s));
    // Large batches: the out and down projections carry the residual add
    // and LayerNorm in their epilogue (same bits as GEMM + launch_ln_add).
    const bool fuse_ln = T >= TC_F16_MIN_M && gemm_ln_supported(H, H) && gemm_ln_supported(H, F);
    // Batches whose GEMMs run on tensor cores also run the short
    // sequences' attention on them (its work list built here, once); small
    // batches keep the mma.sync tile (the same bits as the single-kernel
    // forward).
    const bool att_tc = T >= TC_MIN_M && m->head_dim == 64;
    if (att_tc) PLAUNCH(7, launch_attention_units(d_offsets, nseq, w.cap_seqs, w.att_units.p, s));
    for (const Layer& L : m->layers) {
      EpiParams e{};
      e.M = T;
      e.mode = EPI_QKV;
      e.N = 3 * H;
      e.out16 = qkv;
      e.ldo = 3 * H;
      e.pos = pos;
      e.rope_cos = m->rope_cos.as<float>();
      e.rope_sin = m->rope_sin.as<float>();
      e.head_dim = m->head_dim;
      e.rope_cols = 2 * H;
      TRY(gemm(m, 0, L.qkv, hA, H, e, s));
      if (att_tc)
        PLAUNCH(4, launch_attention_stc(qkv, w.att_units.p, w.cap_seqs, nseq, T, H, m->hp.heads, att,
                                        m->status.as<DevStatus>(), s));
      else
        PLAUNCH(4, launch_attention(qkv, d_offsets, nseq, max_len, H, m->hp.heads, m->head_dim, att, s));
      if (max_len > ATTN_SHORT_MAX)
        PLAUNCH(4, launch_attention_tc(qkv, d_offsets, nseq, T, max_len, ATTN_SHORT_MAX + 1, H, m->hp.heads, att,
                                       m->status.as<DevStatus>(), s));
      EpiParams r{};
      r.M = T;
      r.mode = EPI_F32;
      r.N = H;
      r.out32 = y32;
      r.ldo = H;
      if (fuse_ln) {
        PLAUNCH(1, launch_gemm_ln(L.out.w16.as<__half>(), H, att, H, T, h32, hA, L.attn_w.as<float>(),
                                  L.attn_b.as<float>(), m->hp.ln_eps, ln_part, ln_rows, ln_ctl, m->status.as<DevStatus>(), s));
      } else {
        TRY(gemm(m, 1, L.out, att, H, r, s));
        PLAUNCH(5,
                launch_ln_add(h32, y32, L.attn_w.as<float>(), L.attn_b.as<float>(), m->hp.ln_eps, T, H, h32, hA, s));
      }
      EpiParams g{};
      g.M = T;
      g.mode = EPI_GEGLU;
      g.N = F;
      g.out16 = ff;
      g.ldo = F;
      TRY(gemm(m, 2, L.upgate, hA, H, g, s));
      if (fuse_ln) {
        PLAUNCH(3, launch_gemm_ln(L.down.w16.as<__half>(), F, ff, F, T, h32, hA, L.out_w.as<float>(),
                                  L.out_b.as<float>(), m->hp.ln_eps, ln_part, ln_rows, ln_ctl, m->status.as<DevStatus>(), s));
      } else {
        TRY(gemm(m, 3, L.down, ff, F, r, s));
        PLAUNCH(5, launch_ln_add(h32, y32, L.out_w.as<float>(), L.out_b.as<float>(), m->hp.ln_eps, T, H, h32, hA, s));
      }
    }
  }
  PLAUNCH(7, launch_pool(h32, d_offsets, nseq, H, out_dim, d_out, s));
  return LE_OK;
}

// forward() through the graph cache: a call shape seen before replays its
// graph with one launch; a new small shape runs directly and is captured
// (on the model's capture stream, which executes nothing) for next time.
static int run_forward(le_model* m, const int32_t* d_ids, const int32_t* d_offsets, int nseq, int T, int max_len,
                       int out_dim, float* d_out, cudaStream_t s) {
  if (m->prof.on || T <= 0 || T > GRAPH_MAX_TOKENS)
    return forward(m, d_ids, d_offsets, nseq, T, max_len, out_dim, d_out, s);
  for (auto& g : m->graphs)
    if (g.T == T && g.nseq == nseq && g.max_len == max_len && g.out_dim == out_dim && g.ids == d_ids &&
        g.offsets == d_offsets && g.out == d_out) {
      g.last_use = ++m->graph_clock;
      CK(cudaGraphLaunch(g.exec, s));
      return LE_OK;
    }
  TRY(forward(m, d_ids, d_offsets, nseq, T, max_len, out_dim, d_out, s));
  cudaGraph_t graph = nullptr;
  CK(cudaStreamBeginCapture(m->capture_stream, cudaStreamCaptureModeThreadLocal));
  const int rc = forward(m, d_ids, d_offsets, nseq, T, max_len, out_dim, d_out, m->capture_stream);
  const cudaError_t ce = cudaStreamEndCapture(m->capture_stream, &graph);
  if (rc != LE_OK || ce != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    return rc != LE_OK ? rc : LE_OK;  // the direct run above produced the result
  }
  GraphEntry e;
  const cudaError_t ie = cudaGraphInstantiate(&e.exec, graph, 0);
  cudaGraphDestroy(graph);
  if (ie != cudaSuccess) {
    cudaGetLastError();
    return LE_OK;
  }
  if (m->graphs.size() >= GRAPH_CACHE) {
    auto lru = std::min_element(m->graphs.begin(), m->graphs.end(),
                                [](const GraphEntry& a, const GraphEntry& b) { return a.last_use < b.last_use; });
    cudaGraphExecDestroy(lru->exec);
    m->graphs.erase(lru);
  }
  e.T = T;
  e.nseq = nseq;
  e.max_len = max_len;
  e.out_dim = out_dim;
  e.ids = d_ids;
  e.offsets = d_offsets;
  e.out = d_out;
  e.last_use = ++m->graph_clock;
  m->graphs.push_back(e);
  return LE_OK;
}

// One device's share: chunks of whole sequences of at most CHUNK_TOKENS.
static int embed_host(le_model* m, const int32_t* ids, const int32_t* offs, int nseq, int out_dim, float* out) {
  std::lock_guard<std::mutex> lk(m->mu);
  if (cudaSetDevice(m->dev) != cudaSuccess) return fail(LE_ECUDA, "cudaSetDevice(%d) failed", m->dev);
  cudaStream_t s = m->stream;
  int s0 = 0;
  while (s0 < nseq) {
    int s1 = s0 + 1, maxlen = offs[s0 + 1] - offs[s0];
    while (s1 < nseq && offs[s1 + 1] - offs[s0] <= CHUNK_TOKENS) {
      maxlen = std::max(maxlen, offs[s1 + 1] - offs[s1]);
      s1++;
    }
    const int n = s1 - s0, T = offs[s1] - offs[s0];
    TRY(ensure_ws(m, T, n));
    Workspace& w = m->ws;
    int32_t* hi = w.h_ids.as<int32_t>();
    int32_t* ho = w.h_offsets.as<int32_t>();
    std::memcpy(hi, ids + offs[s0], (size_t)T * 4);
    for (int i = 0; i <= n; i++) ho[i] = offs[s0 + i] - offs[s0];
    bool cap = false;
    TRY(ws_order_begin(m, s, &cap));
    CK(cudaMemcpyAsync(w.ids.p, hi, (size_t)T * 4, cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(w.offsets.p, ho, (size_t)(n + 1) * 4, cudaMemcpyHostToDevice, s));
    TRY(run_forward(m, w.ids.as<int32_t>(), w.offsets.as<int32_t>(), n, T, maxlen, out_dim, w.out.as<float>(), s));
    CK(cudaMemcpyAsync(w.h_out.p, w.out.p, (size_t)n * out_dim * 4, cudaMemcpyDeviceToHost, s));
    TRY(ws_order_end(m, s, cap));
    TRY(model_status(m, s));
    std::memcpy(out + (size_t)s0 * out_dim, w.h_out.p, (size_t)n * out_dim * 4);
    s0 = s1;
  }
  return LE_OK;
}

// ---------------------------------------------------------- GGUF ----------

namespace {

struct Mapped {
  void* p = MAP_FAILED;
  size_t n = 0;
  ~Mapped() {
    if (p != MAP_FAILED) munmap(p, n);
  }
};

struct GgufParsed {
  std::vector<std::string> names;
  std::vector<le_tensor_desc> tensors;
  std::map<std::string, uint32_t> u32;
  std::map<std::string, float> f32;
};

struct Cur {
  const uint8_t* p;
  size_t n, pos;
  bool ok = true;
  template <class T>
  T get() {
    T v{};
    if (!ok || pos + sizeof(T) > n) {
      ok = false;
      return v;
    }
    std::memcpy(&v, p + pos, sizeof(T));
    pos += sizeof(T);
    return v;
  }
  std::string str() {
    uint64_t len = get<uint64_t>();
    if (!ok || pos + len > n) {
      ok = false;
      return {};
    }
    std::string s((const char*)p + pos, len);
    pos += len;
    return s;
  }
};

// Value skipping / capture as internal/gguf/reader.go:390-433; only exact
// uint32 and float32 scalars are kept (reader.go:293-332).
bool gguf_value(Cur& c, uint32_t vt, GgufParsed& g, const std::string* key, int depth) {
  if (depth > 4) return false;
  switch (vt) {
    case 0: case 1: case 7: c.get<uint8_t>(); break;
    case 2: case 3: c.get<uint16_t>(); break;
    case 4: { uint32_t v = c.get<uint32_t>(); if (key) g.u32[*key] = v; break; }
    case 5: c.get<int32_t>(); break;
    case 6: { float v = c.get<float>(); if (key) g.f32[*key] = v; break; }
    case 8: c.str(); break;
    case 9: {
      uint32_t et = c.get<uint32_t>();
      uint64_t len = c.get<uint64_t>();
      if (!c.ok || len > c.n) return false;
      for (uint64_t i = 0; i < len && c.ok; i++)
        if (!gguf_value(c, et, g, nullptr, depth + 1)) return false;
      break;
    }
    case 10: case 11: case 12: c.get<uint64_t>(); break;
    default: return false;
  }
  return c.ok;
}

}  // namespace

static int parse_gguf(const uint8_t* p, size_t n, GgufParsed& g) {
  Cur c{p, n, 0};
  if (c.get<uint32_t>() != 0x46554747u) return fail(LE_EIO, "gguf: invalid magic");
  const uint32_t ver = c.get<uint32_t>();
  if (ver < 2 || ver > 3) return fail(LE_EIO, "gguf: unsupported version: %u", ver);
  const uint64_t nt = c.get<uint64_t>(), nkv = c.get<uint64_t>();
  if (!c.ok || nt > (1u << 20) || nkv > (1u << 20)) return fail(LE_EIO, "gguf: bad header");
  for (uint64_t i = 0; i < nkv; i++) {
    std::string key = c.str();
    uint32_t vt = c.get<uint32_t>();
    if (!c.ok || !gguf_value(c, vt, g, &key, 0)) return fail(LE_EIO, "gguf: reading KV pair %llu", (unsigned long long)i);
  }
  struct Info {
    int32_t nd;
    uint64_t dims[4];
    uint32_t type;
    uint64_t off;
  };
  std::vector<Info> infos;
  for (uint64_t i = 0; i < nt; i++) {
    g.names.push_back(c.str());
    Info in{};
    in.nd = (int32_t)c.get<uint32_t>();
    if (in.nd < 1 || in.nd > 4) return fail(LE_EIO, "gguf: tensor %llu has %d dims", (unsigned long long)i, in.nd);
    for (int d = 0; d < in.nd; d++) in.dims[d] = c.get<uint64_t>();
    in.type = c.get<uint32_t>();
    in.off = c.get<uint64_t>();
    if (!c.ok) return fail(LE_EIO, "gguf: reading tensor %llu", (unsigned long long)i);
    infos.push_back(in);
  }
  const size_t data = (c.pos + 31) & ~(size_t)31;  // reader.go:266-269
  for (size_t i = 0; i < infos.size(); i++) {
    le_tensor_desc t{};
    t.name = g.names[i].c_str();
    t.type = (int32_t)infos[i].type;
    t.n_dims = infos[i].nd;
    uint64_t nel = 1;
    for (int d = 0; d < t.n_dims; d++) {
      t.dims[d] = (int64_t)infos[i].dims[d];
      nel *= infos[i].dims[d];
    }
    const long rb = row_bytes_of(t.type, (long)infos[i].dims[0]);
    t.n_bytes = rb < 0 ? 0 : (int64_t)(rb * (long)(nel / infos[i].dims[0]));
    if (data + infos[i].off + (uint64_t)t.n_bytes > n) return fail(LE_EIO, "gguf: tensor %s out of file", t.name);
    t.data = p + data + infos[i].off;
    g.tensors.push_back(t);
  }
  return LE_OK;
}

// ---------------------------------------------------------- C ABI ---------

extern "C" {

const char* le_last_error(void) { return g_err.c_str(); }

int le_init(int* ndev) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(LE_ECUDA, "no CUDA device: %s", cudaGetErrorString(e));
  }
  int ok = 0;
  for (int d = 0; d < n; d++) {
    cudaDeviceProp p{};
    if (cudaGetDeviceProperties(&p, d) == cudaSuccess && p.major == 10) ok++;
  }
  if (ndev) *ndev = ok;
  if (ok == 0) return fail(LE_ECUDA, "no sm_100 device among %d CUDA devices", n);
  return LE_OK;
}

static const le_tensor_desc* find(const le_tensor_desc* t, int nt, const std::string& name) {
  for (int i = 0; i < nt; i++)
    if (t[i].name && name == t[i].name) return &t[i];
  return nullptr;
}

static int load_impl(int dev, const le_tensor_desc* ts, int nt, const le_hparams* hp, le_model** out,
                     double parse_ms = 0) {
  const double t_start = now_ms();
  if (!ts || !hp || !out) return fail(LE_EINVAL, "null argument");
  *out = nullptr;
  int ndev = 0;
  TRY(le_init(&ndev));
  int total = 0;
  CK(cudaGetDeviceCount(&total));
  if (dev < 0 || dev >= total) return fail(LE_EINVAL, "device %d out of range (%d devices)", dev, total);
  if (hp->n_layers <= 0 || hp->hidden <= 0) return fail(LE_EINVAL, "embed: missing model params in GGUF metadata");
  if (hp->heads <= 0 || hp->hidden % hp->heads || hp->hidden / hp->heads != 64)
    return fail(LE_EINVAL, "head_dim must be 64 (hidden %d, heads %d)", hp->hidden, hp->heads);
  if (hp->hidden % 256 || hp->hidden > 1024) return fail(LE_EINVAL, "hidden %d unsupported (multiple of 256, <= 1024)", hp->hidden);
  if (hp->ffn <= 0 || hp->ffn % 256) return fail(LE_EINVAL, "ffn %d unsupported (multiple of 256)", hp->ffn);
  if (hp->context_length <= 0) return fail(LE_EINVAL, "context_length must be positive");
  CK(cudaSetDevice(dev));
  auto m = std::make_unique<le_model>();
  m->dev = dev;
  m->hp = *hp;
  m->head_dim = hp->hidden / hp->heads;
  CK(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
  CK(cudaStreamCreateWithFlags(&m->capture_stream, cudaStreamNonBlocking));
  CK(cudaEventCreateWithFlags(&m->ws_done, cudaEventDisableTiming));
  CK(cudaDeviceGetAttribute(&m->sms, cudaDevAttrMultiProcessorCount, dev));
  TRY(m->barrier.ensure(small_sync_bytes()));
  cudaStream_t s = m->stream;
  const int H = hp->hidden, F = hp->ffn;
  auto need = [&](const std::string& n) { return find(ts, nt, n); };

  const le_tensor_desc* te = need("token_embd.weight");
  const le_tensor_desc* tt = need("token_types.weight");
  if (!te) return fail(LE_EINVAL, "tensor \"token_embd.weight\" not found");
  if (!tt) return fail(LE_EINVAL, "tensor \"token_types.weight\" not found");
  if (te->dims[0] != H) return fail(LE_EINVAL, "token_embd.weight inner dim %lld != hidden %d", (long long)te->dims[0], H);
  m->emb_type = te->type;
  m->emb_row_bytes = row_bytes_of(te->type, H);
  if (m->emb_row_bytes < 0) return fail(LE_EINVAL, "unsupported embedding type: %d", te->type);
  m->vocab = te->n_dims > 1 ? (int)te->dims[1] : 1;
  if (te->n_bytes < m->emb_row_bytes * m->vocab) return fail(LE_EINVAL, "token_embd.weight too short");
  // 16 spare bytes: the single-kernel forward stages rows with 16-byte loads
  // from the 16-byte boundary below each row.
  TRY(m->emb.ensure((size_t)m->emb_row_bytes * m->vocab + 16));
  {
    const double t0 = now_ms();
    CK(cudaMemcpyAsync(m->emb.p, te->data, (size_t)m->emb_row_bytes * m->vocab, cudaMemcpyHostToDevice, s));
    CK(cudaStreamSynchronize(s));
    m->load.upload_ms += now_ms() - t0;
    m->load.h2d_bytes += (int64_t)m->emb_row_bytes * m->vocab;
  }
  // token_types row 0, exact float32 (bert.go:227), kept in its own buffer.
  {
    const long trb = row_bytes_of(tt->type, H);
    if (trb < 0 || tt->dims[0] != H) return fail(LE_EINVAL, "unsupported token_types tensor");
    DevBuf raw;
    TRY(raw.ensure((size_t)trb));
    CK(cudaMemcpyAsync(raw.p, tt->data, (size_t)trb, cudaMemcpyHostToDevice, s));
    TRY(m->type0.ensure((size_t)H * 4));
    CK(launch_gguf_rows(tt->type, raw.as<uint8_t>(), trb, 1, H, m->type0.as<float>(), s));
    CK(cudaStreamSynchronize(s));
  }
  const le_tensor_desc* nw = need("token_embd_norm.weight");
  const le_tensor_desc* nb = need("token_embd_norm.bias");
  if (!nw || !nb) return fail(LE_EINVAL, "tensor \"token_embd_norm.*\" not found");
  TRY(upload_f32(m->embd_w, nw, H, s));
  TRY(upload_f32(m->embd_b, nb, H, s));

  m->layers.resize(hp->n_layers);
  for (int i = 0; i < hp->n_layers; i++) {
    Layer& L = m->layers[i];
    const std::string p = "blk." + std::to_string(i) + ".";
    const le_tensor_desc* w[5];
    static const char* names[5] = {"attn_qkv", "attn_output", "ffn_up", "ffn_gate", "ffn_down"};
    const int Ks[5] = {H, H, H, H, F}, Ns[5] = {3 * H, H, F, F, H};
    for (int j = 0; j < 5; j++) {
      w[j] = need(p + names[j] + ".weight");
      if (!w[j]) return fail(LE_EINVAL, "tensor \"%s%s.weight\" not found", p.c_str(), names[j]);
      int64_t N = 1;
      for (int d = 1; d < w[j]->n_dims; d++) N *= w[j]->dims[d];
      if (w[j]->dims[0] != Ks[j] || N != Ns[j])
        return fail(LE_EINVAL, "%s%s.weight has shape [%lld, %lld], expected [%d, %d]", p.c_str(), names[j],
                    (long long)w[j]->dims[0], (long long)N, Ks[j], Ns[j]);
      if (row_bytes_of(weight_type(w[j]->type), Ks[j]) < 0)
        return fail(LE_EINVAL, "%s%s.weight: unsupported type %d (F32/Q8_0/Q4_K/Q5_K/Q6_K)", p.c_str(), names[j],
                    w[j]->type);
      if (w[j]->n_bytes < row_bytes_of(weight_type(w[j]->type), Ks[j]) * Ns[j])
        return fail(LE_EINVAL, "%s%s.weight data too short", p.c_str(), names[j]);
    }
    int ty[5];
    for (int j = 0; j < 5; j++) ty[j] = weight_type(w[j]->type);
    if (ty[2] != ty[3])
      return fail(LE_EINVAL, "ffn_up and ffn_gate of layer %d must share a type (%d vs %d)", i, w[2]->type, w[3]->type);
    TRY(make_qmat(L.qkv, ty[0], w[0]->data, nullptr, 3 * H, H, false, s, true, &m->load));
    TRY(make_qmat(L.out, ty[1], w[1]->data, nullptr, H, H, false, s, true, &m->load));
    TRY(make_qmat(L.upgate, ty[2], w[2]->data, w[3]->data, F, H, true, s, true, &m->load));
    TRY(make_qmat(L.down, ty[4], w[4]->data, nullptr, H, F, false, s, true, &m->load));
    const char* nn[4] = {"attn_output_norm.weight", "attn_output_norm.bias", "layer_output_norm.weight",
                         "layer_output_norm.bias"};
    DevBuf* dst[4] = {&L.attn_w, &L.attn_b, &L.out_w, &L.out_b};
    for (int j = 0; j < 4; j++) {
      const le_tensor_desc* t = need(p + nn[j]);
      if (!t) return fail(LE_EINVAL, "tensor \"%s%s\" not found", p.c_str(), nn[j]);
      TRY(upload_f32(*dst[j], t, H, s));
    }
  }
  // ops_simd.go:107-124 (NewRoPETable): freq = f32(1)/f32(pow(base, 2i/d)),
  // theta = freq * f32(pos), cos/sin in float64 rounded to float32.
  {
    const int nrot = m->head_dim / 2, P = hp->context_length;
    std::vector<float> c((size_t)P * nrot), sn((size_t)P * nrot);
    for (int pos = 0; pos < P; pos++)
      for (int i = 0; i < nrot; i++) {
        const float freq = 1.0f / (float)std::pow((double)hp->rope_base, (double)(2 * i) / (double)m->head_dim);
        const float theta = freq * (float)pos;
        c[(size_t)pos * nrot + i] = (float)std::cos((double)theta);
        sn[(size_t)pos * nrot + i] = (float)std::sin((double)theta);
      }
    TRY(m->rope_cos.ensure(c.size() * 4));
    TRY(m->rope_sin.ensure(sn.size() * 4));
    CK(cudaMemcpy(m->rope_cos.p, c.data(), c.size() * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(m->rope_sin.p, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
  }
  TRY(m->status.ensure(sizeof(DevStatus)));
  CK(cudaMemsetAsync(m->status.p, 0, sizeof(DevStatus), s));
  CK(cudaStreamSynchronize(s));
  m->parse_ms = parse_ms;
  m->load_ms = parse_ms + (now_ms() - t_start);
  *out = m.release();
  return LE_OK;
}

int le_model_load(int dev, const le_tensor_desc* tensors, int n_tensors, const le_hparams* hp, le_model** out) {
  return load_impl(dev, tensors, n_tensors, hp, out);
}

int le_model_load_gguf(int dev, const char* path, le_model** out) {
  if (!path || !out) return fail(LE_EINVAL, "null argument");
  const double t0 = now_ms();
  Mapped mp;
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(LE_EIO, "gguf: open %s: %s", path, strerror(errno));
  struct stat st {};
  if (fstat(fd, &st) != 0) {
    close(fd);
    return fail(LE_EIO, "gguf: stat %s failed", path);
  }
  mp.n = (size_t)st.st_size;
  mp.p = mmap(nullptr, mp.n, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (mp.p == MAP_FAILED) return fail(LE_EIO, "gguf: mmap %s failed", path);
  GgufParsed g;
  TRY(parse_gguf((const uint8_t*)mp.p, mp.n, g));
  auto u = [&](const char* k) { auto it = g.u32.find(k); return it == g.u32.end() ? 0u : it->second; };
  auto f = [&](const char* k) { auto it = g.f32.find(k); return it == g.f32.end() ? 0.f : it->second; };
  le_hparams hp{};
  hp.n_layers = (int)u("nomic-bert.block_count");
  hp.hidden = (int)u("nomic-bert.embedding_length");
  hp.ffn = (int)u("nomic-bert.feed_forward_length");
  hp.heads = (int)u("nomic-bert.attention.head_count");
  hp.context_length = (int)u("nomic-bert.context_length");
  hp.ln_eps = f("nomic-bert.attention.layer_norm_epsilon");
  hp.rope_base = f("nomic-bert.rope.freq_base");
  return load_impl(dev, g.tensors.data(), (int)g.tensors.size(), &hp, out, now_ms() - t0);
}

int le_model_free(le_model* m) {
  if (!m) return LE_OK;
  {
    std::lock_guard<std::mutex> lk(m->mu);
    cudaSetDevice(m->dev);
    cudaStreamSynchronize(m->stream);
  }
  delete m;
  return LE_OK;
}

int le_model_load_stats(const le_model* m, le_load_stats* out) {
  if (!m || !out) return fail(LE_EINVAL, "null argument");
  out->parse_ms = m->parse_ms;
  out->upload_ms = m->load.upload_ms;
  out->repack_ms = m->load.repack_ms;
  out->expand_ms = m->load.expand_ms;
  out->total_ms = m->load_ms;
  out->h2d_bytes = m->load.h2d_bytes;
  size_t dev_bytes = m->emb.n + m->type0.n + m->embd_w.n + m->embd_b.n + m->rope_cos.n + m->rope_sin.n;
  for (const Layer& L : m->layers) {
    for (const QMat* q : {&L.qkv, &L.out, &L.upgate, &L.down}) dev_bytes += q->buf.n + q->r16.n + q->w16.n;
    dev_bytes += L.attn_w.n + L.attn_b.n + L.out_w.n + L.out_b.n;
  }
  out->weight_bytes = (int64_t)dev_bytes;
  return LE_OK;
}

int le_model_hparams(const le_model* m, le_hparams* out) {
  if (!m || !out) return fail(LE_EINVAL, "null argument");
  *out = m->hp;
  return LE_OK;
}

static double seq_work(int L) { return 226492416.0 * L + 36864.0 * (double)L * L; }

int le_embed_ids(le_model* const* models, int n_models, const int32_t* ids, const int32_t* offs, int nseq, int out_dim,
                 float* out) {
  if (!models || n_models <= 0 || !offs || (nseq > 0 && (!ids || !out))) return fail(LE_EINVAL, "null argument");
  if (nseq < 0) return fail(LE_EINVAL, "nseq < 0");
  for (int i = 0; i < n_models; i++)
    if (!models[i]) return fail(LE_EINVAL, "model %d is null", i);
  const le_model* m0 = models[0];
  if (out_dim < 1 || out_dim > m0->hp.hidden) return fail(LE_EINVAL, "out_dim %d outside [1, %d]", out_dim, m0->hp.hidden);
  if (nseq == 0) return LE_OK;
  if (offs[0] != 0) return fail(LE_EINVAL, "seq_offsets[0] must be 0");
  for (int s = 0; s < nseq; s++) {
    const int L = offs[s + 1] - offs[s];
    if (L < 0) return fail(LE_EINVAL, "seq_offsets not ascending at %d", s);
    if (L > m0->hp.context_length) return fail(LE_EINVAL, "sequence %d has %d tokens > context_length %d", s, L, m0->hp.context_length);
  }
  for (int i = 0; i < offs[nseq]; i++)
    if (ids[i] < 0 || ids[i] >= m0->vocab) return fail(LE_EINVAL, "token id %d at %d outside vocab %d", ids[i], i, m0->vocab);
  if (n_models == 1) return embed_host(models[0], ids, offs, nseq, out_dim, out);
  // Token-balanced contiguous shards, one thread per device (no collectives).
  double total = 0;
  for (int s = 0; s < nseq; s++) total += seq_work(offs[s + 1] - offs[s]);
  std::vector<int> cut(n_models + 1, nseq);
  cut[0] = 0;
  double acc = 0;
  int k = 1;
  for (int s = 0; s < nseq && k < n_models; s++) {
    acc += seq_work(offs[s + 1] - offs[s]);
    while (k < n_models && acc >= total * k / n_models) cut[k++] = s + 1;
  }
  std::vector<int> rc(n_models, LE_OK);
  std::vector<std::string> msg(n_models);
  std::vector<std::thread> th;
  for (int i = 0; i < n_models; i++) {
    th.emplace_back([&, i] {
      const int a = cut[i], b = cut[i + 1];
      if (b <= a) return;
      std::vector<int32_t> o(b - a + 1);
      for (int j = a; j <= b; j++) o[j - a] = offs[j] - offs[a];
      rc[i] = embed_host(models[i], ids + offs[a], o.data(), b - a, out_dim, out + (size_t)a * out_dim);
      if (rc[i] != LE_OK) msg[i] = g_err;
    });
  }
  for (auto& t : th) t.join();
  for (int i = 0; i < n_models; i++)
    if (rc[i] != LE_OK) return fail(rc[i], "device shard %d: %s", i, msg[i].c_str());
  return LE_OK;
}

int le_embed_ids_device(le_model* m, const int32_t* d_ids, const int32_t* d_offsets, int nseq, int n_tokens, int max_len,
                        int out_dim, float* d_out, void* stream) {
  if (!m || !d_offsets || (nseq > 0 && !d_out)) return fail(LE_EINVAL, "null argument");
  if (out_dim < 1 || out_dim > m->hp.hidden) return fail(LE_EINVAL, "out_dim %d outside [1, %d]", out_dim, m->hp.hidden);
  if (nseq < 0 || n_tokens < 0 || max_len < 0 || max_len > m->hp.context_length)
    return fail(LE_EINVAL, "bad sizes (nseq %d, tokens %d, max_len %d)", nseq, n_tokens, max_len);
  if (n_tokens > LE_MAX_DEVICE_TOKENS)
    return fail(LE_EINVAL, "n_tokens %d exceeds LE_MAX_DEVICE_TOKENS (%d): split the batch", n_tokens,
                LE_MAX_DEVICE_TOKENS);
  std::lock_guard<std::mutex> lk(m->mu);
  CK(cudaSetDevice(m->dev));
  cudaStream_t s = stream ? (cudaStream_t)stream : m->stream;
  TRY(ensure_ws(m, n_tokens, nseq));
  bool cap = false;
  TRY(ws_order_begin(m, s, &cap));
  TRY(run_forward(m, d_ids, d_offsets, nseq, n_tokens, max_len, out_dim, d_out, s));
  return ws_order_end(m, s, cap);
}

int le_sync(le_model* m) {
  if (!m) return fail(LE_EINVAL, "null argument");
  std::lock_guard<std::mutex> lk(m->mu);
  CK(cudaSetDevice(m->dev));
  CK(cudaDeviceSynchronize());
  return model_status(m, m->stream);
}

int le_set_profiling(le_model* m, int enable) {
  if (!m) return fail(LE_EINVAL, "null argument");
  std::lock_guard<std::mutex> lk(m->mu);
  m->prof.on = enable != 0;
  return LE_OK;
}

int le_get_stats(le_model* m, le_stats* out, int reset) {
  if (!m || !out) return fail(LE_EINVAL, "null argument");
  std::lock_guard<std::mutex> lk(m->mu);
  CK(cudaSetDevice(m->dev));
  CK(cudaDeviceSynchronize());
  TRY(m->prof.collect());
  out->launches = m->prof.launches;
  for (int i = 0; i < LE_NCLASS; i++) {
    out->count[i] = m->prof.count[i];
    out->ms[i] = m->prof.ms[i];
  }
  if (reset) {
    m->prof.launches = 0;
    for (int i = 0; i < LE_NCLASS; i++) {
      m->prof.count[i] = 0;
      m->prof.ms[i] = 0;
    }
  }
  return LE_OK;
}

int le_dequant(le_model* m, int layer, int which, int mode, float* out) {
  if (!m || !out) return fail(LE_EINVAL, "null argument");
  if (layer < 0 || layer >= m->hp.n_layers || which < 0 || which > 4 || mode < 0 || mode > 1)
    return fail(LE_EINVAL, "bad layer/which/mode (%d, %d, %d)", layer, which, mode);
  std::lock_guard<std::mutex> lk(m->mu);
  CK(cudaSetDevice(m->dev));
  const Layer& L = m->layers[layer];
  const QMat* q = which == 0 ? &L.qkv : which == 1 ? &L.out : which == 4 ? &L.down : &L.upgate;
  const int K = q->K;
  // Virtual row of output row n (the merged up/gate order for which 2, 3).
  auto vrow = [&](int n) {
    return (which == 2 || which == 3) ? (n / (TILE_N / 2)) * TILE_N + (n % (TILE_N / 2)) + (which == 3 ? TILE_N / 2 : 0)
                                      : n;
  };
  const int n_out = (which == 2 || which == 3) ? m->hp.ffn : q->n_real;
  if (q->qf == QF_F16) {
    // F32 weights: mode 0 is the stored rows themselves, mode 1 their fp16
    // operand values.
    if (mode == 0) {
      const size_t off = which == 3 ? (size_t)n_out * K : 0;
      CK(cudaMemcpyAsync(out, q->buf.as<float>() + off, (size_t)n_out * K * 4, cudaMemcpyDeviceToHost, m->stream));
      CK(cudaStreamSynchronize(m->stream));
      return LE_OK;
    }
    std::vector<__half> h16((size_t)q->n_virt * K);
    CK(cudaMemcpyAsync(h16.data(), q->w16.p, h16.size() * 2, cudaMemcpyDeviceToHost, m->stream));
    CK(cudaStreamSynchronize(m->stream));
    for (int n = 0; n < n_out; n++)
      for (int k = 0; k < K; k++) out[(size_t)n * K + k] = __half2float(h16[(size_t)vrow(n) * K + k]);
    return LE_OK;
  }
  DevBuf d;
  TRY(d.ensure((size_t)q->n_virt * q->K * 4));
  CK(launch_dequant_tiles(q->qf, q->buf.as<uint8_t>(), q->n_virt, q->K, mode, d.as<float>(), m->stream));
  std::vector<float> all((size_t)q->n_virt * q->K);
  CK(cudaMemcpyAsync(all.data(), d.p, all.size() * 4, cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  for (int n = 0; n < n_out; n++) std::memcpy(out + (size_t)n * K, all.data() + (size_t)vrow(n) * K, (size_t)K * 4);
  return LE_OK;
}

int le_qweight_create(int dev, int qtype, const void* wq, int N, int K, le_qweight** out) {
  if (!wq || !out) return fail(LE_EINVAL, "null argument");
  *out = nullptr;
  int ndev = 0;
  TRY(le_init(&ndev));
  CK(cudaSetDevice(dev));
  auto w = std::make_unique<le_qweight>();
  w->dev = dev;
  CK(cudaStreamCreateWithFlags(&w->stream, cudaStreamNonBlocking));
  TRY(make_qmat(w->w, qtype, wq, nullptr, N, K, false, w->stream));
  TRY(w->status.ensure(sizeof(DevStatus)));
  CK(cudaMemset(w->status.p, 0, sizeof(DevStatus)));
  *out = w.release();
  return LE_OK;
}

int le_qgemm_device(le_qweight* w, const float* d_x, int M, float* d_y, void* stream) {
  if (!w || (M > 0 && (!d_x || !d_y))) return fail(LE_EINVAL, "null argument");
  if (M < 0) return fail(LE_EINVAL, "M < 0");
  std::lock_guard<std::mutex> lk(w->mu);
  CK(cudaSetDevice(w->dev));
  cudaStream_t s = stream ? (cudaStream_t)stream : w->stream;
  const int K = w->w.K;
  TRY(w->x16.ensure((size_t)std::max(M, 1) * K * 2));
  CK(launch_f32_to_f16(d_x, (long)M * K, w->x16.as<__half>(), s));
  EpiParams e{};
  e.mode = EPI_F32;
  e.M = M;
  e.N = w->w.n_real;
  e.out32 = d_y;
  e.ldo = w->w.n_real;
  CK(launch_gemm(gemm_w(w->w, w->w.n_real), w->x16.as<__half>(), K, e, w->status.as<DevStatus>(), s));
  return LE_OK;
}

int le_qweight_sync(le_qweight* w) {
  if (!w) return fail(LE_EINVAL, "null argument");
  std::lock_guard<std::mutex> lk(w->mu);
  CK(cudaSetDevice(w->dev));
  CK(cudaDeviceSynchronize());
  return check_status(w->status, w->stream);
}

int le_qweight_free(le_qweight* w) {
  if (!w) return LE_OK;
  cudaSetDevice(w->dev);
  cudaStreamSynchronize(w->stream);
  delete w;
  return LE_OK;
}

int le_qgemm(int dev, int qtype, const void* wq, int N, int K, const float* x, int M, float* y) {
  if (!wq || (M > 0 && (!x || !y))) return fail(LE_EINVAL, "null argument");
  le_qweight* w = nullptr;
  TRY(le_qweight_create(dev, qtype, wq, N, K, &w));
  std::unique_ptr<le_qweight, int (*)(le_qweight*)> guard(w, le_qweight_free);
  if (M == 0) return LE_OK;
  DevBuf dx, dy;
  TRY(dx.ensure((size_t)M * K * 4));
  TRY(dy.ensure((size_t)M * N * 4));
  CK(cudaMemcpyAsync(dx.p, x, (size_t)M * K * 4, cudaMemcpyHostToDevice, w->stream));
  TRY(le_qgemm_device(w, dx.as<float>(), M, dy.as<float>(), nullptr));
  CK(cudaMemcpyAsync(y, dy.p, (size_t)M * N * 4, cudaMemcpyDeviceToHost, w->stream));
  return check_status(w->status, w->stream);
}

// le_qgemm_device_noalloc: le_qgemm_device with its scratch (the status word
// and the fp16 copy of x) in one file-scope device array instead of buffers
// grown per weight.  Layout: [0, 256) DevStatus, then fp16 x [M][K].  The
// array is shared by every call on a device; only the status word has to
// start at zero, and each call clears it first.
static __device__ __align__(256) uint8_t g_noalloc_scratch[256 + (size_t)LE_QGEMM_NOALLOC_MAX_ELEMS * 2];

constexpr int NOALLOC_MAX_DEVICES = 64;
static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[NOALLOC_MAX_DEVICES];

// Device address of the scratch array on the current device `dev`, looked up
// once per device.
static int noalloc_scratch(int dev, uint8_t** out) {
  if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) return fail(LE_EINVAL, "device %d beyond %d", dev, NOALLOC_MAX_DEVICES);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    CK(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    if (!p || reinterpret_cast<uintptr_t>(p) % 256) return fail(LE_ECUDA, "scratch array address %p", p);
    g_noalloc_ptr[dev] = p;
  }
  *out = static_cast<uint8_t*>(g_noalloc_ptr[dev]);
  return LE_OK;
}

int le_qgemm_device_noalloc(le_qweight* w, const float* d_x, int M, float* d_y, void* stream) {
  if (!w || (M > 0 && (!d_x || !d_y))) return fail(LE_EINVAL, "null argument");
  if (M < 0) return fail(LE_EINVAL, "M < 0");
  const int K = w->w.K;
  if ((long long)M * K > LE_QGEMM_NOALLOC_MAX_ELEMS)
    return fail(LE_EINVAL, "M*K = %lld exceeds the scratch limit of %d elements", (long long)M * K,
                LE_QGEMM_NOALLOC_MAX_ELEMS);
  std::lock_guard<std::mutex> lk(w->mu);
  CK(cudaSetDevice(w->dev));
  uint8_t* scratch = nullptr;
  TRY(noalloc_scratch(w->dev, &scratch));
  if (M == 0) return LE_OK;
  cudaStream_t s = stream ? (cudaStream_t)stream : w->stream;
  DevStatus* st = reinterpret_cast<DevStatus*>(scratch);
  __half* x16 = reinterpret_cast<__half*>(scratch + 256);
  CK(cudaMemsetAsync(st, 0, sizeof(DevStatus), s));
  CK(launch_f32_to_f16(d_x, (long)M * K, x16, s));
  EpiParams e{};
  e.mode = EPI_F32;
  e.M = M;
  e.N = w->w.n_real;
  e.out32 = d_y;
  e.ldo = w->w.n_real;
  CK(launch_gemm(gemm_w(w->w, w->w.n_real), x16, K, e, st, s));
  DevStatus h{};
  CK(cudaMemcpyAsync(&h, st, sizeof h, cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  if (h.code != DE_OK)
    return fail(LE_EDEVICE, "kernel failure code %d at site %d (info %d)", h.code, h.where, h.info);
  return LE_OK;
}

int le_info(char* buf, int len) {
  int n = 0, sms = 0;
  cudaDeviceProp p{};
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  if (n > 0 && cudaGetDeviceProperties(&p, 0) == cudaSuccess) sms = p.multiProcessorCount;
  const int w = snprintf(buf, buf ? (size_t)len : 0,
                         "{\"devices\": %d, \"device0\": \"%s\", \"sm_count\": %d, \"arch\": \"sm_100a\", "
                         "\"gemm\": \"%s\", \"operands\": \"fp16\", \"accumulate\": \"fp32\"}",
                         n, n > 0 ? p.name : "", sms, gemm_variant_name());
  return w < 0 ? LE_EINVAL : LE_OK;
}

}  // extern "C"
