/*
 * libllmembed_cuda — C ABI of the B200 (sm_100a) nomic-bert encoder.
 *
 * Drop-in device backend for dbrushchenko/llm-embed's encoder forward pass.
 * The reference computes it in Go + amd64 asm (internal/embed/bert.go,
 * internal/ggml/*); this library replaces everything `Forward` reaches below
 * the Go API.  The host keeps the GGUF reader (internal/gguf/reader.go) and
 * the WordPiece tokenizer (internal/embed/tokenizer.go) and calls these
 * functions with token ids.
 *
 * Conventions
 *   - Every function returns 0 on success or a negative LE_E* code; the
 *     message of the last failure on the calling thread is le_last_error().
 *   - Plain pointers and sizes only.  "host" buffers are ordinary CPU
 *     memory owned by the caller; "device" buffers are CUDA device pointers
 *     on the model's device.
 *   - Thread safety: any function may be called from any thread.  Calls on
 *     one model are serialised by a per-model lock; different models (e.g.
 *     one per GPU) run concurrently.
 *   - No CPU fallback: without a usable sm_100 device le_init fails.
 *
 * Citations are path:line inside the reference project.
 */
#ifndef LLMEMBED_H
#define LLMEMBED_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LE_OK 0
#define LE_EINVAL -1   /* bad argument, shape or unsupported tensor type */
#define LE_ECUDA -2    /* CUDA runtime error */
#define LE_EDEVICE -3  /* kernel reported a failure (bounded wait expired, bounds) */
#define LE_ENOMEM -4   /* device or host allocation failed */
#define LE_EIO -5      /* GGUF file could not be read or parsed */

/* GGML tensor type ids accepted for weights (internal/gguf/reader.go:46-65).
 * Projection weights may also carry ids 15 and 16, which the reference's
 * DequantWeightMatrix (internal/ggml/gemm.go:240) decodes as Q5_K; so does
 * this library.  F32 projection weights are multiplied as fp16 operands. */
#define LE_TYPE_F32 0
#define LE_TYPE_Q8_0 8
#define LE_TYPE_Q4_K 12
#define LE_TYPE_Q5_K 13
#define LE_TYPE_Q6_K 14

typedef struct le_model le_model;

/* One tensor of a parsed GGUF file: what gguf.Open reports
 * (internal/gguf/reader.go:178-184 TensorInfo) plus its bytes.  `data` may
 * point into the caller's mmap; it is only read during le_model_load. */
typedef struct {
  const char* name;  /* e.g. "blk.3.attn_qkv.weight" (bert.go:152-207) */
  int32_t type;      /* GGML type id */
  int32_t n_dims;
  int64_t dims[4];   /* GGUF order: dims[0] is the contiguous (K) dim */
  const void* data;
  int64_t n_bytes;
} le_tensor_desc;

/* Model hyper-parameters read from GGUF KVs (bert.go:98-104). */
typedef struct {
  int32_t n_layers;        /* nomic-bert.block_count */
  int32_t hidden;          /* nomic-bert.embedding_length */
  int32_t ffn;             /* nomic-bert.feed_forward_length */
  int32_t heads;           /* nomic-bert.attention.head_count */
  int32_t context_length;  /* nomic-bert.context_length */
  float ln_eps;            /* nomic-bert.attention.layer_norm_epsilon */
  float rope_base;         /* nomic-bert.rope.freq_base */
} le_hparams;

/* Number of usable sm_100 devices.  Replaces the reference's backend probe
 * (internal/ggml/sgemm.go:237 InitSgemmBackend, mkl_linux.go:45 initMKL). */
int le_init(int* ndev);

/* Upload one full model replica to device `dev` and repack its weights into
 * the tile-blocked layout.  Replaces LoadBertModel + PreDequant +
 * NewRoPETable (bert.go:91, bert.go:542, embedder.go:26-29). */
int le_model_load(int dev, const le_tensor_desc* tensors, int n_tensors, const le_hparams* hp, le_model** out);

/* Convenience: parse a GGUF file (GGUF v2/v3, 32-byte data alignment as
 * internal/gguf/reader.go:219-280) and call le_model_load. */
int le_model_load_gguf(int dev, const char* path, le_model** out);

/* Wall-clock phases of a model load and the replica's footprint (the
 * reference's LoadBertModel + PreDequant, bert.go:91, bert.go:542, run once
 * at Load).  Each phase is timed with the device idle before and after it. */
typedef struct {
  double parse_ms;      /* GGUF mmap + metadata parse (le_model_load_gguf) */
  double upload_ms;     /* host -> device copies of the tensor bytes */
  double repack_ms;     /* tile-blocked repack kernels */
  double expand_ms;     /* fp16 operand matrices (expand or F32 convert) */
  double total_ms;      /* the whole load call, parse included */
  int64_t h2d_bytes;    /* weight and embedding bytes copied to the device */
  int64_t weight_bytes; /* device memory held by the replica's weights */
} le_load_stats;
int le_model_load_stats(const le_model* m, le_load_stats* out);

/* Release a model (bert.go:46 Close). */
int le_model_free(le_model* m);

/* Hyper-parameters of a loaded model. */
int le_model_hparams(const le_model* m, le_hparams* out);

/* Embed packed sequences.  Sequence s is ids[seq_offsets[s] ..
 * seq_offsets[s+1]) (all positions valid; the reference's padding positions
 * carry no information, see bert.go:381-386 and pool.go:17).  Writes the
 * L2-normalised [nseq][out_dim] float32 embeddings to host `out`, truncated
 * and renormalised when out_dim < hidden (Matryoshka, embedder.go:66-68).
 * Sequences are sharded across the given per-device models (one thread per
 * device, token-balanced).  Replaces Embedder.Embed / EmbedBatch
 * (embedder.go:46, embedder.go:75) below tokenisation. */
int le_embed_ids(le_model* const* models, int n_models, const int32_t* ids, const int32_t* seq_offsets, int nseq,
                 int out_dim, float* out);

/* Largest n_tokens of one le_embed_ids_device call (le_embed_ids splits
 * larger batches into calls of at most this many tokens). */
#define LE_MAX_DEVICE_TOKENS 65536

/* Same on device-resident buffers of the model's device, asynchronously on
 * `stream` (a cudaStream_t; NULL = the model's own stream).  d_offsets has
 * nseq+1 entries starting at 0; n_tokens = d_offsets[nseq]; max_len is the
 * longest sequence.  The call returns once the work is enqueued; device
 * errors surface from the next call or from le_sync.  All forwards of one
 * model share its workspace: calls on different streams are ordered on the
 * GPU (each waits for the previous call's completion event), so they run one
 * after another, not concurrently.  A call enqueued while `stream` is being
 * captured into the caller's CUDA graph is not ordered against other calls:
 * the caller must not replay that graph concurrently with other forwards of
 * the model. */
int le_embed_ids_device(le_model* m, const int32_t* d_ids, const int32_t* d_offsets, int nseq, int n_tokens,
                        int max_len, int out_dim, float* d_out, void* stream);

/* Wait for the model's work and report any device-side failure. */
int le_sync(le_model* m);

/* Dequantise weight `which` (0 attn_qkv, 1 attn_output, 2 ffn_up,
 * 3 ffn_gate, 4 ffn_down) of `layer` from the device copy into host
 * out[N][K] float32, GGUF row order.  mode 0: the exact float32 values of
 * DequantWeightMatrix (internal/ggml/gemm.go:221); mode 1: the fp16 tensor
 * core operand values (round-to-nearest of mode 0), widened to float32. */
int le_dequant(le_model* m, int layer, int which, int mode, float* out);

/* Standalone quantised matmul y[M][N] = x[M][K] . W^T for raw GGUF weight
 * bytes wq (N rows of K elements, types Q8_0/Q4_K/Q5_K/Q6_K), host buffers.
 * Replaces gemmOrBatch / MatMulBatch (bert.go:579, internal/ggml/ops.go:418)
 * for one weight. */
int le_qgemm(int dev, int qtype, const void* wq, int N, int K, const float* x, int M, float* y);

/* Device-resident form of le_qgemm for repeated calls: upload + repack once,
 * then y = x . W^T on device buffers (x float32 [M][K], y float32 [M][N]). */
typedef struct le_qweight le_qweight;
int le_qweight_create(int dev, int qtype, const void* wq, int N, int K, le_qweight** out);
int le_qgemm_device(le_qweight* w, const float* d_x, int M, float* d_y, void* stream);
/* Wait for the weight's device work (all streams of its device) and report a
 * kernel failure of an earlier le_qgemm_device call (LE_EDEVICE; the status
 * word is cleared).  le_qgemm_device returns once its work is enqueued, so
 * this is where its device errors surface. */
int le_qweight_sync(le_qweight* w);
int le_qweight_free(le_qweight* w);

/* le_qgemm_device without allocation (no counterpart in the reference: its Go
 * GEMM allocates per call; this entry point exists for callers that must not
 * allocate device memory, e.g. inside a caller-managed memory budget).  The
 * fp16 copy of x and the kernel status word live in one file-scope device
 * array of 256 + 2*LE_QGEMM_NOALLOC_MAX_ELEMS bytes per device, so M*K must
 * not exceed LE_QGEMM_NOALLOC_MAX_ELEMS (LE_EINVAL otherwise).  The call
 * calls no cudaMalloc/cudaFree, runs on `stream` (NULL = the weight's
 * stream), waits for it and returns LE_EDEVICE on a kernel-reported failure.
 * Every call on a device shares the array: calls whose work overlaps on the
 * GPU (other streams, other host threads) race on it. */
#define LE_QGEMM_NOALLOC_MAX_ELEMS (4 * 1024 * 1024)
int le_qgemm_device_noalloc(le_qweight* w, const float* d_x, int M, float* d_y, void* stream);

/* Per-kernel device timing of le_embed_ids / le_embed_ids_device calls.
 * With profiling on, every kernel launch of the forward pass is bracketed by
 * CUDA events on its stream; le_get_stats synchronises and returns the
 * accumulated device time and launch count per kernel class.  `launches`
 * counts every kernel this library launched for the model (profiling on or
 * off).  Classes: 0 QKV GEMM, 1 attention-output GEMM, 2 FFN up/gate GEMM,
 * 3 FFN down GEMM, 4 attention, 5 LayerNorm, 6 embedding gather + LN,
 * 7 positions + mean-pool, 8 the single-kernel forward of small calls
 * (<= 16 tokens; all layers in one launch). */
#define LE_NCLASS 9
typedef struct {
  int64_t launches;
  int64_t count[LE_NCLASS];
  double ms[LE_NCLASS];
} le_stats;
int le_set_profiling(le_model* m, int enable);
int le_get_stats(le_model* m, le_stats* out, int reset);

/* Host tokenizer: internal/embed/tokenizer.go (WordPieceTokenizer,
 * LoadTokenizer, Encode) in C++, for hosts that hand texts to the library.
 * Token ids follow the reference's rules exactly: Go's strings.ToLower,
 * split on unicode.IsSpace and BERT punctuation, greedy longest match over
 * each word's UTF-8 bytes with the U+2581 prefix on the first piece, byte and
 * [UNK]=100 fallbacks, [CLS]=101 ... [SEP]=102, truncation keeping [SEP].
 * A tokenizer is read-only after creation: any number of threads may call
 * le_tokenize on it concurrently. */
typedef struct le_tokenizer le_tokenizer;
/* Vocabulary: token i (token_lens[i] bytes) has id i; a later duplicate wins
 * (tokenizer.go:29-35). */
int le_tokenizer_create(const char* const* tokens, const int32_t* token_lens, int n_tokens, le_tokenizer** out);
/* The vocabulary of a GGUF file's "tokenizer.ggml.tokens" string array
 * (tokenizer.go:24-44, readGGUFStringArray). */
int le_tokenizer_load_gguf(const char* path, le_tokenizer** out);
int le_tokenizer_vocab_size(const le_tokenizer* t, int* n);
int le_tokenizer_free(le_tokenizer* t);
/* Encode texts packed back to back in `text` (text i = bytes
 * text[text_offsets[i] .. text_offsets[i+1]), UTF-8; invalid bytes read as
 * U+FFFD as Go does) with `prefix` (NUL-terminated, may be NULL) prepended
 * (embedder.go:48-51), truncated to max_len ids (>= 2).  Writes offsets
 * [n_texts+1] and the packed ids (text i = ids[offsets[i] .. offsets[i+1])),
 * ready for le_embed_ids; if capacity (in ids) is too small, returns
 * LE_EINVAL with the offsets filled in, so offsets[n_texts] is the size to
 * allocate.  n_texts * max_len is always enough.  nthreads <= 0: all
 * hardware threads. */
int le_tokenize(const le_tokenizer* t, const char* text, const int64_t* text_offsets, int n_texts, const char* prefix,
                int max_len, int32_t* ids, int64_t capacity, int32_t* offsets, int nthreads);

/* Library / device description for health endpoints (sgemm.go:263
 * SgemmInfo): device count, SM count, kernel variants, precision mode. */
int le_info(char* buf, int len);

/* Message of the last failure on this thread ("" if none). */
const char* le_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* LLMEMBED_H */
