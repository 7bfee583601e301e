"""Python host binding of libllmembed_cuda, mirroring the reference's public
API (internal/embed/embedder.go): Load, Embed, EmbedBatch, Dim,
SetTargetDim, plus EmbedIDs for packed batches.

Texts are tokenised on the host (tokenizer.py, a restatement of
internal/embed/tokenizer.go) with the model's GGUF vocabulary and the
TaskPrefix, as Embedder.Embed does; the device library takes token ids, which
Embed / EmbedBatch also accept directly.  There is no CPU fallback: if the
CUDA library is missing or no sm_100 GPU is present, the calls raise.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import numpy as np


_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libllmembed_cuda.so")

LE_OK, LE_EINVAL, LE_ECUDA, LE_EDEVICE, LE_ENOMEM, LE_EIO = 0, -1, -2, -3, -4, -5
WEIGHT_NAMES = ("attn_qkv", "attn_output", "ffn_up", "ffn_gate", "ffn_down")


class LlmEmbedError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"llmembed error {code}: {message}")
        self.code = code


class TensorDesc(C.Structure):
    _fields_ = [("name", C.c_char_p), ("type", C.c_int32), ("n_dims", C.c_int32), ("dims", C.c_int64 * 4),
                ("data", C.c_void_p), ("n_bytes", C.c_int64)]


NCLASS = 9
CLASS_NAMES = ("gemm_qkv", "gemm_attn_out", "gemm_ffn_upgate", "gemm_ffn_down", "attention", "layernorm",
               "embed_ln", "positions_pool", "fused_small")


class Stats(C.Structure):
    _fields_ = [("launches", C.c_int64), ("count", C.c_int64 * NCLASS), ("ms", C.c_double * NCLASS)]


class LoadStats(C.Structure):
    _fields_ = [("parse_ms", C.c_double), ("upload_ms", C.c_double), ("repack_ms", C.c_double),
                ("expand_ms", C.c_double), ("total_ms", C.c_double), ("h2d_bytes", C.c_int64),
                ("weight_bytes", C.c_int64)]


# Largest token count of one device call (LE_MAX_DEVICE_TOKENS).
MAX_DEVICE_TOKENS = 65536


class HParams(C.Structure):
    _fields_ = [("n_layers", C.c_int32), ("hidden", C.c_int32), ("ffn", C.c_int32), ("heads", C.c_int32),
                ("context_length", C.c_int32), ("ln_eps", C.c_float), ("rope_base", C.c_float)]


_lib = None
_lib_lock = threading.Lock()


def lib() -> C.CDLL:
    """The loaded CUDA library (raises if it has not been built)."""
    global _lib
    with _lib_lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise LlmEmbedError(LE_EIO, f"{LIB_PATH} missing: build it with `python -m llm_embed_b200.build`")
            L = C.CDLL(LIB_PATH)
            vp, ip, fp = C.c_void_p, C.POINTER(C.c_int32), C.POINTER(C.c_float)
            L.le_last_error.restype = C.c_char_p
            L.le_init.argtypes = [C.POINTER(C.c_int)]
            L.le_model_load.argtypes = [C.c_int, C.POINTER(TensorDesc), C.c_int, C.POINTER(HParams), C.POINTER(vp)]
            L.le_model_load_gguf.argtypes = [C.c_int, C.c_char_p, C.POINTER(vp)]
            L.le_model_free.argtypes = [vp]
            L.le_model_hparams.argtypes = [vp, C.POINTER(HParams)]
            L.le_model_load_stats.argtypes = [vp, C.POINTER(LoadStats)]
            L.le_embed_ids.argtypes = [C.POINTER(vp), C.c_int, ip, ip, C.c_int, C.c_int, fp]
            L.le_embed_ids_device.argtypes = [vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, vp, vp]
            L.le_sync.argtypes = [vp]
            L.le_dequant.argtypes = [vp, C.c_int, C.c_int, C.c_int, fp]
            L.le_qgemm.argtypes = [C.c_int, C.c_int, vp, C.c_int, C.c_int, fp, C.c_int, fp]
            L.le_qweight_create.argtypes = [C.c_int, C.c_int, vp, C.c_int, C.c_int, C.POINTER(vp)]
            L.le_qgemm_device.argtypes = [vp, vp, C.c_int, vp, vp]
            L.le_qgemm_device_noalloc.argtypes = [vp, vp, C.c_int, vp, vp]
            L.le_qweight_free.argtypes = [vp]
            L.le_qweight_sync.argtypes = [vp]
            L.le_tokenizer_create.argtypes = [C.POINTER(C.c_char_p), ip, C.c_int, C.POINTER(vp)]
            L.le_tokenizer_load_gguf.argtypes = [C.c_char_p, C.POINTER(vp)]
            L.le_tokenizer_vocab_size.argtypes = [vp, C.POINTER(C.c_int)]
            L.le_tokenizer_free.argtypes = [vp]
            L.le_tokenize.argtypes = [vp, C.c_char_p, C.POINTER(C.c_int64), C.c_int, C.c_char_p, C.c_int, ip,
                                      C.c_int64, ip, C.c_int]
            L.le_info.argtypes = [C.c_char_p, C.c_int]
            L.le_set_profiling.argtypes = [vp, C.c_int]
            L.le_get_stats.argtypes = [vp, C.POINTER(Stats), C.c_int]
            _lib = L
        return _lib


def _check(rc: int) -> None:
    if rc != LE_OK:
        raise LlmEmbedError(rc, lib().le_last_error().decode(errors="replace"))


def init() -> int:
    """Number of usable sm_100 devices (raises if none)."""
    n = C.c_int(0)
    _check(lib().le_init(C.byref(n)))
    return n.value


def info() -> str:
    buf = C.create_string_buffer(1024)
    _check(lib().le_info(buf, 1024))
    return buf.value.decode()


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(C.POINTER(t))


def pack(seqs) -> tuple[np.ndarray, np.ndarray]:
    """List of id sequences -> (ids int32, offsets int32 [n+1])."""
    lens = [len(s) for s in seqs]
    offs = np.zeros(len(seqs) + 1, np.int32)
    offs[1:] = np.cumsum(lens, dtype=np.int64)
    ids = np.concatenate([np.asarray(s, np.int32) for s in seqs]) if seqs and offs[-1] else np.zeros(0, np.int32)
    return np.ascontiguousarray(ids, np.int32), offs


class Tokenizer:
    """The library's C++ host tokenizer (le_tokenizer_*): the rules of
    internal/embed/tokenizer.go, multithreaded over a batch of texts.  Same
    Encode/VocabSize interface as tokenizer.WordPieceTokenizer (its Python
    restatement)."""

    def __init__(self, handle):
        self._h = handle

    @classmethod
    def Load(cls, path: str) -> "Tokenizer":
        h = C.c_void_p()
        _check(lib().le_tokenizer_load_gguf(path.encode(), C.byref(h)))
        return cls(h.value)

    @classmethod
    def from_tokens(cls, tokens) -> "Tokenizer":
        toks = [t if isinstance(t, bytes) else t.encode() for t in tokens]
        arr = (C.c_char_p * len(toks))(*toks)
        lens = np.array([len(t) for t in toks], np.int32)
        h = C.c_void_p()
        _check(lib().le_tokenizer_create(arr, _p(lens, C.c_int32), len(toks), C.byref(h)))
        return cls(h.value)

    def VocabSize(self) -> int:
        n = C.c_int(0)
        _check(lib().le_tokenizer_vocab_size(self._h, C.byref(n)))
        return n.value

    @staticmethod
    def pack_texts(texts):
        """Texts as one UTF-8 buffer and int64 offsets [n+1] (le_tokenize's input)."""
        raw = [t if isinstance(t, bytes) else t.encode("utf-8", "surrogatepass") for t in texts]
        toffs = np.zeros(len(raw) + 1, np.int64)
        toffs[1:] = np.cumsum(np.fromiter(map(len, raw), np.int64, len(raw)))
        return b"".join(raw), toffs

    def encode_batch(self, texts, max_len: int, prefix: str = "", nthreads: int = 0):
        """(ids int32, offsets int32 [n+1]) of prefix + text for each text."""
        return self.encode_packed(*self.pack_texts(texts), max_len, prefix, nthreads)

    def encode_packed(self, buf: bytes, toffs: np.ndarray, max_len: int, prefix: str = "", nthreads: int = 0):
        """encode_batch on texts already packed by pack_texts."""
        n = toffs.size - 1
        offs = np.zeros(n + 1, np.int32)
        ids = np.empty(max(n * max_len, 1), np.int32)
        _check(lib().le_tokenize(self._h, buf, toffs.ctypes.data_as(C.POINTER(C.c_int64)), n,
                                 prefix.encode("utf-8", "surrogatepass"), max_len, _p(ids, C.c_int32), ids.size,
                                 _p(offs, C.c_int32), nthreads))
        return ids[:offs[-1]].copy(), offs

    def Encode(self, text, max_len: int) -> tuple[list[int], list[int]]:
        """Encode (tokenizer.go:47-80): token ids and the all-ones mask."""
        ids, _ = self.encode_batch([text], max_len)
        return ids.tolist(), [1] * len(ids)

    def close(self):
        if self._h:
            lib().le_tokenizer_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Embedder:
    """One model replica per device; EmbedIDs shards sequences across them."""

    def __init__(self, handles, hp: HParams, tokenizer: "Tokenizer | None" = None):
        self._handles = (C.c_void_p * len(handles))(*handles)
        self._n = len(handles)
        self.hparams = hp
        self.target_dim = hp.hidden
        self.tokenizer = tokenizer
        # embedder.go:15, 39: prepended to every text before tokenisation.
        self.TaskPrefix = "search_query: "

    # embedder.go:19 Load: model replicas plus the GGUF's tokenizer.
    @classmethod
    def Load(cls, model_path: str, devices=(0,)) -> "Embedder":
        handles = []
        try:
            for d in devices:
                h = C.c_void_p()
                _check(lib().le_model_load_gguf(int(d), model_path.encode(), C.byref(h)))
                handles.append(h.value)
        except Exception:
            for h in handles:
                lib().le_model_free(h)
            raise
        hp = HParams()
        _check(lib().le_model_hparams(handles[0], C.byref(hp)))
        # The model file parsed, so its KV section is readable; a file without
        # tokenizer.ggml.tokens still embeds token ids.
        try:
            tok = Tokenizer.Load(model_path)
        except LlmEmbedError as err:
            if "not found" in str(err):
                tok = None
            else:
                for h in handles:
                    lib().le_model_free(h)
                raise
        return cls(handles, hp, tok)

    @classmethod
    def LoadTensors(cls, tensors, hp: HParams, devices=(0,)) -> "Embedder":
        """le_model_load with caller-parsed tensors: list of
        (name, ggml_type, dims, bytes-like)."""
        arr = (TensorDesc * len(tensors))()
        keep = []
        for i, (name, gtype, dims, data) in enumerate(tensors):
            buf = np.frombuffer(data, np.uint8)
            keep.append((name.encode(), buf))
            arr[i].name = keep[-1][0]
            arr[i].type = gtype
            arr[i].n_dims = len(dims)
            for j, d in enumerate(dims):
                arr[i].dims[j] = d
            arr[i].data = buf.ctypes.data
            arr[i].n_bytes = buf.size
        handles = []
        for d in devices:
            h = C.c_void_p()
            _check(lib().le_model_load(int(d), arr, len(tensors), C.byref(hp), C.byref(h)))
            handles.append(h.value)
        return cls(handles, hp)

    def Close(self) -> None:
        if self._handles is not None:
            for h in self._handles:
                lib().le_model_free(h)
            self._handles = None

    close = Close

    def __del__(self):
        try:
            self.Close()
        except Exception:
            pass

    # embedder.go:136 Dim, :142 SetTargetDim (clamped to [1, hidden])
    def Dim(self) -> int:
        return self.target_dim

    def SetTargetDim(self, dim: int) -> None:
        self.target_dim = max(1, min(int(dim), self.hparams.hidden))

    # Packed batch: the device call of EmbedBatch.
    def EmbedIDs(self, ids, offsets, out_dim: int | None = None) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        offsets = np.ascontiguousarray(offsets, np.int32)
        nseq = offsets.size - 1
        d = self.target_dim if out_dim is None else out_dim
        out = np.empty((nseq, d), np.float32)
        _check(lib().le_embed_ids(self._handles, self._n, _p(ids, C.c_int32), _p(offsets, C.c_int32), nseq, d,
                                  _p(out, C.c_float)))
        return out

    def Tokenize(self, text: str) -> list[int]:
        """TaskPrefix + text through the model's tokenizer, truncated to the
        context length (embedder.go:48-51)."""
        if self.tokenizer is None:
            raise LlmEmbedError(LE_EINVAL, "no tokenizer: load the model from a GGUF file with tokenizer.ggml.tokens")
        return self.tokenizer.Encode(self.TaskPrefix + text, self.hparams.context_length)[0]

    def _ids(self, item) -> list[int]:
        return self.Tokenize(item) if isinstance(item, str) else item

    # embedder.go:46 Embed: a text (or an already tokenised id sequence).
    def Embed(self, text) -> np.ndarray:
        i, o = pack([self._ids(text)])
        return self.EmbedIDs(i, o)[0]

    # embedder.go:75 EmbedBatch: texts (or id sequences), one device call for
    # the whole batch instead of one forward per text; texts are tokenised
    # together by the C++ tokenizer's threads.
    def EmbedBatch(self, texts) -> list[np.ndarray]:
        if len(texts) == 0:
            return []
        if self.tokenizer is not None and all(isinstance(t, str) for t in texts):
            i, o = self.tokenizer.encode_batch(texts, self.hparams.context_length, prefix=self.TaskPrefix)
        else:
            i, o = pack([self._ids(t) for t in texts])
        return list(self.EmbedIDs(i, o))

    def embed_device(self, d_ids: int, d_offsets: int, nseq: int, n_tokens: int, max_len: int, d_out: int,
                     stream: int = 0, replica: int = 0, out_dim: int | None = None) -> None:
        """Asynchronous forward on device pointers of replica `replica`,
        enqueued on the cudaStream_t handle `stream` (0: the model's own
        stream, which does not order with the legacy default stream)."""
        d = self.target_dim if out_dim is None else out_dim
        _check(lib().le_embed_ids_device(self._handles[replica], d_ids, d_offsets, nseq, n_tokens, max_len, d,
                                         d_out, stream or None))

    def sync(self, replica: int = 0) -> None:
        _check(lib().le_sync(self._handles[replica]))

    def load_stats(self, replica: int = 0) -> dict:
        """Wall-clock phases (ms) of the replica's load and its byte counts."""
        st = LoadStats()
        _check(lib().le_model_load_stats(self._handles[replica], C.byref(st)))
        return {f: getattr(st, f) for f, _ in LoadStats._fields_}

    def set_profiling(self, on: bool, replica: int = 0) -> None:
        _check(lib().le_set_profiling(self._handles[replica], 1 if on else 0))

    def stats(self, reset: bool = True, replica: int = 0) -> dict:
        """Launch count and per-class device time (ms) since the last reset."""
        st = Stats()
        _check(lib().le_get_stats(self._handles[replica], C.byref(st), 1 if reset else 0))
        return {"launches": st.launches,
                "classes": {n: {"count": st.count[i], "ms": st.ms[i]} for i, n in enumerate(CLASS_NAMES)}}

    def dequant(self, layer: int, which: int, mode: int = 0) -> np.ndarray:
        hp = self.hparams
        N = [3 * hp.hidden, hp.hidden, hp.ffn, hp.ffn, hp.hidden][which]
        K = hp.ffn if which == 4 else hp.hidden
        out = np.empty((N, K), np.float32)
        _check(lib().le_dequant(self._handles[0], layer, which, mode, _p(out, C.c_float)))
        return out


def qgemm(qtype: int, wq: np.ndarray, N: int, K: int, x: np.ndarray, dev: int = 0) -> np.ndarray:
    """y = x . W^T for raw GGUF weight bytes (le_qgemm)."""
    wq = np.ascontiguousarray(wq, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    M = x.shape[0]
    y = np.empty((M, N), np.float32)
    _check(lib().le_qgemm(dev, qtype, wq.ctypes.data, N, K, _p(x, C.c_float), M, _p(y, C.c_float)))
    return y


class QWeight:
    """Device-resident quantised weight for repeated le_qgemm_device calls."""

    def __init__(self, qtype: int, wq: np.ndarray, N: int, K: int, dev: int = 0):
        wq = np.ascontiguousarray(wq, np.uint8)
        h = C.c_void_p()
        _check(lib().le_qweight_create(dev, qtype, wq.ctypes.data, N, K, C.byref(h)))
        self._h, self.N, self.K = h.value, N, K

    def matmul_device(self, d_x: int, M: int, d_y: int, stream: int = 0) -> None:
        _check(lib().le_qgemm_device(self._h, d_x, M, d_y, stream or None))

    def sync(self) -> None:
        """Wait for the device work; raise on a kernel failure of an earlier
        matmul_device call."""
        _check(lib().le_qweight_sync(self._h))

    # Largest M*K le_qgemm_device_noalloc accepts (LE_QGEMM_NOALLOC_MAX_ELEMS).
    NOALLOC_MAX_ELEMS = 4 * 1024 * 1024

    def matmul_device_noalloc(self, d_x: int, M: int, d_y: int, stream: int = 0) -> None:
        """matmul_device through the entry point that allocates nothing: it
        uses a fixed per-device scratch array shared by all calls (M*K <=
        NOALLOC_MAX_ELEMS) and waits for `stream` before returning."""
        _check(lib().le_qgemm_device_noalloc(self._h, d_x, M, d_y, stream or None))

    def close(self):
        if self._h:
            lib().le_qweight_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
