"""TEST INFRASTRUCTURE — ctypes binding of the CPU restatement oracle.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may
import this package; it is the checker, never the product.  See oracle.h for
what it restates and for its parity status.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

F32, Q8_0, Q4_K, Q5_K, Q6_K = 0, 8, 12, 13, 14
EMUL_FP32, EMUL_FP16, EMUL_BF16, EMUL_TF32 = 0, 1, 2, 3


def build():
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_SO):
            build()
        _lib = C.CDLL(_SO)
        fp, ip, up = C.POINTER(C.c_float), C.POINTER(C.c_int32), C.POINTER(C.c_uint8)
        L = _lib
        L.or_f16_to_f32.restype = C.c_float
        L.or_f16_to_f32.argtypes = [C.c_uint16]
        L.or_row_bytes.restype = C.c_long
        L.or_row_bytes.argtypes = [C.c_int, C.c_long]
        L.or_dequant.argtypes = [C.c_int, up, C.c_long, fp]
        L.or_dequant_matrix.argtypes = [C.c_int, up, C.c_int, C.c_int, fp]
        L.or_layernorm.argtypes = [fp, fp, fp, C.c_float, C.c_int]
        L.or_gelu.argtypes = [fp, C.c_int]
        L.or_softmax.argtypes = [fp, C.c_int]
        L.or_dot_f32.restype = C.c_float
        L.or_dot_f32.argtypes = [fp, fp, C.c_int]
        L.or_rope_table.argtypes = [C.c_int, C.c_int, C.c_float, fp, fp]
        L.or_prepack32.argtypes = [fp, C.c_int, C.c_int, fp]
        L.or_gemm_prepacked32.argtypes = [fp, C.c_int, fp, fp, C.c_int, C.c_int, C.c_int]
        L.or_matmul_batch.argtypes = [C.c_int, up, C.c_int, C.c_int, fp, C.c_int, fp, C.c_int]
        L.or_model_load.restype = C.c_void_p
        L.or_model_load.argtypes = [C.c_char_p, C.c_int, C.c_char_p, C.c_int]
        L.or_model_free.argtypes = [C.c_void_p]
        L.or_model_hparams.argtypes = [C.c_void_p, ip, fp, fp]
        L.or_forward.argtypes = [C.c_void_p, ip, ip, C.c_int, fp, C.c_int]
        L.or_embed_ids.argtypes = [C.c_void_p, ip, ip, C.c_int, C.c_int, fp, C.c_int]
        L.or_model_weight.argtypes = [C.c_void_p, C.c_int, C.c_int, fp]
    return _lib


def _p(a, t):
    return a.ctypes.data_as(C.POINTER(t))


def f16_to_f32(h: int) -> float:
    return lib().or_f16_to_f32(h)


def row_bytes(gtype: int, n: int) -> int:
    return lib().or_row_bytes(gtype, n)


def dequant(gtype: int, data, n: int) -> np.ndarray:
    d = np.ascontiguousarray(np.frombuffer(bytes(data), np.uint8) if not isinstance(data, np.ndarray) else data, np.uint8)
    out = np.empty(n, np.float32)
    if lib().or_dequant(gtype, _p(d, C.c_uint8), n, _p(out, C.c_float)) != 0:
        raise ValueError("unsupported type")
    return out


def dequant_matrix(gtype: int, data: np.ndarray, K: int, N: int) -> np.ndarray:
    d = np.ascontiguousarray(data, np.uint8)
    out = np.empty((N, K), np.float32)
    if lib().or_dequant_matrix(gtype, _p(d, C.c_uint8), K, N, _p(out, C.c_float)) != 0:
        raise ValueError("unsupported type")
    return out


def layernorm(x, w, b, eps):
    x = np.array(x, np.float32)
    lib().or_layernorm(_p(x, C.c_float), _p(np.ascontiguousarray(w, np.float32), C.c_float),
                       _p(np.ascontiguousarray(b, np.float32), C.c_float), eps, x.size)
    return x


def gelu(x):
    x = np.array(x, np.float32)
    lib().or_gelu(_p(x, C.c_float), x.size)
    return x


def softmax(x):
    x = np.array(x, np.float32)
    lib().or_softmax(_p(x, C.c_float), x.size)
    return x


def rope_table(max_seq, head_dim, base):
    c = np.empty((max_seq, head_dim // 2), np.float32)
    s = np.empty_like(c)
    lib().or_rope_table(max_seq, head_dim, base, _p(c, C.c_float), _p(s, C.c_float))
    return c, s


def gemm(A: np.ndarray, B_nk: np.ndarray, nthreads: int = 8) -> np.ndarray:
    """C = A . B^T with the reference's prepacked blocking."""
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B_nk, np.float32)
    M, K = A.shape
    N = B.shape[0]
    packed = np.empty(((N + 31) // 32) * K * 32, np.float32)
    lib().or_prepack32(_p(B, C.c_float), K, N, _p(packed, C.c_float))
    out = np.empty((M, N), np.float32)
    lib().or_gemm_prepacked32(_p(A, C.c_float), M, _p(packed, C.c_float), _p(out, C.c_float), N, K, nthreads)
    return out


def matmul_batch(gtype: int, wq: np.ndarray, K: int, N: int, X: np.ndarray, nthreads: int = 8) -> np.ndarray:
    X = np.ascontiguousarray(X, np.float32)
    wq = np.ascontiguousarray(wq, np.uint8)
    out = np.empty((X.shape[0], N), np.float32)
    if lib().or_matmul_batch(gtype, _p(wq, C.c_uint8), K, N, _p(X, C.c_float), X.shape[0], _p(out, C.c_float), nthreads):
        raise ValueError("unsupported type")
    return out


class Model:
    """Oracle model: LoadBertModel + PreDequant + NewRoPETable."""

    def __init__(self, path: str, emul: int = EMUL_FP32):
        err = C.create_string_buffer(512)
        self._h = lib().or_model_load(path.encode(), emul, err, 512)
        if not self._h:
            raise RuntimeError(err.value.decode())
        o = (C.c_int * 7)()
        eps, base = C.c_float(), C.c_float()
        lib().or_model_hparams(self._h, o, C.byref(eps), C.byref(base))
        self.layers, self.hidden, self.heads, self.head_dim, self.ffn, self.max_seq, self.vocab = list(o)
        self.eps, self.rope_base = eps.value, base.value

    def close(self):
        if self._h:
            lib().or_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, ids, mask=None, nthreads: int = 8) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        mask = np.ones_like(ids) if mask is None else np.ascontiguousarray(mask, np.int32)
        out = np.empty((ids.size, self.hidden), np.float32)
        if lib().or_forward(self._h, _p(ids, C.c_int32), _p(mask, C.c_int32), ids.size, _p(out, C.c_float), nthreads):
            raise ValueError("sequence too long")
        return out

    def embed_ids(self, ids, offsets, out_dim: int | None = None, nthreads: int = 8) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        offsets = np.ascontiguousarray(offsets, np.int32)
        out_dim = out_dim or self.hidden
        nseq = offsets.size - 1
        out = np.empty((nseq, out_dim), np.float32)
        if lib().or_embed_ids(self._h, _p(ids, C.c_int32), _p(offsets, C.c_int32), nseq, out_dim,
                              _p(out, C.c_float), nthreads):
            raise ValueError("bad arguments")
        return out

    def weight(self, layer: int, which: int) -> np.ndarray:
        N = [3 * self.hidden, self.hidden, self.ffn, self.ffn, self.hidden][which]
        K = self.ffn if which == 4 else self.hidden
        out = np.empty((N, K), np.float32)
        if lib().or_model_weight(self._h, layer, which, _p(out, C.c_float)):
            raise ValueError("bad layer/which")
        return out
