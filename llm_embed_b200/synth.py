"""Synthetic nomic-bert GGUF models and token inputs for tests and benchmarks.

The reference (dbrushchenko/llm-embed) only *reads* GGUF files
(internal/gguf/reader.go:219) and only *dequantises* blocks
(internal/ggml/tensor.go:130, quant_q4k.go:27, quant_q5k.go:29,
quant_q6k.go:23); no model file is available offline.  This module writes
random-init models that the reference's loader accepts:

* hparams as uint32 / float32 KVs, exactly the keys bert.go:98-104 reads;
* tensor names of bert.go:152-207, GGUF dims [K, N] (K contiguous);
* tensor data at 32-byte aligned offsets (reader.go:266-269);
* norms and token_types in F32, projections quantised per config.

The quantisers are simple amax / min-max rounding.  Parity does not depend
on quantiser quality (the CUDA path and the oracle read the same bytes); they
only need to produce valid blocks, and they keep fp16 subnormal scales (the
Q6_K super-scales of N(0, 0.02) weights are subnormal), which both decoders
must handle (tensor.go:162-191).

Seeds: tensor number t (in file order) of a model with seed s draws from
numpy.random.default_rng([s, t]); token inputs use default_rng([seed, 1000]).
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass, field

import numpy as np

GGML_F32, GGML_Q8_0, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K = 0, 8, 12, 13, 14
TYPE_NAMES = {"f32": GGML_F32, "q8_0": GGML_Q8_0, "q4_k": GGML_Q4_K, "q5_k": GGML_Q5_K, "q6_k": GGML_Q6_K}
BLOCK = {GGML_F32: (1, 4), GGML_Q8_0: (32, 34), GGML_Q4_K: (256, 144), GGML_Q5_K: (256, 176), GGML_Q6_K: (256, 210)}
WEIGHTS = ("attn_qkv", "attn_output", "ffn_up", "ffn_gate", "ffn_down")


def row_bytes(gtype: int, k: int) -> int:
    bs, ts = BLOCK[gtype]
    return k // bs * ts


def _f16_bits(x: np.ndarray) -> np.ndarray:
    """Round to IEEE half (nearest-even, subnormals kept) and return the bits."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def _f16_value(bits: np.ndarray) -> np.ndarray:
    return bits.view(np.float16).astype(np.float32)


# --------------------------------------------------------------- quantisers --

def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    """[N][K] f32 -> [N][K/32*34] uint8 (tensor.go:256-260 layout)."""
    n, k = w.shape
    b = w.reshape(n, k // 32, 32).astype(np.float32)
    amax = np.abs(b).max(axis=2)
    dbits = _f16_bits(amax / 127.0)
    d = _f16_value(dbits)
    inv = np.where(d > 0, 1.0 / np.where(d > 0, d, 1), 0).astype(np.float32)
    q = np.clip(np.rint(b * inv[..., None]), -128, 127).astype(np.int8)
    out = np.empty((n, k // 32, 34), np.uint8)
    out[..., 0:2] = dbits[..., None].view(np.uint8).reshape(n, k // 32, 2)
    out[..., 2:] = q.view(np.uint8)
    return out.reshape(n, -1)


def _pack_k4_scales(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Pack 8 six-bit (scale, min) pairs into 12 bytes, the inverse of
    getScaleMinK4 (quant_q4k.go:133-140).  sc, mn: [..., 8] uint8 < 64."""
    s = np.zeros(sc.shape[:-1] + (12,), np.uint8)
    s[..., 0:4] = (sc[..., 0:4] & 63) | ((sc[..., 4:8] >> 4) << 6)
    s[..., 4:8] = (mn[..., 0:4] & 63) | ((mn[..., 4:8] >> 4) << 6)
    s[..., 8:12] = (sc[..., 4:8] & 0xF) | ((mn[..., 4:8] & 0xF) << 4)
    return s


def _kquant_minmax(b: np.ndarray, qmax: int):
    """Sub-block (32) min-max quantisation shared by Q4_K (qmax 15) and
    Q5_K (qmax 31).  b: [N, nb, 8, 32] f32."""
    mn = np.minimum(b.min(axis=3), 0.0)
    mx = b.max(axis=3)
    scale = (mx - mn) / qmax
    dbits = _f16_bits(scale.max(axis=2) / 63.0)
    mbits = _f16_bits((-mn).max(axis=2) / 63.0)
    d = _f16_value(dbits)
    dmin = _f16_value(mbits)
    safe = lambda v: np.where(v > 0, v, 1.0)
    sc = np.where(d[..., None] > 0, np.clip(np.rint(scale / safe(d)[..., None]), 0, 63), 0).astype(np.uint8)
    m = np.where(dmin[..., None] > 0, np.clip(np.rint(-mn / safe(dmin)[..., None]), 0, 63), 0).astype(np.uint8)
    d1 = (d[..., None] * sc.astype(np.float32)).astype(np.float32)
    dm1 = (dmin[..., None] * m.astype(np.float32)).astype(np.float32)
    q = np.where(d1[..., None] > 0, np.rint((b + dm1[..., None]) / safe(d1)[..., None]), 0)
    q = np.clip(q, 0, qmax).astype(np.uint8)
    return dbits, mbits, sc, m, q


def quantize_q4_k(w: np.ndarray) -> np.ndarray:
    """[N][K] -> [N][K/256*144] (quant_q4k.go:8-18 layout)."""
    n, k = w.shape
    nb = k // 256
    b = w.reshape(n, nb, 8, 32).astype(np.float32)
    dbits, mbits, sc, m, q = _kquant_minmax(b, 15)
    out = np.zeros((n, nb, 144), np.uint8)
    out[..., 0:2] = dbits[..., None].view(np.uint8).reshape(n, nb, 2)
    out[..., 2:4] = mbits[..., None].view(np.uint8).reshape(n, nb, 2)
    out[..., 4:16] = _pack_k4_scales(sc, m)
    qg = q.reshape(n, nb, 4, 2, 32)  # group of 64 = (low-nibble 32, high-nibble 32)
    out[..., 16:144] = (qg[:, :, :, 0, :] | (qg[:, :, :, 1, :] << 4)).reshape(n, nb, 128)
    return out.reshape(n, -1)


def quantize_q5_k(w: np.ndarray) -> np.ndarray:
    """[N][K] -> [N][K/256*176] (quant_q5k.go:8-27 layout)."""
    n, k = w.shape
    nb = k // 256
    b = w.reshape(n, nb, 8, 32).astype(np.float32)
    dbits, mbits, sc, m, q = _kquant_minmax(b, 31)
    out = np.zeros((n, nb, 176), np.uint8)
    out[..., 0:2] = dbits[..., None].view(np.uint8).reshape(n, nb, 2)
    out[..., 2:4] = mbits[..., None].view(np.uint8).reshape(n, nb, 2)
    out[..., 4:16] = _pack_k4_scales(sc, m)
    qh = np.zeros((n, nb, 32), np.uint8)
    for s in range(8):  # bit s of qh[l] is the high bit of sub-group s, position l
        qh |= ((q[:, :, s, :] >> 4) & 1) << s
    out[..., 16:48] = qh
    qg = (q & 0xF).reshape(n, nb, 4, 2, 32)
    out[..., 48:176] = (qg[:, :, :, 0, :] | (qg[:, :, :, 1, :] << 4)).reshape(n, nb, 128)
    return out.reshape(n, -1)


def quantize_q6_k(w: np.ndarray) -> np.ndarray:
    """[N][K] -> [N][K/256*210] (quant_q6k.go:8-16 layout)."""
    n, k = w.shape
    nb = k // 256
    b = w.reshape(n, nb, 16, 16).astype(np.float32)
    scale = np.abs(b).max(axis=3) / 32.0
    dbits = _f16_bits(scale.max(axis=2) / 127.0)
    d = _f16_value(dbits)
    safe = lambda v: np.where(v > 0, v, 1.0)
    sc = np.where(d[..., None] > 0, np.clip(np.rint(scale / safe(d)[..., None]), -128, 127), 0).astype(np.int8)
    ds = (d[..., None] * sc.astype(np.float32)).astype(np.float32)
    q = np.where(ds[..., None] != 0, np.rint(b / np.where(ds != 0, ds, 1.0)[..., None]), 0)
    q = (np.clip(q, -32, 31) + 32).astype(np.uint8).reshape(n, nb, 256)
    out = np.zeros((n, nb, 210), np.uint8)
    for half in range(2):  # 128-element halves, quant_q6k.go:343-366
        e = q[:, :, half * 128:(half + 1) * 128].reshape(n, nb, 4, 32)  # (+0, +32, +64, +96) x l
        ql = np.zeros((n, nb, 64), np.uint8)
        ql[..., 0:32] = (e[:, :, 0] & 0xF) | ((e[:, :, 2] & 0xF) << 4)
        ql[..., 32:64] = (e[:, :, 1] & 0xF) | ((e[:, :, 3] & 0xF) << 4)
        qh = ((e[:, :, 0] >> 4) & 3) | (((e[:, :, 1] >> 4) & 3) << 2) | (((e[:, :, 2] >> 4) & 3) << 4) | (((e[:, :, 3] >> 4) & 3) << 6)
        out[..., half * 64:(half + 1) * 64] = ql
        out[..., 128 + half * 32:128 + (half + 1) * 32] = qh
    out[..., 192:208] = sc.view(np.uint8)
    out[..., 208:210] = dbits[..., None].view(np.uint8).reshape(n, nb, 2)
    return out.reshape(n, -1)


def quantize(w: np.ndarray, gtype: int) -> np.ndarray:
    if gtype == GGML_F32:
        return np.ascontiguousarray(w, dtype=np.float32).view(np.uint8).reshape(w.shape[0], -1)
    return {GGML_Q8_0: quantize_q8_0, GGML_Q4_K: quantize_q4_k, GGML_Q5_K: quantize_q5_k,
            GGML_Q6_K: quantize_q6_k}[gtype](w)


# ---------------------------------------------------------------- GGUF I/O --

def _gguf_str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


@dataclass
class ModelSpec:
    """Architecture and quantisation of a synthetic nomic-bert model."""
    layers: int = 12
    hidden: int = 768
    heads: int = 12
    ffn: int = 3072
    vocab: int = 30522
    context: int = 2048
    eps: float = 1e-12
    rope_base: float = 1000.0
    embd_type: int = GGML_Q8_0
    # per-projection types (attn_qkv, attn_output, ffn_up, ffn_gate, ffn_down)
    weight_types: tuple = (GGML_Q8_0,) * 5
    seed: int = 0
    std: float = 0.02
    tokens: bool = True  # write tokenizer.ggml.tokens (tokenizer.go:24)


CONFIG_SPECS = {
    # BASELINE.json configs[0] and [2]
    "q8_0": ModelSpec(seed=0),
    # Q4_K for qkv/up/gate, Q6_K for attn_output/ffn_down, Q8_0 token_embd
    "q4_k_m": ModelSpec(weight_types=(GGML_Q4_K, GGML_Q6_K, GGML_Q4_K, GGML_Q4_K, GGML_Q6_K), seed=2),
    # Q6_K and Q5_K variants (token_embd in the same type)
    "q6_k": ModelSpec(weight_types=(GGML_Q6_K,) * 5, embd_type=GGML_Q6_K, seed=3),
    "q5_k": ModelSpec(weight_types=(GGML_Q5_K,) * 5, embd_type=GGML_Q5_K, seed=3),
}


def _tensor_list(spec: ModelSpec):
    """(name, dims [K, N] or [n], type) in file order."""
    H, F = spec.hidden, spec.ffn
    t = [("token_embd.weight", [H, spec.vocab], spec.embd_type),
         ("token_types.weight", [H, 2], GGML_F32),
         ("token_embd_norm.weight", [H], GGML_F32),
         ("token_embd_norm.bias", [H], GGML_F32)]
    dims = {"attn_qkv": [H, 3 * H], "attn_output": [H, H], "ffn_up": [H, F], "ffn_gate": [H, F], "ffn_down": [F, H]}
    for i in range(spec.layers):
        p = f"blk.{i}."
        for w, ty in zip(WEIGHTS, spec.weight_types):
            t.append((p + w + ".weight", dims[w], ty))
            if w == "attn_output":
                t.append((p + "attn_output_norm.weight", [H], GGML_F32))
                t.append((p + "attn_output_norm.bias", [H], GGML_F32))
        t.append((p + "layer_output_norm.weight", [H], GGML_F32))
        t.append((p + "layer_output_norm.bias", [H], GGML_F32))
    return t


def _tensor_data(spec: ModelSpec, idx: int, name: str, dims, gtype: int) -> bytes:
    if name.endswith("norm.weight"):
        return np.ones(dims[0], np.float32).tobytes()
    if name.endswith("norm.bias"):
        return np.zeros(dims[0], np.float32).tobytes()
    rng = np.random.default_rng([spec.seed, idx])
    k, n = dims
    w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(spec.std)).astype(np.float32)
    return quantize(w, gtype).tobytes()


def write_model(path: str, spec: ModelSpec) -> str:
    """Write a GGUF v3 nomic-bert model; returns path."""
    tensors = _tensor_list(spec)
    kv = []
    kv.append(_gguf_str("general.architecture") + struct.pack("<I", 8) + _gguf_str("nomic-bert"))
    for key, val in (("block_count", spec.layers), ("embedding_length", spec.hidden),
                     ("feed_forward_length", spec.ffn), ("attention.head_count", spec.heads),
                     ("context_length", spec.context)):
        kv.append(_gguf_str("nomic-bert." + key) + struct.pack("<II", 4, val))
    kv.append(_gguf_str("nomic-bert.attention.layer_norm_epsilon") + struct.pack("<If", 6, spec.eps))
    kv.append(_gguf_str("nomic-bert.rope.freq_base") + struct.pack("<If", 6, spec.rope_base))
    if spec.tokens:
        vocab = synthetic_vocab(spec.vocab)
        toks = b"".join(_gguf_str(t) for t in vocab)
        kv.append(_gguf_str("tokenizer.ggml.tokens") + struct.pack("<IIQ", 9, 8, spec.vocab) + toks)
    infos, blobs, off = [], [], 0
    for idx, (name, dims, gtype) in enumerate(tensors):
        data = _tensor_data(spec, idx, name, dims, gtype)
        infos.append(_gguf_str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
                     + struct.pack("<IQ", gtype, off))
        pad = (-len(data)) % 32
        blobs.append(data + b"\0" * pad)
        off += len(data) + pad
    header = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv)) + b"".join(kv) + b"".join(infos)
    header += b"\0" * ((-len(header)) % 32)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(header)
        for b in blobs:
            f.write(b)
    os.replace(tmp, path)
    return path


# Synthetic vocabulary: the specials at their BERT ids, then (from id 1000)
# whole words with the SentencePiece prefix, sub-word pieces, letters, digits
# and punctuation with and without the prefix, two CJK characters; the rest
# are filler "▁t<id>" entries.  Enough for the tokenizer's greedy
# matching, fallbacks and [UNK] paths to all occur on ordinary text.
VOCAB_VERSION = 2
_VOCAB_WORDS = ("hello world search query document what is machine learning the cat sat on mat how to cook "
                "pasta quantum computing basics go programming language neural network architecture climate "
                "change effects embedding model a of and in for un token caf \u00fcber").split()
_VOCAB_PIECES = ("ing", "ed", "s", "er", "ly", "ation", "iz", "izer", "able", "ld", "wor", "ize", "ization")
_VOCAB_CHARS = "abcdefghijklmnopqrstuvwxyz0123456789"
_VOCAB_PUNCT = ".,!?;:'\"()-_/"


def synthetic_vocab(n: int) -> list[str]:
    special = {0: "[PAD]", 100: "[UNK]", 101: "[CLS]", 102: "[SEP]", 103: "[MASK]"}
    entries = ["\u2581" + w for w in _VOCAB_WORDS] + list(_VOCAB_PIECES)
    entries += ["\u2581" + c for c in _VOCAB_CHARS] + list(_VOCAB_CHARS)
    entries += ["\u2581" + c for c in _VOCAB_PUNCT] + ["\u2581\u4e2d", "\u2581\u6587"]
    entries = list(dict.fromkeys(entries))  # unique, first occurrence kept
    vocab = [special.get(i, f"\u2581t{i}") for i in range(n)]
    for j, e in enumerate(entries):
        if 1000 + j < n:
            vocab[1000 + j] = e
    return vocab


def cached_model(name_or_spec, directory: str | None = None) -> str:
    """Path of a synthetic model, written once into `directory` (default
    $LLMEMBED_MODEL_DIR or /tmp/llm_embed_b200_models)."""
    spec = CONFIG_SPECS[name_or_spec] if isinstance(name_or_spec, str) else name_or_spec
    directory = directory or os.environ.get("LLMEMBED_MODEL_DIR", "/tmp/llm_embed_b200_models")
    os.makedirs(directory, exist_ok=True)
    tag = "_".join(str(x) for x in (spec.layers, spec.hidden, spec.heads, spec.ffn, spec.vocab, spec.context,
                                      spec.embd_type, *spec.weight_types, spec.seed,
                                      int(spec.tokens) * VOCAB_VERSION))
    path = os.path.join(directory, f"nomic_{tag}.gguf")
    if not os.path.exists(path):
        write_model(path, spec)
    return path


# ----------------------------------------------------------- token inputs --

def config_inputs(config: int, seed: int | None = None):
    """Packed token ids for BASELINE.json configs 0, 2, 3, 4.

    Returns (ids int32 [sum L], offsets int32 [nseq+1]).  Sequences are the
    valid tokens only ([CLS]=101, body ids U[1000, 30522), [SEP]=102); the
    reference's padding positions are masked keys whose exp(-1e9 - max) is
    exactly 0 (ops_simd.go:73-75) and are excluded from the mean pool
    (pool.go:17-24), so dropping them leaves every valid output unchanged."""
    if config == 0:
        lens = [8]
        seed = 0 if seed is None else seed
    elif config == 2:
        seed = 1 if seed is None else seed
        lens = np.random.default_rng([seed, 1000]).integers(16, 129, size=256).tolist()
    elif config == 3:
        seed = 2 if seed is None else seed
        lens = np.random.default_rng([seed, 1000]).integers(64, 257, size=1024).tolist()
    elif config == 4:
        seed = 3 if seed is None else seed
        lens = [512] * 4096
    else:
        raise ValueError(f"config {config} has no token input")
    return make_ids(lens, seed)


def make_ids(lens, seed: int, vocab: int = 30522):
    rng = np.random.default_rng([seed, 1001])
    offs = np.zeros(len(lens) + 1, np.int32)
    offs[1:] = np.cumsum(lens)
    ids = np.empty(int(offs[-1]), np.int32)
    for s, L in enumerate(lens):
        seq = ids[offs[s]:offs[s + 1]]
        if L >= 1:
            seq[0] = 101
        if L >= 2:
            seq[-1] = 102
            seq[1:-1] = rng.integers(1000 if vocab > 2000 else 104, vocab, size=L - 2)
    return ids, offs


def read_gguf(path: str):
    """Minimal GGUF v2/v3 reader (reader.go:219-280 semantics: exact-typed
    scalar KVs, 32-byte data alignment).  Returns (kv, tensors) where tensors
    maps name -> (ggml_type, dims, memoryview of the data)."""
    with open(path, "rb") as f:
        buf = f.read()
    mv = memoryview(buf)
    pos = 0

    def take(fmt):
        nonlocal pos
        v = struct.unpack_from(fmt, buf, pos)
        pos += struct.calcsize(fmt)
        return v[0] if len(v) == 1 else v

    def string():
        nonlocal pos
        n = take("<Q")
        s = bytes(mv[pos:pos + n]).decode(errors="replace")
        pos += n
        return s

    scalar = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<B", 10: "<Q", 11: "<q", 12: "<d"}

    def value(vt):
        if vt in scalar:
            return take(scalar[vt])
        if vt == 8:
            return string()
        if vt == 9:
            et, n = take("<I"), take("<Q")
            return [value(et) for _ in range(n)]
        raise ValueError(f"unknown value type {vt}")

    if take("<I") != 0x46554747:
        raise ValueError("gguf: invalid magic")
    ver = take("<I")
    if ver not in (2, 3):
        raise ValueError(f"gguf: unsupported version {ver}")
    nt, nkv = take("<Q"), take("<Q")
    kv = {}
    for _ in range(nkv):
        key = string()
        vt = take("<I")
        kv[key] = (vt, value(vt))
    infos = []
    for _ in range(nt):
        name = string()
        nd = take("<I")
        dims = [take("<Q") for _ in range(nd)]
        gtype, off = take("<I"), take("<Q")
        infos.append((name, dims, gtype, off))
    data = (pos + 31) & ~31
    tensors = {}
    for name, dims, gtype, off in infos:
        n = int(np.prod(dims))
        nbytes = row_bytes(gtype, dims[0]) * (n // dims[0])
        tensors[name] = (gtype, dims, mv[data + off:data + off + nbytes])
    return kv, tensors
