"""CPU tests: synthetic GGUF models satisfy the reference's loader contract,
quantisers produce valid blocks, and the oracle forward pass has the
reference's properties."""
import numpy as np
import pytest

import oracle
from llm_embed_b200 import synth
from helpers import MODEL_DIR, small_spec


@pytest.fixture(scope="module")
def tiny_path():
    return synth.cached_model(small_spec(layers=1, vocab=600, seed=41), MODEL_DIR)


def test_gguf_kvs_and_tensors(tiny_path):
    """Exactly-typed hparams (bert.go:98-104, reader.go:293-332), tensor names
    (bert.go:152-207), 32-byte aligned data (reader.go:266-269)."""
    kv, tensors = synth.read_gguf(tiny_path)
    for k in ("block_count", "embedding_length", "feed_forward_length", "attention.head_count", "context_length"):
        assert kv["nomic-bert." + k][0] == 4  # uint32
    for k in ("attention.layer_norm_epsilon", "rope.freq_base"):
        assert kv["nomic-bert." + k][0] == 6  # float32
    assert kv["tokenizer.ggml.tokens"][0] == 9 and len(kv["tokenizer.ggml.tokens"][1]) == 600
    assert tensors["token_embd.weight"][1] == [768, 600]
    assert tensors["blk.0.ffn_down.weight"][1] == [3072, 768]
    assert tensors["token_types.weight"][0] == synth.GGML_F32
    m = oracle.Model(tiny_path)
    assert (m.layers, m.hidden, m.heads, m.ffn, m.max_seq, m.vocab) == (1, 768, 12, 3072, 2048, 600)
    assert abs(m.eps - 1e-12) < 1e-18 and m.rope_base == 1000.0
    m.close()


@pytest.mark.parametrize("gtype,tol", [(synth.GGML_Q8_0, 0.01), (synth.GGML_Q6_K, 0.04), (synth.GGML_Q5_K, 0.08),
                                       (synth.GGML_Q4_K, 0.16)])
def test_quantizers_round_trip(gtype, tol):
    rng = np.random.default_rng(3)
    w = rng.standard_normal((64, 768), dtype=np.float32) * np.float32(0.02)
    wq = synth.quantize(w, gtype)
    assert wq.shape == (64, synth.row_bytes(gtype, 768))
    back = oracle.dequant_matrix(gtype, wq, 768, 64)
    rel = np.linalg.norm(back - w) / np.linalg.norm(w)
    assert rel < tol


def test_q6_k_superscale_is_subnormal():
    rng = np.random.default_rng(4)
    w = rng.standard_normal((8, 256), dtype=np.float32) * np.float32(0.02)
    d = synth.quantize_q6_k(w)[:, 208:210].copy().view(np.uint16)
    assert ((d & 0x7C00) == 0).all() and (d != 0).all()


def test_oracle_embeddings_unit_norm_and_batch_invariant(tiny_path):
    m = oracle.Model(tiny_path)
    ids, offs = synth.make_ids([9, 1, 30, 5], seed=1, vocab=600)
    e = m.embed_ids(ids, offs, nthreads=4)
    assert np.allclose(np.linalg.norm(e, axis=1), 1.0, atol=1e-6)
    for i in range(4):
        one = m.embed_ids(ids[offs[i]:offs[i + 1]], np.array([0, offs[i + 1] - offs[i]], np.int32), nthreads=1)
        assert np.array_equal(one[0], e[i])
    m.close()


def test_oracle_padding_is_inert(tiny_path):
    """A padded, masked forward (bert.go:381-386, pool.go:17) gives the same
    pooled embedding as the packed valid tokens."""
    m = oracle.Model(tiny_path)
    ids, offs = synth.make_ids([12], seed=2, vocab=600)
    packed = m.embed_ids(ids, offs, nthreads=2)[0]
    padded = np.concatenate([ids, np.zeros(20, np.int32)])
    mask = np.concatenate([np.ones(12, np.int32), np.zeros(20, np.int32)])
    hid = m.forward(padded, mask)
    pooled = hid[:12].sum(0) / np.float32(12)
    pooled /= np.linalg.norm(pooled.astype(np.float64))
    assert np.allclose(pooled, packed, atol=1e-6)
    m.close()


def test_oracle_gemm_blocking_matches_float64():
    rng = np.random.default_rng(5)
    for M in (1, 6, 7, 13):
        A = rng.standard_normal((M, 300), dtype=np.float32)
        B = rng.standard_normal((70, 300), dtype=np.float32)
        got = oracle.gemm(A, B, 2)
        ref = A.astype(np.float64) @ B.T.astype(np.float64)
        assert np.abs(got - ref).max() < 1e-3


def test_oracle_ops_known_values():
    # GeLU rational tanh clamps at |t| > 4.97 (ops_simd.go:35-39)
    g = oracle.gelu([0.0, 10.0, -10.0])
    assert g[0] == 0.0 and g[1] == 10.0 and g[2] == 0.0
    # softmax: weights more than 10 below the max are exactly 0 (ops_simd.go:73-75)
    p = oracle.softmax([0.0, -10.5, -9.5])
    assert p[1] == 0.0 and p[2] > 0.0 and abs(p.sum() - 1.0) < 1e-6
    # RoPE table row 0 is the identity rotation
    c, s = oracle.rope_table(4, 64, 1000.0)
    assert np.all(c[0] == 1.0) and np.all(s[0] == 0.0)
    x = oracle.layernorm(np.arange(8, dtype=np.float32), np.ones(8), np.zeros(8), 1e-12)
    assert abs(x.mean()) < 1e-6 and abs(x.std() - 1.0) < 1e-4


def test_config_inputs_shapes():
    for cfg, n, lo, hi in ((0, 1, 8, 8), (2, 256, 16, 128), (3, 1024, 64, 256), (4, 4096, 512, 512)):
        ids, offs = synth.config_inputs(cfg)
        L = np.diff(offs)
        assert offs.size == n + 1 and L.min() >= lo and L.max() <= hi
        assert np.all(ids[offs[:-1]] == 101) and np.all(ids[offs[1:] - 1] == 102)
        body = np.delete(ids, np.concatenate([offs[:-1], offs[1:] - 1]))
        assert body.min() >= 1000 and body.max() < 30522
