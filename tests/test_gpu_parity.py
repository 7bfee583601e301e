"""GPU parity of the CUDA path (through the C ABI) against the CPU oracle.

Tolerances:
  * dequantised weights: bit-exact (float32 bits);
  * every embedding: cosine >= 0.99999 and max |diff| <= 2e-3 against the
    oracle's restatement of the reference's Go forward pass.
"""
import json
import os
import threading

import numpy as np
import pytest

import oracle
from llm_embed_b200 import synth
from llm_embed_b200.embed import Embedder, LlmEmbedError, QWeight, info, init, qgemm
from helpers import small_spec

pytestmark = pytest.mark.gpu

COS_MIN = 0.99999
MAX_ABS = 2e-3
NTHREADS = os.cpu_count() or 8


def log_parity(tag, **fields):
    """Append one JSON record to $LLMEMBED_PARITY_LOG (if set): the parity
    figures behind the committed per-config table."""
    path = os.environ.get("LLMEMBED_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps({"case": tag, **fields}) + "\n")


def assert_parity(got, ref, cos_min=COS_MIN, max_abs=MAX_ABS, tag=None):
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    assert got.shape == ref.shape
    assert np.isfinite(got).all()
    nz = np.linalg.norm(ref, axis=1) > 0
    cos = (got * ref).sum(1)[nz] / (np.linalg.norm(got, axis=1)[nz] * np.linalg.norm(ref, axis=1)[nz])
    err = np.abs(got - ref).max() if got.size else 0.0
    if tag:
        log_parity(tag, n=int(got.shape[0]), min_cos=float(cos.min()) if cos.size else 1.0, max_abs=float(err))
    assert (cos.min() if cos.size else 1.0) >= cos_min, f"min cosine {cos.min():.8f}"
    assert err <= max_abs, f"max abs diff {err:.3e}"
    return cos, err


@pytest.fixture(scope="module")
def ndev():
    return init()


def test_init_and_info(ndev):
    assert ndev >= 1
    s = info()
    assert '"arch": "sm_100a"' in s


# ------------------------------------------------------------ dequant -----

@pytest.mark.parametrize("wtype", [synth.GGML_Q8_0, synth.GGML_Q4_K, synth.GGML_Q5_K, synth.GGML_Q6_K])
def test_dequant_bit_exact(model_path, wtype):
    """Every weight of a 2-layer model: device dequant == DequantWeightMatrix
    (gemm.go:221) bit for bit; the fp16 operands == round-to-nearest of it."""
    path = model_path(small_spec(weight_type=wtype, embd_type=wtype))
    _, tensors = synth.read_gguf(path)
    e = Embedder.Load(path)
    try:
        for layer in range(2):
            for which, name in enumerate(synth.WEIGHTS):
                gtype, dims, data = tensors[f"blk.{layer}.{name}.weight"]
                K, N = dims
                ref = oracle.dequant_matrix(gtype, np.frombuffer(data, np.uint8), K, N)
                got = e.dequant(layer, which, mode=0)
                assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), f"{name} layer {layer}"
                got16 = e.dequant(layer, which, mode=1)
                ref16 = ref.astype(np.float16).astype(np.float32)
                assert np.array_equal(got16.view(np.uint32), ref16.view(np.uint32)), f"fp16 {name} layer {layer}"
    finally:
        e.Close()


def test_dequant_subnormal_scales_present(model_path):
    """The Q6_K super-scales of N(0, 0.02) weights are fp16 subnormals; the
    bit-exact test above covers them only if they occur."""
    path = model_path(small_spec(weight_type=synth.GGML_Q6_K, embd_type=synth.GGML_Q6_K))
    _, tensors = synth.read_gguf(path)
    _, _, data = tensors["blk.0.attn_qkv.weight"]
    d = np.frombuffer(data, np.uint8).reshape(-1, 210)[:, 208:210].copy().view(np.uint16)
    assert ((d & 0x7C00) == 0).any()


# ------------------------------------------------------------ forward -----

def _oracle_embed(path, ids, offs, out_dim=None):
    m = oracle.Model(path)
    try:
        return m.embed_ids(ids, offs, out_dim=out_dim, nthreads=NTHREADS)
    finally:
        m.close()


def test_config0_single_embed(model_path):
    """Q8_0 model, batch 1, 8 tokens (seed 0)."""
    path = model_path("q8_0")
    ids, offs = synth.config_inputs(0)
    e = Embedder.Load(path)
    try:
        got = e.Embed(ids)
    finally:
        e.Close()
    ref = _oracle_embed(path, ids, offs)
    assert_parity(got[None], ref, tag="configs[0] q8_0, batch 1, 8 tokens")


@pytest.mark.parametrize("name,config,nseq", [("q8_0", 2, 256), ("q4_k_m", 3, 64), ("q6_k", 4, 16), ("q5_k", 4, 16)])
def test_config_parity(model_path, name, config, nseq):
    """configs[2..4] on their 12-layer models against the oracle: the whole
    configs[2] batch (256 sequences, the tcgen05 GEMMs with the fused
    LayerNorm and the short-sequence attention), 64 configs[3] sequences
    (Q4_K/Q6_K, lengths 64..256: both attention kernels) and 16 configs[4]
    sequences of 512 tokens per Q6_K and Q5_K (8,192 tokens: fused
    LayerNorm, long-sequence attention)."""
    path = model_path(name)
    ids, offs = synth.config_inputs(config)
    offs = offs[:nseq + 1]
    ids = ids[:offs[-1]]
    e = Embedder.Load(path)
    try:
        got = e.EmbedIDs(ids, offs)
    finally:
        e.Close()
    ref = _oracle_embed(path, ids, offs)
    assert_parity(got, ref, tag=f"configs[{config}] {name}, first {nseq} sequences ({int(offs[-1])} tokens)")


def test_edge_lengths(model_path):
    """Empty sequence (zero vector), length 1, 2, ragged, and the maximum
    context length, in one packed call."""
    spec = small_spec(context=2048)
    path = model_path(spec)
    lens = [0, 1, 2, 65, 0, 127, 2048]
    ids, offs = synth.make_ids(lens, seed=5, vocab=spec.vocab)
    e = Embedder.Load(path)
    try:
        got = e.EmbedIDs(ids, offs)
    finally:
        e.Close()
    ref = _oracle_embed(path, ids, offs)
    assert np.all(got[0] == 0) and np.all(got[4] == 0)
    assert_parity(got, ref)


@pytest.mark.parametrize("lens", [
    [128, 129, 64, 65, 16, 1, 130, 63],            # 596 tokens: fused LayerNorm GEMMs
    [128, 129, 1, 64],                             # 322 tokens
    [100, 5, 3],                                   # 108 tokens: mid-size GEMMs, tcgen05 attention
])
def test_attention_length_classes(model_path, lens):
    """Sequences on both sides of every attention boundary (64-key boxes,
    the 128-token short class, the long kernel from 129) in batches that run
    the tensor-core paths, against the oracle; and each sequence equals
    itself in a batch of the other sequences reordered."""
    spec = small_spec(context=512)
    path = model_path(spec)
    ids, offs = synth.make_ids(lens, seed=21, vocab=spec.vocab)
    e = Embedder.Load(path)
    try:
        got = e.EmbedIDs(ids, offs)
        order = list(range(len(lens)))[::-1]
        rid = np.concatenate([ids[offs[i]:offs[i + 1]] for i in order])
        roffs = np.concatenate([[0], np.cumsum([lens[i] for i in order])]).astype(np.int32)
        rev = e.EmbedIDs(rid, roffs)
    finally:
        e.Close()
    for k, i in enumerate(order):
        assert np.array_equal(rev[k].view(np.uint32), got[i].view(np.uint32)), f"sequence {i}"
    ref = _oracle_embed(path, ids, offs)
    assert_parity(got, ref)


def test_short_attention_packing_is_invisible(model_path):
    """The tensor-core short attention packs sequences of at most 64 tokens
    two to a 128-row unit, paired in length order, and runs the units
    longest first.  A sequence's embedding must not depend on its partner:
    the same short sequences in three batches that pair them differently
    (another order, one more short sequence shifting every pair, a lone
    short one left unpaired) give the same bits, and match the oracle."""
    spec = small_spec(context=512)
    path = model_path(spec)
    shorts = [64, 64, 63, 33, 32, 17, 16, 9, 2, 1, 48]
    longs = [65, 128, 129, 97]
    lens = shorts + longs  # 11 short: one left alone
    ids, offs = synth.make_ids(lens, seed=31, vocab=spec.vocab)
    seqs = [ids[offs[i]:offs[i + 1]] for i in range(len(lens))]

    def batch(order, extra=()):
        parts = [seqs[i] for i in order] + list(extra)
        o = np.concatenate([[0], np.cumsum([len(p) for p in parts])]).astype(np.int32)
        return np.concatenate(parts).astype(np.int32), o

    e = Embedder.Load(path)
    try:
        got = e.EmbedIDs(ids, offs)
        order = list(range(len(lens)))[::-1]
        b_ids, b_offs = batch(order)
        rev = e.EmbedIDs(b_ids, b_offs)
        extra = synth.make_ids([40], seed=32, vocab=spec.vocab)[0]
        c_ids, c_offs = batch(range(len(lens)), [extra])  # 12 short: pairs shift
        more = e.EmbedIDs(c_ids, c_offs)
    finally:
        e.Close()
    assert offs[-1] >= 64  # the tensor-core attention path
    for k, i in enumerate(order):
        assert np.array_equal(rev[k].view(np.uint32), got[i].view(np.uint32)), f"reversed, sequence {i}"
    assert np.array_equal(more[:len(lens)].view(np.uint32), got.view(np.uint32))
    assert_parity(got, _oracle_embed(path, ids, offs), tag="short attention packing")


def test_context_length_enforced(model_path):
    spec = small_spec(context=512, seed=12)
    path = model_path(spec)
    e = Embedder.Load(path)
    try:
        ids, offs = synth.make_ids([513], seed=1, vocab=spec.vocab)
        with pytest.raises(LlmEmbedError):
            e.EmbedIDs(ids, offs)
        ids, offs = synth.make_ids([512], seed=1, vocab=spec.vocab)
        assert_parity(e.EmbedIDs(ids, offs), _oracle_embed(path, ids, offs))
    finally:
        e.Close()


@pytest.mark.parametrize("dim", [512, 256, 64, 1])
def test_matryoshka_truncation(model_path, dim):
    """SetTargetDim + truncate/renormalise (embedder.go:66-68, :142)."""
    path = model_path(small_spec())
    ids, offs = synth.make_ids([9, 33, 70], seed=2, vocab=2048)
    e = Embedder.Load(path)
    try:
        e.SetTargetDim(dim)
        assert e.Dim() == dim
        got = e.EmbedIDs(ids, offs)
    finally:
        e.Close()
    ref = _oracle_embed(path, ids, offs, out_dim=dim)
    assert got.shape == (3, dim)
    assert np.allclose(np.linalg.norm(got, axis=1), 1.0, atol=1e-5)
    if dim > 1:
        assert_parity(got, ref)
    else:
        assert np.array_equal(np.sign(got), np.sign(ref))


def test_set_target_dim_clamps(model_path):
    e = Embedder.Load(model_path(small_spec()))
    try:
        e.SetTargetDim(10_000)
        assert e.Dim() == 768
        e.SetTargetDim(0)
        assert e.Dim() == 1
    finally:
        e.Close()


def test_batch_equals_single_bitwise(model_path):
    """EmbedBatch([x]) == Embed(x) and an 8-sequence batch == 8 singles, bit
    for bit (embedder_test.go:116-145, :212-253)."""
    e = Embedder.Load(model_path(small_spec()))
    try:
        ids, offs = synth.make_ids([5, 9, 3, 12, 7, 8, 4, 6], seed=3, vocab=2048)
        seqs = [ids[offs[i]:offs[i + 1]] for i in range(8)]
        batch = e.EmbedBatch(seqs)
        for s, b in zip(seqs, batch):
            one = e.Embed(s)
            assert np.array_equal(one.view(np.uint32), b.view(np.uint32))
        assert np.array_equal(e.EmbedBatch([seqs[0]])[0].view(np.uint32), e.Embed(seqs[0]).view(np.uint32))
    finally:
        e.Close()


@pytest.mark.parametrize("wtype", [synth.GGML_Q8_0, synth.GGML_Q4_K, synth.GGML_Q5_K, synth.GGML_Q6_K])
def test_small_fused_forward(model_path, wtype):
    """Calls of <= 16 tokens run the whole encoder in one cooperative kernel:
    it matches the oracle, and each sequence equals, bit for bit, the same
    sequence inside a 40-token batch run by the separate kernels."""
    path = model_path(small_spec(weight_type=wtype, embd_type=wtype))
    e = Embedder.Load(path)
    try:
        ids, offs = synth.make_ids([3, 7, 1, 5, 6, 9, 4, 5], seed=9, vocab=2048)
        lens = np.diff(offs)
        batch = e.EmbedIDs(ids, offs)                      # 40 tokens: separate kernels
        first = e.EmbedIDs(ids[:16], offs[:5])             # 16 tokens: fused kernel
        assert np.array_equal(first.view(np.uint32), batch[:4].view(np.uint32))
        for i in range(len(lens)):
            one = e.EmbedIDs(ids[offs[i]:offs[i + 1]], np.array([0, lens[i]], np.int32))
            assert np.array_equal(one[0].view(np.uint32), batch[i].view(np.uint32)), f"sequence {i}"
        ref = _oracle_embed(path, ids[:16], offs[:5])
        assert_parity(first, ref)
    finally:
        e.Close()


REF_TEXTS = ["hello world", "what is machine learning", "the cat sat on the mat", "how to cook pasta",
             "quantum computing basics", "go programming language", "neural network architecture",
             "climate change effects"]


def test_embed_text_api(model_path):
    """Embed(text) = TaskPrefix + text through the GGUF's tokenizer, then the
    forward (embedder.go:46-70): equal to embedding those ids, and to the
    oracle; Matryoshka truncation through the text API (TestSetTargetDim)."""
    path = model_path(small_spec())
    e = Embedder.Load(path)
    try:
        assert e.TaskPrefix == "search_query: "
        ids = e.tokenizer.Encode("search_query: hello world", e.hparams.context_length)[0]
        v = e.Embed("hello world")
        assert np.array_equal(v.view(np.uint32), e.Embed(ids).view(np.uint32))
        ref = _oracle_embed(path, np.asarray(ids, np.int32), np.array([0, len(ids)], np.int32))
        assert_parity(v[None], ref)
        assert abs(np.linalg.norm(v) - 1.0) < 1e-5
        e.TaskPrefix = ""
        assert not np.array_equal(e.Embed("hello world"), v)
        e.TaskPrefix = "search_query: "
        e.SetTargetDim(256)
        t = e.Embed("hello world")
        assert t.shape == (256,) and abs(np.linalg.norm(t) - 1.0) < 1e-5
    finally:
        e.Close()


def test_embed_batch_texts_match_singles(model_path):
    """TestEmbedBatchParallel (embedder_test.go:212-253) on its eight texts.
    The reference runs one forward per text, so its batch equals its singles
    bit for bit.  Here the batch (76 tokens) runs the tensor-core GEMMs and
    each single (<= 16 tokens) the single-kernel path: equal within the
    parity tolerance, and bit for bit when the batch stays below 64 tokens."""
    e = Embedder.Load(model_path(small_spec()))
    try:
        batch = e.EmbedBatch(REF_TEXTS)
        singles = [e.Embed(t) for t in REF_TEXTS]
        assert_parity(np.stack(batch), np.stack(singles))
        small = e.EmbedBatch(REF_TEXTS[:4])  # 40 tokens
        for t, b in zip(REF_TEXTS[:4], small):
            assert np.array_equal(e.Embed(t).view(np.uint32), b.view(np.uint32))
    finally:
        e.Close()


def test_graph_replay_matches_direct(model_path):
    """Small calls replay a captured CUDA graph after their first (direct)
    run: repeated calls, and device calls with other output pointers, give
    the same bits as the first call."""
    import torch
    e = Embedder.Load(model_path(small_spec()))
    try:
        ids, offs = synth.make_ids([5, 9, 3], seed=4, vocab=2048)
        first = e.EmbedIDs(ids, offs)
        for _ in range(3):
            assert np.array_equal(e.EmbedIDs(ids, offs).view(np.uint32), first.view(np.uint32))
        d_ids = torch.from_numpy(ids).cuda()
        d_offs = torch.from_numpy(offs).cuda()
        outs = [torch.zeros(3, 768, device="cuda") for _ in range(2)]
        torch.cuda.synchronize()  # the model's stream does not order with torch's
        for _ in range(2):
            for o in outs:
                e.embed_device(d_ids.data_ptr(), d_offs.data_ptr(), 3, int(offs[-1]), 9, o.data_ptr(), 0)
        e.sync()
        for o in outs:
            assert np.array_equal(o.cpu().numpy().view(np.uint32), first.view(np.uint32))
    finally:
        e.Close()


def test_concurrent_calls(model_path):
    """16 threads x 3 calls on one model give the single-thread results
    (embedder_test.go:255-305)."""
    e = Embedder.Load(model_path(small_spec()))
    try:
        ids, offs = synth.make_ids([11, 40, 7, 90], seed=4, vocab=2048)
        ref = e.EmbedIDs(ids, offs)
        errs = []

        def work():
            try:
                for _ in range(3):
                    if not np.array_equal(e.EmbedIDs(ids, offs), ref):
                        errs.append("mismatch")
            except Exception as ex:  # noqa: BLE001
                errs.append(repr(ex))

        th = [threading.Thread(target=work) for _ in range(16)]
        for t in th:
            t.start()
        for t in th:
            t.join()
        assert not errs, errs[:3]
    finally:
        e.Close()


def test_load_from_tensor_descs(model_path):
    """le_model_load with caller-parsed tensors (the path a Go host that keeps
    internal/gguf takes) equals le_model_load_gguf bit for bit."""
    path = model_path(small_spec(weight_type=synth.GGML_Q4_K))
    kv, tensors = synth.read_gguf(path)
    from llm_embed_b200.embed import HParams
    hp = HParams(n_layers=kv["nomic-bert.block_count"][1], hidden=kv["nomic-bert.embedding_length"][1],
                 ffn=kv["nomic-bert.feed_forward_length"][1], heads=kv["nomic-bert.attention.head_count"][1],
                 context_length=kv["nomic-bert.context_length"][1],
                 ln_eps=kv["nomic-bert.attention.layer_norm_epsilon"][1],
                 rope_base=kv["nomic-bert.rope.freq_base"][1])
    a = Embedder.LoadTensors([(n, t, d, bytes(b)) for n, (t, d, b) in tensors.items()], hp)
    b = Embedder.Load(path)
    try:
        ids, offs = synth.make_ids([17, 3], seed=6, vocab=2048)
        assert np.array_equal(a.EmbedIDs(ids, offs), b.EmbedIDs(ids, offs))
    finally:
        a.Close()
        b.Close()


def test_errors_are_reported(model_path, tmp_path):
    e = Embedder.Load(model_path(small_spec()))
    try:
        with pytest.raises(LlmEmbedError) as ex:
            e.EmbedIDs(np.array([101, 5000, 102], np.int32), np.array([0, 3], np.int32))
        assert "outside vocab" in str(ex.value)
        with pytest.raises(LlmEmbedError):
            e.EmbedIDs(np.array([101], np.int32), np.array([0, 1], np.int32), out_dim=0)
        with pytest.raises(LlmEmbedError):
            e.EmbedIDs(np.array([101, 102], np.int32), np.array([0, 2, 1], np.int32))
    finally:
        e.Close()
    with pytest.raises(LlmEmbedError) as ex:
        Embedder.Load(str(tmp_path / "missing.gguf"))
    assert ex.value.code == -5
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUF" + b"\0" * 64)
    with pytest.raises(LlmEmbedError):
        Embedder.Load(str(bad))


def test_multi_device_sharding(model_path, ndev):
    """le_embed_ids over several replicas == one replica, bit for bit."""
    if ndev < 2:
        pytest.skip("one GPU")
    path = model_path(small_spec())
    ids, offs = synth.make_ids(list(range(1, 40)), seed=7, vocab=2048)
    one = Embedder.Load(path)
    many = Embedder.Load(path, devices=list(range(ndev)))
    try:
        assert np.array_equal(one.EmbedIDs(ids, offs), many.EmbedIDs(ids, offs))
    finally:
        one.Close()
        many.Close()


# ------------------------------------------------------------ op sweep -----

QTYPES = [synth.GGML_Q8_0, synth.GGML_Q6_K, synth.GGML_Q5_K, synth.GGML_Q4_K]
SWEEP_KN = [(K, N) for K in (768, 3072) for N in (768, 2304, 3072)]


def _sweep_weight(qtype, K, N):
    rng = np.random.default_rng([0, qtype, K, N])
    w = rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)
    return synth.quantize(w, qtype)


def _row_parity(got, ref, tag):
    """Per output row cosine >= 0.99999 and max |diff| <= 4e-3 * rms(ref):
    fp16 operand rounding of x and W against the float32 reference."""
    rms = float(np.sqrt((ref.astype(np.float64) ** 2).mean()))
    err = float(np.abs(got - ref).max())
    cos = (got * ref).sum(1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(ref, axis=1))
    log_parity(tag, min_cos=float(cos.min()), max_abs=err, max_abs_over_rms=err / rms)
    assert err <= 4e-3 * rms, f"max |diff| {err:.3e} vs rms {rms:.3e}"
    assert cos.min() >= COS_MIN, f"min cosine {cos.min():.8f}"


@pytest.mark.parametrize("qtype", QTYPES)
@pytest.mark.parametrize("M", [8, 512])
@pytest.mark.parametrize("K,N", SWEEP_KN)
def test_qgemm_vs_oracle(qtype, M, K, N):
    """configs[1] op sweep at the oracle-sized M (8, 512) for every K, N and
    type: le_qgemm against the reference's prepacked GEMM
    (gemm_avx512.go:67) and its fused MatMulBatch (ops.go:418)."""
    wq = _sweep_weight(qtype, K, N)
    x = np.random.default_rng([1, qtype, M, K, N]).standard_normal((M, K), dtype=np.float32)
    got = qgemm(qtype, wq, N, K, x)
    wd = oracle.dequant_matrix(qtype, wq, K, N)
    _row_parity(got, oracle.gemm(x, wd, NTHREADS), f"configs[1] type {qtype} M={M} K={K} N={N} vs prepacked gemm")
    _row_parity(got, oracle.matmul_batch(qtype, wq, K, N, x, NTHREADS),
                f"configs[1] type {qtype} M={M} K={K} N={N} vs MatMulBatch")


@pytest.mark.parametrize("qtype", QTYPES)
@pytest.mark.parametrize("K,N", SWEEP_KN)
def test_qgemm_full_size_vs_torch(qtype, K, N):
    """configs[1] at M=32768 (too large for the oracle) for every K, N and
    type: the device result against a torch float32 matmul of the oracle's
    exact dequantised weight."""
    import torch
    M = 32768
    wq = _sweep_weight(qtype, K, N)
    x = torch.randn(M, K, device="cuda", generator=torch.Generator("cuda").manual_seed(K + N))
    y = torch.empty(M, N, device="cuda")
    qw = QWeight(qtype, wq, N, K)
    try:
        qw.matmul_device(x.data_ptr(), M, y.data_ptr())
        qw.sync()
    finally:
        qw.close()
    wd = torch.from_numpy(oracle.dequant_matrix(qtype, wq, K, N)).cuda()
    ref = torch.matmul(x, wd.T)
    rms = ref.double().pow(2).mean().sqrt().item()
    err = (y - ref).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(y, ref, dim=1).min().item()
    log_parity(f"configs[1] type {qtype} M={M} K={K} N={N} vs torch fp32", min_cos=cos, max_abs=err,
               max_abs_over_rms=err / rms)
    assert err <= 4e-3 * rms
    assert cos >= COS_MIN


@pytest.mark.parametrize("qtype", [synth.GGML_Q8_0, synth.GGML_Q4_K, synth.GGML_Q6_K])
def test_gemm_paths_bitwise_equal(qtype):
    """The large-batch kernel (fp16 weights via TMA, M >= 256) and the
    in-shared-memory dequant kernel (64 <= M < 256) use the same fp16 operand
    values and MMA order: rows of an M=256 call equal the same rows computed
    at M=255 and M=64, bit for bit."""
    import torch
    K, N = 768, 2304
    rng = np.random.default_rng([7, qtype])
    w = rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)
    qw = QWeight(qtype, synth.quantize(w, qtype), N, K)
    try:
        x = torch.randn(256, K, device="cuda", generator=torch.Generator("cuda").manual_seed(3))
        outs = {}
        for M in (256, 255, 64):
            y = torch.empty(M, N, device="cuda")
            torch.cuda.synchronize()
            qw.matmul_device(x.data_ptr(), M, y.data_ptr())
            torch.cuda.synchronize()
            outs[M] = y
        assert torch.isfinite(outs[256]).all()
        assert torch.equal(outs[256][:255].view(torch.int32), outs[255].view(torch.int32))
        assert torch.equal(outs[256][:64].view(torch.int32), outs[64].view(torch.int32))
    finally:
        qw.close()


def test_large_batch_rows_match_mid_batch(model_path):
    """Batches of 256+ tokens run the out/down projections with the residual
    LayerNorm fused into the GEMM (three CTA pairs per 256-row block, row
    statistics exchanged through global memory); 64..255 tokens run GEMM +
    separate LayerNorm.  Both reduce each row in the same order, so a
    sequence's embedding is the same bits in either, and in a batch of 939
    or 7,033 tokens, including batches whose last token tile is partial."""
    spec = small_spec()
    e = Embedder.Load(model_path(spec))
    try:
        lens = [37, 5, 61, 18, 29, 44, 90, 12, 73, 55, 8, 101, 66, 23, 48, 77, 31, 59]  # 939 tokens
        ids, offs = synth.make_ids(lens, seed=11, vocab=spec.vocab)
        big = e.EmbedIDs(ids, offs)
        k = 4  # 121 tokens
        mid = e.EmbedIDs(ids[:offs[k]], offs[:k + 1])
        assert offs[k] >= 64 and offs[-1] >= 256 and offs[-1] % 128 != 0
        assert np.array_equal(big[:k].view(np.uint32), mid.view(np.uint32))
        # The 939 tokens followed by more sequences, 7,033 tokens in all.
        more = [101] * 61 + [35]
        ids2, offs2 = synth.make_ids(lens + more, seed=11, vocab=spec.vocab)
        assert np.array_equal(ids2[:offs[-1]], ids) and offs2[-1] >= 7000
        huge = e.EmbedIDs(ids2, offs2)
        assert np.array_equal(huge[:len(lens)].view(np.uint32), big.view(np.uint32))
    finally:
        e.Close()
    ref = _oracle_embed(model_path(spec), ids, offs)
    assert_parity(big, ref)


def test_config2_full_batch_properties(model_path):
    """The full configs[2] batch (256 sequences): unit norms, run-to-run
    bit-identical, and oracle parity of a sample of its sequences."""
    path = model_path("q8_0")
    ids, offs = synth.config_inputs(2)
    e = Embedder.Load(path)
    try:
        a = e.EmbedIDs(ids, offs)
        b = e.EmbedIDs(ids, offs)
    finally:
        e.Close()
    assert np.array_equal(a, b)
    assert np.allclose(np.linalg.norm(a, axis=1), 1.0, atol=1e-5)
    pick = [0, 77, 255]
    sub_ids = np.concatenate([ids[offs[i]:offs[i + 1]] for i in pick])
    sub_offs = np.concatenate([[0], np.cumsum([offs[i + 1] - offs[i] for i in pick])]).astype(np.int32)
    ref = _oracle_embed(path, sub_ids, sub_offs)
    assert_parity(a[pick], ref)
