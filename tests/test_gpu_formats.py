"""GPU tests of the weight formats and call-ordering rules beyond the
quantised configs: the reference's known-answer blocks through the device
repack, dequant and GEMM; F32 projection weights and token embedding
(DequantWeightMatrix case 0, getEmbedding case 0); the type ids 15/16 that
DequantWeightMatrix decodes as Q5_K; and device calls on several streams."""
import json
import os

import numpy as np
import pytest

import oracle
from llm_embed_b200 import synth
from llm_embed_b200.embed import Embedder, HParams, QWeight
from helpers import small_spec
from test_gpu_parity import NTHREADS, assert_parity

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "known_answers.json")
CASES = json.load(open(GOLDEN))["cases"]


def expected_values(case):
    n, v = case["n"], case["values"]
    if "all" in v:
        return np.full(n, v["all"], np.float32)
    if "even" in v:
        return np.where(np.arange(n) % 2 == 0, v["even"], v["odd"]).astype(np.float32)
    if "index_multiple_of_32" in v:
        return np.where(np.arange(n) % 32 == 0, v["index_multiple_of_32"], v["other"]).astype(np.float32)
    return np.repeat(np.asarray(v["per16"], np.float32), 16)


def _hparams(kv):
    return HParams(n_layers=kv["nomic-bert.block_count"][1], hidden=kv["nomic-bert.embedding_length"][1],
                   ffn=kv["nomic-bert.feed_forward_length"][1], heads=kv["nomic-bert.attention.head_count"][1],
                   context_length=kv["nomic-bert.context_length"][1],
                   ln_eps=kv["nomic-bert.attention.layer_norm_epsilon"][1],
                   rope_base=kv["nomic-bert.rope.freq_base"][1])


def _tiny_model_tensors(gtype, qkv_rows):
    """A 1-layer, hidden-256 model (4 heads of 64, FFN 256) whose attn_qkv
    rows are `qkv_rows` (768 GGUF rows of K=256 of type gtype); the other
    tensors random of the same type."""
    H, FF, V = 256, 256, 64
    rng = np.random.default_rng(17)

    def q(n, k):
        return synth.quantize(rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02), gtype).tobytes()

    ones, zeros = np.ones(H, np.float32).tobytes(), np.zeros(H, np.float32).tobytes()
    t = [("token_embd.weight", synth.GGML_Q8_0, [H, V],
          synth.quantize(rng.standard_normal((V, H), dtype=np.float32) * np.float32(0.02), synth.GGML_Q8_0).tobytes()),
         ("token_types.weight", synth.GGML_F32, [H, 2], (rng.standard_normal(2 * H) * 0.02).astype(np.float32).tobytes()),
         ("token_embd_norm.weight", synth.GGML_F32, [H], ones), ("token_embd_norm.bias", synth.GGML_F32, [H], zeros),
         ("blk.0.attn_qkv.weight", gtype, [H, 3 * H], qkv_rows.tobytes()),
         ("blk.0.attn_output.weight", gtype, [H, H], q(H, H)),
         ("blk.0.attn_output_norm.weight", synth.GGML_F32, [H], ones),
         ("blk.0.attn_output_norm.bias", synth.GGML_F32, [H], zeros),
         ("blk.0.ffn_up.weight", gtype, [H, FF], q(FF, H)), ("blk.0.ffn_gate.weight", gtype, [H, FF], q(FF, H)),
         ("blk.0.ffn_down.weight", gtype, [FF, H], q(H, FF)),
         ("blk.0.layer_output_norm.weight", synth.GGML_F32, [H], ones),
         ("blk.0.layer_output_norm.bias", synth.GGML_F32, [H], zeros)]
    hp = HParams(n_layers=1, hidden=H, ffn=FF, heads=4, context_length=512, ln_eps=1e-12, rope_base=1000.0)
    return t, hp


@pytest.mark.parametrize("gtype", sorted({c["type"] for c in CASES}))
def test_known_answer_blocks_device_dequant(gtype):
    """The reference's known-answer blocks (dot_test.go:120-176,
    dot_q5k_test.go:84-222, dot_q6k_test.go:59-104) as the rows of a weight
    uploaded through le_model_load: the device repack + dequant gives the
    known values bit for bit (mode 0) and their fp16 rounding (mode 1)."""
    cases = [c for c in CASES if c["type"] == gtype]
    K, N = 256, 768
    rows, want = [], []
    for r in range(N):
        c = cases[r % len(cases)]
        block = np.frombuffer(bytes.fromhex(c["block"]), np.uint8)
        reps = K // c["n"]
        rows.append(np.tile(block, reps))
        want.append(np.tile(expected_values(c), reps))
    tensors, hp = _tiny_model_tensors(gtype, np.stack(rows))
    want = np.stack(want).astype(np.float32)
    e = Embedder.LoadTensors(tensors, hp)
    try:
        got = e.dequant(0, 0, mode=0)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        got16 = e.dequant(0, 0, mode=1)
        assert np.array_equal(got16.view(np.uint32), want.astype(np.float16).astype(np.float32).view(np.uint32))
    finally:
        e.Close()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
@pytest.mark.parametrize("M", [1, 64, 256])
def test_known_answer_blocks_device_gemm(case, M):
    """Each known-answer block through le_qgemm (the M < 64 CUDA-core path,
    the in-shared-memory dequant tcgen05 path and the fp16-operand TMA path):
    x = the case's constant input gives the case's dot product.  When every
    value is exact in fp16 and the sums are exact in float32, bit for bit."""
    block = np.frombuffer(bytes.fromhex(case["block"]), np.uint8)
    n = case["n"]
    K = 64 if n == 32 else n
    reps = K // n
    wq = np.stack([np.tile(block, reps)] * 256)  # N = 256 identical rows
    qw = QWeight(case["type"], wq, 256, K)
    try:
        x = np.full((M, K), case["x"], np.float32)
        import torch
        dx = torch.from_numpy(x).cuda()
        dy = torch.empty(M, 256, device="cuda")
        torch.cuda.synchronize()
        qw.matmul_device(dx.data_ptr(), M, dy.data_ptr())
        qw.sync()
        y = dy.cpu().numpy()
    finally:
        qw.close()
    vals = np.tile(expected_values(case), reps)
    v16 = vals.astype(np.float16).astype(np.float32)
    want = float((v16.astype(np.float64) * np.float64(np.float16(case["x"]))).sum())
    assert abs(case["dot"] * reps - float((vals.astype(np.float64) * case["x"]).sum())) <= 1e-6 * abs(case["dot"] * reps)
    if np.array_equal(v16, vals) and abs(want) < 2 ** 24:
        assert np.all(y == np.float32(want)), (y.min(), y.max(), want)
    else:
        assert np.abs(y - want).max() <= 1e-6 * abs(want)


def test_f32_weights_and_token_embd(model_path):
    """F32 projection weights (DequantWeightMatrix case 0, gemm.go:257-263)
    and an F32 token embedding (getEmbedding case 0, bert.go:291-294): the
    stored floats come back exactly from le_dequant, and embeddings over the
    small, mid and large batch paths match the oracle."""
    spec = small_spec(weight_type=synth.GGML_F32, embd_type=synth.GGML_F32, seed=13)
    path = model_path(spec)
    _, tensors = synth.read_gguf(path)
    e = Embedder.Load(path)
    try:
        for which, name in enumerate(synth.WEIGHTS):
            _, dims, data = tensors[f"blk.1.{name}.weight"]
            K, N = dims
            ref = np.frombuffer(data, np.float32).reshape(N, K)
            assert np.array_equal(e.dequant(1, which, mode=0).view(np.uint32), ref.view(np.uint32)), name
            ref16 = ref.astype(np.float16).astype(np.float32)
            assert np.array_equal(e.dequant(1, which, mode=1).view(np.uint32), ref16.view(np.uint32)), name
        m = oracle.Model(path)
        try:
            for lens in ([8], [5, 9, 40, 3], [130, 100, 70, 12]):
                ids, offs = synth.make_ids(lens, seed=sum(lens), vocab=spec.vocab)
                got = e.EmbedIDs(ids, offs)
                assert_parity(got, m.embed_ids(ids, offs, nthreads=NTHREADS),
                              tag=f"F32 weights + F32 token_embd, lengths {lens}")
        finally:
            m.close()
    finally:
        e.Close()


def test_weight_type_ids_15_16_decode_as_q5_k(model_path):
    """DequantWeightMatrix (gemm.go:240) reads type ids 15 and 16 as Q5_K:
    a model whose Q5_K projections carry those ids gives the same weights
    and embeddings, bit for bit."""
    path = model_path(small_spec(weight_type=synth.GGML_Q5_K, seed=14))
    kv, tensors = synth.read_gguf(path)
    hp = _hparams(kv)
    plain = [(n, t, d, bytes(b)) for n, (t, d, b) in tensors.items()]
    relabeled = [(n, (15 if ("ffn_" in n or "attn_qkv" in n) else 16) if (t == synth.GGML_Q5_K and n.startswith("blk."))
                  else t, d, b) for n, t, d, b in plain]
    assert any(t == 15 for _, t, _, _ in relabeled) and any(t == 16 for _, t, _, _ in relabeled)
    a = Embedder.LoadTensors(relabeled, hp)
    b = Embedder.LoadTensors(plain, hp)
    try:
        ids, offs = synth.make_ids([17, 3, 90], seed=6, vocab=2048)
        assert np.array_equal(a.EmbedIDs(ids, offs).view(np.uint32), b.EmbedIDs(ids, offs).view(np.uint32))
        for which in range(5):
            assert np.array_equal(a.dequant(0, which).view(np.uint32), b.dequant(0, which).view(np.uint32))
    finally:
        a.Close()
        b.Close()


def test_device_calls_on_two_streams_are_ordered(model_path):
    """le_embed_ids_device calls of one model on two caller streams share the
    model's workspace; the library orders them on the GPU, so interleaved
    calls on two streams give the serial results bit for bit.  The batches
    run the fused-LayerNorm GEMMs, whose statistics words live in the
    workspace, and the short- and long-sequence attention."""
    import torch
    e = Embedder.Load(model_path(small_spec(context=512)))
    try:
        batches = []
        for k, lens in enumerate(([130, 100, 70, 12, 300], [64, 129, 5, 200, 77, 31])):
            ids, offs = synth.make_ids(lens, seed=40 + k, vocab=2048)
            ref = e.EmbedIDs(ids, offs)
            batches.append((torch.from_numpy(ids).cuda(), torch.from_numpy(offs).cuda(), len(lens),
                            int(offs[-1]), max(lens), ref))
        streams = [torch.cuda.Stream(), torch.cuda.Stream()]
        calls = [(batches[(i // 2) % 2], torch.full((batches[(i // 2) % 2][2], 768), float("nan"), device="cuda"))
                 for i in range(8)]
        torch.cuda.synchronize()
        # Back to back, adjacent calls on different streams.
        for i, ((d_ids, d_offs, n, T, maxlen, _), o) in enumerate(calls):
            e.embed_device(d_ids.data_ptr(), d_offs.data_ptr(), n, T, maxlen, o.data_ptr(), streams[i % 2].cuda_stream)
        outs = [(o, b[5]) for b, o in calls]
        torch.cuda.synchronize()
        e.sync()
        for o, ref in outs:
            assert np.array_equal(o.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    finally:
        e.Close()
