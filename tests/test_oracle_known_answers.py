"""The oracle against the reference's own known-answer quant tests
(tests/golden/known_answers.json, made by tests/golden/make_golden.py) and
the reference's internal-consistency checks (fused dot == dequant-then-dot)."""
import json
import os

import numpy as np
import pytest

import oracle
from llm_embed_b200 import synth

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


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_known_answer_dequant(case):
    block = np.frombuffer(bytes.fromhex(case["block"]), np.uint8)
    got = oracle.dequant(case["type"], block, case["n"])
    assert np.array_equal(got, expected_values(case))


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_known_answer_dot(case):
    """The fused dequant.dot of MatMulBatch (ops.go:418) on the case's x."""
    block = np.frombuffer(bytes.fromhex(case["block"]), np.uint8)
    x = np.full((1, case["n"]), case["x"], np.float32)
    got = oracle.matmul_batch(case["type"], block, case["n"], 1, x)[0, 0]
    assert abs(got - case["dot"]) <= 0.01 * max(1.0, abs(case["dot"])) * 1e-3


def test_f16_to_f32_all_patterns():
    """tensor.go:162-191: every non-NaN half converts exactly (subnormals
    normalised, not flushed)."""
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([oracle.f16_to_f32(int(v)) for v in h[::7]], np.float32)
    r = ref[::7]
    ok = np.isnan(r)
    assert np.array_equal(got[~ok].view(np.uint32), r[~ok].view(np.uint32))
    assert np.isnan(got[ok]).all()


@pytest.mark.parametrize("gtype", [synth.GGML_Q4_K, synth.GGML_Q5_K, synth.GGML_Q6_K, synth.GGML_Q8_0])
def test_fused_dot_matches_dequant_then_dot(gtype):
    """dot_q5k_test.go:224-314, dot_q6k_test.go:11-57: the fused dot agrees
    with dequantise-then-dot to relErr 1e-5."""
    rng = np.random.default_rng(42)
    K, N = 768, 16
    w = rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)
    wq = synth.quantize(w, gtype)
    x = (rng.random((3, K), dtype=np.float32) * 2 - 1).astype(np.float32)
    fused = oracle.matmul_batch(gtype, wq, K, N, x)
    wd = oracle.dequant_matrix(gtype, wq, K, N)
    ref = x.astype(np.float64) @ wd.T.astype(np.float64)
    rel = np.abs(fused - ref) / np.maximum(np.abs(ref), 1e-10)
    assert np.median(rel) < 1e-5 and np.abs(fused - ref).max() < 1e-4


def test_q6_k_random_bytes_fixed_scale():
    """dot_q6k_test.go:18-35: random bytes with d = 0x2411."""
    rng = np.random.default_rng(42)
    data = rng.integers(0, 256, size=(3, 210), dtype=np.uint8)
    data[:, 208], data[:, 209] = 0x11, 0x24
    flat = data.reshape(-1)
    x = (rng.random((1, 768), dtype=np.float32) * 2 - 1)
    fused = oracle.matmul_batch(synth.GGML_Q6_K, flat, 768, 1, x)[0, 0]
    wd = oracle.dequant(synth.GGML_Q6_K, flat, 768)
    ref = float(np.dot(wd.astype(np.float64), x[0].astype(np.float64)))
    assert abs(fused - ref) <= 1e-5 * max(abs(ref), 1e-10) + 1e-6
