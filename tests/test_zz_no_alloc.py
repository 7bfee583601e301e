"""le_qgemm_device_noalloc against le_qgemm_device (collected last).

The no-alloc entry point keeps its scratch in one file-scope device array
shared by every call on a device; two calls in a row with different shapes
must each match the allocating entry point on the same weight and input.
"""
import numpy as np
import pytest
import torch

from llm_embed_b200 import synth
from llm_embed_b200.embed import LlmEmbedError, QWeight

pytestmark = pytest.mark.gpu

LE_EINVAL = -1


def _weight(qtype, N, K, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    return QWeight(qtype, synth.quantize(w, qtype), N, K)


def _x(M, K, seed):
    return torch.randn(M, K, device="cuda", generator=torch.Generator("cuda").manual_seed(seed))


@pytest.mark.parametrize("qtype,N,K", [(synth.GGML_Q8_0, 768, 768), (synth.GGML_Q4_K, 1024, 768)])
def test_noalloc_matches_qgemm_device_two_calls(qtype, N, K):
    """Call 1 (tensor-core path, M=512) then call 2 (M=40, small-M path and
    a shorter input over the same scratch) both equal le_qgemm_device."""
    qw = _weight(qtype, N, K, seed=qtype)
    try:
        for M, seed in ((512, 1), (40, 2)):
            x = _x(M, K, seed)
            ref = torch.empty(M, N, device="cuda")
            got = torch.full((M, N), float("nan"), device="cuda")
            torch.cuda.synchronize()
            qw.matmul_device(x.data_ptr(), M, ref.data_ptr())
            torch.cuda.synchronize()
            qw.matmul_device_noalloc(x.data_ptr(), M, got.data_ptr())
            torch.cuda.synchronize()
            assert torch.isfinite(got).all()
            # Same kernels on the same operands: equal up to a 1e-6 tolerance.
            torch.testing.assert_close(got, ref, rtol=1e-6, atol=1e-6)
    finally:
        qw.close()


def test_noalloc_rejects_oversize():
    """M*K beyond the scratch array is LE_EINVAL before any device work."""
    K = 768
    qw = _weight(synth.GGML_Q8_0, 256, K, seed=5)
    try:
        M = QWeight.NOALLOC_MAX_ELEMS // K + 1
        with pytest.raises(LlmEmbedError) as ei:
            qw.matmul_device_noalloc(1 << 20, M, 1 << 20)
        assert ei.value.code == LE_EINVAL
        assert "scratch limit" in str(ei.value)
        # The largest M that fits still runs.
        M = QWeight.NOALLOC_MAX_ELEMS // K
        x = _x(M, K, 6)
        ref = torch.empty(M, 256, device="cuda")
        got = torch.empty(M, 256, device="cuda")
        torch.cuda.synchronize()
        qw.matmul_device(x.data_ptr(), M, ref.data_ptr())
        torch.cuda.synchronize()
        qw.matmul_device_noalloc(x.data_ptr(), M, got.data_ptr())
        torch.cuda.synchronize()
        torch.testing.assert_close(got, ref, rtol=1e-6, atol=1e-6)
    finally:
        qw.close()
