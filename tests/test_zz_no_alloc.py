"""le_qgemm_device_noalloc against le_qgemm_device (collected last).

The no-alloc entry point keeps its scratch in one file-scope device array
shared by every call on a device; two calls in a row with different shapes
must each match the allocating entry point on the same weight and input, and
the calls must leave the device's free memory unchanged.
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
            qw.sync()
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
        qw.sync()
        qw.matmul_device_noalloc(x.data_ptr(), M, got.data_ptr())
        torch.cuda.synchronize()
        torch.testing.assert_close(got, ref, rtol=1e-6, atol=1e-6)
    finally:
        qw.close()


def test_noalloc_leaves_free_memory_unchanged():
    """The entry point's contract: no device allocation.  After every kernel
    it launches has run once (module loading allocates on first use), calls
    at the largest allowed M and at a new, smaller shape on a weight that
    never ran le_qgemm_device leave cudaMemGetInfo's free bytes unchanged,
    while le_qgemm_device on a fresh weight grows its own buffer."""
    K, N = 768, 512
    Mmax = QWeight.NOALLOC_MAX_ELEMS // K
    warm = _weight(synth.GGML_Q8_0, N, K, seed=7)
    fresh = _weight(synth.GGML_Q8_0, N, K, seed=8)
    probe = _weight(synth.GGML_Q8_0, N, K, seed=9)
    try:
        x = _x(Mmax, K, 9)
        y = torch.empty(Mmax, N, device="cuda")
        for M in (Mmax, 100, 40):  # fp16 TMA, in-smem dequant and CUDA-core paths
            warm.matmul_device_noalloc(x.data_ptr(), M, y.data_ptr())
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        for M in (Mmax, 77, 40, Mmax):
            fresh.matmul_device_noalloc(x.data_ptr(), M, y.data_ptr())
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free0
        # The allocating entry point on a weight that has not run yet grows
        # its fp16 input buffer (M*K*2 = 8 MiB here), which free memory shows.
        probe.matmul_device(x.data_ptr(), Mmax, y.data_ptr())
        probe.sync()
        assert torch.cuda.mem_get_info()[0] < free0
    finally:
        warm.close()
        fresh.close()
        probe.close()
