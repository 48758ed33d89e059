"""tsn_gemm_noalloc: the runtime-face GEMM for callers that may not allocate device memory once
running (a real-time audio render thread, a process whose device memory another allocator owns).
Its split-operand scratch is a fixed 8 MiB device array inside the library instead of a cudaMalloc'd
buffer. Checked through the C ABI against tsn_gemm, the allocating entry point, on two calls in a
row (the second reuses the array the first left behind), plus the size limit.

This file sorts last so a run that stops at its first failure has already run every other test."""
import numpy as np
import pytest

import tsn
from conftest import rel_l2

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _case(rng, M, N, K, ldw):
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = (rng.standard_normal((N, ldw), dtype=np.float32) * 0.03).astype(np.float16)
    b = rng.standard_normal(N, dtype=np.float32)
    return (torch.from_numpy(x).cuda(), torch.from_numpy(w.view(np.uint16).astype(np.int16)).cuda(),
            torch.from_numpy(b).cuda())


def test_noalloc_matches_allocating_gemm_twice():
    dev = tsn.Device(0)
    try:
        rng = np.random.default_rng(99)
        for (M, N, K, ldw) in [(376, 3072, 1024, 1024), (154, 1024, 2048, 2112)]:   # second: strided weights
            X, W, B = _case(rng, M, N, K, ldw)
            ref = torch.full((M, N), float("nan"), device="cuda")
            got = torch.full((M, N), float("nan"), device="cuda")
            dev.gemm(True, W, X, ref, B, M, N, K, K, ldw, N)
            dev.gemm_noalloc(W, X, got, B, M, N, K, K, ldw, N)
            dev.commit()
            r, g = ref.cpu().numpy(), got.cpu().numpy()
            assert not np.isnan(g).any()
            assert rel_l2(g, r) < 5e-5
    finally:
        dev.close()


def test_noalloc_rejects_oversize():
    dev = tsn.Device(0)
    try:
        M, N, K = 2048, 1024, 1024          # 4*M*K = 8 MiB of operand scratch plus nothing spare
        X = torch.zeros((M + 64, K), device="cuda")
        W = torch.zeros((N, K), dtype=torch.int16, device="cuda")
        Y = torch.zeros((M + 64, N), device="cuda")
        with pytest.raises(tsn.TsnError) as e:
            dev.gemm_noalloc(W, X, Y, None, M + 64, N, K)
        assert e.value.code == 1 and "8 MiB" in str(e.value)
    finally:
        dev.close()
