"""tsn_gemm_noalloc: the runtime-face GEMM for callers that may not allocate device memory once
running (a real-time audio render thread, where cudaMalloc can take a device-wide lock and stall the
callback; a process whose device memory another framework's pool allocator owns). Its split-operand
scratch is a fixed 8 MiB device array inside the library instead of a cudaMalloc'd buffer.

Checked through the C ABI on two calls in a row (the second reuses the array the first left
behind): against a float64 product of the same f16 weights and f32 X, and against tsn_gemm, the
allocating entry point, with and without bias, with strided weights, at exactly the 8 MiB limit
and one row past it; and that calls after the first change the device's free memory by nothing.

This file sorts last so a run that stops at its first failure has already run every other test."""
import numpy as np
import pytest

import tsn
from conftest import rel_l2

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

LIMIT = 8 << 20          # bytes of the library's static scratch array
GEMM_TOL = 5e-5          # the runtime-face GEMM's gate against float64 (tests/test_gpu_gemm.py)


def _case(rng, M, N, K, ldw, bias=True):
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = (rng.standard_normal((N, ldw), dtype=np.float32) * 0.03).astype(np.float16)
    b = rng.standard_normal(N, dtype=np.float32) if bias else None
    ref = x.astype(np.float64) @ w[:, :K].astype(np.float64).T + (b if bias else 0.0)
    dev_t = (torch.from_numpy(x).cuda(), torch.from_numpy(w.view(np.uint16).astype(np.int16)).cuda(),
             torch.from_numpy(b).cuda() if bias else None)
    return dev_t, ref


CASES = [  # (M, N, K, ldw, bias): 4*M*K (+ 2*N*K when ldw != K) bytes of scratch
    (376, 3072, 1024, 1024, True),        # latent qkv rows of a CFG pair
    (154, 1024, 2048, 2112, True),        # strided weights: packed into the array too
    (188, 6144, 1024, 1024, False),       # no bias
    (2048, 1024, 1024, 1024, True),       # 4*M*K = exactly 8 MiB
]


def test_noalloc_matches_float64_and_allocating_gemm_twice():
    dev = tsn.Device(0)
    try:
        rng = np.random.default_rng(99)
        for (M, N, K, ldw, bias) in CASES:
            (X, W, B), ref = _case(rng, M, N, K, ldw, bias)
            outs = []
            for _ in range(2):      # two calls in a row on the shared array
                got = torch.full((M, N), float("nan"), device="cuda")
                dev.gemm_noalloc(W, X, got, B, M, N, K, K, ldw, N)
                dev.commit()
                outs.append(got.cpu().numpy())
            alloc = torch.full((M, N), float("nan"), device="cuda")
            dev.gemm(True, W, X, alloc, B, M, N, K, K, ldw, N)
            dev.commit()
            a = alloc.cpu().numpy()
            for g in outs:
                assert not np.isnan(g).any(), (M, N, K)
                assert rel_l2(g, ref) < GEMM_TOL, (M, N, K, rel_l2(g, ref))
                assert rel_l2(g, a) < GEMM_TOL, (M, N, K, rel_l2(g, a))
            assert np.array_equal(outs[0], outs[1]), "second call differs from the first"
    finally:
        dev.close()


def test_noalloc_allocates_nothing():
    dev = tsn.Device(0)
    try:
        rng = np.random.default_rng(5)
        M, N, K = 376, 3072, 1024
        (X, W, B), ref = _case(rng, M, N, K, K)
        Y = torch.zeros((M, N), device="cuda")
        dev.gemm_noalloc(W, X, Y, B, M, N, K)        # first call: looks up the array's address
        dev.commit()
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        for _ in range(5):
            dev.gemm_noalloc(W, X, Y, B, M, N, K)
        dev.commit()
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free0, "a call changed the device's free memory"
        assert rel_l2(Y.cpu().numpy(), ref) < GEMM_TOL
    finally:
        dev.close()


def test_noalloc_rejects_oversize():
    dev = tsn.Device(0)
    try:
        M, N, K = 2049, 1024, 1024          # one row past 4*M*K = 8 MiB
        X = torch.zeros((M, K), device="cuda")
        W = torch.zeros((N, K), dtype=torch.int16, device="cuda")
        Y = torch.zeros((M, N), device="cuda")
        assert 4 * M * K > LIMIT
        with pytest.raises(tsn.TsnError) as e:
            dev.gemm_noalloc(W, X, Y, None, M, N, K)
        assert e.value.code == 1 and "8 MiB" in str(e.value)
    finally:
        dev.close()
