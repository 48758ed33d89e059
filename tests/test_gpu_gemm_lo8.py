"""An experimental split-operand GEMM whose low-order product runs on the e4m3 tensor path
(csrc/gemm_lo8.cu, reached only through tsn_selftest_gemm_lo8; no model path uses it).

X = Xh + Xl with Xh = f16(X): Xh·W on the f16 tensor path, e4m3(2^12 Xl)·e4m3(2^wexp W) on the 8-bit
path into a second accumulator, scaled back in the epilogue. The product must stay close to the
float64 one (well inside the error of a single f16 operand) on ragged shapes; the library's split
f16 GEMM reached through the same hook is checked against float64 with the same bound.
"""
import numpy as np
import pytest

import tsn
from conftest import rel_l2

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

WEXP = 11   # weights N(0, 0.03): |W| * 2^11 stays below e4m3's 448


@pytest.fixture(scope="module")
def dev():
    d = tsn.Device(0)
    yield d
    d.close()


def operands(M, N, K, seed=17):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K), dtype=np.float32) * 2.0
    x[:, :8] *= 30.0   # a few large activations (still below the 2^8 where e4m3 would saturate)
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.03).astype(np.float16)
    b = rng.standard_normal(N).astype(np.float32)
    ref = x.astype(np.float64) @ w.astype(np.float64).T + b
    return x, w, b, ref


def run(dev, x, w, b, M, N, K, mode, bn):
    W = torch.from_numpy(w.view(np.uint16).astype(np.int16)).cuda()
    Y = torch.full((M * N + 64,), float("nan"), dtype=torch.float32, device="cuda")
    dev.selftest_gemm_lo8(W, torch.from_numpy(x).cuda(), Y, torch.from_numpy(b).cuda(), M, N, K, WEXP, mode, bn)
    y = Y.cpu().numpy()
    assert np.isnan(y[M * N:]).all(), "wrote past the output"
    return y[:M * N].reshape(M, N)


@pytest.mark.parametrize("M,N,K,bn", [(200, 1000, 1024, 176), (376, 512, 3072, 256), (129, 250, 64, 128),
                                      (376, 1056, 3072, 176)])
def test_lo8_gemm_vs_float64(dev, M, N, K, bn):
    x, w, b, ref = operands(M, N, K)
    y = run(dev, x, w, b, M, N, K, 0, bn)
    e = rel_l2(y, ref)
    single = rel_l2(x.astype(np.float16).astype(np.float64) @ w.astype(np.float64).T + b, ref)
    print(f"M={M} N={N} K={K} bn={bn}: e4m3 low-order product {e:.3g}, single f16 operand {single:.3g}")
    assert np.isfinite(y).all()
    assert e < 2e-5 and e < single / 8, (e, single)


@pytest.mark.parametrize("mode,bn,N", [(1, 128, 512), (1, 256, 512), (2, 176, 1000), (3, 176, 1000), (3, 256, 512),
                                       (3, 128, 250)])
def test_split_f16_through_the_hook_vs_float64(dev, mode, bn, N):
    """mode 1: the library's split GEMM; modes 2 and 3: the same product with 64- and 32-wide K blocks."""
    M, K = 376, 1024
    x, w, b, ref = operands(M, N, K)
    # the f16 residual itself rounds (and goes subnormal below 2^-14): ~4e-6 on these operands
    assert rel_l2(run(dev, x, w, b, M, N, K, mode, bn), ref) < 2e-5


def test_lo8_gemm_timing_vs_split(dev):
    """Times the forms at the shapes of the step's w1/w3 (376 x 8192 x 3072), modulation
    (376 x 131072 x 1024) and qkv (376 x 3072 x 1024) GEMMs: the mean of 10 launches, each timed alone
    after an L2-evicting write, and (+ "warm") without it. Prints the table; asserts only that every
    configuration ran."""
    rows = []
    for M, N, K, tag in [(376, 8192, 3072, "w1/w3"), (376, 131072, 1024, "modulation"), (376, 3072, 1024, "qkv")]:
        rng = np.random.default_rng(1)
        x = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).cuda()
        w = torch.from_numpy((rng.standard_normal((N, K), dtype=np.float32) * 0.03).astype(np.float16).view(np.int16)).cuda()
        Y = torch.empty(M * N, dtype=torch.float32, device="cuda")
        for mode, bn in [(1, 128), (1, 256), (0, 128), (0, 176), (0, 256), (5, 256), (4, 256), (4, 176),
                         (2, 176), (3, 176), (2, 256), (3, 256), (6, 176), (7, 176)]:
            ms = dev.selftest_gemm_lo8(w, x, Y, None, M, N, K, WEXP, mode, bn, reps=10)
            name = ["e4m3 lo", "split f16", "split f16 kb64", "split f16 kb32"][mode & 3] + (", warm L2" if mode & 4 else "")
            rows.append((tag, name, bn, ms * 1e3, 2.0 * M * N * K / (ms * 1e-3) / 1e12))
        del w, Y
    for r in rows:
        print(f"{r[0]:>10}  {r[1]:<20} bn {r[2]:>3}  {r[3]:8.2f} us  {r[4]:6.1f} TFLOP/s (algorithmic)")
    assert all(r[3] > 0 for r in rows)
