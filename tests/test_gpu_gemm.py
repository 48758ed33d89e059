"""The tcgen05 GEMM / conv behind the runtime face (Runtime::gemm / Runtime::conv, src/net.mm:14-49).

Mirrors tools/gemm_bench.cpp and tools/conv_bench.cpp of the reference: seeded inputs, weights
N(0,1)*0.03 rounded to f16, outputs NaN-filled so unwritten elements show up, a guard band
checked for clobbering, shapes of the real DiT. The CPU reference is float64 on the same f16
weights and the f32 X: the runtime face passes X as a split f16 operand (hi + lo), so the
tensor-core product matches the f32-activation product to f32 accumulation error.
"""
import numpy as np
import pytest

import tsn
from conftest import rel_l2

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SHAPES = [  # (M, N, K, bias, xpad, ypad, tag)   tools/gemm_bench.cpp:32-47, DiT rows doubled for CFG
    (376, 6144, 1024, True, 0, 0, "latent adaLN"),
    (376, 3072, 1024, True, 0, 0, "latent qkv"),
    (154, 4096, 1024, False, 0, 0, "text ffn w1"),
    (154, 1024, 4096, False, 0, 0, "text ffn w2"),
    (1024, 1024, 1024, True, 0, 0, "square"),
    (43, 1024, 3072, True, 0, 0, "odd M"),
    (16, 1024, 1024, True, 64, 0, "ldx pad"),
    (77, 1024, 1024, True, 0, 2048, "ldy pad"),
    (1, 6144, 1024, True, 0, 0, "M=1"),
    (50, 100, 72, True, 0, 0, "CUDA-core shape"),
]


@pytest.fixture(scope="module")
def dev():
    d = tsn.Device(0)
    yield d
    d.close()


@pytest.mark.parametrize("M,N,K,bias,xpad,ypad,tag", SHAPES)
def test_gemm_runtime_face(dev, M, N, K, bias, xpad, ypad, tag):
    rng = np.random.default_rng(7)
    ldx, ldy = K + xpad, N + ypad
    x = rng.standard_normal((M, ldx), dtype=np.float32)
    w16 = (rng.standard_normal((N, K), dtype=np.float32) * 0.03).astype(np.float16)
    b = rng.standard_normal(N, dtype=np.float32)
    X = torch.from_numpy(x).cuda()
    W = torch.from_numpy(w16.view(np.uint16).astype(np.int16)).cuda()
    B = torch.from_numpy(b).cuda()
    Y = torch.full((M * ldy + 8,), float("nan"), dtype=torch.float32, device="cuda")
    dev.gemm(True, W, X, Y, B if bias else None, M, N, K, ldx, K, ldy)
    dev.commit()
    y = Y.cpu().numpy()
    assert np.isnan(y[M * ldy:]).all(), "wrote past the output"
    y = y[:M * ldy].reshape(M, ldy)
    if ypad:
        assert np.isnan(y[:, N:]).all(), "clobbered the row padding"
    y = y[:, :N]
    wf = w16.astype(np.float64)
    ref = x[:, :K].astype(np.float64) @ wf.T + (b if bias else 0)
    assert not np.isnan(y).any(), "unwritten outputs"
    assert rel_l2(y, ref) < 5e-5, tag   # f32 tensor-core accumulation over K up to 7168


CONV_CASES = [  # (T, IC, OC, K, pad, bias, tag)  tools/conv_bench.cpp:14-26 (DiT rows)
    (172, 1024, 2816, 3, 1, False, "latent ffn w1 k3"),
    (172, 1024, 1024, 3, 1, True, "latent linear1 k3"),
    (172, 64, 1024, 3, 1, True, "audio_input_proj.0"),
    (172, 1024, 64, 7, 3, True, "final conv k7"),
    (64, 1024, 2816, 3, 1, False, "clip ffn w1"),
]


@pytest.mark.parametrize("T,IC,OC,K,pad,bias,tag", CONV_CASES)
def test_conv_runtime_face(dev, T, IC, OC, K, pad, bias, tag):
    rng = np.random.default_rng(11)
    x = rng.standard_normal((T, IC), dtype=np.float32)
    w16 = (rng.standard_normal((OC, IC, K), dtype=np.float32) * 0.03).astype(np.float16)
    b = rng.standard_normal(OC, dtype=np.float32)
    X = torch.from_numpy(x).cuda()
    W = torch.from_numpy(w16.view(np.uint16).astype(np.int16)).cuda()
    B = torch.from_numpy(b).cuda()
    Y = torch.full((T, OC), float("nan"), dtype=torch.float32, device="cuda")
    dev.conv(True, W, B if bias else None, X, Y, T, T, IC, OC, K, 1, pad, 1)
    dev.commit()
    y = Y.cpu().numpy()
    xp = np.zeros((T + 2 * pad, IC))
    xp[pad:pad + T] = x.astype(np.float64)
    ref = np.zeros((T, OC))
    wf = w16.astype(np.float64)
    for k in range(K):
        ref += xp[k:k + T] @ wf[:, :, k].T
    if bias:
        ref += b
    assert not np.isnan(y).any()
    assert rel_l2(y, ref) < 5e-5, tag   # f32 tensor-core accumulation over K up to 7168


GEMV_CASES = [  # (N, K, bias, wf16): Runtime::gemv (src/net.mm:51-56); f16 rows of <= 1024 stream
    (6144, 1024, True, True),        # one clip/text adaLN modulation
    (1023, 1024, True, True),        # odd N: the last 8-row stage is ragged
    (7, 200, False, True),           # a single partial stage, K not a multiple of 256
    (1, 64, True, True),
    (300, 2048, True, True),         # K above the streaming kernel's limit: the general kernel
    (500, 512, True, False),         # f32 weights: the general kernel
]


@pytest.mark.parametrize("N,K,bias,wf16", GEMV_CASES)
def test_gemv_runtime_face(dev, N, K, bias, wf16):
    rng = np.random.default_rng(13)
    x = rng.standard_normal(K, dtype=np.float32)
    w = rng.standard_normal((N, K), dtype=np.float32) * 0.03
    if wf16:
        w = w.astype(np.float16)
        W = torch.from_numpy(w.view(np.uint16).astype(np.int16)).cuda()
    else:
        W = torch.from_numpy(w).cuda()
    b = rng.standard_normal(N, dtype=np.float32)
    Y = torch.full((N + 8,), float("nan"), dtype=torch.float32, device="cuda")
    outs = []
    for _ in range(2):
        dev.gemv(W, torch.from_numpy(x).cuda(), Y, torch.from_numpy(b).cuda() if bias else None, N, K, 0, wf16)
        dev.commit()
        outs.append(Y.cpu().numpy())
    y = outs[0]
    assert np.isnan(y[N:]).all(), "wrote past the output"
    ref = w.astype(np.float64) @ x.astype(np.float64) + (b if bias else 0)
    assert rel_l2(y[:N], ref) < 1e-5     # f32 sums over K <= 2048
    assert np.array_equal(outs[0][:N], outs[1][:N])


GEMV_JOB_CASES = [  # (Ns, K, nb, nb_cap, act): the step's batched GEMV (t-embedding, clip/text modulations)
    ((6144, 1000, 7, 1), 1024, 2, 2, 0),       # ragged jobs below the largest N, odd N, one-row job
    ((333, 64, 1023), 64, 1, 1, 1),            # short rows, odd last slots, SiLU
    ((5, 6144, 17), 200, 3, 4, 0),             # three arms in the four-arm instance, K not a multiple of 128
    ((1024, 255, 999, 8), 1024, 8, 8, 0),      # eight arms (eight generations in one batch)
    ((7,), 8, 5, 8, 1),                        # the smallest K
    ((3,) * 20, 128, 2, 2, 0),                 # more jobs than one launch carries
]


GEMV_TC_CASES = [  # (Ns, K, nb): the tensor-core form the model runs its clip/text modulations on
    ((6144, 1000, 7, 1), 1024, 2),             # ragged jobs: partial 128-row tiles, one-row job
    ((333, 64, 1023), 64, 1),                  # the smallest K, one arm
    ((1024, 255, 999, 8), 1024, 8),            # eight arms: all 16 rows of the N tile
    ((6144,) * 12 + (2048,) * 2, 1024, 2),     # the step's 14 jobs at the 8 s geometry
    ((130, 129), 512, 3),
]


@pytest.mark.parametrize("Ns,K,nb", GEMV_TC_CASES)
def test_gemv_tc_jobs_vs_f64(dev, Ns, K, nb):
    """gemv_tc_kernel: weights as the tcgen05 M operand, the arms' split x as a 16-row N operand; every
    row within f32 accumulation error of float64 and bit-identical for grids of 148, 37 and 1 CTAs (a
    row's products run in one fixed order whichever CTA takes its tile)."""
    rng = np.random.default_rng(31)
    total = int(sum(Ns))
    w = (rng.standard_normal((total, K), dtype=np.float32) * 0.03).astype(np.float16)
    b = rng.standard_normal(total, dtype=np.float32)
    x = rng.standard_normal((nb, K), dtype=np.float32)
    W = torch.from_numpy(w.view(np.uint16).astype(np.int16)).cuda()
    bd, xd = torch.from_numpy(b).cuda(), torch.from_numpy(x).cuda()
    Y = torch.empty(nb * total + 8, dtype=torch.float32, device="cuda")
    outs = []
    for blocks in (148, 37, 1):
        Y.fill_(float("nan"))
        dev.selftest_gemv_jobs(W, bd, xd, Y, list(Ns), K, nb, nb, 0, blocks, tc=True)
        outs.append(Y.cpu().numpy())
    y = outs[0]
    assert np.isnan(y[nb * total:]).all(), "wrote past the output"
    ref = x.astype(np.float64) @ w.astype(np.float64).T + b
    assert rel_l2(y[:nb * total].reshape(nb, total), ref) < 1e-5
    for o in outs[1:]:
        assert np.array_equal(o[:nb * total], y[:nb * total]), "result depends on the grid"


@pytest.mark.parametrize("Ns,K,nb,nb_cap,act", GEMV_JOB_CASES)
def test_gemv_jobs_ragged_vs_f64(dev, Ns, K, nb, nb_cap, act):
    """gemv_kernel over several jobs of different row counts (src/net.mm:51-56 per job): every row
    within f32 summation error of float64 and, since a row's lane sums and butterfly do not depend on
    which warp or block takes its slot, bit-identical for grids of 148, 37 and 1 blocks."""
    rng = np.random.default_rng(29)
    total = int(sum(Ns))
    w = (rng.standard_normal((total, K), dtype=np.float32) * 0.03).astype(np.float16)
    b = rng.standard_normal(total, dtype=np.float32)
    x = rng.standard_normal((nb, K), dtype=np.float32)
    W = torch.from_numpy(w.view(np.uint16).astype(np.int16)).cuda()
    bd, xd = torch.from_numpy(b).cuda(), torch.from_numpy(x).cuda()
    Y = torch.empty(nb * total + 8, dtype=torch.float32, device="cuda")
    outs = []
    for blocks in (148, 37, 1):
        Y.fill_(float("nan"))
        dev.selftest_gemv_jobs(W, bd, xd, Y, list(Ns), K, nb, nb_cap, act, blocks)
        outs.append(Y.cpu().numpy())
    y = outs[0]
    assert np.isnan(y[nb * total:]).all(), "wrote past the output"
    ref = x.astype(np.float64) @ w.astype(np.float64).T + b
    if act:
        ref = ref / (1.0 + np.exp(-ref))
    assert rel_l2(y[:nb * total].reshape(nb, total), ref) < 1e-5
    for o in outs[1:]:
        assert np.array_equal(o[:nb * total], y[:nb * total]), "result depends on the grid"
