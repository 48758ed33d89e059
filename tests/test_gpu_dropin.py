"""The drop-in boundary end to end: the reference's own, unmodified host code (src/dit.cpp,
src/dit_fwd.cpp, src/net.mm, src/vae.cpp, src/t5.cpp, src/clip.cpp, src/gguf.cpp) and the oracle's
driver, built with src/gpu.mm replaced by the library's tn::gpu::Device
(thinksound-native_b200/integration/gpu_tsn.cpp, oracle/_ref/ts_ref_dit_tsn), run on the GPU.
Every named dispatch of that code then runs on the runtime face (tsn_dispatch and the compat
kernels), and its results must match the same host code on the CPU device (the golden fixtures):
flow rel-L2 <= 1e-3 and every parity tap <= 2e-3 (the path's parity gates), the 4-step sample, the VAE
decode and both text encoders <= 1e-3.
"""
import os

import numpy as np
import pytest

import oracle as O
from conftest import CLIP_SMALL, SEED, T5_SMALL, TINY, make_geom, rel_l2

import tsn

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.access(O.REF_TSN_BIN, os.X_OK),
                                 reason="oracle/_ref/ts_ref_dit_tsn not built (needs the reference tree)")]

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
FLOW_TOL, TAP_TOL = 1e-3, 2e-3


@pytest.fixture(scope="module")
def tiny_gguf(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("dropin") / "tiny.gguf")
    tsn.write_synthetic_gguf(p, make_geom(**TINY), SEED)
    yield p
    os.unlink(p)


def _inputs(g, d):
    O.write_inputs(d, {k[3:]: g[k] for k in g.files if k.startswith("in_")})


def test_reference_forward_on_gpu_device(tiny_gguf, tmp_path):
    g = np.load(os.path.join(GOLDEN, "tiny_forward.npz"))
    T, C, TS = int(g["T"]), int(g["C"]), int(g["TS"])
    _inputs(g, str(tmp_path / "in"))
    O.run_ref("forward", tiny_gguf, T, C, TS, str(tmp_path / "in"), str(tmp_path / "out"), float(g["t"]), "cond",
              binary=O.REF_TSN_BIN)
    taps = O.read_ref_taps(str(tmp_path / "out"))
    assert set(taps) == {k[4:] for k in g.files if k.startswith("tap_")}
    worst = {}
    for name, v in taps.items():
        worst[name] = rel_l2(v, g["tap_" + name])
    print("drop-in forward, rel-L2 per tap:", {k: f"{v:.2e}" for k, v in worst.items()})
    assert worst["flow"] < FLOW_TOL
    assert max(worst.values()) < TAP_TOL


def test_reference_sampler_on_gpu_device(tiny_gguf, tmp_path):
    g = np.load(os.path.join(GOLDEN, "tiny_sample.npz"))
    T, C, TS = int(g["T"]), int(g["C"]), int(g["TS"])
    _inputs(g, str(tmp_path / "in"))
    O.run_ref("sample", tiny_gguf, T, C, TS, str(tmp_path / "in"), str(tmp_path / "out"), int(g["steps"]),
              float(g["cfg"]), binary=O.REF_TSN_BIN)
    x = np.fromfile(str(tmp_path / "out" / "x_final.bin"), np.float32).reshape(T, 64)
    err = rel_l2(x, g["x_final"])
    print("drop-in 4-step sample rel-L2:", err)
    assert err < FLOW_TOL


def test_reference_vae_on_gpu_device(tmp_path):
    g = np.load(os.path.join(GOLDEN, "small_vae.npz"))
    p = str(tmp_path / "vae.gguf")
    tsn.write_synthetic_vae_gguf(p, channels=int(g["channels"]), seed=SEED)
    audio, _ = O.ref_vae(p, g["latent"], workdir=str(tmp_path / "w"), binary=O.REF_TSN_BIN)
    err = rel_l2(audio, g["audio"])
    print("drop-in VAE rel-L2:", err)
    assert err < 1e-3


def test_reference_text_encoders_on_gpu_device(tmp_path):
    gt = np.load(os.path.join(GOLDEN, "small_t5.npz"))
    p = str(tmp_path / "t5.gguf")
    tsn.write_synthetic_t5_gguf(p, seed=SEED, **T5_SMALL)
    out, _, _ = O.ref_encoder("t5", p, gt["ids"], workdir=str(tmp_path / "t5"), binary=O.REF_TSN_BIN)
    e1 = rel_l2(out, gt["out"])
    gc = np.load(os.path.join(GOLDEN, "small_clip.npz"))
    p = str(tmp_path / "clip.gguf")
    tsn.write_synthetic_clip_gguf(p, seed=SEED, **CLIP_SMALL)
    pt, pooled, _ = O.ref_encoder("clip", p, gc["ids"], workdir=str(tmp_path / "clip"), binary=O.REF_TSN_BIN)
    e2, e3 = rel_l2(pt, gc["per_token"]), rel_l2(pooled, gc["pooled"])
    print("drop-in T5 / CLIP per-token / CLIP pooled rel-L2:", e1, e2, e3)
    assert e1 < 1e-3 and e2 < 1e-3 and e3 < 1e-3
