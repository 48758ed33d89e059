"""The GPU VAE decoder (tsn_vae_*) against the reference's VaeModel::decode (src/vae.cpp:17-86).

Gate: decoded audio rel-L2 <= 1e-3 against the reference (the split-weight GEMMs carry the f32
weights to ~2^-22; f16 weights alone would give ~1.3e-3), and repeated decodes bit-identical.
"""
import os

import numpy as np
import pytest

import oracle as O
from conftest import SEED, rel_l2

import tsn

pytestmark = pytest.mark.gpu

AUDIO_TOL = 1e-3
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "small_vae.npz")


@pytest.fixture(scope="module")
def dev():
    d = tsn.Device(0)
    yield d
    d.close()


@pytest.fixture(scope="module")
def vae_gguf(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("vae") / "vae.gguf")
    tsn.write_synthetic_vae_gguf(p, channels=64, seed=SEED)
    yield p
    os.unlink(p)


def _weights(path):
    import gguf_read
    b, kv, tensors, data = gguf_read.read_header(path)

    def W(name):
        ne, ty, off = tensors[name]
        a = np.frombuffer(b, np.float32, int(np.prod(ne)), data + off).astype(np.float64)
        return a.reshape(ne[::-1]) if len(ne) > 1 else a
    return W


def test_vae_decode_vs_reference_golden(dev):
    g = np.load(GOLDEN)
    v = tsn.Vae(dev, channels=int(g["channels"]), seed=SEED)
    audio = v.decode(g["latent"])
    assert audio.shape == g["audio"].shape
    e = rel_l2(audio, g["audio"])
    print("vae audio rel-L2 vs reference:", e)
    assert e < AUDIO_TOL
    again = v.decode(g["latent"])
    assert np.array_equal(audio, again), "repeat decode not bit-identical"


def test_vae_file_equals_synthetic_and_other_lengths(dev, vae_gguf):
    """The GGUF path loads the same weights as the in-memory synthetic model; a second latent length
    (its own plan and graph) matches the float64 restatement of the reference's decode."""
    lat = np.random.default_rng(11).standard_normal((5, 64)).astype(np.float32)
    a = tsn.Vae(dev, gguf=vae_gguf).decode(lat)
    b = tsn.Vae(dev, channels=64, seed=SEED).decode(lat)
    assert np.array_equal(a, b)
    ref = O.vae_decode_np(_weights(vae_gguf), lat)
    assert rel_l2(a, ref) < AUDIO_TOL
    # back to the first length on the same model
    v = tsn.Vae(dev, channels=64, seed=SEED)
    v.decode(lat[:2])
    c = v.decode(lat)
    assert np.array_equal(c, b)
