"""Shared fixtures. GPU tests carry @pytest.mark.gpu; everything else runs on the CPU."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "thinksound-native_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

import tsn  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")
    config.addinivalue_line("markers", "slow: long CPU oracle runs")


# Small DiT used by most parity tests: 2 joint blocks (the second pre_only) + 1 fused block.
TINY = dict(H=256, NH=4, F=512, depth=3, fused_depth=1)
TINY_SEQ = dict(T=24, C=8, TS=16)
# Real widths, fewer blocks.
WIDE = dict(H=1024, NH=16, F=4096, depth=3, fused_depth=1)
WIDE_SEQ = dict(T=188, C=64, TS=77)
SEED = 4242


# Text encoder fixtures (tests/golden/small_t5.npz, small_clip.npz).
T5_SMALL = dict(d_model=256, d_ff=512, layers=2, heads=4)
CLIP_SMALL = dict(hidden=256, layers=2, heads=4)


def t5_ids(seed, n_tok=31):
    """n_tok seeded token ids, EOS (1), pad (0) to 77: the T5 tokenizer's layout."""
    ids = np.zeros(77, np.int32)
    ids[:n_tok] = np.random.default_rng(seed).integers(2, 32000, n_tok)
    ids[n_tok] = 1
    return ids


def clip_ids(seed, n_tok=20):
    """BOS (49406), n_tok seeded ids, EOS (49407) padding to 77: the CLIP tokenizer's layout."""
    ids = np.full(77, 49407, np.int32)
    ids[0] = 49406
    ids[1:1 + n_tok] = np.random.default_rng(seed).integers(1, 49000, n_tok)
    return ids


def make_geom(H, NH, F, depth, fused_depth):
    return tsn.geom(H=H, NH=NH, F=F, depth=depth, fused_depth=fused_depth)


def make_inputs(T, C, TS, H, seed=SEED, L=64):
    """Per-generation conditioning and latent, all N(0,1) f32 (BASELINE config 1 inputs)."""
    rng = np.random.default_rng(seed)
    f = lambda *s: rng.standard_normal(s, dtype=np.float32)  # noqa: E731
    return {"x": f(T, L), "clip_pp": f(C, H), "sync_gather": f(T, H),
            "text_pp_cond": f(TS, H), "text_pp_unc": f(TS, H), "gcmlp_cond": f(H), "gcmlp_unc": f(H)}


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-30))


@pytest.fixture(scope="session")
def tiny_gguf(tmp_path_factory):
    d = tmp_path_factory.mktemp("gguf")
    p = str(d / "tiny.gguf")
    tsn.write_synthetic_gguf(p, make_geom(**TINY), SEED)
    return p


@pytest.fixture(scope="session")
def wide_gguf(tmp_path_factory):
    d = tmp_path_factory.mktemp("gguf_wide")
    p = str(d / "wide.gguf")
    tsn.write_synthetic_gguf(p, make_geom(**WIDE), SEED)
    return p
