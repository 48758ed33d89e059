"""The GPU text encoders (tsn_t5_load / tsn_clip_load / tsn_encoder_encode) against the reference's
T5Model::encode (src/t5.cpp:84-131) and ClipModel::encode (src/clip.cpp:30-101).

Gate: per-token features, and CLIP's pooled projection, within rel-L2 1e-3 of the reference (split f16
activations, and split weights for CLIP's f32 tensors, carry the f32 GEMMs to ~2^-22; attention
keeps P in f16), and repeated encodes bit-identical.
"""
import os

import numpy as np
import pytest

import gguf_read
import oracle as O
from conftest import CLIP_SMALL, SEED, T5_SMALL, clip_ids, rel_l2, t5_ids

import tsn

pytestmark = pytest.mark.gpu

TOL = 1e-3
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def dev():
    d = tsn.Device(0)
    yield d
    d.close()


def _gguf(tmp_path_factory, kind, tag=None, **geom):
    p = str(tmp_path_factory.mktemp(tag or kind) / f"{kind}.gguf")
    (tsn.write_synthetic_t5_gguf if kind == "t5" else tsn.write_synthetic_clip_gguf)(p, seed=SEED, **geom)
    return p


@pytest.fixture(scope="module")
def t5_small(tmp_path_factory):
    p = _gguf(tmp_path_factory, "t5", **T5_SMALL)
    yield p
    os.unlink(p)


@pytest.fixture(scope="module")
def clip_small(tmp_path_factory):
    p = _gguf(tmp_path_factory, "clip", **CLIP_SMALL)
    yield p
    os.unlink(p)


def test_t5_vs_reference_golden(dev, t5_small):
    g = np.load(os.path.join(GOLDEN, "small_t5.npz"))
    e = tsn.TextEncoder(dev, "t5", t5_small)
    assert (e.width, e.ctx, e.layers) == (T5_SMALL["d_model"], 77, T5_SMALL["layers"])
    out = e.encode(g["ids"])
    err = rel_l2(out, g["out"])
    print("t5 rel-L2 vs reference:", err)
    assert err < TOL
    assert np.array_equal(out, e.encode(g["ids"])), "repeat encode not bit-identical"


def test_clip_vs_reference_golden(dev, clip_small):
    g = np.load(os.path.join(GOLDEN, "small_clip.npz"))
    e = tsn.TextEncoder(dev, "clip", clip_small)
    pt, pooled = e.encode(g["ids"])
    e1, e2 = rel_l2(pt, g["per_token"]), rel_l2(pooled, g["pooled"])
    print("clip rel-L2 vs reference: per_token", e1, "pooled", e2)
    assert e1 < TOL and e2 < TOL
    pt2, pooled2 = e.encode(g["ids"])
    assert np.array_equal(pt, pt2) and np.array_equal(pooled, pooled2)


@pytest.mark.parametrize("n_tok", [1, 76])
def test_t5_pad_mask_edges(dev, t5_small, n_tok):
    """One token + EOS (75 padded keys) and a context without padding, against the restatement."""
    ids = t5_ids(SEED + n_tok, n_tok)
    out = tsn.TextEncoder(dev, "t5", t5_small).encode(ids)
    W, kv = gguf_read.device_weights(t5_small)
    assert rel_l2(out, O.t5_encode_np(W, kv, ids)) < TOL


@pytest.mark.parametrize("n_tok", [0, 75])
def test_clip_eot_edges(dev, clip_small, n_tok):
    """EOT at position 1 (empty caption) and at position 76 (full context)."""
    ids = clip_ids(SEED + n_tok, n_tok)
    pt, pooled = tsn.TextEncoder(dev, "clip", clip_small).encode(ids)
    W, kv = gguf_read.device_weights(clip_small)
    rp, rg = O.clip_encode_np(W, kv, ids)
    assert rel_l2(pt, rp) < TOL and rel_l2(pooled, rg) < TOL


def test_wide_geometries(dev, tmp_path_factory):
    """Widths of the real models (T5 d_model 1024 with 16 heads, d_ff 2816; CLIP hidden 512) over
    two layers: many weight tiles per GEMM and K-sliced partial tiles."""
    p = _gguf(tmp_path_factory, "t5", "t5w", d_model=1024, d_ff=2816, layers=2, heads=16)
    ids = t5_ids(SEED + 5, 40)
    out = tsn.TextEncoder(dev, "t5", p).encode(ids)
    W, kv = gguf_read.device_weights(p)
    assert rel_l2(out, O.t5_encode_np(W, kv, ids)) < TOL
    os.unlink(p)
    p = _gguf(tmp_path_factory, "clip", "clipw", hidden=512, layers=2, heads=8)
    ids = clip_ids(SEED + 6, 30)
    pt, pooled = tsn.TextEncoder(dev, "clip", p).encode(ids)
    W, kv = gguf_read.device_weights(p)
    rp, rg = O.clip_encode_np(W, kv, ids)
    assert rel_l2(pt, rp) < TOL and rel_l2(pooled, rg) < TOL
    os.unlink(p)


def test_bad_ids_rejected(dev, t5_small):
    e = tsn.TextEncoder(dev, "t5", t5_small)
    ids = t5_ids(SEED)
    with pytest.raises(tsn.TsnError):
        e.encode(ids[:76])
    bad = ids.copy()
    bad[3] = 32128
    with pytest.raises(tsn.TsnError):
        e.encode(bad)
    bad[3] = -1
    with pytest.raises(tsn.TsnError):
        e.encode(bad)
    assert rel_l2(e.encode(ids), np.load(os.path.join(GOLDEN, "small_t5.npz"))["out"]) < TOL
