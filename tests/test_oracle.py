"""The CPU oracle against the reference's own host code and the committed golden vectors.

* port vs reference build: oracle/port.cpp restates src/dit_fwd.cpp; oracle/_ref/ts_ref_dit runs
  the reference's src/dit_fwd.cpp, src/dit.cpp, src/net.mm and src/gguf.cpp unmodified over the
  same scalar kernels. They must agree bit for bit on every tap the reference dumps
  (src/dit_fwd.cpp:151-301) and on a full CFG step (src/pipeline.cpp:146-148).
* golden: tests/golden/*.npz were produced by the reference build (make_golden.py); the port
  must reproduce them wherever the reference tree is absent (the GPU hosts).
"""
import hashlib
import os

import numpy as np
import pytest

import gguf_read
import oracle as O
from conftest import CLIP_SMALL, SEED, T5_SMALL, TINY, TINY_SEQ, clip_ids, make_geom, make_inputs, rel_l2, t5_ids

import tsn

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")

needs_ref = pytest.mark.skipif(not O.have_ref(), reason="oracle/_ref not built (reference tree absent)")


def _inputs():
    return make_inputs(TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"], TINY["H"])


@needs_ref
def test_port_matches_reference_build_forward(tiny_gguf, tmp_path):
    T, C, TS = TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"]
    inp = _inputs()
    O.write_inputs(str(tmp_path / "in"), inp)
    O.run_ref("forward", tiny_gguf, T, C, TS, str(tmp_path / "in"), str(tmp_path / "out"), 0.5, "cond")
    ref = O.read_ref_taps(str(tmp_path / "out"))
    orc = O.Oracle(tiny_gguf)
    flow = orc.forward(T, C, TS, inp["x"], 0.5, inp["clip_pp"], inp["sync_gather"], inp["text_pp_cond"],
                       inp["gcmlp_cond"], taps=True)
    assert set(ref) == set(O.TAPS)
    for name in O.TAPS:
        mine = flow.ravel() if name == "flow" else orc.tap(name)
        assert mine.shape == ref[name].shape, name
        assert np.array_equal(mine, ref[name]), f"tap {name} differs: rel-L2 {rel_l2(mine, ref[name])}"


@needs_ref
def test_port_matches_reference_build_step(tiny_gguf, tmp_path):
    T, C, TS = TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"]
    inp = _inputs()
    O.write_inputs(str(tmp_path / "in"), inp)
    dt = (1.0 - 1.0 / 24) - 1.0
    O.run_ref("step", tiny_gguf, T, C, TS, str(tmp_path / "in"), str(tmp_path / "out"), 1.0, 5.0, dt)
    x_ref = np.fromfile(str(tmp_path / "out" / "x_out.bin"), np.float32).reshape(T, 64)
    orc = O.Oracle(tiny_gguf)
    x, fc, fu = orc.step(T, C, TS, inp["x"], 1.0, 5.0, np.float32(dt), inp["clip_pp"], inp["sync_gather"],
                         inp["text_pp_cond"], inp["gcmlp_cond"], inp["text_pp_unc"], inp["gcmlp_unc"])
    assert np.array_equal(x, x_ref)
    assert not np.array_equal(fc, fu)   # the arms see different conditioning


def _golden(name):
    p = os.path.join(GOLDEN, name)
    if not os.path.exists(p):
        pytest.skip(f"{name} not generated")
    return dict(np.load(p))


def test_synthetic_gguf_bytes_pinned(tiny_gguf):
    g = _golden("tiny_forward.npz")
    h = hashlib.sha256(open(tiny_gguf, "rb").read()).hexdigest()
    assert h == str(g["gguf_sha256"]), "synthetic weight generator drifted from the golden fixture"


def test_port_reproduces_golden_forward(tiny_gguf):
    g = _golden("tiny_forward.npz")
    T, C, TS = int(g["T"]), int(g["C"]), int(g["TS"])
    orc = O.Oracle(tiny_gguf)
    flow = orc.forward(T, C, TS, g["in_x"], float(g["t"]), g["in_clip_pp"], g["in_sync_gather"],
                       g["in_text_pp_cond"], g["in_gcmlp_cond"], taps=True)
    assert np.array_equal(flow.ravel(), g["tap_flow"])
    for name in O.TAPS:
        if name != "flow":
            assert np.array_equal(orc.tap(name), g[f"tap_{name}"]), name


def test_port_reproduces_golden_sample(tiny_gguf):
    g = _golden("tiny_sample.npz")
    T, C, TS = int(g["T"]), int(g["C"]), int(g["TS"])
    orc = O.Oracle(tiny_gguf)
    x = g["in_x"].copy()
    steps, cfg = int(g["steps"]), float(g["cfg"])
    for s in range(steps):   # src/pipeline.cpp:142-148
        t_curr = np.float32(1.0) - np.float32(s) / np.float32(steps)
        t_prev = np.float32(1.0) - np.float32(s + 1) / np.float32(steps)
        x, _, _ = orc.step(T, C, TS, x, float(t_curr), cfg, float(np.float32(t_prev - t_curr)), g["in_clip_pp"],
                           g["in_sync_gather"], g["in_text_pp_cond"], g["in_gcmlp_cond"], g["in_text_pp_unc"],
                           g["in_gcmlp_unc"])
    assert np.array_equal(x, g["x_final"])


def _splitmix64(x):
    M = (1 << 64) - 1
    x = (x + 0x9E3779B97F4A7C15) & M
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & M
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & M
    return x ^ (x >> 31)


def _normal(key, idx):
    s = 0
    for j in range(3):
        r = _splitmix64((key + 3 * idx + j) & ((1 << 64) - 1))
        s += (r & 0xFFFF) + ((r >> 16) & 0xFFFF) + ((r >> 32) & 0xFFFF) + (r >> 48)
    return np.float32(s - 393210) * np.float32(1.0 / 65536.0)


def _key(name, seed):
    h = 1469598103934665603
    for ch in name.encode():
        h = ((h ^ ch) * 1099511628211) & ((1 << 64) - 1)
    return _splitmix64(h ^ _splitmix64(seed))


def _bf16(f):
    u = int(np.float32(f).view(np.uint32))
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFFFFFF
    return u >> 16


def test_synthetic_values_match_independent_restatement(tiny_gguf):
    """The C generator (include/tsn_synth.h) against a pure-Python restatement, read back from the file."""
    from gguf_read import read_tensor
    key = _key("t_embed.mlp.0.weight", SEED)
    got = read_tensor(tiny_gguf, "t_embed.mlp.0.weight", 16)
    want = np.array([_bf16(_normal(key, i) * np.float32(0.02)) for i in range(16)], np.uint16)
    assert np.array_equal(got, want)
    key = _key("joint_blocks.0.latent_block.attn.q_norm.weight", SEED)
    got = read_tensor(tiny_gguf, "joint_blocks.0.latent_block.attn.q_norm.weight", 16)
    want = np.array([np.float32(1.0) + _normal(key, i) * np.float32(0.02) for i in range(16)], np.float32)
    assert np.array_equal(got, want)


# prep_conditioning / prep_text_arm need the real hidden size (their cond projections read 1024
# inputs); a 2-block model with real widths keeps the reference run short.
PREP_GEOM = dict(H=1024, NH=16, F=4096, depth=2, fused_depth=1)
PREP_SEQ = dict(T=24, C=8, TS=16, sync_S=32)


def prep_inputs(seed=SEED + 11):
    s = PREP_SEQ
    rng = np.random.default_rng(seed)
    f = lambda *d: rng.standard_normal(d, dtype=np.float32)  # noqa: E731
    return {"clip_f": f(s["C"], 1024), "sync_f": f(s["sync_S"], 768), "text_cat_cond": f(s["TS"], 2048),
            "gtext_cond": f(1024), "text_cat_unc": f(s["TS"], 2048), "gtext_unc": f(1024)}


@pytest.fixture(scope="module")
def prep_gguf(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("gguf_prep") / "prep.gguf")
    tsn.write_synthetic_gguf(p, make_geom(**PREP_GEOM), SEED, with_prep=True)
    return p


@pytest.mark.skipif(not O.have_ref(), reason="reference build (oracle/_ref) absent")
def test_port_matches_reference_build_prep(prep_gguf, tmp_path):
    """The port's prep_conditioning + prep_text_arm equal the reference's own host code bit for bit."""
    s = PREP_SEQ
    inp = prep_inputs()
    O.write_inputs(str(tmp_path / "in"), inp)
    O.run_ref("prep", prep_gguf, s["T"], s["C"], s["TS"], str(tmp_path / "in"), str(tmp_path / "out"), s["sync_S"])
    got = O.Oracle(prep_gguf).prep(s["T"], s["C"], s["TS"], s["sync_S"], inp["clip_f"], inp["sync_f"],
                                   inp["text_cat_cond"], inp["gtext_cond"], inp["text_cat_unc"], inp["gtext_unc"])
    for k in O.PREP_OUT:
        ref = np.fromfile(str(tmp_path / "out" / f"{k}.bin"), np.float32)
        assert np.array_equal(got[k].ravel(), ref), k


# ---------------------------------------------------------------- VAE decoder
def _vae_weights(path):
    import gguf_read
    b, kv, tensors, data = gguf_read.read_header(path)

    def W(name):
        ne, ty, off = tensors[name]
        a = np.frombuffer(b, np.float32, int(np.prod(ne)), data + off).astype(np.float64)
        return a.reshape(ne[::-1]) if len(ne) > 1 else a
    return W


@pytest.fixture(scope="module")
def vae_gguf(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("vae") / "vae.gguf")
    tsn.write_synthetic_vae_gguf(p, channels=64, seed=SEED)
    yield p
    os.unlink(p)


def test_vae_synthetic_gguf_bytes_pinned(vae_gguf):
    g = np.load(os.path.join(GOLDEN, "small_vae.npz"))
    assert hashlib.sha256(open(vae_gguf, "rb").read()).hexdigest() == str(g["gguf_sha256"])


def test_vae_restatement_reproduces_golden(vae_gguf):
    """The float64 restatement of VaeModel::decode matches the reference's own decode (golden)."""
    g = np.load(os.path.join(GOLDEN, "small_vae.npz"))
    audio = O.vae_decode_np(_vae_weights(vae_gguf), g["latent"])
    assert audio.shape == g["audio"].shape
    assert rel_l2(audio, g["audio"]) < 1e-5


@needs_ref
def test_vae_reference_build_matches_restatement(vae_gguf, tmp_path):
    lat = np.random.default_rng(7).standard_normal((2, 64)).astype(np.float32)
    audio, js = O.ref_vae(vae_gguf, lat, workdir=str(tmp_path))
    assert js["T_audio"] == 2 * 2048
    assert rel_l2(O.vae_decode_np(_vae_weights(vae_gguf), lat), audio) < 1e-5


# ---------------------------------------------------------------- text encoders


@pytest.fixture(scope="module")
def t5_gguf(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("t5") / "t5.gguf")
    tsn.write_synthetic_t5_gguf(p, seed=SEED, **T5_SMALL)
    yield p
    os.unlink(p)


@pytest.fixture(scope="module")
def clip_gguf(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("clip") / "clip.gguf")
    tsn.write_synthetic_clip_gguf(p, seed=SEED, **CLIP_SMALL)
    yield p
    os.unlink(p)


def test_t5_bucket_known_values():
    """src/t5.cpp:7-20 at 32 buckets, max distance 128: exact below 8, logarithmic to 127, clamped."""
    b = lambda r: O.t5_bucket(r, 32, 128)  # noqa: E731
    assert [b(0), b(1), b(-1), b(7), b(-7)] == [0, 17, 1, 23, 7]
    assert b(8) == 24 and b(-8) == 8
    assert b(200) == 31 and b(-200) == 15 and b(127) == 31


def test_encoder_synthetic_gguf_bytes_pinned(t5_gguf, clip_gguf):
    for path, name in ((t5_gguf, "small_t5.npz"), (clip_gguf, "small_clip.npz")):
        g = np.load(os.path.join(GOLDEN, name))
        assert hashlib.sha256(open(path, "rb").read()).hexdigest() == str(g["gguf_sha256"])


def test_q8_0_blocks_follow_the_synthetic_values(t5_gguf):
    """The writer's Q8_0 blocks decode (to_f32, src/gguf.cpp:216-228) to the seeded normal values
    within half a quantisation step, and every block's largest value maps to +-127."""
    b, kv, tensors, data = gguf_read.read_header(t5_gguf)
    v, ty = gguf_read.tensor_f32(b, tensors, data, "blk.0.q")
    assert ty == 8
    blk = np.frombuffer(b, np.uint8, v.size // 32 * 34, data + tensors["blk.0.q"][2]).reshape(-1, 34)
    q = blk[:, 2:].view(np.int8)
    assert np.all(np.abs(q).max(axis=1) == 127)
    assert np.all(np.abs(v) <= 127 * gguf_read._f16_flush(blk[:, :2].copy().view(np.uint16)[:, 0]).max() * 1.001)


def test_t5_restatement_reproduces_golden(t5_gguf):
    g = np.load(os.path.join(GOLDEN, "small_t5.npz"))
    W, kv = gguf_read.device_weights(t5_gguf)
    assert rel_l2(O.t5_encode_np(W, kv, g["ids"]), g["out"]) < 1e-5


def test_clip_restatement_reproduces_golden(clip_gguf):
    g = np.load(os.path.join(GOLDEN, "small_clip.npz"))
    W, kv = gguf_read.device_weights(clip_gguf)
    pt, pooled = O.clip_encode_np(W, kv, g["ids"])
    assert rel_l2(pt, g["per_token"]) < 1e-5
    assert rel_l2(pooled, g["pooled"]) < 1e-5


@needs_ref
@pytest.mark.parametrize("n_tok", [1, 76])
def test_t5_reference_build_matches_restatement(t5_gguf, tmp_path, n_tok):
    """Edge cases of the pad mask: a single token + EOS (75 pad keys), and no padding at all."""
    ids = t5_ids(SEED + n_tok, n_tok)
    out, _, _ = O.ref_encoder("t5", t5_gguf, ids, workdir=str(tmp_path))
    W, kv = gguf_read.device_weights(t5_gguf)
    assert rel_l2(O.t5_encode_np(W, kv, ids), out) < 1e-5


@needs_ref
@pytest.mark.parametrize("n_tok", [0, 75])
def test_clip_reference_build_matches_restatement(clip_gguf, tmp_path, n_tok):
    """EOT at position 1 (empty caption) and at the last position (a full context)."""
    ids = clip_ids(SEED + n_tok, n_tok)
    pt, pooled, _ = O.ref_encoder("clip", clip_gguf, ids, workdir=str(tmp_path))
    W, kv = gguf_read.device_weights(clip_gguf)
    p2, g2 = O.clip_encode_np(W, kv, ids)
    assert rel_l2(p2, pt) < 1e-5 and rel_l2(g2, pooled) < 1e-5


def test_joint_block_entry_matches_forward_taps(tiny_gguf):
    """oracle_joint_block (the CPU baseline of BASELINE config 1) is joint block 0 of the forward:
    fed the forward's own x_in, conditioning and streams, it reproduces the jb0_* taps."""
    T, C, TS = TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"]
    inp = make_inputs(T, C, TS, TINY["H"])
    orc = O.Oracle(tiny_gguf)
    orc.forward(T, C, TS, inp["x"], 0.5, inp["clip_pp"], inp["sync_gather"], inp["text_pp_cond"], inp["gcmlp_cond"],
                taps=True)
    silu = lambda v: (v / (1.0 + np.exp(-v.astype(np.float64)))).astype(np.float32)  # noqa: E731
    lat, clip, text = orc.joint_block(orc.tap("x_in").reshape(T, -1), inp["clip_pp"], inp["text_pp_cond"],
                                      silu(orc.tap("extended_c")).reshape(T, -1), silu(orc.tap("global_c")))
    for got, name in ((lat, "jb0_lat"), (clip, "jb0_clip"), (text, "jb0_text")):
        assert rel_l2(got, orc.tap(name)) < 1e-5, name
