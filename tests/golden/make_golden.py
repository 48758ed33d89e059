"""Generate the golden fixtures from the reference's own host code (run in the container that holds
the reference tree; the GPU hosts only read the committed .npz files).

    python tests/golden/make_golden.py

tiny_forward.npz  one DitModel::forward (src/dit_fwd.cpp:104-304) of the cond arm on the tiny
                  synthetic DiT (H=256, 4 heads, F=512, 2 joint + 1 fused block; T=24, C=8, TS=16,
                  t=0.5) with every tap the reference dumps, plus the SHA-256 of the weight file.
tiny_sample.npz   4 Euler steps of the sampler loop (src/pipeline.cpp:142-155), CFG 5.0.
small_vae.npz     VaeModel::decode (src/vae.cpp:17-86) of a seeded latent [3, 64] on the synthetic
                  VAE with 64 base channels (widths 1024 ... 64), audio [6144, 2].
small_t5.npz      T5Model::encode (src/t5.cpp:84-131) of seeded ids (31 tokens + EOS, then pad) on
                  the synthetic Q8_0 T5 (d_model 256, d_ff 512, 2 layers, 4 heads): out [77, 256].
small_clip.npz    ClipModel::encode (src/clip.cpp:30-101) of seeded ids (BOS, 20 tokens, EOS padded)
                  on the synthetic f32 MetaCLIP text model (hidden 256, 2 layers, 4 heads):
                  per_token [77, 256], pooled [256].
The weights are regenerated bit-exactly by tsn.write_synthetic_gguf / write_synthetic_vae_gguf /
write_synthetic_t5_gguf / write_synthetic_clip_gguf (seed 4242). `python tests/golden/make_golden.py
vae` (or `encoders`) writes only those fixtures.
"""
import hashlib
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from conftest import CLIP_SMALL, SEED, T5_SMALL, TINY, TINY_SEQ, clip_ids, make_geom, make_inputs, t5_ids  # noqa: E402

import oracle as O  # noqa: E402
import tsn  # noqa: E402


VAE_CH, VAE_T = 64, 3


def vae_latent():
    return np.random.default_rng(SEED).standard_normal((VAE_T, 64)).astype(np.float32)


def make_vae(d):
    gguf = os.path.join(d, "vae.gguf")
    tsn.write_synthetic_vae_gguf(gguf, channels=VAE_CH, seed=SEED)
    sha = hashlib.sha256(open(gguf, "rb").read()).hexdigest()
    lat = vae_latent()
    audio, _ = O.ref_vae(gguf, lat, workdir=os.path.join(d, "vae"))
    np.savez_compressed(os.path.join(HERE, "small_vae.npz"), latent=lat, audio=audio, channels=VAE_CH,
                        gguf_sha256=sha)


def make_encoders(d):
    g = os.path.join(d, "t5.gguf")
    tsn.write_synthetic_t5_gguf(g, seed=SEED, **T5_SMALL)
    sha = hashlib.sha256(open(g, "rb").read()).hexdigest()
    ids = t5_ids(SEED)
    out, _, _ = O.ref_encoder("t5", g, ids, workdir=os.path.join(d, "t5"))
    np.savez_compressed(os.path.join(HERE, "small_t5.npz"), ids=ids, out=out, gguf_sha256=sha, **T5_SMALL)
    g = os.path.join(d, "clip.gguf")
    tsn.write_synthetic_clip_gguf(g, seed=SEED, **CLIP_SMALL)
    sha = hashlib.sha256(open(g, "rb").read()).hexdigest()
    ids = clip_ids(SEED)
    pt, pooled, _ = O.ref_encoder("clip", g, ids, workdir=os.path.join(d, "clip"))
    np.savez_compressed(os.path.join(HERE, "small_clip.npz"), ids=ids, per_token=pt, pooled=pooled, gguf_sha256=sha,
                        **CLIP_SMALL)


def main():
    if not O.have_ref():
        raise SystemExit("oracle/_ref/ts_ref_dit not built (needs the reference tree)")
    if sys.argv[1:] == ["encoders"]:
        with tempfile.TemporaryDirectory() as d:
            make_encoders(d)
        print("wrote small_t5.npz, small_clip.npz")
        return
    if sys.argv[1:] == ["vae"]:
        with tempfile.TemporaryDirectory() as d:
            make_vae(d)
        print("wrote small_vae.npz")
        return
    if not O.have_ref():
        raise SystemExit("oracle/_ref/ts_ref_dit not built (needs the reference tree)")
    T, C, TS = TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"]
    with tempfile.TemporaryDirectory() as d:
        gguf = os.path.join(d, "tiny.gguf")
        tsn.write_synthetic_gguf(gguf, make_geom(**TINY), SEED)
        sha = hashlib.sha256(open(gguf, "rb").read()).hexdigest()
        inp = make_inputs(T, C, TS, TINY["H"])
        O.write_inputs(os.path.join(d, "in"), inp)
        O.run_ref("forward", gguf, T, C, TS, os.path.join(d, "in"), os.path.join(d, "fw"), 0.5, "cond")
        taps = O.read_ref_taps(os.path.join(d, "fw"))
        out = {f"in_{k}": v for k, v in inp.items()}
        out.update({f"tap_{k}": v for k, v in taps.items()})
        out.update(T=T, C=C, TS=TS, t=np.float32(0.5), gguf_sha256=sha, **{k: v for k, v in TINY.items()})
        np.savez_compressed(os.path.join(HERE, "tiny_forward.npz"), **out)

        steps, cfg = 4, 5.0
        O.run_ref("sample", gguf, T, C, TS, os.path.join(d, "in"), os.path.join(d, "sm"), steps, cfg)
        xf = np.fromfile(os.path.join(d, "sm", "x_final.bin"), np.float32).reshape(T, 64)
        out = {f"in_{k}": v for k, v in inp.items()}
        out.update(T=T, C=C, TS=TS, steps=steps, cfg=np.float32(cfg), x_final=xf, gguf_sha256=sha)
        np.savez_compressed(os.path.join(HERE, "tiny_sample.npz"), **out)
        make_vae(d)
        make_encoders(d)
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
