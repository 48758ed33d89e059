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
full_sample.npz   BASELINE config 3 at full size: the 24-step CFG-5 sampler (src/pipeline.cpp:126-155) of
                  the 21-block model (H 1024, 16 heads, F 4096; T 188, clip 64, text 77), initial
                  latent drawn as generate_wav draws it from mt19937(4242); the conditioning inputs
                  are make_inputs(188, 64, 77, 1024) (seed 4242, stored as a SHA-256 only: the tests
                  regenerate them). Holds x0, x_final and, for steps 0, 1, 11, 12 and 23, the step's
                  input x and both arms' flows; and the trajectory's sensitivity: x_final of the
                  reference's own run from x0 perturbed by relative SENS_EPS (the size of the per-step
                  flow gate) Gaussian noise, as its rel-L2 distance from x_final.
                  `python tests/golden/make_golden.py full` writes only this.
long_forward.npz  BASELINE config 4 at full depth: one DitModel::forward per CFG arm of the 21-block model
                  at the 30 s geometry (T 704, clip 240, text 77; S = 1021), t = 0.5, inputs
                  make_inputs(704, 240, 77, 1024) (stored as a SHA-256), flows of both arms.
                  `python tests/golden/make_golden.py long` writes only this.
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


FULL = dict(H=1024, NH=16, F=4096, depth=21, fused_depth=14)
FULL_SEQ = dict(T=188, C=64, TS=77)
FULL_STEPS, FULL_CFG, FULL_DUMP = 24, 5.0, (0, 1, 11, 12, 23)
SENS_EPS = 1e-3


def inputs_sha(inp):
    h = hashlib.sha256()
    for k in sorted(inp):
        h.update(k.encode())
        h.update(np.ascontiguousarray(inp[k], np.float32).tobytes())
    return h.hexdigest()


def make_full(d):
    T, C, TS = FULL_SEQ["T"], FULL_SEQ["C"], FULL_SEQ["TS"]
    gguf = os.path.join(d, "full.gguf")
    tsn.write_synthetic_gguf(gguf, make_geom(**FULL), SEED)
    inp = make_inputs(T, C, TS, FULL["H"])
    O.write_inputs(os.path.join(d, "in"), inp)
    od = os.path.join(d, "full")
    out = O.run_ref("sample", gguf, T, C, TS, os.path.join(d, "in"), od, FULL_STEPS, FULL_CFG, SEED,
                    ",".join(str(s) for s in FULL_DUMP), timeout=7200)
    rd = lambda n: np.fromfile(os.path.join(od, n), np.float32).reshape(T, 64)  # noqa: E731
    res = {"x0": rd("x0.bin"), "x_final": rd("x_final.bin")}
    for s in FULL_DUMP:
        res[f"x_s{s}"] = rd(f"x_s{s}.bin")
        res[f"fc_s{s}"] = rd(f"fc_s{s}.bin")
        res[f"fu_s{s}"] = rd(f"fu_s{s}.bin")
    # sensitivity: the same sampler from x0 + SENS_EPS * rms(x0) * N(0, 1)
    x0 = res["x0"]
    pin = dict(inp)
    noise = np.random.default_rng(1).standard_normal(x0.shape)
    pin["x"] = (x0 + SENS_EPS * np.sqrt(np.mean(x0.astype(np.float64) ** 2)) * noise).astype(np.float32)
    O.write_inputs(os.path.join(d, "pin"), pin)
    pd = os.path.join(d, "pert")
    O.run_ref("sample", gguf, T, C, TS, os.path.join(d, "pin"), pd, FULL_STEPS, FULL_CFG, -1, "", timeout=7200)
    xp = np.fromfile(os.path.join(pd, "x_final.bin"), np.float32).reshape(T, 64).astype(np.float64)
    xf = res["x_final"].astype(np.float64)
    sens = float(np.linalg.norm(xp - xf) / np.linalg.norm(xf))
    np.savez_compressed(os.path.join(HERE, "full_sample.npz"), **res, steps=FULL_STEPS, cfg=np.float32(FULL_CFG),
                        dump_steps=np.array(FULL_DUMP), inputs_sha256=inputs_sha(inp), seconds=O.parse_json_line(out)["seconds"],
                        sens_eps=SENS_EPS, sens_x_final_rel=sens, **{k: v for k, v in FULL.items()}, **FULL_SEQ)


LONG_SEQ = dict(T=704, C=240, TS=77)


def make_long(d):
    T, C, TS = LONG_SEQ["T"], LONG_SEQ["C"], LONG_SEQ["TS"]
    gguf = os.path.join(d, "full.gguf")
    if not os.path.exists(gguf):
        tsn.write_synthetic_gguf(gguf, make_geom(**FULL), SEED)
    inp = make_inputs(T, C, TS, FULL["H"])
    O.write_inputs(os.path.join(d, "lin"), inp)
    flows = {}
    for arm in ("cond", "unc"):
        od = os.path.join(d, "long_" + arm)
        O.run_ref("forward", gguf, T, C, TS, os.path.join(d, "lin"), od, 0.5, arm, timeout=7200)
        flows[f"flow_{arm}"] = np.fromfile(os.path.join(od, "flow.bin"), np.float32).reshape(T, 64)
    np.savez_compressed(os.path.join(HERE, "long_forward.npz"), **flows, t=np.float32(0.5), inputs_sha256=inputs_sha(inp),
                        **{k: v for k, v in FULL.items()}, **LONG_SEQ)


def main():
    if not O.have_ref():
        raise SystemExit("oracle/_ref/ts_ref_dit not built (needs the reference tree)")
    if sys.argv[1:] == ["long"]:
        with tempfile.TemporaryDirectory() as d:
            make_long(d)
        print("wrote long_forward.npz")
        return
    if sys.argv[1:] == ["full"]:
        with tempfile.TemporaryDirectory() as d:
            make_full(d)
        print("wrote full_sample.npz")
        return
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
