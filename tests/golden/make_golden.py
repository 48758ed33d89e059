"""Generate the golden fixtures from the reference's own host code (run in the container that holds
the reference tree; the GPU hosts only read the committed .npz files).

    python tests/golden/make_golden.py

tiny_forward.npz  one DitModel::forward (src/dit_fwd.cpp:104-304) of the cond arm on the tiny
                  synthetic DiT (H=256, 4 heads, F=512, 2 joint + 1 fused block; T=24, C=8, TS=16,
                  t=0.5) with every tap the reference dumps, plus the SHA-256 of the weight file.
tiny_sample.npz   4 Euler steps of the sampler loop (src/pipeline.cpp:142-155), CFG 5.0.
The weights are regenerated bit-exactly by tsn.write_synthetic_gguf (seed 4242).
"""
import hashlib
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from conftest import SEED, TINY, TINY_SEQ, make_geom, make_inputs  # noqa: E402

import oracle as O  # noqa: E402
import tsn  # noqa: E402


def main():
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
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
