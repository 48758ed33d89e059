"""The once-per-generation conditioning (DitModel::prep_conditioning / prep_text_arm,
src/dit.cpp:55-192) on the GPU against the oracle port, which the CPU suite pins bit-for-bit to
the reference's own host code (tests/test_oracle.py::test_port_matches_reference_build_prep)."""
import numpy as np
import pytest

import oracle as O
import tsn
from conftest import SEED, make_geom, make_inputs, rel_l2
from test_oracle import PREP_GEOM, PREP_SEQ, prep_inputs

PREP_TOL = 1e-4     # six chained GEMM/conv stages with split f16 activations (~2^-22 each) and f16 weights


@pytest.fixture(scope="module")
def dev():
    d = tsn.Device(0)
    yield d
    d.close()


@pytest.fixture(scope="module")
def prep_gguf(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("gguf_prep_gpu") / "prep.gguf")
    tsn.write_synthetic_gguf(p, make_geom(**PREP_GEOM), SEED, with_prep=True)
    return p


def gpu_prep(dev, gguf, inp):
    s = PREP_SEQ
    m = tsn.Dit(dev, gguf=gguf)
    m.prepare(s["T"], s["C"], s["TS"], 2)
    m.prep_conditioning(inp["clip_f"], inp["sync_f"], s["sync_S"])
    m.prep_text_arm(0, inp["text_cat_cond"], inp["gtext_cond"])
    m.prep_text_arm(1, inp["text_cat_unc"], inp["gtext_unc"])
    return m


@pytest.mark.gpu
def test_prep_vs_oracle(dev, prep_gguf):
    s, H = PREP_SEQ, PREP_GEOM["H"]
    inp = prep_inputs()
    m = gpu_prep(dev, prep_gguf, inp)
    clip_pp = np.zeros((s["C"], H), np.float32)
    sync_gather = np.zeros((s["T"], H), np.float32)
    text_pp = np.zeros((2, s["TS"], H), np.float32)
    gcmlp = np.zeros((2, H), np.float32)
    m.get_conditioning(clip_pp, sync_gather, text_pp, gcmlp)
    ref = O.Oracle(prep_gguf).prep(s["T"], s["C"], s["TS"], s["sync_S"], inp["clip_f"], inp["sync_f"],
                                   inp["text_cat_cond"], inp["gtext_cond"], inp["text_cat_unc"], inp["gtext_unc"])
    got = {"clip_pp": clip_pp, "sync_gather": sync_gather, "text_pp_cond": text_pp[0], "gcmlp_cond": gcmlp[0],
           "text_pp_unc": text_pp[1], "gcmlp_unc": gcmlp[1]}
    for k in O.PREP_OUT:
        assert rel_l2(got[k], ref[k]) < PREP_TOL, (k, rel_l2(got[k], ref[k]))


@pytest.mark.gpu
def test_prep_then_forward_vs_oracle(dev, prep_gguf):
    """GPU prep feeding the GPU forward gives the oracle's flow (oracle prep feeding the oracle forward)."""
    s, H = PREP_SEQ, PREP_GEOM["H"]
    inp = prep_inputs()
    m = gpu_prep(dev, prep_gguf, inp)
    x = make_inputs(s["T"], s["C"], s["TS"], H, seed=SEED + 5)["x"]
    m.set_x(x)
    flow = np.zeros((2, s["T"], 64), np.float32)
    m.forward(0.5, flow)
    orc = O.Oracle(prep_gguf)
    ref = orc.prep(s["T"], s["C"], s["TS"], s["sync_S"], inp["clip_f"], inp["sync_f"],
                   inp["text_cat_cond"], inp["gtext_cond"], inp["text_cat_unc"], inp["gtext_unc"])
    for arm, sfx in ((0, "cond"), (1, "unc")):
        rf = orc.forward(s["T"], s["C"], s["TS"], x, 0.5, ref["clip_pp"], ref["sync_gather"], ref[f"text_pp_{sfx}"],
                         ref[f"gcmlp_{sfx}"])
        assert rel_l2(flow[arm].ravel(), rf.ravel()) < 1e-3


@pytest.mark.gpu
def test_prep_text_before_conditioning_is_refused(dev, prep_gguf):
    s = PREP_SEQ
    m = tsn.Dit(dev, gguf=prep_gguf)
    m.prepare(s["T"], s["C"], s["TS"], 2)
    inp = prep_inputs()
    with pytest.raises(tsn.TsnError) as e:
        m.prep_text_arm(0, inp["text_cat_cond"], inp["gtext_cond"])
    assert e.value.code == 9
