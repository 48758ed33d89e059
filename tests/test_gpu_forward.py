"""Parity of the fused CUDA forward / sampler (model face) against the CPU oracle.

Gates (north star): flow rel-L2 <= 1e-3 per step, every block tap the reference dumps
(src/dit_fwd.cpp:151-301) <= 2e-3, repeated GPU runs bit-identical
(tools/parity_dump.cpp:136-149). The oracle restates the reference bit-exactly (test_oracle.py).
"""
import os

import numpy as np
import pytest

import oracle as O
import tsn
from conftest import SEED, TINY, TINY_SEQ, WIDE, WIDE_SEQ, make_geom, make_inputs, rel_l2

pytestmark = pytest.mark.gpu

FLOW_TOL = 1e-3
TAP_TOL = 2e-3


@pytest.fixture(scope="module")
def dev():
    d = tsn.Device(0)
    yield d
    d.close()


def gpu_model(dev, gguf, inp, T, C, TS, compute=tsn.TSN_COMPUTE_F16, synthetic=None):
    m = tsn.Dit(dev, gguf=gguf, synthetic=synthetic, compute=compute)
    m.prepare(T, C, TS, 2)
    m.set_conditioning(inp["clip_pp"], inp["sync_gather"], np.stack([inp["text_pp_cond"], inp["text_pp_unc"]]),
                       np.stack([inp["gcmlp_cond"], inp["gcmlp_unc"]]))
    m.set_x(inp["x"])
    return m


def check_taps(m, orc, inp, T, C, TS, t, tap_tol=TAP_TOL, flow_tol=FLOW_TOL):
    flow = np.zeros((2, T, 64), np.float32)
    m.forward_taps(t, flow)
    report = {}
    for arm, sfx in ((0, "cond"), (1, "unc")):
        ref_flow = orc.forward(T, C, TS, inp["x"], t, inp["clip_pp"], inp["sync_gather"], inp[f"text_pp_{sfx}"],
                               inp[f"gcmlp_{sfx}"], taps=True)
        for name in O.TAPS:
            ref = ref_flow.ravel() if name == "flow" else orc.tap(name)
            got = m.tap(name, arm)
            assert got.shape == ref.shape, (name, got.shape, ref.shape)
            e = rel_l2(got, ref)
            report[(arm, name)] = e
        report[(arm, "flow_out")] = rel_l2(flow[arm], ref_flow)
    print("tap rel-L2:", {f"{k[0]}:{k[1]}": round(v, 7) for k, v in report.items()})
    bad = {k: v for k, v in report.items() if v > (flow_tol if k[1] in ("flow", "flow_out") else tap_tol)}
    worst = sorted(report.items(), key=lambda kv: -kv[1])[:6]
    assert not bad, f"over tolerance: {bad}; worst: {worst}"
    return report


def test_tiny_forward_taps_vs_oracle(dev, tiny_gguf):
    T, C, TS = TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"]
    inp = make_inputs(T, C, TS, TINY["H"])
    m = gpu_model(dev, tiny_gguf, inp, T, C, TS)
    check_taps(m, O.Oracle(tiny_gguf), inp, T, C, TS, 0.5)


def test_tiny_golden_flow(dev, tiny_gguf):
    g = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "tiny_forward.npz")))
    T, C, TS = int(g["T"]), int(g["C"]), int(g["TS"])
    inp = {k[3:]: g[k] for k in g if k.startswith("in_")}
    m = gpu_model(dev, tiny_gguf, inp, T, C, TS)
    flow = np.zeros((2, T, 64), np.float32)
    m.forward(float(g["t"]), flow)
    assert rel_l2(flow[0], g["tap_flow"]) < FLOW_TOL


def test_graph_replay_deterministic_and_equal_to_eager(dev, tiny_gguf):
    T, C, TS = TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"]
    inp = make_inputs(T, C, TS, TINY["H"])
    m = gpu_model(dev, tiny_gguf, inp, T, C, TS)
    a = np.zeros((2, T, 64), np.float32)
    b = np.zeros_like(a)
    c = np.zeros_like(a)
    m.forward(0.25, a)
    m.forward(0.25, b)
    m.forward_taps(0.25, c)
    assert np.array_equal(a, b), "repeat forward not bit-identical"
    assert np.array_equal(a, c), "graph replay differs from eager launch"


def test_tile_table_round_trip(dev, tiny_gguf):
    """Tiles read after autotuning and pinned on a fresh model reproduce the tuned forward bit for bit;
    pinning a different valid tile changes the plan but stays within the parity gate."""
    T, C, TS = TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"]
    inp = make_inputs(T, C, TS, TINY["H"])
    m = gpu_model(dev, tiny_gguf, inp, T, C, TS)
    m.autotune()
    tiles = m.tiles()
    assert tiles.shape[1] == 3 and len(tiles) > 0
    a = np.zeros((2, T, 64), np.float32)
    m.forward(0.25, a)
    m2 = gpu_model(dev, tiny_gguf, inp, T, C, TS)
    m2.set_tiles(tiles)
    assert np.array_equal(m2.tiles(), tiles)
    b = np.zeros_like(a)
    m2.forward(0.25, b)
    assert np.array_equal(a, b), "pinned tiles do not reproduce the tuned forward"
    # one GEMM on the narrowest tile without split-K: a valid different plan, same result within the gate
    t3 = tiles.copy()
    t3[0, 1:] = (64, 1)
    m2.set_tiles(t3)
    assert m2.tiles()[0, 1] == 64
    c = np.zeros_like(a)
    m2.forward(0.25, c)
    assert rel_l2(c, a) < 1e-5


def test_pair_kernel_tiles_vs_oracle(dev, tiny_gguf, monkeypatch):
    """The static tile plan, and the CTA-pair GEMM (tile code 2000 + NT: picked by the autotuner and by
    the tile table's 30 s entries) pinned on every GEMM it can serve, with 64- and 96-token tiles,
    without and with K slices: the flow stays within
    the gate of the CPU oracle, and the f32 outputs written through TMA store views equal the
    per-lane store epilogues (TSN_NO_TMA_OUT=1) bit for bit."""
    T, C, TS = TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"]
    inp = make_inputs(T, C, TS, TINY["H"])
    orc = O.Oracle(tiny_gguf)
    refs = [orc.forward(T, C, TS, inp["x"], 0.5, inp["clip_pp"], inp["sync_gather"], inp[f"text_pp_{sfx}"],
                        inp[f"gcmlp_{sfx}"]) for sfx in ("cond", "unc")]
    for code, slices in ((0, 0), (2064, 1), (2064, 2), (2096, 1)):   # 0: the static plan
        flows = []
        for tma in (True, False):
            if tma:
                monkeypatch.delenv("TSN_NO_TMA_OUT", raising=False)
            else:
                monkeypatch.setenv("TSN_NO_TMA_OUT", "1")
            m = gpu_model(dev, tiny_gguf, inp, T, C, TS)
            if slices:
                t = m.tiles().copy()
                t[:, 1], t[:, 2] = code, slices
                m.set_tiles(t)
                assert (m.tiles()[:, 1] == code).any(), "no GEMM took the pair tile"
            flow = np.zeros((2, T, 64), np.float32)
            m.forward(0.5, flow)
            for arm in (0, 1):
                assert rel_l2(flow[arm], refs[arm]) < FLOW_TOL, (code, slices, tma, arm)
            flows.append(flow)
        assert np.array_equal(flows[0], flows[1]), f"TMA-store and per-lane epilogues differ ({code}, K slices {slices})"
    monkeypatch.delenv("TSN_NO_TMA_OUT", raising=False)


def test_synthetic_device_weights_equal_file(dev, tiny_gguf):
    T, C, TS = TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"]
    inp = make_inputs(T, C, TS, TINY["H"])
    a = np.zeros((2, T, 64), np.float32)
    b = np.zeros_like(a)
    gpu_model(dev, tiny_gguf, inp, T, C, TS).forward(0.5, a)
    gpu_model(dev, None, inp, T, C, TS, synthetic=make_geom(**TINY)).forward(0.5, b)
    assert np.array_equal(a, b)


def test_tiny_sample_vs_golden(dev, tiny_gguf):
    g = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "tiny_sample.npz")))
    T, C, TS = int(g["T"]), int(g["C"]), int(g["TS"])
    inp = {k[3:]: g[k] for k in g if k.startswith("in_")}
    m = gpu_model(dev, tiny_gguf, inp, T, C, TS)
    m.sample(int(g["steps"]), float(g["cfg"]))
    x = np.zeros((T, 64), np.float32)
    m.get_x(x)
    # CFG 5 amplifies per-step flow error ~5x into x; 4 steps accumulate
    assert rel_l2(x, g["x_final"]) < 5e-3


def test_tiny_step_vs_oracle(dev, tiny_gguf):
    T, C, TS = TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"]
    inp = make_inputs(T, C, TS, TINY["H"], seed=SEED + 1)
    m = gpu_model(dev, tiny_gguf, inp, T, C, TS)
    t, dt = 1.0, float(np.float32(1.0 - 1.0 / 24) - np.float32(1.0))
    m.step(t, 5.0, dt)
    x = np.zeros((T, 64), np.float32)
    m.get_x(x)
    orc = O.Oracle(tiny_gguf)
    xr, fc, fu = orc.step(T, C, TS, inp["x"], t, 5.0, dt, inp["clip_pp"], inp["sync_gather"], inp["text_pp_cond"],
                          inp["gcmlp_cond"], inp["text_pp_unc"], inp["gcmlp_unc"])
    # compare the update dt*(fu + 5(fc - fu)) itself: x carries the unchanged noise
    assert rel_l2(x - inp["x"], xr - inp["x"]) < 5 * FLOW_TOL


def test_step_host_buffers_match_device_step(dev, tiny_gguf):
    """tsn_dit_step_host (copy in, schedule row, the step graph, copy out) gives the device step's
    bits with pageable numpy buffers, with page-locked buffers, in place (x_in is x_out) and across
    repeated calls at other t and dt."""
    import torch
    T, C, TS = TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"]
    inp = make_inputs(T, C, TS, TINY["H"], seed=SEED + 2)
    m = gpu_model(dev, tiny_gguf, inp, T, C, TS)
    sched = [(1.0, -1.0 / 24), (0.75, -0.05), (0.5, -1.0 / 24)]

    def device_steps(x0, n):
        m.set_x(x0)
        out = []
        for t, dt in sched[:n]:
            m.step(t, 5.0, dt)
            x = np.zeros((T, 64), np.float32)
            m.get_x(x)
            out.append(x)
        return out

    ref = device_steps(inp["x"], 3)
    # pageable buffers
    xo = np.zeros((T, 64), np.float32)
    m.step_host(np.ascontiguousarray(inp["x"]), xo, sched[0][0], 5.0, sched[0][1])
    assert np.array_equal(xo, ref[0])
    # page-locked buffers, then in place on the same pinned buffer for the next steps
    xin = torch.from_numpy(inp["x"].copy()).pin_memory()
    xout = torch.zeros_like(xin).pin_memory()
    m.step_host(xin, xout, sched[0][0], 5.0, sched[0][1])
    assert np.array_equal(xout.numpy(), ref[0])
    for k in (1, 2):
        m.step_host(xout, xout, sched[k][0], 5.0, sched[k][1])
        assert np.array_equal(xout.numpy(), ref[k]), k
    # the first pair again (its graph is cached): the same bits as the first time
    m.step_host(xin, xout, sched[0][0], 5.0, sched[0][1])
    assert np.array_equal(xout.numpy(), ref[0])
    m.close()


def test_bf16_operands_rejected(dev, tiny_gguf):
    """BF16 operands are refused loudly (they cannot meet the 1e-3 flow gate), not silently downgraded."""
    with pytest.raises(tsn.TsnError) as e:
        tsn.Dit(dev, gguf=tiny_gguf, compute=tsn.TSN_COMPUTE_BF16)
    assert e.value.code == 7


def test_wide_forward_taps_vs_oracle(dev, wide_gguf):
    """Real widths (H=1024, 16 heads, F=4096) at the 8 s geometry, 2 joint + 1 fused block."""
    T, C, TS = WIDE_SEQ["T"], WIDE_SEQ["C"], WIDE_SEQ["TS"]
    inp = make_inputs(T, C, TS, WIDE["H"])
    m = gpu_model(dev, wide_gguf, inp, T, C, TS)
    check_taps(m, O.Oracle(wide_gguf), inp, T, C, TS, 0.5)


def test_wide_long_context_taps_vs_oracle(dev, wide_gguf):
    """BASELINE config 4 geometry (30 s: 704 latent rows, 240 clip rows, 77 text rows; joint
    S = 1021, not a multiple of the 64-row attention tiles), real widths, 2 joint + 1 fused block."""
    T, C, TS = 704, 240, 77
    inp = make_inputs(T, C, TS, WIDE["H"], seed=SEED + 3)
    m = gpu_model(dev, wide_gguf, inp, T, C, TS)
    check_taps(m, O.Oracle(wide_gguf), inp, T, C, TS, 0.75)


def test_single_arm_matches_batched(dev, tiny_gguf):
    """arms=1 (one CFG arm per GPU) gives the same flow as the arms=2 batch."""
    T, C, TS = TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"]
    inp = make_inputs(T, C, TS, TINY["H"])
    both = np.zeros((2, T, 64), np.float32)
    gpu_model(dev, tiny_gguf, inp, T, C, TS).forward(0.5, both)
    for arm, sfx in ((0, "cond"), (1, "unc")):
        m = tsn.Dit(dev, gguf=tiny_gguf)
        m.prepare(T, C, TS, 1)
        m.set_conditioning(inp["clip_pp"], inp["sync_gather"], inp[f"text_pp_{sfx}"], inp[f"gcmlp_{sfx}"])
        m.set_x(inp["x"])
        one = np.zeros((1, T, 64), np.float32)
        m.forward(0.5, one)
        assert rel_l2(one[0], both[arm]) < 1e-5


FULL = dict(H=1024, NH=16, F=4096, depth=21, fused_depth=14)


@pytest.fixture(scope="module")
def full_gguf(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("gguf_full") / "full.gguf")
    tsn.write_synthetic_gguf(p, make_geom(**FULL), SEED)
    yield p
    os.unlink(p)


def test_full_depth_forward_vs_oracle(dev, full_gguf):
    """the full 21-block MMDiT (7 joint + 14 fused), 8 s geometry, t = 0.5."""
    T, C, TS = WIDE_SEQ["T"], WIDE_SEQ["C"], WIDE_SEQ["TS"]
    inp = make_inputs(T, C, TS, FULL["H"])
    m = gpu_model(dev, full_gguf, inp, T, C, TS)
    check_taps(m, O.Oracle(full_gguf), inp, T, C, TS, 0.5)


@pytest.mark.parametrize("G", [2, 4])
def test_generations_batched_match_single(dev, tiny_gguf, G):
    """arms = 2G (G generations, each with its cond and uncond arm; G = 4 is bench.py --config5's
    batch) gives each generation its own flow and sampler step. At G = 2 the GEMMs get the same
    tiles as one generation, so the sums, and the results, are those of the single-generation
    model (to 1e-5). At G = 4 (192 latent rows) the tile plan differs, the f32 sums run in another
    order, and an occasional f16 rounding of the FFN down-projection input flips: each generation
    is checked against the CPU oracle instead (flow within the 1e-3 gate), and against the single-
    generation model within the same gate."""
    T, C, TS = TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"]
    gens = [make_inputs(T, C, TS, TINY["H"], seed=SEED + 20 + g) for g in range(G)]
    m = tsn.Dit(dev, gguf=tiny_gguf)
    m.prepare(T, C, TS, 2 * G)
    m.set_conditioning(np.stack([g["clip_pp"] for g in gens]), np.stack([g["sync_gather"] for g in gens]),
                       np.stack([g[k] for g in gens for k in ("text_pp_cond", "text_pp_unc")]),
                       np.stack([g[k] for g in gens for k in ("gcmlp_cond", "gcmlp_unc")]))
    m.set_x(np.stack([g["x"] for g in gens]))
    flowG = np.zeros((2 * G, T, 64), np.float32)
    m.forward(0.5, flowG)
    dt = float(np.float32(1.0 - 1.0 / 24) - np.float32(1.0))
    m.step(1.0, 5.0, dt)
    xG = np.zeros((G, T, 64), np.float32)
    m.get_x(xG)
    tol = 1e-5 if G == 2 else FLOW_TOL
    orc = O.Oracle(tiny_gguf) if G > 2 else None
    for g, inp in enumerate(gens):
        one = gpu_model(dev, tiny_gguf, inp, T, C, TS)
        flow2 = np.zeros((2, T, 64), np.float32)
        one.forward(0.5, flow2)
        assert rel_l2(flowG[2 * g:2 * g + 2], flow2) < tol
        if orc is not None:
            for arm, sfx in ((0, "cond"), (1, "unc")):
                ref = orc.forward(T, C, TS, inp["x"], 0.5, inp["clip_pp"], inp["sync_gather"], inp[f"text_pp_{sfx}"],
                                  inp[f"gcmlp_{sfx}"])
                assert rel_l2(flowG[2 * g + arm], ref) < FLOW_TOL, (g, arm)
        one.step(1.0, 5.0, dt)
        x1 = np.zeros((T, 64), np.float32)
        one.get_x(x1)
        assert rel_l2(xG[g] - inp["x"], x1 - inp["x"]) < tol


@pytest.mark.parametrize("T", [WIDE_SEQ["T"], 96])
def test_grouped_w13_persistent_text_tiles_same_bits(dev, wide_gguf, monkeypatch, T):
    """The joint blocks' grouped w1/w3 launch runs the text stream as persistent 208-wide tile lists
    on the SMs the latent and clip tiles leave free; its outputs are the same dot products as the
    ordinary 256-wide tiles (TSN_NO_PERSIST_GROUP=1), so the flows are bit-identical. At T = 188
    the 80 text tiles come out as 20 lists of four; at T = 96 (96 deep tiles) as 52 lists of one or
    two."""
    C, TS = WIDE_SEQ["C"], WIDE_SEQ["TS"]
    inp = make_inputs(T, C, TS, WIDE["H"])
    flows = []
    for off in (False, True):
        if off:
            monkeypatch.setenv("TSN_NO_PERSIST_GROUP", "1")
        else:
            monkeypatch.delenv("TSN_NO_PERSIST_GROUP", raising=False)
        m = gpu_model(dev, wide_gguf, inp, T, C, TS)
        gemms = [l for l in m.profile_ops().splitlines() if "bn=" in l]
        t = m.tiles().copy()
        for i, l in enumerate(gemms):   # the grouped w1/w3 on 256-wide tiles, the width the table gives at 8 s
            if l.split()[1] == "ffn_w13" and "group=" in l:
                t[i, 1:] = (256, 1)
        m.set_tiles(t)
        ops = [l for l in m.profile_ops().splitlines() if "ffn_w13" in l and "group=" in l]
        assert ops and all(("persist=" in l) != off for l in ops), ops
        flow = np.zeros((2, T, 64), np.float32)
        m.forward(0.5, flow)
        flows.append(flow)
        m.close()
    monkeypatch.delenv("TSN_NO_PERSIST_GROUP", raising=False)
    assert np.array_equal(flows[0], flows[1])


@pytest.mark.parametrize("code", [2192, 2096])
def test_pair_kernel_swiglu_real_widths_vs_oracle(dev, wide_gguf, code):
    """The CTA-pair GEMM with 192- and 96-token tiles (96: an arm's 188 latent rows as 96 + 92)
    pinned on the FFN w1/w3 GEMMs (SwiGLU epilogue through the staged f16 tile) at real widths and
    the 8 s latent length: flow within the gate."""
    T, C, TS = WIDE_SEQ["T"], WIDE_SEQ["C"], WIDE_SEQ["TS"]
    inp = make_inputs(T, C, TS, WIDE["H"])
    m = gpu_model(dev, wide_gguf, inp, T, C, TS)
    gemms = [l for l in m.profile_ops().splitlines() if "bn=" in l]
    t = m.tiles().copy()
    # the single (not grouped) w1/w3 launches: fused blocks, the pre-only joint block, audio_in
    w13 = [i for i, l in enumerate(gemms) if l.split()[1] in ("ffn_w13", "audio_in.w13") and "group=" not in l]
    assert w13
    for i in w13:
        t[i, 1:] = (code, 1)
    m.set_tiles(t)
    assert all(m.tiles()[i, 1] == code for i in w13), "a w1/w3 GEMM did not take the pair tile"
    flow = np.zeros((2, T, 64), np.float32)
    m.forward(0.5, flow)
    orc = O.Oracle(wide_gguf)
    for arm, sfx in ((0, "cond"), (1, "unc")):
        ref = orc.forward(T, C, TS, inp["x"], 0.5, inp["clip_pp"], inp["sync_gather"], inp[f"text_pp_{sfx}"],
                          inp[f"gcmlp_{sfx}"])
        assert rel_l2(flow[arm], ref) < FLOW_TOL
