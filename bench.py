"""MMDiT CFG denoise steps/s on B200 (BASELINE.json metric), one JSON line on rank 0.

A step is one rectified-flow Euler step of the sampler (src/pipeline.cpp:146-148): the 21-block
MMDiT forward for the cond and uncond arms (batched) plus the CFG-Euler update, on the 8 s
geometry of BASELINE config 2/3 (T=188 latent rows, 64 clip rows, 77 text rows, H=1024, 16 heads,
F=4096) with seeded synthetic weights N(0,0.02) generated on the device.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl tsn|reference]

Multi-GPU (torchrun, one process per GPU): every rank samples its own generation (data-parallel
generations) with no cross-GPU traffic in the timed region; value is the
steps of all ranks divided by the slowest rank's device time (weak scaling).
With --cfg-split, ranks 2k and 2k+1 share one generation instead: each runs one CFG arm and the
pair all-gathers the two flows every step (BASELINE config 3 on 2 GPUs; a latency mode).
With --config5, the ranks share BASELINE config 5: 64 independent 24-step generations (seeds
0..63, contiguous seed ranges per rank), --gens-per-forward of them batched in each forward, and
one gather of the final latents to rank 0; the line reports generations/s.

--impl reference times the reference's own CPU implementation of the path (the reference's
src/dit_fwd.cpp built over the scalar kernel transliteration in oracle/_ref; the oracle port when
that build is absent) on the host cores, same config and metric; rank 0 only.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "thinksound-native_b200"))

METRIC = "MMDiT CFG denoise steps/s (8 s audio) at 1/2/4/8 B200; % of step roofline"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=48)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="tsn", choices=["tsn", "reference"])
    ap.add_argument("--T", type=int, default=188)
    ap.add_argument("--C", type=int, default=64)
    ap.add_argument("--TS", type=int, default=77)
    ap.add_argument("--H", type=int, default=1024)
    ap.add_argument("--F", type=int, default=4096)
    ap.add_argument("--depth", type=int, default=21)
    ap.add_argument("--fused", type=int, default=14)
    ap.add_argument("--cfg", type=float, default=5.0)
    ap.add_argument("--seed", type=int, default=4242)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--profile-ops", action="store_true", help="print one line per launch of an eager step to stderr")
    ap.add_argument("--autotune", action="store_true",
                    help="time every tile candidate at load instead of the library's built-in tile table (the tuned "
                         "forward may then differ from other processes' in the last bits)")
    ap.add_argument("--cfg-split", action="store_true", help="one CFG arm per rank, pairs of ranks per generation")
    ap.add_argument("--trace-ops", action="store_true",
                    help="print per-CTA phase stamps (medians) of one launch of each op kind of a fused block to stderr")
    ap.add_argument("--cpu-configs", action="store_true",
                    help="time BASELINE configs 1 and 2 on the host cores (oracle port / reference build)")
    ap.add_argument("--cfg-split-eager", action="store_true", help="--cfg-split with the steps issued from the host")
    ap.add_argument("--long", action="store_true", help="BASELINE config 4 geometry: 30 s audio (T=704, clip 240, text 77)")
    ap.add_argument("--config5", action="store_true", help="64 generations x 24 steps, data-parallel, final gather")
    ap.add_argument("--gens-per-forward", type=int, default=4, help="config 5: generations batched per forward (1-4)")
    ap.add_argument("--generations", type=int, default=64)
    ap.add_argument("--vae", action="store_true",
                    help="the VAE decoder after the sampler (src/vae.cpp): decode T latent frames, synthetic f32 weights")
    ap.add_argument("--vae-channels", type=int, default=128)
    ap.add_argument("--encoders", action="store_true",
                    help="the text encoders before the sampler (src/t5.cpp, src/clip.cpp) at full size, synthetic weights")
    ap.add_argument("--encoder-layers", type=int, default=24)
    return ap.parse_args()


def apply_long(a):
    if a.long:
        a.T, a.C, a.TS = 704, 240, 77


def geom_kwargs(a):
    return dict(H=a.H, NH=a.H // 64, F=a.F, depth=a.depth, fused_depth=a.fused)


def workload(a, what=None):
    geo = "30 s audio geometry (config 4)" if (a.T, a.C) == (704, 240) else "8 s audio geometry" if a.T == 188 else \
        f"T={a.T} geometry"
    what = what or (f"config{'4' if (a.T, a.C) == (704, 240) else '2/3'}: {a.depth}-block MMDiT CFG Euler step "
                    f"({a.depth - a.fused} joint + {a.fused} fused), {geo}, cond+uncond batched")
    return {"workload": what,
            "T": a.T, "clip_S": a.C, "text_S": a.TS, "H": a.H, "heads": a.H // 64, "F": a.F, "cfg": a.cfg,
            "weights": "synthetic BF16 N(0,0.02) -> f16 operands (reference weight conversion)",
            "l2": "inputs larger than L2: every step streams ~3.1 GB of weights from HBM (L2 126 MB)"}


# ------------------------------------------------------------------------------------ FLOPs
def step_flops_bytes(a):
    """Algorithmic FLOPs (2*M*N*K over every GEMM/conv/GEMV + 4*S^2*H attention, both arms) and
    weight bytes (BF16/f16 once per step) of one CFG step, counted from src/dit_fwd.cpp:104-304."""
    H, F, L, T, C, TS, B = a.H, a.F, 64, a.T, a.C, a.TS, 2
    nj, nf = a.depth - a.fused, a.fused
    params = 0
    fl = 0

    def lin(rows, n, k):
        nonlocal params, fl
        params += n * k
        fl += 2 * B * rows * n * k

    lin(1, H, H); lin(1, H, H)                       # t_embed (M=1 per arm on the reference)
    lin(T, H, 3 * L); lin(T, 2 * F, 3 * H); lin(T, H, 3 * F)    # audio_input_proj
    for i in range(nj):
        pre = i == nj - 1
        lin(T, 6 * H, H); lin(T, 3 * H, H)
        lin(1, (2 if pre else 6) * H, H); lin(C, 3 * H, H)
        lin(1, (2 if pre else 6) * H, H); lin(TS, 3 * H, H)
        lin(T, H, 3 * H); lin(T, 2 * F, 3 * H); lin(T, H, 3 * F)
        if not pre:
            lin(C, H, 3 * H); lin(C, 2 * F, 3 * H); lin(C, H, 3 * F)
            lin(TS, H, H); lin(TS, 2 * F, H); lin(TS, H, F)
        S = T + C + TS
        fl += 4 * B * S * S * H
    for _ in range(nf):
        lin(T, 6 * H, H); lin(T, 3 * H, H)
        lin(T, H, 3 * H); lin(T, 2 * F, 3 * H); lin(T, H, 3 * F)
        fl += 4 * B * T * T * H
    lin(T, 2 * H, H); lin(T, L, 7 * H)
    return fl, 2 * params


def dominant_gemm(profile_text):
    """The GEMM (name + tile configuration) with the largest device time per step in the eager
    per-op profile: (name, desc, launches, mean ms per launch, algorithmic FLOPs per launch)."""
    groups = {}
    for line in profile_text.splitlines():
        p = line.split()
        if len(p) < 7 or "bn=" not in line:
            continue
        name, ms = p[1], float(p[2])
        flops = float(p[-1].split("=")[1])
        desc = " ".join(p[6:-1])
        g = groups.setdefault((name, desc), [0, 0.0, flops])
        g[0] += 1
        g[1] += ms
    (name, desc), (n, tot, flops) = max(groups.items(), key=lambda kv: kv[1][1])
    return name, desc, n, tot / n, flops


def measured_traffic(name, desc):
    """DRAM bytes per launch of that GEMM from the committed ncu summary (profiles/), or None."""
    p = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    if not os.path.exists(p):
        return None, None
    d = json.load(open(p))
    for k in d.get("kernels", []):
        if k["op"] == name and k["tile"] in desc:
            return k["dram_bytes_per_launch"], k["source"]
    return None, None


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


# ------------------------------------------------------------------------------------ clocks
class Clocks:
    def __init__(self, gpu_index, enabled=True):
        self.proc = None
        self.path = None
        if not enabled:
            return
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={gpu_index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                try:
                    rows.append((float(f[1]), float(f[2]), f[5:9]))
                except ValueError:
                    pass
        os.unlink(self.path)
        if not rows:
            return None
        load = [r for r in rows if r[0] > 0.5 * r[1]] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in load for i, v in enumerate(r[2]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in load), "sm_max_mhz": max(r[1] for r in rows),
                "samples": len(rows), "samples_under_load": len(load), "reasons": reasons}


# ------------------------------------------------------------------------------------ CPU arms
def cpu_reference_steps(a, reps, threads):
    """Time `reps` CFG steps of the reference's host code (oracle/_ref) or the oracle port on the
    host cores; returns (seconds per step list, kind, sample description)."""
    import numpy as np

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    tmp = tempfile.mkdtemp(prefix="tsn_cpu_")
    gguf = os.path.join(tmp, "dit.gguf")
    # written by the oracle library: the CPU arms never load the GPU library
    O.write_synthetic_gguf(gguf, seed=a.seed, **geom_kwargs(a))
    rng = np.random.default_rng(a.seed)
    f = lambda *s: rng.standard_normal(s, dtype=np.float32)  # noqa: E731
    inp = {"x": f(a.T, 64), "clip_pp": f(a.C, a.H), "sync_gather": f(a.T, a.H), "text_pp_cond": f(a.TS, a.H),
           "text_pp_unc": f(a.TS, a.H), "gcmlp_cond": f(a.H), "gcmlp_unc": f(a.H)}
    try:
        if O.have_ref():
            O.write_inputs(os.path.join(tmp, "in"), inp)
            out = O.run_ref("step", gguf, a.T, a.C, a.TS, os.path.join(tmp, "in"), os.path.join(tmp, "out"),
                            0.5, a.cfg, -1.0 / 24, reps, threads=threads)
            secs = O.parse_json_line(out)["seconds"]
            kind = "reference"
        else:
            os.environ["OMP_NUM_THREADS"] = str(threads)
            orc = O.Oracle(gguf)
            secs = []
            x = inp["x"]
            for _ in range(reps):
                t0 = time.perf_counter()
                x, _, _ = orc.step(a.T, a.C, a.TS, x, 0.5, a.cfg, -1.0 / 24, inp["clip_pp"], inp["sync_gather"],
                                   inp["text_pp_cond"], inp["gcmlp_cond"], inp["text_pp_unc"], inp["gcmlp_unc"])
                secs.append(time.perf_counter() - t0)
            kind = "port"
    finally:
        for fn in os.listdir(tmp):
            p = os.path.join(tmp, fn)
            if os.path.isdir(p):
                for g in os.listdir(p):
                    os.unlink(os.path.join(p, g))
                os.rmdir(p)
            else:
                os.unlink(p)
        os.rmdir(tmp)
    sample = (f"{len(secs)} full CFG step(s) ({a.depth} blocks, T={a.T}, clip {a.C}, text {a.TS}, both arms + cfg_euler) "
              f"of the {'reference host code (src/dit_fwd.cpp) over the scalar kernel transliteration' if kind == 'reference' else 'oracle port'}, "
              f"f32 activations, OpenMP over output rows")
    return secs, kind, sample


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    reps = a.warmup + a.steps
    secs, kind, sample = cpu_reference_steps(a, reps, threads)
    timed = secs[a.warmup:] if len(secs) > a.warmup else secs
    value = len(timed) / sum(timed)
    print(json.dumps({
        "metric": METRIC, "impl": "reference", "value": value, "unit": "steps/s", "n_gpus": a.gpus,
        "steps": len(timed), "warmup": a.warmup, "ms_per_step": 1e3 * sum(timed) / len(timed),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload(a),
        "cpu_baseline": {"value": value, "unit": "steps/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ------------------------------------------------------------------------------------ GPU arm
def run_tsn(a):
    import numpy as np
    import torch

    import tsn

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    stream = torch.cuda.Stream()
    dev = tsn.Device(local, stream=stream.cuda_stream)
    m = tsn.Dit(dev, synthetic=tsn.geom(**geom_kwargs(a)), seed=a.seed)
    m.prepare(a.T, a.C, a.TS, 2)
    rng = np.random.default_rng(a.seed + 1000 * rank)     # per-rank generation (config 5: seeds per generation)
    f = lambda *s: rng.standard_normal(s, dtype=np.float32)  # noqa: E731
    m.set_conditioning(f(a.C, a.H), f(a.T, a.H), f(2, a.TS, a.H), f(2, a.H))
    m.set_x(f(a.T, 64))
    tiles_desc = "built-in B200 tile table (fixed per GEMM shape, cost model for unlisted shapes): the same bits " \
                 "in every process"
    if a.autotune:
        rep = m.autotune()
        tiles_desc = "autotuned per shape at load"
        if a.profile_ops and rank == 0:
            print(rep, file=sys.stderr, flush=True)
    total = a.warmup + a.steps
    m.schedule(min(total, 1024), a.cfg)

    with torch.cuda.stream(stream):
        m.run_steps(a.warmup)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        clocks = Clocks(local, enabled=not a.no_clocks)
        time.sleep(0.3 if clocks.proc else 0)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        m.run_steps(a.steps)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        clk = clocks.stop()
    x = np.zeros((a.T, 64), np.float32)
    m.get_x(x)
    finite = bool(np.isfinite(x).all())

    # e2e: the public host-buffer step (tsn_dit_step_host): H2D of x and the step's schedule row,
    # the step, D2H of x, every step
    e2e_ms = None
    h2d = a.T * 64 * 4 + a.H * 4 + 4
    d2h = a.T * 64 * 4
    if not a.no_e2e:
        xin = torch.from_numpy(f(a.T, 64)).pin_memory()
        xout = torch.empty_like(xin).pin_memory()
        for _ in range(2):
            m.step_host(xin, xout, 0.5, a.cfg, -1.0 / 24)
        if dist:
            dist.barrier()
        with torch.cuda.stream(stream):
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            for i in range(a.steps):
                m.step_host(xout if i else xin, xout, 0.5, a.cfg, -1.0 / 24)
            s1.record(stream)
            torch.cuda.synchronize()
            e2e_ms = s0.elapsed_time(s1)

    prof = m.profile_step()
    kps = m.kernels_per_step()
    ops_text = m.profile_ops()
    if a.trace_ops and rank == 0:
        trace_ops(m, ops_text)
    if a.profile_ops and rank == 0:
        print(ops_text, file=sys.stderr, flush=True)
    times = torch.tensor([ms, e2e_ms or 0.0], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms, e2e_ms = float(times[0]), float(times[1]) if e2e_ms is not None else None

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        threads = os.cpu_count() or 1
        secs, kind, sample = cpu_reference_steps(a, 1, threads)
        cpu = {"value": 1.0 / secs[-1], "unit": "steps/s", "cores": threads, "kind": kind, "sample": sample}

    if rank == 0:
        flops, wbytes = step_flops_bytes(a)
        hbm, tf_burst, tf_sus, src = peaks()
        step_ms = ms / a.steps
        compute_ms = flops / (tf_sus * 1e12) * 1e3
        hbm_ms = wbytes / (hbm * 1e9) * 1e3
        bound_ms = max(compute_ms, hbm_ms)
        g_ms = prof["gemm_ms"]
        g_tf = prof["gemm_flops"] / (g_ms * 1e-3) / 1e12 if g_ms > 0 else 0.0
        d_name, d_desc, d_n, d_ms, d_flops = dominant_gemm(ops_text)
        d_tf = d_flops / (d_ms * 1e-3) / 1e12
        traffic, t_src = measured_traffic(d_name, d_desc)
        out = {
            "metric": METRIC, "value": world * a.steps / (ms * 1e-3), "unit": "steps/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 (split hi+lo activations), f32 accumulate", "data": "synthetic",
            "config": workload(a),
            "parallelism": f"dp{world} (one generation per GPU, no data-path collective)",
            "gemm_tiles": tiles_desc,
            # dominant kernel: the GEMM with the most device time per step, each launch timed with
            # CUDA events on its stream (eager per-op pass after the timed region), against the
            # burst bf16 peak (a kernel timed alone)
            "roofline": {"bound": "tensor", "achieved": d_tf, "peak": tf_burst, "unit": "TFLOP/s",
                         "frac": d_tf / tf_burst, "traffic": traffic,
                         "kernel": f"gemm_tc_kernel {d_name} ({d_desc})", "launches_per_step": d_n,
                         "ms_per_launch": d_ms, "algorithmic_flops_per_launch": d_flops,
                         "peak_source": f"{src} bf16_tflops (burst)", "traffic_source": t_src,
                         "all_gemms": {"achieved_tflops": g_tf, "frac_of_sustained": g_tf / tf_sus,
                                       "algorithmic_flops_per_step": prof["gemm_flops"], "gemm_ms_per_step": g_ms,
                                       "gemm_launches_per_step": prof["gemm_launches"]},
                         "attention_ms_per_step": prof["attn_ms"], "other_ms_per_step": prof["other_ms"]},
            "step_roofline": {"algorithmic_gflop": flops / 1e9, "weight_gb": wbytes / 1e9, "compute_ms": compute_ms,
                              "hbm_ms": hbm_ms, "bound": "tensor" if compute_ms >= hbm_ms else "hbm",
                              "roofline_ms": bound_ms, "frac": bound_ms / step_ms,
                              "peaks": f"{src}: {tf_sus} TFLOP/s sustained bf16, {hbm} GB/s"},
            "cpu_baseline": cpu,
            "e2e": ({"value": world * a.steps / (e2e_ms * 1e-3), "unit": "steps/s", "h2d_bytes_per_step": h2d,
                     "d2h_bytes_per_step": d2h} if e2e_ms else None),
            "gpu_launches": kps * a.steps,
            "clocks": clk,
            "x_finite": finite,
        }
        print(json.dumps(out), flush=True)
    m.close()
    dev.close()
    if dist:
        dist.destroy_process_group()


def trace_ops(m, ops_text):
    """Per-CTA phase stamps (tsn_dit_trace_op) of the first launch of each op kind past the joint
    blocks, as medians over the CTAs (us), one JSON line per launch on stderr. GEMMs and the short
    attention stamp 8 phases (entry, setup / upstream done, first operand stage / Q landed, MMA done /
    every score product done, epilogue done / row max known, exit), adaLN and GEMV launches 3 (entry,
    upstream done, exit)."""
    import numpy as np

    names = {}
    for line in ops_text.splitlines():
        p = line.split()
        if len(p) > 2 and p[0].isdigit():
            names[int(p[0])] = (p[1], " ".join(p[2:]))
    first = {}
    start = max(names) // 3 if names else 0
    for i, (n, _) in sorted(names.items()):
        if i >= start and n not in first:
            first[n] = i
    for n, i in first.items():
        try:
            st = m.trace_op(i).astype(np.int64)
        except Exception:   # not a stamped launch
            continue
        if len(st) == 0:
            continue
        med = lambda b, e: float(np.median(st[:, e] - st[:, b]) / 1e3)  # noqa: E731
        if st[:, 5].max() > 0:
            ph = {"upstream+setup": med(0, 1), "to_first_data": med(1, 2), "main": med(2, 3), "epilogue": med(3, 4),
                  "to_exit": med(4, 5)}
        else:
            ph = {"to_upstream_done": med(0, 1), "work": med(1, 2)}
        print(json.dumps({"trace_op": n, "op": i, "ctas": int(len(st)), "median_us": {k: round(v, 2) for k, v in ph.items()},
                          "desc": names[i][1][:80]}), file=sys.stderr, flush=True)


def run_cfg_split(a):
    """Pairs of ranks sample one generation each, one CFG arm per rank (tsn.cfg_split)."""
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    import tsn
    from tsn import cfg_split

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world < 2 or world % 2:
        if rank == 0:
            print(json.dumps({"metric": METRIC, "error": "--cfg-split needs an even number of ranks"}), flush=True)
        return
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    pairs = [dist.new_group([2 * k, 2 * k + 1]) for k in range(world // 2)]
    group, arm = pairs[rank // 2], rank % 2
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        dev = tsn.Device(local, stream=stream.cuda_stream)
        m = tsn.Dit(dev, synthetic=tsn.geom(**geom_kwargs(a)), seed=a.seed)
        m.prepare(a.T, a.C, a.TS, 1)
        rng = np.random.default_rng(a.seed + 1000 * (rank // 2))     # one generation per pair
        f = lambda *s: rng.standard_normal(s, dtype=np.float32)  # noqa: E731
        clip, sync, text, gc, x0 = f(a.C, a.H), f(a.T, a.H), f(2, a.TS, a.H), f(2, a.H), f(a.T, 64)
        m.set_conditioning(clip, sync, text[arm], gc[arm])
        m.set_x(x0)
        if a.autotune:
            m.autotune()
        sampler = cfg_split.CfgSplitSampler(m, dev, a.T, group=group)
        xs = torch.from_numpy(x0).cuda()
        x = torch.empty_like(xs)
        # each step (this arm's forward, the NCCL all-gather of the two flows, the CFG update) is
        # replayed from one CUDA graph; --cfg-split-eager runs the steps from the host instead
        if not a.cfg_split_eager:
            sampler.graph_capture(xs, a.cfg)
            sampler.graph_run(xs, a.warmup)
        else:
            x.copy_(xs)
            sampler.sample(x, a.warmup, a.cfg)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if not a.cfg_split_eager:
            m.set_x(xs)
            m.split_schedule(a.steps)
            e0.record(stream)
            for _ in range(a.steps):
                sampler.graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            m.get_x(x)
            sampler.graph_release()
        else:
            x.copy_(xs)
            e0.record(stream)
            sampler.sample(x, a.steps, a.cfg)
            e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        times = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
        ms = float(times[0])
        finite = bool(torch.isfinite(x).all())
        if rank == 0:
            flops, wbytes = step_flops_bytes(a)
            hbm, _, tf_sus, src = peaks()
            compute_ms = flops / 2 / (tf_sus * 1e12) * 1e3     # each GPU does one arm
            hbm_ms = wbytes / (hbm * 1e9) * 1e3                 # ... but streams every weight
            step_ms = ms / a.steps
            print(json.dumps({
                "metric": METRIC, "value": (world // 2) * a.steps / (ms * 1e-3), "unit": "steps/s", "n_gpus": world,
                "steps": a.steps, "warmup": a.warmup, "ms_per_step": step_ms, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f16 (split hi+lo activations), f32 accumulate",
                "data": "synthetic",
                "config": workload(a, f"config2/3 CFG pair split: {a.depth}-block MMDiT CFG Euler step, one arm per GPU, "
                                      f"8 s audio geometry" if a.T == 188 else None),
                "parallelism": f"cfg-split x{world // 2} (one CFG arm per GPU, NCCL all-gather of the flow every step"
                               f"{', steps from the host' if a.cfg_split_eager else ', every step one CUDA graph'})",
                "step_roofline": {"compute_ms": compute_ms, "hbm_ms": hbm_ms, "roofline_ms": max(compute_ms, hbm_ms),
                                  "frac": max(compute_ms, hbm_ms) / step_ms,
                                  "peaks": f"{src}: {tf_sus} TFLOP/s sustained bf16, {hbm} GB/s"},
                "x_finite": finite}), flush=True)
        m.close()
        dev.close()
    for g in pairs:
        dist.destroy_process_group(g)
    dist.destroy_process_group()


def run_config5(a):
    """`generations` independent 24-step generations split over the ranks as
    contiguous seed ranges, G = --gens-per-forward of them sampled together (arms = 2G); the final
    latents are gathered to rank 0 once at the end."""
    import datetime

    import numpy as np
    import torch

    import tsn

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    G = max(1, min(4, a.gens_per_forward))
    per_rank = (a.generations + world - 1) // world
    mine = list(range(rank * per_rank, min(a.generations, (rank + 1) * per_rank)))
    steps = 24
    stream = torch.cuda.Stream()
    dev = tsn.Device(local, stream=stream.cuda_stream)
    m = tsn.Dit(dev, synthetic=tsn.geom(**geom_kwargs(a)), seed=a.seed)
    m.prepare(a.T, a.C, a.TS, 2 * G)

    def inputs(gens):
        xs, cps, sgs, tps, gcs = [], [], [], [], []
        for g in gens:
            rng = np.random.default_rng(g)                     # per-generation seed (config 5: seeds 0..63)
            f = lambda *s: rng.standard_normal(s, dtype=np.float32)  # noqa: E731
            cps.append(f(a.C, a.H)); sgs.append(f(a.T, a.H)); tps.append(f(2, a.TS, a.H)); gcs.append(f(2, a.H))
            xs.append(f(a.T, 64))
        return (np.stack(cps), np.stack(sgs), np.concatenate(tps), np.concatenate(gcs), np.stack(xs))

    def run_batch(gens):
        cp, sg, tp, gc, x = inputs(gens + [gens[-1]] * (G - len(gens)))   # a short last batch repeats
        m.set_conditioning(cp, sg, tp, gc)
        m.set_x(x)
        m.schedule(steps, a.cfg)
        m.run_steps(steps)
        out = np.zeros((G, a.T, 64), np.float32)
        m.get_x(out)
        return out[:len(gens)]

    with torch.cuda.stream(stream):
        m.set_conditioning(*inputs(list(range(G)))[:4])
        m.set_x(inputs(list(range(G)))[4])
        if a.autotune:
            m.autotune()
        run_batch(list(range(G)))                               # warm-up
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        finals = [run_batch(mine[i:i + G]) for i in range(0, len(mine), G)]
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        x_all = np.concatenate(finals) if finals else np.zeros((0, a.T, 64), np.float32)
        times = torch.tensor([ms], dtype=torch.float64, device="cuda")
        if dist:
            dist.all_reduce(times, op=dist.ReduceOp.MAX)
            # the only cross-GPU traffic: the final latents to rank 0
            buf = torch.zeros(per_rank, a.T, 64, dtype=torch.float32, device="cuda")
            buf[:len(mine)] = torch.from_numpy(x_all).cuda()
            gathered = [torch.empty_like(buf) for _ in range(world)] if rank == 0 else None
            dist.gather(buf, gathered, dst=0)
        ms = float(times[0])
        finite = bool(np.isfinite(x_all).all())
        if rank == 0:
            gen_s = a.generations / (ms * 1e-3)
            print(json.dumps({
                "metric": "config 5: independent 8 s generations/s (24-step CFG-5 sampler), data-parallel",
                "value": gen_s, "unit": "generations/s", "n_gpus": world, "generations": a.generations,
                "gens_per_forward": G, "steps_per_generation": steps, "seconds": ms * 1e-3,
                "cfg_steps_per_s": gen_s * steps, "higher_is_better": True, "scaling": "strong",
                "data": "synthetic",
                "config": workload(a, f"config5: {a.generations} independent generations x {steps} CFG-{a.cfg:g} Euler "
                                      f"steps, {a.depth}-block MMDiT, 8 s audio geometry, final latents gathered"),
                "parallelism": f"dp{world}, {G} generation(s) per forward",
                "x_finite": finite}), flush=True)
    m.close()
    dev.close()
    if dist:
        dist.destroy_process_group()


def run_vae(a):
    """The VAE decode of one 8 s latent [T, 64] -> stereo audio [T * 2048, 2] (the step after the
    sampler, src/vae.cpp:17-86): device time of the decode graph, end-to-end time through
    tsn_vae_decode with host buffers, the split-weight GEMMs' algorithmic rate, and the reference's
    own decode (oracle/_ref over the scalar kernels) on a bounded sample of latent frames."""
    import time

    import numpy as np

    import tsn

    dev = tsn.Device(0)
    v = tsn.Vae(dev, channels=a.vae_channels, seed=a.seed)
    lat = np.random.default_rng(a.seed).standard_normal((a.T, 64)).astype(np.float32)
    for _ in range(max(a.warmup, 3)):
        v.decode(lat)
    dev_ms, wall = [], []
    for _ in range(a.steps):
        t0 = time.perf_counter()
        v.decode(lat)
        wall.append(time.perf_counter() - t0)
        dev_ms.append(v.last_ms())
    ms = max(dev_ms)
    flops = v.flops()
    _, peak, _, peak_src = peaks()
    line = {
        "metric": "VAE decodes/s of one 8 s latent (T=188 -> 385024 stereo samples)",
        "value": 1000.0 / ms, "unit": "decodes/s", "n_gpus": 1, "steps": a.steps, "warmup": max(a.warmup, 3),
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16 split activations x f16 split weights (f32 weights as hi+lo), f32 accumulate",
        "data": "synthetic",
        "config": {"workload": "VAE decoder (src/vae.cpp): conv k7 64->16C, 5 upsampling blocks (strides 8,8,4,4,2, "
                               "3 residual units each), snake, conv k7 C->2", "T": a.T, "channels": a.vae_channels,
                   "weights": "synthetic f32 (seed %d)" % a.seed},
        "roofline": {"bound": "tensor", "achieved": flops / (ms * 1e-3) / 1e12, "peak": peak, "unit": "TFLOP/s",
                     "frac": flops / (ms * 1e-3) / 1e12 / peak, "algorithmic_flops_per_step": flops,
                     "peak_source": f"{peak_src} bf16_tflops (burst)",
                     "note": "2·M·N·K over every conv; each K step issues three split products"},
        "e2e": {"value": 1.0 / max(wall), "unit": "decodes/s", "h2d_bytes_per_step": lat.nbytes,
                "d2h_bytes_per_step": a.T * 2048 * 2 * 4},
        "gpu_launches": v.launches() * a.steps,
    }
    if not a.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        if O.have_ref():
            frames = 2
            _, js = O.ref_vae(write_vae_fixture(a), lat[:frames])
            sec = min(js["seconds"]) * a.T / frames
            line["cpu_baseline"] = {"value": 1.0 / sec, "unit": "decodes/s", "cores": js["threads"], "kind": "reference",
                                    "sample": f"the reference's decode of {frames} latent frames, scaled to {a.T}"}
    print(json.dumps(line), flush=True)


def run_encoders(a):
    """The two text encoders at full size (T5 v1.1 XL: d_model 2048, d_ff 5120, 32 heads, Q8_0 file;
    MetaCLIP text: hidden 1024, 16 heads, f32 file; 24 layers each, 77 tokens): device time of each
    encode graph, end-to-end time through tsn_encoder_encode with host buffers, the weight-streaming
    rate against HBM, and the reference's own encodes (oracle/_ref over the scalar kernels). One
    JSON line per encoder."""
    import tempfile
    import time

    import numpy as np

    import tsn

    def t5_ids(seed, n):     # n ids, EOS (1), pad (0): the T5 tokenizer's layout
        ids = np.zeros(77, np.int32)
        ids[:n] = np.random.default_rng(seed).integers(2, 32000, n)
        ids[n] = 1
        return ids

    def clip_ids(seed, n):   # BOS, n ids, EOS padding: the CLIP tokenizer's layout
        ids = np.full(77, 49407, np.int32)
        ids[0] = 49406
        ids[1:1 + n] = np.random.default_rng(seed).integers(1, 49000, n)
        return ids

    hbm, _, _, peak_src = peaks()
    dev = tsn.Device(0)
    L = a.encoder_layers
    for kind in ("t5", "clip"):
        path = os.path.join(tempfile.gettempdir(), f"tsn_bench_{kind}_{L}_{a.seed}.gguf")
        if not os.path.exists(path):
            if kind == "t5":
                tsn.write_synthetic_t5_gguf(path, d_model=2048, d_ff=5120, layers=L, heads=32, seed=a.seed)
            else:
                tsn.write_synthetic_clip_gguf(path, hidden=1024, layers=L, heads=16, seed=a.seed)
        e = tsn.TextEncoder(dev, kind, path)
        ids = t5_ids(a.seed, 40) if kind == "t5" else clip_ids(a.seed, 30)
        for _ in range(max(a.warmup, 3)):
            e.encode(ids)
        dev_ms, wall = [], []
        for _ in range(a.steps):
            t0 = time.perf_counter()
            e.encode(ids)
            wall.append(time.perf_counter() - t0)
            dev_ms.append(e.last_ms())
        ms = max(dev_ms)
        wb = e.weight_bytes()
        if a.profile_ops:
            print(e.profile_ops(), file=sys.stderr, flush=True)
        line = {
            "metric": f"{kind} encodes/s (77 tokens)", "value": 1000.0 / ms, "unit": "encodes/s", "n_gpus": 1,
            "steps": a.steps, "warmup": max(a.warmup, 3), "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "f16 split activations x " + ("f16 weights (Q8_0 file)" if kind == "t5" else "f16 split weights (f32 file)")
                     + ", f32 accumulate",
            "data": "synthetic",
            "config": {"workload": "T5Model::encode (src/t5.cpp)" if kind == "t5" else "ClipModel::encode (src/clip.cpp)",
                       "width": e.width, "layers": e.layers, "tokens": e.ctx, "weights": "synthetic (seed %d)" % a.seed},
            "roofline": {"bound": "hbm", "achieved": wb / (ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": wb / (ms * 1e-3) / 1e9 / hbm, "traffic": None,
                         "algorithmic_bytes_per_step": wb, "peak_source": f"{peak_src} hbm_gbs",
                         "note": "weights streamed once per encode (2 B per f16 weight, 4 B per split f32 weight); "
                                 "77-row activations are negligible", "tflops": e.flops() / (ms * 1e-3) / 1e12},
            "e2e": {"value": 1.0 / max(wall), "unit": "encodes/s", "h2d_bytes_per_step": ids.nbytes,
                    "d2h_bytes_per_step": e.ctx * e.width * 4 + (e.width * 4 if kind == "clip" else 0)},
            "gpu_launches": e.launches() * a.steps,
        }
        if not a.no_cpu_baseline:
            sys.path.insert(0, os.path.join(ROOT, "oracle"))
            import oracle as O
            if O.have_ref():
                _, _, js = O.ref_encoder(kind, path, ids)
                sec = min(js["seconds"])
                line["cpu_baseline"] = {"value": 1.0 / sec, "unit": "encodes/s", "cores": js["threads"],
                                        "kind": "reference", "sample": "one full encode of the reference build"}
        e.close()
        print(json.dumps(line), flush=True)


def run_cpu_configs(a):
    """The CPU baselines of BASELINE.md's table, on this host's cores: config 1 (one full joint block,
    both CFG arms, T = 24, clip 8, text 77, H 1024, F 4096; the oracle port's joint block over a
    two-joint-block synthetic file, inputs N(0,1) from the seed) and config 2 (one full CFG step of
    the reference's host code, as the reference arm runs it); config 3 as 24 x config 2. One JSON line
    each."""
    import numpy as np

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    threads = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(threads)
    T, C, TS, H = 24, 8, 77, a.H
    with tempfile.TemporaryDirectory(prefix="tsn_cfg1_") as d:
        gguf = os.path.join(d, "two_joint.gguf")
        O.write_synthetic_gguf(gguf, H=H, NH=H // 64, F=a.F, depth=2, fused_depth=0, seed=a.seed)
        orc = O.Oracle(gguf)
        rng = np.random.default_rng(a.seed)
        f = lambda *sh: rng.standard_normal(sh, dtype=np.float32)  # noqa: E731
        lat, clip, text, extc, gc = f(T, H), f(C, H), f(2, TS, H), f(T, H), f(2, H)
        orc.joint_block(lat, clip, text[0], extc, gc[0])          # warm-up
        secs = []
        for _ in range(max(3, a.steps // 8)):
            t0 = time.perf_counter()
            for arm in (0, 1):
                orc.joint_block(lat, clip, text[arm], extc, gc[arm])
            secs.append(time.perf_counter() - t0)
        orc.close()
    c1 = min(secs)
    print(json.dumps({"metric": "config 1 (CPU): one MMDiT joint block, both CFG arms", "value": c1 * 1e3, "unit": "ms",
                      "higher_is_better": False, "cores": threads, "kind": "port", "reps": len(secs),
                      "config": {"T": T, "clip_S": C, "text_S": TS, "H": H, "F": a.F, "arms": 2},
                      "sample": "joint block 0 of the oracle port (scalar restatement of the reference kernels, "
                                "bit-exact to the reference build), f32, OpenMP over output rows"}), flush=True)
    step_secs, kind, sample = cpu_reference_steps(a, 2, threads)
    c2 = min(step_secs)
    print(json.dumps({"metric": "config 2 (CPU): one CFG step, 21 blocks, 8 s", "value": c2 * 1e3, "unit": "ms",
                      "higher_is_better": False, "cores": threads, "kind": kind, "reps": len(step_secs),
                      "config": workload(a), "sample": sample}), flush=True)
    print(json.dumps({"metric": "config 3 (CPU, extrapolated): 24-step CFG-5 denoise, 8 s", "value": 24 * c2,
                      "unit": "s", "higher_is_better": False, "cores": threads, "kind": kind,
                      "sample": "24 x the config 2 step time (extrapolated, not run)"}), flush=True)


def write_vae_fixture(a):
    import tempfile

    import tsn
    p = os.path.join(tempfile.gettempdir(), f"tsn_bench_vae_{a.vae_channels}_{a.seed}.gguf")
    if not os.path.exists(p):
        tsn.write_synthetic_vae_gguf(p, channels=a.vae_channels, seed=a.seed)
    return p


def main():
    a = parse()
    apply_long(a)
    if a.cpu_configs:
        run_cpu_configs(a)
    elif a.vae:
        run_vae(a)
    elif a.encoders:
        run_encoders(a)
    elif a.impl == "reference":
        run_reference(a)
    elif a.cfg_split:
        run_cfg_split(a)
    elif a.config5:
        run_config5(a)
    else:
        run_tsn(a)


if __name__ == "__main__":
    main()
