"""CFG split over a pair of ranks (one CFG arm per rank, flows all-gathered every step).

The CPU test runs the pair as two gloo processes with the oracle as each rank's forward and checks
that both ranks end with the same x as the single-process reference step loop, bit for bit. The
GPU test runs the same protocol on two GPUs over NCCL (it needs two visible devices), once step by
step from the host and once with every step replayed from one captured CUDA graph (forward, NCCL
all-gather, update), which must give the same bits."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import SEED, TINY, TINY_SEQ, make_inputs, rel_l2

import tsn
from tsn import cfg_split

STEPS, CFG = 3, 5.0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _euler_ref(fc, fu, x, cfg, dt):
    """cfg_euler (shaders/ops_conv.metal:194-201) in f32, as the oracle computes it."""
    v = fu + (fc - fu) * np.float32(cfg)
    return (x + np.float32(dt) * v).astype(np.float32)


def _cpu_rank(rank, port, gguf, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), OMP_NUM_THREADS="2")
    import torch.distributed as dist
    import oracle as O
    dist.init_process_group("gloo", rank=rank, world_size=2)
    try:
        T, C, TS = TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"]
        inp = make_inputs(T, C, TS, TINY["H"], seed=SEED + 7)
        sfx = "cond" if rank == 0 else "unc"
        orc = O.Oracle(gguf)

        def forward(x, t):
            return orc.forward(T, C, TS, x, float(t), inp["clip_pp"], inp["sync_gather"], inp[f"text_pp_{sfx}"],
                               inp[f"gcmlp_{sfx}"]).reshape(T, 64)

        def all_gather(mine):
            parts = [torch.empty(T, 64) for _ in range(2)]
            dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(mine)))
            return parts[0].numpy(), parts[1].numpy()

        x = cfg_split.loop(STEPS, CFG, inp["x"].copy(), forward, all_gather, _euler_ref)
        np.save(os.path.join(out_dir, f"x{rank}.npy"), x)
    finally:
        dist.destroy_process_group()


def test_cfg_split_pair_matches_reference_loop(tiny_gguf, tmp_path):
    import oracle as O
    port = _free_port()
    mp.start_processes(_cpu_rank, args=(port, tiny_gguf, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    x0, x1 = np.load(tmp_path / "x0.npy"), np.load(tmp_path / "x1.npy")
    assert np.array_equal(x0, x1), "the two ranks' replicas of x diverged"
    # single process: the reference step (both arms + cfg_euler) with the same schedule
    T, C, TS = TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"]
    inp = make_inputs(T, C, TS, TINY["H"], seed=SEED + 7)
    orc = O.Oracle(tiny_gguf)
    x = inp["x"].copy()
    for t, dt in cfg_split.schedule(STEPS):
        x, _, _ = orc.step(T, C, TS, x, float(t), CFG, float(dt), inp["clip_pp"], inp["sync_gather"],
                           inp["text_pp_cond"], inp["gcmlp_cond"], inp["text_pp_unc"], inp["gcmlp_unc"])
    assert np.array_equal(x0, x)


def test_schedule_is_the_reference_f32_schedule():
    """t_s = 1 - s/steps and dt = t_{s+1} - t_s, each operation rounded to f32 (src/pipeline.cpp:142-145)."""
    for steps in (1, 4, 24, 50):
        sch = cfg_split.schedule(steps)
        assert len(sch) == steps
        for s, (t, dt) in enumerate(sch):
            t_ref = np.float32(np.float32(1.0) - np.float32(np.float32(s) / np.float32(steps)))
            t_nx = np.float32(np.float32(1.0) - np.float32(np.float32(s + 1) / np.float32(steps)))
            assert t == t_ref and dt == np.float32(t_nx - t_ref)
        assert sch[0][0] == np.float32(1.0)


class _RankFailed(RuntimeError):
    pass


def _failing_rank(rank, port, out_dir, fail_step):
    """One rank of the pair; pair rank 1 fails in its forward of `fail_step` (a host exception, as a
    failed library call would raise), leaves the loop and the group without joining that step's
    all-gather, and exits 0. Pair rank 0 must see its all-gather end with an error (the peer closed
    the group, or the group's 5 s timeout) instead of waiting for good."""
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=5))
    calls = [0]

    def forward(x, t):
        if rank == 1 and calls[0] == fail_step:
            raise _RankFailed(f"rank 1 forward failed at step {calls[0]}")
        calls[0] += 1
        return (x * np.float32(0.5 + 0.25 * rank)).astype(np.float32)

    def all_gather(mine):
        parts = [torch.empty(mine.shape) for _ in range(2)]
        dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(mine)))
        return parts[0].numpy(), parts[1].numpy()

    t0 = time.monotonic()
    outcome = "finished"
    try:
        cfg_split.loop(4, CFG, np.ones((8, 64), np.float32), forward, all_gather, _euler_ref)
    except _RankFailed:
        outcome = "failed"
    except RuntimeError:
        outcome = "peer_lost"
    finally:
        try:
            dist.destroy_process_group()
        except RuntimeError:
            pass
    with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
        f.write(f"{outcome} {calls[0]} {time.monotonic() - t0:.3f}")


def test_cfg_split_rank_failure_ends_the_peer_collective(tmp_path):
    """A rank that fails between steps (its forward raises before the step's all-gather) leaves the
    pair; the other rank's next all-gather returns an error within the group's timeout, after the
    steps both ranks completed. Host-only (gloo), no GPU."""
    fail_step = 2
    mp.start_processes(_failing_rank, args=(_free_port(), str(tmp_path), fail_step), nprocs=2, join=True,
                       start_method="spawn")
    o0, n0, s0 = (tmp_path / "r0.txt").read_text().split()
    o1, n1, _ = (tmp_path / "r1.txt").read_text().split()
    assert (o1, int(n1)) == ("failed", fail_step)
    assert o0 == "peer_lost", "the surviving rank's collective did not end with an error"
    assert int(n0) == fail_step + 1     # it ran its own forward of the failed step, then lost the peer
    assert float(s0) < 60.0


def _gpu_rank(rank, port, gguf, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        st = torch.cuda.Stream()
        with torch.cuda.stream(st):
            dev = tsn.Device(rank, stream=st.cuda_stream)
            T, C, TS = TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"]
            inp = make_inputs(T, C, TS, TINY["H"], seed=SEED + 7)
            sfx = "cond" if rank == 0 else "unc"
            m = tsn.Dit(dev, gguf=gguf)
            m.prepare(T, C, TS, 1)
            m.set_conditioning(inp["clip_pp"], inp["sync_gather"], inp[f"text_pp_{sfx}"], inp[f"gcmlp_{sfx}"])
            x = torch.from_numpy(inp["x"]).cuda()
            xg = x.clone()
            sampler = cfg_split.CfgSplitSampler(m, dev, T)
            sampler.sample(x, STEPS, CFG)
            torch.cuda.synchronize()
            np.save(os.path.join(out_dir, f"g{rank}.npy"), x.cpu().numpy())
            sampler.sample_graph(xg, STEPS, CFG)          # every step replayed from one CUDA graph
            torch.cuda.synchronize()
            np.save(os.path.join(out_dir, f"gg{rank}.npy"), xg.cpu().numpy())
            m.close()
            dev.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_cfg_split_two_gpus(tiny_gguf, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import oracle as O
    port = _free_port()
    mp.start_processes(_gpu_rank, args=(port, tiny_gguf, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    x0, x1 = np.load(tmp_path / "g0.npy"), np.load(tmp_path / "g1.npy")
    assert np.array_equal(x0, x1), "the two GPUs' replicas of x diverged"
    # the graph-replayed sampler issues the same kernels in the same order: the same bits
    assert np.array_equal(np.load(tmp_path / "gg0.npy"), x0) and np.array_equal(np.load(tmp_path / "gg1.npy"), x0)
    T, C, TS = TINY_SEQ["T"], TINY_SEQ["C"], TINY_SEQ["TS"]
    inp = make_inputs(T, C, TS, TINY["H"], seed=SEED + 7)
    orc = O.Oracle(tiny_gguf)
    x = inp["x"].copy()
    for t, dt in cfg_split.schedule(STEPS):
        x, _, _ = orc.step(T, C, TS, x, float(t), CFG, float(dt), inp["clip_pp"], inp["sync_gather"],
                           inp["text_pp_cond"], inp["gcmlp_cond"], inp["text_pp_unc"], inp["gcmlp_unc"])
    # the update dt*(fu + 5(fc - fu)) summed over the steps: x carries the unchanged noise
    assert rel_l2(x0 - inp["x"], x - inp["x"]) < 5e-3
