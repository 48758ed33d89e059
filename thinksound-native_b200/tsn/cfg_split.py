"""Two-rank CFG split of the sampler loop (src/pipeline.cpp:126-155).

The reference runs, per Euler step, the conditional and the unconditional forward one after the
other and then ``cfg_euler`` (shaders/ops_conv.metal:194-201). Here the two arms run on the two
ranks of a pair: the rank with pair rank ``arm`` (0 conditional, 1 unconditional) owns a model
prepared with ``arms = 1`` and that arm's conditioning. After every forward the pair all-gathers
the two flows ``[T, 64]`` f32 (47 KiB at 8 s) in arm order, and both ranks apply the same
``cfg_euler`` to their replica of x, so x stays bit-identical on the two ranks with no other
exchange.

:func:`loop` is the protocol with the three steps passed in; :class:`CfgSplitSampler` binds them
to the library (one ``Dit`` per rank) and to ``torch.distributed`` (NCCL all-gather on the stream
the library runs on). :meth:`CfgSplitSampler.sample_graph` runs the same protocol with one step
(this arm's forward, the all-gather, the update) captured in a CUDA graph and replayed, so a step
costs no host round trip.
"""
from __future__ import annotations

import numpy as np


def schedule(steps: int):
    """(t, dt) of every step in f32, as src/pipeline.cpp:142-145 computes them:
    t_s = 1 - s/steps and dt = t_{s+1} - t_s."""
    one, n = np.float32(1.0), np.float32(steps)
    out = []
    for s in range(steps):
        t = one - np.float32(s) / n
        t_next = one - np.float32(s + 1) / n
        out.append((t, np.float32(t_next - t)))
    return out


def loop(steps: int, cfg: float, x, forward, all_gather, euler):
    """Run the sampler with the arms split over a pair of ranks.

    forward(x, t) -> this rank's flow; all_gather(flow) -> (flow_cond, flow_uncond) in arm order;
    euler(flow_cond, flow_uncond, x, cfg, dt) -> updated x. Every rank of the pair calls the same
    collective once per step, in the same order."""
    for t, dt in schedule(steps):
        mine = forward(x, t)
        fc, fu = all_gather(mine)
        x = euler(fc, fu, x, cfg, dt)
    return x


class CfgSplitSampler:
    """The pair's sampler on GPUs: ``dit`` is prepared with ``arms = 1`` and holds this rank's arm
    conditioning; ``dev`` is the library device running on torch's current stream (so the NCCL
    all-gather is ordered with the library's launches); ``group`` is the pair's process group, in
    which pair rank 0 is the conditional arm."""

    def __init__(self, dit, dev, T: int, latent_dim: int = 64, group=None):
        import torch
        self.dit, self.dev, self.group = dit, dev, group
        self.n = T * latent_dim
        self.mine = torch.empty(T, latent_dim, dtype=torch.float32, device="cuda")
        self.flows = torch.empty(2, T, latent_dim, dtype=torch.float32, device="cuda")

    def forward(self, x, t):
        self.dit.set_x(x)
        self.dit.forward(float(t), self.mine)
        return self.mine

    def all_gather(self, mine):
        import torch.distributed as dist
        dist.all_gather_into_tensor(self.flows, mine, group=self.group)
        return self.flows[0], self.flows[1]

    def euler(self, fc, fu, x, cfg, dt):
        self.dev.cfg_euler(fc, fu, x, self.n, float(cfg), float(dt))
        return x

    def sample(self, x, steps: int, cfg: float):
        """x: this rank's replica of the latent [T, 64] f32 on the device, updated in place."""
        return loop(steps, cfg, x, self.forward, self.all_gather, self.euler)

    # ------------------------------------------------------------------ one CUDA graph per step
    def _one_step(self, cfg):
        import torch.distributed as dist
        self.dit.split_forward(self.mine)
        dist.all_gather_into_tensor(self.flows, self.mine, group=self.group)
        self.dit.split_update(self.flows, float(cfg))

    def graph_capture(self, x0, cfg: float):
        """Capture one sampler step in a CUDA graph: the library's stream-ordered split calls
        (tsn_dit_split_forward / tsn_dit_split_update) and the NCCL all-gather, on the library's
        stream (torch's current stream, which must not be the default stream). One eager step runs
        first (it loads the kernels and warms the communicator). x0: device [T, 64]."""
        import torch
        self.dit.set_x(x0)
        self.dit.split_schedule(1)
        self._one_step(cfg)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=torch.cuda.current_stream()):
            self._one_step(cfg)

    def graph_run(self, x0, steps: int):
        """The sampler from x0 over `steps` steps, each replayed from the captured graph (no host
        round trip per step); x stays on the device (read it with the model's get_x)."""
        self.dit.set_x(x0)
        self.dit.split_schedule(steps)
        for _ in range(steps):
            self.graph.replay()

    def graph_release(self):
        """Release the graph (it holds NCCL work: release it before destroying the process group)."""
        import torch
        torch.cuda.synchronize()
        self.graph = None

    def sample_graph(self, x, steps: int, cfg: float):
        """:meth:`sample` with each step replayed from one CUDA graph; x (device [T, 64]) is the start
        latent and receives the result."""
        x0 = x.clone()
        self.graph_capture(x0, cfg)
        try:
            self.graph_run(x0, steps)
            self.dit.get_x(x)
        finally:
            self.graph_release()
        return x
