"""Benchmark of the SCOPE sparse-attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c3] [--impl ours|reference|flex]

One step = one layer of configuration C3 (B=1, H=16, T=131072, D=64, bf16,
block 128, K=16 spectral frequencies, sliding 8 / local 2 / half 4 / global
1 / budget 8 pointer blocks): the fused pointer selection + mask build, the
attention forward with the spectral bias (qk_aug, the reference default) and
the backward for q, k, v and the spectral coefficients.  Heads are sharded
across the N ranks; the outputs and pointer statistics are all-gathered over
NCCL (the path's only collective).  Metric: active-block attention TFLOP/s
fwd+bwd = 14 * bs^2 * D * sum(kv_num_blocks) / step time, whole job.

The same line carries:
  * ``gpu_reference``: the reference's GPU path on this GPU, same layer and
    inputs -- torch.compile(flex_attention) (Inductor Triton) fwd + bwd with
    the reference's BlockMask.from_kv_blocks and qk_aug tensor ops (run as
    ``--impl flex`` in a child process, N = 1);
  * ``decoder``: configuration C4, the 24-layer SCOPE decoder trained
    data-parallel over the N ranks (tokens/s per GPU, the metric's second half);
  * ``roofline``, ``phases_ms``, ``cpu_baseline``, ``e2e``, ``clocks``,
    ``coeff_block`` (the SpectralBias coefficient block kernel).

--impl reference times the reference's CPU path on the host cores (the
numpy port of its mask builder + torch's compiled CPU flex_attention, forward
only: the reference has no CPU backward).  --impl flex prints the
gpu_reference measurement on its own; it is not the driver's reference arm.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from scope_b200 import PointerBlockMaskBuilder, SpectralScoreMod, flex_attention, trig_tables  # noqa: E402
from scope_b200 import _lib, shard  # noqa: E402
from scope_b200.synth import BETA, CONFIGS, SCALE, make_inputs  # noqa: E402

METRIC = "active-block attn TFLOP/s fwd+bwd at T=128k; tokens/s/GPU at 1/2/4/8 B200"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """SM clock and throttle reasons sampled every 10 ms (NVML) during the
    timed region."""
    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4}

    def __init__(self, index: int, period: float = 0.01):
        self.index, self.period, self.rows = index, period, []
        self._stop = threading.Event()
        self.nvml = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            # the physical GPU behind this process's device `index`, by PCI address
            pr = torch.cuda.get_device_properties(self.index)
            bus = "%08X:%02X:%02X.0" % (int(pr.pci_domain_id), int(pr.pci_bus_id), int(pr.pci_device_id))
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            self.nvml, self.h = pynvml, h
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
        except Exception:
            self.nvml = None
        return self

    def _poll(self):
        nv, h = self.nvml, self.h
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.rows.append((sm, rs))
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *a):
        self._stop.set()
        if self.nvml:
            self.t.join(timeout=2)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        reasons = sorted({n for _, rs in self.rows for n, b in self.REASONS.items() if rs & b})
        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.rows), "source": "NVML, 10 ms"}


def setup_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


class Workload:
    """The per-rank inputs of one C3 layer (this rank's head shard)."""

    def __init__(self, cfg, rank, world, device, seed=0):
        self.heads = shard.head_slice(cfg.H, rank, world)
        hp = cfg.H // world
        self.cfg, self.rank, self.world, self.hp = cfg, rank, world, hp
        x = make_inputs(cfg, device=device, seed=seed, heads=self.heads)
        self.x = x
        self.cos_t, self.sin_t = trig_tables(x["omegas"], cfg.T)
        self.builder = PointerBlockMaskBuilder(
            num_heads=hp, M=cfg.M, pointer_local_blocks=cfg.local_eff, pointer_half_blocks=cfg.half_blocks,
            pointer_global_blocks=cfg.global_blocks, pointer_budget_blocks=cfg.budget_blocks,
            pointer_budget_is_total=cfg.budget_is_total, pointer_budget_temp=cfg.budget_temp, debug_stats=True)
        self.leaves = {n: x[n].detach().requires_grad_(True) for n in ("q", "k", "v", "coeff_cos", "coeff_sin")}
        self.gather_out = self.stats_out = None    # all-gather receive buffers (N > 1)

    def build(self):
        x = self.x
        return self.builder.select_and_build(pointer_logits=x["logits"], gumbel=x["gumbel"], tau=self.cfg.select_tau,
                                             docs=x["docs"], budget_rep=x["budget_rep"],
                                             block_size=self.cfg.block_size)

    def step(self):
        """mask build -> forward -> (async all-gathers of the output heads and of the
        pointer statistics) -> backward"""
        L = self.leaves
        for t in L.values():
            t.grad = None
        bm = self.build()
        sm = SpectralScoreMod(coeff_cos=L["coeff_cos"], coeff_sin=L["coeff_sin"], cos_tab=self.cos_t,
                              sin_tab=self.sin_t, beta=BETA, impl="qk_aug")
        out = flex_attention(L["q"][None], L["k"][None], L["v"][None], bm, score_mod=sm, scale=SCALE,
                             head_major_out=self.world > 1)
        works = []
        if self.world > 1:
            # out[0] is this rank's [H/N, T, D] head-major slice: the gather lands it in the
            # [H, T, D] output without a copy or permute
            if self.gather_out is None:
                self.gather_out = shard.gather_buffer(self.cfg.T, self.cfg.H, self.cfg.D, self.world,
                                                      out.dtype, out.device)
                self.stats_out = shard.stats_buffer(bm.stats, self.world)
            works.append(shard.gather_heads(out[0].detach(), self.gather_out, async_op=True)[1])
            works.append(shard.gather_stats(bm.stats, self.stats_out, async_op=True)[1])
        out.backward(self.x["do"][None])
        for w in works:
            w.wait()
        return bm, out


def capture_step(wl, world):
    """The step captured in a CUDA graph (kernels, memsets and, at N > 1, the
    NCCL all-gathers), after warm-up steps on a side stream; replaying it
    costs the host ~10 us instead of the Python launch path of the mask
    builder, the custom ops and autograd.  Every rank captures or none does
    (a rank that fails reports it and all ranks run the step eagerly).
    Returns (graph or None, launches per step, reason)."""
    L = _lib.lib()
    torch.cuda.synchronize()
    n0 = L.scope_launch_count()
    wl.step()
    torch.cuda.synchronize()
    per_step = L.scope_launch_count() - n0
    graph, why = None, ""
    try:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                wl.step()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            wl.step()
        torch.cuda.synchronize()
        graph = g
    except Exception as e:  # the eager step is measured instead
        why = f"{type(e).__name__}: {e}"[:200]
    ok = torch.tensor([1 if graph is not None else 0], device="cuda", dtype=torch.int32)
    if world > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if int(ok.item()) == 0:
        graph = None
        why = why or "another rank could not capture the step"
    return graph, per_step, why


def active_pairs(bm):
    return int(bm.kv_num_blocks.sum().item())


def time_steps(fn, steps, world):
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(steps):
        fn()
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
        dist.barrier()
    return ms


# DRAM bytes (read + write) of one launch of each phase's dominant kernel, from
# single ncu --set full captures of this build (cold L2, as ncu replays), and
# the units that launch processed.  Refresh them with a new capture when a
# kernel changes.
NCU_TRAFFIC = {
    "builder": {"bytes": 71.20e6 + 1.82e6, "units": 16,
                "capture": "ncu build_kernel, C3 (16 heads, 1024 q blocks each)"},
    "forward": {"bytes": 349.86e6 + 55.44e6, "units": 59741,
                "capture": "ncu fwd_kernel<32,0>, C3 with 4 of 16 heads (59,741 active pairs)"},
    "backward": {"bytes": 1023.21e6 + 486.42e6, "units": 59741,
                 "capture": "ncu dkvq_kernel<32,0,0> (prep, plan and finish kernels not included), "
                            "C3 with 4 of 16 heads (59,741 active pairs)"},
}


def gpu_hold(ms=30.0):
    """Keep the current stream busy for about `ms` (a device-side sleep), so
    that the host enqueues the work that follows before the GPU reaches it:
    events recorded after the hold then time device work, not host launch
    gaps."""
    torch.cuda._sleep(int(ms * 1e-3 * 2.0e9))


def phase_times(wl, reps=5):
    """Median device time of each phase of the step, with CUDA events on the
    stream the kernels are launched on (the current stream); each repetition
    is queued behind a device-side hold, so host launch overhead is not
    counted.  One untimed repetition goes first (the caching allocator may
    grow, and synchronise, on the first eager step after a graph capture), and
    the median drops a repetition the host still fell behind on."""
    s = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    samples = [[], [], []]
    L = wl.leaves
    for rep in range(reps + 1):
        for t in L.values():
            t.grad = None
        gpu_hold()
        ev[0].record(s)
        bm = wl.build()
        ev[1].record(s)
        sm = SpectralScoreMod(coeff_cos=L["coeff_cos"], coeff_sin=L["coeff_sin"], cos_tab=wl.cos_t,
                              sin_tab=wl.sin_t, beta=BETA, impl="qk_aug")
        out = flex_attention(L["q"][None], L["k"][None], L["v"][None], bm, score_mod=sm, scale=SCALE)
        ev[2].record(s)
        out.backward(wl.x["do"][None])
        ev[3].record(s)
        torch.cuda.synchronize()
        if rep > 0:
            for i in range(3):
                samples[i].append(ev[i].elapsed_time(ev[i + 1]))
    return [statistics.median(x) for x in samples]


class E2EPipeline:
    """The step through the public API from pinned host buffers, every step:
    H2D of all of its inputs, the step, D2H of its output and gradients.
    Copies run on their own streams so that the inputs of step i+1 travel
    while step i computes and the results of step i travel back while step
    i+1 computes (PCIe carries H2D and D2H at the same time); the device
    inputs are double buffered."""

    IN = ("q", "k", "v", "do", "coeff_cos", "coeff_sin", "logits", "gumbel", "budget_rep")

    def __init__(self, wl, host):
        self.wl, self.host = wl, host
        self.dev = [{n: wl.x[n].detach().clone() for n in self.IN} for _ in range(2)]
        self.s_h2d, self.s_d2h = torch.cuda.Stream(), torch.cuda.Stream()
        self.free = [None, None]        # compute done with a slot's inputs
        self.i = 0

    def start(self, ev0):
        self.s_h2d.wait_event(ev0)

    def step(self):
        k = self.i % 2
        cur = torch.cuda.current_stream()
        dev = self.dev[k]
        if self.free[k] is not None:
            self.s_h2d.wait_event(self.free[k])
        with torch.cuda.stream(self.s_h2d):
            for n, h in self.host["in"].items():
                dev[n].copy_(h, non_blocking=True)
        cur.wait_stream(self.s_h2d)
        wl, L = self.wl, self.wl.leaves
        for n in ("q", "k", "v", "coeff_cos", "coeff_sin"):
            L[n].data = dev[n]
        wl.x["do"] = dev["do"]
        wl.x["logits"], wl.x["gumbel"], wl.x["budget_rep"] = dev["logits"], dev["gumbel"], dev["budget_rep"]
        bm, out = wl.step()
        self.free[k] = cur.record_event()
        self.s_d2h.wait_stream(cur)
        res = [("out", out[0].detach())] + [("d" + n, L[n].grad) for n in ("q", "k", "v", "coeff_cos", "coeff_sin")]
        with torch.cuda.stream(self.s_d2h):
            for n, t in res:
                t.record_stream(self.s_d2h)
                self.host["out"][n].copy_(t, non_blocking=True)
        self.i += 1

    def finish(self):
        cur = torch.cuda.current_stream()
        cur.wait_stream(self.s_h2d)
        cur.wait_stream(self.s_d2h)


def time_e2e(pipe, steps, world):
    """Device time of `steps` pipelined end-to-end steps: from an event before
    the first H2D to one after the last D2H, max over ranks."""
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    pipe.start(e0)
    for _ in range(steps):
        pipe.step()
    pipe.finish()
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
        dist.barrier()
    return ms


def score_mod_leg(wl, cfg, bm, pairs, *, reps=5):
    """The layer with the score_mod closure (scoped_medium.py:425-457) instead of
    qk_aug: Fourier sum in the QK MMA, b0, slope * Δ and the softplus gate
    per element, their gradients from per-query column sums.  Same mask and
    inputs as the step; fwd and bwd each timed with CUDA events after a
    device-side hold (TFLOP/s on active block pairs, as the headline)."""
    from scope_b200 import SpectralScoreMod, flex_attention
    hp, T, D, bs = wl.hp, cfg.T, cfg.D, 128
    g = torch.Generator(device="cuda").manual_seed(17)
    dev = wl.x["q"].device
    extra = {"b0": 0.1 * torch.randn(hp, T, generator=g, device=dev),
             "slope": 0.01 * torch.tanh(torch.randn(hp, T, generator=g, device=dev)),
             "delta_main": torch.rand(hp, T, generator=g, device=dev) * 4096.0,
             "width": 32.0 + torch.rand(hp, T, generator=g, device=dev) * 224.0}
    L = wl.leaves
    lv = {n: t.detach().requires_grad_(True) for n, t in extra.items()}
    s = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    fw, bw = [], []
    for rep in range(reps + 2):
        for t in list(L.values()) + list(lv.values()):
            t.grad = None
        sm = SpectralScoreMod(coeff_cos=L["coeff_cos"], coeff_sin=L["coeff_sin"], cos_tab=wl.cos_t,
                              sin_tab=wl.sin_t, beta=BETA, b0=lv["b0"], slope=lv["slope"],
                              delta_main=lv["delta_main"], width=lv["width"], gate="softplus", impl="score_mod")
        gpu_hold()
        ev[0].record(s)
        out = flex_attention(L["q"][None], L["k"][None], L["v"][None], bm, score_mod=sm, scale=SCALE)
        ev[1].record(s)
        out.backward(wl.x["do"][None])
        ev[2].record(s)
        torch.cuda.synchronize()
        if rep >= 2:
            fw.append(ev[0].elapsed_time(ev[1]))
            bw.append(ev[1].elapsed_time(ev[2]))
    f_ms, b_ms = statistics.median(fw), statistics.median(bw)
    fl = 14 * bs * bs * D * pairs
    return {"workload": f"{cfg.name} layer, score_mod closure (K={cfg.K}, b0, slope, softplus gate)",
            "forward_ms": f_ms, "backward_ms": b_ms, "tflops": fl / ((f_ms + b_ms) * 1e-3) / 1e12,
            "forward_tflops": 4 * bs * bs * D * pairs / (f_ms * 1e-3) / 1e12,
            "backward_tflops": 10 * bs * bs * D * pairs / (b_ms * 1e-3) / 1e12}


def torch_teacher_mass(q_sel, k_sel, q_pos, k_pos, docs, scale):
    """The reference teacher's dense block-mass loop (scoped_medium.py:1793-1819)
    as the same eager torch ops on the GPU: per query block, bf16 scores
    against every key, the document-causal mask, softmax, column sums
    scattered into kv blocks."""
    H, L, _ = q_sel.shape
    dev = q_sel.device
    bs = 128
    nb = L // bs
    k_idx = torch.arange(L, device=dev)
    k_blocks = torch.floor_divide(k_idx, bs)
    mass_all = torch.zeros(H, nb, nb, device=dev)
    for qb in range(nb):
        qs, qe = qb * bs, (qb + 1) * bs
        scores = torch.matmul(q_sel[:, qs:qe], k_sel.transpose(-2, -1)) * scale
        scores = scores + torch.matmul(q_pos[:, qs:qe], k_pos.transpose(-2, -1)) * scale
        q_idx = torch.arange(qs, qe, device=dev)
        mask = (docs[qs:qe][:, None] == docs[None, :]) & (q_idx[:, None] >= k_idx[None, :])
        w = torch.softmax(scores.float().masked_fill(~mask, -1.0e9), dim=-1)
        m = torch.zeros(H, nb, device=dev)
        m.scatter_add_(1, k_blocks[None].expand(H, -1), w.sum(dim=1))
        mass_all[:, qb] = m
    return mass_all


def teacher_leg(cfg, heads, *, L=4096, reps=5):
    """The spectral teacher's block mass (scoped_medium.py:1793-1819) at the
    reference's default teacher length (4096 tokens) on this rank's heads, K
    of the config with the slope column: this package's kernel
    (teacher_block_mass) against the reference's loop as eager torch ops on
    the same GPU, each timed with CUDA events (median of `reps`)."""
    from scope_b200 import teacher_block_mass
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(29)
    K = cfg.K
    q = torch.randn(heads, L, 64, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(heads, L, 64, generator=g, device=dev).to(torch.bfloat16)
    s_aug = math.sqrt(BETA / SCALE)
    cc = 0.3 * torch.randn(heads, L, K, generator=g, device=dev)
    cs = 0.3 * torch.randn(heads, L, K, generator=g, device=dev)
    ph = torch.tensor([math.pi * 2.0 ** (-i) for i in range(K)], device=dev)[:, None] * torch.arange(L, device=dev)
    ct = torch.cos(ph).to(torch.bfloat16).float().T[None].expand(heads, L, K)
    st = torch.sin(ph).to(torch.bfloat16).float().T[None].expand(heads, L, K)
    slope = 0.01 * torch.tanh(torch.randn(heads, L, generator=g, device=dev))
    pos = torch.arange(L, device=dev, dtype=torch.float32)[None, :, None].expand(heads, L, 1)
    q_pos = (torch.cat([cc * ct + cs * st, cc * st - cs * ct, -slope[..., None]], -1) * s_aug).to(torch.bfloat16)
    k_pos = (torch.cat([ct, st, pos], -1) * s_aug).to(torch.bfloat16)
    cuts = torch.zeros(L, dtype=torch.int64, device=dev)
    cuts[[700, 1500, 2600]] = 1
    docs = cuts.cumsum(0)
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn):
        for _ in range(2):
            fn()
        ts = []
        for _ in range(reps):
            torch.cuda.synchronize()
            e0.record(s)
            fn()
            e1.record(s)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    ours = timed(lambda: teacher_block_mass(q, k, docs, scale=SCALE, q_pos=q_pos, k_pos=k_pos))
    ref = timed(lambda: torch_teacher_mass(q, k, q_pos, k_pos, docs, SCALE))
    diff = (teacher_block_mass(q, k, docs, scale=SCALE, q_pos=q_pos, k_pos=k_pos) -
            torch_teacher_mass(q, k, q_pos, k_pos, docs, SCALE)).abs().max().item()
    return {"workload": f"teacher block mass, {heads} heads x {L} tokens, K={K} + slope, 4 documents",
            "ours_ms": ours, "reference_torch_ms": ref, "ours_over_reference": ref / ours,
            "max_abs_diff_vs_reference_ops": diff,
            "note": "reference = scoped_medium.py:1793-1819 as eager torch ops on this GPU (bf16 matmuls round "
                    "the scores to bf16; the kernel keeps them in float32)"}


def coeff_block(wl, cfg, hbm, *, reps=10, cpu=True):
    """The SpectralBias coefficient block (model/attn_bias.py:306-324, 419-478)
    on this rank's heads at the bench's T, M = 8 pointers, K of the config:
    the fused kernel (scope_spectral_coeffs) timed with CUDA events over `reps`
    calls (q, 2^17 tokens x 16 heads of bf16, is larger than L2), its HBM
    roofline (q read once, every output written once), and on the host the
    oracle's restatement of the reference's CPU computation on a bounded
    sample (one head, 8192 tokens)."""
    from scope_b200 import SpectralCoefficients, spectral_coefficients
    from scope_b200.coeff import OUT_NAMES
    H, T, K, M = wl.hp, cfg.T, cfg.K, 8
    n_out = 5 * M + 1
    sc = SpectralCoefficients(head_dim=64, num_heads=H, L_train=T, K=K, M=M, seed=7)
    g = torch.Generator().manual_seed(8)
    sc.load_weights(sc.w1[0], torch.randn(128, generator=g) * 0.1, torch.randn(n_out, 128, generator=g) * 0.08,
                    sc.b2[0] + torch.randn(n_out, generator=g) * 0.5)
    q = wl.x["q"].detach()
    kw = dict(omegas=sc.omegas, log_omegas=sc.log_omegas, M=M, delta_cap=float(min(sc.delta_star_max, T - 1)),
              logw_min=sc.logw_min, logw_max=sc.logw_max)
    w = [t[0].to(device=q.device, dtype=torch.bfloat16) for t in (sc.w1, sc.b1, sc.w2, sc.b2)]
    outs = [spectral_coefficients(q, *w, **kw) for _ in range(3)]
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gpu_hold()
    e0.record(s)
    for _ in range(reps):
        spectral_coefficients(q, *w, **kw)
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    tok = H * T
    byts = tok * (64 * 2 + (2 * K + 3 * M + 4) * 4)
    res = {"kernel": "scope_spectral_coeffs", "workload": f"{H} heads x T={T}, K={K}, M={M}, shared MLP 64-128-{n_out}",
           "ms": ms, "tokens_per_s": tok / (ms * 1e-3),
           "roofline": {"bound": "hbm", "achieved": byts / (ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                        "frac": byts / (ms * 1e-3) / 1e9 / hbm, "algorithmic_bytes": byts},
           "mlp_tflops": 2 * tok * (64 * 128 + 128 * n_out) / (ms * 1e-3) / 1e12}
    # backward: dL/dy kernel + the MLP replay (library GEMMs), from unit upstream gradients
    # of the coefficients and the slope, with q and the weights requiring grad
    from scope_b200.coeff import coeff_dy
    qg = q.detach().requires_grad_(True)
    wg = [t.detach().float().requires_grad_(True) for t in w]
    ups = None
    for i in range(3 + reps):
        if i == 3:
            torch.cuda.synchronize()
            gpu_hold()
            e0.record(s)
        qg.grad = None                       # a training step starts from cleared gradients
        for t in wg:
            t.grad = None
        o = spectral_coefficients(qg, *wg, **kw)
        if ups is None:
            ups = [torch.ones_like(o.coeff_cos), torch.ones_like(o.coeff_sin), torch.ones_like(o.slope)]
        torch.autograd.backward([o.coeff_cos, o.coeff_sin, o.slope], ups)
    e1.record(s)
    torch.cuda.synchronize()
    res["fwd_bwd_ms"] = e0.elapsed_time(e1) / reps
    yb = o.mlp_out if o.mlp_out is not None else spectral_coefficients(q, *w, **kw, return_mlp=True).mlp_out
    torch.cuda.synchronize()
    gpu_hold()
    e0.record(s)
    for _ in range(reps):
        coeff_dy(yb, [ups[0], ups[1], ups[2]] + [None] * 6, **kw, use_slope=True, subtract_b0=True, c_scale=sc.c_scale,
                 width_min=sc.width_min, width_max=sc.width_max, eps=sc.eps)
    e1.record(s)
    torch.cuda.synchronize()
    res["dy_kernel_ms"] = e0.elapsed_time(e1) / reps
    del outs
    if cpu:
        from oracle import coeff_oracle as CO   # the CPU baseline only
        n = 8192
        qc = q[:1, :n].cpu()[None]
        wc = [t[0] for t in (sc.w1, sc.b1, sc.w2, sc.b2)]
        t0 = time.perf_counter()
        y = CO.mlp(qc, *[t.to(torch.bfloat16) for t in wc])
        CO.heads(y.float(), M=M, omegas=sc.omegas.cpu(), log_omegas=sc.log_omegas.cpu(),
                 delta_cap=kw["delta_cap"], logw_min=sc.logw_min, logw_max=sc.logw_max, use_slope=True,
                 subtract_b0=True, c_scale=sc.c_scale, width_min=sc.width_min, width_max=sc.width_max, eps=sc.eps)
        dt = time.perf_counter() - t0
        res["cpu_baseline"] = {"value": n / dt, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
                               "sample": f"1 head x {n} tokens: the oracle's torch-CPU restatement of the reference's "
                                         "MLP and mixture"}
    return res


def decoder_bench(rank, world, *, steps=4, warmup=2, T=65536):
    """Configuration C4: the 24-layer SCOPE decoder (scope_b200.decoder) trained
    data-parallel, one sequence of T uniform token ids per rank (shifted
    targets), forward + backward + bucketed gradient all-reduce + AdamW step.
    Returns tokens/s per GPU (the metric's second half) and the model FLOP rate
    (6 x matmul parameters per token plus 14 bs^2 D per active block pair)."""
    from scope_b200.decoder import BucketedAllReduce, ScopeDecoder, synthetic_tokens
    torch.manual_seed(0)
    model = ScopeDecoder(max_seq_len=T).cuda()
    opt = torch.optim.AdamW(model.parameters(), lr=1e-4, betas=(0.9, 0.95), fused=True)
    dp = BucketedAllReduce(model.parameters()) if world > 1 else None
    inp, tgt = synthetic_tokens(T, seed=1000 + rank, device="cuda")

    def step():
        if dp is not None:
            dp.zero_grad()
        else:
            opt.zero_grad(set_to_none=False)
        model(inp, tgt).backward()
        if dp is not None:
            dp.wait()
        opt.step()

    for _ in range(warmup):
        step()
    ms = time_steps(step, steps, world) / steps
    pairs = model.attention_pairs()
    flops = model.flops_per_token() * T + 14 * 128 * 128 * 64 * pairs
    res = {"workload": "c4: 24 layers, d_model 1024, 16 heads x 64, MLP 4x, vocab 50304, T=65536 per GPU, "
                       "SCOPE attention (K=8, pointer mask: local 8, 4 pointer blocks) on every layer",
           "tokens_per_s_per_gpu": T / (ms * 1e-3), "tokens_per_s": world * T / (ms * 1e-3), "ms_per_step": ms,
           "steps": steps, "warmup": warmup, "parallelism": f"dp{world}",
           "model_tflops_per_gpu": flops / (ms * 1e-3) / 1e12, "attention_block_pairs_per_layer": pairs / 24,
           "params": sum(p.numel() for p in model.parameters()), "optimizer": "AdamW (fused)",
           "grad_allreduce": "bucketed, overlapped with the backward (NCCL)" if world > 1 else "none (1 GPU)"}
    del model, opt, dp
    torch.cuda.empty_cache()
    return res


def cpu_reference(cfg, *, warmup=1, steps=3, heads=1, seconds_budget=60.0):
    """The reference's CPU path on a bounded sample: the numpy port of its
    mask builder, then the attention forward (the reference raises
    NotImplementedError for a CPU backward) over ``heads`` heads of the config
    on the qk_aug inputs -- torch's compiled CPU flex_attention, the kernel the
    reference's flex_attention call runs on a CPU, or, where Inductor cannot
    build that kernel on the host (it needs AVX-512 / AVX2 micro-GEMMs), the
    oracle's block-sparse restatement of the same algorithm on every 4th q
    block of the sample."""
    from oracle import mask_oracle as MO
    from oracle import attn_oracle as AO
    from torch.nn.attention.flex_attention import BlockMask, flex_attention as torch_flex
    if os.path.exists("/usr/bin/g++") and not os.environ.get("CXX"):
        os.environ["CXX"] = "/usr/bin/g++"   # Inductor's C++ flex template needs a g++ with libgomp
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    x = make_inputs(cfg, device="cpu", seed=0, heads=slice(0, heads))
    T, bs = cfg.T, cfg.block_size
    QB = T // bs
    docs = x["docs"].long()

    def document_causal(b, h, q_idx, kv_idx):
        return (q_idx >= kv_idx) & (docs[q_idx] == docs[kv_idx])

    cos_t, sin_t = AO.trig_tables(x["omegas"], T)
    qa, ka, va = AO.qk_aug_inputs(x["q"].float(), x["k"].float(), x["v"].float(), x["coeff_cos"], x["coeff_sin"],
                                  cos_t, sin_t, beta=BETA, scale=SCALE)
    fa = torch.compile(torch_flex, dynamic=False)
    mode = {"kernel": "compiled"}
    sample_rows = range(0, QB, 4)

    def one():
        t0 = time.perf_counter()
        cen = MO.select_pointer_blocks(x["logits"].numpy(), x["gumbel"].numpy(), M=cfg.M, tau=cfg.select_tau)
        m = MO.build_pointer_blockmask(docs=x["docs"].numpy(), block_size=bs, M=cfg.M, centres=cen,
                                       budget_rep=x["budget_rep"].numpy(), local_blocks=cfg.local_eff,
                                       half_blocks=cfg.half_blocks, global_blocks_max=cfg.global_blocks,
                                       budget_blocks=cfg.budget_blocks, budget_is_total=cfg.budget_is_total,
                                       budget_temp=cfg.budget_temp, with_transpose=False)
        kvi = torch.from_numpy(MO.flex_padded(m["kv_packed"], QB))[None]
        kvn = torch.from_numpy(m["kv_num"])[None]
        t_build = time.perf_counter() - t0
        if mode["kernel"] == "compiled":
            try:
                bmk = BlockMask.from_kv_blocks(kvn, kvi, torch.zeros_like(kvn), torch.zeros_like(kvi), BLOCK_SIZE=bs,
                                               mask_mod=document_causal)
                fa(qa[None], ka[None], va[None], block_mask=bmk, scale=SCALE)
                return time.perf_counter() - t0, int(m["kv_num"].sum())
            except Exception as e:  # Inductor could not build the CPU kernel on this host
                mode["kernel"] = "oracle"
                mode["why"] = f"{type(e).__name__}"
                t0 = time.perf_counter() - t_build
        _, pairs = AO.block_sparse_forward(qa, ka, va, kvn[0], kvi[0], docs, scale=SCALE, block_size=bs,
                                           q_blocks=sample_rows)
        return time.perf_counter() - t0, pairs

    for _ in range(max(1, warmup)):      # the first call compiles
        one()
    times, P = [], 0
    t_start = time.perf_counter()
    for _ in range(max(1, steps)):
        dt, P = one()
        times.append(dt)
        if time.perf_counter() - t_start > seconds_budget:
            break
    sec = sum(times) / len(times)
    fwd_flops = 4 * bs * bs * 64 * P
    if mode["kernel"] == "compiled":
        what = "torch.compile'd CPU flex_attention"
    else:
        what = (f"the oracle's block-sparse fp32 forward on every 4th q block (the compiled CPU flex kernel "
                f"failed to build here: {mode['why']})")
    return {"value": fwd_flops / sec / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{cfg.name} with {heads} of {cfg.H} heads (T={T}), forward only (the reference has no CPU "
                      f"backward): numpy port of the mask builder + {what} on the qk_aug inputs, "
                      f"{len(times)} timed steps", "seconds_per_step": sec}


def torch_builder_ops(logits, gumbel, budget_rep, *, tau, M, L, p, G, budget_rem, temp, docs=None,
                      block_size=128):
    """The reference builder's steps (model/attn_bias.py:688-837) as eager torch
    ops on the GPU -- the document starts of each block (change points, running
    max), Gumbel top-M over the causal candidates, stick-breaking radius
    allocation with largest-remainder rounding, the local / pointer / global
    window entries with their document clamps, then sort, de-duplicate and
    pack (unique blocks ascending, repeats after).  Timed beside this
    package's builder kernel as the GPU-torch form of the same work; its lists
    equal the oracle's (a CPU test checks that)."""
    H, QB, _ = logits.shape
    dev = logits.device
    qb = torch.arange(QB, device=dev)
    dsp = dsl = torch.zeros(QB, dtype=torch.long, device=dev)
    if docs is not None:
        T = docs.shape[0]
        tok = torch.arange(T, device=dev)
        change = torch.ones(T, dtype=torch.bool, device=dev)
        change[1:] = docs[1:] != docs[:-1]
        dst = torch.where(change, tok, torch.zeros_like(tok)).cummax(0).values
        dsp = torch.div(dst[(qb + 1) * block_size - 1], block_size, rounding_mode="floor")
        dsl = torch.div(dst[qb * block_size], block_size, rounding_mode="floor")
    causal = qb[None, :] <= qb[:, None]
    s = torch.where(causal, logits / tau + gumbel, torch.full_like(logits, -float("inf")))
    cen = torch.topk(s, M, dim=-1).indices                                   # [H, QB, M]
    cen = torch.maximum(torch.minimum(cen, qb[None, :, None]), dsp[None, :, None])
    # radius: M - 1 stick fractions, the last piece the rest; largest-remainder rounding
    u = torch.sigmoid(budget_rep[..., : M - 1] / temp)
    rem = torch.full(u.shape[:-1], float(budget_rem), device=dev)
    pieces = []
    for m in range(M - 1):
        b = u[..., m] * rem
        pieces.append(b)
        rem = rem - b
    pieces.append(rem)
    alloc = torch.stack(pieces, -1)
    fl = torch.floor(alloc)
    fr = alloc - fl
    left = (budget_rem - fl.sum(-1, keepdim=True)).clamp(0, M)
    rank = torch.sort(torch.sort(-fr, dim=-1, stable=True).indices, dim=-1).indices
    r = (fl + (rank < left).float()).clamp(0, p).long()
    # window entries
    local = torch.maximum((qb[:, None] - torch.arange(L, device=dev)[None, :]).clamp(min=0), dsl[:, None])
    local = local.expand(H, QB, L)
    offs = torch.arange(-p, p + 1, device=dev)
    w = (cen[..., None] + offs).clamp(0, QB - 1)
    w = torch.maximum(torch.minimum(w, qb[None, :, None, None]), dsp[None, :, None, None])
    w = torch.where(offs.abs() <= r[..., None], w, cen[..., None]).reshape(H, QB, -1)
    glob = torch.minimum(dsp[:, None] + torch.arange(G, device=dev)[None, :], qb[:, None]).expand(H, QB, G)
    ent = torch.cat([local, w, glob], -1)
    srt = ent.sort(-1).values
    first = torch.ones_like(srt, dtype=torch.bool)
    first[..., 1:] = srt[..., 1:] != srt[..., :-1]
    key = (~first).long() * QB + srt
    packed = srt.gather(-1, torch.sort(key, dim=-1, stable=True).indices)
    return first.sum(-1).to(torch.int32), packed.to(torch.int32)


def run_flex(args):
    """torch's compiled flex_attention (Inductor Triton) on the GPU: the
    reference's GPU path for this layer, on the same inputs and mask.  The
    qk_aug dims are formed by the reference's torch ops (scoped_medium.py:
    380-421), the call is the compiled standalone flex_attention of
    scoped_medium.py:37-50 and :422, the mask is the reference's
    BlockMask.from_kv_blocks call (model/attn_bias.py:851-874) over the
    flex-padded lists of this configuration (built by this package's builder:
    the reference's builder sources do not travel to the GPU box).  Times the
    step (from_kv_blocks + qk_aug prep + forward + backward to q, k, v and the
    coefficients) and each phase with CUDA events on the current stream."""
    from torch.nn.attention.flex_attention import BlockMask, flex_attention as torch_flex
    from scope_b200.synth import build_config_mask
    torch.cuda.set_device(0)
    cfg = CONFIGS[args.config]
    if args.heads:
        import dataclasses
        cfg = dataclasses.replace(cfg, H=args.heads)
    dev = torch.device("cuda", 0)
    x = make_inputs(cfg, device=dev, seed=0)
    H, T, D, K, bs = cfg.H, cfg.T, cfg.D, cfg.K, cfg.block_size
    b = PointerBlockMaskBuilder(num_heads=H, M=cfg.M, pointer_local_blocks=cfg.local_eff,
                                pointer_half_blocks=cfg.half_blocks, pointer_global_blocks=cfg.global_blocks,
                                pointer_budget_blocks=cfg.budget_blocks, pointer_budget_is_total=cfg.budget_is_total,
                                pointer_budget_temp=cfg.budget_temp)
    bmp = b.select_and_build(pointer_logits=x["logits"], gumbel=x["gumbel"], tau=cfg.select_tau, docs=x["docs"],
                             budget_rep=x["budget_rep"], block_size=bs, layout="flex_padded")
    P = int(bmp.kv_num_blocks.sum().item())
    docs = x["docs"].long()

    def document_causal(b_, h, q_idx, kv_idx):
        q_ = q_idx.to(torch.long)
        k_ = kv_idx.to(torch.long)
        return (q_ >= k_) & (docs[q_] == docs[k_])

    kvn, kvi = bmp.kv_num_blocks.contiguous(), bmp.kv_indices.contiguous()

    def make_mask():
        return BlockMask.from_kv_blocks(kvn, kvi, torch.zeros_like(kvn), torch.zeros_like(kvi), BLOCK_SIZE=bs,
                                        mask_mod=document_causal)

    cos_t, sin_t = trig_tables(x["omegas"], T)
    leaves = {n: x[n].detach().requires_grad_(True) for n in ("q", "k", "v", "coeff_cos", "coeff_sin")}
    s_aug = math.sqrt(BETA / SCALE)

    def prep():
        # the reference's qk_aug ops (scoped_medium.py:384-421), B = 1
        ct = cos_t.transpose(0, 1).to(torch.float32)[None].expand(H, T, K)
        st = sin_t.transpose(0, 1).to(torch.float32)[None].expand(H, T, K)
        cc, cs = leaves["coeff_cos"], leaves["coeff_sin"]
        q_pos = (torch.cat([cc * ct + cs * st, cc * st - cs * ct], -1) * s_aug).to(torch.bfloat16)
        k_pos = (torch.cat([ct, st], -1) * s_aug).to(torch.bfloat16)
        qa = torch.cat([leaves["q"], q_pos], -1)
        ka = torch.cat([leaves["k"], k_pos], -1)
        va = torch.cat([leaves["v"], leaves["v"].new_zeros(H, T, q_pos.shape[-1])], -1)
        return qa[None], ka[None], va[None]

    fa = torch.compile(torch_flex, dynamic=False)
    do = x["do"][None]
    s = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]

    def step(acc=None):
        for t in leaves.values():
            t.grad = None
        ev[0].record(s)
        bmask = make_mask()
        ev[1].record(s)
        qa, ka, va = prep()
        ev[2].record(s)
        y = fa(qa, ka, va, block_mask=bmask, scale=SCALE)[..., :D]
        ev[3].record(s)
        y.backward(do)
        ev[4].record(s)
        if acc is not None:
            torch.cuda.synchronize()
            for i in range(4):
                acc[i] += ev[i].elapsed_time(ev[i + 1])

    t0 = time.perf_counter()
    step()
    torch.cuda.synchronize()
    compile_s = time.perf_counter() - t0
    for _ in range(max(args.warmup, 3) - 1):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(args.steps):
        step()
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    acc = [0.0] * 4
    reps = 3
    for _ in range(reps):
        step(acc)
    ph = [a / reps for a in acc]
    # the builder's work as eager torch ops on the GPU, beside this package's kernel
    L_, p_, G_ = cfg.local_eff, cfg.half_blocks, cfg.global_blocks
    # integer radius budget (model/attn_bias.py:724-734)
    if cfg.budget_is_total:
        extra = max(min(cfg.budget_blocks, L_ + cfg.M + 2 * cfg.M * p_) - L_ - cfg.M, 0)
    else:
        extra = max(0, cfg.budget_blocks)
    brem = min(extra // 2, cfg.M * p_)
    bkw = dict(tau=cfg.select_tau, M=cfg.M, L=L_, p=p_, G=G_, budget_rem=brem, temp=cfg.budget_temp,
               docs=x["docs"].long(), block_size=bs)
    for _ in range(3):
        torch_builder_ops(x["logits"], x["gumbel"], x["budget_rep"], **bkw)
    torch.cuda.synchronize()
    e0.record(s)
    for _ in range(5):
        torch_builder_ops(x["logits"], x["gumbel"], x["budget_rep"], **bkw)
    e1.record(s)
    torch.cuda.synchronize()
    torch_builder_ms = e0.elapsed_time(e1) / 5
    flops = 14 * bs * bs * D * P
    res = {"impl": "torch.compile(flex_attention), Inductor Triton, on the GPU", "value": flops / (ms * 1e-3) / 1e12,
           "unit": "TFLOP/s", "ms_per_step": ms, "active_block_pairs": P, "steps": args.steps,
           "phases_ms": {"from_kv_blocks_ms": ph[0], "qk_aug_prep_ms": ph[1], "forward_ms": ph[2],
                         "backward_ms": ph[3]},
           "attention_tflops": flops / ((ph[2] + ph[3]) * 1e-3) / 1e12, "compile_s": compile_s,
           "builder_torch_ops_ms": torch_builder_ms,
           "builder_note": "the reference builder's steps as eager torch ops on this GPU (torch_builder_ops); "
                           "with BlockMask.from_kv_blocks (from_kv_blocks_ms) that is its mask path",
           "config": {"workload": f"{cfg.name}: the same layer, head dim 64 + {2 * K} qk_aug dims", "H": H, "T": T,
                      "block_size": bs, "K": K}}
    return res


def gpu_reference_subprocess(args, timeout_s=480):
    """run_flex in a child process (bounded in time; a compile failure or
    a slow compile cannot take the bench down with it)."""
    cmd = [sys.executable, os.path.abspath(__file__), "--impl", "flex", "--config", args.config, "--steps", "5",
           "--warmup", "3"]
    if args.heads:
        cmd += ["--heads", str(args.heads)]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout_s)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"torch.compile(flex_attention) did not finish within {timeout_s} s"}
    for ln in reversed(r.stdout.splitlines()):
        if ln.startswith("{"):
            try:
                return json.loads(ln)
            except ValueError:
                break
    tail = (r.stderr or r.stdout).strip().splitlines()[-1:] or ["no output"]
    return {"unavailable": f"flex_attention run failed (rc {r.returncode}): {tail[0][:200]}"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg = CONFIGS[args.config]
    res = cpu_reference(cfg, warmup=args.warmup, steps=args.steps)
    line = {"metric": METRIC, "value": res["value"], "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": res["seconds_per_step"] * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{cfg.name}: one SCOPE attention layer, 1-head CPU sample", "T": cfg.T,
                       "H": 1, "block_size": cfg.block_size, "K": cfg.K, "spectral_impl": "qk_aug"},
            "impl": "reference",
            "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": res["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c3")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "flex"])
    ap.add_argument("--no-gpu-reference", action="store_true")
    ap.add_argument("--no-decoder", action="store_true")
    ap.add_argument("--no-score-mod", action="store_true", help="skip the score_mod-closure layer leg")
    ap.add_argument("--no-teacher", action="store_true", help="skip the teacher block-mass leg")
    ap.add_argument("--no-graph", action="store_true", help="time the step eagerly instead of as a CUDA graph")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--heads", type=int, default=0,
                    help="run only this many heads of the config (a smaller case, e.g. for profiling)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.impl == "flex":
        print(json.dumps(run_flex(args)), flush=True)
        return
    args.warmup = max(args.warmup, 3)
    rank, world, local = setup_dist()
    cfg = CONFIGS[args.config]
    if args.heads:
        import dataclasses
        cfg = dataclasses.replace(cfg, H=args.heads)
    wl = Workload(cfg, rank, world, "cuda")
    bm0 = wl.build()
    P_local = active_pairs(bm0)
    for _ in range(args.warmup):
        wl.step()
    torch.cuda.synchronize()
    L = _lib.lib()
    graph, per_step, graph_why = (None, 0, "disabled (--no-graph)")
    if not args.no_graph:
        graph, per_step, graph_why = capture_step(wl, world)
    step_fn = graph.replay if graph is not None else wl.step
    for _ in range(2):
        step_fn()
    torch.cuda.synchronize()
    n0 = L.scope_launch_count()
    with ClockSampler(local) as clk:
        ms = time_steps(step_fn, args.steps, world)
    # a graph replay launches the captured kernels without calling the library
    launches = per_step * args.steps if graph is not None else L.scope_launch_count() - n0
    P_t = torch.tensor([P_local], device="cuda", dtype=torch.int64)
    if world > 1:
        dist.all_reduce(P_t)
    P = int(P_t.item())
    bs, D = cfg.block_size, cfg.D
    flops = 14 * bs * bs * D * P
    ms_step = ms / args.steps
    value = flops / (ms_step * 1e-3) / 1e12

    # per-phase device times (builder / forward / backward) on this rank
    ph = phase_times(wl)
    # the mask builder alone against its HBM roofline: the causal candidate logits and
    # Gumbel noise read, the lists and counts written (block_info, the zeroed bitmap and
    # statistics included in the time)
    QBc = cfg.QB
    mb_bytes = wl.hp * (QBc * (QBc + 1) // 2) * 8 + wl.hp * QBc * (4 + 4 * bm0.kv_indices.shape[-1])
    torch.cuda.synchronize()
    s0 = torch.cuda.current_stream()
    eb0, eb1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gpu_hold()
    eb0.record(s0)
    for _ in range(10):
        wl.build()
    eb1.record(s0)
    torch.cuda.synchronize()
    mb_ms = eb0.elapsed_time(eb1) / 10
    hbm_peak = peaks()[0]
    mask_builder = {"kernel": "scope_mask_build (+ block_info, zeroed bitmap and statistics)", "ms": mb_ms,
                    "algorithmic_bytes": mb_bytes, "achieved_gbs": mb_bytes / (mb_ms * 1e-3) / 1e9,
                    "peak_gbs": hbm_peak, "frac": mb_bytes / (mb_ms * 1e-3) / 1e9 / hbm_peak,
                    "unit": "GB/s", "bound": "hbm"}
    hbm, bf16, src = peaks()
    f_fwd, f_bwd = 4 * bs * bs * D * P_local, 10 * bs * bs * D * P_local
    phases = {"mask_build_ms": ph[0], "forward_ms": ph[1], "backward_ms": ph[2]}
    dom = int(max(range(3), key=lambda i: ph[i]))
    if dom == 0:
        # builder: algorithmic bytes = causal candidate logits + noise read + lists written
        QB = cfg.QB
        byts = wl.hp * (QB * (QB + 1) // 2) * 8 + wl.hp * QB * (4 + 4 * bm0.kv_indices.shape[-1])
        ach = byts / (ph[0] * 1e-3) / 1e9
        roof = {"kernel": "scope mask builder", "bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s"}
    else:
        fl = f_fwd if dom == 1 else f_bwd
        ach = fl / (ph[dom] * 1e-3) / 1e12
        roof = {"kernel": "attention " + ("forward" if dom == 1 else "backward"), "bound": "tensor",
                "achieved": ach, "peak": bf16, "unit": "TFLOP/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["peak_source"] = f"{src} (MEASURED_PEAKS.json burst)" if src == "measured" else "fallback"
    # DRAM traffic of the dominant kernel from one ncu capture of this build
    # (dram__bytes_read.sum + dram__bytes_write.sum), scaled to this launch
    cap = NCU_TRAFFIC["builder" if dom == 0 else ("forward" if dom == 1 else "backward")]
    units = wl.hp if dom == 0 else P_local
    roof["traffic"] = cap["bytes"] / cap["units"] * units
    roof["traffic_unit"] = "bytes per launch"
    roof["traffic_source"] = cap["capture"] + ", scaled to this launch's " + ("heads" if dom == 0 else "active pairs")

    e2e = None
    if not args.no_e2e:
        host = {"in": {n: wl.x[n].detach().cpu().pin_memory() for n in E2EPipeline.IN},
                "out": {"out": torch.empty(cfg.T, wl.hp, D, dtype=torch.bfloat16).pin_memory().permute(1, 0, 2)}}
        for n in ("q", "k", "v"):
            host["out"]["d" + n] = torch.empty(cfg.T, wl.hp, D, dtype=torch.bfloat16).pin_memory().permute(1, 0, 2)
        for n in ("coeff_cos", "coeff_sin"):
            host["out"]["d" + n] = torch.empty_like(wl.x[n], device="cpu").pin_memory()
        pipe = E2EPipeline(wl, host)
        for _ in range(2):
            pipe.step()
        pipe.finish()
        torch.cuda.synchronize()
        # enough steps that the pipeline's fill (the first H2D) and drain (the last
        # D2H), which overlap nothing, do not dominate the per-step figure: over 20
        # steps they add about a tenth of a step to each
        e_steps = max(20, args.steps)
        ms_e = time_e2e(pipe, e_steps, world)
        h2d = sum(t.numel() * t.element_size() for t in host["in"].values())
        d2h = sum(t.numel() * t.element_size() for t in host["out"].values())
        e2e = {"value": flops / (ms_e / e_steps * 1e-3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
               "ms_per_step": ms_e / e_steps, "steps": e_steps,
               "note": "pipelined: step i+1's inputs travel while step i computes and step i's results "
                       "travel back; the first H2D and the last D2H are inside the timed region"}

    coeff = coeff_block(wl, cfg, hbm, cpu=(rank == 0 and world == 1 and not args.no_cpu_baseline))
    smod = None if args.no_score_mod else score_mod_leg(wl, cfg, bm0, P_local)
    teacher = None if args.no_teacher else teacher_leg(cfg, wl.hp)

    decoder = None
    if not args.no_decoder and not args.heads and args.config == "c3":
        decoder = decoder_bench(rank, world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            r = cpu_reference(cfg, warmup=1, steps=3, seconds_budget=20.0)
            cpu = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
        except Exception as e:  # the baseline is reported, not required
            cpu = {"value": None, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port",
                   "sample": f"failed: {type(e).__name__}: {e}"[:300]}

    gref = None
    if rank == 0 and world == 1 and not args.no_gpu_reference:
        # torch's compiled flex_attention (Triton) on this GPU, same layer and inputs,
        # in a child process (this process's buffers stay resident meanwhile)
        torch.cuda.synchronize()
        gref = gpu_reference_subprocess(args)
        if "value" in gref:
            gref["ours_over_reference"] = value / gref["value"]
            ours_attn = (4 + 10) * bs * bs * D * P_local / ((ph[1] + ph[2]) * 1e-3) / 1e12
            gref["ours_attention_tflops"] = ours_attn
            gref["attention_ours_over_reference"] = ours_attn / gref["attention_tflops"]
            if "builder_torch_ops_ms" in gref:
                # the mask path: torch ops + BlockMask.from_kv_blocks against this package's builder phase
                gref["mask_ours_over_reference"] = (gref["builder_torch_ops_ms"] +
                                                    gref["phases_ms"]["from_kv_blocks_ms"]) / ph[0]

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": f"{cfg.name}: one SCOPE attention layer, select+build, fwd+bwd",
                           "B": 1, "H": cfg.H, "T": cfg.T, "D": D, "block_size": bs, "K": cfg.K,
                           "spectral_impl": "qk_aug", "parallelism": f"heads/{world}",
                           "active_block_pairs": P, "l2": "inputs larger than L2 (q,k,v,dO 1 GiB)"},
                "roofline": roof, "phases_ms": phases, "cpu_baseline": cpu, "e2e": e2e,
                "clocks": clk.summary(), "gpu_launches": int(launches), "coeff_block": coeff,
                "gpu_reference": gref, "decoder": decoder, "mask_builder": mask_builder, "score_mod": smod,
                "teacher": teacher,
                "step_launch": {"cuda_graph": graph is not None, "kernels_per_step": per_step,
                                "note": graph_why or "the timed steps replay one CUDA graph of the whole step"}}
        print(json.dumps(line), flush=True)
    # a graph holding NCCL work must be destroyed before the process group, or the
    # exit waits for good: reset() frees the graph and its executable even while
    # references to it (step_fn is its bound replay) remain
    torch.cuda.synchronize()
    if graph is not None:
        graph.reset()
    del step_fn, graph
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
