#!/usr/bin/env python3
"""Rollout throughput benchmark: the reference's headline metric, rollout
env-steps per second at 1/2/4/8 B200 against the reference's CPU path.

One "step" = one 128-tick rollout of one GPU's env shard: observe -> masks ->
learner act -> opponent act -> step (device auto-reset) -> crate recycling
every 16 ticks, captured as one CUDA graph.  value = envs * ticks * ranks /
max-over-ranks device time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--config cfg2|cfg4|cfg5]

--config selects the workload (default cfg2, the headline): cfg2 = N=5632,
MLP learner seat 0 vs astar seat 1; cfg4 = N=65536, self-play (one MLP for
both seats, one N=256 GEMM), plus one PPO update on the seat-0 buffer timed
separately; cfg5 = N=5632, CNN learner vs greedy.

Multi-GPU (weak scaling, no data-path collective in the rollout): launched
with torch.distributed.run, each rank runs its own shard; cfg4's PPO update
all-reduces gradients and advantage statistics over NCCL.  --impl reference
times the CPU restatement of the reference algorithm (oracle/, the reference
itself is Python and cannot be shipped) on the host's cores for the same
workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [ROOT, os.path.join(ROOT, "qqt-gpu-sim_b200")]

METRIC = "rollout env-steps/sec (sim+obs+policy+sample) at 1/2/4/8 B200 vs ref CPU"
UNIT = "env-steps/s"

CONFIGS = {
    "cfg2": dict(envs=5632, learner="mlp", seats=(0,), opponent="astar", ppo=False, cpu=(352, 16),
                 ref_per=None,
                 workload="cfg2: 13x13 pillar corridor (bricks p=0.7), P=2, N=5632 envs per "
                          "GPU, random-init MLP learner seat 0 (view_perm) vs astar seat 1, "
                          "128-tick rollout"),
    "cfg4": dict(envs=65536, learner="mlp", seats=(0, 1), opponent=None, ppo=True, cpu=(512, 8),
                 ref_per=512,
                 workload="cfg4: cfg2 map, N=65536 envs per GPU, self-play (one random-init "
                          "MLP for both seats, one N=256 GEMM), 128-tick rollout; PPO update "
                          "(4 epochs x 8 minibatches, seat-0 buffer) timed separately"),
    "cfg3": dict(envs=16384, learner=None, seats=(), opponent=None, ppo=False, cpu=(64, 1),
                 ref_per=None,
                 workload="cfg3: chain/danger stress, 13x13 border-wall map, N=16384 envs per GPU, "
                          "20-40 bombs per env (fuse U{1..30}, blast U{1..5}); one step = step "
                          "(IDLE, no reset) + danger map + obs + masks + astar V_safe/V_opp and "
                          "actions for both players, from the same stress state every step"),
    "cfg5": dict(envs=5632, learner="cnn", seats=(0,), opponent="greedy", ppo=False, cpu=(64, 8),
                 ref_per=64,
                 workload="cfg5: cfg2 map, N=5632 envs per GPU, random-init CNN learner seat 0 "
                          "vs greedy seat 1, 128-tick rollout"),
}
CFG = CONFIGS["cfg2"]
N_ENVS = 5632      # from the config; --envs overrides for profiling cases
TICKS = 128

# Algorithmic bytes per env per launch (reference dtypes, compulsory traffic).
OBS_ROW = 2368 * 2
ALG_BYTES = {
    "step": 169 * (1 + 1 + 1 + 1 + 2 + 1 + 2) * 2 - 169 + 280 + 32 + 8 + 1,
    "observe": 169 * (1 + 1 + 1 + 1 + 2 + 2) + 56 + OBS_ROW + 14,
    # the step with the next observation: the step's bytes + the row and masks
    "step+observe": 169 * (1 + 1 + 1 + 1 + 2 + 1 + 2) * 2 - 169 + 280 + 32 + 8 + 1 + OBS_ROW + 14,
    "astar": 169 * (1 + 1 + 1 + 2) + 169 * 2 + 10 + 20 + 16,
    "greedy": 169 * (1 + 1 + 1 + 2) + 169 * 2 + 10 + 20 + 16,
    "policy": OBS_ROW,           # + per seat: masks, uniforms, actions, log-prob, value
    "flush": 169 * 8 + 16,
}
POLICY_PER_SEAT = 5 + 2 + 8 + 16 + 4 + 4
MLP_FLOPS = 2 * (2366 * 128 + 128 * 128 + 3 * 128 * 64 + 64 * 8)
# CNN policy per sample (train/model.py:77-101): convs 14->16, 16->32, 32->64 (3x3),
# 64->8 (1x1) on 13x13, Linear(1352->128), the 128x128 layer, heads: 9.07 MFLOP
CNN_FLOPS = 2 * (169 * 9 * (14 * 16 + 16 * 32 + 32 * 64) + 169 * 64 * 8 + 1352 * 128 +
                 128 * 128 + 3 * 128 * 64 + 64 * 8)


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return (float(m["hbm_gbs"]), float(m.get("bf16_tflops_sustained", m["bf16_tflops"])),
                "measured")
    except Exception:
        return 6650.0, 1400.0, "fallback"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons every 10 ms while running,
    through NVML (nvidia-smi's library); the GPU is found by its PCI bus id,
    so CUDA_VISIBLE_DEVICES remapping does not matter."""

    # nvmlClocksEventReason* bits
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
            "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device_index):
        self.device_index = device_index
        self.rows = []
        self._stop = threading.Event()
        self._t = None
        self._err = None

    def _handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        try:
            pr = torch.cuda.get_device_properties(self.device_index)
            bus = "%08x:%02x:%02x.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.device_index)

    def __enter__(self):
        try:
            nv, h = self._handle()
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        except Exception as e:          # no NVML: the line says "unsampled"
            self._err = repr(e)
            return self

        def run():
            while not self._stop.is_set():
                try:
                    self.rows.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                      nv.nvmlDeviceGetCurrentClocksEventReasons(h)))
                except Exception as e:
                    self._err = repr(e)
                self._stop.wait(0.01)
        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t is not None:
            self._t.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"],
                    "error": self._err}
        reasons = sorted({k for _, r in self.rows for k, bit in self.BITS.items() if r & bit})
        return {"sm_mhz": statistics.median(m for m, _ in self.rows), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.rows), "source": "nvml, 10 ms"}


def _template(cfg, n, seed):
    from qqt_b200 import scenarios
    return scenarios.corridor_template(cfg, n, seed)


# --------------------------------------------------------------- CPU legs

def cpu_leg(n_per, ticks, procs, seed=0, conf="cfg2"):
    """The oracle's rollout tick (oracle/cpu_rollout.py) on `procs` spawned
    processes of n_per envs each: a 40-tick warm-up into a bomb-rich
    mid-game state, then `ticks` timed ticks (the slowest shard's time).
    Returns (env-steps/s, env-steps, seconds)."""
    from oracle.cpu_rollout import ShardPool
    pool = ShardPool(conf, n_per, procs, seed=seed, root=ROOT)
    try:
        steps, dt = pool.run(ticks)
    finally:
        pool.close()
    return steps / dt, steps, dt


# ------------------------------------------------------------ GPU leg

def build_engine(device, rank, slots=None, groups=1):
    """The rank's env shard as `groups` independent env groups (one sim, bot
    and rollout buffer each; one shared policy pack)."""
    import torch
    from qqt_b200 import scenarios
    from qqt_b200.bots import make_bot
    from qqt_b200.config import SimConfig
    from qqt_b200.policy import B200Policy
    from qqt_b200.policy_init import init_params
    from qqt_b200.rollout import Rollout, RolloutGroups
    from qqt_b200.sim import B200Sim
    cfg = SimConfig(**scenarios.CFG2)
    if N_ENVS % groups:
        raise ValueError("envs per GPU must divide into the groups")
    n = N_ENVS // groups
    tmpl = _template(cfg, N_ENVS, 1 + rank)
    pol = B200Policy(init_params(cfg.obs_shape, CFG["learner"], seed=1), cfg.obs_shape, 2,
                     seats=CFG["seats"], device=device, arch=CFG["learner"])
    ros = []
    for g in range(groups):
        part = {k: v[g * n:(g + 1) * n] for k, v in tmpl.items()}
        sim = B200Sim(cfg, n, device=device, seed=1 + rank + 1000 * g, template=part)
        sim.set_template(part, apply=False, seed=1 + rank + 1000 * g, swap_spawns=False)
        bot = make_bot(sim, CFG["opponent"], mode=True) if CFG["opponent"] else None
        ros.append(Rollout(sim, pol, bot, T=TICKS, slots=slots))
    gen = torch.Generator(device=device).manual_seed(1234 + rank)
    return RolloutGroups(ros), gen


def graph_kernel_times(grp):
    """Per-call device durations inside the captured rollout: a second graph
    of the same T-tick rollout (same streams and concurrency) with a pair of
    external timing events around every engine call, replayed once after the
    timed region.  Returns name -> (launches per rollout of one group, mean
    ms per call)."""
    import torch
    bot_name = CFG["opponent"] or "bot"
    marks = []

    def probe(name, fn):
        a = torch.cuda.Event(enable_timing=True, external=True)
        b = torch.cuda.Event(enable_timing=True, external=True)
        a.record()
        out = fn()
        b.record()
        marks.append((bot_name if name == "bot" else name, a, b))
        return out

    for ro in grp.ros:
        ro.probe = probe
    try:
        grp.capture()
    finally:
        for ro in grp.ros:
            ro.probe = None
    grp.replay()
    torch.cuda.synchronize()
    grp.graph, grp.graphs = None, []
    times = {}
    for name, a, b in marks:
        times.setdefault(name, []).append(a.elapsed_time(b))
    g = len(grp.ros)
    return {k: (len(v) // g, sum(v) / len(v)) for k, v in times.items()}


def _launches_per_rollout():
    """Kernels per rollout of one env group: per tick policy (fused MLP: 1;
    CNN: trunk + linear/tail per seat), bot (astar: cap + field; greedy: 1)
    and the step (which also writes the next observation); a separate observe
    on the first tick; the crate recycling every 16 ticks (which rewrites the
    crate channel of the step's next-tick rows with one torch copy, not
    counted here)."""
    pol = 1 if CFG["learner"] == "mlp" else 1 + len(CFG["seats"])
    bot = {"astar": 2, "greedy": 1, None: 0}[CFG["opponent"]]
    flushes = TICKS // 16
    return TICKS * (pol + bot + 1) + 1 + flushes


def ppo_leg(grp, device):
    """cfg4: one PPO update (4 epochs x 8 minibatches) on the seat-0 rollout
    buffer, after a bootstrap value for the state the rollout ended in;
    device time by CUDA events."""
    import torch
    from qqt_b200.ppo import MLPActorCritic, PPOConfig, ppo_update
    ro = grp.ros[0]
    sim, buf, pol = ro.sim, ro.buf, ro.learner
    cfg = PPOConfig(epochs=4, minibatches=8, lr=1e-4, entropy_coef=0.03, entropy_final=0.03)
    model = MLPActorCritic(sim.cfg.obs_shape, 2).to(device)
    model.load_state_dict({k: v.clone() for k, v in pol.params.items()}, strict=False)
    opt = torch.optim.Adam(model.parameters(), lr=cfg.lr, eps=1e-5)
    n = sim.num_envs
    rows = torch.zeros((n, sim.obs_stride), dtype=torch.float16, device=device)
    mm = torch.ones((n, 2, 5), dtype=torch.bool, device=device)
    bm = torch.ones((n, 2, 2), dtype=torch.bool, device=device)
    acts = torch.zeros((n, 2, 2), dtype=torch.int64, device=device)
    last = torch.zeros((len(ro.seats), n), dtype=torch.float32, device=device)
    u = torch.rand((len(ro.seats), n, 2), device=device)
    data = {"obs": buf.obs_rows, "mm": buf.mm[:, :, 0], "bm": buf.bm[:, :, 0],
            "act": buf.act[:, :, 0], "logp": buf.logp[:, 0], "val": buf.val[:, 0],
            "rew": buf.rew[:, :, 0], "done": buf.done, "dmg": buf.dmg[:, :, 0]}

    def update():
        obs, mmv, bmv = sim.observe_and_mask(rows, mm, bm, danger=False)
        pol.act_seats(obs, [mmv[:, s] for s in ro.seats], [bmv[:, s] for s in ro.seats], u,
                      [acts[:, s] for s in ro.seats], None, last)
        st = ppo_update(model, opt, data, last[0], cfg, cfg.entropy_coef, pid=0, profile=prof)
        pol.load_state_dict({k: p.detach() for k, p in model.state_dict().items()
                             if k in pol.params})
        return st

    # the first update also grows the allocator's pools (multi-GB minibatch
    # blocks) and creates the optimizer state; a training loop pays that once
    times = []
    prof = {}
    for _ in range(2):
        prof.clear()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        stats = update()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    ms = times[-1]
    ar_ms = sum(x.elapsed_time(y) for x, y in prof.get("allreduce_events", []))
    samples = buf.done.numel()
    return {"ms": round(ms, 2), "first_update_ms": round(times[0], 2), "samples": samples,
            "samples_per_s": round(samples / (ms / 1e3), 1),
            "minibatches": cfg.epochs * cfg.minibatches,
            "grad_allreduce_ms": round(ar_ms, 3),
            "grad_allreduce_share": round(ar_ms / ms, 5),
            "grad_allreduce_bytes": 345288 * 4,
            "includes": "bootstrap value, GAE kernel, advantage stats, 32 x (row gather, fused "
                        "forward, backward kernels, gradient all-reduce, clip, Adam), policy "
                        "repack; the second of two updates on the same rollout",
            "losses": {k: round(v, 5) for k, v in stats.items()}}


def gpu_bench(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = f"cuda:{local}"
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(device))
    groups = 1 if CFG["ppo"] else args.groups
    grp, gen = build_engine(device, rank, args.slots, groups)
    # first tick eagerly (one-time set-up: resolve tiers, ticker state)
    for ro in grp.ros:
        ro.draws.generate(gen)
        ro.tick(0)
    grp.collect()                    # finish a full eager rollout for a warm state
    n_inst = grp.ros[0].sim.num_envs
    grp.capture()
    pool = [[RolloutDrawsPool.make(ro.draws, gen) for ro in grp.ros]
            for _ in range(min(args.steps + args.warmup, 4))]
    l2 = torch.empty((64 << 20,), dtype=torch.float32, device=device)   # 256 MB > L2

    def one_step(i, ev):
        a, b = ev
        a.record()
        for ro, ts in zip(grp.ros, pool[i % len(pool)]):
            RolloutDrawsPool.load(ro.draws, ts)
        grp.replay()
        b.record()

    for i in range(args.warmup):
        one_step(i, (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)))
        l2.zero_()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            one_step(i, evs[i])
            l2.zero_()                      # flush L2 between timed steps (not timed)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in evs)
    t_max = torch.tensor([ms], device=device)
    if dist:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    ms = float(t_max.item())
    value = N_ENVS * TICKS * world * args.steps / (ms / 1e3)

    # ---- e2e: public API with host-fed draws and a host read of the rewards.
    # Two graphs read two draw-buffer sets: step i+1's draws are copied from
    # pinned host memory into one set (copy stream) while step i's graph runs
    # on the other, as a training loop streams its next rollout's draws.  One
    # timed region spans every step: the first copy, all replays, all copies,
    # every reward read and the L2 flushes.
    grp.capture(double_buffer=True)
    sets = [[t for d in ds for t in d.tensors()] for ds in grp.draw_sets]
    host_draws = [t.detach().cpu().pin_memory() for t in sets[0]]
    h2d = sum(t.numel() * t.element_size() for t in host_draws)
    rew_host = [torch.empty((ro.buf.rew.shape[0], ro.sim.num_envs), dtype=torch.float32).pin_memory()
                for ro in grp.ros]
    d2h = sum(r.numel() * 4 for r in rew_host)
    main = torch.cuda.current_stream(device)
    cs = torch.cuda.Stream(device)
    used = [torch.cuda.Event(), torch.cuda.Event()]       # replay on set k done
    landed = [torch.cuda.Event(), torch.cuda.Event()]     # copy into set k done
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for dst, src in zip(sets[0], host_draws):
        dst.copy_(src, non_blocking=True)
    for i in range(args.steps):
        k = i % 2
        if i + 1 < args.steps:
            with torch.cuda.stream(cs):
                if i >= 1:
                    cs.wait_event(used[1 - k])
                for dst, src in zip(sets[1 - k], host_draws):
                    dst.copy_(src, non_blocking=True)
                landed[1 - k].record(cs)
        if i >= 1:
            main.wait_event(landed[k])
        grp.replay(k)
        used[k].record(main)
        for ro, rh in zip(grp.ros, rew_host):
            rh.copy_(ro.buf.rew[:, :, 0], non_blocking=True)
        l2.zero_()
    b.record()
    b.synchronize()
    e_ms = a.elapsed_time(b)
    t_e = torch.tensor([e_ms], device=device)
    if dist:
        dist.all_reduce(t_e, op=dist.ReduceOp.MAX)
    e_value = N_ENVS * TICKS * world * args.steps / (float(t_e.item()) / 1e3)
    grp.graph, grp.graphs = None, []
    torch.cuda.synchronize()
    # per-kernel durations for the roofline: the same rollout graph with
    # timing events around each call (after the timed regions)
    kt = graph_kernel_times(grp)

    ppo = None
    if CFG["ppo"]:
        ppo = ppo_leg(grp, device)
        t_p = torch.tensor([ppo["ms"]], device=device)
        if dist:
            dist.all_reduce(t_p, op=dist.ReduceOp.MAX)
        ppo["ms"] = round(float(t_p.item()), 2)
        ppo["samples_per_s"] = round(ppo["samples"] * world / (ppo["ms"] / 1e3), 1)

    out = None
    if rank == 0:
        hbm, tflops, src = _peaks()
        per = {}
        n_seats = len(CFG["seats"])
        for k, (launches, mean_ms) in kt.items():
            if launches == 0:
                continue
            byt = ALG_BYTES["policy"] + n_seats * POLICY_PER_SEAT if k == "policy" else \
                ALG_BYTES.get(k, 169 * 8)
            per[k] = {"launches_per_rollout": launches, "mean_ms": round(mean_ms, 5),
                      "share": None, "alg_bytes_per_launch": byt * n_inst}
        tot = sum(v["launches_per_rollout"] * v["mean_ms"] for v in per.values())
        for v in per.values():
            v["share"] = round(v["launches_per_rollout"] * v["mean_ms"] / tot, 4)
        dom = max((k for k in per if k != "flush"), key=lambda k: per[k]["share"])
        d = per[dom]
        achieved = d["alg_bytes_per_launch"] / (d["mean_ms"] / 1e3) / 1e9
        # the CNN policy is a dense contraction (9.07 MFLOP per 4.7 KB row): its
        # roofline is the tensor pipe (the sustained bf16 peak: it is timed inside
        # the rollout graph); every other dominant kernel here is bandwidth-bound
        tensor_bound = dom == "policy" and CFG["learner"] == "cnn"
        if tensor_bound:
            d["alg_flops_per_launch"] = CNN_FLOPS * n_inst * n_seats
            achieved = d["alg_flops_per_launch"] / (d["mean_ms"] / 1e3) / 1e12
        # ncu traffic was captured for the default cfg2 shard (2 groups of 2816 envs)
        traffic = _ncu_traffic(dom) if args.config == "cfg2" and n_inst == 2816 else None
        cores = args.cpu_procs
        cpu_base = None
        if world == 1:
            cpu_v, cpu_steps, cpu_dt = cpu_leg(args.cpu_envs, args.cpu_ticks, cores,
                                               conf=args.config)
            cpu_base = {"value": round(cpu_v, 1), "unit": UNIT, "cores": cores, "kind": "port",
                        "sample": f"oracle (numpy restatement of the reference tick), "
                                  f"{cores} process(es) x {args.cpu_envs} envs of the same "
                                  f"workload: {args.cpu_ticks} mid-game ticks timed after a "
                                  f"40-tick warm-up into a bomb-rich state ({cpu_steps} "
                                  f"env-steps in {cpu_dt:.2f} s)"}
        out = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 sim, fp16xfp16->f32 tensor-core policy",
            "data": "synthetic (seeded template maps, random-init policy, device RNG draws)",
            "config": {"workload": CFG["workload"], "envs_per_gpu": N_ENVS, "ticks": TICKS,
                       "env_groups_per_gpu": groups,
                       "parallelism": f"env shards x{world}, no rollout collective",
                       "l2": "flushed (256 MB write) between timed steps; each step also "
                             "writes its T x N observation buffer (> L2)",
                       "cuda_graph": True,
                       "draws": "value: sampling / bot / crate draws generated on the device "
                                "before the timed region, copied device-to-device into the "
                                "graph's draw buffers inside it; e2e: copied from pinned host "
                                "memory inside the timed region"},
            "e2e": {"value": round(e_value, 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": _launches_per_rollout() * groups * args.steps,
            "roofline": {"kernel": dom, "bound": "tensor" if tensor_bound else "hbm",
                         "achieved": round(achieved, 1),
                         "peak": tflops if tensor_bound else hbm,
                         "unit": "TFLOP/s" if tensor_bound else "GB/s",
                         "frac": round(achieved / (tflops if tensor_bound else hbm), 4),
                         "peak_source": src, "traffic": traffic,
                         "per_kernel": per},
            "cpu_baseline": cpu_base,
            "clocks": clk.summary(),
        }
        if ppo is not None:
            out["ppo_update"] = ppo
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return out


# ------------------------------------------------------------ cfg3 stress

def _stress_state(cfg, n, seed):
    """Env-major numpy state of the cfg3 stress case."""
    import numpy as np
    from qqt_b200 import scenarios
    p = cfg.n_players
    fuse, owner, blast = scenarios.bomb_stress(n, cfg, seed)
    wall = np.broadcast_to(scenarios.border_walls(cfg.height, cfg.width), fuse.shape).copy()
    spawn = np.array(scenarios.open_spawns(cfg), np.float32)
    return {"wall": wall, "brick": np.zeros_like(wall), "crate": np.zeros_like(wall),
            "recycle": np.zeros_like(wall), "fuse": fuse, "owner": owner, "bomb_blast": blast,
            "pos": np.broadcast_to(spawn, (n, p, 2)).copy(), "alive": np.ones((n, p), bool),
            "hp": np.full((n, p), cfg.max_hp, np.uint8), "invuln": np.zeros((n, p), np.int64),
            "t": np.full(n, 40, np.int64)}


def _stress_oracle_worker(args):
    n, seed = args
    import numpy as np
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(1)
    except Exception:
        pass
    from oracle import qqt_oracle as O
    from qqt_b200 import scenarios
    from qqt_b200.config import SimConfig
    cfg = SimConfig(**scenarios.CFG1)
    p = cfg.n_players
    st = _stress_state(cfg, n, seed)
    full = {"since_bomb": np.full((n, p), cfg.place_dist_cooldown, np.int32),
            "bombs_cap": np.full((n, p), cfg.growth_bombs_start, np.int64),
            "blast_cap": np.full((n, p), cfg.growth_blast_start, np.int64),
            "spd_g": np.full((n, p), cfg.growth_speed_start, np.float32),
            "pending_lost": np.zeros((n, p), np.int64), "combo": np.zeros((n, p), np.int64),
            "last_hit": np.full((n, p), -10 ** 9, np.int64),
            "lo_bombs": np.full((n, p), cfg.growth_bombs_start, np.int64),
            "lo_blast": np.full((n, p), cfg.growth_blast_start, np.int64),
            "lo_spd": np.full((n, p), cfg.growth_speed_start, np.float32),
            "crate_prob": np.full(n, cfg.growth_crate_prob, np.float32),
            "hazard": np.zeros(n, bool)}
    st.update(full)
    rng = np.random.default_rng(seed)
    acts = np.zeros((n, p, 2), np.int64)
    acts[..., 0] = 4
    t0 = time.perf_counter()
    rb = rng.random((2, n, p)).astype(np.float32)
    O.step(cfg, st, acts, rb[0], rb[1])
    obs, _ = O.observe(cfg, st)
    obs32 = obs.astype(np.float16).astype(np.float32)
    mm, bm = O.legal_mask(cfg, st)
    for pid in range(p):
        O.astar_attack(cfg, st, obs32[:, 2 * p + 1], mm[:, pid], bm[:, pid], pid,
                       rng.random((n, 5)).astype(np.float32), return_fields=True)
    return n, time.perf_counter() - t0


def stress_bench(args):
    """cfg3: device time of step + danger/obs/masks + both players' astar
    fields and actions, restarted from the stress state every step."""
    import torch
    from qqt_b200 import scenarios
    from qqt_b200.bots import AstarBot
    from qqt_b200.config import SimConfig
    from qqt_b200.sim import B200Sim
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = f"cuda:{local}"
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(device))
    cfg = SimConfig(**scenarios.CFG1)
    n, p = N_ENVS, cfg.n_players
    sim = B200Sim(cfg, n, device=device, seed=7 + rank)
    sim.load_numpy_state(_stress_state(cfg, n, 7 + rank))
    snap = {k: v.clone() for k, v in sim._buf.items()}
    acts = torch.zeros((n, p, 2), dtype=torch.int64, device=device)
    acts[..., 0] = 4
    gen = torch.Generator(device=device).manual_seed(99 + rank)
    draws = (torch.rand((n, p), device=device, generator=gen),
             torch.rand((n, p), device=device, generator=gen))
    bots = []
    for pid in range(p):
        b = AstarBot(sim, mode=False)
        b.keep_fields = True
        bots.append(b)
    noise = torch.rand((p, n, 5), device=device, generator=gen)
    l2 = torch.empty((64 << 20,), dtype=torch.float32, device=device)

    def restore():
        for k, v in snap.items():
            sim._buf[k].copy_(v)

    def tick():
        sim.step(acts, auto_reset=False, crate_draws=draws, info_planes=False)
        obs, mm, bm = sim.observe_and_mask(danger=True)
        for pid, b in enumerate(bots):
            b.feed(noise=noise[pid])
            b.act(obs, mm[:, pid], bm[:, pid], pid)

    restore()
    tick()                                  # first step: records the blast tiers

    def timed_tick(ev):
        restore()
        l2.zero_()                          # flush L2 (not timed)
        ev[0].record()
        tick()
        ev[1].record()

    mk = lambda: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))  # noqa: E731
    for _ in range(args.warmup):
        timed_tick(mk())
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    evs = [mk() for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        for ev in evs:
            timed_tick(ev)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in evs)
    t_max = torch.tensor([ms], device=device)
    if dist:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
        dist.destroy_process_group()
    ms = float(t_max.item())
    if rank != 0:
        return None
    value = n * world * args.steps / (ms / 1e3)
    cpu_n = args.cpu_envs
    steps_c, dt_c = _stress_oracle_worker((cpu_n, 0))
    hbm, _, src = _peaks()
    alg = ALG_BYTES["step"] + ALG_BYTES["observe"] + 169 * 4 + p * (ALG_BYTES["astar"] + 2 * 169 * 4)
    return {"metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 sim", "data": "synthetic (seeded bomb-stress states)",
            "config": {"workload": CFG["workload"], "envs_per_gpu": n,
                       "l2": "flushed (256 MB write) before each timed step"},
            "e2e": None, "gpu_launches": (1 + 1 + 2 * p) * args.steps,
            "roofline": {"kernel": "stress tick", "bound": "hbm",
                         "achieved": round(alg * value / world / 1e9, 1), "peak": hbm,
                         "unit": "GB/s", "frac": round(alg * value / world / 1e9 / hbm, 4),
                         "peak_source": src, "traffic": None},
            "cpu_baseline": {"value": round(steps_c / dt_c, 1), "unit": UNIT, "cores": 1,
                             "kind": "port",
                             "sample": f"oracle, {cpu_n} envs x 1 stress tick"},
            "clocks": clk.summary()}


def _ncu_traffic(kernel):
    """DRAM bytes per launch from the committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(kernel)
    except Exception:
        return None


class RolloutDrawsPool:
    @staticmethod
    def make(dr, gen):
        import torch
        ts = [torch.empty_like(t) for t in dr.tensors()]
        for t in ts[:3]:
            t.uniform_(generator=gen)
        ts[3].random_(0, 2, generator=gen)
        ts[4].random_(60, 240, generator=gen)
        return ts

    @staticmethod
    def load(dr, ts):
        for dst, src in zip(dr.tensors(), ts):
            dst.copy_(src, non_blocking=True)


def reference_arm(args):
    """Time the CPU restatement of the reference tick (oracle/cpu_rollout.py)
    on every host core, on this arm's workload: one spawned process per
    core, each holding a shard of the GPU's envs (the whole shard for cfg2;
    512 envs per process for cfg4 and 64 for cfg5, whose full shards would
    take minutes per tick), warmed up 40 ticks into a bomb-rich mid-game
    state; every step then plays `--ref-ticks` ticks on all shards at once
    and is timed by the slowest shard.  cfg3 times the stress tick."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    procs = args.cpu_procs_ref or max(1, len(os.sched_getaffinity(0)))
    if args.config == "cfg3":
        return _reference_stress(args, procs)
    per = N_ENVS // procs if CFG["ref_per"] is None else min(CFG["ref_per"], N_ENVS // procs)
    from oracle.cpu_rollout import ShardPool
    pool = ShardPool(args.config, per, procs, seed=0, root=ROOT)
    try:
        for _ in range(args.warmup):
            pool.run(args.ref_ticks)
        vals = [pool.run(args.ref_ticks) for _ in range(args.steps)]
    finally:
        pool.close()
    steps = sum(s for s, _ in vals)
    dt = sum(d for _, d in vals)
    value = steps / dt
    sample = (f"oracle restatement of the reference tick, {procs} processes x {per} envs "
              f"({per * procs} of the {N_ENVS}-env shard), 40-tick warm-up, then "
              f"{args.warmup} untimed and {args.steps} timed steps of {args.ref_ticks} ticks")
    return {"impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": UNIT,
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 sim, f64 policy (numpy)", "data": "synthetic",
            "config": {"workload": CFG["workload"], "envs_per_gpu": N_ENVS,
                       "sample_envs": per * procs, "ticks_per_step": args.ref_ticks,
                       "warmup_ticks": 40},
            "cpu_baseline": {"value": round(value, 1), "unit": UNIT, "cores": procs,
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 1), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def _reference_stress(args, procs):
    import multiprocessing as mp
    per = max(1, N_ENVS // procs)
    ctx = mp.get_context("spawn")
    vals = []
    with ctx.Pool(procs) as pool:
        for i in range(args.warmup + args.steps):
            res = pool.map(_stress_oracle_worker, [(per, 100 * i + j) for j in range(procs)])
            if i >= args.warmup:
                vals.append((sum(r[0] for r in res), max(r[1] for r in res)))
    steps = sum(s for s, _ in vals)
    dt = sum(d for _, d in vals)
    value = steps / dt
    return {"impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": UNIT,
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 sim", "data": "synthetic",
            "config": {"workload": CFG["workload"], "envs_per_gpu": N_ENVS},
            "cpu_baseline": {"value": round(value, 1), "unit": UNIT, "cores": procs,
                             "kind": "port",
                             "sample": f"oracle stress tick, {procs} processes x {per} envs"},
            "e2e": {"value": round(value, 1), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


# ------------------------------------------------------- phase stamps

PHASES = {
    2: ("step (lane 0 of every warp of every 4th block)",
        [0, 16, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 18, 19, 20, 21, 22, 14, 15, 17],
        ["tile staging", "per-env set-up", "countdown + placement", "placement bonus",
         "movement", "chain explosion", "damage", "clearing + bomb list", "t / done",
         "rewards", "danger standing", "terminal rewards", "outputs", "device reset",
         "danger paint", "observation: player info", "observation: zero row",
         "observation: channels", "observation: row out", "legal masks", "player stores",
         "barrier + write-back"], True),
    3: ("astar bot (lane 0 of every warp of every 4th block)",
        [0, 1, 2, 3, 4],
        ["tile staging", "field set-up", "relaxation (V_safe, V_opp)", "scoring + bomb rule"],
        True),
    1: ("MLP policy, epilogue warp 2 (one record per CTA)",
        [0, 1, 7, 8, 9, 10, 11, 12, 13, 14],
        ["set-up (barriers, TMEM)", "layer 1 (wait for its MMAs)", "LN1 + operand",
         "layer-2 MMAs", "LN2 + operand", "head MMAs", "output layers",
         "logit reduce + sampling", "exit"], False),
    # the same kernel's producer (thread 0) and MMA-issuer stamps
    11: ("MLP policy, layer-1 producer / MMA issuer (one record per CTA)",
         [0, 1, 2, 3, 4, 5],
         ["set-up (barriers, TMEM, K-tile flags)", "first TMA issued", "rest of the TMAs issued",
          "last MMAs issued", "last MMAs complete"], False, 1),
}


def phase_table(rec, kid):
    """Per-phase durations (us) of kernel `kid` from phase-stamp records:
    the k-th record of a (block[, warp], phase) is that block's k-th launch."""
    import numpy as np
    title, order, names, by_warp = PHASES[kid][:4]
    kid = PHASES[kid][4] if len(PHASES[kid]) > 4 else kid
    w0 = rec[:, 0]
    t = rec[:, 1].astype(np.int64)
    k = (w0 >> np.uint64(56)).astype(np.int64)
    ph = ((w0 >> np.uint64(48)) & np.uint64(0xff)).astype(np.int64)
    blk = ((w0 >> np.uint64(8)) & np.uint64(0xffffff)).astype(np.int64)
    wp = (w0 & np.uint64(0xff)).astype(np.int64)
    key = blk * 64 + wp if by_warp else blk
    cols = []
    for p in order:
        m = (k == kid) & (ph == p)
        kk, tt = key[m], t[m]
        o = np.lexsort((tt, kk))
        kk, tt = kk[o], tt[o]
        start = np.r_[0, np.flatnonzero(kk[1:] != kk[:-1]) + 1]
        occ = np.arange(len(kk)) - np.repeat(start, np.diff(np.r_[start, len(kk)]))
        cols.append(dict(zip(zip(kk.tolist(), occ.tolist()), tt.tolist())))
    common = set(cols[0])
    for c in cols[1:]:
        common &= set(c)
    if not common:
        return [f"{title}: no records"]
    keys = sorted(common)
    T = np.array([[c[x] for c in cols] for x in keys], dtype=np.int64)
    D = np.diff(T, axis=1) / 1000.0
    tot = (T[:, -1] - T[:, 0]) / 1000.0
    out = [f"{title}: {len(keys)} samples, total mean {tot.mean():.2f} us, "
           f"p50 {np.median(tot):.2f}, p95 {np.percentile(tot, 95):.2f}"]
    for j, nm in enumerate(names):
        out.append(f"  {nm:36s} mean {D[:, j].mean():6.2f}  p50 {np.median(D[:, j]):6.2f}"
                   f"  p95 {np.percentile(D[:, j], 95):6.2f}")
    return out


def launch_spans(rec, kid, p_start, p_end, by_warp):
    """(first start, last start, last end) in ns of every launch of kernel
    `kid` from phase-stamp records: the k-th record of a block (or warp) at
    phase p_start / p_end belongs to that block's k-th launch."""
    import numpy as np
    w0 = rec[:, 0]
    t = rec[:, 1].astype(np.int64)
    k = (w0 >> np.uint64(56)).astype(np.int64)
    ph = ((w0 >> np.uint64(48)) & np.uint64(0xff)).astype(np.int64)
    blk = ((w0 >> np.uint64(8)) & np.uint64(0xffffff)).astype(np.int64)
    key = blk * 64 + (w0 & np.uint64(0xff)).astype(np.int64) if by_warp else blk
    occ_t = {}
    for p in (p_start, p_end):
        m = (k == kid) & (ph == p)
        kk, tt = key[m], t[m]
        o = np.lexsort((tt, kk))
        kk, tt = kk[o], tt[o]
        start = np.r_[0, np.flatnonzero(kk[1:] != kk[:-1]) + 1]
        occ = np.arange(len(kk)) - np.repeat(start, np.diff(np.r_[start, len(kk)]))
        for oc in np.unique(occ):
            occ_t.setdefault(int(oc), {})[p] = tt[occ == oc]
    out = [(v[p_start].min(), v[p_start].max(), v[p_end].max())
           for _, v in sorted(occ_t.items()) if p_start in v and p_end in v]
    return np.array(out, dtype=np.int64).reshape(-1, 3)


def relax_histogram(rec):
    """The astar relaxation's sweep-phase counts (stamp ids 40 + n)."""
    import numpy as np
    w0 = rec[:, 0]
    k = (w0 >> np.uint64(56)).astype(np.int64)
    ph = ((w0 >> np.uint64(48)) & np.uint64(0xff)).astype(np.int64)
    n = ph[(k == 3) & (ph >= 40)] - 40
    if len(n) == 0:
        return []
    vals, cnt = np.unique(n, return_counts=True)
    top = ", ".join(f"{v}: {c / len(n):.1%}" for v, c in zip(vals, cnt) if c / len(n) >= 0.01)
    return [f"astar relaxation sweep phases per env: mean {n.mean():.2f} ({top})"]


def chain_summary(rec):
    """How one tick's policy -> step chain lines up, from the launches'
    first / last block stamps: the gap from a step's end to the next policy
    start, how early the step's first blocks start before its policy ends
    (staging under programmatic launch), the step's end after its policy's,
    and each kernel's span and block start spread."""
    import numpy as np
    S = launch_spans(rec, 2, 0, 17, True)
    P = launch_spans(rec, 1, 0, 14, False)
    if len(S) == 0 or len(P) == 0:
        return ["chain: no step / policy launches recorded"]
    se = np.sort(S[:, 2])
    gap_sp = [p[0] - se[se <= p[0]][-1] for p in P if (se <= p[0]).any()]
    # a step's policy: the latest policy that ended after the step started
    early, after = [], []
    for s in S:
        cand = P[(P[:, 2] >= s[0]) & (P[:, 0] <= s[0])]
        if len(cand):
            pe = cand[:, 2].max()
            early.append(pe - s[0])
            after.append(s[2] - pe)
    f = lambda v: f"{np.mean(v) / 1e3:.2f}" if len(v) else "-"
    # what gates a step's start: its policy's layer 1 (the programmatic
    # trigger, stamp 5 of the last CTA) or the bot of the same tick (the
    # latest astar launch that ended before the step started)
    L1 = launch_spans(rec, 1, 0, 5, False)
    A = launch_spans(rec, 3, 0, 4, True)
    after_l1, after_bot, bot_vs_pol = [], [], []
    for s in S:
        cand = L1[(L1[:, 2] <= s[0])]
        if len(cand):
            after_l1.append(s[0] - cand[:, 2].max())
        ab = A[A[:, 2] <= s[0]]
        if len(ab):
            after_bot.append(s[0] - ab[:, 2].max())
    for a in A:
        cand = P[np.abs(P[:, 0] - a[0]) < 15000]
        if len(cand):
            bot_vs_pol.append(a[2] - cand[np.argmin(np.abs(cand[:, 0] - a[0])), 0])
    return [
        f"chain: step end -> next policy start {f(gap_sp)} us; step's first block starts "
        f"{f(early)} us before its policy ends; step ends {f(after)} us after it",
        f"  step launch span {f(S[:, 2] - S[:, 0])} us (block start spread {f(S[:, 1] - S[:, 0])}); "
        f"policy span {f(P[:, 2] - P[:, 0])} us (CTA start spread {f(P[:, 1] - P[:, 0])})",
        f"  a step's first block starts {f(after_l1)} us after its policy's layer 1 ends and "
        f"{f(after_bot)} us after the latest bot launch ended; a bot launch ends "
        f"{f(bot_vs_pol)} us after the policy launch nearest its start began "
        f"(bot span {f(A[:, 2] - A[:, 0])} us)"]


def phase_stamps_leg(args):
    """Per-phase durations of the step and policy kernels, from the
    phase-stamp build of the library (build.py --phase-stamps): one captured
    rollout of the configured workload after warm-up replays, then 20 policy
    launches of one env group alone.  Prints tables, no JSON line."""
    import ctypes
    import numpy as np
    import torch
    from qqt_b200 import _capi
    _capi.LIB_PATH = os.path.join(os.path.dirname(_capi.LIB_PATH), "libqqt_b200_phase.so")
    L = _capi.lib()
    cap = 8_000_000

    def read():
        buf = np.zeros((cap, 2), np.uint64)
        n = ctypes.c_uint32(0)
        _capi.check(L.qqt_phase_read(buf.ctypes.data, cap, ctypes.byref(n)), "qqt_phase_read")
        return buf[: n.value]

    torch.cuda.set_device(0)
    grp, gen = build_engine("cuda:0", 0, args.slots, 1 if CFG["ppo"] else args.groups)
    for ro in grp.ros:
        ro.draws.generate(gen)
        ro.tick(0)
    grp.collect()
    grp.capture()
    for _ in range(3):
        for ro in grp.ros:
            ro.draws.generate(gen)
        grp.replay()
    for ro in grp.ros:
        ro.draws.generate(gen)
    torch.cuda.synchronize()
    _capi.check(L.qqt_phase_reset(), "qqt_phase_reset")
    grp.replay()
    torch.cuda.synchronize()
    rec = read()
    lines = [f"phase stamps, {args.config}: {N_ENVS} envs per GPU in {len(grp.ros)} group(s), "
             f"one {TICKS}-tick rollout replay ({len(rec)} records)"]
    for kid in (2, 3, 1, 11):
        lines += phase_table(rec, kid)
    lines += relax_histogram(rec)
    lines += chain_summary(rec)
    ro = grp.ros[0]
    b = 5 % ro.slots
    obs, mm, bm, acts = ro.buf.obs(b), ro.buf.mm[b], ro.buf.bm[b], ro.buf.act[b]
    seats = list(ro.seats)
    for tiles in (ro.buf.tiles[b], None):
        pol = lambda: ro.learner.act_seats(obs, [mm[:, s] for s in seats],
                                           [bm[:, s] for s in seats], ro.draws.u_net[b],
                                           [acts[:, s] for s in seats], ro.buf.logp[b],
                                           ro.buf.val[b], obs_tiles=tiles)
        for _ in range(5):
            pol()
        torch.cuda.synchronize()
        _capi.check(L.qqt_phase_reset(), "qqt_phase_reset")
        for _ in range(20):
            pol()
            torch.cuda.synchronize()
        lines.append(f"policy alone: 20 launches over one group's {ro.sim.num_envs} envs, "
                     + ("with" if tiles is not None else "without") + " the rows' K-tile flags")
        rec = read()
        lines += phase_table(rec, 1)
        lines += phase_table(rec, 11)
    print("\n".join(lines), file=sys.stderr)


def main():
    # exactly one line on stdout: libraries (NCCL's version banner, ...) print
    # to file descriptor 1, so it points at stderr and the JSON line goes to a
    # saved copy of the original stdout
    json_fd = os.dup(1)
    sys.stdout.flush()
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="cfg2", choices=sorted(CONFIGS))
    ap.add_argument("--cpu-envs", type=int, default=0,
                    help="CPU baseline envs per process (0: per config)")
    ap.add_argument("--cpu-ticks", type=int, default=0,
                    help="CPU baseline timed ticks after the warm-up (0: per config)")
    ap.add_argument("--cpu-procs", type=int, default=1)
    ap.add_argument("--cpu-procs-ref", type=int, default=0)
    ap.add_argument("--ref-ticks", type=int, default=4)
    ap.add_argument("--envs", type=int, default=0, help="envs per GPU (profiling cases)")
    ap.add_argument("--ticks", type=int, default=128, help="ticks per rollout (multiple of 16)")
    ap.add_argument("--groups", type=int, default=2,
                    help="independent env groups per GPU, each on its own stream")
    ap.add_argument("--slots", type=int, default=0,
                    help="rollout-buffer slots (0 = one per tick; fewer = ring, profiling only)")
    ap.add_argument("--phase-stamps", action="store_true",
                    help="print per-phase kernel durations from the phase-stamp build "
                         "(build.py --phase-stamps) instead of the JSON line")
    args = ap.parse_args()
    global CFG, N_ENVS, TICKS
    CFG = CONFIGS[args.config]
    N_ENVS, TICKS = args.envs or CFG["envs"], args.ticks
    args.cpu_envs = args.cpu_envs or CFG["cpu"][0]
    args.cpu_ticks = args.cpu_ticks or CFG["cpu"][1]
    if TICKS % 16:
        raise SystemExit("--ticks must be a multiple of 16")
    if args.phase_stamps:
        phase_stamps_leg(args)
        out = None
    elif args.impl == "reference":
        out = reference_arm(args)
    elif args.config == "cfg3":
        out = stress_bench(args)
    else:
        out = gpu_bench(args)
    if out is not None:
        os.write(json_fd, (json.dumps(out) + "\n").encode())
    os.close(json_fd)


if __name__ == "__main__":
    main()
