#!/usr/bin/env python3
"""Time the reference's own eager-torch CPU rollout tick against the oracle
port (oracle/cpu_rollout.py) on the same workload and machine --
BASELINE INFRASTRUCTURE ONLY, run where the reference source tree exists
(it is imported, not copied):

    python oracle/time_reference.py --ref /path/to/qqt-gpu-sim [--envs 5632]

The GPU box cannot import the reference, so bench.py's CPU legs time the
port; this script ties the port's speed to the reference's own.

Workload (cfg2): the pillar-corridor template, a random-init MLP learner on
seat 0 (ActorCritic.act, the reference's Categorical sampling) against the
reference's astar bot (make_bot, mode ticker on) on seat 1, step with
auto-reset, flush_recycle every 16 ticks -- the collect tick of
train/ppo.py:213-271.  Both sides play a 40-tick warm-up into a bomb-rich
mid-game state and then time `--ticks` ticks.  The reference runs in one
process with torch using every core; the port runs one process per core,
each holding an equal shard of the envs.  One JSON line per measurement.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path[:0] = [REPO, os.path.join(REPO, "qqt-gpu-sim_b200"), os.path.join(REPO, "tests", "golden")]


def time_reference(ref_root, n, warm, ticks, threads):
    import torch
    from make_golden import load_params, load_reference, set_state
    from qqt_b200 import scenarios
    from qqt_b200.policy_init import init_params
    R = load_reference(ref_root)
    torch.set_num_threads(threads)
    ts, rbots = R["ts"], R["bots"]
    cfg = R["SimConfig"](map_mode="corridor", open_fraction=0.0, speed=3.0, max_steps=1800)
    h, w, p = cfg.height, cfg.width, cfg.n_players
    sim = ts.BatchedSim(cfg, n, device="cpu", seed=1)
    wall, brick = scenarios.pillar_corridor(n, h, w, seed=1)
    set_state(sim, {"wall": wall, "brick": brick})
    sp = np.array(scenarios.corner_spawns(cfg), dtype=np.float32)
    sim.pos.copy_(torch.from_numpy(np.broadcast_to(sp, (n, p, 2)).copy()))
    model = R["ActorCritic"](cfg.obs_shape, arch="mlp")
    load_params(model, init_params(cfg.obs_shape, arch="mlp", seed=1))
    model.eval()
    bot = rbots.make_bot(sim, "astar")
    stage = {"observe+mask": 0.0, "learner": 0.0, "astar": 0.0, "step+flush": 0.0}

    def tick(i, timed):
        t0 = time.perf_counter()
        obs = sim.observe()
        mm, bm = sim.legal_mask()
        t1 = time.perf_counter()
        acts = torch.zeros((n, p, 2), dtype=torch.long)
        with torch.no_grad():
            a0, _, _ = model.act(obs, mm[:, 0], bm[:, 0], 0)
        acts[:, 0] = a0
        t2 = time.perf_counter()
        acts[:, 1] = bot.act(obs, mm[:, 1], bm[:, 1], 1)
        t3 = time.perf_counter()
        sim.step(acts)
        if i % 16 == 15:
            sim.flush_recycle()
        t4 = time.perf_counter()
        if timed:
            for k, dt in zip(stage, (t1 - t0, t2 - t1, t3 - t2, t4 - t3)):
                stage[k] += dt

    for i in range(warm):
        tick(i, False)
    t0 = time.perf_counter()
    for i in range(warm, warm + ticks):
        tick(i, True)
    dt = time.perf_counter() - t0
    return {"impl": "reference eager torch (CPU)", "envs": n, "threads": threads,
            "warmup_ticks": warm, "ticks": ticks, "seconds": round(dt, 3),
            "env_steps_per_s": round(n * ticks / dt, 1),
            "stage_share": {k: round(v / dt, 3) for k, v in stage.items()}}


def time_port(n, warm, ticks, procs):
    from oracle.cpu_rollout import ShardPool
    pool = ShardPool("cfg2", n // procs, procs, seed=0, warm=warm, root=REPO)
    try:
        steps, dt = pool.run(ticks)
    finally:
        pool.close()
    return {"impl": "oracle port (numpy)", "envs": steps // ticks, "processes": procs,
            "warmup_ticks": warm, "ticks": ticks, "seconds": round(dt, 3),
            "env_steps_per_s": round(steps / dt, 1)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="root of the reference source tree")
    ap.add_argument("--envs", type=int, default=5632)
    ap.add_argument("--warm", type=int, default=40)
    ap.add_argument("--ticks", type=int, default=16)
    args = ap.parse_args()
    cores = len(os.sched_getaffinity(0))
    print(json.dumps(time_port(args.envs, args.warm, args.ticks, cores)), flush=True)
    print(json.dumps(time_port(args.envs // cores, args.warm, args.ticks, 1)), flush=True)
    print(json.dumps(time_reference(args.ref, args.envs, args.warm, args.ticks, cores)),
          flush=True)
    print(json.dumps(time_reference(args.ref, args.envs // cores, args.warm, args.ticks, 1)),
          flush=True)


if __name__ == "__main__":
    main()
