#!/usr/bin/env python3
"""Generate golden vectors by running the reference implementation itself.

Run in a container that holds the reference source tree (it is imported, not
copied):

    python tests/golden/make_golden.py --ref /path/to/qqt-gpu-sim

Two import shims are applied before the reference loads: `triton` is blocked
so movement uses the eager torch path, and the missing `sim.dev.synchronize`
that `train/ppo.py` imports is provided.  Every random draw the rollout makes
(bot samplers and noise, mode-ticker integers, crate-pickup uniforms, learner
sampling uniforms) is fed from a recorded numpy stream, so the oracle and the
CUDA engine can replay the same trajectory.

Outputs (compressed npz, all env-major like the reference tensors):
  kat_states.npz   the reference's own known-answer states
                   (deploy/ref_state.json, deploy/sweep_states.json) with
                   their danger / obs / masks / covered / triggered
  traj_cfg1.npz    open border map, random bots p=0.05, 256 ticks
  traj_cfg2.npz    pillar corridor, MLP learner vs astar, 128 ticks
  traj_cfg4.npz    pillar corridor, self-play MLP (both seats), 64 ticks
  traj_cfg5.npz    pillar corridor, CNN learner vs greedy, 48 ticks
  traj_hunter.npz  pillar corridor with bricks p=0.3 and crates on 12 % of the
                   free cells, MLP learner vs the hunter bot (astar with the
                   crate layer), 128 ticks, with V_crate fields
  stress_cfg3.npz  bomb stress: one idle step, danger/obs/masks, V fields
  hazard_wave.npz  the reference's hazard-wave placement on seeded states,
                   its draws fed from the engine's keyed generator
  ckpt_adapt.npz   adapt_first_conv on seeded models (2 <-> 3 players), and
  ref_ckpt_mlp.pt  a checkpoint written by the reference's save_ckpt
  ckpt_adapt_lstm.npz  adapt_first_conv on the LSTM architecture
  mapgen_fed.npz   per-episode level generation (reset_) with recorded draws
  danger_walls.npz danger map and chain resolution with bombs on wall cells
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from functools import partial

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "qqt-gpu-sim_b200"))

from qqt_b200 import scenarios  # noqa: E402
from qqt_b200.policy_init import init_params  # noqa: E402


def load_reference(ref_root):
    sys.modules["triton"] = None
    sys.path.insert(0, ref_root)
    import torch  # noqa: F401
    import sim.dev
    sim.dev.synchronize = lambda *a, **k: None
    import sim.bots as rbots
    import sim.torch_sim as rts
    from sim.blast import danger_map, resolve_explosions
    from sim.config import SimConfig
    from sim.obs import encode_obs, legal_mask
    from train.model import ActorCritic
    return dict(bots=rbots, ts=rts, SimConfig=SimConfig, danger_map=danger_map,
                resolve=resolve_explosions, encode_obs=encode_obs,
                legal_mask=legal_mask, ActorCritic=ActorCritic, root=ref_root)


class FedTorch:
    """Stand-in for the `torch` module inside sim/bots.py: rand/randint come
    from a numpy stream and are recorded in call order."""

    def __init__(self, real, rng):
        self._real = real
        self._rng = rng
        self.log = []

    def rand(self, *size, device=None, **kw):
        shape = size[0] if len(size) == 1 and isinstance(size[0], tuple) else size
        v = self._rng.random(shape).astype(np.float32)
        self.log.append(("rand", v))
        return self._real.from_numpy(v)

    def randint(self, low, high, size, device=None, **kw):
        v = self._rng.integers(low, high, size=size).astype(np.int64)
        self.log.append(("randint", v))
        return self._real.from_numpy(v)

    def __getattr__(self, name):
        return getattr(self._real, name)


def state_np(sim):
    import torch
    out = {}
    names = {"wall": "wall", "brick": "brick", "crate": "crate",
             "recycle": "_recycle_crate", "fuse": "fuse", "owner": "owner",
             "bomb_blast": "bomb_blast", "pos": "pos", "alive": "alive",
             "hp": "hp", "since_bomb": "since_bomb", "t": "t",
             "bombs_cap": "bombs_cap", "blast_cap": "blast_cap", "spd_g": "spd_g",
             "invuln": "invuln", "pending_lost": "_pending_lost", "combo": "_combo",
             "last_hit": "_last_hit", "lo_bombs": "_lo_bombs", "lo_blast": "_lo_blast",
             "lo_spd": "_lo_spd", "crate_prob": "crate_prob", "hazard": "_hazard"}
    for k, attr in names.items():
        v = getattr(sim, attr)
        assert isinstance(v, torch.Tensor)
        out[k] = v.detach().cpu().numpy().copy()
    return out


def set_state(sim, st):
    import torch
    names = {"wall": "wall", "brick": "brick", "crate": "crate",
             "recycle": "_recycle_crate", "fuse": "fuse", "owner": "owner",
             "bomb_blast": "bomb_blast", "pos": "pos"}
    for k, attr in names.items():
        if k in st:
            getattr(sim, attr).copy_(torch.from_numpy(np.asarray(st[k])))


def load_params(model, params):
    import torch
    sd = model.state_dict()
    for k in sd:
        sd[k] = torch.from_numpy(params[k])
    model.load_state_dict(sd)


def masked_sample_np(logits, mask, u):
    z = np.where(mask, logits.astype(np.float64), np.finfo(np.float32).min)
    m = z.max(-1, keepdims=True)
    e = np.exp(z - m)
    cs = np.cumsum(e, -1)
    s = cs[:, -1:]
    a = np.minimum(((u[:, None] * s) > cs).sum(-1), z.shape[-1] - 1)
    logp = np.take_along_axis(z, a[:, None], 1)[:, 0] - m[:, 0] - np.log(s[:, 0])
    return a.astype(np.int64), logp


def rollout(R, cfg, n, ticks, seed, template, learner_arch, opp_kind, rng_seed,
            obs_every=4, bomb_rate=0.05):
    import torch
    torch.set_num_threads(4)
    ts, rbots = R["ts"], R["bots"]
    rng = np.random.default_rng(rng_seed)
    fed = FedTorch(torch, rng)
    rbots.torch = fed
    h, w, p = cfg.height, cfg.width, cfg.n_players
    border = scenarios.border_walls(h, w)
    orig_open = ts.make_open_obstacles
    if template == "open_border":
        ts.make_open_obstacles = lambda c, count, gen, dev: \
            torch.from_numpy(np.broadcast_to(border, (count, h, w)).copy())
    try:
        sim = ts.BatchedSim(cfg, n, device="cpu", seed=seed)
        if template in ("corridor", "sparse_crates"):
            bp = 0.7 if template == "corridor" else 0.3
            wall, brick = scenarios.pillar_corridor(n, h, w, seed=seed, brick_p=bp)
            st0 = {"wall": wall, "brick": brick}
            if template == "sparse_crates":
                # crates on 12 % of the free cells (corner L cells kept clear),
                # so that the hunter's crate layer has targets it can reach
                keep = np.zeros((h, w), bool)
                for r, c in scenarios.corner_l_cells(h, w):
                    keep[r, c] = True
                crng = np.random.default_rng(seed + 100)
                st0["crate"] = ~wall & ~brick & ~keep[None] & (crng.random(wall.shape) < 0.12)
            set_state(sim, st0)
            sp = np.array(scenarios.corner_spawns(cfg), dtype=np.float32)
            sim.pos.copy_(torch.from_numpy(np.broadcast_to(sp, (n, p, 2)).copy()))
        init = state_np(sim)
        models = {}
        seats = []
        if learner_arch is not None:
            m = R["ActorCritic"](cfg.obs_shape, arch=learner_arch)
            params = init_params(cfg.obs_shape, arch=learner_arch, seed=seed)
            load_params(m, params)
            m.eval()
            models[0] = m
            seats.append(("net", 0))
        else:
            seats.append(("bot", 0))
        if opp_kind == "self":
            models[1] = models[0]
            seats.append(("net", 1))
        else:
            seats.append(("bot", 1))
        bots = {}
        for kind, pid in seats:
            if kind == "bot":
                kname = opp_kind if pid == 1 else "random"
                if kname == "random":
                    bots[pid] = rbots.BotWrapper(
                        sim, partial(rbots.random_attack, bomb_rate=bomb_rate), "random")
                else:
                    bots[pid] = rbots.make_bot(sim, kname)
        rec = {k: [] for k in ("mm", "bm", "actions", "reward", "done", "winner",
                               "rb_hit", "rb_grow", "u_net", "logits_m", "logits_b",
                               "value", "logp", "draws_kind", "state", "n_alive")}
        obs_ticks, obs_rec, dng_rec = [], [], []
        reset_rec, flush_rec = [], []
        fields_rec = []
        vcrate_rec = []
        bot_draws = []
        for t in range(ticks):
            obs = sim.observe()
            mm, bm = sim.legal_mask()
            if t % obs_every == 0:
                obs_ticks.append(t)
                obs_rec.append(obs.numpy().copy())
                dng_rec.append(sim._dng_cache.numpy().copy() if sim._dng_cache is not None
                               else np.zeros((n, h, w), np.float32))
            acts = torch.zeros((n, p, 2), dtype=torch.long)
            u_net = np.zeros((n, p, 2), dtype=np.float64)
            lm = np.zeros((n, p, 5), np.float32)
            lb = np.zeros((n, p, 2), np.float32)
            val = np.zeros((n, p), np.float32)
            lp = np.zeros((n, p), np.float64)
            tick_draws = {}
            for kind, pid in seats:
                if kind == "net":
                    with torch.no_grad():
                        ml, bl, v = models[pid](obs, pid)
                    u = rng.random((n, 2))
                    u_net[:, pid] = u
                    am, l1 = masked_sample_np(ml.numpy(), mm[:, pid].numpy(), u[:, 0])
                    ab, l2 = masked_sample_np(bl.numpy(), bm[:, pid].numpy(), u[:, 1])
                    acts[:, pid, 0] = torch.from_numpy(am)
                    acts[:, pid, 1] = torch.from_numpy(ab)
                    lm[:, pid], lb[:, pid], val[:, pid] = ml.numpy(), bl.numpy(), v.numpy()
                    lp[:, pid] = l1 + l2
                else:
                    fed.log.clear()
                    a = bots[pid].act(obs, mm[:, pid], bm[:, pid], pid)
                    acts[:, pid] = a
                    tick_draws[pid] = list(fed.log)
            bot_draws.append(tick_draws)
            if opp_kind in ("astar", "hunter") and t % 8 == 0:
                dng = obs.float()[:, 2 * p + 1]
                blk = sim.wall | sim.brick | (sim.fuse > 0)
                vs = rbots._dijkstra_field(sim, dng < 0.35, dng, blocked=blk)
                src = torch.zeros(n, h, w, dtype=torch.bool)
                r0 = sim.pos[:, 0, 0].floor().long().clamp(0, h - 1)
                c0 = sim.pos[:, 0, 1].floor().long().clamp(0, w - 1)
                src.view(n, -1)[torch.arange(n), r0 * w + c0] = sim.alive[:, 0]
                vo = rbots._dijkstra_field(sim, src, dng, blocked=blk)
                fields_rec.append((t, vs.numpy().copy(), vo.numpy().copy()))
                if opp_kind == "hunter":
                    vc = rbots._dijkstra_field(sim, sim.crate, dng, blocked=blk)
                    vcrate_rec.append(vc.numpy().copy())
            rb = rng.random((2, n, p)).astype(np.float32)
            buf = np.zeros(n * (2 * p + 1), dtype=np.float32)
            buf[: n * p] = rb[0].reshape(-1)
            buf[n * p: 2 * n * p] = rb[1].reshape(-1)
            sim._rand_buf = torch.from_numpy(buf)
            r, d, info = sim.step(acts, auto_reset=False)
            rec["mm"].append(mm.numpy().copy())
            rec["bm"].append(bm.numpy().copy())
            rec["actions"].append(acts.numpy().copy())
            rec["reward"].append(r.numpy().copy())
            rec["done"].append(d.numpy().copy())
            rec["winner"].append(info["winner"].numpy().copy())
            rec["n_alive"].append(info["n_alive"].numpy().copy())
            rec["rb_hit"].append(rb[0])
            rec["rb_grow"].append(rb[1])
            rec["u_net"].append(u_net)
            rec["logits_m"].append(lm)
            rec["logits_b"].append(lb)
            rec["value"].append(val)
            rec["logp"].append(lp)
            rec["state"].append(state_np(sim))
            if bool(d.any()):
                sim.reset_(d)
                reset_rec.append((t, state_np(sim)))
            if t % 16 == 15:
                gstate = sim.gen.get_state().numpy().copy()
                sim.flush_recycle()
                flush_rec.append((t, gstate, state_np(sim)))
    finally:
        ts.make_open_obstacles = orig_open
        rbots.torch = torch
    out = {"init_" + k: v for k, v in init.items()}
    for k in ("mm", "bm", "actions", "reward", "done", "winner", "rb_hit", "rb_grow",
              "u_net", "logits_m", "logits_b", "value", "logp", "n_alive"):
        out[k] = np.stack(rec[k])
    skeys = [k for k in rec["state"][0] if k != "wall"]
    for k in skeys:
        out["st_" + k] = np.stack([s[k] for s in rec["state"]])
    out["obs_ticks"] = np.array(obs_ticks)
    out["obs"] = np.stack(obs_rec)
    out["danger"] = np.stack(dng_rec)
    out["reset_ticks"] = np.array([t for t, _ in reset_rec], dtype=np.int64)
    for i, (t, s) in enumerate(reset_rec):
        for k in skeys:
            out[f"reset{i}_{k}"] = s[k]
    out["flush_ticks"] = np.array([t for t, _, _ in flush_rec], dtype=np.int64)
    for i, (t, g, s) in enumerate(flush_rec):
        out[f"flush{i}_gen"] = g
        for k in ("crate", "recycle", "pending_lost"):
            out[f"flush{i}_{k}"] = s[k]
    if fields_rec:
        out["field_ticks"] = np.array([t for t, _, _ in fields_rec])
        out["vsafe"] = np.stack([a for _, a, _ in fields_rec])
        out["vopp"] = np.stack([b for _, _, b in fields_rec])
    if vcrate_rec:
        out["vcrate"] = np.stack(vcrate_rec)
    # bot draws per tick and seat, flattened in call order
    for pid in (0, 1):
        kinds = []
        for t, td in enumerate(bot_draws):
            for j, (kind, v) in enumerate(td.get(pid, [])):
                out[f"draw_p{pid}_t{t}_{j}"] = v
                kinds.append((t, j, kind))
        if kinds:
            out[f"draw_p{pid}_index"] = np.array([[t, j, 0 if k == "rand" else 1]
                                                  for t, j, k in kinds], dtype=np.int64)
    return out


def kat_states(R, ref_root):
    import torch
    cfg = R["SimConfig"](height=13, width=13, n_players=2, map_mode="corridor",
                         speed=3.0, max_steps=1800, obs_extra_enabled=True, obs_fp16=False)
    with open(os.path.join(ref_root, "deploy", "ref_state.json")) as f:
        states = [json.load(f)]
    with open(os.path.join(ref_root, "deploy", "sweep_states.json")) as f:
        states += json.load(f)["states"]
    h, w = 13, 13
    keys = ("wall", "brick", "fuse", "owner", "bomb_blast", "crate")
    dt = {"wall": bool, "brick": bool, "crate": bool, "fuse": np.int16,
          "owner": np.int8, "bomb_blast": np.int16}
    out = {k: [] for k in keys + ("pos", "alive", "t", "invuln", "bombs_cap",
                                 "blast_cap", "danger", "obs", "mm", "bm",
                                 "covered", "triggered")}
    for s in states:
        st = s["state"]
        for k in keys:
            out[k].append(np.array(st[k], dtype=dt[k]).reshape(h, w))
        out["pos"].append(np.array(st["pos"], np.float32).reshape(2, 2))
        out["alive"].append(np.array(st["alive"], bool))
        out["t"].append(st["t"])
        out["invuln"].append(np.array(st["invuln"], np.int64))
        out["bombs_cap"].append(np.array(st["bombs_cap"], np.int64))
        out["blast_cap"].append(np.array(st["blast_cap"], np.int64))
        # recompute with the reference and check it against the stored answer
        T = {k: torch.from_numpy(out[k][-1][None]) for k in keys}
        bmap = torch.where(T["bomb_blast"] > 0, T["bomb_blast"].long(), cfg.blast)
        dng = R["danger_map"](T["fuse"], T["wall"], bmap, cfg.fuse, T["brick"], cfg.max_chain)
        pos = torch.from_numpy(out["pos"][-1][None])
        alive = torch.from_numpy(out["alive"][-1][None])
        tt = torch.tensor([st["t"]])
        inv = torch.from_numpy(out["invuln"][-1][None])
        bp = torch.from_numpy(out["bombs_cap"][-1][None])
        obs = R["encode_obs"](cfg, T["wall"], T["fuse"], T["owner"], pos, alive, tt,
                              T["brick"], T["bomb_blast"], T["crate"], inv, bp,
                              danger_precomputed=dng)
        mm, bm = R["legal_mask"](cfg, T["wall"], T["fuse"], T["owner"], pos, alive,
                                 T["brick"], bp)
        cov, trig = R["resolve"](T["fuse"], T["owner"], T["wall"], bmap, cfg.max_chain,
                                 T["brick"])
        assert np.array_equal(np.array(s["danger"], np.float32), dng[0].numpy().reshape(-1))
        assert np.array_equal(np.array(s["obs"], np.float32), obs[0].numpy().reshape(-1))
        assert np.array_equal(np.array(s["mm"], bool), mm[0].numpy())
        assert np.array_equal(np.array(s["covered"], bool), cov[0].numpy().reshape(-1))
        out["danger"].append(dng[0].numpy())
        out["obs"].append(obs[0].numpy())
        out["mm"].append(mm[0].numpy())
        out["bm"].append(bm[0].numpy())
        out["covered"].append(cov[0].numpy())
        out["triggered"].append(trig[0].numpy())
    return {k: np.stack([np.asarray(x) for x in v]) for k, v in out.items()}


def danger_walls_golden(R):
    """The reference's danger_map and resolve_explosions (sim/blast.py:43-317)
    on seeded 13 x 13 states with interior walls and bricks and 10-24 bombs
    per env placed on any cell, walls included (a player standing on a wall
    cell can place a bomb there: an open map's obstacle may cover an open
    spawn), some of them going off this tick (fuse 0, owner set)."""
    import torch
    cfg = R["SimConfig"](height=13, width=13, n_players=2, map_mode="corridor", speed=3.0)
    n, h, w = 48, 13, 13
    rng = np.random.default_rng(77)
    wall = rng.random((n, h, w)) < 0.15
    brick = ~wall & (rng.random((n, h, w)) < 0.15)
    fuse = np.zeros((n, h, w), np.int16)
    owner = np.full((n, h, w), -1, np.int8)
    blast = np.zeros((n, h, w), np.int16)
    for e in range(n):
        k = int(rng.integers(10, 25))
        cells = rng.choice(h * w, size=k, replace=False)
        walled = np.flatnonzero(wall[e].reshape(-1))
        if walled.size:                        # at least two bombs on wall cells
            cells[:2] = rng.choice(walled, size=min(2, walled.size), replace=False)[:2] \
                if walled.size >= 2 else np.repeat(walled, 2)[:2]
        cells = np.unique(cells)
        fuse.reshape(n, -1)[e, cells] = rng.integers(0, 31, size=cells.size)
        owner.reshape(n, -1)[e, cells] = rng.integers(0, 2, size=cells.size)
        blast.reshape(n, -1)[e, cells] = rng.integers(1, 6, size=cells.size)
    T = {k: torch.from_numpy(v) for k, v in
         dict(wall=wall, brick=brick, fuse=fuse, owner=owner, bomb_blast=blast).items()}
    bmap = torch.where(T["bomb_blast"] > 0, T["bomb_blast"].long(), cfg.blast)
    dng = R["danger_map"](T["fuse"], T["wall"], bmap, cfg.fuse, T["brick"], cfg.max_chain)
    cov, trig = R["resolve"](T["fuse"], T["owner"], T["wall"], bmap, cfg.max_chain, T["brick"])
    return {"wall": wall, "brick": brick, "fuse": fuse, "owner": owner, "bomb_blast": blast,
            "danger": dng.numpy(), "covered": cov.numpy(), "triggered": trig.numpy(),
            "max_chain": np.int64(cfg.max_chain), "fuse_max": np.int64(cfg.fuse),
            "blast": np.int64(cfg.blast)}


def stress(R, cfg, n, seed):
    import torch
    ts, rbots = R["ts"], R["bots"]
    h, w, p = cfg.height, cfg.width, cfg.n_players
    border = scenarios.border_walls(h, w)
    orig_open = ts.make_open_obstacles
    ts.make_open_obstacles = lambda c, count, gen, dev: \
        torch.from_numpy(np.broadcast_to(border, (count, h, w)).copy())
    rng = np.random.default_rng(seed + 100)
    fed = FedTorch(torch, rng)
    rbots.torch = fed
    try:
        sim = ts.BatchedSim(cfg, n, device="cpu", seed=seed)
        fuse, owner, blast = scenarios.bomb_stress(n, cfg, seed)
        set_state(sim, {"fuse": fuse, "owner": owner, "bomb_blast": blast})
        sp = np.array(scenarios.open_spawns(cfg), dtype=np.float32)
        sim.pos.copy_(torch.from_numpy(np.broadcast_to(sp, (n, p, 2)).copy()))
        init = state_np(sim)
        acts = torch.zeros((n, p, 2), dtype=torch.long)
        acts[..., 0] = 4
        rb = rng.random((2, n, p)).astype(np.float32)
        buf = np.zeros(n * (2 * p + 1), dtype=np.float32)
        buf[: n * p] = rb[0].reshape(-1)
        buf[n * p: 2 * n * p] = rb[1].reshape(-1)
        sim._rand_buf = torch.from_numpy(buf)
        r, d, info = sim.step(acts, auto_reset=False)
        after = state_np(sim)
        obs = sim.observe()
        mm, bm = sim.legal_mask()
        dng = obs.float()[:, 2 * p + 1]
        blk = sim.wall | sim.brick | (sim.fuse > 0)
        out = {"init_" + k: v for k, v in init.items()}
        out.update({"after_" + k: v for k, v in after.items()})
        out.update(reward=r.numpy(), done=d.numpy(), covered=info["blast"].numpy(),
                   triggered=info["trig"].numpy(), obs=obs.numpy(), mm=mm.numpy(),
                   bm=bm.numpy(), rb_hit=rb[0], rb_grow=rb[1],
                   danger=sim._dng_cache.numpy())
        for pid in range(p):
            vs = rbots._dijkstra_field(sim, dng < 0.35, dng, blocked=blk)
            src = torch.zeros(n, h, w, dtype=torch.bool)
            o = 1 - pid
            ro = sim.pos[:, o, 0].floor().long().clamp(0, h - 1)
            co = sim.pos[:, o, 1].floor().long().clamp(0, w - 1)
            src.view(n, -1)[torch.arange(n), ro * w + co] = sim.alive[:, o]
            vo = rbots._dijkstra_field(sim, src, dng, blocked=blk)
            out[f"vsafe{pid}"] = vs.numpy()
            out[f"vopp{pid}"] = vo.numpy()
            fed.log.clear()
            a = rbots.astar_attack(sim, obs, mm[:, pid], bm[:, pid], pid)
            out[f"astar_act{pid}"] = a.numpy()
            out[f"astar_noise{pid}"] = fed.log[0][1]
    finally:
        ts.make_open_obstacles = orig_open
        rbots.torch = torch
    return out


RESET_CFGS = {
    "open_default": dict(),
    "open_obstacles": dict(open_obstacle_max=6, height=11, width=11),
    "corridor_default": dict(map_mode="corridor", speed=3.0, max_steps=1800),
    "corridor_dense": dict(map_mode="corridor", wall_density=0.45, random_wall_rows=False),
    "corridor_mixed": dict(map_mode="corridor", open_fraction=0.3, ring_fraction=0.3,
                           pure_open_fraction=0.1, wall_density=0.25, open_obstacle_max=3),
    "pillars_open": dict(wall_density=0.6, height=11, width=11),
}


def reset_modes(R):
    """Initial states of BatchedSim(cfg, 24, seed=999) plus a second reset_ of
    every other env, for several map modes (host generator parity)."""
    import torch
    out = {}
    for name, kw in RESET_CFGS.items():
        cfg = R["SimConfig"](**kw)
        sim = R["ts"].BatchedSim(cfg, 24, device="cpu", seed=999)
        for k, v in state_np(sim).items():
            out[f"{name}__init__{k}"] = v
        mask = torch.zeros(24, dtype=torch.bool)
        mask[::2] = True
        sim.reset_(mask)
        for k, v in state_np(sim).items():
            out[f"{name}__again__{k}"] = v
    return out


def ppo_golden(R):
    """compute_gae + one ppo_update (2 epochs x 2 minibatches) of the
    reference on a seeded 8-tick, 24-env buffer, minibatch permutations
    recorded."""
    import torch
    import train.ppo as rppo
    cfg = R["SimConfig"](**scenarios.CFG2)
    T, n = 8, 24
    rng = np.random.default_rng(21)
    shp = (T, n) + tuple(cfg.obs_shape)
    obs = (rng.random(shp) * (rng.random(shp) < 0.3)).astype(np.float16)
    mm = rng.random((T, n, 5)) < 0.8
    mm[..., 4] = True
    bm = rng.random((T, n, 2)) < 0.7
    bm[..., 0] = True
    model = R["ActorCritic"](cfg.obs_shape, arch="mlp")
    load_params(model, init_params(cfg.obs_shape, "mlp", seed=9))
    buf = rppo.RolloutBuffer(T, n, cfg.obs_shape, "cpu", obs_dtype=torch.float16, arch="mlp")
    with torch.no_grad():
        for t in range(T):
            o = torch.from_numpy(obs[t])
            ml, bl, v = model(o, 0)
            u = rng.random((n, 2))
            am, l1 = masked_sample_np(ml.numpy(), mm[t], u[:, 0])
            ab, l2 = masked_sample_np(bl.numpy(), bm[t], u[:, 1])
            buf.add(o, torch.from_numpy(mm[t]), torch.from_numpy(bm[t]),
                    torch.from_numpy(np.stack([am, ab], -1)),
                    torch.from_numpy((l1 + l2).astype(np.float32)), v,
                    torch.from_numpy(rng.normal(0, 0.5, n).astype(np.float32)),
                    torch.from_numpy((rng.random(n) < 0.05).astype(np.float32)),
                    torch.from_numpy(rng.random(n) < 0.1))
    last_val = torch.from_numpy(rng.normal(0, 0.3, n).astype(np.float32))
    adv, ret = rppo.compute_gae(buf, last_val, 0.995, 0.95)
    pcfg = rppo.PPOConfig(epochs=2, minibatches=2, lr=1e-4)
    opt = torch.optim.Adam(model.parameters(), lr=1e-4, eps=1e-5)
    perms = []
    real = rppo.torch

    class PermTorch:
        def randperm(self, k, device=None, **kw):
            p = torch.from_numpy(rng.permutation(k).astype(np.int64))
            perms.append(p.numpy().copy())
            return p

        def __getattr__(self, name):
            return getattr(real, name)

    rppo.torch = PermTorch()
    try:
        stats = rppo.ppo_update(model, opt, buf, last_val, pcfg, entropy_coef=0.03)
    finally:
        rppo.torch = real
    out = {"obs": obs, "mm": mm, "bm": bm, "act": buf.act.numpy(), "logp": buf.logp.numpy(),
           "val": buf.val.numpy(), "rew": buf.rew.numpy(), "done": buf.done.numpy(),
           "dmg": buf.dmg.numpy(), "last_val": last_val.numpy(), "adv": adv.numpy(),
           "ret": ret.numpy(), "n_perms": np.array(len(perms)),
           "stats": np.array([stats[k] for k in ("pg", "vf", "ent", "kl", "clipfrac")])}
    for i, p in enumerate(perms):
        out[f"perm{i}"] = p
    for k, v in model.state_dict().items():
        out["param__" + k] = v.numpy().copy()
    return out


def ckpt_golden(R):
    """Checkpoint format and first-layer migration (train/train.py:92-158,
    243-260, 307-331): the reference's adapt_first_conv on seeded random
    models (3x3 grid, 2 <-> 3 players, mlp and cnn), and one checkpoint
    written by the reference's own save_ckpt (saved beside this file as
    ref_ckpt_mlp.pt)."""
    import argparse as _ap
    import torch
    from sim.config import n_obs_channels
    from train.curriculum import CurriculumState
    from train.model_pool import ModelPool
    from train.train import adapt_first_conv, save_ckpt
    AC = R["ActorCritic"]
    out = {}
    seed = 0
    for arch in ("mlp", "cnn"):
        for p_old, p_new in ((2, 3), (3, 2)):
            torch.manual_seed(100 + seed)
            seed += 1
            old_shape = (n_obs_channels(p_old), 3, 3)
            new_shape = (n_obs_channels(p_new), 3, 3)
            m = AC(old_shape, arch=arch, n_players=p_old)
            with torch.no_grad():
                for prm in m.parameters():
                    prm.normal_(0.0, 0.1)
            nm = adapt_first_conv(m, new_shape, arch=arch, n_players=p_new)
            tag = f"{arch}_{p_old}to{p_new}"
            first = "conv0.weight" if arch == "cnn" else "shared.0.weight"
            out[f"{tag}__old"] = m.state_dict()[first].numpy().copy()
            out[f"{tag}__new"] = nm.state_dict()[first].numpy().copy()
            # every other key is copied through unchanged (same shapes)
            out[f"{tag}__keys"] = np.array(sorted(nm.state_dict().keys()))
    # a checkpoint written by the reference itself
    torch.manual_seed(7)
    m = AC((14, 3, 3), arch="mlp", n_players=2)
    with torch.no_grad():
        for prm in m.parameters():
            prm.normal_(0.0, 0.1)
    opt = torch.optim.Adam(m.parameters(), lr=1e-4, eps=1e-5)
    cs = CurriculumState(stage_idx=2, episodes_in_stage=37, recent_wins=[1.0, 0.0, 0.5])
    args = _ap.Namespace(num_envs=64, arch="mlp", lr=1e-4)
    path = os.path.join(HERE, "ref_ckpt_mlp.pt")
    save_ckpt(path, learner=m, opt=opt, pool=ModelPool(), cstate=cs, global_step=12345,
              elo=1012.5, args=args, fixed_elo={"astar": 990.0})
    return out


def ckpt_lstm_golden(R):
    """adapt_first_conv on the LSTM architecture (train/train.py:140-147: its
    local CNN's first layer l_conv1 takes the observation's channels in
    view order), seeded random models, 2 <-> 3 players."""
    import torch
    from sim.config import n_obs_channels
    from train.train import adapt_first_conv
    AC = R["ActorCritic"]
    out = {}
    for i, (p_old, p_new) in enumerate(((2, 3), (3, 2))):
        torch.manual_seed(200 + i)
        old_shape = (n_obs_channels(p_old), 13, 13)
        new_shape = (n_obs_channels(p_new), 13, 13)
        m = AC(old_shape, arch="lstm", n_players=p_old)
        with torch.no_grad():
            for prm in m.parameters():
                prm.normal_(0.0, 0.1)
        nm = adapt_first_conv(m, new_shape, arch="lstm", n_players=p_new)
        tag = f"lstm_{p_old}to{p_new}"
        out[f"{tag}__old"] = m.state_dict()["l_conv1.weight"].numpy().copy()
        out[f"{tag}__new"] = nm.state_dict()["l_conv1.weight"].numpy().copy()
    return out


class FedDraws:
    """Stand-in for `torch` inside sim/torch_sim.py and sim/mapgen.py during
    reset_: rand / randint come from recorded 24-bit integer keys k (rand =
    k / 2^24 as float32; randint = low + (k * (high - low)) >> 24), logged in
    call order; a (count, H*W) rand (the obstacle permutation keys) gets
    distinct keys per row, so its argsort has no ties."""

    def __init__(self, real, rng, cells):
        self._real, self._rng, self._cells = real, rng, cells
        self.log = []

    def rand(self, *size, generator=None, device=None, dtype=None, **kw):
        shape = tuple(size[0]) if len(size) == 1 and isinstance(size[0], (tuple, list)) \
            else tuple(size)
        if len(shape) == 2 and shape[1] == self._cells:
            k = np.stack([self._rng.choice(1 << 24, size=shape[1], replace=False)
                          for _ in range(shape[0])]) if shape[0] else np.zeros(shape, np.int64)
        else:
            k = self._rng.integers(0, 1 << 24, size=shape)
        self.log.append(("rand", k.astype(np.int64)))
        return self._real.from_numpy(k.astype(np.float32) * np.float32(1.0 / 16777216.0))

    def randint(self, low, high, size, generator=None, device=None, **kw):
        k = self._rng.integers(0, 1 << 24, size=size).astype(np.int64)
        self.log.append(("randint", k))
        return self._real.from_numpy(low + ((k * (high - low)) >> 24))

    def __getattr__(self, name):
        return getattr(self._real, name)


def _route_mapgen_draws(cfg, n, idx, log):
    """Per-env draw arrays (the oracle's map_reset keys) from the calls the
    reference's reset_ made, in its call order (sim/torch_sim.py:178-420)."""
    h, w = cfg.height, cfg.width
    C = h * w
    unit = np.float32(1.0 / 16777216.0)
    d = {"kind_u": np.zeros(n, np.float32), "obst_n": np.zeros(n, np.int64),
         "obst_key": np.zeros((n, C), np.int64), "ring_u": np.zeros((n, C), np.float32),
         "top": np.zeros(n, np.int64), "vstart_u": np.zeros((n, 4), np.float32),
         "vlen_u": np.zeros((n, 4), np.float32), "vact_u": np.zeros((n, 4), np.float32),
         "hstart_u": np.zeros(n, np.float32), "hlen_u": np.zeros(n, np.float32),
         "hact_u": np.zeros(n, np.float32), "swap_u": np.zeros(n, np.float32),
         "hazard_u": np.zeros(n, np.float32)}
    calls = list(log)
    pop = lambda: calls.pop(0)  # noqa: E731
    nmax = cfg.open_obstacle_max
    if cfg.map_mode == "corridor":
        r = pop()[1].astype(np.float32) * unit
        d["kind_u"][idx] = r
        pf = np.float32(cfg.pure_open_fraction)
        po = np.float32(cfg.pure_open_fraction + cfg.open_fraction)
        pr = np.float32(cfg.pure_open_fraction + cfg.open_fraction + cfg.ring_fraction)
        opn = r < po
        ring = ~opn & (r < pr)
        corr = ~(opn | ring)
        assert (r < pf).sum() <= opn.sum()
        if opn.any() and nmax > 0:
            k = pop()[1]
            d["obst_n"][idx[opn]] = (k * (nmax + 1)) >> 24
            d["obst_key"][idx[opn]] = pop()[1]
        if ring.any():
            d["ring_u"][idx[ring]] = pop()[1].reshape(-1, C).astype(np.float32) * unit
        if corr.any():
            ci = idx[corr]
            if cfg.random_wall_rows:
                d["top"][ci] = (pop()[1] * (cfg.top_wall_rows + 1)) >> 24
            if cfg.wall_density > 0:
                c0 = (w - cfg.corridor_width) // 2
                c1 = c0 + cfg.corridor_width
                ne = len([c for c in (c0, c0 + 1, c1 - 2, c1 - 1) if c0 <= c < c1])
                if ne:
                    for key in ("vstart_u", "vlen_u", "vact_u"):
                        d[key][ci, :ne] = pop()[1].astype(np.float32) * unit
                if c1 - c0 > 4:
                    for key in ("hstart_u", "hlen_u", "hact_u"):
                        d[key][ci] = pop()[1].astype(np.float32) * unit
    elif nmax > 0:
        k = pop()[1]
        d["obst_n"][idx] = (k * (nmax + 1)) >> 24
        d["obst_key"][idx] = pop()[1]
    d["swap_u"][idx] = pop()[1].astype(np.float32) * unit
    if cfg.hazard_fraction > 0:
        d["hazard_u"][idx] = pop()[1].astype(np.float32) * unit
    assert not calls, f"unrouted draws: {[c[0] for c in calls]}"
    return d


def mapgen_golden(R):
    """Per-episode level generation (sim/torch_sim.py:178-420, sim/mapgen.py)
    run by the reference with its generator's draws fed and recorded: for
    several configurations (mixed pure-open / open / ring / corridor maps,
    random and fixed wall rows, edge brick segments, open obstacles, cross
    crates, hazard envs, opponent boost tiers 0-2, two and three players, an
    open-mode map), the state before and after reset_ of a random subset of
    envs, and the draws routed per env (tests/test_oracle_golden.py replays
    them through oracle.map_reset)."""
    import torch
    import sim.mapgen as rmg
    ts = R["ts"]
    SC = R["SimConfig"]
    scen = [
        ("mixed", dict(map_mode="corridor", pure_open_fraction=0.2, open_fraction=0.3,
                       ring_fraction=0.2, random_wall_rows=True, wall_density=0.45,
                       open_obstacle_max=6, hazard_fraction=0.3, speed=3.0), 64, 0),
        ("fixed_rows", dict(map_mode="corridor", open_fraction=0.25, ring_fraction=0.25,
                            random_wall_rows=False, wall_density=0.25, open_obstacle_max=3,
                            speed=3.0), 48, 1),
        ("three_players", dict(map_mode="corridor", n_players=3, open_fraction=0.3,
                               ring_fraction=0.3, wall_density=0.45, open_obstacle_max=4,
                               speed=3.0), 48, 2),
        ("open_mode", dict(map_mode="open", open_obstacle_max=5, hazard_fraction=0.2,
                           speed=3.0), 40, 1),
        ("corridor_11", dict(map_mode="corridor", height=11, width=11, corridor_width=5,
                             top_wall_rows=3, open_fraction=0.2, ring_fraction=0.0,
                             wall_density=0.45, speed=3.0), 40, 0),
    ]
    out = {}
    names = []
    for si, (name, kw, n, boost) in enumerate(scen):
        cfg = SC(**kw)
        sim = ts.BatchedSim(cfg, n, device="cpu", seed=50 + si)
        rng = np.random.default_rng(900 + si)
        boosts = rng.integers(0, 3, n) if boost else np.zeros(n, np.int64)
        sim._opp_boost.copy_(torch.from_numpy(boosts))
        mask = rng.random(n) < 0.7
        pre = state_np(sim)
        fed = FedDraws(torch, rng, cfg.height * cfg.width)
        old = (ts.torch, rmg.torch)
        ts.torch, rmg.torch = fed, fed
        try:
            sim.reset_(torch.from_numpy(mask))
        finally:
            ts.torch, rmg.torch = old
        idx = np.nonzero(mask)[0]
        draws = _route_mapgen_draws(cfg, n, idx, fed.log)
        post = state_np(sim)
        tag = f"s{si}"
        names.append(name)
        out[f"{tag}__cfg"] = np.array(json.dumps(kw))
        out[f"{tag}__mask"] = mask
        out[f"{tag}__boost"] = boosts.astype(np.int64)
        for k, v in pre.items():
            out[f"{tag}__pre_{k}"] = v
        for k, v in post.items():
            out[f"{tag}__post_{k}"] = v
        out[f"{tag}__post_is_open"] = sim._is_open.numpy().copy()
        out[f"{tag}__post_map_kind"] = sim._map_kind.numpy().copy()
        for k, v in draws.items():
            out[f"{tag}__draw_{k}"] = v
    out["scenarios"] = np.array(names)
    return out


def hazard_golden(R):
    """Hazard wave placement (sim/torch_sim.py:1404-1466) run by the
    reference itself on seeded states, with its randint / rand / randperm
    fed the engine's keyed draws (oracle.hazard_draws_keyed), so that the
    placement rules (free cells, the dead-player cell rule, blast formula,
    offsets) are pinned independently of the random source."""
    import torch
    sys.path.insert(0, REPO)
    from oracle import qqt_oracle as O
    from qqt_b200.config import SimConfig as BSC
    rts = R["ts"]
    kw = dict(map_mode="open", hazard_fraction=1.0, speed=3.0)
    cfg_r, cfg_b = R["SimConfig"](**kw), BSC(**kw)
    n, h, w, p = 32, cfg_b.height, cfg_b.width, cfg_b.n_players
    rng = np.random.default_rng(21)
    wall = np.broadcast_to(scenarios.border_walls(h, w), (n, h, w)).copy()
    wall |= (rng.random((n, h, w)) < 0.08)
    brick = (rng.random((n, h, w)) < 0.2) & ~wall
    fuse = np.where(rng.random((n, h, w)) < 0.1, rng.integers(1, 30, (n, h, w)), 0).astype(np.int16)
    fuse[wall] = 0
    owner = np.where(fuse > 0, rng.integers(0, p + 1, (n, h, w)), -1).astype(np.int8)
    blast = np.where(fuse > 0, rng.integers(1, 8, (n, h, w)), 0).astype(np.int16)
    pos = (rng.integers(1, h - 1, (n, p, 2)) + 0.5).astype(np.float32)
    alive = rng.random((n, p)) < 0.8
    hazard = rng.random(n) < 0.7
    t = rng.choice([50, 100, 600, 1200, 49], n).astype(np.int64)
    st = {"wall": wall, "brick": brick, "fuse": fuse, "owner": owner, "bomb_blast": blast,
          "pos": pos, "alive": alive, "hazard": hazard, "t": t}
    seed = 0x1234ABCD5678
    draws = O.hazard_draws_keyed(cfg_b, st, seed)

    class Fed:
        def __init__(self):
            self.perm = list(draws["perm"])

        def randint(self, low, high, size, device=None, **k):
            return torch.from_numpy(draws["cnt"].copy())

        def rand(self, *size, device=None, **k):
            return torch.from_numpy(draws["u"].copy())

        def randperm(self, m, device=None, **k):
            pr = self.perm.pop(0)
            assert pr.size == m
            return torch.from_numpy(pr.astype(np.int64))

        def __getattr__(self, name):
            return getattr(torch, name)

    sim = rts.BatchedSim(cfg_r, n, device="cpu", seed=0)
    set_state(sim, st)
    sim.alive.copy_(torch.from_numpy(alive))
    sim._hazard.copy_(torch.from_numpy(hazard))
    sim.t.copy_(torch.from_numpy(t))
    real = rts.torch
    rts.torch = Fed()
    try:
        sim._hazard_wave()
    finally:
        rts.torch = real
    out = {"pre_" + k: np.asarray(v) for k, v in st.items()}
    out["seed"] = np.array(seed, np.uint64)
    out["n_wave_envs"] = np.array(len(draws["envs"]))
    for k in ("fuse", "owner", "bomb_blast"):
        out["post_" + k] = getattr(sim, k).numpy().copy()
    return out


def local_view_golden(R):
    """The reference's local_view_features (sim/obs.py:241-340) on seeded
    states: P = 2 (corridor) and P = 3 (open) configurations, envs from bomb
    free to 40 bombs (fewer bombs than slots leaves non-bomb filler slots),
    players next to the border (clipped windows), fp16 observations from
    the reference's own observe(); only_p0 both ways."""
    import torch
    sys.path.insert(0, R["root"])
    from sim.obs import local_view_features
    rts = R["ts"]
    out = {}
    for tag, kw, n, seed in (("p2", dict(map_mode="corridor", speed=3.0, max_steps=1800), 40, 31),
                             ("p3", dict(map_mode="open", n_players=3), 24, 32)):
        cfg = R["SimConfig"](**kw)
        h, w, p = cfg.height, cfg.width, cfg.n_players
        rng = np.random.default_rng(seed)
        wall = np.broadcast_to(scenarios.border_walls(h, w), (n, h, w)).copy()
        wall |= (rng.random((n, h, w)) < 0.08)
        brick = (rng.random((n, h, w)) < 0.2) & ~wall
        dens = rng.choice([0.0, 0.01, 0.03, 0.1, 0.25], n)[:, None, None]
        fuse = np.where(rng.random((n, h, w)) < dens, rng.integers(1, 31, (n, h, w)), 0)
        fuse = fuse.astype(np.int16)
        fuse[wall] = 0
        owner = np.where(fuse > 0, rng.integers(0, p, (n, h, w)), -1).astype(np.int8)
        blast = np.where(fuse > 0, rng.integers(1, 6, (n, h, w)), 0).astype(np.int16)
        pos = (rng.integers(1, h - 1, (n, p, 2)) + rng.random((n, p, 2)) * 0.98 + 0.01)
        pos = pos.astype(np.float32)
        alive = rng.random((n, p)) < 0.8
        hp = rng.integers(0, cfg.max_hp + 1, (n, p)).astype(np.uint8)
        t = rng.integers(0, cfg.max_steps, n).astype(np.int64)
        sim = rts.BatchedSim(cfg, n, device="cpu", seed=0)
        set_state(sim, {"wall": wall, "brick": brick, "fuse": fuse, "owner": owner,
                        "bomb_blast": blast, "pos": pos})
        sim.alive.copy_(torch.from_numpy(alive))
        sim.hp.copy_(torch.from_numpy(hp).to(sim.hp.dtype))
        sim.t.copy_(torch.from_numpy(t))
        obs = sim.observe()
        st = {"wall": wall, "brick": brick, "fuse": fuse, "owner": owner, "bomb_blast": blast,
              "pos": pos, "alive": alive, "hp": hp, "t": t}
        for k, v in st.items():
            out[f"{tag}__{k}"] = np.asarray(v)
        out[f"{tag}__obs"] = obs.numpy().copy()
        for only in (False, True):
            loc, rel, glob = local_view_features(sim.cfg, obs, sim.pos, sim.alive, sim.t,
                                                 sim.fuse, sim.hp, only_p0=only)
            sfx = "p0" if only else "all"
            out[f"{tag}__{sfx}__local"] = loc.numpy().copy()
            out[f"{tag}__{sfx}__rel"] = rel.numpy().copy()
            out[f"{tag}__{sfx}__glob"] = glob.numpy().copy()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="root of the reference source tree")
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    R = load_reference(args.ref)
    SC = R["SimConfig"]
    jobs = {
        "kat_states": lambda: kat_states(R, args.ref),
        "traj_cfg1": lambda: rollout(R, SC(**scenarios.CFG1), 16, 256, 0, "open_border",
                                     None, "random", rng_seed=10, obs_every=8),
        "traj_cfg2": lambda: rollout(R, SC(**scenarios.CFG2), 24, 128, 1, "corridor",
                                     "mlp", "astar", rng_seed=11, obs_every=4),
        "traj_cfg4": lambda: rollout(R, SC(**scenarios.CFG2), 12, 64, 4, "corridor",
                                     "mlp", "self", rng_seed=14, obs_every=8),
        "traj_cfg5": lambda: rollout(R, SC(**scenarios.CFG2), 8, 48, 3, "corridor",
                                     "cnn", "greedy", rng_seed=13, obs_every=8),
        "traj_hunter": lambda: rollout(R, SC(**scenarios.CFG2), 24, 128, 2, "sparse_crates",
                                       "mlp", "hunter", rng_seed=15, obs_every=8),
        "stress_cfg3": lambda: stress(R, SC(**scenarios.CFG1), 48, 5),
        "reset_modes": lambda: reset_modes(R),
        "ppo_update": lambda: ppo_golden(R),
        "ckpt_adapt": lambda: ckpt_golden(R),
        "ckpt_adapt_lstm": lambda: ckpt_lstm_golden(R),
        "mapgen_fed": lambda: mapgen_golden(R),
        "danger_walls": lambda: danger_walls_golden(R),
        "hazard_wave": lambda: hazard_golden(R),
        "local_view": lambda: local_view_golden(R),
    }
    for name, fn in jobs.items():
        if args.only and name not in args.only.split(","):
            continue
        out = fn()
        path = os.path.join(HERE, name + ".npz")
        np.savez_compressed(path, **out)
        print(f"{name}: {os.path.getsize(path) / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
