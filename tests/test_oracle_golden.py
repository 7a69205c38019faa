"""Pin the CPU oracle against golden vectors produced by the reference itself.

The oracle is the checker for every GPU parity test, so it must reproduce
the reference bit for bit on integer/boolean state and float32 positions,
danger and observations (rewards within 1e-6, policy outputs within the
float32-vs-float64 gap).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import goldens as G
from oracle import qqt_oracle as O
from qqt_b200 import scenarios
from qqt_b200.config import SimConfig
from qqt_b200.policy_init import init_params


def kat_cfg():
    return SimConfig(height=13, width=13, n_players=2, map_mode="corridor", speed=3.0,
                     max_steps=1800, obs_extra_enabled=True, obs_fp16=False)


def test_kat_states_danger_obs_masks_resolve():
    g = G.load("kat_states")
    cfg = kat_cfg()
    n = g["wall"].shape[0]
    st = {k: g[k] for k in ("wall", "brick", "fuse", "owner", "bomb_blast", "crate",
                            "pos", "alive", "invuln", "bombs_cap", "blast_cap")}
    st["t"] = g["t"].astype(np.int64)
    bmap = O.blast_map(st["bomb_blast"], cfg.blast)
    # the known-answer files use the dynamic full-length chain (max_chain rounds)
    dng = O.danger_map(st["fuse"], st["wall"], bmap, st["brick"], cfg.fuse, cfg.max_chain)
    assert np.array_equal(dng, g["danger"])
    obs = O.encode_obs(cfg, st, dng)
    assert np.array_equal(obs, g["obs"])
    mm, bm = O.legal_mask(cfg, st)
    assert np.array_equal(mm, g["mm"]) and np.array_equal(bm, g["bm"])
    cov, trig = O.resolve_explosions(st["fuse"], st["owner"], st["wall"], bmap,
                                     st["brick"], cfg.max_chain - 1)
    assert np.array_equal(cov, g["covered"]) and np.array_equal(trig, g["triggered"])
    assert n == 61


def _bot_act(kind, cfg, st, obs16, mm, bm, pid, draws, ticker, bomb_rate):
    dng = obs16[:, 2 * cfg.n_players + 1].astype(np.float32)
    if kind == "random":
        u_move = draws[0][1][:, 0]
        u_bomb = draws[1][1]
        return O.random_attack(st["alive"][:, pid], mm[:, pid], bm[:, pid],
                               u_move, u_bomb, bomb_rate)
    if kind == "greedy":
        return O.greedy_attack(cfg, st, dng, mm[:, pid], bm[:, pid], pid, draws[0][1])
    if kind == "hunter":
        noise = [v for k, v in draws if k == "rand"][0]
        return O.astar_attack(cfg, st, dng, mm[:, pid], bm[:, pid], pid, noise, mode=None,
                              eat_crates=True)
    if kind == "astar":
        ints = [v for k, v in draws if k == "randint"]
        noise = [v for k, v in draws if k == "rand"][0]
        if ticker[0] is None:
            ticker[0] = O.ModeTicker(ints[0], ints[1])
            ints = ints[2:]
        nm = ints[0] if ints else np.zeros(len(noise), np.int64)
        nt = ints[1] if ints else np.zeros(len(noise), np.int64)
        mode = ticker[0].advance(nm, nt)
        return O.astar_attack(cfg, st, dng, mm[:, pid], bm[:, pid], pid, noise, mode=mode)
    raise ValueError(kind)


def replay(name, cfg, learner, opp, bomb_rate=0.05, check_every_state=True):
    g = G.load(name)
    st = G.init_state(g)
    wall = st["wall"]
    n, p = st["alive"].shape
    T = g["reward"].shape[0]
    obs_ticks = list(g["obs_ticks"])
    reset_ticks = list(g["reset_ticks"])
    flush_ticks = list(g["flush_ticks"])
    params = None
    if learner is not None:
        params = init_params(cfg.obs_shape, arch=learner, seed=_seed_of(name))
    ticker = [None]
    stats = {"logit_err": 0.0, "act_mismatch": 0}
    for t in range(T):
        obs, dng = O.observe(cfg, st)
        obs16 = obs.astype(np.float16)
        if t in obs_ticks:
            i = obs_ticks.index(t)
            assert np.array_equal(obs16, g["obs"][i]), f"{name} t={t}: obs"
        mm, bm = O.legal_mask(cfg, st)
        assert np.array_equal(mm, g["mm"][t]) and np.array_equal(bm, g["bm"][t]), \
            f"{name} t={t}: masks"
        acts = g["actions"][t]
        seats = [0, 1]
        for pid in seats:
            is_net = (pid == 0 and learner is not None) or (pid == 1 and opp == "self")
            if is_net and learner == "mlp":
                u = g["u_net"][t][:, pid]
                a, lp, v, ml, bl = O.mlp_act(params, obs16.astype(np.float32), mm[:, pid],
                                             bm[:, pid], pid, p, u[:, 0], u[:, 1])
                ref_ml = g["logits_m"][t][:, pid]
                err = np.abs(ml - ref_ml).max() / max(1e-6, np.abs(ref_ml).max())
                stats["logit_err"] = max(stats["logit_err"], float(err))
                stats["act_mismatch"] += int((a != acts[:, pid]).any(-1).sum())
            elif not is_net:
                kind = "random" if (pid == 0 or opp == "random") else opp
                draws = G.bot_draws(g, pid, t)
                a = _bot_act(kind, cfg, st, obs16, mm, bm, pid, draws, ticker, bomb_rate)
                assert np.array_equal(a, acts[:, pid]), f"{name} t={t}: bot seat {pid}"
        r, d, info = O.step(cfg, st, acts, g["rb_hit"][t], g["rb_grow"][t])
        assert np.array_equal(d, g["done"][t]), f"{name} t={t}: done"
        assert np.array_equal(info["winner"], g["winner"][t]), f"{name} t={t}: winner"
        assert np.allclose(r, g["reward"][t], atol=1e-6, rtol=0), \
            f"{name} t={t}: reward max err {np.abs(r - g['reward'][t]).max()}"
        ref = G.state_at(g, t, wall)
        bad = G.compare_state(ref, st)
        assert not bad, f"{name} t={t}: state differs in {bad}"
        if t in reset_ticks:
            i = reset_ticks.index(t)
            rs = G.reset_state(g, i, wall)
            for k in rs:
                st[k][d] = rs[k][d]
            bad = G.compare_state(rs, st)
            assert not bad, f"{name} t={t}: post-reset state differs in {bad}"
        if t in flush_ticks:
            i = flush_ticks.index(t)
            gen = torch.Generator().manual_seed(0)
            gen.set_state(torch.from_numpy(g[f"flush{i}_gen"]))
            O.flush_recycle(cfg, st, gen)
            for k in ("crate", "recycle", "pending_lost"):
                assert np.array_equal(st[k], g[f"flush{i}_{k}"]), f"{name} t={t}: flush {k}"
    return stats


def _seed_of(name):
    return {"traj_cfg2": 1, "traj_cfg4": 4, "traj_cfg5": 3, "traj_hunter": 2}.get(name, 0)


def test_traj_cfg1_random_bots():
    replay("traj_cfg1", SimConfig(**scenarios.CFG1), None, "random")


def test_traj_cfg2_mlp_vs_astar():
    stats = replay("traj_cfg2", SimConfig(**scenarios.CFG2), "mlp", "astar")
    assert stats["logit_err"] < 1e-4
    assert stats["act_mismatch"] == 0


def test_traj_cfg4_selfplay_mlp():
    stats = replay("traj_cfg4", SimConfig(**scenarios.CFG2), "mlp", "self")
    assert stats["logit_err"] < 1e-4
    assert stats["act_mismatch"] == 0


def test_stress_cfg3_step_danger_fields():
    g = G.load("stress_cfg3")
    cfg = SimConfig(**scenarios.CFG1)
    st = G.init_state(g)
    n, p = st["alive"].shape
    acts = np.zeros((n, p, 2), np.int64)
    acts[..., 0] = 4
    r, d, info = O.step(cfg, st, acts, g["rb_hit"], g["rb_grow"])
    assert np.array_equal(info["blast"], g["covered"])
    assert np.array_equal(info["trig"], g["triggered"])
    assert np.allclose(r, g["reward"], atol=1e-6)
    after = G.init_state(g, "after_")
    assert not G.compare_state(after, st)
    obs, dng = O.observe(cfg, st)
    assert np.array_equal(dng, g["danger"])
    assert np.array_equal(obs.astype(np.float16), g["obs"])
    mm, bm = O.legal_mask(cfg, st)
    assert np.array_equal(mm, g["mm"]) and np.array_equal(bm, g["bm"])
    d16 = g["obs"][:, 2 * p + 1].astype(np.float32)
    for pid in range(p):
        a, vs, vo = O.astar_attack(cfg, st, d16, mm[:, pid], bm[:, pid], pid,
                                   g[f"astar_noise{pid}"], mode=None, return_fields=True)
        assert np.array_equal(vs, g[f"vsafe{pid}"])
        assert np.array_equal(vo, g[f"vopp{pid}"])
        assert np.array_equal(a, g[f"astar_act{pid}"])


def test_traj_cfg2_dijkstra_fields():
    g = G.load("traj_cfg2")
    cfg = SimConfig(**scenarios.CFG2)
    wall = g["init_wall"]
    h, w = cfg.height, cfg.width
    for i, t in enumerate(g["field_ticks"]):
        st = G.init_state(g) if t == 0 else G.state_at(g, t - 1, wall)
        if t > 0 and (t - 1) in list(g["reset_ticks"]):
            pytest.skip("reset between ticks")
        obs, _ = O.observe(cfg, st)
        d16 = obs.astype(np.float16)[:, 2 * cfg.n_players + 1].astype(np.float32)
        blk = st["wall"] | st["brick"] | (st["fuse"] > 0)
        vs = O.dijkstra_field(d16 < np.float32(0.35), d16, blk)
        n = st["fuse"].shape[0]
        r0 = np.clip(np.floor(st["pos"][:, 0, 0]).astype(int), 0, h - 1)
        c0 = np.clip(np.floor(st["pos"][:, 0, 1]).astype(int), 0, w - 1)
        src = np.zeros((n, h * w), bool)
        src[np.arange(n), r0 * w + c0] = st["alive"][:, 0]
        vo = O.dijkstra_field(src.reshape(n, h, w), d16, blk)
        assert np.array_equal(vs, g["vsafe"][i]) and np.array_equal(vo, g["vopp"][i])


def test_traj_hunter_mlp_vs_hunter():
    """The hunter bot (astar with the crate layer, sim/bots.py:376-431,
    557-561) replayed tick by tick against the reference's trajectory."""
    stats = replay("traj_hunter", SimConfig(**scenarios.CFG2), "mlp", "hunter")
    assert stats["logit_err"] < 1e-4
    assert stats["act_mismatch"] == 0


def test_traj_hunter_crate_fields_and_eat_branch():
    """V_crate (sources = crate cells) bit-exact at the recorded ticks, and
    the crate branch decides some of the hunter's moves in this trajectory."""
    g = G.load("traj_hunter")
    cfg = SimConfig(**scenarios.CFG2)
    wall = g["init_wall"]
    eat_moves = 0
    for i, t in enumerate(g["field_ticks"]):
        st = G.init_state(g) if t == 0 else G.state_at(g, t - 1, wall)
        if t > 0 and (t - 1) in list(g["reset_ticks"]):
            continue
        if t > 0 and (t - 1) in list(g["flush_ticks"]):      # crates recycled after the step
            j = list(g["flush_ticks"]).index(t - 1)
            for k in ("crate", "recycle", "pending_lost"):
                st[k] = g[f"flush{j}_{k}"].copy()
        obs, _ = O.observe(cfg, st)
        d16 = obs.astype(np.float16)[:, 2 * cfg.n_players + 1].astype(np.float32)
        blk = st["wall"] | st["brick"] | (st["fuse"] > 0)
        vc = O.dijkstra_field(st["crate"], d16, blk)
        assert np.array_equal(vc, g["vcrate"][i])
        mm, bm = O.legal_mask(cfg, st)
        noise = [v for k, v in G.bot_draws(g, 1, t) if k == "rand"][0]
        a_eat = O.astar_attack(cfg, st, d16, mm[:, 1], bm[:, 1], 1, noise, eat_crates=True)
        a_plain = O.astar_attack(cfg, st, d16, mm[:, 1], bm[:, 1], 1, noise)
        assert np.array_equal(a_eat, g["actions"][t][:, 1])
        eat_moves += int((a_eat[:, 0] != a_plain[:, 0]).sum())
    assert eat_moves > 0


def test_hazard_wave_matches_reference():
    """Hazard-wave placement (sim/torch_sim.py:1404-1466): the restatement
    with the engine's keyed draws equals the reference fed the same draws."""
    g = G.load("hazard_wave")
    cfg = SimConfig(map_mode="open", hazard_fraction=1.0, speed=3.0)
    st = {k[4:]: v.copy() for k, v in g.items() if k.startswith("pre_")}
    draws = O.hazard_draws_keyed(cfg, st, int(g["seed"]))
    assert len(draws["envs"]) == int(g["n_wave_envs"]) > 0
    O.hazard_wave(cfg, st, draws)
    for k in ("fuse", "owner", "bomb_blast"):
        assert np.array_equal(st[k], g["post_" + k]), k
    assert (g["post_owner"] == cfg.n_players).sum() > (g["pre_owner"] == cfg.n_players).sum()


def test_template_reset_gives_the_reference_reset_state():
    """oracle.template_reset (the restatement of the engine's device
    auto-reset) on the cfg1 open-border template reproduces the reference's
    own post-reset state (sim/torch_sim.py:178-420) for every env that ended
    in the 256-tick cfg1 trajectory, all state keys, when it is given the
    spawn swap the reference's generator drew (read from the golden)."""
    g = G.load("traj_cfg1")
    cfg = SimConfig(**scenarios.CFG1)
    wall = g["init_wall"]
    n = wall.shape[0]
    tmpl = scenarios.open_border_template(cfg, n)
    assert np.array_equal(tmpl["wall"], np.broadcast_to(wall, tmpl["wall"].shape))
    spawn0 = tmpl["spawn"][:, 0]
    swaps = []
    for i, t in enumerate(g["reset_ticks"]):
        st = G.state_at(g, t, wall)
        done = g["done"][t]
        rs = G.reset_state(g, i, wall)
        swap = done & ~np.all(rs["pos"][:, 0] == spawn0, axis=-1)
        swaps += list(swap[done])
        episode = np.zeros(n, np.int64)
        O.template_reset(cfg, st, tmpl, done, swap=swap, episode=episode)
        bad = G.compare_state(rs, st)
        assert not bad, f"t={t}: template reset differs from the reference in {bad}"
        assert np.array_equal(episode, done.astype(np.int64))
    assert any(swaps) and not all(swaps), "both swap outcomes are exercised"


def test_template_swap_draws_are_keyed():
    """The device reset's spawn-swap draw is a pure function of (seed, env,
    episode): fixed values, about half swap, and a new episode redraws."""
    ep = np.zeros(4096, np.int64)
    a = O.template_swap_draws(7, ep)
    assert np.array_equal(a, O.template_swap_draws(7, ep))
    assert 0.45 < a.mean() < 0.55
    b = O.template_swap_draws(7, ep + 1)
    assert 0.4 < (a != b).mean() < 0.6
    c = O.template_swap_draws(8, ep)
    assert (a != c).any()


def test_map_reset_matches_the_reference_level_generator():
    """oracle.map_reset, fed the draws the reference's reset_ consumed (its
    generator replaced by recorded 24-bit keys), rebuilds exactly the
    reference's post-reset state (sim/torch_sim.py:178-420, sim/mapgen.py):
    every state key, is_open and map_kind, for reset and untouched envs, in
    five configurations (mixed pure-open / open / ring / corridor maps with
    random or fixed wall rows and edge brick segments, open obstacles, cross
    crates, hazard envs, opponent boost tiers, three players, an open-mode
    map, an 11 x 11 board)."""
    import json
    g = G.load("mapgen_fed")
    kinds = set()
    for si, name in enumerate(g["scenarios"]):
        tag = f"s{si}"
        cfg = SimConfig(**json.loads(str(g[f"{tag}__cfg"])))
        st = {k: np.array(g[f"{tag}__pre_{k}"], copy=True) for k in G.STATE_KEYS}
        mask = g[f"{tag}__mask"]
        n = mask.shape[0]
        dr = {k[len(tag) + 7:]: g[k] for k in g if k.startswith(f"{tag}__draw_")}
        aux = {"is_open": np.zeros(n, bool), "map_kind": np.zeros(n, np.int64)}
        pre_open = g[f"{tag}__post_is_open"].copy()
        pre_kind = g[f"{tag}__post_map_kind"].copy()
        aux["is_open"][~mask] = pre_open[~mask]
        aux["map_kind"][~mask] = pre_kind[~mask]
        O.map_reset(cfg, st, mask, dr, opp_boost=g[f"{tag}__boost"], aux=aux)
        post = {k: g[f"{tag}__post_{k}"] for k in G.STATE_KEYS}
        bad = G.compare_state(post, st)
        assert not bad, f"{name}: state differs in {bad}"
        assert np.array_equal(aux["is_open"], pre_open), f"{name}: is_open"
        assert np.array_equal(aux["map_kind"], pre_kind), f"{name}: map_kind"
        kinds |= set(aux["map_kind"][mask].tolist())
    assert kinds == {0, 1, 2}, "corridor, open and ring levels all generated"


def test_mapgen_keyed_draws_are_in_range():
    cfg = SimConfig(map_mode="corridor", open_obstacle_max=6, top_wall_rows=4)
    d = O.mapgen_draws_keyed(cfg, 123, np.arange(500) % 7)
    assert d["obst_n"].min() >= 0 and d["obst_n"].max() == 6
    assert d["top"].min() == 0 and d["top"].max() == 4
    assert d["obst_key"].shape == (500, 169) and d["obst_key"].max() < (1 << 24)
    for k in ("kind_u", "ring_u", "vstart_u", "hact_u", "swap_u", "hazard_u"):
        assert 0.0 <= d[k].min() and d[k].max() < 1.0
    again = O.mapgen_draws_keyed(cfg, 123, np.arange(500) % 7)
    assert all(np.array_equal(d[k], again[k]) for k in d)


def test_danger_and_chains_with_bombs_on_walls():
    """Bombs on wall cells (a player standing on an obstacle can place one):
    the reference's danger map spreads stage B from the weights with walls
    zeroed, while stage A still lets such a bomb raise the bombs its flame
    reaches; the oracle's danger map and chain resolution equal the
    reference's on 48 seeded states (tests/golden/danger_walls.npz)."""
    g = G.load("danger_walls")
    assert int(((g["fuse"] > 0) & g["wall"]).sum()) > 50
    bmap = O.blast_map(g["bomb_blast"], int(g["blast"]))
    dng = O.danger_map(g["fuse"], g["wall"], bmap, g["brick"], int(g["fuse_max"]),
                       int(g["max_chain"]))
    assert np.array_equal(dng, g["danger"])
    cov, trig = O.resolve_explosions(g["fuse"], g["owner"], g["wall"], bmap, g["brick"],
                                     int(g["max_chain"]) - 1)
    assert np.array_equal(cov, g["covered"]) and np.array_equal(trig, g["triggered"])
