"""GPU parity: the CUDA engine (through the C ABI) against the reference's
golden trajectories and the CPU oracle.

Bar: integer / boolean state, masks and bot actions bit-exact; positions,
danger and fp16 observations bit-exact (the kernels keep the reference's
float32 operation order); rewards within 1e-6 absolute (the reference sums
the placement chain bonus over cells in a different order); path fields
bit-exact.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import goldens as G

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from qqt_b200 import scenarios
    from qqt_b200.bots import AstarBot, GreedyBot, HunterBot, RandomBot
    from qqt_b200.config import SimConfig
    from qqt_b200.sim import B200Sim, tile_flags
    from qqt_b200 import _capi


@pytest.fixture(autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    yield
    torch.cuda.synchronize()
    assert _capi.device_error() == 0, "device error word set"


def _np(t):
    return t.detach().cpu().numpy()


def _sim_from_state(cfg, st):
    n = st["alive"].shape[0]
    sim = B200Sim(cfg, n, device="cuda", seed=0)
    sim.load_numpy_state(st)
    return sim


def test_kat_states_observe_masks():
    g = G.load("kat_states")
    cfg = SimConfig(height=13, width=13, n_players=2, map_mode="corridor", speed=3.0,
                    max_steps=1800, obs_extra_enabled=True, obs_fp16=False)
    n = g["wall"].shape[0]
    st = {k: g[k] for k in ("wall", "brick", "fuse", "owner", "bomb_blast", "crate", "pos",
                            "alive", "invuln", "bombs_cap", "blast_cap")}
    st["t"] = g["t"].astype(np.int64)
    st["recycle"] = np.zeros_like(st["wall"])
    sim = _sim_from_state(cfg, st)
    obs, mm, bm = sim.observe_and_mask()
    assert np.array_equal(_np(sim.danger()), g["danger"])
    assert np.array_equal(_np(obs), g["obs"])
    assert np.array_equal(_np(mm), g["mm"]) and np.array_equal(_np(bm), g["bm"])


def _replay(name, cfg, learner, opp, bomb_rate=0.05, field_check=False):
    g = G.load(name)
    st = G.init_state(g)
    wall = st["wall"]
    n, p = st["alive"].shape
    sim = _sim_from_state(cfg, st)
    T = g["reward"].shape[0]
    obs_ticks = list(g["obs_ticks"])
    reset_ticks = list(g["reset_ticks"])
    flush_ticks = list(g["flush_ticks"])
    field_ticks = list(g["field_ticks"]) if "field_ticks" in g else []
    bots = {}
    for pid in (0, 1):
        is_net = (pid == 0 and learner is not None) or (pid == 1 and opp == "self")
        if is_net:
            continue
        kind = "random" if (pid == 0 or opp == "random") else opp
        bots[pid] = {"random": lambda: RandomBot(sim, bomb_rate), "greedy": lambda: GreedyBot(sim),
                     "astar": lambda: AstarBot(sim, mode=True),
                     "hunter": lambda: HunterBot(sim)}[kind]()
        if kind in ("astar", "hunter"):
            bots[pid].keep_fields = field_check
    for t in range(T):
        obs, mm, bm = sim.observe_and_mask()
        assert np.array_equal(_np(mm), g["mm"][t]), f"{name} t={t}: move mask"
        assert np.array_equal(_np(bm), g["bm"][t]), f"{name} t={t}: bomb mask"
        if t in obs_ticks:
            assert np.array_equal(_np(obs), g["obs"][obs_ticks.index(t)]), f"{name} t={t}: obs"
        for pid, bot in bots.items():
            draws = G.bot_draws(g, pid, t)
            if isinstance(bot, RandomBot):
                bot.feed(u_move=draws[0][1][:, 0], u_bomb=draws[1][1])
            elif isinstance(bot, (GreedyBot, HunterBot)):
                bot.feed(noise=[v for k, v in draws if k == "rand"][0])
            else:
                ints = [v for k, v in draws if k == "randint"]
                noise = [v for k, v in draws if k == "rand"][0]
                feed = {"noise": noise}
                if bot.mode is None:
                    feed["mode0"], feed["timer0"] = ints[0], ints[1]
                    ints = ints[2:]
                if ints:
                    feed["new_mode"], feed["new_timer"] = ints[0], ints[1]
                elif (bot.calls + 1) % 16 == 0:
                    feed["new_mode"] = np.zeros(n, np.int64)
                    feed["new_timer"] = np.zeros(n, np.int64)
                bot.feed(**feed)
            a = bot.act(obs, mm[:, pid], bm[:, pid], pid)
            assert np.array_equal(_np(a), g["actions"][t][:, pid]), f"{name} t={t}: bot {pid}"
            if field_check and t in field_ticks and pid == 1:
                i = field_ticks.index(t)
                assert np.array_equal(_np(bot.vsafe), g["vsafe"][i]), f"{name} t={t}: V_safe"
                assert np.array_equal(_np(bot.vopp), g["vopp"][i]), f"{name} t={t}: V_opp"
                if "vcrate" in g:
                    assert np.array_equal(_np(bot.vcrate), g["vcrate"][i]), f"{name} t={t}: V_crate"
        acts = torch.from_numpy(g["actions"][t]).cuda()
        rb = (torch.from_numpy(g["rb_hit"][t]).cuda(), torch.from_numpy(g["rb_grow"][t]).cuda())
        r, d, info = sim.step(acts, auto_reset=False, crate_draws=rb)
        assert np.array_equal(_np(d), g["done"][t]), f"{name} t={t}: done"
        assert np.array_equal(_np(info["winner"]), g["winner"][t]), f"{name} t={t}: winner"
        err = np.abs(_np(r) - g["reward"][t]).max()
        assert err <= 1e-6, f"{name} t={t}: reward err {err}"
        got = sim.numpy_state()
        got["wall"] = got["wall"]
        bad = G.compare_state(G.state_at(g, t, wall), got)
        assert not bad, f"{name} t={t}: state differs in {bad}"
        if t in reset_ticks:
            rs = G.reset_state(g, reset_ticks.index(t), wall)
            sim.load_numpy_state(rs)
        if t in flush_ticks:
            i = flush_ticks.index(t)
            sim.gen.set_state(torch.from_numpy(g[f"flush{i}_gen"]))
            sim.flush_recycle()
            got = sim.numpy_state()
            for k in ("crate", "recycle", "pending_lost"):
                assert np.array_equal(got[k], g[f"flush{i}_{k}"]), f"{name} t={t}: flush {k}"


def test_traj_cfg1_random_bots_gpu():
    _replay("traj_cfg1", SimConfig(**scenarios.CFG1), None, "random")


def test_traj_cfg2_astar_gpu():
    _replay("traj_cfg2", SimConfig(**scenarios.CFG2), "mlp", "astar", field_check=True)


def test_traj_hunter_gpu():
    _replay("traj_hunter", SimConfig(**scenarios.CFG2), "mlp", "hunter", field_check=True)


def test_traj_cfg5_greedy_gpu():
    _replay("traj_cfg5", SimConfig(**scenarios.CFG2), "cnn", "greedy")


def test_stress_cfg3_gpu():
    g = G.load("stress_cfg3")
    cfg = SimConfig(**scenarios.CFG1)
    st = G.init_state(g)
    n, p = st["alive"].shape
    sim = _sim_from_state(cfg, st)
    acts = torch.zeros((n, p, 2), dtype=torch.int64, device="cuda")
    acts[..., 0] = 4
    r, d, info = sim.step(acts, auto_reset=False,
                          crate_draws=(torch.from_numpy(g["rb_hit"]).cuda(),
                                       torch.from_numpy(g["rb_grow"]).cuda()))
    assert np.array_equal(_np(info["blast"]), g["covered"])
    assert np.array_equal(_np(info["trig"]), g["triggered"])
    assert np.abs(_np(r) - g["reward"]).max() <= 1e-6
    assert not G.compare_state(G.init_state(g, "after_"), sim.numpy_state())
    obs, mm, bm = sim.observe_and_mask()
    assert np.array_equal(_np(sim.danger()), g["danger"])
    assert np.array_equal(_np(obs), g["obs"])
    assert np.array_equal(_np(mm), g["mm"]) and np.array_equal(_np(bm), g["bm"])
    for pid in range(p):
        bot = AstarBot(sim, mode=False)
        bot.keep_fields = True
        bot.feed(noise=g[f"astar_noise{pid}"])
        a = bot.act(obs, mm[:, pid], bm[:, pid], pid)
        assert np.array_equal(_np(bot.vsafe), g[f"vsafe{pid}"])
        assert np.array_equal(_np(bot.vopp), g[f"vopp{pid}"])
        assert np.array_equal(_np(a), g[f"astar_act{pid}"])


def test_hazard_waves_vs_oracle():
    """Hazard waves in the step kernel (sim/torch_sim.py:1404-1466) against
    the oracle restatement with the same keyed draws, tick by tick (waves
    every 8 ticks, counts kept below the free-cell pool)."""
    from oracle import qqt_oracle as O
    cfg = SimConfig(map_mode="open", speed=3.0, hazard_fraction=1.0, hazard_wave_ticks=8,
                    hazard_bombs_min=2, hazard_bombs_max=6, hazard_blast_min=2,
                    hazard_blast_max=5, hazard_ramp_seconds=2.0)
    n, p = 40, cfg.n_players
    sim = B200Sim(cfg, n, device="cuda", seed=3)
    sim.hazard_seed = 0xC0FFEE1234
    st = sim.numpy_state()
    assert st["hazard"].all()
    rng = np.random.default_rng(5)
    waves = 0
    for t in range(40):
        acts = np.zeros((n, p, 2), np.int64)
        acts[..., 0] = rng.integers(0, 5, (n, p))
        r, d, _ = sim.step(torch.from_numpy(acts).cuda(), auto_reset=False)
        before = int((st["owner"] == p).sum())
        o_r, o_d, _ = O.step(cfg, st, acts, np.zeros((n, p), np.float32),
                             np.zeros((n, p), np.float32), hazard_seed=sim.hazard_seed)
        waves += int((st["owner"] == p).sum()) > before
        got = sim.numpy_state()
        for k in ("fuse", "owner", "bomb_blast", "brick", "pos", "hp", "alive", "t"):
            assert np.array_equal(got[k], st[k]), f"t={t}: {k}"
        assert np.array_equal(_np(d), o_d), f"t={t}: done"
        assert np.abs(_np(r) - o_r).max() <= 1e-6, f"t={t}: reward"
    assert waves >= 3
    torch.cuda.synchronize()
    assert _capi.device_error() == 0


@pytest.mark.parametrize("shape", [(11, 11, 2), (13, 13, 3), (13, 13, 2)],
                         ids=["11x11_p2", "13x13_p3", "13x13_p2"])
def test_step_instances_vs_oracle(shape):
    """The step kernel is compiled per shape: the two-player 13x13 tick has
    the player count and the grid fixed at compile time, two players on any
    other grid have the player count fixed, and every other shape runs the
    runtime-shape kernel.  Each against the oracle tick by tick over 50
    ticks (random moves and bombs; the 30-tick fuses go off), with and without
    the fused next-tick observation, which must equal a stand-alone
    observe of the same state (its K-tile flags those of the rows).  The astar bot is compiled the same way:
    every 5th tick each player's astar action (no mode ticker) against the
    oracle's on the same state and noise."""
    from oracle import qqt_oracle as O
    h, w, p = shape
    cfg = SimConfig(height=h, width=w, n_players=p, map_mode="open", speed=3.0)
    n = 48
    fused = B200Sim(cfg, n, device="cuda", seed=11)
    st = fused.numpy_state()
    plain = _sim_from_state(cfg, {k: v.copy() for k, v in st.items()})
    rows = torch.zeros((n, fused.obs_stride), dtype=torch.float16, device="cuda")
    mm = torch.zeros((n, p, 5), dtype=torch.bool, device="cuda")
    bm = torch.zeros((n, p, 2), dtype=torch.bool, device="cuda")
    tiles = torch.zeros((n, 4), dtype=torch.int32, device="cuda")
    ref_rows = torch.zeros_like(rows)
    ref_mm, ref_bm = torch.zeros_like(mm), torch.zeros_like(bm)
    rng = np.random.default_rng(7)
    zeros = np.zeros((n, p), np.float32)
    exploded = 0
    for t in range(50):
        if t % 5 == 0:
            obs, omm, obm = plain.observe_and_mask()
            d16 = O.observe(cfg, st)[0].astype(np.float16).astype(np.float32)[:, 2 * p + 1]
            o_mm, o_bm = O.legal_mask(cfg, st)
            for pid in range(p):
                noise = rng.random((n, 5), dtype=np.float32)
                bot = AstarBot(plain, mode=False)
                bot.feed(noise=torch.from_numpy(noise).cuda())
                a_gpu = _np(bot.act(obs, omm[:, pid], obm[:, pid], pid))
                a_ref = O.astar_attack(cfg, st, d16, o_mm[:, pid], o_bm[:, pid], pid, noise)
                assert np.array_equal(a_gpu, a_ref), f"t={t}: astar actions of player {pid}"
        acts = np.zeros((n, p, 2), np.int64)
        acts[..., 0] = rng.integers(0, 5, (n, p))
        acts[..., 1] = rng.random((n, p)) < 0.3
        a = torch.from_numpy(acts).cuda()
        r, d, _ = fused.step(a, auto_reset=False, next_obs=(rows, mm, bm, tiles))
        r2, d2, _ = plain.step(a, auto_reset=False)
        plain.observe_and_mask(ref_rows, ref_mm, ref_bm, danger=False)
        owned = st["owner"] >= 0
        o_r, o_d, _ = O.step(cfg, st, acts, zeros, zeros)
        exploded += int((owned & (st["owner"] < 0)).sum())
        got, got2 = fused.numpy_state(), plain.numpy_state()
        for k in ("fuse", "owner", "bomb_blast", "brick", "pos", "hp", "alive", "t"):
            assert np.array_equal(got[k], st[k]), f"t={t}: {k} (fused)"
            assert np.array_equal(got2[k], st[k]), f"t={t}: {k}"
        assert np.array_equal(_np(d), o_d) and np.array_equal(_np(d2), o_d), f"t={t}: done"
        assert np.abs(_np(r) - o_r).max() <= 1e-6 and np.abs(_np(r2) - o_r).max() <= 1e-6
        assert torch.equal(rows.view(torch.int16), ref_rows.view(torch.int16)), f"t={t}: rows"
        assert torch.equal(mm, ref_mm) and torch.equal(bm, ref_bm), f"t={t}: masks"
        assert torch.equal(tiles, tile_flags(rows)), f"t={t}: K-tile flags"
    assert exploded > 0


def test_danger_and_chains_with_bombs_on_walls_gpu():
    """Bombs on wall cells (tests/golden/danger_walls.npz, the reference's own
    danger_map and resolve_explosions): the observe kernel's danger map, and
    the step's flames and exploded bombs from the state one tick earlier
    (every bomb's fuse one higher, so that the step's countdown lands on the
    golden state), bit-exact."""
    g = G.load("danger_walls")
    cfg = SimConfig(height=13, width=13, n_players=2, map_mode="corridor", speed=3.0,
                    chain_cap_rounds=int(g["max_chain"]))
    n = g["wall"].shape[0]
    sim = B200Sim(cfg, n, device="cuda", seed=0)
    st = sim.numpy_state()
    for k in ("wall", "brick", "fuse", "owner", "bomb_blast"):
        st[k] = g[k].copy()
    st["crate"][:] = False
    sim.load_numpy_state(st)
    sim.observe_and_mask()
    assert np.array_equal(_np(sim.danger()), g["danger"])
    bomb = (g["fuse"] > 0) | ((g["fuse"] == 0) & (g["owner"] >= 0))
    st["fuse"] = np.where(bomb, g["fuse"] + 1, 0).astype(np.int16)
    sim.load_numpy_state(st)
    acts = torch.zeros((n, 2, 2), dtype=torch.int64, device="cuda")
    acts[..., 0] = 4
    rb = torch.zeros((n, 2), dtype=torch.float32, device="cuda")
    _, _, info = sim.step(acts, auto_reset=False, crate_draws=(rb, rb))
    assert np.array_equal(_np(info["blast"]), g["covered"])
    assert np.array_equal(_np(info["trig"]), g["triggered"])
