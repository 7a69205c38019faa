"""GPU parity of the device auto-reset with per-episode level generation
(qqt_map_reset) against the oracle's restatement `map_reset` fed the same
counter-based draws (`mapgen_draws_keyed`).  `map_reset` itself rebuilds
the reference's own reset_ bit for bit when fed the reference's draws
(tests/test_oracle_golden.py, sim/torch_sim.py:178-420, sim/mapgen.py).

* reset_ of random env subsets, twice in a row (the episode counters
  advance), in six configurations: mixed pure-open / open / ring /
  corridor levels with random wall rows, edge brick segments, obstacles,
  cross crates and hazard envs; fixed wall rows; three players; an
  open-mode map with obstacles; an 11 x 11 board; opponent boost tiers
  0, 1 and 2 -- every state key plus is_open and map_kind, bit-exact;
* a rollout of 40 ticks with episodes forced to end (timeouts and deaths)
  through qqt_step_observe + qqt_map_reset: state, rewards, done and the
  new episodes' observation rows and masks every tick.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from oracle import qqt_oracle as O
    from qqt_b200 import _capi
    from qqt_b200.config import SimConfig
    from qqt_b200.sim import B200Sim, tile_flags

CONFIGS = {
    "mixed": dict(map_mode="corridor", pure_open_fraction=0.2, open_fraction=0.3,
                  ring_fraction=0.2, random_wall_rows=True, wall_density=0.45,
                  open_obstacle_max=6, hazard_fraction=0.3, speed=3.0),
    "fixed_rows": dict(map_mode="corridor", open_fraction=0.25, ring_fraction=0.25,
                       random_wall_rows=False, wall_density=0.25, open_obstacle_max=3,
                       speed=3.0),
    "three_players": dict(map_mode="corridor", n_players=3, open_fraction=0.3,
                          ring_fraction=0.3, wall_density=0.45, open_obstacle_max=4, speed=3.0),
    "open_mode": dict(map_mode="open", open_obstacle_max=5, hazard_fraction=0.2, speed=3.0),
    "corridor_11": dict(map_mode="corridor", height=11, width=11, corridor_width=5,
                        top_wall_rows=3, open_fraction=0.2, wall_density=0.45, speed=3.0),
    "plain_corridor": dict(map_mode="corridor", open_fraction=0.0, speed=3.0, max_steps=1800),
}
REW_TOL = 1e-6


@pytest.fixture(autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    yield
    torch.cuda.synchronize()
    assert _capi.device_error() == 0, "device error word set"


def _np(t):
    return t.detach().cpu().numpy()


def _aux(sim):
    return {"is_open": _np(sim._is_open).copy(), "map_kind": _np(sim._map_kind).copy()}


def _cmp(sim, st, aux, where):
    got = sim.numpy_state()
    bad = [k for k in O.STATE_KEYS if k in got and not np.array_equal(got[k], st[k])]
    assert not bad, f"{where}: state differs in {bad}"
    assert np.array_equal(_np(sim._is_open), aux["is_open"]), f"{where}: is_open"
    assert np.array_equal(_np(sim._map_kind), aux["map_kind"]), f"{where}: map_kind"


@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_device_map_reset_vs_oracle(name):
    cfg = SimConfig(**CONFIGS[name])
    n, seed = 256, 0xA11CE + len(name)
    sim = B200Sim(cfg, n, device="cuda", seed=7, map_reset="device")
    sim._mapgen.seed = seed
    rng = np.random.default_rng(len(name))
    boost = rng.integers(0, 3, n).astype(np.int64)
    sim._opp_boost.copy_(torch.from_numpy(boost))
    kinds = set()
    for rep in range(3):
        # arbitrary mid-game values everywhere, so that every reset field shows
        st = sim.numpy_state()
        st["fuse"][:] = rng.integers(0, 5, st["fuse"].shape)
        st["owner"][:] = rng.integers(-1, cfg.n_players, st["owner"].shape)
        st["hp"][:] = rng.integers(0, cfg.max_hp + 1, st["hp"].shape)
        st["t"][:] = rng.integers(0, 500, n)
        st["bombs_cap"][:] = rng.integers(1, 9, st["bombs_cap"].shape)
        st["spd_g"][:] = rng.random(st["spd_g"].shape).astype(np.float32) + 1
        st["crate"][:] = rng.random(st["crate"].shape) < 0.2
        sim.load_numpy_state(st)
        aux = _aux(sim)
        mask = rng.random(n) < (1.0 if rep == 0 else 0.6)
        episode = _np(sim._mg_episode).copy()
        dr = O.mapgen_draws_keyed(cfg, seed, episode)
        sim.reset_(torch.from_numpy(mask))
        torch.cuda.synchronize()
        O.map_reset(cfg, st, mask, dr, opp_boost=boost, aux=aux)
        _cmp(sim, st, aux, f"{name} rep {rep}")
        assert np.array_equal(_np(sim._mg_episode), episode + mask)
        kinds |= set(aux["map_kind"][mask].tolist())
    if cfg.map_mode == "corridor" and cfg.open_fraction > 0 and cfg.ring_fraction > 0:
        assert kinds == {0, 1, 2}


def test_device_map_reset_rollout_with_fused_observation():
    cfg = SimConfig(**CONFIGS["mixed"])
    n, p, T, seed = 128, cfg.n_players, 40, 0xBEEF
    sim = B200Sim(cfg, n, device="cuda", seed=3, map_reset="device")
    sim._mapgen.seed = seed
    sim.hazard_seed = 0x5A5A5A5A      # hazard waves with fixed keyed draws
    st = sim.numpy_state()
    aux = _aux(sim)
    rng = np.random.default_rng(5)
    rows = torch.zeros((n, sim.obs_stride), dtype=torch.float16, device="cuda")
    nmm = torch.zeros((n, p, 5), dtype=torch.bool, device="cuda")
    nbm = torch.zeros((n, p, 2), dtype=torch.bool, device="cuda")
    tiles = torch.zeros((n, 4), dtype=torch.int32, device="cuda")
    k_in = cfg.n_channels * cfg.n_cells
    ends = 0
    for t in range(T):
        if t % 8 == 3:
            e = rng.permutation(n)[: n // 3]
            st["t"][e] = cfg.max_steps - 1
            sim.load_numpy_state({"t": st["t"]})
        acts = np.stack([rng.integers(0, 5, (n, p)), rng.integers(0, 2, (n, p))], -1)
        rb = rng.random((2, n, p)).astype(np.float32)
        episode = _np(sim._mg_episode).copy()
        r, d, _ = sim.step(torch.from_numpy(acts).cuda(), auto_reset=True,
                           crate_draws=(torch.from_numpy(rb[0]).cuda(),
                                        torch.from_numpy(rb[1]).cuda()),
                           next_obs=(rows, nmm, nbm, tiles))
        torch.cuda.synchronize()
        o_r, o_d, _ = O.step(cfg, st, acts, rb[0], rb[1], hazard_seed=sim.hazard_seed)
        O.map_reset(cfg, st, o_d, O.mapgen_draws_keyed(cfg, seed, episode),
                    opp_boost=np.zeros(n, np.int64), aux=aux)
        ends += int(o_d.sum())
        assert np.array_equal(_np(d), o_d), f"t={t}: done"
        assert np.abs(_np(r) - o_r).max() <= REW_TOL, f"t={t}: reward"
        _cmp(sim, st, aux, f"t={t}")
        obs, _ = O.observe(cfg, st)
        mm, bm = O.legal_mask(cfg, st)
        got = _np(rows[:, :k_in]).view(np.uint16)
        assert np.array_equal(got, obs.astype(np.float16).reshape(n, -1).view(np.uint16)), \
            f"t={t}: next observation rows"
        assert np.array_equal(_np(nmm), mm) and np.array_equal(_np(nbm), bm), f"t={t}: masks"
        # K-tile flags: exact for rows the step wrote, every tile for rows
        # the level generator rewrote
        exact = tile_flags(rows)
        assert torch.equal(tiles[~d], exact[~d]), f"t={t}: K-tile flags"
        assert bool((tiles[d] == -1).all()), f"t={t}: K-tile flags of reset rows"
    assert ends >= n, f"only {ends} episodes ended"
