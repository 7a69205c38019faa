"""GPU parity of the cfg3 chain/danger stress workload at its benchmark size
(N=16384 envs, 20-40 bombs per env with fuse U{1..30} and blast U{1..5} on
the open-border map): one step with both seats idle and no reset, then the
danger map, observation and legal masks of the post-step state, then the
astar bot's path fields V_safe and V_opp and its actions for both players
-- all against the oracle for every env, bit-exact (rewards within 1e-6
absolute, as for the reference's own goldens).  Deep chains exercise the
8-round truncation of the resolver and of danger stage A."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from oracle import qqt_oracle as O
    from qqt_b200 import _capi, scenarios
    from qqt_b200.bots import AstarBot
    from qqt_b200.config import SimConfig
    from qqt_b200.sim import B200Sim


@pytest.fixture(autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    yield
    torch.cuda.synchronize()
    assert _capi.device_error() == 0, "device error word set"


def _np(t):
    return t.detach().cpu().numpy()


def test_stress_cfg3_full_size_vs_oracle():
    cfg = SimConfig(**scenarios.CFG1)
    n, p = 16384, cfg.n_players
    sim = B200Sim(cfg, n, device="cuda", seed=7)
    fuse, owner, blast = scenarios.bomb_stress(n, cfg, seed=7)
    st = sim.numpy_state()
    st["wall"] = np.broadcast_to(scenarios.border_walls(cfg.height, cfg.width), fuse.shape).copy()
    st["brick"][:] = False
    st["fuse"], st["owner"], st["bomb_blast"] = fuse, owner, blast
    st["pos"][:] = np.array(scenarios.open_spawns(cfg), np.float32)
    st["t"][:] = 40
    sim.load_numpy_state(st)
    assert (fuse > 0).sum(axis=(1, 2)).min() >= 20
    rng = np.random.default_rng(99)
    rb = rng.random((2, n, p)).astype(np.float32)
    acts = np.zeros((n, p, 2), np.int64)
    acts[..., 0] = 4
    r, d, info = sim.step(torch.from_numpy(acts).cuda(), auto_reset=False,
                          crate_draws=(torch.from_numpy(rb[0]).cuda(),
                                       torch.from_numpy(rb[1]).cuda()))
    o_r, o_d, o_info = O.step(cfg, st, acts, rb[0], rb[1])
    assert np.array_equal(_np(info["blast"]), o_info["blast"]), "flames"
    assert np.array_equal(_np(info["trig"]), o_info["trig"]), "exploded bombs"
    assert o_info["trig"].sum(axis=(1, 2)).max() >= 10, "deep chains occur"
    assert np.array_equal(_np(d), o_d)
    assert np.abs(_np(r) - o_r).max() <= 1e-6
    got = sim.numpy_state()
    bad = [k for k in O.STATE_KEYS if k in got and not np.array_equal(got[k], st[k])]
    assert not bad, f"post-step state differs in {bad}"
    obs, mm, bm = sim.observe_and_mask()
    o_obs, o_dng = O.observe(cfg, st)
    o_mm, o_bm = O.legal_mask(cfg, st)
    assert np.array_equal(_np(sim.danger()), o_dng), "danger map"
    assert np.array_equal(_np(obs), o_obs.astype(np.float16)), "observation"
    assert np.array_equal(_np(mm), o_mm) and np.array_equal(_np(bm), o_bm), "legal masks"
    d16 = o_obs.astype(np.float16)[:, 2 * p + 1].astype(np.float32)
    for pid in range(p):
        bot = AstarBot(sim, mode=False)
        bot.keep_fields = True
        noise = rng.random((n, 5)).astype(np.float32)
        bot.feed(noise=noise)
        a = bot.act(obs, mm[:, pid], bm[:, pid], pid)
        o_a, vs, vo = O.astar_attack(cfg, st, d16, o_mm[:, pid], o_bm[:, pid], pid, noise,
                                     mode=None, return_fields=True)
        assert np.array_equal(_np(bot.vsafe), vs), f"V_safe of player {pid}"
        assert np.array_equal(_np(bot.vopp), vo), f"V_opp of player {pid}"
        assert np.array_equal(_np(a), o_a), f"astar actions of player {pid}"
