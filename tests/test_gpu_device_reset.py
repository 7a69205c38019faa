"""GPU parity of the device auto-reset (the template branch of the step
kernel) against the oracle's restatement `template_reset`, which is itself
pinned to the reference's own reset state (tests/test_oracle_golden.py,
sim/torch_sim.py:178-420).

* episodes forced to end by timeout (t = max_steps - 1) and by death (hp 1
  with a bomb about to explode underfoot), several times per env, through
  qqt_step and qqt_step_observe: state (every key), done, winner, died and
  damage flags after every tick, and with the fused observation the next
  tick's rows and legal masks, bit-exact; rewards within 1e-6;
* cfg1 at its benchmark size (N=64, 256 ticks, random bots on both seats)
  with the device reset on, observing and stepping through the public
  B200Sim API, tick by tick against the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from oracle import qqt_oracle as O
    from qqt_b200 import _capi, scenarios
    from qqt_b200.bots import RandomBot
    from qqt_b200.config import SimConfig
    from qqt_b200.sim import B200Sim


# rewards: within 1e-6 absolute, the bar of the reference goldens: the
# combo term's gap_factor ** gap is CUDA's powf on the device and the C
# library's powf in numpy, which may differ in the last bit
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


def _cmp_state(got, st, where):
    bad = [k for k in O.STATE_KEYS if k in got and not np.array_equal(got[k], st[k])]
    assert not bad, f"{where}: state differs in {bad}"


def _force_ends(cfg, st, rng, n, tick):
    """Pick envs to end on this tick: a third by timeout, a third by the
    death of one player (hp 1, no invulnerability, a bomb with fuse 1 and
    blast 2 on its centre cell).  Returns the keys poked."""
    e = rng.permutation(n)
    k = n // 3
    st["t"][e[:k]] = cfg.max_steps - 1
    h, w = cfg.height, cfg.width
    for i in e[k:2 * k]:
        pl = int(rng.integers(0, 2))
        if not st["alive"][i, pl]:
            continue
        r = min(max(int(np.floor(st["pos"][i, pl, 0])), 0), h - 1)
        c = min(max(int(np.floor(st["pos"][i, pl, 1])), 0), w - 1)
        st["hp"][i, pl] = 1
        st["invuln"][i, pl] = 0
        st["fuse"][i, r, c] = 1
        st["owner"][i, r, c] = pl
        st["bomb_blast"][i, r, c] = 2
    return ("t", "hp", "invuln", "fuse", "owner", "bomb_blast")


@pytest.mark.parametrize("fused", [False, True])
def test_device_reset_vs_template_reset(fused):
    cfg = SimConfig(**scenarios.CFG2)
    n, p, T = 96, cfg.n_players, 44
    tmpl = scenarios.corridor_template(cfg, n, seed=17)
    sim = B200Sim(cfg, n, device="cuda", seed=17, template=tmpl)
    seed = 0x5EED0F
    sim.set_template(tmpl, apply=False, seed=seed, swap_spawns=True)
    st = sim.numpy_state()
    episode = np.zeros(n, np.int64)
    rng = np.random.default_rng(101)
    rows = torch.zeros((n, sim.obs_stride), dtype=torch.float16, device="cuda")
    nmm = torch.zeros((n, p, 5), dtype=torch.bool, device="cuda")
    nbm = torch.zeros((n, p, 2), dtype=torch.bool, device="cuda")
    k_in = cfg.n_channels * cfg.n_cells
    resets = np.zeros(n, np.int64)
    for t in range(T):
        if t % 10 == 5:
            keys = _force_ends(cfg, st, rng, n, t)
            sim.load_numpy_state({k: st[k] for k in keys})
        acts = np.stack([rng.integers(0, 5, (n, p)), rng.integers(0, 2, (n, p))], -1)
        rb = rng.random((2, n, p)).astype(np.float32)
        hp0 = st["hp"].astype(np.int32)
        kw = dict(auto_reset=True,
                  crate_draws=(torch.from_numpy(rb[0]).cuda(), torch.from_numpy(rb[1]).cuda()))
        if fused:
            kw["next_obs"] = (rows, nmm, nbm)
        r, d, info = sim.step(torch.from_numpy(acts).cuda(), **kw)
        torch.cuda.synchronize()
        o_r, o_d, o_info = O.step(cfg, st, acts, rb[0], rb[1])
        o_hit = ((hp0 - st["hp"].astype(np.int32)) > 0) & ~o_d[:, None]
        swap = O.template_swap_draws(seed, episode)
        O.template_reset(cfg, st, tmpl, o_d, swap=swap, episode=episode)
        resets += o_d
        assert np.array_equal(_np(d), o_d), f"t={t}: done"
        assert np.abs(_np(r) - o_r).max() <= REW_TOL, f"t={t}: reward"
        assert np.array_equal(_np(info["winner"]), o_info["winner"]), f"t={t}: winner"
        assert np.array_equal(_np(info["died"]), o_info["died"]), f"t={t}: died"
        assert np.array_equal(_np(info["hit"]), o_hit), f"t={t}: damage flags"
        _cmp_state(sim.numpy_state(), st, f"t={t}")
        if fused:
            obs, _ = O.observe(cfg, st)
            mm, bm = O.legal_mask(cfg, st)
            got = _np(rows[:, :k_in]).view(np.uint16)
            want = obs.astype(np.float16).reshape(n, -1).view(np.uint16)
            assert np.array_equal(got, want), f"t={t}: next observation rows"
            assert np.array_equal(_np(nmm), mm) and np.array_equal(_np(nbm), bm), f"t={t}: masks"
    tm = sim._tmpl_buf["episode"]
    assert np.array_equal(_np(tm), episode), "per-env episode counters"
    assert (resets >= 2).sum() >= n // 4, "many envs run two or more episodes"
    assert (resets >= 3).any()


def test_cfg1_benchmark_size_device_reset_vs_oracle():
    """cfg1 (N=64, 256 ticks, random bots with bomb rate 0.05 on both seats,
    the open-border map re-applied with a keyed spawn swap by every device
    reset): observation, masks, both seats' actions, rewards, done and the
    whole state every tick."""
    cfg = SimConfig(**scenarios.CFG1)
    n, p, T = 64, cfg.n_players, 256
    tmpl = scenarios.open_border_template(cfg, n)
    sim = B200Sim(cfg, n, device="cuda", seed=0, template=tmpl)
    seed = 0xC0FFEE
    sim.set_template(tmpl, apply=False, seed=seed, swap_spawns=True)
    bots = [RandomBot(sim, 0.05), RandomBot(sim, 0.05)]
    st = sim.numpy_state()
    episode = np.zeros(n, np.int64)
    rng = np.random.default_rng(0)
    ends = 0
    for t in range(T):
        obs, mm, bm = sim.observe_and_mask()
        o_obs, _ = O.observe(cfg, st)
        o_mm, o_bm = O.legal_mask(cfg, st)
        assert np.array_equal(_np(obs), o_obs.astype(np.float16)), f"t={t}: obs"
        assert np.array_equal(_np(mm), o_mm) and np.array_equal(_np(bm), o_bm), f"t={t}: masks"
        u = rng.random((p, 2, n)).astype(np.float32)
        acts = torch.empty((n, p, 2), dtype=torch.int64, device="cuda")
        o_acts = np.zeros((n, p, 2), np.int64)
        for pid, bot in enumerate(bots):
            bot.feed(u_move=u[pid, 0], u_bomb=u[pid, 1])
            bot.act(obs, mm[:, pid], bm[:, pid], pid, out=acts[:, pid])
            o_acts[:, pid] = O.random_attack(st["alive"][:, pid], o_mm[:, pid], o_bm[:, pid],
                                             u[pid, 0], u[pid, 1], 0.05)
        assert np.array_equal(_np(acts), o_acts), f"t={t}: actions"
        r, d, _ = sim.step(acts, auto_reset=True)
        o_r, o_d, _ = O.step(cfg, st, o_acts, None, None)
        O.template_reset(cfg, st, tmpl, o_d, swap=O.template_swap_draws(seed, episode),
                         episode=episode)
        ends += int(o_d.sum())
        assert np.array_equal(_np(d), o_d), f"t={t}: done"
        assert np.abs(_np(r) - o_r).max() <= REW_TOL, f"t={t}: reward"
        _cmp_state(sim.numpy_state(), st, f"t={t}")
    assert ends >= 8, f"only {ends} episodes ended in 256 ticks"
