"""GPU parity of the benchmarked rollout itself: cfg2 at its benchmark shape
(N=5632 as two env groups of 2816 on their own streams, 128 ticks, MLP
learner on seat 0 vs the astar bot on seat 1, device auto-reset and crate
recycling), captured as the benchmark captures it (two CUDA graphs over two
draw-buffer sets, `capture(double_buffer=True)`) and replayed from a
mid-game state, against the oracle on seeded subsets of envs of both groups
for all 128 ticks of both graphs: observation rows, legal masks, both
seats' actions, done and damage flags every tick and the whole state at the
end bit-exact, rewards within 1e-6.

Envs are independent except for one batch-wide value: the astar bot's
chain scan reaches out to the maximum blast_cap of its seat over the whole
batch (sim/bots.py:484).  Each env group is its own sim, so that batch is
the group, as it would be for a separate reference process; the rollout
records each tick's value (`Rollout.cap_log`) and the subset oracle uses
it.  Group 1 is given larger blast caps than group 0, so the two groups'
values differ and each is checked to be its own group's maximum.

The learner samples from float32 tensor-core logits, the oracle from
float64 logits: a sampled action may differ only where u*S falls within
1e-5 of a category boundary (a near tie); such an env continues with the
engine's action.
"""

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
    from qqt_b200.policy import B200Policy
    from qqt_b200.policy_init import init_params
    from qqt_b200.rollout import Rollout, RolloutGroups
    from qqt_b200.sim import B200Sim, _recycle_exclusion

N_ENVS, GROUPS, T = 5632, 2, 128
SUBSET = 192


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


def _build():
    """The benchmark's engine for rank 0 (bench.py build_engine, cfg2)."""
    cfg = SimConfig(**scenarios.CFG2)
    n = N_ENVS // GROUPS
    tmpl = scenarios.corridor_template(cfg, N_ENVS, 1)
    pol = B200Policy(init_params(cfg.obs_shape, "mlp", seed=1), cfg.obs_shape, 2, seats=(0,))
    ros, tmpls = [], []
    for g in range(GROUPS):
        part = {k: v[g * n:(g + 1) * n] for k, v in tmpl.items()}
        sim = B200Sim(cfg, n, device="cuda", seed=1 + 1000 * g, template=part)
        sim.set_template(part, apply=False, seed=1 + 1000 * g, swap_spawns=False)
        ro = Rollout(sim, pol, AstarBot(sim, mode=True), T=T)
        ro.cap_log = torch.zeros((T,), dtype=torch.int32, device="cuda")
        ros.append(ro)
        tmpls.append(part)
    return cfg, pol, RolloutGroups(ros), tmpls


def _near_tie(logits, mask, u, a, b, tol=1e-5):
    z = np.where(mask, logits, np.finfo(np.float32).min).astype(np.float64)
    e = np.exp(z - z.max())
    cs = np.cumsum(e)
    x = float(u) * cs[-1]
    lo, hi = min(a, b), max(a, b)
    return min(abs(x - cs[k]) for k in range(lo, hi)) <= tol * cs[-1]


def _logp(logits, mask, a):
    z = np.where(mask, logits, np.finfo(np.float32).min).astype(np.float64)
    m = z.max(-1, keepdims=True)
    s = np.exp(z - m).sum(-1)
    return np.take_along_axis(z, a[:, None], 1)[:, 0] - m[:, 0] - np.log(s)


def _oracle_group(cfg, params, ro, tmpl, start, sub, calls0, flush0, draws, bufs, cap_log):
    """Replay one group's subset on the oracle; returns the near-tie count."""
    p = cfg.n_players
    st = {k: np.array(v[sub], copy=True) for k, v in start["state"].items()}
    st["resolve_tiers"] = np.int64(start["tiers"])
    tm = {k: np.asarray(v)[sub] for k, v in tmpl.items()}
    ticker = O.ModeTicker(start["mode"][sub], start["timer"][sub])
    ticker.tick = calls0
    episode = start["episode"][sub].copy()
    excl = _recycle_exclusion(cfg)
    n = sub.size
    k_in = cfg.n_channels * cfg.n_cells
    ties = 0
    flushes = 0
    for t in range(T):
        obs, _ = O.observe(cfg, st)
        obs16 = obs.astype(np.float16)
        mm, bm = O.legal_mask(cfg, st)
        got = bufs["obs_rows"][t][:, :k_in]
        assert np.array_equal(got.view(np.uint16), obs16.reshape(n, -1).view(np.uint16)), \
            f"t={t}: observation rows"
        assert np.array_equal(bufs["mm"][t], mm), f"t={t}: move mask"
        assert np.array_equal(bufs["bm"][t], bm), f"t={t}: bomb mask"
        obs32 = obs16.astype(np.float32)
        u = draws["u_net"][t, 0][sub]
        a0, _, v0, ml, bl = O.mlp_act(params, obs32, mm[:, 0], bm[:, 0], 0, p, u[:, 0], u[:, 1])
        acts = bufs["act"][t].copy()
        for i in np.nonzero((acts[:, 0] != a0).any(-1))[0]:
            for j, (lg, mk) in enumerate(((ml, mm[:, 0]), (bl, bm[:, 0]))):
                if acts[i, 0, j] != a0[i, j]:
                    assert _near_tie(lg[i], mk[i], u[i, j], acts[i, 0, j], a0[i, j]), \
                        f"t={t}: learner action of env {sub[i]} is not a near tie"
                    ties += 1
        lp = _logp(ml, mm[:, 0], acts[:, 0, 0]) + _logp(bl, bm[:, 0], acts[:, 0, 1])
        assert np.abs(bufs["logp"][t, 0] - lp).max() <= 1e-3, f"t={t}: log-prob"
        assert np.abs(bufs["val"][t, 0] - v0).max() <= 2e-3 * max(np.abs(v0).max(), 1e-3), \
            f"t={t}: value"
        k = ticker.tick + 1
        jj = (k // 16) % draws["tick_mode"].shape[0]
        mode = ticker.advance(draws["tick_mode"][jj][sub], draws["tick_timer"][jj][sub])
        a1 = O.astar_attack(cfg, st, obs32[:, 2 * p + 1], mm[:, 1], bm[:, 1], 1,
                            draws["noise"][t][sub], mode=mode, cap_max=int(cap_log[t]))
        assert np.array_equal(acts[:, 1], a1), f"t={t}: astar actions"
        assert int(cap_log[t]) >= int(st["blast_cap"][:, 1].max()), f"t={t}: chain-scan length"
        hp0 = st["hp"].astype(np.int32)
        rew, done, _ = O.step(cfg, st, acts, draws["crate"][t, 0][sub], draws["crate"][t, 1][sub])
        dmg = ((hp0 - st["hp"].astype(np.int32)) > 0) & ~done[:, None]
        O.template_reset(cfg, st, tm, done, swap=None, episode=episode)
        assert np.abs(bufs["rew"][t] - rew).max() <= REW_TOL, f"t={t}: reward"
        assert np.array_equal(bufs["done"][t], done), f"t={t}: done"
        assert np.array_equal(bufs["dmg"][t], dmg), f"t={t}: damage flags"
        if t % ro.flush_every == ro.flush_every - 1:
            flushes += 1
            O.flush_recycle_keyed(cfg, st, excl, ro.sim._flush_seed, flush0 + flushes, envs=sub)
    return st, episode, ties


def test_benchmark_rollout_graphs_vs_oracle():
    cfg, pol, grp, tmpls = _build()
    gen = torch.Generator(device="cuda").manual_seed(1234)
    for ro in grp.ros:
        ro.draws.generate(gen)
        ro.tick(0)
    grp.collect()                      # a full eager rollout: a mid-game state
    # larger blast caps on seat 1 in a few envs of group 1: the groups'
    # chain-scan lengths differ
    s1 = grp.ros[1].sim
    cap = s1.blast_cap.clone()
    cap[:8, 1] = cfg.growth_blast_max
    s1.blast_cap = cap
    calls0 = [ro.opponent.calls for ro in grp.ros]
    flush0 = [getattr(ro.sim, "_flush_count", 0) for ro in grp.ros]
    grp.capture(double_buffer=True)
    for d in grp.draw_sets[1]:
        d.generate(gen)                # new draws for the second graph
    params = {k: v.cpu().numpy() for k, v in pol.params.items()}
    rng = np.random.default_rng(2024)
    n = N_ENVS // GROUPS
    ties = 0
    for which in (0, 1):
        starts = []
        for ro in grp.ros:
            starts.append({"state": ro.sim.numpy_state(), "mode": _np(ro.opponent.mode),
                           "timer": _np(ro.opponent.timer),
                           "episode": _np(ro.sim._tmpl_buf["episode"]),
                           "tiers": int(ro.sim._tiers.item())})
        grp.replay(which)
        torch.cuda.synchronize()
        logs = [_np(ro.cap_log) for ro in grp.ros]
        for g, ro in enumerate(grp.ros):
            assert logs[g][0] == int(starts[g]["state"]["blast_cap"][:, 1].max()), \
                f"group {g}: tick-0 chain-scan length is the group's maximum"
        if which == 0:
            assert logs[1][0] > logs[0][0], "the two groups' chain-scan lengths differ"
        for g, ro in enumerate(grp.ros):
            sub = np.sort(rng.choice(n, SUBSET, replace=False))
            if g == 1:
                sub = np.union1d(sub, np.arange(8))
            b, si = ro.buf, torch.from_numpy(sub).cuda()
            bufs = {k: _np(getattr(b, k)[:, si]) for k in ("obs_rows", "mm", "bm", "act", "rew",
                                                          "done", "dmg")}
            bufs.update({k: _np(getattr(b, k)[:, :, si]) for k in ("logp", "val")})
            dr = {k: _np(getattr(grp.draw_sets[which][g], k))
                  for k in ("u_net", "noise", "crate", "tick_mode", "tick_timer")}
            f0 = flush0[g] + which * (T // ro.flush_every)
            st, episode, k = _oracle_group(cfg, params, ro, tmpls[g], starts[g], sub, calls0[g],
                                           f0, dr, bufs, logs[g])
            ties += k
            got = ro.sim.numpy_state()
            bad = [key for key in O.STATE_KEYS if key in got
                   and not np.array_equal(got[key][sub], st[key])]
            assert not bad, f"graph {which} group {g}: end state differs in {bad}"
            assert np.array_equal(_np(ro.sim._tmpl_buf["episode"])[sub], episode)
    assert ties <= 4, f"{ties} near-tie learner samples"
