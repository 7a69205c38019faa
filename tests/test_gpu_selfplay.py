"""GPU replay of the reference's cfg4 self-play trajectory (both seats on one
random-init MLP, 12 envs, 64 ticks, tests/golden/traj_cfg4.npz) through the
rollout engine: `Rollout(seats=(0, 1))` runs both seats as one two-seat
policy launch (N = 256 output columns: seat 0's and seat 1's view of W0)
and the step with its fused next observation, as the cfg4 benchmark does
(train/ppo.py:215-249, `_opponent_actions` in self-play).

Bar: legal masks, observations (at the recorded ticks), both seats'
sampled actions, done flags and the whole state bit-exact to the
reference's own trajectory every tick; rewards within 1e-6 (the reference
sums the placement chain bonus in another order); log-probabilities within
1e-4 and the logits of both seats within 2e-3 relative of the reference's.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import goldens as G

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from qqt_b200 import _capi, scenarios
    from qqt_b200.config import SimConfig
    from qqt_b200.policy import B200Policy
    from qqt_b200.policy_init import init_params
    from qqt_b200.rollout import Rollout
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


def _rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-12))


def test_traj_cfg4_selfplay_rollout_gpu():
    g = G.load("traj_cfg4")
    cfg = SimConfig(**scenarios.CFG2)
    st = G.init_state(g)
    wall = st["wall"]
    n, p = st["alive"].shape
    T = g["reward"].shape[0]
    assert len(g["reset_ticks"]) == 0
    tmpl = {"wall": st["wall"], "brick": st["brick"], "crate": st["crate"], "spawn": st["pos"],
            "bombs_cap": st["bombs_cap"], "blast_cap": st["blast_cap"], "spd": st["spd_g"],
            "crate_prob": st["crate_prob"]}
    sim = B200Sim(cfg, n, device="cuda", seed=4, template=tmpl)
    sim.load_numpy_state(st)
    params = init_params(cfg.obs_shape, "mlp", seed=4)
    pol = B200Policy(params, cfg.obs_shape, p, seats=(0, 1))
    # crate recycling at the trajectory's flush ticks runs on the host
    # generator below, in the reference's draw order
    ro = Rollout(sim, pol, None, T=T, flush_every=0)
    ro.draws.u_net.copy_(torch.from_numpy(g["u_net"].transpose(0, 2, 1, 3).copy()))
    ro.draws.crate[:, 0].copy_(torch.from_numpy(g["rb_hit"]))
    ro.draws.crate[:, 1].copy_(torch.from_numpy(g["rb_grow"]))
    obs_ticks = list(g["obs_ticks"])
    flush_ticks = list(g["flush_ticks"])
    buf = ro.buf
    k_in = cfg.n_channels * cfg.n_cells
    for t in range(T):
        ro.tick(t)
        torch.cuda.synchronize()
        assert np.array_equal(_np(buf.mm[t]), g["mm"][t]), f"t={t}: move mask"
        assert np.array_equal(_np(buf.bm[t]), g["bm"][t]), f"t={t}: bomb mask"
        if t in obs_ticks:
            obs = _np(buf.obs_rows[t, :, :k_in]).reshape(g["obs"][0].shape)
            assert np.array_equal(obs, g["obs"][obs_ticks.index(t)]), f"t={t}: obs"
            # both seats' logits through the same two-seat launch
            logits, acts2, logp2 = pol.forward_logits(buf.obs(t), buf.mm[t], buf.bm[t],
                                                      ro.draws.u_net[t])
            lg = _np(logits)
            for s in range(2):
                assert _rel(lg[s, :, :5], g["logits_m"][t][:, s]) <= 2e-3, f"t={t}: seat {s}"
                assert _rel(lg[s, :, 5:7], g["logits_b"][t][:, s]) <= 2e-3, f"t={t}: seat {s}"
            assert np.array_equal(np.stack([_np(a) for a in acts2], 1), g["actions"][t])
            assert np.abs(_np(logp2).T - g["logp"][t]).max() <= 1e-4
        assert np.array_equal(_np(buf.act[t]), g["actions"][t]), f"t={t}: actions"
        lp = _np(buf.logp[t]).T
        assert np.abs(lp - g["logp"][t]).max() <= 1e-4, f"t={t}: log-prob"
        assert np.array_equal(_np(buf.done[t]), g["done"][t]), f"t={t}: done"
        err = np.abs(_np(buf.rew[t]) - g["reward"][t]).max()
        assert err <= 1e-6, f"t={t}: reward err {err}"
        got = sim.numpy_state()
        bad = G.compare_state(G.state_at(g, t, wall), got)
        assert not bad, f"t={t}: state differs in {bad}"
        if t in flush_ticks:
            i = flush_ticks.index(t)
            sim.gen.set_state(torch.from_numpy(g[f"flush{i}_gen"]))
            rows = buf.obs_rows[t + 1] if t + 1 < T else None
            sim.flush_recycle(on_device=False, obs_rows=rows)
            got = sim.numpy_state()
            for k in ("crate", "recycle", "pending_lost"):
                assert np.array_equal(got[k], g[f"flush{i}_{k}"]), f"t={t}: flush {k}"
