"""The drop-in claim, tested: the reference's own collection tick
(SelfPlayRunner.collect, train/ppo.py:213-289) written against the
reference's API -- `sim.observe()`, `sim.legal_mask()`, the learner's
`act(obs, mm, bm, pid)`, the bot's `act(obs, mm, bm, pid)`, attribute pokes
`sim.owner.clone()`, `sim.fuse.clone()`, `sim.hp[:, 0].clone()`,
`sim.step(actions)` with its default auto-reset, `info["winner"]`,
`info["died"]`, the crate-pickup draws through `sim._rand_buf`, and
`sim.flush_recycle()` every 16 ticks -- runs unchanged on B200Sim, B200Policy
and the B200 astar bot, and gives the same trajectory as the engine's own
graph-capturable rollout (qqt_b200.rollout.Rollout, checked against the
oracle elsewhere) fed the same draws: observations, masks, actions, rewards,
done and damage flags every tick and the end state; the collect loop's
health statistics (suicides, bombs, danger standing) run on the pokes.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from qqt_b200 import _capi, scenarios
    from qqt_b200.bots import AstarBot
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


class _FedLearner:
    """The reference learner's interface (ActorCritic.act(obs, mm, bm, pid)
    -> (actions, logp, value)); its sampling uniforms come from a recorded
    stream, one (N, 2) block per call, instead of Categorical.sample."""

    def __init__(self, pol, u):
        self.pol, self.u, self.calls = pol, u, 0

    def act(self, obs, mm, bm, pid):
        u = self.u[self.calls]
        self.calls += 1
        return self.pol.act(obs, mm, bm, pid, u=u)


def _make(n, seed):
    cfg = SimConfig(**scenarios.CFG2)
    tmpl = scenarios.corridor_template(cfg, n, seed)
    sim = B200Sim(cfg, n, device="cuda", seed=seed, template=tmpl)
    sim.set_template(tmpl, apply=False, seed=seed, swap_spawns=True)
    bot = AstarBot(sim, mode=True)
    rng = np.random.default_rng(seed)
    bot.mode = torch.from_numpy(rng.integers(0, 2, n)).cuda()
    bot.timer = torch.from_numpy(rng.integers(60, 240, n)).cuda()
    return cfg, sim, bot


def test_reference_collect_protocol_runs_on_b200sim():
    n, T = 256, 48
    cfg, sim_a, bot_a = _make(n, 23)
    _, sim_b, bot_b = _make(n, 23)
    p = cfg.n_players
    pol = B200Policy(init_params(cfg.obs_shape, "mlp", seed=1), cfg.obs_shape, p, seats=(0,))
    # engine rollout on sim A
    ro = Rollout(sim_a, pol, bot_a, T=T)
    ro.draws.generate(torch.Generator(device="cuda").manual_seed(5))
    ro.collect()
    torch.cuda.synchronize()
    dr = ro.draws
    # the reference's collect tick on sim B, through its public surface only
    learner = _FedLearner(pol, dr.u_net[:, 0])
    sim = sim_b
    dng_ch = 2 * p + 1
    st_sui = torch.zeros(n, dtype=torch.long, device="cuda")
    st_bmb = torch.zeros(n, dtype=torch.long, device="cuda")
    st_dt = torch.zeros(n, dtype=torch.long, device="cuda")
    st_dv = torch.zeros(n, dtype=torch.float32, device="cuda")
    k_in = cfg.n_channels * cfg.n_cells
    for i in range(T):
        obs = sim.observe()
        mmask, bmask = sim.legal_mask()
        assert torch.equal(obs.reshape(n, -1).view(torch.int16),
                           ro.buf.obs_rows[i, :, :k_in].view(torch.int16)), f"t={i}: obs"
        assert torch.equal(mmask, ro.buf.mm[i]) and torch.equal(bmask, ro.buf.bm[i])
        actions = torch.zeros((n, p, 2), dtype=torch.long, device="cuda")
        with torch.no_grad():
            a0, logp, value = learner.act(obs, mmask[:, 0], bmask[:, 0], 0)
        actions[:, 0] = a0
        feed = {"noise": dr.noise[i]}
        if (bot_b.calls + 1) % 16 == 0:
            k = (bot_b.calls + 1) // 16
            feed["new_mode"] = dr.tick_mode[k % dr.tick_mode.shape[0]]
            feed["new_timer"] = dr.tick_timer[k % dr.tick_timer.shape[0]]
        bot_b.feed(**feed)
        actions[:, 1] = bot_b.act(obs, mmask[:, 1], bmask[:, 1], 1)
        assert torch.equal(actions, ro.buf.act[i]), f"t={i}: actions"
        assert torch.allclose(logp, ro.buf.logp[i, 0]) and torch.allclose(value, ro.buf.val[i, 0])
        owner_snap = sim.owner.clone()
        fuse_snap = sim.fuse.clone()
        hp0 = sim.hp[:, 0].clone()
        sim._rand_buf = torch.cat([dr.crate[i, 0].reshape(-1), dr.crate[i, 1].reshape(-1)])
        reward, done, info = sim.step(actions)
        dmg = (hp0 - sim.hp[:, 0]).clamp(min=0) > 0
        if i % 16 == 15:
            sim.flush_recycle()
        assert torch.equal(reward, ro.buf.rew[i]), f"t={i}: reward"
        assert torch.equal(done, ro.buf.done[i]), f"t={i}: done"
        # the reference's damage flag, read after the auto-reset step, is
        # the engine's "hp lost in an env that continued"
        assert torch.equal(dmg, ro.buf.dmg[i, :, 0]), f"t={i}: damage flag"
        # health statistics of the collect loop (train/ppo.py:277-287)
        died0 = info["died"][:, 0]
        own_live = ((owner_snap == 0) & (fuse_snap > 0)).flatten(1).sum(dim=1)
        st_sui += (died0 & (own_live > 0)).long()
        st_bmb += (a0[:, 1] == 1).long()
        h, w = cfg.height, cfg.width
        cy = sim.pos[:, 0, 0].floor().long().clamp(0, h - 1)
        cx = sim.pos[:, 0, 1].floor().long().clamp(0, w - 1)
        foot = obs[:, dng_ch].float().flatten(1).gather(1, (cy * w + cx).unsqueeze(1)).squeeze(1)
        st_dt += (foot > 0.04).long()
        st_dv += foot
        assert info["winner"].dtype == torch.bool and tuple(info["winner"].shape) == (n, p)
    ga, gb = sim_a.numpy_state(), sim_b.numpy_state()
    bad = [k for k in ga if not np.array_equal(ga[k], gb[k])]
    assert not bad, f"end state differs in {bad}"
    # the statistics read from the pokes equal the same sums over the
    # engine rollout's own buffers
    assert int(st_bmb.sum()) == int(ro.buf.act[:, :, 0, 1].sum())
    assert int(st_dt.sum()) > 0 and float(st_dv.sum()) > 0 and int(st_sui.sum()) >= 0


def test_batchedsim_graph_api():
    """BatchedSim's CUDA-graph surface (capture_graph / graph_refill_rand /
    graph_step / graph_actions, sim/torch_sim.py:649-699) on B200Sim: each
    replay equals an eager observe -> legal_mask -> step(auto_reset=False)
    of an identical sim fed the same actions and draws."""
    n = 128
    cfg, sim_g, _ = _make(n, 31)
    _, sim_e, _ = _make(n, 31)
    p = cfg.n_players
    d = "cuda"
    acts = torch.zeros((n, p, 2), dtype=torch.long, device=d)
    bufs = (torch.zeros((n,) + tuple(cfg.obs_shape), dtype=torch.float16, device=d),
            torch.zeros((n, p, 5), dtype=torch.bool, device=d),
            torch.zeros((n, p, 2), dtype=torch.bool, device=d),
            torch.zeros((n, p), dtype=torch.float32, device=d),
            torch.zeros((n,), dtype=torch.float32, device=d),
            torch.zeros((n, p), dtype=torch.float32, device=d))
    gen = torch.Generator(device=d).manual_seed(3)
    # the three warm-up ticks of capture_graph, mirrored on the eager sim
    sim_g.capture_graph(acts, *bufs)
    assert sim_g.graph_actions() is acts
    sim_e._rand_buf = torch.empty_like(sim_g._rand_buf)
    sim_e._rand_buf.copy_(sim_g._rand_buf)
    for _ in range(3):
        sim_e.observe()
        sim_e.legal_mask()
        sim_e.step(acts, auto_reset=False)
    for t in range(24):
        acts.copy_(torch.stack([torch.randint(0, 5, (n, p), device=d, generator=gen),
                                torch.randint(0, 2, (n, p), device=d, generator=gen)], -1))
        sim_g.graph_refill_rand()
        sim_e._rand_buf.copy_(sim_g._rand_buf)
        sim_g.graph_step()
        obs = sim_e.observe().clone()
        mm, bm = sim_e.legal_mask()
        r, done, info = sim_e.step(acts, auto_reset=False)
        torch.cuda.synchronize()
        assert torch.equal(bufs[0], obs) and torch.equal(bufs[1], mm) and torch.equal(bufs[2], bm)
        assert torch.equal(bufs[3], r) and torch.equal(bufs[4], done.float())
        assert torch.equal(bufs[5], info["winner"].float()), f"t={t}"
    ga, ge = sim_g.numpy_state(), sim_e.numpy_state()
    assert not [k for k in ga if not np.array_equal(ga[k], ge[k])]
