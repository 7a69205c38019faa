"""GPU parity of the rollout tick protocol as the benchmark runs it
(train/ppo.py:213-271): observe -> legal masks -> MLP learner (seat 0) on a
side stream || astar bot (seat 1) -> step(auto_reset) -> crate recycling
every 16 ticks, all through qqt_b200.rollout.

* eager ticks vs the oracle protocol, tick by tick: observation rows, masks,
  both seats' actions, rewards and done flags bit-exact (log-prob and value
  within the policy tolerance); the device crate recycling is checked against
  the oracle's restatement of its counter-based draws;
* a captured CUDA graph of the same rollout, replayed from the same start,
  reproduces the eager buffers bit for bit;
* two env groups on their own streams (RolloutGroups) equal the two groups
  run one after the other.
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
    from qqt_b200.sim import B200Sim, _recycle_exclusion, tile_flags


@pytest.fixture(autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    yield
    torch.cuda.synchronize()
    assert _capi.device_error() == 0, "device error word set"


def _make(n, T, seed, pol=None):
    """One env group exactly as the benchmark builds it, with explicit
    ticker start draws and generated rollout draws."""
    cfg = SimConfig(**scenarios.CFG2)
    tmpl = scenarios.corridor_template(cfg, n, seed)
    sim = B200Sim(cfg, n, device="cuda", seed=seed, template=tmpl)
    sim.set_template(tmpl, apply=False, seed=seed, swap_spawns=False)
    if pol is None:
        pol = B200Policy(init_params(cfg.obs_shape, "mlp", seed=1), cfg.obs_shape, 2, seats=(0,))
    bot = AstarBot(sim, mode=True)
    rng = np.random.default_rng(seed)
    bot.mode = torch.from_numpy(rng.integers(0, 2, n)).cuda()
    bot.timer = torch.from_numpy(rng.integers(60, 240, n)).cuda()
    ro = Rollout(sim, pol, bot, T=T)
    ro.draws.generate(torch.Generator(device="cuda").manual_seed(seed))
    return cfg, sim, pol, bot, ro


def _snapshot(sim, bot):
    return (sim.numpy_state(), bot.mode.clone(), bot.timer.clone(), bot.calls,
            getattr(sim, "_flush_count", 0))


def _restore(sim, bot, snap):
    st, mode, timer, calls, flush_count = snap
    sim.load_numpy_state(st)
    bot.mode.copy_(mode)
    bot.timer.copy_(timer)
    bot.calls = calls
    sim._flush_count = flush_count


def _buffers(ro):
    b = ro.buf
    return {k: getattr(b, k).clone() for k in ("obs_rows", "mm", "bm", "act", "logp", "val",
                                                "rew", "done", "dmg")}


def test_rollout_ticks_vs_oracle():
    n, T, p = 64, 48, 2
    cfg, sim, pol, bot, ro = _make(n, T, seed=5)
    st = sim.numpy_state()
    ticker = O.ModeTicker(bot.mode.cpu().numpy(), bot.timer.cpu().numpy())
    params = {k: v.cpu().numpy() for k, v in pol.params.items()}
    dr = {k: getattr(ro.draws, k).cpu().numpy()
          for k in ("u_net", "noise", "crate", "tick_mode", "tick_timer")}
    excl = _recycle_exclusion(cfg)
    k_in = cfg.obs_shape[0] * cfg.height * cfg.width
    for t in range(T):
        ro.tick(t)
        torch.cuda.synchronize()
        obs, _ = O.observe(cfg, st)
        obs16 = obs.astype(np.float16).reshape(n, -1)
        mm, bm = O.legal_mask(cfg, st)
        got = ro.buf.obs_rows[t, :, :k_in].cpu().numpy()
        assert np.array_equal(got.view(np.uint16), obs16.view(np.uint16)), f"t={t} obs"
        assert np.array_equal(ro.buf.mm[t].cpu().numpy(), mm), f"t={t} move mask"
        assert np.array_equal(ro.buf.bm[t].cpu().numpy(), bm), f"t={t} bomb mask"
        obs32 = obs16.astype(np.float32).reshape((n,) + tuple(cfg.obs_shape))
        u = dr["u_net"][t, 0]
        a0, lp0, v0, _, _ = O.mlp_act(params, obs32, mm[:, 0], bm[:, 0], 0, p, u[:, 0], u[:, 1])
        k = ticker.tick + 1
        j = (k // 16) % dr["tick_mode"].shape[0]
        mode = ticker.advance(dr["tick_mode"][j], dr["tick_timer"][j])
        a1 = O.astar_attack(cfg, st, obs32[:, 2 * p + 1], mm[:, 1], bm[:, 1], 1, dr["noise"][t],
                            mode=mode)
        acts = ro.buf.act[t].cpu().numpy()
        assert int((acts[:, 0] != a0).any(-1).sum()) == 0, f"t={t} learner actions"
        assert np.array_equal(acts[:, 1], a1), f"t={t} astar actions"
        assert np.abs(ro.buf.logp[t, 0].cpu().numpy() - lp0).max() <= 1e-3
        assert np.abs(ro.buf.val[t, 0].cpu().numpy() - v0).max() <= 2e-3 * max(np.abs(v0).max(), 1e-3)
        hp0 = st["hp"].astype(np.int32)
        rew, done, _ = O.step(cfg, st, acts, dr["crate"][t, 0], dr["crate"][t, 1])
        dmg = ((hp0 - st["hp"].astype(np.int32)) > 0) & ~done[:, None]
        assert np.array_equal(ro.buf.dmg[t].cpu().numpy(), dmg), f"t={t} damage flags"
        assert not done.any(), "no episode ends inside this rollout (resets not exercised here)"
        assert np.array_equal(ro.buf.rew[t].cpu().numpy(), rew), f"t={t} reward"
        assert np.array_equal(ro.buf.done[t].cpu().numpy(), done), f"t={t} done"
        if t % 16 == 15:
            O.flush_recycle_keyed(cfg, st, excl, sim._flush_seed, sim._flush_count)
        got_st = sim.numpy_state()
        bad = [k for k in O.STATE_KEYS if k in got_st and not np.array_equal(got_st[k], st[k])]
        assert not bad, f"t={t} state differs: {bad}"


def test_device_flush_vs_keyed_restatement():
    """k_flush_recycle on states with lost attribute layers for both seats."""
    n = 96
    cfg, sim, pol, bot, ro = _make(n, 16, seed=9)
    rng = np.random.default_rng(3)
    st = sim.numpy_state()
    st["pending_lost"] = rng.integers(0, 4, (n, 2)).astype(np.int64)
    st["t"] = rng.integers(0, 1000, n).astype(np.int64)
    st["brick"] &= rng.random(st["brick"].shape) < 0.5
    sim.load_numpy_state(st)
    for count in (1, 2):
        sim.flush_recycle(on_device=True)
        torch.cuda.synchronize()
        O.flush_recycle_keyed(cfg, st, _recycle_exclusion(cfg), sim._flush_seed, count)
        got = sim.numpy_state()
        for k in ("crate", "recycle", "pending_lost"):
            assert np.array_equal(got[k], st[k]), f"flush {count}: {k}"
        st["pending_lost"] = rng.integers(0, 3, (n, 2)).astype(np.int64)
        sim.load_numpy_state({"pending_lost": st["pending_lost"]})


def test_graph_replay_equals_eager():
    n, T = 256, 32
    cfg, sim, pol, bot, ro = _make(n, T, seed=11)
    ro.tick(0)                        # one-time first-step set-up, outside the compared run
    snap = _snapshot(sim, bot)
    ro.collect()
    torch.cuda.synchronize()
    eager = _buffers(ro)
    end_eager = sim.numpy_state()
    _restore(sim, bot, snap)
    ro.capture()
    ro.replay()
    torch.cuda.synchronize()
    graph = _buffers(ro)
    for k in eager:
        assert torch.equal(eager[k], graph[k]), f"graph replay differs in {k}"
    end_graph = sim.numpy_state()
    for k in end_eager:
        assert np.array_equal(end_eager[k], end_graph[k]), f"end state {k}"


def test_groups_equal_sequential_groups():
    n, T = 128, 32
    made = [_make(n, T, seed=21 + g) for g in range(2)]
    pol = made[0][2]
    made[1] = _make(n, T, seed=22, pol=pol)
    for m in made:
        m[4].tick(0)
    snaps = [_snapshot(m[1], m[3]) for m in made]
    for m in made:
        m[4].collect()
    torch.cuda.synchronize()
    seq = [_buffers(m[4]) for m in made]
    for m, s in zip(made, snaps):
        _restore(m[1], m[3], s)
    grp = RolloutGroups([m[4] for m in made])
    grp.capture()
    grp.replay()
    torch.cuda.synchronize()
    for g, m in enumerate(made):
        got = _buffers(m[4])
        for k in got:
            assert torch.equal(seq[g][k], got[k]), f"group {g}: {k}"


def test_step_observe_equals_step_then_observe():
    """qqt_step_observe's rows and masks equal observe_and_mask of the
    post-step state, for envs that continue and envs that time out and are
    reset to their template on the device."""
    n, T = 96, 40
    cfg, sim, pol, bot, ro = _make(n, T, seed=31)
    for t in range(24):                       # mid-game: bombs, flames, crates
        ro.tick(t)
    st = sim.numpy_state()
    st["t"][::2] = cfg.max_steps - 1          # every other env ends on this step
    sim.load_numpy_state({"t": st["t"]})
    acts = ro.buf.act[23].clone()
    draws = (ro.draws.crate[23, 0], ro.draws.crate[23, 1])
    snap = _snapshot(sim, bot)
    rows = torch.zeros_like(ro.buf.obs_rows[0])
    mm = torch.zeros_like(ro.buf.mm[0])
    bm = torch.zeros_like(ro.buf.bm[0])
    tiles = torch.zeros((n, 4), dtype=torch.int32, device="cuda")
    _, done_f, _ = sim.step(acts, auto_reset=True, crate_draws=draws,
                            next_obs=(rows, mm, bm, tiles))
    fused_state = sim.numpy_state()
    done_f = done_f.clone()
    _restore(sim, bot, snap)
    _, done_s, _ = sim.step(acts, auto_reset=True, crate_draws=draws)
    ref_rows = torch.zeros_like(rows)
    ref_mm, ref_bm = torch.zeros_like(mm), torch.zeros_like(bm)
    sim.observe_and_mask(ref_rows, ref_mm, ref_bm, danger=False)
    torch.cuda.synchronize()
    assert bool(done_f[::2].all()) and torch.equal(done_f, done_s)
    got = sim.numpy_state()
    for k in fused_state:
        assert np.array_equal(fused_state[k], got[k]), f"state {k}"
    assert torch.equal(rows.view(torch.int16), ref_rows.view(torch.int16)), "observation rows"
    assert torch.equal(mm, ref_mm) and torch.equal(bm, ref_bm), "legal masks"
    assert torch.equal(tiles, tile_flags(rows)), "K-tile flags of the written rows"


@pytest.mark.parametrize("on_device", [True, False])
def test_flush_rewrites_the_crate_channel_of_fused_rows(on_device):
    """A crate recycle changes only the observation's crate channel: the
    step's fused next-tick rows, after flush_recycle(obs_rows=...) rewrites
    that channel, equal a fresh observe of the post-recycle state (device
    and host recycle paths)."""
    n = 96
    cfg, sim, pol, bot, ro = _make(n, 40, seed=13)
    for t in range(20):
        ro.tick(t)
    rng = np.random.default_rng(8)
    lost = rng.integers(0, 4, (n, 2)).astype(np.int64)
    sim.load_numpy_state({"pending_lost": lost})
    rows = torch.zeros_like(ro.buf.obs_rows[0])
    mm = torch.zeros_like(ro.buf.mm[0])
    bm = torch.zeros_like(ro.buf.bm[0])
    tiles = torch.zeros((n, 4), dtype=torch.int32, device="cuda")
    sim.step(ro.buf.act[19].clone(), auto_reset=True,
             crate_draws=(ro.draws.crate[19, 0], ro.draws.crate[19, 1]),
             next_obs=(rows, mm, bm, tiles))
    before = sim.numpy_state()["crate"].copy()
    sim.flush_recycle(on_device=on_device, obs_rows=rows, obs_tiles=tiles)
    ref_rows = torch.zeros_like(rows)
    ref_mm, ref_bm = torch.zeros_like(mm), torch.zeros_like(bm)
    sim.observe_and_mask(ref_rows, ref_mm, ref_bm, danger=False)
    torch.cuda.synchronize()
    after = sim.numpy_state()["crate"]
    assert (after.astype(int) - before.astype(int)).sum() > 0, "the recycle dropped crates"
    assert torch.equal(rows.view(torch.int16), ref_rows.view(torch.int16))
    assert torch.equal(mm, ref_mm) and torch.equal(bm, ref_bm)
    # the K-tile flags still cover every nonzero tile of the rewritten rows
    assert not bool((tile_flags(rows) & ~tiles).any()), "a nonzero K tile lost its flag"


def test_rollout_tile_flags_cover_the_rows():
    """Every tick's K-tile flags in a rollout buffer cover the tick's rows
    (the policy skips unflagged tiles); they are exact for rows the step
    wrote, and over-report only the crate channel after a crate recycle."""
    n, T = 256, 40
    cfg, sim, pol, bot, ro = _make(n, T, seed=17)
    ro.collect()
    torch.cuda.synchronize()
    for t in range(T):
        exact = tile_flags(ro.buf.obs_rows[t])
        flags = ro.buf.tiles[t]
        assert not bool((exact & ~flags).any()), f"t={t}: a nonzero K tile lost its flag"
        if t % ro.flush_every != 0:
            assert torch.equal(flags, exact), f"t={t}: K-tile flags"


def test_double_buffered_graphs_read_their_own_draws():
    """capture(double_buffer=True): the second graph reads the second set of
    draw buffers; with the same draws in both sets the two graphs produce
    the same rollout, and new draws in the second set change only what the
    second graph produces."""
    n, T = 128, 32
    made = [_make(n, T, seed=41 + g) for g in range(2)]
    made[1] = _make(n, T, seed=42, pol=made[0][2])
    for m in made:
        m[4].tick(0)
    snaps = [_snapshot(m[1], m[3]) for m in made]
    grp = RolloutGroups([m[4] for m in made])
    grp.capture(double_buffer=True)
    assert len(grp.graphs) == 2 and len(grp.draw_sets) == 2

    def run(which):
        for m, s in zip(made, snaps):
            _restore(m[1], m[3], s)
        grp.replay(which)
        torch.cuda.synchronize()
        return [_buffers(m[4]) for m in made]

    a = run(0)
    b = run(1)
    for g in range(2):
        for k in a[g]:
            assert torch.equal(a[g][k], b[g][k]), f"group {g}: {k}"
    gen = torch.Generator(device="cuda").manual_seed(99)
    for d in grp.draw_sets[1]:
        d.generate(gen)
    c = run(1)
    assert any(not torch.equal(a[g]["act"], c[g]["act"]) for g in range(2))
    again = run(0)
    for g in range(2):
        for k in a[g]:
            assert torch.equal(a[g][k], again[g][k]), f"group {g}: {k} (set 0 untouched)"
