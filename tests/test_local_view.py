"""LSTM local-view features (sim/obs.py:241-340): the oracle against the
reference's own outputs (tests/golden/local_view.npz) on the CPU, and the
device kernel (`qqt_local_view`) against the oracle on the GPU.

Everything is compared bit for bit except one thing the reference leaves
open: cells at equal L1 distance in the bomb slots come out in torch.topk's
order, which it does not specify (CPU and CUDA differ), and slots past the
last live bomb hold whichever non-bomb cells topk returns.  For those the
test checks what is defined: the same count of bomb slots, the same sorted
distances, the same cells for every distance class that fits entirely,
live bombs at the stated distance in a class cut by the slot count, and
empty type / padding fields in the filler slots.  The oracle and the
kernel use one order (ascending flat cell index within a distance) and
match each other exactly.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import goldens as G
from oracle import qqt_oracle as O
from qqt_b200.config import SimConfig

CFGS = {"p2": dict(map_mode="corridor", speed=3.0, max_steps=1800),
        "p3": dict(map_mode="open", n_players=3)}


def _case(tag):
    g = G.load("local_view")
    st = {k.split("__", 1)[1]: g[k] for k in g if k.startswith(tag + "__") and k.count("__") == 1}
    return SimConfig(**CFGS[tag]), st, g


def _bomb_slots_match(ref, ours, fuse, cell, n_opp):
    """ref / ours: (MAX_T, 6) rel rows of one (env, player)."""
    w = fuse.shape[1]
    rb, ob = ref[n_opp:].astype(np.float64), ours[n_opp:].astype(np.float64)
    assert np.array_equal(rb[:, 3], ob[:, 3])                 # bomb / filler pattern
    live = rb[:, 3] > 0
    assert np.all(rb[~live][:, [2, 4, 5]] == 0) and np.all(ob[~live][:, [2, 4, 5]] == 0)
    d_ref = np.abs(rb[live, 0]) + np.abs(rb[live, 1])
    d_our = np.abs(ob[live, 0]) + np.abs(ob[live, 1])
    assert np.array_equal(d_ref, d_our) and np.all(np.diff(d_ref) >= 0)
    cy, cx = int(cell[0]), int(cell[1])
    bombs = np.argwhere(fuse > 0)
    dist_all = np.abs(bombs[:, 0] - cy) + np.abs(bombs[:, 1] - cx)
    for d in np.unique(d_ref):
        sel_r = {(int(a), int(b)) for a, b in rb[live][d_ref == d][:, :2]}
        sel_o = {(int(a), int(b)) for a, b in ob[live][d_our == d][:, :2]}
        n_class = int((dist_all == d).sum())
        if n_class == len(sel_r):                               # whole class inside
            assert sel_r == sel_o
        for bx, by in sel_o:                                    # cut class: valid bombs
            assert fuse[cy + by, cx + bx] > 0 and abs(bx) + abs(by) == d
    assert rb[:, 3].sum() == min(len(bombs), len(rb))
    _ = w


@pytest.mark.parametrize("tag", ["p2", "p3"])
@pytest.mark.parametrize("only_p0", [False, True])
def test_oracle_matches_reference(tag, only_p0):
    cfg, st, g = _case(tag)
    sfx = "p0" if only_p0 else "all"
    obs = g[f"{tag}__obs"]
    loc, rel, glob = O.local_view_features(cfg, obs, st["pos"], st["alive"], st["t"], st["fuse"],
                                           st["hp"], only_p0)
    assert loc.dtype == obs.dtype and rel.dtype == obs.dtype and glob.dtype == obs.dtype
    assert np.array_equal(loc, g[f"{tag}__{sfx}__local"])
    assert np.array_equal(glob, g[f"{tag}__{sfx}__glob"])
    rref = g[f"{tag}__{sfx}__rel"]
    n_opp = cfg.n_players - 1
    assert np.array_equal(rel[:, :, :n_opp], rref[:, :, :n_opp])
    cell = np.floor(st["pos"]).astype(np.int64)
    for e in range(rel.shape[0]):
        for m in range(rel.shape[1]):
            _bomb_slots_match(rref[e, m], rel[e, m], st["fuse"][e], cell[e, m], n_opp)


def test_golden_exercises_ties_and_filler():
    """The fixture holds envs with no bombs, with fewer bombs than slots, with
    more, and players whose window leaves the grid."""
    _, st, g = _case("p2")
    nb = (st["fuse"] > 0).reshape(len(st["fuse"]), -1).sum(1)
    assert (nb == 0).any() and ((nb > 0) & (nb < 9)).any() and (nb > 9).any()
    cell = np.floor(st["pos"]).astype(np.int64)
    assert (cell.min(-1) < 3).any()


@pytest.mark.gpu
@pytest.mark.parametrize("tag", ["p2", "p3"])
@pytest.mark.parametrize("only_p0", [False, True])
def test_kernel_matches_oracle_and_reference(tag, only_p0):
    """qqt_local_view on the golden states and the reference's own fp16
    observations: bit-exact against the oracle (same tie order), and
    against the reference's outputs as above."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from qqt_b200 import _capi
    from qqt_b200.sim import B200Sim
    cfg, st, g = _case(tag)
    n = st["pos"].shape[0]
    sim = B200Sim(cfg, n, device="cuda", seed=0)
    sim.load_numpy_state({k: st[k] for k in ("wall", "brick", "fuse", "owner", "bomb_blast",
                                             "pos", "alive", "hp", "t")})
    obs = g[f"{tag}__obs"]
    rows = torch.zeros((n, sim.obs_stride), dtype=torch.float16, device="cuda")
    rows[:, :obs[0].size] = torch.from_numpy(obs.reshape(n, -1)).cuda()
    loc, rel, glob = sim.local_view_features(rows, only_p0=only_p0)
    torch.cuda.synchronize()
    assert _capi.device_error() == 0
    loc, rel, glob = (t.cpu().numpy() for t in (loc, rel, glob))
    ol, orl, og = O.local_view_features(cfg, obs, st["pos"], st["alive"], st["t"], st["fuse"],
                                        st["hp"], only_p0)
    assert np.array_equal(loc, ol) and np.array_equal(rel, orl) and np.array_equal(glob, og)
    sfx = "p0" if only_p0 else "all"
    assert np.array_equal(loc, g[f"{tag}__{sfx}__local"])
    assert np.array_equal(glob, g[f"{tag}__{sfx}__glob"])
    n_opp = cfg.n_players - 1
    rref = g[f"{tag}__{sfx}__rel"]
    assert np.array_equal(rel[:, :, :n_opp], rref[:, :, :n_opp])
    cell = np.floor(st["pos"]).astype(np.int64)
    for e in range(n):
        for m in range(rel.shape[1]):
            _bomb_slots_match(rref[e, m], rel[e, m], st["fuse"][e], cell[e, m], n_opp)
    # the view observe() returns is accepted as well
    sim._obs.copy_(rows)
    l2, r2, g2 = sim.local_view_features(sim.obs_view(), only_p0=only_p0)
    assert np.array_equal(l2.cpu().numpy(), loc) and np.array_equal(g2.cpu().numpy(), glob)
