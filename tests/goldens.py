"""Loading helpers for the golden vectors in tests/golden/ (test-only)."""

from __future__ import annotations

import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

STATE_KEYS = ("wall", "brick", "crate", "recycle", "fuse", "owner", "bomb_blast",
              "pos", "alive", "hp", "since_bomb", "t", "bombs_cap", "blast_cap",
              "spd_g", "invuln", "pending_lost", "combo", "last_hit", "lo_bombs",
              "lo_blast", "lo_spd", "crate_prob", "hazard")


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def init_state(g, prefix="init_"):
    return {k: np.array(g[prefix + k], copy=True) for k in STATE_KEYS}


def state_at(g, t, wall):
    st = {k: np.array(g["st_" + k][t], copy=True) for k in STATE_KEYS if k != "wall"}
    st["wall"] = wall.copy()
    return st


def reset_state(g, i, wall):
    st = {k: np.array(g[f"reset{i}_{k}"], copy=True) for k in STATE_KEYS if k != "wall"}
    st["wall"] = wall.copy()
    return st


def bot_draws(g, pid, t):
    """List of (kind, array) draws seat `pid` made at tick t, in call order."""
    key = f"draw_p{pid}_index"
    if key not in g:
        return []
    idx = g[key]
    rows = idx[idx[:, 0] == t]
    return [("rand" if k == 0 else "randint", g[f"draw_p{pid}_t{t}_{j}"])
            for _, j, k in rows]


def compare_state(ref, got, keys=None, envs=None):
    """Names of state entries that differ (floats compared exactly)."""
    bad = []
    for k in keys or STATE_KEYS:
        a, b = np.asarray(ref[k]), np.asarray(got[k])
        if envs is not None:
            a, b = a[envs], b[envs]
        if a.shape != b.shape or not np.array_equal(a, b):
            bad.append(k)
    return bad
