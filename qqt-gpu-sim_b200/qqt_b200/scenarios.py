"""Seeded map templates and start states for the benchmark configurations.

The benchmark configurations describe their own maps instead of the
reference's random level generator:
  * "open border": a ring of permanent walls on rows/cols 0 and H-1, no
    bricks, the reference's open spawns (sim/config.py:581-584);
  * "pillar corridor": border ring, permanent pillars at every (r, c) with
    both coordinates even in 2..H-3, bricks with probability p on every other
    free cell except the 3-cell L at each inner corner, spawns at the inner
    corners (1.5, 1.5) and (H-1.5, W-1.5);
  * "bomb stress": the open-border map with 20-40 bombs per env at uniform
    free cells, fuse U{1..30}, blast U{1..5}, owner U{0,1}.

Everything is numpy on the host; the engine uploads the result once.
"""

from __future__ import annotations

import numpy as np

from .config import SimConfig


def border_walls(h: int, w: int) -> np.ndarray:
    wall = np.zeros((h, w), dtype=bool)
    wall[0, :] = wall[-1, :] = True
    wall[:, 0] = wall[:, -1] = True
    return wall


def corner_l_cells(h: int, w: int) -> set[tuple[int, int]]:
    cells = set()
    for r, c, dr, dc in ((1, 1, 1, 1), (1, w - 2, 1, -1),
                         (h - 2, 1, -1, 1), (h - 2, w - 2, -1, -1)):
        cells |= {(r, c), (r + dr, c), (r, c + dc)}
    return cells


def pillar_corridor(n: int, h: int, w: int, seed: int, brick_p: float = 0.7):
    """(wall (n,h,w), brick (n,h,w)) for the pillar corridor template."""
    wall = border_walls(h, w)
    for r in range(2, h - 2, 2):
        for c in range(2, w - 2, 2):
            wall[r, c] = True
    keep_free = np.zeros((h, w), dtype=bool)
    for r, c in corner_l_cells(h, w):
        keep_free[r, c] = True
    rng = np.random.default_rng(seed)
    draw = rng.random((n, h, w)) < brick_p
    brick = draw & ~wall[None] & ~keep_free[None]
    return np.broadcast_to(wall, (n, h, w)).copy(), brick


def corner_spawns(cfg: SimConfig) -> list[tuple[float, float]]:
    h, w = float(cfg.height), float(cfg.width)
    corners = [(1.5, 1.5), (h - 1.5, w - 1.5), (1.5, w - 1.5), (h - 1.5, 1.5)]
    return corners[: cfg.n_players]


def open_spawns(cfg: SimConfig) -> list[tuple[float, float]]:
    h, w = float(cfg.height), float(cfg.width)
    row = (h - 1) / 2.0 + 0.5
    return [(row, (w - 1) * (i + 1) / (cfg.n_players + 1) + 0.5)
            for i in range(cfg.n_players)]


def bomb_stress(n: int, cfg: SimConfig, seed: int, lo: int = 20, hi: int = 40):
    """(fuse, owner, bomb_blast) planes (n,h,w) for the chain/danger stress case."""
    h, w = cfg.height, cfg.width
    wall = border_walls(h, w)
    free = np.flatnonzero(~wall.reshape(-1))
    rng = np.random.default_rng(seed)
    fuse = np.zeros((n, h * w), dtype=np.int16)
    owner = np.full((n, h * w), -1, dtype=np.int8)
    blast = np.zeros((n, h * w), dtype=np.int16)
    counts = rng.integers(lo, hi + 1, size=n)
    for e in range(n):
        cells = rng.choice(free, size=int(counts[e]), replace=False)
        fuse[e, cells] = rng.integers(1, 31, size=cells.size)
        blast[e, cells] = rng.integers(1, 6, size=cells.size)
        owner[e, cells] = rng.integers(0, 2, size=cells.size)
    return (fuse.reshape(n, h, w), owner.reshape(n, h, w), blast.reshape(n, h, w))


# Benchmark configurations (SimConfig keyword arguments).
CFG1 = dict(height=13, width=13, n_players=2, map_mode="open", speed=3.0, tick_hz=10)
CFG2 = dict(map_mode="corridor", open_fraction=0.0, speed=3.0, max_steps=1800)


def open_border_template(cfg, n: int) -> dict:
    """Per-env template of the cfg1 workload: the open-border map, the
    reference's open spawns and the start attributes its open-map reset
    gives both seats at opponent boost 0 (bombs max_bombs, blast `blast`,
    speed 1.0: sim/torch_sim.py:200-224); crate_prob keeps the construction
    value (an open-map reset leaves it alone).  With swap_spawns the device
    reset swaps the two spawns with probability 1/2, as the reference's
    open-map reset does (sim/torch_sim.py:229-240)."""
    p, h, w = cfg.n_players, cfg.height, cfg.width
    wall = np.broadcast_to(border_walls(h, w), (n, h, w)).copy()
    spawn = np.broadcast_to(np.array(cfg.spawn_pos(), np.float32), (n, p, 2)).copy()
    return {"wall": wall, "brick": np.zeros_like(wall), "spawn": spawn,
            "bombs_cap": np.full((n, p), cfg.max_bombs, np.int64),
            "blast_cap": np.full((n, p), cfg.blast, np.int64),
            "spd": np.full((n, p), 1.0, np.float32),
            "crate_prob": np.full((n,), cfg.growth_crate_prob, np.float32)}


def corridor_template(cfg, n: int, seed: int) -> dict:
    """Per-env map template of the cfg2 workload: border walls, permanent
    pillars, bricks with p=0.7 (corner L cells kept free), corner spawns and
    the growth start values; fed to `B200Sim(template=...)` and applied again
    by every device auto-reset."""
    p = cfg.n_players
    wall, brick = pillar_corridor(n, cfg.height, cfg.width, seed=seed)
    spawn = np.broadcast_to(np.array(corner_spawns(cfg), np.float32), (n, p, 2)).copy()
    return {"wall": wall, "brick": brick, "spawn": spawn,
            "bombs_cap": np.full((n, p), cfg.growth_bombs_start, np.int64),
            "blast_cap": np.full((n, p), cfg.growth_blast_start, np.int64),
            "spd": np.full((n, p), cfg.growth_speed_start, np.float32),
            "crate_prob": np.full((n,), cfg.growth_crate_prob, np.float32)}
