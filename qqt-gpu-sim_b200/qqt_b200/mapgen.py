"""Reset-time level generation on the host CPU generator.

Maps are generated once per episode on the host, as in the reference
(sim/mapgen.py, called from BatchedSim.reset_, sim/torch_sim.py:178-420);
the draws use the same torch CPU generator calls in the same order, so a
B200 engine and a reference simulator built with the same seed produce the
same maps.  Outputs are (count, H, W) bool tensors on the CPU.
"""

from __future__ import annotations

import torch

DIRS4 = ((-1, 0), (1, 0), (0, -1), (0, 1))


def _clear_around(mask: torch.Tensor, cells, h: int, w: int) -> None:
    for r, c in cells:
        mask[:, r, c] = False
        for dr, dc in DIRS4:
            if 0 <= r + dr < h and 0 <= c + dc < w:
                mask[:, r + dr, c + dc] = False


def walls(cfg, count: int, gen: torch.Generator, top_rows=None) -> torch.Tensor:
    """Permanent walls (sim/mapgen.py:15-62)."""
    h, w = cfg.height, cfg.width
    if cfg.map_mode == "corridor":
        if cfg.random_wall_rows:
            if top_rows is None:
                top_rows = torch.randint(0, cfg.top_wall_rows + 1, (count,), generator=gen)
            rows = torch.arange(h).view(1, -1)
            bot = cfg.top_wall_rows - top_rows
            band = (rows < top_rows.view(-1, 1)) | (rows >= (h - bot).view(-1, 1))
            wall = band.unsqueeze(2).expand(count, h, w).clone()
        else:
            wall = torch.zeros((count, h, w), dtype=torch.bool)
            wall[:, : cfg.top_wall_rows] = True
    elif cfg.wall_density <= 0:
        return torch.zeros((count, h, w), dtype=torch.bool)
    else:
        rr = torch.arange(h).view(-1, 1)
        cc = torch.arange(w).view(1, -1)
        pillars = (rr % 2 == 1) & (cc % 2 == 1)
        keep = torch.rand((count, h, w), generator=gen) < cfg.wall_density
        wall = pillars.unsqueeze(0) & keep
    _clear_around(wall, cfg.spawn_cells(), h, w)
    return wall


def open_obstacles(cfg, count: int, gen: torch.Generator) -> torch.Tensor:
    """0..open_obstacle_max single permanent walls per map (sim/mapgen.py:65-95)."""
    h, w = cfg.height, cfg.width
    wall = torch.zeros((count, h, w), dtype=torch.bool)
    k = cfg.open_obstacle_max
    if k <= 0 or count == 0:
        return wall
    n_obst = torch.randint(0, k + 1, (count,), generator=gen)
    order = torch.rand((count, h * w), generator=gen).argsort(dim=1)[:, :k]
    take = torch.arange(k).unsqueeze(0) < n_obst.unsqueeze(1)
    env = torch.arange(count).unsqueeze(1).expand(count, k)
    wall[env[take], (order // w)[take].clamp(0, h - 1), (order % w)[take].clamp(0, w - 1)] = True
    _clear_around(wall, cfg.spawn_cells(), h, w)
    return wall


def bricks(cfg, count: int, gen: torch.Generator, top_rows=None) -> torch.Tensor:
    """Destructible bricks for corridor maps (sim/mapgen.py:98-194)."""
    h, w = cfg.height, cfg.width
    if cfg.map_mode != "corridor":
        return torch.zeros((count, h, w), dtype=torch.bool)
    if cfg.random_wall_rows and top_rows is None:
        top_rows = torch.randint(0, cfg.top_wall_rows + 1, (count,), generator=gen)
    top = top_rows if cfg.random_wall_rows else None
    c0 = (w - cfg.corridor_width) // 2
    c1 = c0 + cfg.corridor_width
    rr = torch.arange(h).view(-1, 1)
    cc = torch.arange(w).view(1, -1)
    side = (cc < c0) | (cc >= c1)
    if top is None:
        out = (side & ~(rr < cfg.top_wall_rows)).expand(count, h, w).clone()
    else:
        in_top = torch.arange(h).view(1, -1) < top.view(-1, 1)
        out = (side.unsqueeze(0) & ~in_top.unsqueeze(2)).expand(count, h, w).clone()
    if cfg.wall_density > 0:
        edge = [c for c in (c0, c0 + 1, c1 - 2, c1 - 1) if c0 <= c < c1]
        ne = len(edge)
        if ne:
            if top is None:
                starts = (torch.rand((count, ne), generator=gen)
                          * (h - cfg.top_wall_rows - 4) + cfg.top_wall_rows).long()
            else:
                bot = cfg.top_wall_rows - top
                span = (h - bot.view(-1, 1) - 4 - top.view(-1, 1)).clamp(min=1)
                starts = (torch.rand((count, ne), generator=gen) * span
                          + top.view(-1, 1)).long()
            lens = 2 + (torch.rand((count, ne), generator=gen) * 3).long()
            on = torch.rand((count, ne), generator=gen) < cfg.wall_density
            rows = torch.arange(h).view(1, 1, -1)
            seg = on.unsqueeze(-1) & (rows >= starts.unsqueeze(-1)) \
                & (rows < (starts + lens).unsqueeze(-1))
            for i, col in enumerate(edge):
                out[:, :, col] |= seg[:, i]
        if c1 - c0 > 4:
            hs = (torch.rand((count,), generator=gen) * (c1 - c0 - 4) + c0).long()
            hl = 2 + (torch.rand((count,), generator=gen) * 3).long()
            hon = torch.rand((count,), generator=gen) < cfg.wall_density
            cols = torch.arange(c0, c1).view(1, -1)
            hseg = hon.view(-1, 1) & (cols >= hs.view(-1, 1)) & (cols < (hs + hl).view(-1, 1))
            if top is None:
                for r in range(cfg.top_wall_rows, cfg.top_wall_rows + min(2, h - cfg.top_wall_rows)):
                    out[:, r, c0:c1] |= hseg
            else:
                env = torch.arange(count).view(-1, 1).expand(count, 2)
                hr = top.view(-1, 1) + torch.arange(2).view(1, -1)
                out[env, hr, c0:c1] |= hseg.unsqueeze(1).expand(count, 2, c1 - c0)
    _clear_around(out, cfg.spawn_cells(), h, w)
    return out


def ring_walls(cfg, count: int) -> torch.Tensor:
    """Central permanent block of the ring map (sim/mapgen.py:230-242)."""
    h, w = cfg.height, cfg.width
    r0 = (h - cfg.ring_center_h) // 2
    c0 = (w - cfg.ring_center_w) // 2
    wall = torch.zeros((count, h, w), dtype=torch.bool)
    wall[:, r0:r0 + cfg.ring_center_h, c0:c0 + cfg.ring_center_w] = True
    return wall


def ring_bricks(cfg, count: int, gen: torch.Generator) -> torch.Tensor:
    """Sparse bricks on the band around the ring block (sim/mapgen.py:197-227)."""
    h, w = cfg.height, cfg.width
    r0 = (h - cfg.ring_center_h) // 2
    c0 = (w - cfg.ring_center_w) // 2
    r1, c1 = r0 + cfg.ring_center_h, c0 + cfg.ring_center_w
    band = torch.zeros((count, h, w), dtype=torch.bool)
    band[:, r0 - 1:r1 + 1, c0 - 1:c1 + 1] = True
    band[:, r0:r1, c0:c1] = False
    draw = torch.rand((count, h, w), generator=gen)
    out = band & (draw < cfg.ring_brick_density)
    _clear_around(out, cfg.ring_spawn_cells(), h, w)
    return out


def open_spawns(cfg) -> list[tuple[float, float]]:
    h, w = float(cfg.height), float(cfg.width)
    row = (h - 1) / 2.0 + 0.5
    return [(row, (w - 1) * (i + 1) / (cfg.n_players + 1) + 0.5) for i in range(cfg.n_players)]


def open_cross_cells(cfg) -> list[tuple[int, int]]:
    """Central cross band of open maps minus the open spawns' neighbourhoods
    (sim/torch_sim.py:465-506)."""
    h, w = cfg.height, cfg.width
    near = set()
    for y, x in open_spawns(cfg):
        r, c = int(y), int(x)
        near.add((r, c))
        for dr, dc in DIRS4:
            if 0 <= r + dr < h and 0 <= c + dc < w:
                near.add((r + dr, c + dc))
    cy, cx = (h - 1) // 2, (w - 1) // 2
    cross = {(r, c) for c in range(w) for r in (cy - 1, cy)} \
        | {(r, c) for r in range(h) for c in (cx - 1, cx)}
    return sorted(cross - near)
