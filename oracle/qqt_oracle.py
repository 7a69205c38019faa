"""CPU oracle for the rollout hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference algorithms that the B200 kernels
replace.  It exists to check the CUDA path (tests/, __graft_entry__.smoke())
and to time the CPU baseline leg of bench.py; the product never imports it.

Parity pin: every function here is checked against golden vectors produced by
running the reference implementation itself (tests/golden/make_golden.py,
which imports the reference from its source tree and feeds it the same random
draws) and against the reference's committed known-answer files
(deploy/ref_state.json, deploy/sweep_states.json).

Formulation: the reference propagates fronts by shifting whole planes one cell
at a time.  Here each target cell instead looks back k cells along a ray
(`_behind`) and keeps an "open path" mask, which yields the same coverage /
danger values.  All float32 arithmetic follows the reference's operation
order so that positions, rewards and danger compare bit-exactly; the policy
forward is computed in float64 as the accuracy reference for the fp16/fp32
GPU path.

Layouts are the reference's env-major ones: planes (N, H, W), per-player
(N, P), positions (N, P, 2).
"""

from __future__ import annotations

import numpy as np

F32 = np.float32
EPS = F32(1e-4)                 # sim/move.py:33
DIRS4 = ((-1, 0), (1, 0), (0, -1), (0, 1))   # up, down, left, right
MOVE_IDLE = 4


# ----------------------------------------------------------------- helpers

def _behind(x: np.ndarray, dr: int, dc: int, k: int, fill) -> np.ndarray:
    """out[..., i, j] = x[..., i - k*dr, j - k*dc]; `fill` outside the grid.

    The value of the cell k steps *behind* (i, j) for a ray travelling in
    direction (dr, dc).
    """
    out = np.full_like(x, fill)
    h, w = x.shape[-2], x.shape[-1]
    sr, sc = dr * k, dc * k
    i0, i1 = max(0, sr), min(h, h + sr)
    j0, j1 = max(0, sc), min(w, w + sc)
    if i0 < i1 and j0 < j1:
        out[..., i0:i1, j0:j1] = x[..., i0 - sr:i1 - sr, j0 - sc:j1 - sc]
    return out


def blast_map(bomb_blast: np.ndarray, default_blast: int) -> np.ndarray:
    """Per-cell blast length; 0 falls back to cfg.blast (sim/torch_sim.py:727-730)."""
    return np.where(bomb_blast > 0, bomb_blast.astype(np.int64), default_blast)


def fuse_weight(fuse: np.ndarray, fuse_max: int) -> np.ndarray:
    """Danger weight of a bomb: clamp(1 - (f-1)/FUSE, 0)^2 (sim/blast.py:218-220)."""
    raw = F32(1.0) - (fuse.astype(F32) - F32(1.0)) / F32(fuse_max)
    raw = np.maximum(raw, F32(0.0))
    return np.where(fuse > 0, raw * raw, F32(0.0)).astype(F32)


# ------------------------------------------------------------ fire / chains

def fire_cover(sources, wall, solid, blast, brick, max_b: int) -> np.ndarray:
    """Cross-shaped flame coverage from `sources` (sim/blast.py:43-98).

    A cell c is covered when it is a firing source, or when some firing
    source s = c - k*d (k <= blast(s)) sees it along direction d with every
    cell strictly between them non-wall and non-solid, and c is not a wall.
    Solid cells (live bombs, bricks) are covered but stop the ray.

    `max_b` is the reference's blast-tier bound: a source whose blast
    exceeds it emits no rays (only its own cell burns), exactly like the
    tier loop `for b in 1..b_max` of sim/blast.py:90-97.
    """
    seed = sources & ~wall & ~brick
    cov = seed.copy()
    clear = ~wall & ~solid
    emit = seed & (blast <= max_b)
    for dr, dc in DIRS4:
        open_path = np.ones_like(seed)
        for k in range(1, max_b + 1):
            src = _behind(emit & (blast >= k), dr, dc, k, False)
            cov |= open_path & src & ~wall
            open_path &= _behind(clear, dr, dc, k, False)
    return cov


def resolve_explosions(fuse, owner, wall, blast, brick, rounds: int, tier_cap=None):
    """(covered, triggered) after the initial blast plus `rounds` chain rounds.

    sim/blast.py:101-155 with the fixed round count used on the rollout path
    (min(max_chain-1, chain_cap_rounds), sim/torch_sim.py:809-833).
    `tier_cap`: blast tiers considered (None = all present).
    """
    triggered = (fuse == 0) & (owner >= 0)
    live = fuse > 0
    solid = live | brick
    max_b = (int(blast.max()) if blast.size else 0) if tier_cap is None else int(tier_cap)
    covered = fire_cover(triggered, wall, solid, blast, brick, max_b)
    for _ in range(rounds):
        newly = live & covered & ~triggered
        if not newly.any():
            break
        covered = covered | fire_cover(newly, wall, solid, blast, brick, max_b)
        triggered = triggered | newly
    return covered, triggered


def danger_map(fuse, wall, blast, brick, fuse_max: int, rounds_a: int) -> np.ndarray:
    """Chain-corrected danger map (sim/blast.py:158-317).

    Stage A (rounds_a rounds): a bomb that a front bomb's flame reaches takes
    the front's weight if larger, and joins the next front.  Stage B: every
    non-wall cell takes the max weight over the bombs whose flame reaches it.
    """
    bombed = fuse > 0
    w = fuse_weight(fuse, fuse_max)
    solid = bombed | brick
    clear = ~wall & ~solid
    max_b = int(blast.max()) if blast.size else 0

    def reach_max(values):
        best = np.zeros(values.shape, dtype=F32)
        for dr, dc in DIRS4:
            open_path = np.ones(values.shape, dtype=bool)
            for k in range(1, max_b + 1):
                v = _behind(np.where(bombed & (blast >= k), values, F32(0.0)),
                            dr, dc, k, F32(0.0))
                best = np.maximum(best, np.where(open_path & ~wall, v, F32(0.0)))
                open_path &= _behind(clear, dr, dc, k, False)
        return best

    if rounds_a > 0:
        cur = w.copy()
        front = np.where(bombed, w, F32(0.0))
        for _ in range(rounds_a):
            spread = np.where(bombed, reach_max(front), F32(0.0))
            newly = (spread > cur) & bombed
            cur = np.maximum(cur, spread)
            front = np.where(newly, spread, F32(0.0))
            if not newly.any():
                break
        weight = cur
    else:
        weight = w
    # stage B spreads the weights with walls zeroed (sim/blast.py:297: seed =
    # weight * passable): a bomb on a wall cell casts no rays here, although
    # in stage A it still raises the bombs its flame reaches
    seed = np.where(wall, F32(0.0), weight)
    return np.maximum(seed, reach_max(seed)).astype(F32)


# ------------------------------------------------------------- movement

def _impassable_pair(blocked_flat, r0, c0, r1, c1, y, x, rad, h, w):
    """Either of two cells blocks this player (sim/move.py:154-181)."""
    oob = ((r0 < 0) | (r0 >= h) | (c0 < 0) | (c0 >= w)
           | (r1 < 0) | (r1 >= h) | (c1 < 0) | (c1 >= w))
    i0 = np.clip(r0, 0, h - 1) * w + np.clip(c0, 0, w - 1)
    i1 = np.clip(r1, 0, h - 1) * w + np.clip(c1, 0, w - 1)
    s0 = np.take_along_axis(blocked_flat, i0, axis=1)
    s1 = np.take_along_axis(blocked_flat, i1, axis=1)
    ra = np.floor(y - rad).astype(np.int64)
    rb = np.floor(y + rad).astype(np.int64)
    ca = np.floor(x - rad).astype(np.int64)
    cb = np.floor(x + rad).astype(np.int64)
    in0 = (r0 >= ra) & (r0 <= rb) & (c0 >= ca) & (c0 <= cb)
    in1 = (r1 >= ra) & (r1 <= rb) & (c1 >= ca) & (c1 <= cb)
    return oob | (s0 & ~in0) | (s1 & ~in1)


def resolve_axis(coord, delta, other, y, x, blocked_flat, rad, h, w, vertical):
    """Slide along one axis and stop flush against the first blocking cell.

    (N, K) arrays; sim/move.py:184-231.  Every float op keeps the reference's
    order so the stop positions agree to the bit.
    """
    rad = F32(rad)
    sgn = np.sign(delta).astype(F32)
    old_lead = np.floor((coord - delta) + sgn * rad).astype(np.int64)
    new_lead = np.floor(coord + sgn * rad).astype(np.int64)
    lo = np.minimum(old_lead, new_lead)
    hi = np.maximum(old_lead, new_lead)
    span0 = np.floor(other - rad).astype(np.int64)
    span1 = np.floor(other + rad).astype(np.int64)

    def hit(lead):
        if vertical:
            return _impassable_pair(blocked_flat, lead, span0, lead, span1,
                                    y, x, rad, h, w)
        return _impassable_pair(blocked_flat, span0, lead, span1, lead,
                                y, x, rad, h, w)

    hit_lo, hit_hi = hit(lo), hit(hi)
    pos_dir = sgn > 0
    first_lead = np.where(pos_dir, hi, lo)
    second_lead = np.where(pos_dir, lo, hi)
    first_hit = np.where(pos_dir, hit_hi, hit_lo)
    second_hit = np.where(pos_dir, hit_lo, hit_hi)
    has = first_hit | second_hit
    first = np.where(first_hit, first_lead, np.where(second_hit, second_lead, 0))
    ff = first.astype(F32)
    stop = np.where(pos_dir, (ff - rad) - EPS, ((ff + F32(1.0)) + rad) + EPS)
    return np.where(has, stop, coord).astype(F32)


def step_table(step_len: float) -> np.ndarray:
    dirs = ((-1.0, 0.0), (1.0, 0.0), (0.0, -1.0), (0.0, 1.0))
    return np.array([[dy * step_len, dx * step_len] for dy, dx in dirs]
                    + [[0.0, 0.0]], dtype=F32)


def move_players(cfg, pos, move, alive, blocked, spd):
    """New positions after one tick of AABB sliding (sim/move.py:234-279)."""
    n, p, _ = pos.shape
    h, w, rad = cfg.height, cfg.width, cfg.radius
    bflat = blocked.reshape(n, -1)
    delta = step_table(cfg.step_len)[np.clip(move, 0, 4)] * spd[..., None]
    moving = alive & (move != MOVE_IDLE)
    delta = np.where(moving[..., None], delta, F32(0.0)).astype(F32)
    dy, dx = delta[..., 0], delta[..., 1]
    y, x = pos[..., 0], pos[..., 1]
    ny = resolve_axis(y + dy, dy, x, y, x, bflat, rad, h, w, True)
    nx = resolve_axis(x + dx, dx, y, y, x, bflat, rad, h, w, False)
    out = np.empty_like(pos)
    out[..., 0] = np.clip(np.where(dy != 0, ny, y), F32(rad), F32(h - rad))
    out[..., 1] = np.clip(np.where(dx != 0, nx, x), F32(rad), F32(w - rad))
    return out


def center_flat(pos, w, h, clamp=True):
    cell = np.floor(pos).astype(np.int64)
    flat = cell[..., 0] * w + cell[..., 1]
    return np.clip(flat, 0, h * w - 1) if clamp else flat


# ---------------------------------------------------------- obs and masks

def live_counts(owner, fuse, p):
    """(N, P) live bomb count per player."""
    n = owner.shape[0]
    live = fuse > 0
    return np.stack([((owner == i) & live).reshape(n, -1).sum(1)
                     for i in range(p)], axis=1)


def encode_obs(cfg, st, danger) -> np.ndarray:
    """Shared (N, C, H, W) float32 observation (sim/obs.py:48-136)."""
    n, p = st["alive"].shape
    h, w = cfg.height, cfg.width
    obs = np.zeros((n, cfg.n_channels, h, w), dtype=F32)
    fuse, owner, pos, alive = st["fuse"], st["owner"], st["pos"], st["alive"]
    fuse_norm = fuse.astype(F32) / F32(cfg.fuse)
    for i in range(p):
        obs[:, i] = _splat(pos[:, i], alive[:, i], h, w)
        obs[:, p + i] = np.where((owner == i) & (fuse > 0), fuse_norm, F32(0.0))
    obs[:, 2 * p] = (st["wall"] | st["brick"]).astype(F32)
    obs[:, 2 * p + 1] = danger
    obs[:, 2 * p + 2] = (st["t"].astype(F32) / F32(cfg.max_steps))[:, None, None]
    if not cfg.obs_extra_enabled:
        return obs
    obs[:, 2 * p + 3] = st["crate"].astype(F32)
    flat = center_flat(pos, w, h, clamp=False)
    rows = np.arange(n)
    for i in range(p):
        ch = obs[:, 2 * p + 4 + i].reshape(n, -1)
        ch[rows, flat[:, i]] = ((st["invuln"][:, i] > 0) & alive[:, i]).astype(F32)
    caps = st["bombs_cap"]
    cap = np.maximum(caps.astype(F32), F32(1.0))
    avail = np.maximum((caps - live_counts(owner, fuse, p)).astype(F32), F32(0.0))
    base = 3 * p + 4
    for i in range(p):
        a = alive[:, i].astype(F32)
        obs[:, base + i].reshape(n, -1)[rows, flat[:, i]] = (avail[:, i] / cap[:, i]) * a
        obs[:, base + p + i].reshape(n, -1)[rows, flat[:, i]] = \
            (cap[:, i] / F32(cfg.growth_bombs_max)) * a
    return obs


def _splat(pos_me, gate, h, w):
    """Bilinear splat of one player position, mass 1 (sim/obs.py:25-45)."""
    n = pos_me.shape[0]
    fy = np.clip(pos_me[:, 0] - F32(0.5), F32(0.0), F32(h - 1.0))
    fx = np.clip(pos_me[:, 1] - F32(0.5), F32(0.0), F32(w - 1.0))
    y0 = np.clip(np.floor(fy).astype(np.int64), 0, h - 1)
    x0 = np.clip(np.floor(fx).astype(np.int64), 0, w - 1)
    y1 = np.clip(y0 + 1, 0, h - 1)
    x1 = np.clip(x0 + 1, 0, w - 1)
    wy = np.clip(fy - y0.astype(F32), F32(0.0), F32(1.0))
    wx = np.clip(fx - x0.astype(F32), F32(0.0), F32(1.0))
    g = gate.astype(F32)
    out = np.zeros((n, h * w), dtype=F32)
    rows = np.arange(n)
    for yy, wyy in ((y0, F32(1.0) - wy), (y1, wy)):
        for xx, wxx in ((x0, F32(1.0) - wx), (x1, wx)):
            np.add.at(out, (rows, yy * w + xx), (wyy * wxx) * g)
    return out.reshape(n, h, w)


def legal_mask(cfg, st):
    """(move_mask (N,P,5), bomb_mask (N,P,2)) (sim/obs.py:139-229)."""
    n, p = st["alive"].shape
    h, w, rad = cfg.height, cfg.width, cfg.radius
    fuse, alive, pos = st["fuse"], st["alive"], st["pos"]
    blocked = (st["wall"] | (fuse > 0) | st["brick"]).reshape(n, -1)
    step = F32(cfg.step_len)
    y, x = pos[..., 0], pos[..., 1]
    mm = np.ones((n, p, 5), dtype=bool)
    for d, (sgn, vertical) in enumerate(((-1, True), (1, True), (-1, False), (1, False))):
        dv = np.full_like(y, step) if sgn > 0 else np.full_like(y, -step)
        if vertical:
            ny = resolve_axis(y + dv, dv, x, y, x, blocked, rad, h, w, True)
            moved = np.abs(ny - y) > F32(2e-4)
        else:
            nx = resolve_axis(x + dv, dv, y, y, x, blocked, rad, h, w, False)
            moved = np.abs(nx - x) > F32(2e-4)
        mm[..., d] = moved
    mm = (mm & alive[..., None]) | ~alive[..., None]
    flat = center_flat(pos, w, h, clamp=False)
    ff = fuse.reshape(n, -1)
    bb = (fuse > 0) | st["brick"]
    bbf = bb.reshape(n, -1)
    live = live_counts(st["owner"], fuse, p)
    rows = np.arange(n)
    bm = np.ones((n, p, 2), dtype=bool)
    for i in range(p):
        under = ff[rows, flat[:, i]] > 0
        under_b = bbf[rows, flat[:, i]]
        ok = ~under & ~under_b & (live[:, i] < st["bombs_cap"][:, i]) & alive[:, i]
        bm[:, i, 1] = ok | ~alive[:, i]
    return mm, bm


# ------------------------------------------------------------------ step

def _rounds_resolve(cfg):
    return min(cfg.max_chain - 1, cfg.chain_cap_rounds)


def _rounds_danger(cfg):
    return min(cfg.max_chain, cfg.chain_cap_rounds) if cfg.max_chain > 1 else 0


def place_bombs(cfg, st, bomb, alive0):
    """Sequential per-player placement (sim/torch_sim.py:1357-1402)."""
    n, p = alive0.shape
    h, w = cfg.height, cfg.width
    fuse = st["fuse"].reshape(n, -1)
    owner = st["owner"].reshape(n, -1)
    bblast = st["bomb_blast"].reshape(n, -1)
    brick = st["brick"].reshape(n, -1)
    flat = center_flat(st["pos"], w, h)
    rows = np.arange(n)
    placed = np.zeros((n, p), dtype=bool)
    for me in range(p):
        idx = flat[:, me]
        live = ((owner == me) & (fuse > 0)).sum(1)
        cur = fuse[rows, idx]
        ok = (alive0[:, me] & (bomb[:, me] == 1) & (cur <= 0)
              & ~brick[rows, idx] & (live < st["bombs_cap"][:, me]))
        placed[:, me] = ok
        fuse[rows[ok], idx[ok]] = cfg.fuse
        owner[rows[ok], idx[ok]] = me
        bblast[rows[ok], idx[ok]] = st["blast_cap"][ok, me].astype(np.int16)
    return placed


def place_predict_reward(cfg, st, placed, alive0):
    """Immediate placement bonus: cover + chain (+ dist) (sim/torch_sim.py:1263-1355)."""
    n, p = alive0.shape
    h, w = cfg.height, cfg.width
    if not (cfg.place_cover_reward or cfg.place_chain_reward or cfg.place_dist_reward):
        return np.zeros((n, p), dtype=F32)
    fuse, owner = st["fuse"], st["owner"]
    live = fuse > 0
    bm = blast_map(st["bomb_blast"], cfg.blast)
    frac = np.clip(fuse.astype(F32) / F32(cfg.fuse), F32(0.0), F32(1.0))
    weight = F32(cfg.chain_time_factor) + F32(1.0 - cfg.chain_time_factor) * (F32(1.0) - frac)
    flat = center_flat(st["pos"], w, h)
    rows = np.arange(n)
    placed_map = np.zeros((n, h * w), dtype=bool)
    for me in range(p):                       # later players overwrite earlier
        placed_map[rows, flat[:, me]] = placed[:, me]
    placed_map = placed_map.reshape(n, h, w)
    cover = np.zeros((n, p), dtype=F32)
    dist_pts = np.zeros((n, p), dtype=F32)
    chain = np.zeros((n, p), dtype=F32)
    cooldown_ok = st["since_bomb"] >= cfg.place_dist_cooldown
    cell_f = np.floor(st["pos"]).astype(F32)
    max_b = int(bm.max())
    for me in range(p):
        seed = np.zeros((n, h * w), dtype=bool)
        seed[rows, flat[:, me]] = placed[:, me]
        cov = fire_cover(seed.reshape(n, h, w), st["wall"], live | st["brick"],
                         bm, st["brick"], max_b)
        cflat = cov.reshape(n, -1)
        for o in range(p):
            if o == me:
                continue
            under = cflat[rows, flat[:, o]]
            cover[:, me] += (under & alive0[:, o]).astype(F32)
            if cfg.place_dist_reward > 0:
                d = np.sqrt(((cell_f[:, me] - cell_f[:, o]) ** 2).sum(-1)).astype(F32)
                ok = placed[:, me] & ~under & (d < cfg.place_dist_radius) \
                    & cooldown_ok[:, me] & alive0[:, o]
                gain = np.maximum(F32(1.0) - d / F32(cfg.place_dist_radius), F32(0.0))
                dist_pts[:, me] += (ok * gain).astype(F32)
        chained = cov & live & (owner >= 0) & ~placed_map
        chain[:, me] = np.where(chained, weight, F32(0.0)).reshape(n, -1).sum(1, dtype=F32)
    bonus = (F32(cfg.place_cover_reward) * cover + F32(cfg.place_dist_reward) * dist_pts
             + F32(cfg.place_chain_reward) * chain)
    return (bonus * alive0.astype(F32)).astype(F32)


def step(cfg, st, actions, rb_hit, rb_grow, explore_coef=1.0, hazard_seed=None):
    """One tick, in place on `st` (sim/torch_sim.py:895-1261), no auto-reset.

    rb_hit / rb_grow: (N, P) float32 uniforms for crate pickup (the
    reference's `_rand_buf` layout).  hazard_seed: with cfg.hazard_fraction
    > 0, the hazard wave after the tick count (sim/torch_sim.py:1042-1049)
    with the engine's keyed draws (`hazard_draws_keyed`).  Returns (reward
    (N,P) f32, done (N,), info dict with covered/triggered/died/winner/n_alive).
    """
    n, p = st["alive"].shape
    h, w = cfg.height, cfg.width
    rows = np.arange(n)
    alive0 = st["alive"].copy()
    a0f = alive0.astype(F32)
    hp_before = st["hp"].astype(np.int32)
    move, bomb = actions[..., 0], actions[..., 1]
    coef = F32(explore_coef)

    st["fuse"][...] = np.where(st["fuse"] > 0, st["fuse"] - 1, st["fuse"])
    placed = place_bombs(cfg, st, bomb, alive0)
    place_bonus = place_predict_reward(cfg, st, placed, alive0)
    st["since_bomb"] += 1
    st["since_bomb"][placed] = 0

    blocked = st["wall"] | st["brick"] | (st["fuse"] > 0)
    st["pos"][...] = move_players(cfg, st["pos"], move, alive0, blocked, st["spd_g"])

    bmap = blast_map(st["bomb_blast"], cfg.blast)
    # The reference compiles resolve once, on the first step, with that step's
    # hint max(bomb_blast.max(), cfg.blast) bound into the closure
    # (sim/torch_sim.py:818-832): later steps keep those blast tiers.
    if int(st.get("resolve_tiers", -1)) < 0:
        st["resolve_tiers"] = np.int64(max(int(st["bomb_blast"].max()), int(cfg.blast)))
    covered, triggered = resolve_explosions(st["fuse"], st["owner"], st["wall"], bmap,
                                            st["brick"], _rounds_resolve(cfg),
                                            tier_cap=int(st["resolve_tiers"]))
    chain_bonus = np.zeros((n, p), dtype=F32)
    if cfg.chain_blast_bonus > 0 and cfg.max_chain > 1:
        nat = (triggered & (st["fuse"] == 0)).reshape(n, -1)
        own = st["owner"].reshape(n, -1)
        chained = (triggered.reshape(n, -1) & ~nat)
        for pl in range(p):
            fired = np.minimum((nat & (own == pl)).sum(1), 1)
            cross = (chained & (own != pl)).sum(1)
            chain_bonus[:, pl] = F32(cfg.chain_blast_bonus) * (cross * fired).astype(F32)
    if cfg.map_mode == "corridor":
        st["crate"] |= st["brick"] & covered
    st["brick"] &= ~covered

    flat = center_flat(st["pos"], w, h)
    hit = alive0 & covered.reshape(n, -1)[rows[:, None], flat]
    hit_eff = hit & (st["invuln"] <= 0)
    hp_new = np.maximum(st["hp"].astype(np.int32) - hit_eff.astype(np.int32), 0)
    died = hit_eff & (hp_new == 0)
    st["hp"][...] = hp_new.astype(np.uint8)
    st["alive"][...] = alive0 & ~died
    st["invuln"][...] = np.maximum(st["invuln"] - 1, 0)
    st["invuln"][hit_eff] = cfg.invuln_ticks

    st["fuse"][triggered] = 0
    st["owner"][triggered] = -1
    st["bomb_blast"][triggered] = 0
    st["t"] += 1
    if cfg.hazard_fraction > 0 and hazard_seed is not None:
        hazard_wave(cfg, st, hazard_draws_keyed(cfg, st, hazard_seed))
    n_alive = st["alive"].sum(1)
    done = (n_alive <= 1) | (st["t"] >= cfg.max_steps)

    dmg = np.maximum(hp_before - st["hp"].astype(np.int32), 0).astype(F32)
    dealt = dmg.sum(1, keepdims=True, dtype=F32) - dmg
    hr = F32(cfg.hit_reward)
    reward = (((-F32(cfg.step_penalty)) * a0f + hr * dealt) - hr * dmg
              + (coef * place_bonus) * a0f)

    if cfg.hit_attr_penalty > 0:
        hit_any = (dmg > 0) & alive0
        pen = cfg.hit_attr_penalty
        nb = np.maximum(st["bombs_cap"] - pen, st["lo_bombs"])
        nz = np.maximum(st["blast_cap"] - pen, st["lo_blast"])
        ns = np.maximum(st["spd_g"] - F32(pen * cfg.growth_speed_step), st["lo_spd"])
        lost = (((st["bombs_cap"] - nb) + (st["blast_cap"] - nz)).astype(F32)
                + np.round((st["spd_g"] - ns) / F32(cfg.growth_speed_step))).astype(np.int64)
        st["bombs_cap"][...] = np.where(hit_any, nb, st["bombs_cap"])
        st["blast_cap"][...] = np.where(hit_any, nz, st["blast_cap"])
        st["spd_g"][...] = np.where(hit_any, ns, st["spd_g"])
        st["pending_lost"] += lost * hit_any
    reward = reward + (coef * chain_bonus) * a0f

    if cfg.map_mode == "corridor":
        flat = center_flat(st["pos"], w, h)
        stood = st["crate"].reshape(n, -1)[rows[:, None], flat]
        reward = reward + (F32(cfg.brick_reward) * stood.astype(F32)) * a0f
        rec = st["recycle"].reshape(n, -1)[rows[:, None], flat]
        prob = np.where(rec, F32(cfg.recycle_crate_prob), st["crate_prob"][:, None])
        hits = stood & (rb_hit < prob) & alive0
        _grow(cfg, st, hits.astype(np.int64) * alive0, rb_grow)
        st["crate"].reshape(n, -1)[rows[:, None], flat] = False
        st["recycle"].reshape(n, -1)[rows[:, None], flat] = False

    danger = danger_map(st["fuse"], st["wall"], blast_map(st["bomb_blast"], cfg.blast),
                        st["brick"], cfg.fuse, _rounds_danger(cfg))
    flat = center_flat(st["pos"], w, h)
    standing = danger.reshape(n, -1)[rows[:, None], flat]
    reward = reward - (F32(explore_coef * cfg.danger_penalty) * standing) * a0f

    if cfg.combo_reward > 0:
        hit_this = dmg > 0
        for me in range(p):
            dm = dealt[:, me]
            c = st["combo"][:, me].copy()
            gap = np.maximum(st["t"] - st["last_hit"][:, me], 0).astype(F32)
            factor = np.power(F32(cfg.combo_gap_factor), gap).astype(F32)
            inc = (dm > 0).astype(np.int64)
            now = (c + inc) * inc
            pts = ((now.astype(F32) * F32(cfg.combo_reward)) * factor) * np.minimum(dm, F32(1.0))
            reward[:, me] = reward[:, me] + pts * a0f[:, me]
            st["combo"][:, me] = np.where(inc > 0, now, c)
            st["last_hit"][:, me] = np.where(inc > 0, st["t"], st["last_hit"][:, me])
            st["combo"][:, me] = np.where(hit_this[:, me], 0, st["combo"][:, me])

    alive = st["alive"]
    death_done = done & (n_alive == 1)
    winner = death_done[:, None] & alive & (n_alive == 1)[:, None]
    loser = death_done[:, None] & ~alive & (n_alive == 1)[:, None]
    hpf = st["hp"].astype(F32)
    all_alive = done & (n_alive == p)
    if not cfg.win_hp_scaled:
        reward = reward + F32(cfg.win_bonus) * (winner.astype(F32) - loser.astype(F32))
        if cfg.timeout_draw:
            tot = hpf.sum(1, dtype=F32)
            for me in range(p):
                opp = (tot - hpf[:, me]) / F32(p - 1)
                diff = hpf[:, me] - opp
                reward[:, me] = reward[:, me] + ((F32(cfg.win_bonus / cfg.max_hp) * diff)
                                                 * all_alive.astype(F32)) * coef
    else:
        scale = coef if cfg.timeout_draw else F32(1.0)
        tot = hpf.sum(1, dtype=F32)
        for me in range(p):
            diff = hpf[:, me] - (tot - hpf[:, me]) / F32(p - 1)
            base = F32(cfg.win_bonus / cfg.max_hp) * diff
            reward[:, me] = reward[:, me] + (base * death_done.astype(F32)
                                             + (base * all_alive.astype(F32)) * scale)
    info = {"n_alive": n_alive, "blast": covered, "trig": triggered,
            "died": died, "winner": winner}
    return reward.astype(F32), done, info


def _grow(cfg, st, hits, rb):
    """Crate-driven growth of bombs/blast/speed (sim/torch_sim.py:862-893)."""
    attr = np.floor(rb * F32(3.0)).astype(np.int64)
    if cfg.crate_speed_only:
        attr = np.where(st["hazard"][:, None], 2, attr)
    st["bombs_cap"][...] = np.minimum(st["bombs_cap"] + (attr == 0) * hits,
                                      cfg.growth_bombs_max)
    st["blast_cap"][...] = np.minimum(st["blast_cap"] + (attr == 1) * hits,
                                      cfg.growth_blast_max)
    add = ((attr == 2) * hits).astype(F32) * F32(cfg.growth_speed_step)
    st["spd_g"][...] = np.minimum(st["spd_g"] + add, F32(cfg.growth_speed_max))


def observe(cfg, st):
    """danger + obs (fp32) for the current state (sim/torch_sim.py:605-627)."""
    dng = danger_map(st["fuse"], st["wall"], blast_map(st["bomb_blast"], cfg.blast),
                     st["brick"], cfg.fuse, _rounds_danger(cfg))
    return encode_obs(cfg, st, dng), dng


# -------------------------------------------------- LSTM local-view features

LV_K = 7          # local window side (sim/obs.py:252)
LV_MAX_T = 10     # relative-target slots (sim/obs.py:238)
LV_GLOB = 5       # global scalars (sim/obs.py:239)


def local_view_features(cfg, obs, pos, alive, t, fuse, hp, only_p0=False):
    """Per-player features of the LSTM policy from the shared observation
    (sim/obs.py:241-340).  obs (N, C, H, W) in its storage dtype; pos (N,P,2)
    f32, alive (N,P), t (N,), fuse (N,H,W), hp (N,P).  Returns local
    (N,Po,C,7,7), rel (N,Po,10,6) and glob (N,Po,5) in obs's dtype, Po = 1
    with only_p0 else P.

      local  the 7x7 window of every channel centred on the player's cell,
             zero outside the grid (sim/obs.py:257-282)
      rel    slots 0..P-2: opponent (me + i + 1) % P as [row delta, column
             delta, alive, 0, 0, 0]; slots P-1..9: cells ordered by L1
             distance from the player's cell, live bombs first (distance of a
             non-bomb cell counts as 1e6), as [column delta, row delta, 0,
             is-bomb, 0, 0] (sim/obs.py:284-322)
      glob   [t / max_steps, hp / max_hp, danger under the player, bombs /
             max_bombs, sum(fuse) / (max_bombs * fuse)] (sim/obs.py:324-338)

    Cells at equal distance are taken in ascending flat index; the reference
    leaves that order to torch.topk (sim/obs.py:306-309), which does not
    specify it (its CPU and CUDA implementations differ).
    """
    n, P, _ = pos.shape
    c, h, w = obs.shape[1], cfg.height, cfg.width
    half = LV_K // 2
    po = 1 if only_p0 else P
    dt = obs.dtype
    cell = np.floor(pos).astype(np.int64)
    pad = np.pad(obs, ((0, 0), (0, 0), (half, half), (half, half)))
    rows = np.arange(n)
    local = np.empty((n, po, c, LV_K, LV_K), dt)
    for m in range(po):
        for dy in range(LV_K):
            ys = np.clip(cell[:, m, 0] + dy, 0, h + 2 * half - 1)
            for dx in range(LV_K):
                xs = np.clip(cell[:, m, 1] + dx, 0, w + 2 * half - 1)
                local[:, m, :, dy, dx] = pad[rows, :, ys, xs]
    rel = np.zeros((n, po, LV_MAX_T, 6), dt)
    n_opp = P - 1
    for m in range(po):
        for i in range(n_opp):
            opp = (m + i + 1) % P
            rel[:, m, i, 0] = (pos[:, opp, 0] - pos[:, m, 0]).astype(F32)
            rel[:, m, i, 1] = (pos[:, opp, 1] - pos[:, m, 1]).astype(F32)
            rel[:, m, i, 2] = alive[:, opp]
    k = min(LV_MAX_T - n_opp, h * w)
    if k > 0:
        gy = np.arange(h).reshape(1, h, 1)
        gx = np.arange(w).reshape(1, 1, w)
        for m in range(po):
            cy, cx = cell[:, m, 0], cell[:, m, 1]
            dist = np.abs(gy - cy.reshape(n, 1, 1)) + np.abs(gx - cx.reshape(n, 1, 1))
            dist = np.where(fuse > 0, dist, 1000000).reshape(n, -1)
            order = np.argsort(dist, axis=1, kind="stable")[:, :k]
            vals = np.take_along_axis(dist, order, 1)
            for j in range(k):
                gi = order[:, j]
                rel[:, m, n_opp + j, 0] = (gi % w).astype(F32) - cx.astype(F32)
                rel[:, m, n_opp + j, 1] = (gi // w).astype(F32) - cy.astype(F32)
                rel[:, m, n_opp + j, 3] = vals[:, j] < 100000
    glob = np.zeros((n, po, LV_GLOB), dt)
    # dtype(t) / max_steps: the division runs in float32 and rounds to dtype
    glob[..., 0] = (t.astype(dt).astype(F32) / F32(cfg.max_steps)).astype(dt)[:, None]
    glob[..., 1] = (hp[:, :po].astype(dt).astype(F32) / F32(cfg.max_hp)).astype(dt)
    danger = obs[:, 2 * cfg.n_players + 1].reshape(n, -1)
    glob[..., 2] = np.take_along_axis(danger, (cell[:, :po, 0] * w + cell[:, :po, 1]), 1)
    nb = (fuse > 0).reshape(n, -1).sum(1).astype(F32)
    glob[..., 3] = (nb / F32(cfg.max_bombs))[:, None]
    fs = fuse.reshape(n, -1).astype(F32).sum(1, dtype=F32)
    glob[..., 4] = (fs / F32(cfg.max_bombs * cfg.fuse))[:, None]
    return local, rel, glob


# ------------------------------------------------------------------- bots

def sample_legal(mask, u):
    """Inverse-CDF sample over legal entries (sim/bots.py:36-46); u: (N,) f32."""
    cs = np.cumsum(mask.astype(F32), axis=-1, dtype=F32)
    s = np.maximum(cs[:, -1:], F32(1e-6))
    return ((u[:, None].astype(F32) * s) > cs).sum(-1).astype(np.int64)


def random_attack(alive_me, mm, bm, u_move, u_bomb, bomb_rate):
    """Uniform legal move, bomb with probability bomb_rate (sim/bots.py:49-58)."""
    move = sample_legal(mm, u_move)
    bomb = ((u_bomb < F32(bomb_rate)) & bm[:, 1]).astype(np.int64)
    move = np.where(alive_me, move, MOVE_IDLE)
    bomb = np.where(alive_me, bomb, 0)
    return np.stack([move, bomb], axis=-1)


def _cells(pos, pid, h, w):
    r = np.clip(np.floor(pos[:, pid, 0]).astype(np.int64), 0, h - 1)
    c = np.clip(np.floor(pos[:, pid, 1]).astype(np.int64), 0, w - 1)
    return r, c


def _candidates(r, c, h, w):
    rows = np.stack([np.clip(r - 1, 0, h - 1), np.clip(r + 1, 0, h - 1), r, r, r], 1)
    cols = np.stack([c, c, np.clip(c - 1, 0, w - 1), np.clip(c + 1, 0, w - 1), c], 1)
    return rows, cols


def greedy_attack(cfg, st, danger_obs, mm, bm, pid, noise):
    """Chebyshev approach with a hard danger filter (sim/bots.py:95-176).

    danger_obs: (N, H, W) float32 read from the fp16 observation; noise (N,5).
    """
    n, p = st["alive"].shape
    h, w = cfg.height, cfg.width
    pos = st["pos"]
    dflat = danger_obs.reshape(n, -1)
    blocked = (st["wall"] | st["brick"]).reshape(n, -1)
    r, c = _cells(pos, pid, h, w)
    rows = np.arange(n)
    own = dflat[rows, r * w + c]
    cr, cc = _candidates(r, c, h, w)
    cflat = cr * w + cc
    dng = np.take_along_axis(dflat, cflat, 1)
    blk = np.take_along_axis(blocked, cflat, 1)
    dist = np.full((n, 5), F32(1e9), dtype=F32)
    for o in range(p):
        if o == pid:
            continue
        ro, co = _cells(pos, o, h, w)
        d = np.maximum(np.abs(cr - ro[:, None]), np.abs(cc - co[:, None])).astype(F32)
        d = np.where(st["alive"][:, o][:, None], d, F32(1e9))
        dist = np.minimum(dist, d)
    inf = F32(np.inf)
    nz = F32(0.05) * noise.astype(F32)
    best = np.zeros(n, dtype=np.int64)
    best_s = np.full(n, inf, dtype=F32)
    esc_s = np.full(n, inf, dtype=F32)
    esc_d = np.zeros(n, dtype=np.int64)
    for d in range(5):
        legal = mm[:, d] & ~blk[:, d]
        s = np.where(legal, (dist[:, d] + F32(2.0) * dng[:, d]) + nz[:, d], inf)
        better = s < best_s
        best_s = np.where(better, s, best_s)
        best = np.where(better, d, best)
        e = np.where(legal, dng[:, d], inf)
        eb = e < esc_s
        esc_s = np.where(eb, e, esc_s)
        esc_d = np.where(eb, d, esc_d)
    use_safe = (best_s < inf) & (dng[rows, best] < F32(0.35))
    move = np.where(use_safe, best, esc_d)
    place = (bm[:, 1] & (dist[:, MOVE_IDLE] < st["blast_cap"][:, pid].astype(F32))
             & (own < F32(0.2))).astype(np.int64)
    dead = ~st["alive"][:, pid]
    return np.stack([np.where(dead, MOVE_IDLE, move), np.where(dead, 0, place)], -1)


def dijkstra_field(sources, danger, blocked, lam=2.0):
    """Multi-source shortest-path cost field, exact fixed point (sim/bots.py:179-238).

    cost(c) = 1 + lam*danger(c) (inf when blocked); dist = min over paths of
    the left-to-right float32 sum of entered-cell costs.  The reference's
    Jacobi passes stop at the same fixed point, which any convergent
    relaxation order reaches.
    """
    n = sources.shape[0]
    h, w = sources.shape[-2:]
    cost = F32(1.0) + F32(lam) * danger.astype(F32)
    cost = np.where(blocked, F32(np.inf), cost).astype(F32)
    dist = np.where(sources, F32(0.0), F32(np.inf)).astype(F32)
    for _ in range(h * w + 1):
        best = np.full_like(dist, F32(np.inf))
        best[:, 1:, :] = np.minimum(best[:, 1:, :], dist[:, :-1, :])
        best[:, :-1, :] = np.minimum(best[:, :-1, :], dist[:, 1:, :])
        best[:, :, 1:] = np.minimum(best[:, :, 1:], dist[:, :, :-1])
        best[:, :, :-1] = np.minimum(best[:, :, :-1], dist[:, :, 1:])
        new = np.minimum(dist, best + cost)
        if np.array_equal(new, dist):
            break
        dist = new
    return dist.reshape(n, h * w)


def _splitmix_unit(x):
    """SplitMix64 finaliser (S. Vigna's published mixer) -> the top 24 bits as
    a float in [0, 1): the device's counter-based uniform."""
    x = np.asarray(x, dtype=np.uint64)
    with np.errstate(over="ignore"):
        x = x + np.uint64(0x9E3779B97F4A7C15)
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    x = x ^ (x >> np.uint64(31))
    return (x >> np.uint64(40)).astype(np.float32) * np.float32(1.0 / 16777216.0)


def flush_recycle_keyed(cfg, st, excl, seed, counter, envs=None):
    """Crate recycling with counter-based draws (the engine's device variant of
    sim/torch_sim.py:549-596): for each player p (in order) of each env with
    pending_lost > 0, the min(lost, #available) available cells (not wall,
    not brick, not in `excl`) with the smallest keys u(key + cell) get a
    crate and a recycle mark (ties -> lower cell); key = seed ^ counter*G ^
    (e << 20) ^ (p << 52) ^ t_e*M.  Checker for k_flush_recycle.  envs:
    the engine's env index of each row of `st` (a subset of a larger sim);
    None = 0..N-1."""
    n = st["wall"].shape[0]
    p = st["alive"].shape[1]
    h, w = cfg.height, cfg.width
    cells = np.arange(h * w, dtype=np.uint64)
    ex = np.zeros(h * w, bool)
    ex[list(excl)] = True
    G = np.uint64(0x9E3779B97F4A7C15)
    M = np.uint64(0xD1B54A32D192ED03)
    with np.errstate(over="ignore"):
        for pl in range(p):
            for e in range(n):
                lost = int(st["pending_lost"][e, pl])
                if lost <= 0:
                    continue
                ge = e if envs is None else int(envs[e])
                key = (np.uint64(seed) ^ (np.uint64(counter) * G) ^ (np.uint64(ge) << np.uint64(20))
                       ^ (np.uint64(pl) << np.uint64(52)) ^ (np.uint64(st["t"][e]) * M))
                avail = ~(st["wall"][e].reshape(-1) | st["brick"][e].reshape(-1) | ex)
                k = _splitmix_unit(key + cells)
                idx = np.nonzero(avail)[0]
                order = idx[np.lexsort((idx, k[idx]))][:min(lost, idx.size)]
                st["crate"][e].reshape(-1)[order] = True
                st["recycle"][e].reshape(-1)[order] = True
                st["pending_lost"][e, pl] = 0
    return st


def template_swap_draws(seed, episode, envs=None):
    """Spawn-swap decisions of the device auto-reset: env e in its episode
    `episode[e]` swaps seats 0 and 1 when u(seed ^ (e << 32) ^ episode[e])
    < 0.5 (the keyed stand-in for the reference's host draw
    `torch.rand(count, generator=gen) < 0.5`, sim/torch_sim.py:229-240).
    envs: the engine's env index of each entry (a subset of a larger sim);
    None = 0..N-1."""
    ep = np.asarray(episode, dtype=np.int64).astype(np.uint64)
    e = (np.arange(ep.shape[0]) if envs is None else np.asarray(envs)).astype(np.uint64)
    return _splitmix_unit(np.uint64(seed) ^ (e << np.uint64(32)) ^ ep) < np.float32(0.5)


def template_reset(cfg, st, tmpl, mask, swap=None, episode=None):
    """Reset the envs in `mask` to their per-env templates, in place.

    Restates the reset branch of the engine's step (the device auto-reset)
    on the reference's reset_ field list (sim/torch_sim.py:178-420):
      * map: wall, brick from the template; crate from the template (the
        reference clears crates, sim/torch_sim.py:385, and lays an open
        map's cross crates afterwards, :392-396: a template carries the
        crates an episode starts with); recycle marks cleared (:386);
      * bombs: fuse 0, owner -1, bomb_blast 0 (:397-399);
      * players: spawn positions from the template, seats 0 and 1 swapped
        where `swap` is set (:229-240 / :374-383); bombs_cap, blast_cap,
        spd_g and the growth floors lo_* from the template's start
        attributes (:209-224 and the corridor/ring/open branches); alive,
        hp = max_hp (:400-401), since_bomb = place_dist_cooldown (:404),
        invuln 0 (:405), pending_lost 0, combo 0, last_hit -10**9
        (:387-389);
      * env: t = 0 (:406), crate_prob from the template (:284, :317, :348),
        hazard off (:420; templates carry no hazard waves).
    tmpl: dict of wall, brick, crate (N,H,W) bool, spawn (N,P,2) f32,
    bombs_cap, blast_cap (N,P) int, spd (N,P) f32, crate_prob (N,) f32.
    swap: (N,) bool or None (no swap).  episode: (N,) int64 counter,
    incremented for every reset env when given.
    """
    idx = np.nonzero(np.asarray(mask, bool))[0]
    if idx.size == 0:
        return st
    p = st["alive"].shape[1]
    st["wall"][idx] = tmpl["wall"][idx]
    st["brick"][idx] = tmpl["brick"][idx]
    st["crate"][idx] = tmpl["crate"][idx] if "crate" in tmpl else False
    st["recycle"][idx] = False
    st["fuse"][idx] = 0
    st["owner"][idx] = -1
    st["bomb_blast"][idx] = 0
    pos = np.array(tmpl["spawn"][idx], dtype=F32, copy=True)
    if swap is not None and p >= 2:
        sw = np.asarray(swap, bool)[idx]
        pos[sw, 0], pos[sw, 1] = tmpl["spawn"][idx][sw, 1], tmpl["spawn"][idx][sw, 0]
    st["pos"][idx] = pos
    st["alive"][idx] = True
    st["hp"][idx] = cfg.max_hp
    st["since_bomb"][idx] = cfg.place_dist_cooldown
    st["invuln"][idx] = 0
    st["pending_lost"][idx] = 0
    st["combo"][idx] = 0
    st["last_hit"][idx] = -10 ** 9
    for cap, lo, src in (("bombs_cap", "lo_bombs", "bombs_cap"),
                         ("blast_cap", "lo_blast", "blast_cap"), ("spd_g", "lo_spd", "spd")):
        st[cap][idx] = tmpl[src][idx]
        st[lo][idx] = tmpl[src][idx]
    st["crate_prob"][idx] = tmpl["crate_prob"][idx]
    st["hazard"][idx] = False
    st["t"][idx] = 0
    if episode is not None:
        episode[idx] += 1
    return st


def _u24(x):
    """SplitMix64 finaliser -> the top 24 bits as an integer (the device's
    counter-based draw before scaling)."""
    x = np.asarray(x, dtype=np.uint64)
    with np.errstate(over="ignore"):
        x = x + np.uint64(0x9E3779B97F4A7C15)
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    x = x ^ (x >> np.uint64(31))
    return (x >> np.uint64(40)).astype(np.int64)


def hazard_key(seed, e, t, j):
    """Key of draw family j (0: count, 1: cell order, 2: blast) for env e at
    tick t (after the step's increment)."""
    with np.errstate(over="ignore"):
        return (np.uint64(seed) ^ (np.uint64(e) << np.uint64(20))
                ^ (np.uint64(t) * np.uint64(0xD1B54A32D192ED03)) ^ (np.uint64(j) << np.uint64(56)))


def hazard_wave_envs(cfg, st):
    """Envs whose wave lands this tick (sim/torch_sim.py:1428)."""
    return st["hazard"] & (st["t"] > 0) & (st["t"] % cfg.hazard_wave_ticks == 0)


def hazard_free_cells(cfg, st, e):
    """Free cells of env e for the wave (sim/torch_sim.py:1431-1437): no wall,
    brick or live bomb; each player's centre cell (in player order) is then
    set to "not alive" (a dead player's cell becomes free even if blocked)."""
    h, w = cfg.height, cfg.width
    free = (~st["wall"][e] & ~st["brick"][e] & (st["fuse"][e] <= 0)).reshape(-1).copy()
    flat = center_flat(st["pos"][e:e + 1], w, h)[0]
    for pl in range(st["alive"].shape[1]):
        free[flat[pl]] = not st["alive"][e, pl]
    return free


def hazard_draws_keyed(cfg, st, seed):
    """The engine's draws for this tick's waves: per wave env e (ascending)
    a bomb count, an order of the free cells and one uniform per bomb, all
    counter-based (SplitMix64 of hazard_key(seed, e, t, family) + index).
    Returned in the reference's shapes: cnt (W,), u (sum cnt,), and per env
    the permutation of its free-cell list that randperm would give."""
    envs = np.nonzero(hazard_wave_envs(cfg, st))[0]
    span = cfg.hazard_bombs_max - cfg.hazard_bombs_min + 1
    cnt, us, perms = [], [], []
    hw = cfg.height * cfg.width
    for e in envs:
        t = int(st["t"][e])
        c = cfg.hazard_bombs_min + int((_u24(hazard_key(seed, e, t, 0)) * span) >> 24)
        cnt.append(c)
        pool = np.nonzero(hazard_free_cells(cfg, st, e))[0]
        keys = _u24(hazard_key(seed, e, t, 1) + np.arange(hw, dtype=np.uint64))[pool]
        perms.append(np.lexsort((pool, keys)))          # ascending key, ties -> lower cell
        u = (_u24(hazard_key(seed, e, t, 2) + np.arange(c, dtype=np.uint64)).astype(np.float32)
             * np.float32(1.0 / 16777216.0))
        us.append(u)
    return {"envs": envs, "cnt": np.array(cnt, np.int64),
            "u": np.concatenate(us) if us else np.zeros(0, np.float32), "perm": perms}


def hazard_wave(cfg, st, draws):
    """Place this tick's wave bombs (sim/torch_sim.py:1404-1466) from explicit
    draws: per wave env, min(cnt, #free) cells pool[perm[:c]] get fuse =
    cfg.fuse, owner = P (no player), and blast = min + floor(u^x * (max - min
    + 1)) clamped, x = 1 - 0.8 * clamp(t / ramp_ticks, 0, 1); the blasts are
    computed over all the wave's bombs in order and handed out with an
    offset that advances by the clamped count (as the reference does)."""
    envs = draws["envs"]
    if len(envs) == 0:
        return st
    p = st["alive"].shape[1]
    cnt = draws["cnt"]
    ramp = F32(cfg.hazard_ramp_seconds * cfg.tick_hz)
    frac = np.clip(st["t"][envs].astype(F32) / ramp, F32(0.0), F32(1.0))
    ex = (F32(1.0) - F32(0.8) * frac).astype(F32)
    ex_b = np.repeat(ex, cnt)
    u = draws["u"].astype(F32)
    v = np.power(u.astype(np.float64), ex_b.astype(np.float64)).astype(F32)
    lo, hi = cfg.hazard_blast_min, cfg.hazard_blast_max
    blast = (F32(lo) + np.floor(v * F32(hi - lo + 1))).astype(F32)
    blast = np.clip(blast, F32(lo), F32(hi)).astype(np.int16)
    w = cfg.width
    off = 0
    for i, e in enumerate(envs):
        pool = np.nonzero(hazard_free_cells(cfg, st, e))[0]
        c = min(int(cnt[i]), pool.size)
        if c <= 0:
            continue
        pick = pool[draws["perm"][i][:c]]
        y, x = pick // w, pick % w
        st["fuse"][e, y, x] = cfg.fuse
        st["owner"][e, y, x] = p
        st["bomb_blast"][e, y, x] = blast[off:off + c]
        off += c
    return st


class ModeTicker:
    """astar approach/flee mode switcher with fed draws (sim/bots.py:241-264)."""

    def __init__(self, mode0, timer0):
        self.mode = np.asarray(mode0, dtype=np.int64).copy()
        self.timer = np.asarray(timer0, dtype=np.int64).copy()
        self.tick = 0

    def advance(self, new_mode, new_timer):
        self.tick += 1
        self.timer -= 1
        if self.tick % 16 == 0:
            sw = self.timer <= 0
            self.mode = np.where(sw, new_mode, self.mode)
            self.timer = np.where(sw, new_timer, self.timer)
        return self.mode


def astar_attack(cfg, st, danger_obs, mm, bm, pid, noise, mode=None, cap_max=None,
                 return_fields=False, eat_crates=False):
    """Danger-aware path-field bot (sim/bots.py:267-508).

    cap_max: batch max of blast_cap[:, pid] (the reference's chain scan
    length, sim/bots.py:484); computed here when None.  eat_crates: the
    `hunter` bot's crate layer (sim/bots.py:376-431, make_bot "hunter" at
    sim/bots.py:557-561): with >= 2 of the bomb / blast / speed attributes
    under 70 % of their growth caps and a crate on the board, descend the
    crate field (sources = crate cells) instead of approaching.
    """
    n, p = st["alive"].shape
    h, w = cfg.height, cfg.width
    pos, fuse = st["pos"], st["fuse"]
    rows = np.arange(n)
    dflat = danger_obs.reshape(n, -1).astype(F32)
    r, c = _cells(pos, pid, h, w)
    own = dflat[rows, r * w + c]
    threat = (st["owner"] == pid) & (fuse > 0)
    for _ in range(int(cfg.growth_blast_max)):
        nb = threat.copy()
        nb[:, 1:, :] |= threat[:, :-1, :]
        nb[:, :-1, :] |= threat[:, 1:, :]
        nb[:, :, 1:] |= threat[:, :, :-1]
        nb[:, :, :-1] |= threat[:, :, 1:]
        threat = nb
    block_all = st["wall"] | st["brick"] | (fuse > 0)
    dng2 = danger_obs.astype(F32)
    v_safe = dijkstra_field(dng2 < F32(0.35), dng2, block_all)
    opp_src = np.zeros((n, h * w), dtype=bool)
    for o in range(p):
        if o == pid:
            continue
        ro, co = _cells(pos, o, h, w)
        opp_src[rows, ro * w + co] = st["alive"][:, o]
    v_opp = dijkstra_field(opp_src.reshape(n, h, w), dng2, block_all)

    cr, cc = _candidates(r, c, h, w)
    cflat = cr * w + cc
    vopp = np.take_along_axis(v_opp, cflat, 1)
    vsafe = np.take_along_axis(v_safe, cflat, 1)
    dng = np.take_along_axis(dflat, cflat, 1)
    thr = np.take_along_axis(threat.reshape(n, -1), cflat, 1).astype(F32)
    blk = np.take_along_axis((st["wall"] | st["brick"]).reshape(n, -1), cflat, 1)
    legal = mm & ~blk
    inf = F32(np.inf)
    nz = F32(0.05) * noise.astype(F32)
    two = F32(2.0)

    app = ((vopp + two * dng) + two * thr) + nz
    app = np.where(dng >= F32(0.5), inf, app)
    app = np.where(legal, app, inf)
    app_ok = np.isfinite(app.min(1))
    use_esc = (own >= F32(0.35)) | ~app_ok
    esc = (vsafe * F32(100.0) + two * thr) + nz
    idle_col = np.arange(5) == 4
    esc = np.where(use_esc[:, None] & idle_col[None], inf, esc)
    esc = np.where(legal, esc, inf)
    v_crate = None
    if eat_crates:
        fr = np.stack([st["bombs_cap"][:, pid].astype(F32) / F32(cfg.growth_bombs_max),
                       st["blast_cap"][:, pid].astype(F32) / F32(cfg.growth_blast_max),
                       st["spd_g"][:, pid].astype(F32) / F32(cfg.growth_speed_max)], 0)
        hungry = (fr < F32(0.7)).sum(0) >= 2
        has_crate = st["crate"].reshape(n, -1).any(1)
        eat_on = hungry & has_crate & st["alive"][:, pid]
        v_crate = dijkstra_field(st["crate"], dng2, block_all)
        vcrate = np.take_along_axis(v_crate, cflat, 1)
        eat = (vcrate * F32(100.0) + two * dng) + nz
        eat = np.where(dng >= F32(0.5), inf, eat)
        eat = np.where(legal, eat, inf)
        no_idle = np.where(~idle_col[None], eat, inf).min(1)
        eat = np.where(idle_col[None] & (no_idle[:, None] < eat[:, 4:5]), inf, eat)
        eat_on = eat_on & np.isfinite(eat.min(1))
        app = np.where(eat_on[:, None], eat, app)
    score = np.where(use_esc[:, None], esc, app)
    if mode is not None:
        vf = np.minimum(vopp, F32(1e3))
        flee = ((-vf + two * dng) + two * thr) + nz
        flee = np.where(dng >= F32(0.5), inf, flee)
        flee = np.where(legal, flee, inf)
        flee = np.where(use_esc[:, None], esc, flee)
        score = np.where((mode == 1)[:, None], flee, score)
    move = np.argmin(score, 1).astype(np.int64)
    any_legal = legal.any(1)
    no_path = ~np.isfinite(score).any(1)
    dl = np.where(legal, dng, inf)
    dmv = np.where(~idle_col[None], dl, inf)
    fb = np.where(np.isfinite(dmv.min(1)), np.argmin(dmv, 1), np.argmin(dl, 1))
    move = np.where(no_path & any_legal, fb, move)

    cap = st["blast_cap"][:, pid].astype(np.int64)
    big = 10 ** 9
    dr_o = np.full(n, big, dtype=np.int64)
    dc_o = np.full(n, big, dtype=np.int64)
    for o in range(p):
        if o == pid:
            continue
        ro, co = _cells(pos, o, h, w)
        dr_o = np.where(st["alive"][:, o], np.abs(r - ro), dr_o)
        dc_o = np.where(st["alive"][:, o], np.abs(c - co), dc_o)
    aligned = ((dr_o == 0) & (dc_o <= cap)) | ((dc_o == 0) & (dr_o <= cap))
    manh = np.minimum(dr_o + dc_o, 10 ** 8)
    near = manh <= np.maximum(cap + 1, 1)
    chain = np.zeros(n, dtype=bool)
    kmax = int(cap.max()) if cap_max is None else int(cap_max)
    for k in range(1, kmax + 1):
        for dr, dc in DIRS4:
            rr, cc2 = r + dr * k, c + dc * k
            inb = (rr >= 0) & (rr < h) & (cc2 >= 0) & (cc2 < w)
            f = fuse[rows, np.clip(rr, 0, h - 1), np.clip(cc2, 0, w - 1)]
            chain |= inb & (f > 0) & (f <= 10)
    can = bm[:, 1]
    can_escape = (legal & (dng < F32(0.35)) & ~(thr > 0)).any(1)
    place = (can & (aligned | near | chain) & (own < F32(0.2)) & can_escape)
    if mode is not None:
        flee_place = can & (aligned | near) & (own < F32(0.2)) & can_escape
        place = np.where(mode == 1, flee_place, place)
    dead = ~st["alive"][:, pid]
    out = np.stack([np.where(dead, MOVE_IDLE, move),
                    np.where(dead, 0, place.astype(np.int64))], -1)
    if return_fields:
        return (out, v_safe, v_opp, v_crate) if eat_crates else (out, v_safe, v_opp)
    return out


# ----------------------------------------------------------------- policy

def _ln(x, g, b, eps=1e-5):
    m = x.mean(-1, keepdims=True)
    v = ((x - m) ** 2).mean(-1, keepdims=True)
    return (x - m) / np.sqrt(v + eps) * g + b


def inv_cols(cfg_c, h, w, p, pid):
    """Column gather that folds the seat's view permutation into W0 (train/model.py:127-138)."""
    base = 2 * p + 3
    perm = [pid, p + pid] + [i for i in range(p) if i != pid] \
        + [p + i for i in range(p) if i != pid] + [2 * p, 2 * p + 1, 2 * p + 2] \
        + list(range(base, cfg_c))
    inv = np.argsort(np.asarray(perm))
    hw = h * w
    return np.concatenate([np.arange(hw) + int(inv[k]) * hw for k in range(cfg_c)])


def mlp_forward(params, obs, pid, p):
    """float64 MLP forward -> (move_logits, bomb_logits, value) (train/model.py:191-196).

    params: dict of numpy arrays keyed like ActorCritic's state_dict.
    """
    n, c, h, w = obs.shape
    x = obs.reshape(n, -1).astype(np.float64)
    W0 = params["shared.0.weight"].astype(np.float64)[:, inv_cols(c, h, w, p, pid)]
    z = x @ W0.T + params["shared.0.bias"]
    z = np.maximum(_ln(z, params["shared.1.weight"], params["shared.1.bias"]), 0)
    z = z @ params["shared.3.weight"].T.astype(np.float64) + params["shared.3.bias"]
    z = np.maximum(_ln(z, params["shared.4.weight"], params["shared.4.bias"]), 0)

    def head(name):
        a = np.maximum(z @ params[f"{name}.0.weight"].T.astype(np.float64)
                       + params[f"{name}.0.bias"], 0)
        return a @ params[f"{name}.2.weight"].T.astype(np.float64) + params[f"{name}.2.bias"]

    return head("move_head"), head("bomb_head"), head("critic")[:, 0]


def cnn_forward(params, obs, pid, p):
    """float64 CNN forward -> (move_logits, bomb_logits, value) (train/model.py:77-101, 187-196).

    Uses torch's float64 convolutions on the CPU as the accuracy reference.
    """
    import torch
    import torch.nn.functional as F
    T = lambda k: torch.from_numpy(np.asarray(params[k], dtype=np.float64))  # noqa: E731
    n, c, h, w = obs.shape
    base = 2 * p + 3
    perm = [pid, p + pid] + [i for i in range(p) if i != pid] \
        + [p + i for i in range(p) if i != pid] + [2 * p, 2 * p + 1, 2 * p + 2] + list(range(base, c))
    inv = torch.from_numpy(np.argsort(np.asarray(perm)))
    x = torch.from_numpy(obs.astype(np.float64))
    x = F.conv2d(x, T("conv0.weight")[:, inv], T("conv0.bias"), padding=1)
    for ln, conv, pad in (("conv.0", "conv.2", 1), ("conv.3", "conv.5", 1), ("conv.6", "conv.8", 0)):
        g = T(ln + ".weight")
        x = torch.relu(F.layer_norm(x, tuple(g.shape), g, T(ln + ".bias"), 1e-5))
        x = F.conv2d(x, T(conv + ".weight"), T(conv + ".bias"), padding=pad)
    g = T("conv.9.weight")
    x = torch.relu(F.layer_norm(x, tuple(g.shape), g, T("conv.9.bias"), 1e-5)).reshape(n, -1)
    z = x.numpy() @ np.asarray(params["shared.0.weight"], np.float64).T + params["shared.0.bias"]
    z = np.maximum(_ln(z, params["shared.1.weight"], params["shared.1.bias"]), 0)
    z = z @ np.asarray(params["shared.3.weight"], np.float64).T + params["shared.3.bias"]
    z = np.maximum(_ln(z, params["shared.4.weight"], params["shared.4.bias"]), 0)

    def head(name):
        a = np.maximum(z @ np.asarray(params[f"{name}.0.weight"], np.float64).T
                       + params[f"{name}.0.bias"], 0)
        return a @ np.asarray(params[f"{name}.2.weight"], np.float64).T + params[f"{name}.2.bias"]

    return head("move_head"), head("bomb_head"), head("critic")[:, 0]


def masked_sample(logits, mask, u):
    """Inverse-CDF draw from the masked categorical (train/model.py:216-245).

    Masked logits take float32's lowest finite value; a = #{k : u*S > cs_k}
    where cs is the running sum of exp(z - max z).  Returns (action, logp).
    """
    z = np.where(mask, logits, np.finfo(np.float32).min).astype(np.float64)
    m = z.max(-1, keepdims=True)
    e = np.exp(z - m)
    cs = np.cumsum(e, -1)
    s = cs[:, -1:]
    a = np.minimum(((u[:, None] * s) > cs).sum(-1), z.shape[-1] - 1)
    logp = np.take_along_axis(z, a[:, None], 1)[:, 0] - m[:, 0] - np.log(s[:, 0])
    return a.astype(np.int64), logp


def mlp_act(params, obs, mm, bm, pid, p, u_move, u_bomb):
    ml, bl, v = mlp_forward(params, obs, pid, p)
    am, lm = masked_sample(ml, mm, u_move.astype(np.float64))
    ab, lb = masked_sample(bl, bm, u_bomb.astype(np.float64))
    return np.stack([am, ab], -1), lm + lb, v, ml, bl


# ------------------------------------------------------------------ state

STATE_KEYS = ("wall", "brick", "crate", "recycle", "fuse", "owner", "bomb_blast",
              "pos", "alive", "hp", "since_bomb", "t", "bombs_cap", "blast_cap",
              "spd_g", "invuln", "pending_lost", "combo", "last_hit", "lo_bombs",
              "lo_blast", "lo_spd", "crate_prob", "hazard")


def copy_state(st):
    return {k: np.array(v, copy=True) for k, v in st.items()}


# --------------------------------------------------------- crate recycling

def recycle_exclusion(cfg):
    """Flat cells where recycled crates never land (sim/torch_sim.py:465-533):
    the 4-neighbourhoods of the open / mode / ring spawns plus the open
    map's central cross band."""
    h, w = cfg.height, cfg.width
    near = lambda r, c: {(r, c)} | {(r + dr, c + dc) for dr, dc in DIRS4
                                    if 0 <= r + dr < h and 0 <= c + dc < w}
    row = (h - 1) / 2.0 + 0.5
    open_sp = [(int(row), int((w - 1) * (i + 1) / (cfg.n_players + 1) + 0.5))
               for i in range(cfg.n_players)]
    open_excl = set()
    for r, c in open_sp:
        open_excl |= near(r, c)
    cy, cx = (h - 1) // 2, (w - 1) // 2
    cross = {(r, c) for c in range(w) for r in (cy - 1, cy)} \
        | {(r, c) for r in range(h) for c in (cx - 1, cx)}
    cross -= open_excl
    excl = set(open_excl)
    for r, c in list(cfg.spawn_cells()) + list(cfg.ring_spawn_cells()):
        excl |= near(r, c)
    excl |= cross
    return np.array(sorted(r * w + c for r, c in excl), dtype=np.int64)


def flush_recycle(cfg, st, gen):
    """Drop one crate per lost attribute layer on random free cells.

    sim/torch_sim.py:549-596; `gen` is a torch CPU generator in the same
    state as the reference's `sim.gen` (randperm draws, player-major, env
    order).
    """
    import torch
    n, p = st["pending_lost"].shape
    hw = cfg.height * cfg.width
    if st["pending_lost"].sum() <= 0:
        return
    excl = recycle_exclusion(cfg)
    for pl in range(p):
        lost = st["pending_lost"][:, pl]
        idx = np.flatnonzero(lost > 0)
        if idx.size == 0:
            continue
        avail = (~st["wall"][idx] & ~st["brick"][idx]).reshape(-1, hw).copy()
        avail[:, excl] = False
        crate = st["crate"].reshape(n, -1)
        rec = st["recycle"].reshape(n, -1)
        for i, e in enumerate(idx):
            cells = np.flatnonzero(avail[i])
            if cells.size == 0:
                continue
            k = min(int(lost[e]), cells.size)
            perm = torch.randperm(cells.size, generator=gen)[:k].numpy()
            crate[e, cells[perm]] = True
            rec[e, cells[perm]] = True
    st["pending_lost"][...] = 0


# ------------------------------------------------ per-episode map generation
#
# The reference draws every new episode's level from its host generator
# (BatchedSim.reset_, sim/torch_sim.py:178-420, with sim/mapgen.py).  The
# engine's device reset draws the same quantities from a counter-based hash
# keyed by (seed, env, episode, draw family, index), so that a reset needs
# no host round trip.  `map_reset` builds the levels from a dict of per-env
# draws in either form; it is pinned to the reference by feeding it the
# draws the reference consumed (tests/golden/mapgen_fed.npz), and the device
# kernel is compared with it on `mapgen_draws_keyed`.

MG_KIND, MG_OBST_N, MG_OBST_KEY, MG_RING, MG_TOP, MG_VSEG, MG_HSEG, MG_HAZARD = range(1, 9)


def _mg_hash(seed, envs, episode, fam, index):
    """SplitMix64 finaliser of (seed ^ e << 32 ^ episode ^ fam << 56) + index
    -> 24-bit integers, shape (n,) or (n, k) for an index vector."""
    e = np.asarray(envs, dtype=np.int64).astype(np.uint64)
    ep = np.asarray(episode, dtype=np.int64).astype(np.uint64)
    with np.errstate(over="ignore"):
        key = np.uint64(seed) ^ (e << np.uint64(32)) ^ ep ^ (np.uint64(fam) << np.uint64(56))
        idx = np.asarray(index, dtype=np.int64).astype(np.uint64)
        x = key[:, None] + idx[None, :] if idx.ndim else key + idx
    return _u24(x)


def mapgen_draws_keyed(cfg, seed, episode, envs=None):
    """The device reset's per-env draws for each env's current episode:
    uniforms u = k / 2^24 of 24-bit keys k, integer draws low + (k * range)
    >> 24 (the stand-in for the generator's randint)."""
    episode = np.asarray(episode, dtype=np.int64)
    n = episode.shape[0]
    envs = np.arange(n) if envs is None else np.asarray(envs)
    C = cfg.height * cfg.width
    unit = np.float32(1.0 / 16777216.0)

    def u(fam, index=0):
        return _mg_hash(seed, envs, episode, fam, index).astype(np.float32) * unit

    return {
        "kind_u": u(MG_KIND),
        "obst_n": (_mg_hash(seed, envs, episode, MG_OBST_N, 0)
                   * (cfg.open_obstacle_max + 1)) >> 24,
        "obst_key": _mg_hash(seed, envs, episode, MG_OBST_KEY, np.arange(C)),
        "ring_u": u(MG_RING, np.arange(C)),
        "top": (_mg_hash(seed, envs, episode, MG_TOP, 0) * (cfg.top_wall_rows + 1)) >> 24,
        "vstart_u": u(MG_VSEG, 3 * np.arange(4)),
        "vlen_u": u(MG_VSEG, 3 * np.arange(4) + 1),
        "vact_u": u(MG_VSEG, 3 * np.arange(4) + 2),
        "hstart_u": u(MG_HSEG, 0), "hlen_u": u(MG_HSEG, 1), "hact_u": u(MG_HSEG, 2),
        "swap_u": template_swap_draws_u(seed, episode, envs),
        "hazard_u": u(MG_HAZARD),
    }


def template_swap_draws_u(seed, episode, envs=None):
    """The spawn-swap uniform of template_swap_draws (swap when < 0.5)."""
    ep = np.asarray(episode, dtype=np.int64).astype(np.uint64)
    e = (np.arange(ep.shape[0]) if envs is None else np.asarray(envs)).astype(np.uint64)
    return _splitmix_unit(np.uint64(seed) ^ (e << np.uint64(32)) ^ ep)


def _clear4(mask, cells, h, w):
    for r, c in cells:
        mask[r, c] = False
        for dr, dc in DIRS4:
            if 0 <= r + dr < h and 0 <= c + dc < w:
                mask[r + dr, c + dc] = False


def _open_spawn_pos(cfg):
    h, w = float(cfg.height), float(cfg.width)
    row = (h - 1) / 2.0 + 0.5
    return np.array([(row, (w - 1) * (i + 1) / (cfg.n_players + 1) + 0.5)
                     for i in range(cfg.n_players)], dtype=F32)


def _open_cross(cfg):
    """Cross-band crate cells of an open map (sim/torch_sim.py:465-506)."""
    h, w = cfg.height, cfg.width
    near = set()
    for y, x in _open_spawn_pos(cfg):
        r, c = int(y), int(x)
        near.add((r, c))
        for dr, dc in DIRS4:
            if 0 <= r + dr < h and 0 <= c + dc < w:
                near.add((r + dr, c + dc))
    cy, cx = (h - 1) // 2, (w - 1) // 2
    cross = {(r, c) for c in range(w) for r in (cy - 1, cy)} \
        | {(r, c) for r in range(h) for c in (cx - 1, cx)}
    return sorted(cross - near)


def _opp_start(cfg, boost, b0, z0, s0):
    """Seat-1 start attributes by opponent boost tier (sim/torch_sim.py:433-453):
    0 = seat 0's, 1 = x opp_hist_mult rounded (half to even) and capped, 2 =
    the opp_growth_* constants; float32 arithmetic."""
    m = F32(cfg.opp_hist_mult)
    if boost == 2:
        return int(cfg.opp_growth_bombs), int(cfg.opp_growth_blast), F32(cfg.opp_growth_speed)
    if boost == 1:
        b = min(np.rint(F32(b0) * m), F32(cfg.growth_bombs_max))
        z = min(np.rint(F32(z0) * m), F32(cfg.growth_blast_max))
        s = min(F32(s0) * m, F32(cfg.growth_speed_max))
        return int(b), int(z), F32(s)
    return int(b0), int(z0), F32(s0)


def map_reset(cfg, st, mask, dr, opp_boost=None, aux=None):
    """Reset the envs in `mask` to new levels built from the draws `dr`
    (mapgen_draws_keyed's keys), in place: the reference's reset_
    (sim/torch_sim.py:178-420) with sim/mapgen.py's make_walls (:15-62),
    make_open_obstacles (:65-95), make_bricks (:98-194), make_ring_bricks
    (:197-227) and make_ring_walls (:230-242).  opp_boost: (N,) tier per env
    (default 0).  aux: optional dict receiving "is_open" (N,) bool and
    "map_kind" (N,) int64 (1 open, 2 ring, 0 corridor)."""
    h, w, p = cfg.height, cfg.width, cfg.n_players
    corridor = cfg.map_mode == "corridor"
    rows = np.arange(h)[:, None]
    cols = np.arange(w)[None, :]
    c0 = (w - cfg.corridor_width) // 2
    c1 = c0 + cfg.corridor_width
    T = cfg.top_wall_rows
    edge = [c for c in (c0, c0 + 1, c1 - 2, c1 - 1) if c0 <= c < c1]
    r0 = (h - cfg.ring_center_h) // 2
    q0 = (w - cfg.ring_center_w) // 2
    r1, q1 = r0 + cfg.ring_center_h, q0 + cfg.ring_center_w
    cross = _open_cross(cfg)
    spawn = {"corr": np.array(cfg.spawn_pos(), F32), "open": _open_spawn_pos(cfg),
             "ring": np.array(cfg.ring_spawns(), F32)}
    t_pure = F32(cfg.pure_open_fraction)
    t_open = F32(cfg.pure_open_fraction + cfg.open_fraction)
    t_ring = F32(cfg.pure_open_fraction + cfg.open_fraction + cfg.ring_fraction)
    dens = F32(cfg.wall_density)
    for e in np.nonzero(np.asarray(mask, bool))[0]:
        if corridor:
            r = F32(dr["kind_u"][e])
            kind = "pure" if r < t_pure else ("open" if r < t_open else
                                               ("ring" if r < t_ring else "corr"))
        else:
            kind = "openmode"
        wall = np.zeros((h, w), bool)
        brick = np.zeros((h, w), bool)
        if kind in ("pure", "open", "openmode"):
            k = cfg.open_obstacle_max
            if k > 0:
                key = np.asarray(dr["obst_key"][e])
                order = np.argsort(key, kind="stable")[:k]
                for cell in order[: int(dr["obst_n"][e])]:
                    wall[min(cell // w, h - 1), min(cell % w, w - 1)] = True
                _clear4(wall, cfg.spawn_cells(), h, w)
            if kind == "pure":
                wall[:] = False
        elif kind == "ring":
            wall[r0:r1, q0:q1] = True
            band = np.zeros((h, w), bool)
            band[r0 - 1:r1 + 1, q0 - 1:q1 + 1] = True
            band[r0:r1, q0:q1] = False
            brick = band & (np.asarray(dr["ring_u"][e], F32).reshape(h, w) < F32(cfg.ring_brick_density))
            _clear4(brick, cfg.ring_spawn_cells(), h, w)
        else:
            top = int(dr["top"][e]) if cfg.random_wall_rows else None
            if top is not None:
                bot = T - top
                wall = np.broadcast_to((rows < top) | (rows >= h - bot), (h, w)).copy()
                brick = ((cols < c0) | (cols >= c1)) & ~(rows < top)
            else:
                wall[:T] = True
                brick = ((cols < c0) | (cols >= c1)) & ~(rows < T)
            _clear4(wall, cfg.spawn_cells(), h, w)
            if cfg.wall_density > 0:
                if top is None:
                    span, base = F32(h - T - 4), F32(T)
                else:
                    span, base = F32(max(h - (T - top) - 4 - top, 1)), F32(top)
                for i, col in enumerate(edge):
                    start = int(F32(F32(dr["vstart_u"][e][i]) * span) + base)
                    ln = 2 + int(F32(dr["vlen_u"][e][i]) * F32(3.0))
                    if F32(dr["vact_u"][e][i]) < dens:
                        brick[max(start, 0):max(start + ln, 0), col] = True
                if c1 - c0 > 4:
                    hs = int(F32(F32(dr["hstart_u"][e]) * F32(c1 - c0 - 4)) + F32(c0))
                    hl = 2 + int(F32(dr["hlen_u"][e]) * F32(3.0))
                    if F32(dr["hact_u"][e]) < dens:
                        band_rows = range(T, T + min(2, h - T)) if top is None else (top, top + 1)
                        seg = (np.arange(c0, c1) >= hs) & (np.arange(c0, c1) < hs + hl)
                        for rr in band_rows:
                            brick[rr, c0:c1] |= seg
            _clear4(brick, cfg.spawn_cells(), h, w)
        st["wall"][e] = wall
        st["brick"][e] = brick
        # start attributes of seats 0 and 1 (other seats keep theirs)
        if kind == "openmode":
            b0, z0, s0 = int(cfg.max_bombs), int(cfg.blast), F32(1.0)
        elif kind in ("pure", "open"):
            b0, z0, s0 = int(cfg.open_growth_bombs), int(cfg.open_growth_blast), F32(cfg.open_growth_speed)
        else:
            b0, z0, s0 = (int(cfg.growth_bombs_start), int(cfg.growth_blast_start),
                          F32(cfg.growth_speed_start))
        bo = 0 if opp_boost is None else int(opp_boost[e])
        caps = [(b0, z0, s0), _opp_start(cfg, bo, b0, z0, s0)]
        for pl, (bb, zz, ss) in enumerate(caps[:p]):
            st["bombs_cap"][e, pl] = st["lo_bombs"][e, pl] = bb
            st["blast_cap"][e, pl] = st["lo_blast"][e, pl] = zz
            st["spd_g"][e, pl] = st["lo_spd"][e, pl] = ss
        if corridor:
            st["crate_prob"][e] = {"pure": F32(1.0), "open": F32(1.0), "ring": F32(cfg.ring_crate_prob),
                                   "corr": F32(cfg.growth_crate_prob)}[kind]
        sp = spawn["corr" if kind == "corr" else ("ring" if kind == "ring" else "open")]
        pos = sp.copy()
        if F32(dr["swap_u"][e]) < F32(0.5) and p >= 2:
            pos[[0, 1]] = pos[[1, 0]]
        st["pos"][e] = pos
        st["crate"][e] = False
        if corridor and cfg.open_crate_cross and kind in ("pure", "open"):
            for rr, cc in cross:
                st["crate"][e, rr, cc] = True
        st["recycle"][e] = False
        st["pending_lost"][e] = 0
        st["combo"][e] = 0
        st["last_hit"][e] = -10 ** 9
        st["fuse"][e] = 0
        st["owner"][e] = -1
        st["bomb_blast"][e] = 0
        st["alive"][e] = True
        st["hp"][e] = cfg.max_hp
        st["since_bomb"][e] = cfg.place_dist_cooldown
        st["invuln"][e] = 0
        st["t"][e] = 0
        if cfg.hazard_fraction > 0:
            hz = F32(dr["hazard_u"][e]) < F32(cfg.hazard_fraction)
            st["hazard"][e] = hz
            if hz:
                st["bombs_cap"][e] = 0
        else:
            st["hazard"][e] = False
        if aux is not None:
            aux["is_open"][e] = corridor and kind in ("pure", "open")
            aux["map_kind"][e] = {"openmode": 1, "pure": 1, "open": 1, "ring": 2, "corr": 0}[kind]
    return st
