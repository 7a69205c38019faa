"""B200Sim: the reference `BatchedSim` API on the B200 kernels.

State lives on the device with env-major planes [N][H*W] (a warp simulates
one env and reads its planes as one contiguous run; a block of 8 envs
stages 8 consecutive rows), per-player arrays [P][N] and positions
[P][2][N].  The public attributes (`sim.fuse`, `sim.pos`, ...) are torch
views with the reference's shapes ((N,H,W), (N,P), (N,P,2)) -- the planes
plain contiguous tensors -- so bots, tests and callers that index or poke
them work unchanged and without copies; assigning to an attribute copies
into the device buffer.

Per tick the engine runs three library calls (observe, one step, plus the
policy and bot calls made by the caller); nothing in `observe`, `legal_mask`
or a template-reset `step` synchronises the host, so a tick can be captured
into a CUDA graph.  Reference call sites: sim/torch_sim.py:53-1466.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _capi as capi
from . import mapgen
from .config import SimConfig

_PLANES = {"wall": torch.bool, "brick": torch.bool, "crate": torch.bool,
           "_recycle_crate": torch.bool, "fuse": torch.int16, "owner": torch.int8,
           "bomb_blast": torch.int16}
_PLAYER = {"alive": torch.bool, "hp": torch.uint8, "since_bomb": torch.int32,
           "bombs_cap": torch.int64, "blast_cap": torch.int64, "spd_g": torch.float32,
           "invuln": torch.int64, "_pending_lost": torch.int64, "_combo": torch.int64,
           "_last_hit": torch.int64, "_lo_bombs": torch.int64, "_lo_blast": torch.int64,
           "_lo_spd": torch.float32}
_ENV = {"t": torch.int64, "crate_prob": torch.float32, "_hazard": torch.bool,
        "_is_open": torch.bool, "_map_kind": torch.int64, "_opp_boost": torch.int64}
# ctypes QqtState field -> attribute name
_CSTATE = {"wall": "wall", "brick": "brick", "crate": "crate", "recycle": "_recycle_crate",
           "fuse": "fuse", "owner": "owner", "bomb_blast": "bomb_blast", "pos": "pos",
           "alive": "alive", "hp": "hp", "since_bomb": "since_bomb", "t": "t",
           "bombs_cap": "bombs_cap", "blast_cap": "blast_cap", "spd_g": "spd_g",
           "invuln": "invuln", "pending_lost": "_pending_lost", "combo": "_combo",
           "last_hit": "_last_hit", "lo_bombs": "_lo_bombs", "lo_blast": "_lo_blast",
           "lo_spd": "_lo_spd", "crate_prob": "crate_prob", "hazard": "_hazard"}


def check_tile_flags(tiles: torch.Tensor, n: int) -> None:
    """K-tile flags of n observation rows: a contiguous (n, 4) int32 tensor
    whose storage starts on a 16-byte boundary."""
    if (tiles.dtype != torch.int32 or tuple(tiles.shape) != (n, 4) or not tiles.is_contiguous()
            or tiles.data_ptr() % 16):
        raise ValueError("K-tile flags must be a contiguous, 16-byte aligned (N, 4) int32 tensor")


def tile_flag_words(lo: int, hi: int, device) -> torch.Tensor:
    """(4,) int32 flag words of every 64-entry K tile that overlaps row
    entries [lo, hi): tile t is bit min(t >> 2, 31) of word t & 3."""
    words = [0, 0, 0, 0]
    for t in range(lo // 64, (hi + 63) // 64):
        words[t & 3] |= 1 << min(t >> 2, 31)
    return torch.tensor([w - (1 << 32) if w >= 1 << 31 else w for w in words],
                        dtype=torch.int32, device=device)


def tile_flags(rows: torch.Tensor) -> torch.Tensor:
    """(N, 4) int32 K-tile flags of fp16 observation rows (N, stride) -- bit
    min(t >> 2, 31) of word t & 3 set when entries [64 t, 64 t + 64) of the
    row hold a nonzero bit pattern -- for callers that build rows
    themselves (the step's fused observation writes the same words)."""
    n, k = rows.shape
    kt = (k + 63) // 64
    bits = rows.contiguous().view(torch.int16) != 0
    if kt * 64 != k:
        bits = torch.nn.functional.pad(bits, (0, kt * 64 - k))
    nz = bits.view(n, kt, 64).any(-1).to(torch.int64)
    t = torch.arange(kt, device=rows.device)
    shifted = nz << torch.clamp(t >> 2, max=31)
    words = torch.zeros((n, 4), dtype=torch.int64, device=rows.device)
    for t0 in range(kt):
        words[:, t0 & 3] |= shifted[:, t0]
    words = torch.where(words >= 1 << 31, words - (1 << 32), words)
    return words.to(torch.int32)


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def make_ccfg(cfg: SimConfig, n_envs: int, explore_coef: float = 1.0,
              obs_stride: int | None = None) -> capi.QqtCfg:
    """Scalar config for the kernels; float fields are the float32 values the
    reference multiplies by (double products rounded once)."""
    c = capi.QqtCfg()
    hw = cfg.height * cfg.width
    fp32 = not cfg.obs_fp16
    stride = obs_stride or _round_up(cfg.n_channels * hw, 4 if fp32 else 8)
    ints = dict(n_envs=n_envs, height=cfg.height, width=cfg.width, n_players=cfg.n_players,
                fuse=cfg.fuse, blast=cfg.blast, max_steps=cfg.max_steps,
                invuln_ticks=cfg.invuln_ticks, max_hp=cfg.max_hp,
                resolve_rounds=min(cfg.max_chain - 1, cfg.chain_cap_rounds),
                danger_rounds=(min(cfg.max_chain, cfg.chain_cap_rounds)
                               if cfg.max_chain > 1 else 0),
                corridor=int(cfg.map_mode == "corridor"),
                hit_attr_penalty=cfg.hit_attr_penalty, growth_bombs_max=cfg.growth_bombs_max,
                growth_blast_max=cfg.growth_blast_max,
                place_dist_cooldown=cfg.place_dist_cooldown,
                crate_speed_only=int(cfg.crate_speed_only), timeout_draw=int(cfg.timeout_draw),
                win_hp_scaled=int(cfg.win_hp_scaled), combo_on=int(cfg.combo_reward > 0),
                obs_extra=int(cfg.obs_extra_enabled), obs_channels=cfg.n_channels,
                obs_stride=stride, obs_fp32=int(fp32))
    floats = dict(radius=cfg.radius, step_len=cfg.step_len, move_eps2=2e-4,
                  step_penalty=cfg.step_penalty, hit_reward=cfg.hit_reward,
                  brick_reward=cfg.brick_reward,
                  danger_penalty=explore_coef * cfg.danger_penalty,
                  explore_coef=explore_coef, place_cover_reward=cfg.place_cover_reward,
                  place_chain_reward=cfg.place_chain_reward,
                  place_dist_reward=cfg.place_dist_reward,
                  place_dist_radius=cfg.place_dist_radius,
                  chain_time_factor=cfg.chain_time_factor,
                  chain_time_rest=1.0 - cfg.chain_time_factor,
                  growth_speed_step=cfg.growth_speed_step,
                  growth_speed_max=cfg.growth_speed_max,
                  pen_speed=cfg.hit_attr_penalty * cfg.growth_speed_step,
                  recycle_crate_prob=cfg.recycle_crate_prob, combo_reward=cfg.combo_reward,
                  combo_gap_factor=cfg.combo_gap_factor, win_bonus=cfg.win_bonus,
                  win_bonus_per_hp=cfg.win_bonus / cfg.max_hp,
                  chain_blast_bonus=(cfg.chain_blast_bonus if cfg.max_chain > 1 else 0.0),
                  obs_growth_bombs_max=float(cfg.growth_bombs_max), fuse_f=float(cfg.fuse),
                  max_steps_f=float(cfg.max_steps), h_minus_rad=cfg.height - cfg.radius,
                  w_minus_rad=cfg.width - cfg.radius)
    for k, v in ints.items():
        setattr(c, k, int(v))
    for k, v in floats.items():
        setattr(c, k, float(v))
    # hazard waves (sim/torch_sim.py:1404-1466); the seed is set per step
    c.hazard_on = int(cfg.hazard_fraction > 0)
    c.hazard_wave_ticks = int(cfg.hazard_wave_ticks)
    c.hazard_bombs_min, c.hazard_bombs_max = int(cfg.hazard_bombs_min), int(cfg.hazard_bombs_max)
    c.hazard_blast_min, c.hazard_blast_max = int(cfg.hazard_blast_min), int(cfg.hazard_blast_max)
    c.hazard_ramp_ticks = float(cfg.hazard_ramp_seconds * cfg.tick_hz)
    return c


class B200Sim:
    """Drop-in for `sim.torch_sim.BatchedSim` backed by libqqt_b200.so."""

    def __init__(self, cfg: SimConfig, num_envs: int, device: str | torch.device = "cuda",
                 seed: int = 0, template: dict | None = None, map_reset: str = "host") -> None:
        """map_reset: "host" builds every new episode's level on the host
        generator in the reference's draw order (bit-compatible with a
        reference BatchedSim of the same seed); "device" builds it on the GPU
        from counter-based draws (qqt_map_reset), so resets -- the initial one
        included -- never return to the host.  A template (set_template)
        replaces both with a fixed per-env level."""
        self.cfg = cfg
        self.num_envs = n = int(num_envs)
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("B200Sim runs on a CUDA device only (no CPU fallback)")
        capi.lib()
        self.gen = torch.Generator(device="cpu").manual_seed(seed)
        self._flush_seed = (int(seed) * 0x2545F4914F6CDD1D + 0x1234567) & ((1 << 64) - 1)
        h, w, p = cfg.height, cfg.width, cfg.n_players
        hw = h * w
        d = self.device
        self._buf = {}
        for k, dt in _PLANES.items():
            self._buf[k] = torch.zeros((n, hw), dtype=dt, device=d)
        self._buf["owner"].fill_(-1)
        for k, dt in _PLAYER.items():
            self._buf[k] = torch.zeros((p, n), dtype=dt, device=d)
        self._buf["pos"] = torch.zeros((p, 2, n), dtype=torch.float32, device=d)
        for k, dt in _ENV.items():
            self._buf[k] = torch.zeros((n,), dtype=dt, device=d)
        self._buf["alive"].fill_(True)
        self._buf["hp"].fill_(cfg.max_hp)
        self._buf["_last_hit"].fill_(-10 ** 9)
        self._buf["crate_prob"].fill_(cfg.growth_crate_prob)
        self._buf["_lo_bombs"].fill_(cfg.growth_bombs_start)
        self._buf["_lo_blast"].fill_(cfg.growth_blast_start)
        self._buf["_lo_spd"].fill_(cfg.growth_speed_start)
        self._buf["spd_g"].fill_(1.0)
        self._explore_coef = 1.0
        # hazard-wave draws: keyed by (seed, env, tick); None derives a new
        # seed for every step call, an int fixes it (parity checks)
        self.hazard_seed: int | None = None
        self._hazard_calls = 0
        self._hazard_base = (int(seed) * 0x9E3779B97F4A7C15 + 0x5851F42D4C957F2D) & ((1 << 64) - 1)
        self.speed_mult = None
        self._rand_buf: torch.Tensor | None = None
        self._ccfg = make_ccfg(cfg, n, 1.0)
        self.obs_stride = int(self._ccfg.obs_stride)
        obs_dt = torch.float16 if cfg.obs_fp16 else torch.float32
        self._obs = torch.zeros((n, self.obs_stride), dtype=obs_dt, device=d)
        self._danger = torch.zeros((n, hw), dtype=torch.float32, device=d)
        self._mm = torch.ones((n, p, 5), dtype=torch.bool, device=d)
        self._bm = torch.ones((n, p, 2), dtype=torch.bool, device=d)
        self._reward = torch.zeros((n, p), dtype=torch.float32, device=d)
        self._done = torch.zeros((n,), dtype=torch.bool, device=d)
        self._died = torch.zeros((n, p), dtype=torch.bool, device=d)
        self._winner = torch.zeros((n, p), dtype=torch.bool, device=d)
        self._hit = torch.zeros((n, p), dtype=torch.bool, device=d)
        self._n_alive = torch.zeros((n,), dtype=torch.int64, device=d)
        self._covered = torch.zeros((n, hw), dtype=torch.bool, device=d)
        self._triggered = torch.zeros((n, hw), dtype=torch.bool, device=d)
        self._reset_mask = torch.zeros((n,), dtype=torch.bool, device=d)
        self._tiers = torch.full((1,), -1, dtype=torch.int32, device=d)
        self._first_step = True
        nb = int(capi.lib().qqt_step_scratch_bytes(ctypes.byref(self._ccfg)))
        self._step_scratch = torch.zeros((max(nb, 256),), dtype=torch.uint8, device=d)
        # K-tile flag words of the observation's crate channel (a recycle
        # rewrites it), made here so no later call copies from the host
        ch = 2 * cfg.n_players + 3
        self._crate_tile_words = (tile_flag_words(ch * hw, (ch + 1) * hw, d)
                                  if cfg.n_channels > ch else None)
        self._tmpl = None
        self._mapgen = None
        self._cstate = self._make_cstate()
        self._cout = self._make_cout()
        if map_reset not in ("host", "device"):
            raise ValueError("map_reset is 'host' or 'device'")
        if template is not None:
            self.set_template(template, apply=True)
        else:
            if map_reset == "device":
                self.enable_device_map_reset(seed)
            self.reset_all()

    # ------------------------------------------------------------ views
    def _view(self, key):
        b = self._buf[key]
        n, cfg = self.num_envs, self.cfg
        if key in _PLANES:
            return b.view(n, cfg.height, cfg.width)
        if key in _PLAYER:
            return b.t()
        if key == "pos":
            return b.permute(2, 0, 1)
        return b

    def _make_cstate(self):
        s = capi.QqtState()
        for f, key in _CSTATE.items():
            setattr(s, f, self._buf[key].data_ptr())
        return s

    def _make_cout(self):
        o = capi.QqtStepOut()
        o.reward = self._reward.data_ptr()
        o.done = self._done.data_ptr()
        o.died = self._died.data_ptr()
        o.winner = self._winner.data_ptr()
        o.n_alive = self._n_alive.data_ptr()
        o.covered = self._covered.data_ptr()
        o.triggered = self._triggered.data_ptr()
        o.reset_mask = self._reset_mask.data_ptr()
        o.hit = self._hit.data_ptr()
        return o

    def _stream(self):
        return capi.stream_ptr(self.device)

    # ----------------------------------------------------- templates / reset
    def set_template(self, template: dict, apply: bool = True, seed: int = 0,
                     swap_spawns: bool = False) -> None:
        """Install per-env reset templates and switch auto-reset to the device.

        template: numpy/torch arrays, env-major like the reference:
          wall, brick (N,H,W) bool; optional crate (N,H,W); spawn (N,P,2);
          bombs_cap, blast_cap (N,P) int; spd (N,P) float; crate_prob (N,).
        Done envs are then reset inside the step kernel to their template,
        with no host round trip (the benchmark configurations' reset rule).
        """
        n, p, hw = self.num_envs, self.cfg.n_players, self.cfg.n_cells
        d = self.device
        T = lambda a, dt: torch.as_tensor(np.asarray(a)).to(d, dt)  # noqa: E731
        tm = {
            "wall": T(template["wall"], torch.bool).reshape(n, hw).contiguous(),
            "brick": T(template["brick"], torch.bool).reshape(n, hw).contiguous(),
            "crate": T(template.get("crate", np.zeros((n, hw), bool)), torch.bool)
            .reshape(n, hw).contiguous(),
            "spawn": T(template["spawn"], torch.float32).permute(1, 2, 0).contiguous(),
            "bombs_cap": T(template["bombs_cap"], torch.int64).t().contiguous(),
            "blast_cap": T(template["blast_cap"], torch.int64).t().contiguous(),
            "spd": T(template["spd"], torch.float32).t().contiguous(),
            "crate_prob": T(template["crate_prob"], torch.float32).contiguous(),
            "episode": torch.zeros((n,), dtype=torch.int64, device=d),
        }
        self._tmpl_buf = tm
        c = capi.QqtTemplate()
        for k in ("wall", "brick", "crate", "spawn", "bombs_cap", "blast_cap", "spd",
                  "crate_prob", "episode"):
            setattr(c, k, tm[k].data_ptr())
        c.seed = int(seed) & ((1 << 64) - 1)
        c.swap_spawns = int(swap_spawns)
        c.since_bomb0 = int(self.cfg.place_dist_cooldown)
        self._tmpl = c
        if apply:
            self._apply_template(torch.ones(n, dtype=torch.bool, device=d))

    def enable_device_map_reset(self, seed: int = 0) -> None:
        """Generate each ended episode's next level on the device (the
        reference's reset_, sim/torch_sim.py:178-420, with counter-based
        draws keyed by (seed, env, episode)): `reset_`, `reset_all` and
        `step(auto_reset=True)` then run qqt_map_reset and never synchronise
        the host.  Installing a template afterwards takes precedence."""
        cfg, n, d = self.cfg, self.num_envs, self.device
        if cfg.n_players > 4:
            raise ValueError("device level generation supports up to 4 players")
        self._mg_episode = torch.zeros((n,), dtype=torch.int64, device=d)
        self._mapgen = _make_mapgen(cfg, seed, self._mg_episode, self._buf["_opp_boost"],
                                    self._buf["_is_open"], self._buf["_map_kind"])

    def _device_map_reset(self, done: torch.Tensor, rows=None, mm=None, bm=None,
                          tiles=None) -> None:
        capi.check(capi.lib().qqt_map_reset(
            ctypes.byref(self._ccfg), ctypes.byref(self._cstate), ctypes.byref(self._mapgen),
            done.data_ptr(), capi.ptr(rows), capi.ptr(mm), capi.ptr(bm), capi.ptr(tiles),
            self._stream()),
            "qqt_map_reset")

    def _apply_template(self, mask: torch.Tensor) -> None:
        tm, b = self._tmpl_buf, self._buf
        idx = mask.nonzero(as_tuple=True)[0]
        if idx.numel() == 0:
            return
        for k in ("wall", "brick"):
            b[k][idx] = tm[k][idx]
        b["crate"][idx] = tm["crate"][idx]
        b["_recycle_crate"][idx] = False
        b["fuse"][idx] = 0
        b["owner"][idx] = -1
        b["bomb_blast"][idx] = 0
        b["pos"][:, :, idx] = tm["spawn"][:, :, idx]
        b["bombs_cap"][:, idx] = tm["bombs_cap"][:, idx]
        b["blast_cap"][:, idx] = tm["blast_cap"][:, idx]
        b["spd_g"][:, idx] = tm["spd"][:, idx]
        b["_lo_bombs"][:, idx] = tm["bombs_cap"][:, idx]
        b["_lo_blast"][:, idx] = tm["blast_cap"][:, idx]
        b["_lo_spd"][:, idx] = tm["spd"][:, idx]
        b["crate_prob"][idx] = tm["crate_prob"][idx]
        self._reset_common(idx)

    def _reset_common(self, idx) -> None:
        b, cfg = self._buf, self.cfg
        b["_recycle_crate"][idx] = False
        b["_pending_lost"][:, idx] = 0
        b["_combo"][:, idx] = 0
        b["_last_hit"][:, idx] = -10 ** 9
        b["fuse"][idx] = 0
        b["owner"][idx] = -1
        b["bomb_blast"][idx] = 0
        b["alive"][:, idx] = True
        b["hp"][:, idx] = cfg.max_hp
        b["since_bomb"][:, idx] = cfg.place_dist_cooldown
        b["invuln"][:, idx] = 0
        b["t"][idx] = 0

    def reset_all(self) -> None:
        self.reset_(torch.ones((self.num_envs,), dtype=torch.bool, device=self.device))

    def _opp_start(self, idx, b0, z0, s0):
        """Seat-1 start attributes by opponent boost tier (sim/torch_sim.py:433-453)."""
        cfg = self.cfg
        bo = self._buf["_opp_boost"][idx].cpu()
        m = cfg.opp_hist_mult
        b = torch.where(bo == 2, torch.full_like(b0, cfg.opp_growth_bombs),
                        torch.where(bo == 1, (b0 * m).round().clamp(max=cfg.growth_bombs_max), b0))
        z = torch.where(bo == 2, torch.full_like(z0, cfg.opp_growth_blast),
                        torch.where(bo == 1, (z0 * m).round().clamp(max=cfg.growth_blast_max), z0))
        s = torch.where(bo == 2, torch.full_like(s0, cfg.opp_growth_speed),
                        torch.where(bo == 1, (s0 * m).clamp(max=cfg.growth_speed_max), s0))
        return b.long(), z.long(), s

    def reset_(self, mask: torch.Tensor) -> None:
        """Reset the masked envs on the host generator (sim/torch_sim.py:178-420).

        With a device template installed, envs reset to their template
        instead (the benchmark configurations)."""
        if self._tmpl is not None:
            self._apply_template(mask.to(self.device))
            return
        if self._mapgen is not None:
            flags = mask.to(self.device, torch.bool).contiguous().view(torch.uint8)
            self._device_map_reset(flags)
            return
        cfg, b, d = self.cfg, self._buf, self.device
        idx_cpu = mask.detach().to("cpu").nonzero(as_tuple=True)[0]
        count = int(idx_cpu.numel())
        if count == 0:
            return
        idx = idx_cpu.to(d)
        hw, p, gen = cfg.n_cells, cfg.n_players, self.gen
        b["_is_open"][idx] = False
        put = lambda key, rows, val: b[key].__setitem__(rows, val)  # noqa: E731
        if cfg.map_mode != "corridor":
            wall = mapgen.open_obstacles(cfg, count, gen)
            put("wall", idx, wall.reshape(count, hw).to(d))
            put("brick", idx, False)
            b0 = torch.full((count,), float(cfg.max_bombs))
            z0 = torch.full((count,), float(cfg.blast))
            s0 = torch.full((count,), 1.0)
            ob, oz, os_ = self._opp_start(idx, b0, z0, s0)
            caps = [(cfg.max_bombs, cfg.blast, 1.0), (ob, oz, os_)]
            self._set_caps(idx, caps)
            b["_map_kind"][idx] = 1
            pos = torch.tensor(cfg.spawn_pos(), dtype=torch.float32)
            pos = pos.unsqueeze(0).expand(count, -1, -1).clone()
            sw = torch.rand(count, generator=gen) < 0.5
        else:
            r = torch.rand(count, generator=gen)
            pf = cfg.pure_open_fraction
            is_pure = r < pf
            is_open = ~is_pure & (r < pf + cfg.open_fraction)
            is_ring = ~(is_pure | is_open) & (r < pf + cfg.open_fraction + cfg.ring_fraction)
            is_corr = ~(is_pure | is_open | is_ring)
            wall = torch.zeros((count, cfg.height, cfg.width), dtype=torch.bool)
            brick = torch.zeros_like(wall)
            bcap = torch.zeros((count, p), dtype=torch.long)
            zcap = torch.zeros((count, p), dtype=torch.long)
            scap = torch.zeros((count, p), dtype=torch.float32)
            cprob = torch.zeros((count,), dtype=torch.float32)
            kind = torch.zeros((count,), dtype=torch.long)
            opn = is_pure | is_open
            if opn.any():
                no = int(opn.sum())
                wa = mapgen.open_obstacles(cfg, no, gen)
                wa[is_pure[opn]] = False
                wall[opn] = wa
                self._fill_caps(bcap, zcap, scap, opn, idx, cfg.open_growth_bombs,
                                cfg.open_growth_blast, cfg.open_growth_speed)
                cprob[opn] = 1.0
                kind[opn] = 1
            if is_ring.any():
                nr = int(is_ring.sum())
                wall[is_ring] = mapgen.ring_walls(cfg, nr)
                brick[is_ring] = mapgen.ring_bricks(cfg, nr, gen)
                self._fill_caps(bcap, zcap, scap, is_ring, idx, cfg.growth_bombs_start,
                                cfg.growth_blast_start, cfg.growth_speed_start)
                cprob[is_ring] = cfg.ring_crate_prob
                kind[is_ring] = 2
            if is_corr.any():
                nc = int(is_corr.sum())
                tr = (torch.randint(0, cfg.top_wall_rows + 1, (nc,), generator=gen)
                      if cfg.random_wall_rows else None)
                wall[is_corr] = mapgen.walls(cfg, nc, gen, top_rows=tr)
                brick[is_corr] = mapgen.bricks(cfg, nc, gen, top_rows=tr)
                self._fill_caps(bcap, zcap, scap, is_corr, idx, cfg.growth_bombs_start,
                                cfg.growth_blast_start, cfg.growth_speed_start)
                cprob[is_corr] = cfg.growth_crate_prob
            put("wall", idx, wall.reshape(count, hw).to(d))
            put("brick", idx, brick.reshape(count, hw).to(d))
            # seats 0 and 1 only: the reference's reset_ leaves the start
            # attributes of any further seat as they were
            q = min(p, 2)
            b["bombs_cap"][:q, idx] = bcap[:, :q].t().to(d)
            b["blast_cap"][:q, idx] = zcap[:, :q].t().to(d)
            b["spd_g"][:q, idx] = scap[:, :q].t().to(d)
            b["_lo_bombs"][:q, idx] = bcap[:, :q].t().to(d)
            b["_lo_blast"][:q, idx] = zcap[:, :q].t().to(d)
            b["_lo_spd"][:q, idx] = scap[:, :q].t().to(d)
            b["crate_prob"][idx] = cprob.to(d)
            b["_map_kind"][idx] = kind.to(d)
            b["_is_open"][idx] = opn.to(d)
            pos = torch.zeros((count, p, 2), dtype=torch.float32)
            if opn.any():
                pos[opn] = torch.tensor(mapgen.open_spawns(cfg), dtype=torch.float32)
            if is_ring.any():
                pos[is_ring] = torch.tensor(cfg.ring_spawns(), dtype=torch.float32)
            if is_corr.any():
                pos[is_corr] = torch.tensor(cfg.spawn_pos(), dtype=torch.float32)
            sw = torch.rand(count, generator=gen) < 0.5
        if bool(sw.any()):
            tmp = pos[sw, 0].clone()
            pos[sw, 0] = pos[sw, 1]
            pos[sw, 1] = tmp
        b["pos"][:, :, idx] = pos.permute(1, 2, 0).to(d)
        b["crate"][idx] = False
        self._reset_common(idx)
        if cfg.open_crate_cross and cfg.map_mode == "corridor":
            open_idx = idx[b["_is_open"][idx]]
            if open_idx.numel():
                cells = torch.tensor([r * cfg.width + c for r, c in mapgen.open_cross_cells(cfg)],
                                     dtype=torch.long, device=d)
                b["crate"][open_idx.unsqueeze(1), cells.unsqueeze(0)] = True
        if cfg.hazard_fraction > 0:
            hz = torch.rand(count, generator=gen) < cfg.hazard_fraction
            b["_hazard"][idx] = hz.to(d)
            hz_idx = idx[hz.to(d)]
            if hz_idx.numel():
                b["bombs_cap"][:, hz_idx] = 0
        else:
            b["_hazard"][idx] = False

    def _set_caps(self, idx, caps):
        b, d = self._buf, self.device
        for pl, (bb, zz, ss) in enumerate(caps[:2]):
            for key, v in (("bombs_cap", bb), ("blast_cap", zz), ("spd_g", ss)):
                val = v.to(d) if isinstance(v, torch.Tensor) else v
                b[key][pl, idx] = val
                lo = {"bombs_cap": "_lo_bombs", "blast_cap": "_lo_blast", "spd_g": "_lo_spd"}[key]
                b[lo][pl, idx] = val

    def _fill_caps(self, bcap, zcap, scap, sel, idx, b_start, z_start, s_start):
        k = int(sel.sum())
        b0 = torch.full((k,), float(b_start))
        z0 = torch.full((k,), float(z_start))
        s0 = torch.full((k,), float(s_start))
        ob, oz, os_ = self._opp_start(idx[sel.to(idx.device)], b0, z0, s0)
        bcap[sel, 0], zcap[sel, 0], scap[sel, 0] = b_start, z_start, s_start
        bcap[sel, 1], zcap[sel, 1], scap[sel, 1] = ob, oz, os_

    def set_opp_boost(self, v: int) -> None:
        self._buf["_opp_boost"].fill_(int(v))

    def set_explore_coef(self, v: float) -> None:
        self._explore_coef = float(v)
        self._ccfg = make_ccfg(self.cfg, self.num_envs, self._explore_coef, self.obs_stride)

    # -------------------------------------------------------------- tick
    def observe(self) -> torch.Tensor:
        """(N, C, H, W) shared observation (fp16 by default); a view of a
        persistent, row-padded buffer (sim/torch_sim.py:605-627)."""
        capi.check(capi.lib().qqt_observe(ctypes.byref(self._ccfg), ctypes.byref(self._cstate),
                                          self._obs.data_ptr(), self._danger.data_ptr(), None,
                                          None, self._stream()), "qqt_observe")
        return self.obs_view()

    def obs_view(self) -> torch.Tensor:
        cfg = self.cfg
        c = cfg.n_channels * cfg.n_cells
        return self._obs[:, :c].view(self.num_envs, cfg.n_channels, cfg.height, cfg.width)

    def observe_and_mask(self, obs_out=None, mm_out=None, bm_out=None, danger=True):
        """observe() and legal_mask() in one launch.

        obs_out (N, obs_stride) / mm_out (N,P,5) / bm_out (N,P,2): optional
        contiguous slots (rollout-buffer rows) written directly."""
        ob = self._obs if obs_out is None else obs_out
        mm = self._mm if mm_out is None else mm_out
        bm = self._bm if bm_out is None else bm_out
        capi.check(capi.lib().qqt_observe(ctypes.byref(self._ccfg), ctypes.byref(self._cstate),
                                          ob.data_ptr(), self._danger.data_ptr() if danger else None,
                                          mm.data_ptr(), bm.data_ptr(), self._stream()),
                   "qqt_observe")
        cfg = self.cfg
        c = cfg.n_channels * cfg.n_cells
        view = ob[:, :c].view(self.num_envs, cfg.n_channels, cfg.height, cfg.width)
        return view, mm, bm

    def local_view_features(self, obs: torch.Tensor | None = None, only_p0: bool = False):
        """Per-player LSTM features (sim/obs.py:241-340) -> (local (N,Po,C,7,7),
        rel (N,Po,10,6), glob (N,Po,5)) in the observation's dtype, Po = 1 with
        only_p0 else P.  obs: observation rows of this sim's layout ((N,
        obs_stride) rows, or the (N,C,H,W) view observe() returns); None
        reads the sim's own buffer (the last observe()).  Bomb slots at equal
        distance come in ascending cell order (the reference leaves their
        order to torch.topk)."""
        rows = self._obs if obs is None else obs
        if rows.dim() == 4:                      # a view of (N, obs_stride) rows
            if rows.stride(0) != self.obs_stride:
                raise ValueError("pass observation rows (N, obs_stride) or observe()'s view")
            rows = torch.as_strided(rows, (rows.shape[0], self.obs_stride), (self.obs_stride, 1))
        if tuple(rows.shape) != (self.num_envs, self.obs_stride) or rows.dtype != self._obs.dtype:
            raise ValueError("observation rows must be (N, obs_stride) of the sim's dtype")
        cfg = self.cfg
        po = 1 if only_p0 else cfg.n_players
        n, c = self.num_envs, cfg.n_channels
        kw = dict(dtype=rows.dtype, device=self.device)
        local = torch.empty((n, po, c, 7, 7), **kw)
        rel = torch.empty((n, po, 10, 6), **kw)
        glob = torch.empty((n, po, 5), **kw)
        capi.check(capi.lib().qqt_local_view(ctypes.byref(self._ccfg), ctypes.byref(self._cstate),
                                             rows.data_ptr(), int(cfg.max_bombs), int(only_p0),
                                             local.data_ptr(), rel.data_ptr(), glob.data_ptr(),
                                             self._stream()), "qqt_local_view")
        return local, rel, glob

    def danger(self) -> torch.Tensor:
        """(N, H, W) float32 danger map computed by the last observe()."""
        return self._danger.view(self.num_envs, self.cfg.height, self.cfg.width)

    def legal_mask(self):
        """(move_mask (N,P,5) bool, bomb_mask (N,P,2) bool) (sim/obs.py:170-229)."""
        capi.check(capi.lib().qqt_legal_mask(ctypes.byref(self._ccfg),
                                             ctypes.byref(self._cstate), self._mm.data_ptr(),
                                             self._bm.data_ptr(), self._stream()),
                   "qqt_legal_mask")
        return self._mm, self._bm

    def _crate_draws(self):
        n, p = self.num_envs, self.cfg.n_players
        if self._rand_buf is not None:
            rb = self._rand_buf
            return (rb[: n * p].view(n, p).contiguous(),
                    rb[n * p: 2 * n * p].view(n, p).contiguous())
        r = torch.rand(n * p * 2, device=self.device).view(p, 2, n)
        return r[:, 0, :].t().contiguous(), r[:, 1, :].t().contiguous()

    def step(self, actions: torch.Tensor, auto_reset: bool = True, crate_draws=None,
             hit_out: torch.Tensor | None = None, next_obs=None,
             reward_out: torch.Tensor | None = None, done_out: torch.Tensor | None = None,
             info_planes: bool = True):
        """One tick (sim/torch_sim.py:895-1261) -> (reward (N,P), done (N,), info).

        With a template installed, done envs reset on the device inside the
        same kernel; otherwise auto_reset resets them on the host generator.
        `crate_draws`: optional (rb_hit, rb_grow) (N,P) float tensors.
        `reward_out` (N,P) float32 / `done_out` (N,) bool: contiguous slots
        (e.g. rollout-buffer rows) written directly instead of the engine's
        own buffers.  info_planes=False skips writing info["blast"] /
        info["trig"] (the flame and exploded-bomb planes).
        `next_obs` = (rows, mm, bm) or (rows, mm, bm, tiles): the same kernel
        also writes the next tick's observation rows (N, obs_stride) fp16 and
        legal masks, and, given `tiles` (N, 4) int32, each row's
        nonzero-K-tile flags for the MLP policy (`B200Policy.act_seats`).
        """
        acts = actions
        if acts.device != self.device or acts.dtype != torch.int64 or not acts.is_contiguous():
            acts = acts.to(self.device, torch.int64).contiguous()
        cout = self._cout
        reward, done = self._reward, self._done
        hit = self._hit
        if reward_out is not None or done_out is not None or hit_out is not None or not info_planes:
            cout = capi.QqtStepOut.from_buffer_copy(self._cout)
            if hit_out is not None:
                if hit_out.dtype != torch.bool or not hit_out.is_contiguous():
                    raise ValueError("hit_out must be a contiguous bool (N, P) slot")
                cout.hit = hit_out.data_ptr()
                hit = hit_out
            if not info_planes:
                cout.covered = None
                cout.triggered = None
            if reward_out is not None:
                cout.reward = reward_out.data_ptr()
                reward = reward_out
            if done_out is not None:
                cout.done = done_out.data_ptr()
                done = done_out
        rb_hit = rb_grow = None
        if self.cfg.map_mode == "corridor":
            rb_hit, rb_grow = crate_draws if crate_draws is not None else self._crate_draws()
            rb_hit = rb_hit.to(self.device, torch.float32).contiguous()
            rb_grow = rb_grow.to(self.device, torch.float32).contiguous()
        dev_reset = auto_reset and (self._tmpl is not None or self._mapgen is not None)
        map_reset = dev_reset and self._tmpl is None
        if self.cfg.hazard_fraction > 0:
            if self.hazard_seed is not None:
                hs = int(self.hazard_seed)
            else:
                self._hazard_calls += 1
                hs = (self._hazard_base ^ (self._hazard_calls * 0xD1B54A32D192ED03)) & ((1 << 64) - 1)
            self._ccfg.hazard_seed_lo = hs & 0xFFFFFFFF
            self._ccfg.hazard_seed_hi = (hs >> 32) & 0xFFFFFFFF
        if next_obs is not None:
            if auto_reset and not dev_reset:
                raise ValueError("next_obs needs the device auto-reset (a template) or no reset")
            rows, nmm, nbm = next_obs[:3]
            tiles = next_obs[3] if len(next_obs) > 3 else None
            if rows.dtype != torch.float16 or rows.stride(1) != 1 or rows.stride(0) != self.obs_stride:
                raise ValueError("next_obs rows must be fp16 with the engine's row stride")
            for m in (nmm, nbm):
                if m.dtype != torch.bool or not m.is_contiguous():
                    raise ValueError("next_obs masks must be contiguous bool tensors")
            if tiles is not None:
                check_tile_flags(tiles, self.num_envs)
            tmpl = ctypes.byref(self._tmpl) if dev_reset and not map_reset else None
            rc = capi.lib().qqt_step_observe(
                ctypes.byref(self._ccfg), ctypes.byref(self._cstate), acts.data_ptr(),
                capi.ptr(rb_hit), capi.ptr(rb_grow), self._tiers.data_ptr(), int(self._first_step),
                ctypes.byref(cout), tmpl, self._step_scratch.data_ptr(), rows.data_ptr(),
                nmm.data_ptr(), nbm.data_ptr(), capi.ptr(tiles), self._stream())
            capi.check(rc, "qqt_step_observe")
            if map_reset:
                self._device_map_reset(done, rows, nmm, nbm, tiles)
        else:
            tmpl = ctypes.byref(self._tmpl) if dev_reset and not map_reset else None
            rc = capi.lib().qqt_step(ctypes.byref(self._ccfg), ctypes.byref(self._cstate),
                                     acts.data_ptr(), capi.ptr(rb_hit), capi.ptr(rb_grow),
                                     self._tiers.data_ptr(), int(self._first_step),
                                     ctypes.byref(cout), tmpl, self._step_scratch.data_ptr(),
                                     self._stream())
            capi.check(rc, "qqt_step")
            if map_reset:
                self._device_map_reset(done)
        self._first_step = False
        n, h, w = self.num_envs, self.cfg.height, self.cfg.width
        info = {"n_alive": self._n_alive, "died": self._died, "winner": self._winner, "hit": hit,
                "blast": self._covered.view(n, h, w),
                "trig": self._triggered.view(n, h, w)}
        if auto_reset and not dev_reset:
            if bool(done.any()):
                info = {k: v.clone() for k, v in info.items()}
                self.reset_(done.clone())
        return reward, done, info

    # --------------------------------------------- CUDA graph of one tick
    def capture_graph(self, actions: torch.Tensor, obs_buf: torch.Tensor,
                      mmask_buf: torch.Tensor, bmask_buf: torch.Tensor,
                      reward_buf: torch.Tensor, done_buf: torch.Tensor,
                      winner_buf: torch.Tensor) -> None:
        """Capture observe -> legal_mask -> step(auto_reset=False) writing
        into fixed buffers as one CUDA graph (BatchedSim.capture_graph,
        sim/torch_sim.py:649-678); `graph_step()` replays it.  The step reads
        `actions` in place and its crate-pickup draws from `_rand_buf`
        (n*(2P+1) floats, the reference's layout), which
        `graph_refill_rand()` refills between replays.  Like the reference,
        three eager warm-up ticks run first (they advance the state)."""
        n, p = self.num_envs, self.cfg.n_players
        self._g = torch.cuda.CUDAGraph()
        self._gbufs = (obs_buf, mmask_buf, bmask_buf, reward_buf, done_buf, winner_buf)
        self._actions = actions
        self._rand_buf = torch.rand(n * (2 * p + 1), device=self.device)
        for _ in range(3):
            self._graph_body()
        torch.cuda.synchronize(self.device)
        with torch.cuda.graph(self._g):
            self._graph_body()
        torch.cuda.synchronize(self.device)

    def _graph_body(self) -> None:
        obs_buf, mmask_buf, bmask_buf, reward_buf, done_buf, winner_buf = self._gbufs
        obs_buf.copy_(self.observe())
        mm, bm = self.legal_mask()
        mmask_buf.copy_(mm)
        bmask_buf.copy_(bm)
        reward, done, info = self.step(self._actions, auto_reset=False)
        reward_buf.copy_(reward)
        done_buf.copy_(done.float())
        winner_buf.copy_(info["winner"].float())

    def graph_step(self) -> None:
        """Replay the captured tick (BatchedSim.graph_step)."""
        self._g.replay()

    def graph_refill_rand(self) -> None:
        """New uniforms for the captured step's draws, outside the graph
        (BatchedSim.graph_refill_rand)."""
        if self._rand_buf is not None:
            self._rand_buf.uniform_()

    def graph_actions(self) -> torch.Tensor:
        """The action buffer the captured step reads (BatchedSim.graph_actions)."""
        return self._actions

    # ------------------------------------------------------------ recycle
    def flush_recycle(self, on_device: bool | None = None, obs_rows: torch.Tensor | None = None,
                      obs_tiles: torch.Tensor | None = None):
        """Drop one crate per lost attribute layer on random free cells
        (sim/torch_sim.py:549-596).

        on_device=False (default without a template): host generator draws in
        the reference's order, bit-compatible with the reference; True
        (default with a template): one kernel, counter-based draws, no host
        round trip.  obs_rows: observation rows (N, obs_stride) of the current
        state (e.g. written by the step's fused observe); their crate channel
        is rewritten from the crate plane, the one channel a recycle changes
        (crates block neither movement nor flames), so they equal a fresh
        observe() afterwards.  obs_tiles: those rows' K-tile flags (N, 4)
        int32 (see `step`'s next_obs); the crate channel's tiles are flagged
        in every row."""
        if on_device is None:
            on_device = self._tmpl is not None or self._mapgen is not None
        if on_device:
            self._flush_count = getattr(self, "_flush_count", 0) + 1
            words = (ctypes.c_uint32 * 14)(*self._excl_words())
            rc = capi.lib().qqt_flush_recycle(ctypes.byref(self._ccfg), ctypes.byref(self._cstate),
                                              words, int(self._flush_seed), self._flush_count,
                                              self._stream())
            capi.check(rc, "qqt_flush_recycle")
        else:
            self._flush_host()
        if obs_rows is not None:
            self._rewrite_crate_channel(obs_rows, obs_tiles)

    def _rewrite_crate_channel(self, rows: torch.Tensor, tiles=None) -> None:
        cfg = self.cfg
        ch, hw = 2 * cfg.n_players + 3, cfg.n_cells
        if cfg.n_channels <= ch:
            return                       # no crate channel in this layout
        rows[:, ch * hw:(ch + 1) * hw].copy_(self._buf["crate"].reshape(self.num_envs, hw))
        if tiles is not None:
            check_tile_flags(tiles, self.num_envs)
            tiles.bitwise_or_(self._crate_tile_words)

    def _flush_host(self) -> None:
        cfg = self.cfg
        lost = self._buf["_pending_lost"]
        if not bool((lost.sum() > 0).item()):
            return
        n, p, hw = self.num_envs, cfg.n_players, cfg.n_cells
        excl = torch.tensor(_recycle_exclusion(cfg), dtype=torch.long)
        lost_cpu = lost.cpu()
        for pl in range(p):
            lp = lost_cpu[pl]
            idx = (lp > 0).nonzero(as_tuple=True)[0]
            if idx.numel() == 0:
                continue
            idx_d = idx.to(self.device)
            avail = (~self._buf["wall"][idx_d] & ~self._buf["brick"][idx_d]).cpu()
            avail[:, excl] = False
            rows, cols = [], []
            for i, e in enumerate(idx.tolist()):
                cells = avail[i].nonzero(as_tuple=True)[0]
                if cells.numel() == 0:
                    continue
                k = min(int(lp[e]), int(cells.numel()))
                pick = cells[torch.randperm(cells.numel(), generator=self.gen)[:k]]
                rows.append(pick)
                cols.append(torch.full_like(pick, e))
            if rows:
                r = torch.cat(rows).to(self.device)
                c = torch.cat(cols).to(self.device)
                self._buf["crate"][c, r] = True
                self._buf["_recycle_crate"][c, r] = True
        lost.zero_()

    def _excl_words(self):
        w = getattr(self, "_excl_cache", None)
        if w is None:
            w = [0] * 14
            for c in _recycle_exclusion(self.cfg):
                w[c >> 5] |= 1 << (c & 31)
            self._excl_cache = w
        return w

    # --------------------------------------------------------- snapshots
    def state_dict(self) -> dict:
        keys = ("wall", "brick", "crate", "fuse", "owner", "bomb_blast", "pos", "alive", "hp",
                "since_bomb", "t")
        return {k: getattr(self, k).clone() for k in keys}

    def load_state_dict(self, snap: dict) -> None:
        for key, val in snap.items():
            getattr(self, key).copy_(val)

    def load_numpy_state(self, st: dict) -> None:
        """Write an env-major numpy state (oracle/golden key names) into the
        device buffers."""
        names = {"recycle": "_recycle_crate", "pending_lost": "_pending_lost",
                 "combo": "_combo", "last_hit": "_last_hit", "lo_bombs": "_lo_bombs",
                 "lo_blast": "_lo_blast", "lo_spd": "_lo_spd", "hazard": "_hazard"}
        for k, v in st.items():
            key = names.get(k, k)
            if key not in self._buf:
                continue
            self._view(key).copy_(torch.as_tensor(np.asarray(v)).to(self.device))

    def numpy_state(self) -> dict:
        names = {"_recycle_crate": "recycle", "_pending_lost": "pending_lost",
                 "_combo": "combo", "_last_hit": "last_hit", "_lo_bombs": "lo_bombs",
                 "_lo_blast": "lo_blast", "_lo_spd": "lo_spd", "_hazard": "hazard"}
        out = {}
        for key in list(_PLANES) + list(_PLAYER) + ["pos", "t", "crate_prob", "_hazard"]:
            out[names.get(key, key)] = self._view(key).cpu().numpy().copy()
        return out


def _make_prop(key):
    def get(self):
        return self._view(key)

    def set_(self, value):
        self._view(key).copy_(torch.as_tensor(value).to(self.device))

    return property(get, set_)


for _k in list(_PLANES) + list(_PLAYER) + ["pos"] + list(_ENV):
    setattr(B200Sim, _k, _make_prop(_k))


def _cell_bits(cells, w: int) -> list[int]:
    words = [0] * capi.MG_WORDS
    for r, c in cells:
        i = r * w + c
        words[i >> 5] |= 1 << (i & 31)
    return words


def _with_neighbours(cells, h: int, w: int):
    out = set()
    for r, c in cells:
        out.add((r, c))
        for dr, dc in mapgen.DIRS4:
            if 0 <= r + dr < h and 0 <= c + dc < w:
                out.add((r + dr, c + dc))
    return sorted(out)


def _make_mapgen(cfg, seed, episode, opp_boost, is_open, map_kind) -> capi.QqtMapGen:
    """The level generator's parameters for qqt_map_reset (sim/config.py
    fields, the reference's reset_ geometry): thresholds as the float32
    values the reference compares against, spawn positions, and the cell
    sets that stay fixed between episodes."""
    g = capi.QqtMapGen()
    h, w, p = cfg.height, cfg.width, cfg.n_players
    g.seed = int(seed) & ((1 << 64) - 1)
    g.episode = episode.data_ptr()
    g.opp_boost = opp_boost.data_ptr()
    g.is_open = is_open.data_ptr()
    g.map_kind = map_kind.data_ptr()
    g.corridor_mode = int(cfg.map_mode == "corridor")
    pf, of, rf = cfg.pure_open_fraction, cfg.open_fraction, cfg.ring_fraction
    g.cut_pure, g.cut_open, g.cut_ring = pf, pf + of, pf + of + rf
    g.obst_max = int(cfg.open_obstacle_max)
    g.random_wall_rows = int(cfg.random_wall_rows)
    g.top_wall_rows = int(cfg.top_wall_rows)
    c0 = (w - cfg.corridor_width) // 2
    c1 = c0 + cfg.corridor_width
    g.corr_c0, g.corr_c1 = c0, c1
    edge = [c for c in (c0, c0 + 1, c1 - 2, c1 - 1) if c0 <= c < c1]
    g.n_edge = len(edge)
    for i, c in enumerate(edge):
        g.edge_cols[i] = c
    g.wall_density = cfg.wall_density
    g.ring_density = cfg.ring_brick_density
    g.hazard_fraction = cfg.hazard_fraction
    r0 = (h - cfg.ring_center_h) // 2
    q0 = (w - cfg.ring_center_w) // 2
    g.ring_r0, g.ring_r1 = r0, r0 + cfg.ring_center_h
    g.ring_c0, g.ring_c1 = q0, q0 + cfg.ring_center_w
    g.open_cross = int(cfg.open_crate_cross)
    starts = [(cfg.growth_bombs_start, cfg.growth_blast_start, cfg.growth_speed_start),
              (cfg.open_growth_bombs, cfg.open_growth_blast, cfg.open_growth_speed),
              (cfg.max_bombs, cfg.blast, 1.0)]
    for i, (b, z, sp) in enumerate(starts):
        g.start_bombs[i], g.start_blast[i], g.start_spd[i] = int(b), int(z), float(sp)
    for i, cp in enumerate((cfg.growth_crate_prob, 1.0, cfg.ring_crate_prob)):
        g.crate_prob_kind[i] = cp
    g.opp_bombs2, g.opp_blast2 = int(cfg.opp_growth_bombs), int(cfg.opp_growth_blast)
    g.opp_spd2, g.opp_mult = cfg.opp_growth_speed, cfg.opp_hist_mult
    g.bombs_max, g.blast_max = int(cfg.growth_bombs_max), int(cfg.growth_blast_max)
    g.spd_max = cfg.growth_speed_max
    for k, pos in enumerate((cfg.spawn_pos(), mapgen.open_spawns(cfg), cfg.ring_spawns())):
        for i in range(p):
            g.spawn[k][i][0], g.spawn[k][i][1] = float(pos[i][0]), float(pos[i][1])
    for name, cells in (("clear_spawn", _with_neighbours(cfg.spawn_cells(), h, w)),
                        ("clear_ring", _with_neighbours(cfg.ring_spawn_cells(), h, w)),
                        ("cross", mapgen.open_cross_cells(cfg))):
        words = _cell_bits(cells, w)
        arr = getattr(g, name)
        for i, v in enumerate(words):
            arr[i] = v
    return g


def _recycle_exclusion(cfg) -> list[int]:
    """Cells that never receive recycled crates: the 4-neighbourhoods of the
    open, mode and ring spawns plus the open cross band (sim/torch_sim.py:508-533)."""
    h, w = cfg.height, cfg.width
    excl = set()
    spawn_sets = [[(int(y), int(x)) for y, x in mapgen.open_spawns(cfg)],
                  list(cfg.spawn_cells()), list(cfg.ring_spawn_cells())]
    for spawns in spawn_sets:
        for r, c in spawns:
            excl.add((r, c))
            for dr, dc in mapgen.DIRS4:
                if 0 <= r + dr < h and 0 <= c + dc < w:
                    excl.add((r + dr, c + dc))
    excl |= set(mapgen.open_cross_cells(cfg))
    return sorted(r * w + c for r, c in excl)
