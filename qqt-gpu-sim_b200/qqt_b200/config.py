"""Game constants, observation layout and the frozen level configuration.

Field names, defaults and validation follow the reference's `SimConfig`
(sim/config.py:102-603) so a reference config object ports unchanged; the
channel layout and the per-seat view permutation follow sim/config.py:69-99.

Observation layout (one shared tensor per env, (N, C, H, W), C = 5P+4):
    0 .. P-1        player i position, bilinear splat of mass 1
    P .. 2P-1       fuse/FUSE of player i's live bombs
    2P              wall | brick
    2P+1            danger map
    2P+2            t / max_steps
    2P+3            crate
    2P+4 .. 3P+3    invulnerability flag at player i's centre cell
    3P+4 .. 4P+3    available bombs / cap at player i's centre cell
    4P+4 .. 5P+3    cap / growth_bombs_max at player i's centre cell
"""

from __future__ import annotations

from dataclasses import dataclass

MOVE_UP, MOVE_DOWN, MOVE_LEFT, MOVE_RIGHT, MOVE_IDLE = 0, 1, 2, 3, 4
N_MOVES = 5
N_BOMB = 2
# (dy, dx) per move action; MOVE_IDLE has no displacement.
DIRS = ((-1.0, 0.0), (1.0, 0.0), (0.0, -1.0), (0.0, 1.0))

# Compile-time limits of the CUDA kernels (cells per env and seats per env).
KERNEL_LIMITS = {"max_h": 21, "max_w": 21, "max_players": 4}
CUDA_LIMITS = KERNEL_LIMITS


def obs_extra(n_players: int) -> int:
    """World-information tail channels: crate + 3 per-player planes."""
    return 1 + 3 * n_players


def n_obs_channels(n_players: int) -> int:
    return 2 * n_players + 3 + obs_extra(n_players)


def view_perm(me: int, n_players: int, c: int | None = None) -> tuple[int, ...]:
    """View channel j reads stored channel view_perm(me)[j].

    Own position and fuse come first, then the opponents in ascending id,
    then wall/danger/progress; the world tail is left in place
    (sim/config.py:77-94).
    """
    p = n_players
    base = 2 * p + 3
    if c is None:
        c = base + obs_extra(p)
    opp = [i for i in range(p) if i != me]
    head = [me, p + me] + opp + [p + i for i in opp]
    return tuple(head + [2 * p, 2 * p + 1, 2 * p + 2] + list(range(base, c)))


@dataclass(frozen=True)
class SimConfig:
    height: int = 13
    width: int = 13
    n_players: int = 2
    tick_hz: int = 10
    speed: float = 3.6
    radius: float = 0.3
    max_steps: int = 600
    fuse: int = 30
    blast: int = 2
    max_bombs: int = 10
    max_chain: int = 16
    chain_cap_rounds: int = 8
    step_penalty: float = 0.001
    wall_density: float = 0.0
    map_mode: str = "open"
    corridor_width: int = 5
    top_wall_rows: int = 4
    random_wall_rows: bool = True
    open_obstacle_max: int = 0
    growth_crate_prob: float = 0.50
    brick_reward: float = 0.15
    growth_bombs_start: int = 2
    growth_blast_start: int = 2
    growth_speed_start: float = 1.0
    growth_bombs_max: int = 10
    growth_blast_max: int = 7
    growth_speed_max: float = 2.1
    growth_speed_step: float = 0.15
    open_fraction: float = 0.0
    open_growth_bombs: int = 3
    open_growth_blast: int = 3
    open_growth_speed: float = 0.84
    open_crate_cross: bool = True
    hit_attr_penalty: int = 2
    opp_boost: bool = False
    opp_hist_mult: float = 1.3
    opp_growth_bombs: int = 6
    opp_growth_blast: int = 6
    opp_growth_speed: float = 1.68
    recycle_crate_prob: float = 1.0
    ring_fraction: float = 0.0
    pure_open_fraction: float = 0.0
    ring_center_h: int = 7
    ring_center_w: int = 7
    ring_brick_density: float = 0.4
    ring_crate_prob: float = 1.0
    hazard_fraction: float = 0.0
    hazard_wave_ticks: int = 50
    hazard_bombs_min: int = 4
    hazard_bombs_max: int = 30
    hazard_blast_min: int = 4
    hazard_blast_max: int = 8
    hazard_ramp_seconds: float = 60.0
    crate_speed_only: bool = False
    place_cover_reward: float = 0.05
    place_chain_reward: float = 0.20
    chain_time_factor: float = 0.15
    place_dist_reward: float = 0.0
    place_dist_radius: float = 4.0
    place_dist_cooldown: int = 15
    chain_blast_bonus: float = 0.0
    suicide_penalty: float = 0.0
    combo_reward: float = 0.10
    combo_gap_factor: float = 0.9
    approach_reward: float = 0.0
    approach_dist: float = 5.0
    approach_gate: float = 3.0
    chase_reward: float = 0.0
    chase_adj: float = 0.05
    invuln_ticks: int = 30
    max_hp: int = 5
    timeout_draw: bool = True
    hit_reward: float = 1.5
    win_bonus: float = 10.0
    win_hp_scaled: bool = False
    danger_penalty: float = 0.015
    passivity_ticks: int = 20
    passivity_penalty: float = 0.0
    obs_extra_enabled: bool = True
    obs_fp16: bool = True

    def __post_init__(self) -> None:
        lim = KERNEL_LIMITS
        if not 2 <= self.n_players <= lim["max_players"]:
            raise ValueError(f"n_players must be in 2..{lim['max_players']}")
        if self.height > lim["max_h"] or self.width > lim["max_w"]:
            raise ValueError("map larger than the kernels' compile-time limit")
        if self.height < 5 or self.width < 5:
            raise ValueError("map must be at least 5x5")
        if self.map_mode not in ("open", "corridor"):
            raise ValueError(f"map_mode must be open/corridor, got {self.map_mode}")
        if self.map_mode == "corridor":
            if not 3 <= self.corridor_width <= self.width - 2:
                raise ValueError("corridor_width must be in [3, width-2]")
            if self.corridor_width < 2 * self.n_players - 1:
                raise ValueError("corridor_width too small for the spawns")
            if not 1 <= self.top_wall_rows <= self.height - 3:
                raise ValueError("top_wall_rows must be in [1, height-3]")
            total = self.pure_open_fraction + self.open_fraction + self.ring_fraction
            if not 0.0 <= total <= 1.0:
                raise ValueError("map fractions must sum to at most 1")
        if not 0.0 < self.radius < 0.5:
            raise ValueError("radius must be in (0, 0.5)")
        if self.step_len >= 2.0:
            raise ValueError("per-tick displacement too large")
        if self.map_mode == "corridor" and \
                self.step_len * self.growth_speed_max >= 2.0:
            raise ValueError("grown per-tick displacement too large")
        if self.place_dist_radius <= 0:
            raise ValueError("place_dist_radius must be positive")
        if not 0 <= self.place_dist_cooldown < self.passivity_ticks:
            raise ValueError("place_dist_cooldown must be in [0, passivity_ticks)")
        if not 1 <= self.hazard_bombs_min <= self.hazard_bombs_max:
            raise ValueError("hazard bomb counts out of order")
        if not 1 <= self.hazard_blast_min <= self.hazard_blast_max:
            raise ValueError("hazard blast range out of order")

    @property
    def step_len(self) -> float:
        return self.speed / self.tick_hz

    @property
    def n_cells(self) -> int:
        return self.height * self.width

    @property
    def n_channels(self) -> int:
        base = 2 * self.n_players + 3
        return base + (obs_extra(self.n_players) if self.obs_extra_enabled else 0)

    @property
    def obs_shape(self) -> tuple[int, int, int]:
        return (self.n_channels, self.height, self.width)

    def view_perm(self, me: int) -> tuple[int, ...]:
        return view_perm(me, self.n_players)

    @property
    def game_seconds(self) -> float:
        return self.max_steps / self.tick_hz

    def spawn_pos(self) -> list[tuple[float, float]]:
        """Spawn centres (sim/config.py:561-584)."""
        h, w = float(self.height), float(self.width)
        if self.map_mode == "corridor":
            row = (self.top_wall_rows + (self.height - 1)) / 2.0 + 0.5
            c0 = (w - self.corridor_width) / 2.0 + 0.5
            step = (self.corridor_width - 2) / max(1, self.n_players - 1)
            return [(row, c0 + 1.0 + i * step) for i in range(self.n_players)]
        row = (h - 1) / 2.0 + 0.5
        return [(row, (w - 1) * (i + 1) / (self.n_players + 1) + 0.5)
                for i in range(self.n_players)]

    def spawn_cells(self) -> list[tuple[int, int]]:
        return [(int(y), int(x)) for y, x in self.spawn_pos()]

    def ring_spawns(self) -> list[tuple[float, float]]:
        h, w = float(self.height), float(self.width)
        corners = [(1.5, 1.5), (1.5, w - 0.5), (h - 0.5, w - 0.5), (h - 0.5, 1.5)]
        return corners[: self.n_players]

    def ring_spawn_cells(self) -> list[tuple[int, int]]:
        return [(int(y), int(x)) for y, x in self.ring_spawns()]
