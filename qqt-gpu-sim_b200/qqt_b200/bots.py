"""Rule bots on the B200 kernels, with the reference's `.act` interface.

`make_bot(sim, kind)` returns an object with `.act(obs, mmask, bmask, pid)
-> (N, 2) int64` and `is_bot = True`, like sim/bots.py:511-562.  Random
draws (samplers, noise, the astar mode ticker) are taken on the device with
torch's generator, or from `feed(...)` for parity runs that replay a
recorded stream.
"""

from __future__ import annotations

import ctypes

import torch

from . import _capi as capi


def _rows(t: torch.Tensor, width: int):
    """(pointer, row stride) of an (N, width) view whose rows are equally spaced."""
    if t.dim() != 2 or t.shape[1] != width or t.stride(1) != 1:
        t = t.reshape(-1, width).contiguous()
    return t, t.data_ptr(), t.stride(0)


def _as_u8(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.uint8) if t.dtype == torch.bool else t.to(torch.uint8)


class _Bot:
    is_bot = True

    def __init__(self, sim, name):
        self.sim = sim
        self.name = name
        self._fed = None

    def feed(self, **draws) -> None:
        """Use these draws (device or host tensors) for the next act() call."""
        self._fed = {k: torch.as_tensor(v).to(self.sim.device) for k, v in draws.items()}

    def _take(self, key, shape, kind="rand", lo=0, hi=1):
        if self._fed is not None and key in self._fed:
            return self._fed[key].to(torch.float32 if kind == "rand" else torch.int64).contiguous()
        if kind == "rand":
            return torch.rand(shape, device=self.sim.device)
        return torch.randint(lo, hi, shape, device=self.sim.device)

    def _io(self, mmask, bmask, out=None):
        mm, mp, ms = _rows(_as_u8(mmask), 5)
        bm, bp, bs = _rows(_as_u8(bmask), 2)
        if out is None:
            out = torch.empty((self.sim.num_envs, 2), dtype=torch.int64, device=self.sim.device)
        elif out.dtype != torch.int64 or out.stride(1) != 1:
            raise ValueError("out must be an int64 (N, 2) view with unit inner stride")
        return (mm, bm), mp, ms, bp, bs, out

    def __repr__(self):
        return f"B200Bot({self.name})"


class RandomBot(_Bot):
    """Uniform legal move + bomb with probability bomb_rate (sim/bots.py:49-58)."""

    def __init__(self, sim, bomb_rate: float = 0.10):
        super().__init__(sim, "random")
        self.bomb_rate = bomb_rate

    def act(self, obs, mmask, bmask, pid: int, out=None):
        n = self.sim.num_envs
        keep, mp, ms, bp, bs, act = self._io(mmask, bmask, out)
        u_move = self._take("u_move", (n,))
        u_bomb = self._take("u_bomb", (n,))
        self._fed = None
        s = self.sim
        rc = capi.lib().qqt_random_act(ctypes.byref(s._ccfg), ctypes.byref(s._cstate), mp, ms,
                                       bp, bs, pid, u_move.data_ptr(), u_bomb.data_ptr(),
                                       float(self.bomb_rate), act.data_ptr(), act.stride(0),
                                       s._stream())
        capi.check(rc, "qqt_random_act")
        return act


class GreedyBot(_Bot):
    """Chebyshev approach with a hard danger filter (sim/bots.py:95-176)."""

    def __init__(self, sim):
        super().__init__(sim, "greedy")

    def act(self, obs, mmask, bmask, pid: int, out=None):
        n = self.sim.num_envs
        keep, mp, ms, bp, bs, act = self._io(mmask, bmask, out)
        noise = self._take("noise", (n, 5))
        self._fed = None
        s = self.sim
        o = _obs_ptr(s, obs)
        rc = capi.lib().qqt_greedy_act(ctypes.byref(s._ccfg), ctypes.byref(s._cstate), o, mp, ms,
                                       bp, bs, pid, noise.data_ptr(), act.data_ptr(),
                                       act.stride(0), s._stream())
        capi.check(rc, "qqt_greedy_act")
        return act


class AstarBot(_Bot):
    """Danger-aware path-field bot with the approach/flee ticker (sim/bots.py:179-508)."""

    def __init__(self, sim, mode: bool = True):
        super().__init__(sim, "astar")
        self.use_mode = mode
        self.mode = None
        self.timer = None
        self.calls = 0
        self._scratch = torch.zeros(64, dtype=torch.uint8, device=sim.device)
        self.vsafe = None
        self.vopp = None
        self.keep_fields = False

    def act(self, obs, mmask, bmask, pid: int, out=None):
        s = self.sim
        n, hw = s.num_envs, s.cfg.n_cells
        keep, mp, ms, bp, bs, act = self._io(mmask, bmask, out)
        mode_p = timer_p = nm_p = nt_p = None
        tick16 = 0
        if self.use_mode:
            if self.mode is None:
                self.mode = self._take("mode0", (n,), "int", 0, 2).clone()
                self.timer = self._take("timer0", (n,), "int", 60, 240).clone()
            self.calls += 1
            tick16 = int(self.calls % 16 == 0)
            mode_p, timer_p = self.mode.data_ptr(), self.timer.data_ptr()
            if tick16:
                nm = self._take("new_mode", (n,), "int", 0, 2)
                nt = self._take("new_timer", (n,), "int", 60, 240)
                nm_p, nt_p = nm.data_ptr(), nt.data_ptr()
        noise = self._take("noise", (n, 5))
        self._fed = None
        if self.keep_fields:
            if self.vsafe is None:
                self.vsafe = torch.empty((n, hw), dtype=torch.float32, device=s.device)
                self.vopp = torch.empty((n, hw), dtype=torch.float32, device=s.device)
            vs, vo = self.vsafe.data_ptr(), self.vopp.data_ptr()
        else:
            vs = vo = None
        o = _obs_ptr(s, obs)
        rc = capi.lib().qqt_astar_act(ctypes.byref(s._ccfg), ctypes.byref(s._cstate), o, mp, ms,
                                      bp, bs, pid, noise.data_ptr(), mode_p, timer_p, tick16,
                                      nm_p, nt_p, act.data_ptr(), act.stride(0), vs, vo,
                                      self._scratch.data_ptr(), s._stream())
        capi.check(rc, "qqt_astar_act")
        return act

    def chain_scan_len(self) -> torch.Tensor:
        """(1,) int32 device view of the last act()'s chain-scan length: the
        maximum over the batch of the seat's blast_cap (sim/bots.py:484),
        which the library reduces into the first word of the bot's scratch
        before the bot kernel reads it."""
        return self._scratch[:4].view(torch.int32)


class HunterBot(_Bot):
    """The hunter: astar with the crate layer and no mode ticker
    (make_bot "hunter", sim/bots.py:557-561; crate layer sim/bots.py:376-431).

    keep_fields=True keeps V_safe, V_opp and V_crate of the last call in
    .vsafe / .vopp / .vcrate."""

    def __init__(self, sim):
        super().__init__(sim, "hunter")
        self._scratch = torch.zeros(64, dtype=torch.uint8, device=sim.device)
        self.vsafe = self.vopp = self.vcrate = None
        self.keep_fields = False

    def act(self, obs, mmask, bmask, pid: int, out=None):
        s = self.sim
        n, hw = s.num_envs, s.cfg.n_cells
        keep, mp, ms, bp, bs, act = self._io(mmask, bmask, out)
        noise = self._take("noise", (n, 5))
        self._fed = None
        vs = vo = vc = None
        if self.keep_fields:
            if self.vsafe is None:
                self.vsafe, self.vopp, self.vcrate = (
                    torch.empty((n, hw), dtype=torch.float32, device=s.device) for _ in range(3))
            vs, vo, vc = self.vsafe.data_ptr(), self.vopp.data_ptr(), self.vcrate.data_ptr()
        o = _obs_ptr(s, obs)
        rc = capi.lib().qqt_hunter_act(ctypes.byref(s._ccfg), ctypes.byref(s._cstate), o, mp, ms,
                                       bp, bs, pid, noise.data_ptr(), act.data_ptr(),
                                       act.stride(0), vs, vo, vc, self._scratch.data_ptr(),
                                       s._stream())
        capi.check(rc, "qqt_hunter_act")
        return act


def _obs_ptr(sim, obs) -> int:
    """Pointer to a row-padded fp16 observation with the engine's stride."""
    if obs.dtype != torch.float16:
        raise ValueError("bots read the fp16 observation")
    if obs.dim() == 4 and obs.stride(0) == sim.obs_stride:
        return obs.data_ptr()
    flat = obs.reshape(obs.shape[0], -1)
    buf = torch.zeros((obs.shape[0], sim.obs_stride), dtype=torch.float16, device=sim.device)
    buf[:, : flat.shape[1]] = flat
    sim._obs_copy = buf
    return buf.data_ptr()


def make_bot(sim, kind: str, mode: bool = True, bomb_rate: float = 0.10):
    """kind in {"random", "greedy", "astar", "hunter", "idle"} (sim/bots.py:538-562)."""
    if kind == "random":
        return RandomBot(sim, bomb_rate)
    if kind == "greedy":
        return GreedyBot(sim)
    if kind == "astar":
        return AstarBot(sim, mode=mode)
    if kind == "hunter":
        return HunterBot(sim)
    if kind == "idle":
        return IdleBot(sim)
    raise ValueError(f"unknown bot kind: {kind}")


class IdleBot(_Bot):
    """Never moves, never bombs (sim/bots.py:61-71)."""

    def __init__(self, sim):
        super().__init__(sim, "idle")

    def act(self, obs, mmask, bmask, pid: int, out=None):
        n = self.sim.num_envs
        if out is None:
            out = torch.zeros((n, 2), dtype=torch.int64, device=self.sim.device)
        out[:, 0] = 4
        out[:, 1] = 0
        return out
