"""Rollout collection on the device: the B200 counterpart of
SelfPlayRunner.collect (train/ppo.py:197-314).

Tick protocol (ppo.py:213-271): observe -> legal masks -> learner act ->
opponent act -> step(auto_reset) -> crate recycling every 16 ticks.  Every
kernel writes straight into its row of a device-resident rollout buffer
(observation rows, masks, actions, log-probs, values, rewards, done flags),
so a tick moves no data besides what the kernels themselves read and write,
and the whole T-tick rollout can be captured into one CUDA graph.  The step
kernel also writes the next tick's observation and masks (qqt_step_observe),
except before a crate recycling, which changes the board after the step:
the tick after it (and the first tick of a rollout) observes on its own.

Random draws for a rollout (learner sampling uniforms, bot noise, the astar
mode-ticker integers, crate-pickup uniforms) are inputs in `RolloutDraws`;
`RolloutDraws.generate` fills them on the device.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .bots import AstarBot, GreedyBot, RandomBot
from .policy import B200Policy


class DeviceRolloutBuffer:
    """(T, N, ...) buffers; obs rows keep the engine's padded stride."""

    def __init__(self, T, n, p, n_seats, obs_stride, obs_shape, device):
        d = torch.device(device)
        self.T, self.n, self.p = T, n, p
        self.obs_shape = obs_shape
        self.obs_rows = torch.zeros((T, n, obs_stride), dtype=torch.float16, device=d)
        # per row, which 64-entry K tiles hold a nonzero (written by the
        # step's fused observation; the MLP policy skips all-zero tiles)
        self.tiles = torch.full((T, n, 4), -1, dtype=torch.int32, device=d)
        self.mm = torch.ones((T, n, p, 5), dtype=torch.bool, device=d)
        self.bm = torch.ones((T, n, p, 2), dtype=torch.bool, device=d)
        self.act = torch.zeros((T, n, p, 2), dtype=torch.int64, device=d)
        self.logp = torch.zeros((T, n_seats, n), dtype=torch.float32, device=d)
        self.val = torch.zeros((T, n_seats, n), dtype=torch.float32, device=d)
        self.rew = torch.zeros((T, n, p), dtype=torch.float32, device=d)
        self.done = torch.zeros((T, n), dtype=torch.bool, device=d)
        self.dmg = torch.zeros((T, n, p), dtype=torch.bool, device=d)   # hp lost, env not ended

    def obs(self, t):
        c, h, w = self.obs_shape
        return self.obs_rows[t, :, : c * h * w].view(self.n, c, h, w)


@dataclass
class RolloutDraws:
    u_net: torch.Tensor        # (T, S, N, 2)
    noise: torch.Tensor        # (T, N, 5)   opponent bot noise / random-bot uniforms
    crate: torch.Tensor        # (T, 2, N, P) crate-pickup uniforms (hit, grow)
    tick_mode: torch.Tensor    # (T // 16 + 1, N) astar ticker new modes
    tick_timer: torch.Tensor   # (T // 16 + 1, N) astar ticker new timers

    @staticmethod
    def empty(T, n, p, n_seats, device):
        d = torch.device(device)
        k = T // 16 + 1
        return RolloutDraws(torch.zeros((T, n_seats, n, 2), device=d),
                            torch.zeros((T, n, 5), device=d),
                            torch.zeros((T, 2, n, p), device=d),
                            torch.zeros((k, n), dtype=torch.int64, device=d),
                            torch.zeros((k, n), dtype=torch.int64, device=d))

    def generate(self, gen: torch.Generator | None = None) -> None:
        for t in (self.u_net, self.noise, self.crate):
            t.uniform_(generator=gen)
        self.tick_mode.random_(0, 2, generator=gen)
        self.tick_timer.random_(60, 240, generator=gen)

    def tensors(self):
        return [self.u_net, self.noise, self.crate, self.tick_mode, self.tick_timer]


class Rollout:
    """T-tick collection of `sim` with a B200Policy learner and an opponent.

    learner: B200Policy whose seats are the learning/network seats (one seat
    vs a bot, or both seats for self-play); opponent: a bot from
    qqt_b200.bots for the remaining seat, or None for self-play.
    """

    def __init__(self, sim, learner: B200Policy, opponent=None, T: int = 128,
                 flush_every: int = 16, slots: int | None = None):
        self.sim, self.learner, self.opponent = sim, learner, opponent
        self.T = T
        self.flush_every = flush_every
        cfg = sim.cfg
        self.p = cfg.n_players
        self.seats = learner.seats
        self.opp_seat = next(i for i in range(self.p) if i not in self.seats) \
            if opponent is not None else None
        # `slots` < T keeps only the last `slots` ticks (a ring), e.g. for
        # profiling large env counts without a full T-tick buffer
        self.slots = slots or T
        self.buf = DeviceRolloutBuffer(self.slots, sim.num_envs, self.p, len(self.seats),
                                       sim.obs_stride, cfg.obs_shape, sim.device)
        # the learner and the opponent both read only this tick's observation
        # and masks: they run as two concurrent branches (the bot on a side
        # stream) that join before the step
        self.side = torch.cuda.Stream(sim.device) if opponent is not None else None
        self.draws = RolloutDraws.empty(T, sim.num_envs, self.p, len(self.seats), sim.device)
        self.graph = None
        # the fused observation writes fp16 rows with the engine's stride
        self.fuse_observe = bool(sim.cfg.obs_fp16) and sim.obs_stride % 8 == 0
        self._ready = -1      # tick whose observation the last step already wrote
        # probe(name, fn) wraps each engine call of a tick (e.g. timing events
        # around it); None runs the calls directly
        self.probe = None
        # cap_log: a (T,) int32 device tensor, or None; when set, every tick
        # also records the astar opponent's chain-scan length (the batch
        # maximum of its seat's blast_cap, sim/bots.py:484) in cap_log[t],
        # so a check of a subset of envs can replay the bot's bomb rule
        self.cap_log = None

    def _run(self, name, fn):
        # an NVTX range per engine call (visible to Nsight Systems in eager
        # ticks and at graph capture; a no-op without a profiler attached)
        torch.cuda.nvtx.range_push("qqt:" + name)
        try:
            return fn() if self.probe is None else self.probe(name, fn)
        finally:
            torch.cuda.nvtx.range_pop()

    def tick(self, t: int) -> None:
        sim, buf, dr = self.sim, self.buf, self.draws
        b = t % self.slots
        tiles = None
        if self._ready == t:
            obs, mm, bm = buf.obs(b), buf.mm[b], buf.bm[b]
            tiles = buf.tiles[b]
        else:
            obs, mm, bm = self._run("observe", lambda: sim.observe_and_mask(
                buf.obs_rows[b], buf.mm[b], buf.bm[b], danger=False))
        acts = buf.act[b]
        main = torch.cuda.current_stream(sim.device)

        def learner():
            self.learner.act_seats(obs, [mm[:, s] for s in self.seats],
                                   [bm[:, s] for s in self.seats], dr.u_net[t],
                                   [acts[:, s] for s in self.seats], buf.logp[b], buf.val[b],
                                   obs_tiles=tiles)
        # the opponent bot runs on the side stream and the learner's policy
        # on the tick's stream right before the step, so the step (launched
        # as the policy's programmatic dependent) can stage its state while
        # the policy finishes
        if self.opponent is not None:
            o = self.opp_seat
            bot = self.opponent
            self.feed_opponent(t)
            self.side.wait_stream(main)
            with torch.cuda.stream(self.side):
                self._run("bot", lambda: bot.act(obs, mm[:, o], bm[:, o], o, out=acts[:, o]))
                if self.cap_log is not None and isinstance(bot, AstarBot):
                    self.cap_log[t:t + 1].copy_(bot.chain_scan_len())
        self._run("policy", learner)
        if self.opponent is not None:
            main.wait_stream(self.side)
        flush = bool(self.flush_every) and t % self.flush_every == self.flush_every - 1
        nxt = None
        if self.fuse_observe and t + 1 < self.T:
            # after a crate recycle only the crate channel of the next rows
            # changes; flush_recycle rewrites it (no stand-alone observe)
            b1 = (t + 1) % self.slots
            nxt = (buf.obs_rows[b1], buf.mm[b1], buf.bm[b1], buf.tiles[b1])
        self._run("step+observe" if nxt is not None else "step", lambda: sim.step(
            acts, auto_reset=True, crate_draws=(dr.crate[t, 0], dr.crate[t, 1]),
            reward_out=buf.rew[b], done_out=buf.done[b], hit_out=buf.dmg[b],
            info_planes=False, next_obs=nxt))
        self._ready = t + 1 if nxt is not None else -1
        if flush:
            self._run("flush", lambda: sim.flush_recycle(
                obs_rows=nxt[0] if nxt is not None else None,
                obs_tiles=nxt[3] if nxt is not None else None))

    def feed_opponent(self, t: int) -> None:
        """Hand the opponent bot its draws for tick t (noise; the astar mode
        ticker's new modes/timers every 16th call)."""
        bot, dr = self.opponent, self.draws
        if isinstance(bot, AstarBot):
            feed = {"noise": dr.noise[t]}
            if bot.use_mode and (bot.calls + 1) % 16 == 0:
                k = (bot.calls + 1) // 16
                feed["new_mode"] = dr.tick_mode[k % dr.tick_mode.shape[0]]
                feed["new_timer"] = dr.tick_timer[k % dr.tick_timer.shape[0]]
            bot.feed(**feed)
        elif isinstance(bot, GreedyBot):
            bot.feed(noise=dr.noise[t])
        elif isinstance(bot, RandomBot):
            bot.feed(u_move=dr.noise[t, :, 0], u_bomb=dr.noise[t, :, 1])

    def collect(self) -> DeviceRolloutBuffer:
        """Run T ticks eagerly (kernel launches only; no host synchronisation
        when the sim resets on the device)."""
        for t in range(self.T):
            self.tick(t)
        return self.buf

    def capture(self) -> None:
        """Capture one full T-tick rollout into a CUDA graph (call after at
        least one eager tick so first-step set-up is done)."""
        if isinstance(self.opponent, AstarBot) and self.opponent.mode is None:
            raise RuntimeError("run one eager tick before capture (ticker init)")
        s = torch.cuda.Stream(self.sim.device)
        s.wait_stream(torch.cuda.current_stream(self.sim.device))
        g = torch.cuda.CUDAGraph()
        calls0 = self.opponent.calls if isinstance(self.opponent, AstarBot) else 0
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self.collect()
        torch.cuda.current_stream(self.sim.device).wait_stream(s)
        if isinstance(self.opponent, AstarBot):
            self.opponent.calls = calls0   # capture did not run the ticks
        self.graph = g

    def replay(self) -> DeviceRolloutBuffer:
        """Replay the captured rollout (T ticks)."""
        self.graph.replay()
        if isinstance(self.opponent, AstarBot):
            self.opponent.calls += self.T
        return self.buf


class RolloutGroups:
    """Several independent env groups (one `Rollout` each, with its own sim
    state, bot and draws) ticked on their own streams, so one group's
    simulation kernels overlap another group's policy and bot kernels; the
    whole T-tick rollout of every group is still one CUDA graph.

    `Rollout.tick` has no cross-group dependency: each group's kernels are
    ordered only by its own stream (plus its bot side stream)."""

    def __init__(self, rollouts):
        self.ros = list(rollouts)
        dev = self.ros[0].sim.device
        self.device = dev
        self.T = self.ros[0].T
        self.streams = [torch.cuda.Stream(dev) for _ in self.ros]
        self.graph = None

    @property
    def num_envs(self) -> int:
        return sum(r.sim.num_envs for r in self.ros)

    def collect(self):
        main = torch.cuda.current_stream(self.device)
        for s in self.streams:
            s.wait_stream(main)
        for t in range(self.T):
            for ro, s in zip(self.ros, self.streams):
                with torch.cuda.stream(s):
                    ro.tick(t)
        for s in self.streams:
            main.wait_stream(s)
        return [r.buf for r in self.ros]

    def _capture_one(self):
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        g = torch.cuda.CUDAGraph()
        calls0 = [r.opponent.calls if isinstance(r.opponent, AstarBot) else 0 for r in self.ros]
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self.collect()
        torch.cuda.current_stream(self.device).wait_stream(s)
        for r, c in zip(self.ros, calls0):
            if isinstance(r.opponent, AstarBot):
                r.opponent.calls = c
        return g

    def capture(self, double_buffer: bool = False) -> None:
        """Capture the T-tick rollout of every group as one CUDA graph.

        double_buffer: also capture a second graph that reads a second set of
        draw buffers (`draw_sets[1]`), so a caller can copy the next
        rollout's host-fed draws into one set while the graph of the other
        runs (`replay(which)`)."""
        for ro in self.ros:
            if isinstance(ro.opponent, AstarBot) and ro.opponent.mode is None:
                raise RuntimeError("run one eager tick before capture (ticker init)")
        first = [ro.draws for ro in self.ros]
        self.graphs = [self._capture_one()]
        self.draw_sets = [first]
        if double_buffer:
            second = []
            for ro in self.ros:
                d = ro.draws
                ro.draws = RolloutDraws(*(torch.empty_like(t) for t in d.tensors()))
                for a, b in zip(ro.draws.tensors(), d.tensors()):
                    a.copy_(b)
                second.append(ro.draws)
            self.graphs.append(self._capture_one())
            self.draw_sets.append(second)
            for ro, d in zip(self.ros, first):
                ro.draws = d
        self.graph = self.graphs[0]

    def replay(self, which: int = 0):
        """Replay the captured rollout; `which` picks the draw-buffer set
        (double-buffered capture)."""
        self.graphs[which].replay()
        for r in self.ros:
            if isinstance(r.opponent, AstarBot):
                r.opponent.calls += r.T
        return [r.buf for r in self.ros]
