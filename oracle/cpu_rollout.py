"""The rollout tick on the CPU oracle -- BASELINE AND TEST INFRASTRUCTURE ONLY.

This restates the reference's collection tick (SelfPlayRunner.collect,
train/ppo.py:213-271: observe -> legal masks -> learner act -> opponent act
-> step(auto_reset) -> crate recycling every 16 ticks) on the numpy oracle
in qqt_oracle.py, for a shard of envs of one benchmark configuration.  It
is what bench.py times as the CPU baseline and as its reference arm (the
reference is a Python package that cannot travel to the GPU box; this is
its restatement), and nothing in the product imports it.

`ShardPool` runs one shard per spawned process (so no process inherits GPU
state), each pinned to one BLAS thread.  Every shard first plays a warm-up
of 40 ticks into a bomb-rich mid-game state; each `run(ticks)` then plays
the next ticks of every shard concurrently and reports the env-steps and
the slowest shard's time (process start-up and warm-up excluded).

Random draws come from a seeded numpy stream per shard: the learner's
sampling uniforms, the bot's noise and mode-ticker integers, the crate
pickup uniforms; crate recycling uses the reference's host draw order
(qqt_oracle.flush_recycle) with a seeded torch generator.
"""

from __future__ import annotations

import time

import numpy as np

WARMUP_TICKS = 40

# learner, learner seats, opponent (None = self-play on both seats)
CONFS = {"cfg2": ("mlp", (0,), "astar"), "cfg4": ("mlp", (0, 1), None),
         "cfg5": ("cnn", (0,), "greedy")}


class OracleShard:
    """One shard of n envs of a benchmark configuration on the oracle."""

    def __init__(self, conf: str, n: int, seed: int):
        import torch
        from oracle import qqt_oracle as O
        from qqt_b200 import scenarios
        from qqt_b200.config import SimConfig
        from qqt_b200.policy_init import init_params
        self.O = O
        self.learner, self.seats, self.opponent = CONFS[conf]
        self.cfg = cfg = SimConfig(**scenarios.CFG2)
        self.n, p = n, cfg.n_players
        tm = scenarios.corridor_template(cfg, n, seed)
        self.tmpl = tm
        z = np.zeros_like(tm["wall"])
        self.st = {"wall": tm["wall"].copy(), "brick": tm["brick"].copy(), "crate": z.copy(),
                   "recycle": z.copy(), "fuse": np.zeros(z.shape, np.int16),
                   "owner": np.full(z.shape, -1, np.int8), "bomb_blast": np.zeros(z.shape, np.int16),
                   "pos": tm["spawn"].copy(), "alive": np.ones((n, p), bool),
                   "hp": np.full((n, p), cfg.max_hp, np.uint8),
                   "since_bomb": np.full((n, p), cfg.place_dist_cooldown, np.int32),
                   "t": np.zeros(n, np.int64), "bombs_cap": tm["bombs_cap"].copy(),
                   "blast_cap": tm["blast_cap"].copy(), "spd_g": tm["spd"].copy(),
                   "invuln": np.zeros((n, p), np.int64), "pending_lost": np.zeros((n, p), np.int64),
                   "combo": np.zeros((n, p), np.int64),
                   "last_hit": np.full((n, p), -10 ** 9, np.int64),
                   "lo_bombs": tm["bombs_cap"].copy(), "lo_blast": tm["blast_cap"].copy(),
                   "lo_spd": tm["spd"].copy(), "crate_prob": tm["crate_prob"].copy(),
                   "hazard": np.zeros(n, bool)}
        self.params = {k: v.numpy() if hasattr(v, "numpy") else np.asarray(v)
                       for k, v in init_params(cfg.obs_shape, self.learner, seed=1).items()}
        self.rng = np.random.default_rng(seed)
        self.ticker = O.ModeTicker(self.rng.integers(0, 2, n), self.rng.integers(60, 240, n))
        self.gen = torch.Generator().manual_seed(seed)
        self.tick = 0

    def _learner(self, obs32, mm, bm, pid):
        O, p = self.O, self.cfg.n_players
        u = self.rng.random((self.n, 2))
        if self.learner == "mlp":
            return O.mlp_act(self.params, obs32, mm[:, pid], bm[:, pid], pid, p,
                             u[:, 0], u[:, 1])[0]
        ml, bl, _ = O.cnn_forward(self.params, obs32, pid, p)
        am, _ = O.masked_sample(ml, mm[:, pid], u[:, 0])
        ab, _ = O.masked_sample(bl, bm[:, pid], u[:, 1])
        return np.stack([am, ab], -1)

    def run(self, ticks: int):
        """Play `ticks` ticks; returns (env-steps, seconds)."""
        O, cfg, st, n = self.O, self.cfg, self.st, self.n
        p = cfg.n_players
        dch = 2 * p + 1
        t0 = time.perf_counter()
        for _ in range(ticks):
            obs, _ = O.observe(cfg, st)
            obs32 = obs.astype(np.float16).astype(np.float32)
            mm, bm = O.legal_mask(cfg, st)
            acts = np.zeros((n, p, 2), np.int64)
            for pid in self.seats:
                acts[:, pid] = self._learner(obs32, mm, bm, pid)
            if self.opponent == "astar":
                mode = self.ticker.advance(self.rng.integers(0, 2, n),
                                           self.rng.integers(60, 240, n))
                acts[:, 1] = O.astar_attack(cfg, st, obs32[:, dch], mm[:, 1], bm[:, 1], 1,
                                            self.rng.random((n, 5)).astype(np.float32), mode=mode)
            elif self.opponent == "greedy":
                acts[:, 1] = O.greedy_attack(cfg, st, obs32[:, dch], mm[:, 1], bm[:, 1], 1,
                                             self.rng.random((n, 5)).astype(np.float32))
            rb = self.rng.random((2, n, p)).astype(np.float32)
            _, done, _ = O.step(cfg, st, acts, rb[0], rb[1])
            if done.any():
                O.template_reset(cfg, st, self.tmpl, done)
            self.tick += 1
            if self.tick % 16 == 0:
                O.flush_recycle(cfg, st, self.gen)
        return n * ticks, time.perf_counter() - t0


def _shard_loop(conn, conf, n, seed, warm):
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(1)
    except Exception:
        pass
    import torch
    torch.set_num_threads(1)
    shard = OracleShard(conf, n, seed)
    shard.run(warm)
    conn.send(("ready", 0, 0.0))
    while True:
        msg = conn.recv()
        if msg is None:
            break
        steps, dt = shard.run(int(msg))
        conn.send(("done", steps, dt))
    conn.close()


class ShardPool:
    """`procs` oracle shards of `n_per` envs each, in spawned processes."""

    def __init__(self, conf: str, n_per: int, procs: int, seed: int = 0,
                 warm: int = WARMUP_TICKS, root: str | None = None):
        import multiprocessing as mp
        import os
        import sys
        if root is not None:
            # spawned children import the packages from the repository root
            for pth in (root, os.path.join(root, "qqt-gpu-sim_b200")):
                if pth not in sys.path:
                    sys.path.insert(0, pth)
            os.environ["PYTHONPATH"] = os.pathsep.join(
                [root, os.path.join(root, "qqt-gpu-sim_b200"), os.environ.get("PYTHONPATH", "")])
        ctx = mp.get_context("spawn")
        self.conns, self.procs = [], []
        for i in range(procs):
            a, b = ctx.Pipe()
            pr = ctx.Process(target=_shard_loop, args=(b, conf, n_per, seed + i, warm), daemon=True)
            pr.start()
            self.conns.append(a)
            self.procs.append(pr)
        try:
            for c, pr in zip(self.conns, self.procs):
                tag, _, _ = self._recv(c, pr)
                if tag != "ready":
                    raise RuntimeError(f"oracle shard sent {tag!r} instead of ready")
        except BaseException:
            self.close()
            raise
        self.n = n_per * procs

    @staticmethod
    def _recv(conn, proc, timeout: float = 900.0):
        """The shard's next message; raises instead of waiting for good when
        the process has died or stays silent past `timeout` seconds."""
        import time as _t
        end = _t.monotonic() + timeout
        while not conn.poll(1.0):
            if not proc.is_alive():
                raise RuntimeError(f"oracle shard process exited with code {proc.exitcode}")
            if _t.monotonic() > end:
                raise RuntimeError("oracle shard process did not answer in time")
        return conn.recv()

    def run(self, ticks: int):
        """Every shard plays `ticks` ticks at once; returns (env-steps,
        seconds of the slowest shard)."""
        for c in self.conns:
            c.send(ticks)
        res = [self._recv(c, pr) for c, pr in zip(self.conns, self.procs)]
        return sum(r[1] for r in res), max(r[2] for r in res)

    def close(self):
        for c in self.conns:
            try:
                c.send(None)
            except Exception:
                pass
        for pr in self.procs:
            pr.join(timeout=10)
            if pr.is_alive():
                pr.terminate()
