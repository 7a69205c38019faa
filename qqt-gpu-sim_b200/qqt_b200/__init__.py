"""B200-native rollout engine for the batched Bomberman environment.

Public API mirrors the reference package layout:
  make_sim(cfg, num_envs, backend="b200")   -> B200Sim (BatchedSim API)
  bots.make_bot(sim, kind)                  -> bot with .act(obs, mm, bm, pid)
  policy.B200Policy(state_dict, ...)        -> ActorCritic(mlp) forward/act
"""

from .config import (DIRS, MOVE_DOWN, MOVE_IDLE, MOVE_LEFT, MOVE_RIGHT, MOVE_UP, N_BOMB,
                     N_MOVES, SimConfig, n_obs_channels, obs_extra, view_perm)


def make_sim(cfg, num_envs, backend="b200", device=None, seed=0, template=None,
             map_reset="host"):
    """Backend factory (sim/factory.py:11-36) with the B200 engine as "b200".

    "auto" picks "b200" when a CUDA device is present; there is no CPU
    fallback inside this package.  map_reset: "host" (levels from the host
    generator in the reference's draw order) or "device" (levels built on
    the GPU from counter-based draws; resets never leave the device).
    """
    from .sim import B200Sim
    if backend in ("auto", "b200", "cuda"):
        return B200Sim(cfg, num_envs, device=device or "cuda", seed=seed, template=template,
                       map_reset=map_reset)
    raise ValueError(f"unknown backend: {backend}")


__all__ = ["SimConfig", "make_sim", "view_perm", "n_obs_channels", "obs_extra", "N_MOVES",
           "N_BOMB", "MOVE_UP", "MOVE_DOWN", "MOVE_LEFT", "MOVE_RIGHT", "MOVE_IDLE", "DIRS"]
