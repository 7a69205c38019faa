"""PPO update for the MLP actor-critic (train/ppo.py:37-51, 101-110, 364-437),
with data-parallel gradient averaging over NCCL.

The rollout side runs on the B200 kernels (qqt_b200.rollout); this module is
the update step: GAE on the device (`qqt_gae` kernel), global advantage
normalisation, the reference's oversampling of damage / terminal frames,
clipped policy and value losses with an entropy bonus, a gradient all-reduce
across ranks (`torch.distributed`, NCCL on GPUs, gloo on CPU), gradient-norm
clipping and Adam.  The network is a torch restatement of ActorCritic(mlp)
with the reference's parameter names, so its parameters feed B200Policy's
packed weights directly (`B200Policy.repack()` after each update).
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from .config import view_perm


@dataclass
class PPOConfig:
    rollout_steps: int = 128
    epochs: int = 4
    minibatches: int = 4
    gamma: float = 0.995
    gae_lambda: float = 0.95
    clip_eps: float = 0.2
    value_coef: float = 0.5
    entropy_coef: float = 0.05
    entropy_final: float = 0.03
    max_grad_norm: float = 0.5
    lr: float = 3e-4
    oversample_dying: int = 3


def inv_cols(n_players: int, c: int, h: int, w: int, pid: int) -> torch.Tensor:
    """Column gather folding seat `pid`'s view permutation into W0
    (train/model.py:127-138): column block k of the gathered weight is
    block argsort(perm)[k] of W0."""
    perm = np.asarray(view_perm(pid, n_players, c))
    inv = np.argsort(perm)
    hw = h * w
    return torch.from_numpy(np.concatenate([np.arange(hw) + int(inv[k]) * hw for k in range(c)]))


class MLPActorCritic(nn.Module):
    """ActorCritic(arch="mlp") for training (same parameter names)."""

    def __init__(self, obs_shape, n_players: int = 2, n_moves: int = 5, n_bomb: int = 2):
        super().__init__()
        c, h, w = obs_shape
        self.obs_shape = tuple(obs_shape)
        self.k_in = c * h * w
        self.n_players = n_players
        self.shared = nn.Sequential(nn.Linear(c * h * w, 128), nn.LayerNorm(128), nn.ReLU(),
                                    nn.Linear(128, 128), nn.LayerNorm(128), nn.ReLU())
        self.move_head = nn.Sequential(nn.Linear(128, 64), nn.ReLU(), nn.Linear(64, n_moves))
        self.bomb_head = nn.Sequential(nn.Linear(128, 64), nn.ReLU(), nn.Linear(64, n_bomb))
        self.critic = nn.Sequential(nn.Linear(128, 64), nn.ReLU(), nn.Linear(64, 1))
        for pid in range(n_players):
            self.register_buffer(f"inv_cols_{pid}", inv_cols(n_players, c, h, w, pid),
                                 persistent=False)

    def forward(self, obs: torch.Tensor, pid: int = 0):
        n = obs.shape[0]
        # (N, C, H, W) or the engine's row-padded (N, stride >= C*H*W) rows
        x = obs.reshape(n, -1)[:, : self.k_in].to(self.shared[0].weight.dtype)
        w0 = self.shared[0].weight[:, getattr(self, f"inv_cols_{pid}")]
        x = F.linear(x, w0, self.shared[0].bias)
        x = self.shared[1:](x)
        return self.move_head(x), self.bomb_head(x), self.critic(x).squeeze(-1)

    @staticmethod
    def _masked(logits, mask):
        z = torch.where(mask, logits, torch.full_like(logits, torch.finfo(logits.dtype).min))
        logz = z - torch.logsumexp(z, -1, keepdim=True)
        return logz

    def evaluate(self, obs, mm, bm, actions, pid: int = 0):
        """(log-prob of `actions`, entropy, value) under the masked heads
        (train/model.py:247-256)."""
        ml, bl, v = self(obs, pid)
        lm = self._masked(ml, mm)
        lb = self._masked(bl, bm)
        logp = lm.gather(-1, actions[..., :1]).squeeze(-1) + lb.gather(-1, actions[..., 1:]).squeeze(-1)
        low = torch.finfo(lm.dtype).min
        ent = -(lm.clamp(min=low) * lm.exp()).sum(-1) - (lb.clamp(min=low) * lb.exp()).sum(-1)
        return logp, ent, v


def gae(rew, done, val, last_val, gamma, lam):
    """(adv, ret) (T, N) with the device kernel (CUDA tensors) or the same
    recurrence on the host (CPU tensors)."""
    T, n = done.shape
    if rew.is_cuda:
        from . import _capi as capi
        adv = torch.empty((T, n), dtype=torch.float32, device=rew.device)
        ret = torch.empty_like(adv)
        d8 = done.to(torch.uint8).contiguous()
        rc = capi.lib().qqt_gae(rew.data_ptr(), rew.stride(0), d8.data_ptr(), val.data_ptr(),
                                val.stride(0), last_val.contiguous().data_ptr(), T, n,
                                ctypes.c_double(gamma), ctypes.c_double(lam), adv.data_ptr(),
                                ret.data_ptr(), capi.stream_ptr(rew.device))
        capi.check(rc, "qqt_gae")
        return adv, ret
    adv = torch.zeros((T, n), dtype=torch.float32)
    g = torch.zeros(n, dtype=torch.float32)
    for t in reversed(range(T)):
        nonterm = 1.0 - done[t].float()
        nv = last_val if t == T - 1 else val[t + 1]
        delta = rew[t] + gamma * nv * nonterm - val[t]
        g = delta + gamma * lam * nonterm * g
        adv[t] = g
    return adv, adv + val


def _all_reduce(t, op=None):
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=op or dist.ReduceOp.SUM)
        return dist.get_world_size()
    return 1


def ppo_update(model: MLPActorCritic, opt, data: dict, last_val, cfg: PPOConfig,
               entropy_coef: float, pid: int = 0, perm_fn=None) -> dict:
    """One PPO update over a (T, N) rollout shard (train/ppo.py:364-437).

    data: obs (T,N,C,H,W) fp16 (or row-padded view), mm (T,N,5), bm (T,N,2),
    act (T,N,2), logp/val/rew (T,N), done (T,N) bool, dmg (T,N) bool.
    Advantage statistics and gradients are reduced over all ranks of the
    default process group when one is initialised.  perm_fn(n) -> index
    permutation (defaults to torch.randperm on the data's device).
    """
    dev = data["rew"].device
    adv, ret = gae(data["rew"], data["done"], data["val"], last_val, cfg.gamma, cfg.gae_lambda)
    T, n = adv.shape
    total = T * n
    flat = lambda x: x.reshape(total, *x.shape[2:])  # noqa: E731
    obs = flat(data["obs"])
    mm, bm, act = flat(data["mm"]), flat(data["bm"]), flat(data["act"])
    old_logp, old_val = flat(data["logp"]), flat(data["val"])
    adv, ret = flat(adv), flat(ret)
    # global mean / unbiased std of the advantages over every rank's shard
    stats = torch.stack([adv.sum(), (adv * adv).sum(),
                         torch.tensor(float(total), device=dev)]).to(torch.float64)
    world = _all_reduce(stats)
    cnt = stats[2]
    mean = stats[0] / cnt
    var = (stats[1] - cnt * mean * mean) / (cnt - 1)
    std = math.sqrt(max(float(var), 0.0)) if world > 1 else float(adv.std())
    adv = (adv - (mean.float() if world > 1 else adv.mean())) / (std + 1e-8)

    base = torch.arange(total, device=dev)
    over = cfg.oversample_dying
    pool = base
    if over > 1:
        rare = flat(data["dmg"]) | flat(data["done"]).bool()
        if bool(rare.any()):
            rare_idx = rare.nonzero(as_tuple=False).squeeze(1)
            pool = torch.cat([base, rare_idx.repeat(over - 1)])
    mb = max(1, total // cfg.minibatches)
    perm_fn = perm_fn or (lambda k: torch.randperm(k, device=dev))
    # statistics stay on the device; one host read at the end
    out = {k: torch.zeros((), device=dev) for k in ("pg", "vf", "ent", "kl", "clipfrac")}
    updates = 0
    params = [p for p in model.parameters()]
    for _ in range(cfg.epochs):
        perm = pool[perm_fn(pool.numel())][:total]
        for start in range(0, total, mb):
            sel = perm[start:start + mb]
            logp, ent, value = model.evaluate(obs[sel], mm[sel], bm[sel], act[sel], pid)
            ratio = (logp - old_logp[sel]).exp()
            a = adv[sel]
            pg = -torch.min(ratio * a, ratio.clamp(1 - cfg.clip_eps, 1 + cfg.clip_eps) * a).mean()
            v_clip = old_val[sel] + (value - old_val[sel]).clamp(-cfg.clip_eps, cfg.clip_eps)
            vf = 0.5 * torch.max((value - ret[sel]) ** 2, (v_clip - ret[sel]) ** 2).mean()
            ent_m = ent.mean()
            loss = pg + cfg.value_coef * vf - entropy_coef * ent_m
            opt.zero_grad(set_to_none=True)
            loss.backward()
            grads = [p.grad for p in params if p.grad is not None]
            if grads:
                buf = torch.cat([g.reshape(-1) for g in grads])
                w = _all_reduce(buf)
                if w > 1:
                    buf /= w
                    off = 0
                    for g in grads:
                        g.copy_(buf[off:off + g.numel()].view_as(g))
                        off += g.numel()
            torch.nn.utils.clip_grad_norm_(params, cfg.max_grad_norm)
            opt.step()
            with torch.no_grad():
                out["pg"] += pg.detach()
                out["vf"] += vf.detach()
                out["ent"] += ent_m.detach()
                out["kl"] += (old_logp[sel] - logp).mean().detach()
                out["clipfrac"] += ((ratio - 1).abs() > cfg.clip_eps).float().mean()
            updates += 1
    return {k: float(v) / max(1, updates) for k, v in out.items()}
