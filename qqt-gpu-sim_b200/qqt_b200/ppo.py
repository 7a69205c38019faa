"""PPO update for the MLP actor-critic (train/ppo.py:37-51, 101-110, 364-437),
with data-parallel gradient averaging over NCCL.

The rollout side runs on the B200 kernels (qqt_b200.rollout); this module is
the update step: GAE on the device (`qqt_gae` kernel), global advantage
normalisation, the reference's oversampling of damage / terminal frames,
clipped policy and value losses with an entropy bonus, a gradient all-reduce
across ranks (`torch.distributed`, NCCL on GPUs, gloo on CPU), gradient-norm
clipping and Adam.  The network is ActorCritic(mlp) with the reference's
parameter names, so its parameters feed B200Policy's packed weights directly
(`B200Policy.repack()` after each update).

On the GPU every minibatch runs on the kernels of csrc/train_mlp.cu from the
rollout's float16 observation rows: the minibatch's rows are gathered by a
kernel (the reference's `obs[sel]`); `evaluate` is one fused tcgen05 forward
(all four layers, the masked log-softmax of both heads, entropy and value,
keeping the two pre-LayerNorm activations); the PPO loss over the per-row
(logp, entropy, value) stays in torch autograd; its gradients go back
through two persistent tcgen05 kernels (heads + LN2, trunk + LN1) and the
first layer's weight-gradient GEMM.  Products carry float32 accuracy
through fp16 hi/lo operand splits.  CPU tensors (the gloo tests) take the
torch restatement of the same network.
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


def _aligned(buf: torch.Tensor, align: int) -> int:
    base = buf.data_ptr()
    return base + (-base) % align


def obs_rows(obs: torch.Tensor, k_in: int) -> torch.Tensor:
    """2-D float16 observation rows the kernels read: (n, stride) with stride
    >= k_in a multiple of 8 and 16-byte aligned rows.  The rollout buffer's
    row-padded observations qualify as they are; anything else (an (n, C, H,
    W) float16 batch) is copied once into zero-padded rows."""
    n = obs.shape[0]
    if obs.dtype != torch.float16:
        raise TypeError(f"observations must be float16 (the rollout's storage), got {obs.dtype}")
    if (obs.dim() == 2 and obs.stride(1) == 1 and obs.shape[1] >= k_in and obs.stride(0) % 8 == 0
            and obs.data_ptr() % 16 == 0):
        return obs
    flat = obs.reshape(n, -1)[:, :k_in]
    rows = torch.zeros((n, (k_in + 7) // 8 * 8), dtype=torch.float16, device=obs.device)
    rows[:, :k_in] = flat
    return rows


def gather_rows(rows: torch.Tensor, idx: torch.Tensor, out: torch.Tensor | None = None):
    """out[i] = rows[idx[i]] on the device (`qqt_gather_rows`); rows as
    obs_rows returns them, idx int64 on the same device."""
    from . import _capi as capi
    n = idx.numel()
    if out is None:
        out = torch.empty((n, rows.shape[1]), dtype=rows.dtype, device=rows.device)
    idx = idx.to(torch.int64).contiguous()
    rb = rows.shape[1] * rows.element_size()
    rb16 = (rb + 15) // 16 * 16
    if rb16 > rows.stride(0) * rows.element_size():
        raise ValueError("rows must be padded to a 16-byte multiple")
    capi.check(capi.lib().qqt_gather_rows(rows.data_ptr(), rows.shape[0],
                                          rows.stride(0) * rows.element_size(), idx.data_ptr(),
                                          n, out.data_ptr(), out.stride(0) * out.element_size(),
                                          rb16, capi.stream_ptr(rows.device)),
               "qqt_gather_rows")
    return out


class _Layer1(torch.autograd.Function):
    """Linear(k_in -> 128) with seat pid's view permutation folded into W0's
    column order (train/model.py:127-138, 149-150) on the B200 kernels.
    Forward: h1 = x W0p^T + b0 (qqt_l1_forward); backward: dW0
    (qqt_l1_wgrad, in W0's own column order) and db0 = sum of dL/dh1.  The
    observations are data, so no input gradient is formed."""

    @staticmethod
    def forward(ctx, rows, w0, b0, k_in, geom):
        from . import _capi as capi
        n_players, channels, hw, pid = geom
        L, dev = capi.lib(), rows.device
        st = capi.stream_ptr(dev)
        w0c, b0c = w0.detach().contiguous(), b0.detach().contiguous()
        pack = torch.empty(int(L.qqt_l1_pack_bytes(k_in)) + 256, dtype=torch.uint8, device=dev)
        pk = _aligned(pack, 256)
        capi.check(L.qqt_l1_pack(w0c.data_ptr(), k_in, n_players, channels, hw, pid, pk, st),
                   "qqt_l1_pack")
        n = rows.shape[0]
        h1 = torch.empty((n, w0.shape[0]), dtype=torch.float32, device=dev)
        capi.check(L.qqt_l1_forward(pk, rows.data_ptr(), n, rows.stride(0), k_in,
                                    b0c.data_ptr(), h1.data_ptr(), st), "qqt_l1_forward")
        ctx.save_for_backward(rows)
        ctx.k_in, ctx.geom = k_in, geom
        return h1

    @staticmethod
    def backward(ctx, dh1):
        from . import _capi as capi
        (rows,) = ctx.saved_tensors
        n_players, channels, hw, pid = ctx.geom
        L, dev = capi.lib(), rows.device
        dh1 = dh1.contiguous()
        n = rows.shape[0]
        dw0 = torch.empty((dh1.shape[1], ctx.k_in), dtype=torch.float32, device=dev)
        work = torch.empty(int(L.qqt_l1_wgrad_work_bytes(n, ctx.k_in)) + 1024, dtype=torch.uint8,
                           device=dev)
        capi.check(L.qqt_l1_wgrad(rows.data_ptr(), n, rows.stride(0), ctx.k_in, None, 0,
                                  dh1.data_ptr(), n_players, channels, hw, pid, dw0.data_ptr(),
                                  _aligned(work, 1024), capi.stream_ptr(dev)), "qqt_l1_wgrad")
        return None, dw0, dh1.sum(0), None, None


class _MLPTrain(torch.autograd.Function):
    """ActorCritic(mlp).evaluate (train/model.py:121-153, 247-256) on the B200
    kernels: returns per-row (logp of the recorded actions, entropy, value);
    backward gives every parameter's gradient in the reference's layouts.
    rows: the batch's observation rows, or, with idx (int64 row ids), a
    larger row buffer whose rows idx the batch reads in place (TMA gather).
    params: the 20 tensors in state_dict order."""

    @staticmethod
    def forward(ctx, rows, idx, mm, bm, act, geom, *params):
        from . import _capi as capi
        n_players, c, hw, pid = geom
        k_in = c * hw
        L, dev = capi.lib(), rows.device
        st = capi.stream_ptr(dev)
        pc = [p.detach().contiguous() for p in params]
        pack = torch.empty(int(L.qqt_mlp_pack_bytes(k_in, 1)) + 256, dtype=torch.uint8, device=dev)
        pk = _aligned(pack, 256)
        ptrs = (ctypes.c_void_p * 20)(*[p.data_ptr() for p in pc])
        pids = (ctypes.c_int32 * 2)(pid, 0)
        capi.check(L.qqt_mlp_pack(ptrs, k_in, n_players, c, hw, 1, pids, pk, st), "qqt_mlp_pack")
        idx = None if idx is None else idx.to(torch.int64).contiguous()
        n = rows.shape[0] if idx is None else idx.numel()
        mm8 = mm.contiguous().view(torch.uint8)
        bm8 = bm.contiguous().view(torch.uint8)
        a64 = act.to(torch.int64).contiguous()
        logp, ent, v = (torch.empty(n, dtype=torch.float32, device=dev) for _ in range(3))
        h1, h2 = (torch.empty((n, 128), dtype=torch.float32, device=dev) for _ in range(2))
        capi.check(L.qqt_mlp_train_forward(pk, rows.data_ptr(), n, rows.stride(0), k_in,
                                           None if idx is None else idx.data_ptr(),
                                           0 if idx is None else rows.shape[0],
                                           mm8.data_ptr(), mm8.stride(0), bm8.data_ptr(),
                                           bm8.stride(0), a64.data_ptr(), a64.stride(0),
                                           logp.data_ptr(), ent.data_ptr(), v.data_ptr(),
                                           h1.data_ptr(), h2.data_ptr(), st),
                   "qqt_mlp_train_forward")
        ctx.save_for_backward(rows, mm8, bm8, a64, h1, h2)
        ctx.idx = idx
        ctx.pack, ctx.pk, ctx.geom = pack, pk, geom
        ctx.shapes = [p.shape for p in params]
        return logp, ent, v

    @staticmethod
    def backward(ctx, gl, ge, gv):
        from . import _capi as capi
        rows, mm8, bm8, a64, h1, h2 = ctx.saved_tensors
        idx = ctx.idx
        n_players, c, hw, pid = ctx.geom
        k_in = c * hw
        L, dev = capi.lib(), rows.device
        st = capi.stream_ptr(dev)
        n = h1.shape[0]
        g = torch.zeros((3, n), dtype=torch.float32, device=dev)
        for i, gi in enumerate((gl, ge, gv)):
            if gi is not None:
                g[i] = gi
        grads = [torch.empty(s, dtype=torch.float32, device=dev) for s in ctx.shapes]
        dh1 = torch.empty((n, 128), dtype=torch.float32, device=dev)
        work = torch.empty(int(L.qqt_mlp_train_work_bytes(n)) + 1024, dtype=torch.uint8,
                           device=dev)
        ptrs = (ctypes.c_void_p * 20)(*[t.data_ptr() for t in grads])
        capi.check(L.qqt_mlp_train_backward(ctx.pk, n, k_in, h1.data_ptr(), h2.data_ptr(),
                                            mm8.data_ptr(), mm8.stride(0), bm8.data_ptr(),
                                            bm8.stride(0), a64.data_ptr(), a64.stride(0),
                                            g.data_ptr(), ptrs, dh1.data_ptr(),
                                            _aligned(work, 1024), st),
                   "qqt_mlp_train_backward")
        wk = torch.empty(int(L.qqt_l1_wgrad_work_bytes(n, k_in)) + 1024, dtype=torch.uint8,
                         device=dev)
        capi.check(L.qqt_l1_wgrad(rows.data_ptr(), n, rows.stride(0), k_in,
                                  None if idx is None else idx.data_ptr(),
                                  0 if idx is None else rows.shape[0], dh1.data_ptr(),
                                  n_players, c, hw, pid, grads[0].data_ptr(),
                                  _aligned(wk, 1024), st), "qqt_l1_wgrad")
        return (None, None, None, None, None, None, *grads)


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
        if obs.is_cuda:
            c, h, w = self.obs_shape
            x = _Layer1.apply(obs_rows(obs, self.k_in), self.shared[0].weight,
                              self.shared[0].bias, self.k_in, (self.n_players, c, h * w, pid))
        else:
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

    def evaluate(self, obs, mm, bm, actions, pid: int = 0, rows_idx=None):
        """(log-prob of `actions`, entropy, value) under the masked heads
        (train/model.py:247-256).  rows_idx (CUDA only): the batch is rows
        rows_idx of the row buffer `obs` (the reference's obs[sel]), read in
        place by the kernels' TMA gathers -- no copy of the batch, for callers
        short of memory; on a rollout buffer far larger than L2 a
        `gather_rows` copy first is about 4x faster."""
        if obs.is_cuda:
            c, h, w = self.obs_shape
            return _MLPTrain.apply(obs_rows(obs, self.k_in), rows_idx, mm, bm, actions,
                                   (self.n_players, c, h * w, pid), *self.parameters())
        if rows_idx is not None:
            obs = obs[rows_idx]
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


SIDE_BYTES = 48   # packed per-row side data: act int64 x2 | logp, val, adv, ret f32 | mm u8 x5, bm u8 x2


def _pack_side(mm, bm, act, logp, val, adv, ret):
    """The per-row fields a minibatch reads besides the observation, packed
    into one 48-byte row each (one gather per minibatch on the device)."""
    n = act.shape[0]
    side = torch.zeros((n, SIDE_BYTES), dtype=torch.uint8, device=act.device)
    side.view(torch.int64)[:, 0:2] = act.to(torch.int64)
    side.view(torch.float32)[:, 4:8] = torch.stack([logp, val, adv, ret], 1).to(torch.float32)
    side[:, 32:37] = mm.to(torch.bool).view(torch.uint8)
    side[:, 37:39] = bm.to(torch.bool).view(torch.uint8)
    return side


def _side_views(sg):
    """(mm, bm, act, logp, val, adv, ret) views of gathered side rows."""
    f = sg.view(torch.float32)
    return (sg[:, 32:37].view(torch.bool), sg[:, 37:39].view(torch.bool),
            sg.view(torch.int64)[:, 0:2], f[:, 4], f[:, 5], f[:, 6], f[:, 7])


def sampling_pool(total: int, rare: torch.Tensor, copies: int) -> torch.Tensor:
    """Row indices that every epoch's permutation draws its `total` rows
    from (oversampling of dying frames, train/ppo.py:377-392): each row
    once, in order, followed -- when `copies` > 1 and some row is rare (hp
    lost in an env that continued, or an episode end) -- by the list of
    rare rows repeated copies - 1 times.  Rare frames are a handful per
    episode; the extra copies raise their chance of being drawn without
    changing the number of rows an epoch trains on."""
    rows = torch.arange(total, device=rare.device)
    if copies <= 1:
        return rows
    rare_rows = torch.nonzero(rare).flatten()
    if rare_rows.numel() == 0:
        return rows
    return torch.cat([rows] + [rare_rows] * (copies - 1))


def ppo_update(model: MLPActorCritic, opt, data: dict, last_val, cfg: PPOConfig,
               entropy_coef: float, pid: int = 0, perm_fn=None,
               profile: dict | None = None) -> dict:
    """One PPO update over a (T, N) rollout shard (train/ppo.py:364-437).

    data: obs (T,N,C,H,W) fp16 (or row-padded view), mm (T,N,5), bm (T,N,2),
    act (T,N,2), logp/val/rew (T,N), done (T,N) bool, dmg (T,N) bool.
    Advantage statistics and gradients are reduced over all ranks of the
    default process group when one is initialised.  perm_fn(n) -> index
    permutation (defaults to torch.randperm on the data's device).
    profile: a dict that, on CUDA, receives a list of (start, end) CUDA
    event pairs around every minibatch's gradient all-reduce under
    "allreduce_events" (read after a synchronize).
    """
    dev = data["rew"].device
    adv, ret = gae(data["rew"], data["done"], data["val"], last_val, cfg.gamma, cfg.gae_lambda)
    T, n = adv.shape
    total = T * n

    def by_row(x):
        # (T, N, ...) -> (T*N, ...): one training row per (tick, env)
        return x.reshape(total, *x.shape[2:])

    obs = by_row(data["obs"])
    if obs.is_cuda:
        obs = obs_rows(obs, model.k_in)
    mm, bm, act = by_row(data["mm"]), by_row(data["bm"]), by_row(data["act"])
    old_logp, old_val = by_row(data["logp"]), by_row(data["val"])
    adv, ret = by_row(adv), by_row(ret)
    # global mean / unbiased std of the advantages over every rank's shard
    stats = torch.stack([adv.sum(), (adv * adv).sum(),
                         torch.tensor(float(total), device=dev)]).to(torch.float64)
    world = _all_reduce(stats)
    cnt = stats[2]
    mean = stats[0] / cnt
    var = (stats[1] - cnt * mean * mean) / (cnt - 1)
    std = math.sqrt(max(float(var), 0.0)) if world > 1 else float(adv.std())
    adv = (adv - (mean.float() if world > 1 else adv.mean())) / (std + 1e-8)

    pool = sampling_pool(total, by_row(data["dmg"]) | by_row(data["done"]).bool(),
                         cfg.oversample_dying)
    mb = max(1, total // cfg.minibatches)
    perm_fn = perm_fn or (lambda k: torch.randperm(k, device=dev))
    # statistics stay on the device; one host read at the end
    out = {k: torch.zeros((), device=dev) for k in ("pg", "vf", "ent", "kl", "clipfrac")}
    updates = 0
    xg = sg = None
    side = _pack_side(mm, bm, act, old_logp, old_val, adv, ret) if obs.is_cuda else None
    params = [p for p in model.parameters()]
    for _ in range(cfg.epochs):
        perm = pool[perm_fn(pool.numel())][:total]
        for start in range(0, total, mb):
            sel = perm[start:start + mb]
            if side is not None:
                # one gather of the packed per-row fields instead of one index op each
                if sg is None or sg.shape[0] < sel.numel():
                    sg = torch.empty((sel.numel(), SIDE_BYTES), dtype=torch.uint8, device=dev)
                s_mm, s_bm, s_act, s_lp, s_val, s_adv, s_ret = _side_views(
                    gather_rows(side, sel, sg[:sel.numel()]))
            else:
                s_mm, s_bm, s_act = mm[sel], bm[sel], act[sel]
                s_lp, s_val, s_adv, s_ret = old_logp[sel], old_val[sel], adv[sel], ret[sel]
            if obs.is_cuda:
                # the minibatch's rows copied whole into one reused block (whole
                # 4.7 KB rows stream at HBM speed; reading them in place with
                # TMA gathers, evaluate(rows_idx=sel), fetches 128-byte pieces
                # of random rows and measured 4x slower); the previous
                # minibatch's backward has finished reading the block
                if xg is None or xg.shape[0] < sel.numel():
                    xg = torch.empty((sel.numel(), obs.shape[1]), dtype=obs.dtype, device=dev)
                x = gather_rows(obs, sel, xg[:sel.numel()])
            else:
                x = obs[sel]
            logp, ent, value = model.evaluate(x, s_mm, s_bm, s_act, pid)
            ratio = (logp - s_lp).exp()
            a = s_adv
            pg = -torch.min(ratio * a, ratio.clamp(1 - cfg.clip_eps, 1 + cfg.clip_eps) * a).mean()
            v_clip = s_val + (value - s_val).clamp(-cfg.clip_eps, cfg.clip_eps)
            vf = 0.5 * torch.max((value - s_ret) ** 2, (v_clip - s_ret) ** 2).mean()
            ent_m = ent.mean()
            loss = pg + cfg.value_coef * vf - entropy_coef * ent_m
            opt.zero_grad(set_to_none=True)
            loss.backward()
            grads = [p.grad for p in params if p.grad is not None]
            if grads:
                buf = torch.cat([g.reshape(-1) for g in grads])
                ev = None
                if profile is not None and buf.is_cuda:
                    ev = (torch.cuda.Event(enable_timing=True),
                          torch.cuda.Event(enable_timing=True))
                    ev[0].record()
                w = _all_reduce(buf)
                if ev is not None:
                    ev[1].record()
                    profile.setdefault("allreduce_events", []).append(ev)
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
                out["kl"] += (s_lp - logp).mean().detach()
                out["clipfrac"] += ((ratio - 1).abs() > cfg.clip_eps).float().mean()
            updates += 1
    return {k: float(v) / max(1, updates) for k, v in out.items()}
