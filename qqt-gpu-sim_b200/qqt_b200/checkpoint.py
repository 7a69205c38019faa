"""Checkpoints in the reference's training format.

The reference trainer writes one `torch.save` dict per checkpoint
(train/train.py:307-331, `save_ckpt`, format_version 2) and reads it back in
three places: `--resume` (train/train.py:515-547), `load_fixed_checkpoint`
for frozen sparring partners (train/train.py:243-260), and `adapt_first_conv`
when the player count, and with it the channel count, changes between
curriculum stages (train/train.py:92-158).  This module writes and reads the
same dict, so a checkpoint moves between the two trainers in either
direction, and loads one straight into the B200 policy.

Keys (all written, all read back by the reference): format_version, model
(state_dict, reference parameter names), obs_shape, n_players, arch, opt
(optimizer state_dict), pool ({max_size, k, snapshots}), fixed_elo,
curriculum ({stage_idx, episodes_in_stage, recent_wins}), global_step, elo,
args, torch_rng, py_rng.
"""

from __future__ import annotations

import os
import random

import numpy as np
import torch

FORMAT_VERSION = 2
# the layer whose input channels are the observation's, per architecture
# (the LSTM's is the first convolution of its local-view CNN)
FIRST_LAYER = {"cnn": "conv0.weight", "mlp": "shared.0.weight", "lstm": "l_conv1.weight"}
POLICY_ARCHS = ("mlp", "cnn")     # the architectures B200Policy runs


def obs_extra(n_players: int) -> int:
    """Extra world-information channels after the 2P+3 view channels
    (sim/config.py:69-74)."""
    return 1 + 3 * n_players


def infer_players(c: int) -> int:
    """Player count from a channel count (train/model.py:44-51): the 5P+4
    layout (with the extra channels) first, else the old 2P+3 one."""
    if (c - 4) % 5 == 0:
        return (c - 4) // 5
    return (c - 3) // 2


def save_ckpt(path: str, *, model: dict, obs_shape, n_players: int, arch: str,
              opt: dict | None = None, pool: dict | None = None, fixed_elo: dict | None = None,
              curriculum: dict | None = None, global_step: int = 0, elo: float = 1000.0,
              args: dict | None = None) -> None:
    """Write a format-2 checkpoint (train/train.py:307-331).

    model: state_dict with the reference's parameter names (tensors or
    arrays); opt: an optimizer state_dict; pool: the ELO pool's state
    (default: an empty pool with the reference's defaults); curriculum: the
    curriculum state fields.  The file is written to `path + ".tmp"` and
    renamed over `path`, so an interrupted save leaves the old file intact.
    """
    if arch not in FIRST_LAYER:
        raise ValueError(f"unsupported arch {arch}")
    d = os.path.dirname(path)
    if d:
        os.makedirs(d, exist_ok=True)
    state = {k: (v.detach().cpu() if torch.is_tensor(v) else torch.from_numpy(np.asarray(v)))
             for k, v in model.items()}
    ck = {
        "format_version": FORMAT_VERSION,
        "model": state,
        "obs_shape": tuple(int(x) for x in obs_shape),
        "n_players": int(n_players),
        "arch": arch,
        "opt": opt if opt is not None else {"state": {}, "param_groups": []},
        "pool": pool if pool is not None else {"max_size": 12, "k": 16.0, "snapshots": []},
        "fixed_elo": dict(fixed_elo or {}),
        "curriculum": dict(curriculum or {"stage_idx": 0, "episodes_in_stage": 0,
                                          "recent_wins": []}),
        "global_step": int(global_step),
        "elo": float(elo),
        "args": dict(args or {}),
        "torch_rng": torch.get_rng_state(),
        "py_rng": random.getstate(),
    }
    tmp = path + ".tmp"
    torch.save(ck, tmp)
    os.replace(tmp, path)


def load_ckpt(path: str, map_location="cpu") -> dict:
    """Read a checkpoint; like the reference's --resume, anything but
    format_version 2 is rejected (train/train.py:515-519)."""
    ck = torch.load(path, map_location=map_location, weights_only=False)
    if ck.get("format_version") != FORMAT_VERSION:
        raise ValueError("checkpoint uses an old observation layout (format_version "
                         f"{ck.get('format_version')!r}); only format_version 2 loads")
    return ck


def adapt_first_layer(state: dict, old_shape, new_shape, arch: str,
                      old_players: int | None = None, new_players: int | None = None,
                      new_state: dict | None = None) -> dict:
    """Migrate a state_dict to a new channel count (train/train.py:92-158).

    The first layer's input channels are in view order: [0] own position,
    [1] own bomb fuses, [2 .. P] the opponents' positions, [P+1 .. 2P-1]
    their fuses, [2P .. 2P+2] wall / danger / progress.  The two own
    channels and the three map channels are carried over by position, the
    opponent blocks up to min(P_old, P_new) - 1 opponents; every other
    input channel of the new layer (new opponents, the extra world channels)
    starts at zero.  Keys whose shapes match are copied; `new_state` supplies
    the rest (the new model's initial values), otherwise they are absent.
    """
    if arch not in FIRST_LAYER:
        raise ValueError(f"unsupported arch {arch!r} (one of {sorted(FIRST_LAYER)})")
    old_shape, new_shape = tuple(old_shape), tuple(new_shape)
    out = {k: (v.clone() if torch.is_tensor(v) else torch.as_tensor(np.array(v)))
           for k, v in (new_state or {}).items()}
    if old_shape == new_shape:
        return {k: (v.clone() if torch.is_tensor(v) else torch.as_tensor(np.array(v)))
                for k, v in state.items()}
    op = old_players if old_players is not None else infer_players(old_shape[0])
    np_ = new_players if new_players is not None else infer_players(new_shape[0])
    keep = min(op, np_) - 1
    first = FIRST_LAYER[arch]
    for k, v in state.items():
        v = v if torch.is_tensor(v) else torch.as_tensor(np.array(v))
        if k != first:
            if new_state is not None and (k not in out or tuple(out[k].shape) != tuple(v.shape)):
                continue      # dropped, or the new init stays (shape changed, not migrated)
            out[k] = v.clone()
            continue
        if arch in ("cnn", "lstm"):
            # a convolution: input channels on dimension 1
            w = torch.zeros((v.shape[0], new_shape[0]) + tuple(v.shape[2:]), dtype=v.dtype)
            w[:, :2] = v[:, :2]
            w[:, 2 * np_:2 * np_ + 3] = v[:, 2 * op:2 * op + 3]
            if keep > 0:
                w[:, 2:2 + keep] = v[:, 2:2 + keep]
                w[:, np_ + 1:np_ + 1 + keep] = v[:, op + 1:op + 1 + keep]
        else:
            hw = new_shape[1] * new_shape[2]
            w = torch.zeros((v.shape[0], new_shape[0] * hw), dtype=v.dtype)
            w[:, :2 * hw] = v[:, :2 * hw]
            w[:, 2 * np_ * hw:(2 * np_ + 3) * hw] = v[:, 2 * op * hw:(2 * op + 3) * hw]
            if keep > 0:
                w[:, 2 * hw:(2 + keep) * hw] = v[:, 2 * hw:(2 + keep) * hw]
                w[:, (np_ + 1) * hw:(np_ + 1 + keep) * hw] = \
                    v[:, (op + 1) * hw:(op + 1 + keep) * hw]
        out[k] = w
    return out


def load_policy(path: str, device="cuda", target_shape=None, seats=(0,), new_state=None):
    """A checkpoint as a B200Policy (the reference's load_fixed_checkpoint,
    train/train.py:243-260): the arch and player count come from the file;
    a different `target_shape` migrates the first layer (adapt_first_layer;
    `new_state` supplies keys whose shapes change otherwise)."""
    from .policy import B200Policy
    ck = load_ckpt(path)
    arch = ck.get("arch", "cnn")
    if arch not in POLICY_ARCHS:
        raise ValueError(f"B200Policy runs the {' and '.join(POLICY_ARCHS)} architectures, not "
                         f"{arch!r}; load_ckpt and adapt_first_layer still read and migrate "
                         "this checkpoint's weights")
    shape = tuple(ck["obs_shape"])
    n_p = ck.get("n_players") or infer_players(shape[0])
    sd = dict(ck["model"])
    if target_shape is not None and tuple(target_shape) != shape:
        sd = adapt_first_layer(sd, shape, target_shape, arch, n_p, None, new_state)
        shape = tuple(target_shape)
        n_p = infer_players(shape[0])
    return B200Policy(sd, shape, n_p, seats=seats, device=device, arch=arch)
