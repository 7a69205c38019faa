"""Seeded random initialisation of the reference policy's parameters.

The benchmark configurations use fp32 weights drawn from N(0, 0.02), zero
biases and LayerNorm (1, 0) for every layer of the reference `ActorCritic`
(train/model.py:54-165).  Parameters are returned as a dict of numpy arrays
keyed exactly like the reference's state_dict, so the same dict loads into
the reference model, the oracle and the B200 policy.
"""

from __future__ import annotations

import numpy as np


def mlp_param_shapes(obs_shape, n_moves=5, n_bomb=2):
    c, h, w = obs_shape
    flat = c * h * w
    shapes = {
        "shared.0.weight": (128, flat), "shared.0.bias": (128,),
        "shared.1.weight": (128,), "shared.1.bias": (128,),
        "shared.3.weight": (128, 128), "shared.3.bias": (128,),
        "shared.4.weight": (128,), "shared.4.bias": (128,),
    }
    shapes.update(_head_shapes(n_moves, n_bomb))
    return shapes


def cnn_param_shapes(obs_shape, n_moves=5, n_bomb=2):
    c, h, w = obs_shape
    shapes = {
        "conv0.weight": (16, c, 3, 3), "conv0.bias": (16,),
        "conv.0.weight": (16, h, w), "conv.0.bias": (16, h, w),
        "conv.2.weight": (32, 16, 3, 3), "conv.2.bias": (32,),
        "conv.3.weight": (32, h, w), "conv.3.bias": (32, h, w),
        "conv.5.weight": (64, 32, 3, 3), "conv.5.bias": (64,),
        "conv.6.weight": (64, h, w), "conv.6.bias": (64, h, w),
        "conv.8.weight": (8, 64, 1, 1), "conv.8.bias": (8,),
        "conv.9.weight": (8, h, w), "conv.9.bias": (8, h, w),
        "shared.0.weight": (128, 8 * h * w), "shared.0.bias": (128,),
        "shared.1.weight": (128,), "shared.1.bias": (128,),
        "shared.3.weight": (128, 128), "shared.3.bias": (128,),
        "shared.4.weight": (128,), "shared.4.bias": (128,),
    }
    shapes.update(_head_shapes(n_moves, n_bomb))
    return shapes


def _head_shapes(n_moves, n_bomb):
    out = {}
    for name, k in (("move_head", n_moves), ("bomb_head", n_bomb), ("critic", 1)):
        out[f"{name}.0.weight"] = (64, 128)
        out[f"{name}.0.bias"] = (64,)
        out[f"{name}.2.weight"] = (k, 64)
        out[f"{name}.2.bias"] = (k,)
    return out


_NORM_KEYS = ("shared.1.", "shared.4.", "conv.0.", "conv.3.", "conv.6.", "conv.9.")


def init_params(obs_shape, arch: str = "mlp", seed: int = 0, std: float = 0.02):
    """dict name -> float32 array: weights N(0, std), biases 0, norms (1, 0)."""
    shapes = (mlp_param_shapes if arch == "mlp" else cnn_param_shapes)(obs_shape)
    rng = np.random.default_rng(seed)
    out = {}
    for name in sorted(shapes):
        shp = shapes[name]
        if name.startswith(_NORM_KEYS):
            fill = 1.0 if name.endswith("weight") else 0.0
            out[name] = np.full(shp, fill, dtype=np.float32)
        elif name.endswith("bias"):
            out[name] = np.zeros(shp, dtype=np.float32)
        else:
            out[name] = rng.normal(0.0, std, size=shp).astype(np.float32)
    return out
