"""Host reset parity: B200Sim built with the reference's seed generates the
same maps, spawns and attributes as BatchedSim (the reference's
test_parity_after_shared_reset check), for several map modes, at
construction and after a partial reset_."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import goldens as G

pytestmark = pytest.mark.gpu

CASES = {
    "open_default": dict(),
    "open_obstacles": dict(open_obstacle_max=6, height=11, width=11),
    "corridor_default": dict(map_mode="corridor", speed=3.0, max_steps=1800),
    "corridor_dense": dict(map_mode="corridor", wall_density=0.45, random_wall_rows=False),
    "corridor_mixed": dict(map_mode="corridor", open_fraction=0.3, ring_fraction=0.3,
                           pure_open_fraction=0.1, wall_density=0.25, open_obstacle_max=3),
    "pillars_open": dict(wall_density=0.6, height=11, width=11),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_reset_matches_reference(name):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from qqt_b200.config import SimConfig
    from qqt_b200.sim import B200Sim
    g = G.load("reset_modes")
    sim = B200Sim(SimConfig(**CASES[name]), 24, device="cuda", seed=999)
    ref = {k: g[f"{name}__init__{k}"] for k in G.STATE_KEYS}
    bad = G.compare_state(ref, sim.numpy_state())
    assert not bad, f"{name} init differs in {bad}"
    mask = torch.zeros(24, dtype=torch.bool)
    mask[::2] = True
    sim.reset_(mask)
    ref = {k: g[f"{name}__again__{k}"] for k in G.STATE_KEYS}
    bad = G.compare_state(ref, sim.numpy_state())
    assert not bad, f"{name} second reset differs in {bad}"
