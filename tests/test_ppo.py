"""PPO update parity (train/ppo.py:101-110, 364-437) and the data-parallel
gradient average.

CPU: the torch restatement reproduces the reference's compute_gae exactly and
its ppo_update (same minibatch permutations) to float32 rounding; two gloo
ranks each holding half a minibatch average to the single-process gradient
over the union.  GPU: the GAE kernel reproduces the reference bit for bit and
the update on the device tracks the reference parameters.
"""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import goldens as G
from qqt_b200 import scenarios
from qqt_b200.config import SimConfig
from qqt_b200.policy_init import init_params
from qqt_b200.ppo import MLPActorCritic, PPOConfig, gae, ppo_update


def _model(device="cpu"):
    cfg = SimConfig(**scenarios.CFG2)
    m = MLPActorCritic(cfg.obs_shape, 2).to(device)
    sd = m.state_dict()
    p = init_params(cfg.obs_shape, "mlp", seed=9)
    m.load_state_dict({k: torch.from_numpy(p[k]) for k in sd})
    return m


def _data(g, device):
    d = {k: torch.from_numpy(np.asarray(g[k])).to(device)
         for k in ("obs", "mm", "bm", "act", "logp", "val", "rew", "dmg")}
    d["done"] = torch.from_numpy(g["done"] > 0.5).to(device)
    return d


def _run(device, g):
    model = _model(device)
    opt = torch.optim.Adam(model.parameters(), lr=1e-4, eps=1e-5)
    perms = [torch.from_numpy(g[f"perm{i}"]).to(device) for i in range(int(g["n_perms"]))]
    it = iter(perms)
    stats = ppo_update(model, opt, _data(g, device), torch.from_numpy(g["last_val"]).to(device),
                       PPOConfig(epochs=2, minibatches=2, lr=1e-4), 0.03,
                       perm_fn=lambda k: next(it))
    return model, stats


def test_gae_matches_reference_cpu():
    g = G.load("ppo_update")
    adv, ret = gae(torch.from_numpy(g["rew"]), torch.from_numpy(g["done"] > 0.5),
                   torch.from_numpy(g["val"]), torch.from_numpy(g["last_val"]), 0.995, 0.95)
    assert np.array_equal(adv.numpy(), g["adv"]) and np.array_equal(ret.numpy(), g["ret"])


def test_ppo_update_matches_reference_cpu():
    g = G.load("ppo_update")
    model, stats = _run("cpu", g)
    for k, v in model.state_dict().items():
        ref = g["param__" + k]
        err = np.abs(v.numpy() - ref).max()
        assert err <= 1e-5 * max(1.0, np.abs(ref).max()), f"{k}: {err}"
    ref_stats = g["stats"]
    got = np.array([stats[k] for k in ("pg", "vf", "ent", "kl", "clipfrac")])
    assert np.allclose(got, ref_stats, rtol=1e-4, atol=1e-6)


def _dp_worker(rank, world, port, path, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(0)
    model = _model("cpu")
    g = np.load(path)
    obs = torch.from_numpy(g["obs"][0].astype(np.float32))
    half = obs.shape[0] // world
    sl = slice(rank * half, (rank + 1) * half)
    act = torch.from_numpy(g["act"][0])
    mm = torch.from_numpy(g["mm"][0])
    bm = torch.from_numpy(g["bm"][0])
    logp, ent, v = model.evaluate(obs[sl], mm[sl], bm[sl], act[sl])
    (logp.mean() + 0.5 * (v ** 2).mean() - 0.03 * ent.mean()).backward()
    flat = torch.cat([p.grad.reshape(-1) for p in model.parameters()])
    dist.all_reduce(flat)
    flat /= world
    if rank == 0:
        q.put(flat.numpy())
    dist.destroy_process_group()


def test_data_parallel_gradient_average_gloo():
    import multiprocessing as mp
    import socket
    g = G.load("ppo_update")
    path = os.path.join(G.GOLDEN, "ppo_update.npz")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dp_worker, args=(r, 2, port, path, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    model = _model("cpu")
    obs = torch.from_numpy(g["obs"][0].astype(np.float32))
    logp, ent, v = model.evaluate(obs, torch.from_numpy(g["mm"][0]), torch.from_numpy(g["bm"][0]),
                                  torch.from_numpy(g["act"][0]))
    (logp.mean() + 0.5 * (v ** 2).mean() - 0.03 * ent.mean()).backward()
    ref = torch.cat([p.grad.reshape(-1) for p in model.parameters()]).numpy()
    assert np.abs(got - ref).max() <= 1e-6 * max(1.0, np.abs(ref).max())


@pytest.mark.gpu
def test_gae_kernel_bit_exact_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    g = G.load("ppo_update")
    adv, ret = gae(torch.from_numpy(g["rew"]).cuda(), torch.from_numpy(g["done"] > 0.5).cuda(),
                   torch.from_numpy(g["val"]).cuda(), torch.from_numpy(g["last_val"]).cuda(),
                   0.995, 0.95)
    assert np.array_equal(adv.cpu().numpy(), g["adv"]) and np.array_equal(ret.cpu().numpy(), g["ret"])


@pytest.mark.gpu
def test_ppo_update_gpu_tracks_reference():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    torch.backends.cuda.matmul.allow_tf32 = False
    g = G.load("ppo_update")
    model, _ = _run("cuda", g)
    for k, v in model.state_dict().items():
        ref = g["param__" + k]
        err = np.abs(v.cpu().numpy() - ref).max()
        assert err <= 1e-4 * max(1.0, np.abs(ref).max()), f"{k}: {err}"


def test_packed_side_rows_round_trip():
    """The per-row fields a minibatch reads (actions, old log-prob and value,
    advantage, return, legal masks) packed into one 48-byte row each: the
    views of gathered rows equal the fields indexed one by one."""
    from qqt_b200.ppo import SIDE_BYTES, _pack_side, _side_views
    g = torch.Generator().manual_seed(3)
    n = 257
    mm = torch.rand((n, 5), generator=g) < 0.6
    bm = torch.rand((n, 2), generator=g) < 0.6
    act = torch.randint(0, 5, (n, 2), generator=g)
    f = [torch.randn(n, generator=g) for _ in range(4)]
    side = _pack_side(mm, bm, act, *f)
    assert side.shape == (n, SIDE_BYTES) and side.dtype == torch.uint8
    sel = torch.randint(0, n, (100,), generator=g)
    s_mm, s_bm, s_act, s_lp, s_val, s_adv, s_ret = _side_views(side[sel])
    assert torch.equal(s_mm, mm[sel]) and torch.equal(s_bm, bm[sel])
    assert torch.equal(s_act, act[sel])
    for got, want in zip((s_lp, s_val, s_adv, s_ret), f):
        assert torch.equal(got, want[sel])
