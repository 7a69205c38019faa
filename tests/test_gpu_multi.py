"""Data-parallel PPO over NCCL on two GPUs (skipped with fewer than two).

* the NCCL-averaged gradient of two ranks, each holding half of a minibatch,
  equals the single-GPU gradient over the union (train/ppo.py's data-parallel
  contract: all_reduce(SUM) / world);
* a full `ppo_update` on two ranks with their own env shards leaves the two
  parameter replicas bit-identical, and different from the start.

Ranks are spawned processes, one per GPU; NVLS is off and the process group
has a short timeout, so a failing rank ends the others' collectives with an
error instead of a wait.
"""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import goldens as G

pytestmark = pytest.mark.gpu


def _need_two():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")


def _model(device):
    from qqt_b200 import scenarios
    from qqt_b200.config import SimConfig
    from qqt_b200.policy_init import init_params
    from qqt_b200.ppo import MLPActorCritic
    cfg = SimConfig(**scenarios.CFG2)
    model = MLPActorCritic(cfg.obs_shape, 2).to(device)
    params = init_params(cfg.obs_shape, "mlp", seed=9)
    model.load_state_dict({k: torch.from_numpy(params[k]) for k in model.state_dict()})
    return model


def _init(rank, world, port):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device(f"cuda:{rank}"))
    return dist


def _grad_worker(rank, world, port, q):
    import sys
    sys.path[:0] = [os.path.dirname(os.path.abspath(__file__))]
    dist = _init(rank, world, port)
    try:
        dev = f"cuda:{rank}"
        g = G.load("ppo_update")
        model = _model(dev)
        obs = torch.from_numpy(g["obs"][0]).to(dev)
        half = obs.shape[0] // world
        sl = slice(rank * half, (rank + 1) * half)
        act = torch.from_numpy(g["act"][0]).to(dev)
        mm = torch.from_numpy(g["mm"][0]).to(dev)
        bm = torch.from_numpy(g["bm"][0]).to(dev)
        logp, ent, v = model.evaluate(obs[sl], mm[sl], bm[sl], act[sl])
        (logp.mean() + 0.5 * (v ** 2).mean() - 0.03 * ent.mean()).backward()
        flat = torch.cat([p.grad.reshape(-1) for p in model.parameters()])
        dist.all_reduce(flat)
        flat /= world
        if rank == 0:
            q.put(flat.cpu().numpy())
    finally:
        dist.destroy_process_group()


def _update_worker(rank, world, port, q):
    import sys
    sys.path[:0] = [os.path.dirname(os.path.abspath(__file__))]
    dist = _init(rank, world, port)
    try:
        from qqt_b200.ppo import PPOConfig, ppo_update
        dev = f"cuda:{rank}"
        g = G.load("ppo_update")
        model = _model(dev)
        start = torch.cat([p.detach().reshape(-1) for p in model.parameters()]).clone()
        opt = torch.optim.Adam(model.parameters(), lr=1e-4, eps=1e-5)
        T, n = g["rew"].shape
        half = n // world
        sl = slice(rank * half, (rank + 1) * half)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a[:, sl])).to(dev)  # noqa: E731
        data = {"obs": t(g["obs"]), "mm": t(g["mm"]), "bm": t(g["bm"]), "act": t(g["act"]),
                "logp": t(g["logp"]), "val": t(g["val"]), "rew": t(g["rew"]),
                "done": t(g["done"] > 0.5), "dmg": t(g["dmg"])}
        last = torch.from_numpy(g["last_val"][sl]).to(dev)
        gen = torch.Generator(device=dev).manual_seed(5)
        cfg = PPOConfig(epochs=2, minibatches=2)
        ppo_update(model, opt, data, last, cfg, 0.03, pid=0,
                   perm_fn=lambda k: torch.randperm(k, device=dev, generator=gen))
        flat = torch.cat([p.detach().reshape(-1) for p in model.parameters()])
        moved = float((flat - start).abs().max())
        both = [torch.zeros_like(flat) for _ in range(world)]
        dist.all_gather(both, flat)
        if rank == 0:
            q.put((moved, float((both[0] - both[1]).abs().max())))
    finally:
        dist.destroy_process_group()


def _spawn(target, world=2):
    import multiprocessing as mp
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        got = q.get(timeout=180)
    finally:
        for p in procs:
            p.join(timeout=120)
    for p in procs:
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    return got


def test_nccl_gradient_average_two_gpus():
    _need_two()
    got = _spawn(_grad_worker)
    g = G.load("ppo_update")
    model = _model("cuda:0")
    obs = torch.from_numpy(g["obs"][0]).cuda()
    logp, ent, v = model.evaluate(obs, torch.from_numpy(g["mm"][0]).cuda(),
                                  torch.from_numpy(g["bm"][0]).cuda(),
                                  torch.from_numpy(g["act"][0]).cuda())
    (logp.mean() + 0.5 * (v ** 2).mean() - 0.03 * ent.mean()).backward()
    ref = torch.cat([p.grad.reshape(-1) for p in model.parameters()]).cpu().numpy()
    assert np.abs(got - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


def test_ppo_update_replicas_stay_identical_two_gpus():
    _need_two()
    moved, diff = _spawn(_update_worker)
    assert moved > 0.0, "the update did not change the parameters"
    assert diff == 0.0, f"replicas diverged by {diff}"
