"""GPU check of the tcgen05 policy kernel's failure path, written in the
form this pool allows: a bounded wait that runs out and returns, with no
trap and nothing in flight.

qqt_test_set_wait_polls(k) makes every fused-MLP launch start with one
bounded mbarrier wait of k polls on a barrier that nothing completes at
that point, before any TMA copy or MMA is issued.  The wait expires exactly
as a production wait that runs out does: QQT_DEV_TIMEOUT goes into the
error word and the kernel takes its abort path (the abort flag, the
epilogue warps' AND-barrier, the split-K cluster's closing barrier, TMEM
freed).  The launch must end, write no outputs, raise only QQT_DEV_TIMEOUT,
and the next launch with the check off must give the same outputs as
before: its TMEM allocation succeeds, so the aborted CTAs freed theirs.
Both the one-CTA instance (more than 16 row tiles) and the split-K cluster
instance (up to 16 row tiles), with one and two seats.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from qqt_b200 import _capi, scenarios
    from qqt_b200.config import SimConfig
    from qqt_b200.policy import B200Policy
    from qqt_b200.policy_init import init_params

QQT_DEV_TIMEOUT = 1 << 3


@pytest.fixture(autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    yield
    _capi.lib().qqt_test_set_wait_polls(0)
    torch.cuda.synchronize()
    assert _capi.device_error() == 0, "device error word set"


def _inputs(cfg, n, p, seats, seed):
    rng = np.random.default_rng(seed)
    c, h, w = cfg.obs_shape
    k = c * h * w
    stride = (k + 7) // 8 * 8
    rows = torch.zeros((n, stride), dtype=torch.float16, device="cuda")
    vals = (rng.random((n, k)) * (rng.random((n, k)) < 0.3)).astype(np.float16)
    rows[:, :k] = torch.from_numpy(vals).cuda()
    mm = rng.random((n, p, 5)) < 0.8
    mm[..., 4] = True
    bm = rng.random((n, p, 2)) < 0.7
    bm[..., 0] = True
    u = rng.random((len(seats), n, 2)).astype(np.float32)
    return (rows[:, :k].view(n, c, h, w), torch.from_numpy(mm).cuda(),
            torch.from_numpy(bm).cuda(), torch.from_numpy(u).cuda())


def _run(pol, obs, mm, bm, u, S, n):
    logits = torch.full((S, n, 8), 12345.0, dtype=torch.float32, device="cuda")
    logp = torch.full((S, n), 12345.0, dtype=torch.float32, device="cuda")
    acts = [torch.full((n, 2), -7, dtype=torch.int64, device="cuda") for _ in range(S)]
    pol.act_seats(obs, [mm[:, s] for s in pol.seats], [bm[:, s] for s in pol.seats], u, acts,
                  logp, None, logits)
    torch.cuda.synchronize()
    return logits, logp, torch.stack(acts)


@pytest.mark.parametrize("n,seats", [(4096, (0,)), (512, (0,)), (2816, (0, 1)), (384, (0, 1))])
def test_policy_wait_expiry_takes_the_abort_path(n, seats):
    cfg = SimConfig(**scenarios.CFG2)
    p = cfg.n_players
    pol = B200Policy(init_params(cfg.obs_shape, "mlp", seed=5), cfg.obs_shape, p, seats=seats)
    obs, mm, bm, u = _inputs(cfg, n, p, seats, seed=n)
    S = len(seats)
    ref = _run(pol, obs, mm, bm, u, S, n)
    assert _capi.device_error() == 0
    assert int((ref[2] < 0).sum()) == 0
    lib = _capi.lib()
    assert lib.qqt_test_set_wait_polls(64) == 0
    try:
        got = _run(pol, obs, mm, bm, u, S, n)
        err = _capi.device_error()
    finally:
        lib.qqt_test_set_wait_polls(0)
    assert err == QQT_DEV_TIMEOUT, f"error word {err:#x}"
    assert bool((got[0] == 12345.0).all()) and bool((got[1] == 12345.0).all()), \
        "an aborted launch writes no outputs"
    assert bool((got[2] == -7).all())
    again = _run(pol, obs, mm, bm, u, S, n)
    assert _capi.device_error() == 0
    for a, b in zip(ref, again):
        assert torch.equal(a, b), "the launch after an abort gives the same outputs"
