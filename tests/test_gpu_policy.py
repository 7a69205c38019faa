"""GPU parity of the MLP policy (tcgen05 first layer + fused heads).

Contract: logits and values within 2e-3 relative to the largest reference
magnitude of that output; sampled actions equal the oracle's inverse-CDF
draw except where the uniform lands within float32 rounding of a CDF
boundary (counted, must be 0 on these seeds).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import goldens as G

pytestmark = pytest.mark.gpu
REL_TOL = 2e-3

if torch.cuda.is_available():
    from oracle import qqt_oracle as O
    from qqt_b200 import scenarios
    from qqt_b200.config import SimConfig
    from qqt_b200.policy import B200Policy
    from qqt_b200.policy_init import init_params
    from qqt_b200 import _capi


@pytest.fixture(autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    yield
    torch.cuda.synchronize()
    assert _capi.device_error() == 0, "device error word set"


def _padded(obs16: np.ndarray) -> torch.Tensor:
    n = obs16.shape[0]
    k = obs16[0].size
    stride = (k + 7) // 8 * 8
    buf = torch.zeros((n, stride), dtype=torch.float16, device="cuda")
    buf[:, :k] = torch.from_numpy(obs16.reshape(n, -1)).cuda()
    return buf[:, :k].view(obs16.shape)


def _rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-12))


def test_mlp_logits_vs_reference_goldens():
    g = G.load("traj_cfg2")
    cfg = SimConfig(**scenarios.CFG2)
    params = init_params(cfg.obs_shape, "mlp", seed=1)
    pol = B200Policy(params, cfg.obs_shape, 2, seats=(0,))
    for i, t in enumerate(g["obs_ticks"][:8]):
        obs = _padded(g["obs"][i])
        mm = torch.from_numpy(g["mm"][t]).cuda()
        bm = torch.from_numpy(g["bm"][t]).cuda()
        u = torch.from_numpy(g["u_net"][t][:, 0].astype(np.float32)).cuda().view(1, -1, 2)
        logits, acts, logp = pol.forward_logits(obs, mm, bm, u)
        lg = logits[0].cpu().numpy()
        assert _rel(lg[:, :5], g["logits_m"][t][:, 0]) <= REL_TOL
        assert _rel(lg[:, 5:7], g["logits_b"][t][:, 0]) <= REL_TOL
        assert _rel(lg[:, 7], g["value"][t][:, 0]) <= REL_TOL
        assert np.array_equal(acts[0].cpu().numpy(), g["actions"][t][:, 0])
        assert np.abs(logp[0].cpu().numpy() - g["logp"][t][:, 0]).max() <= 1e-4


@pytest.mark.parametrize("seats", [(0,), (1,), (0, 1)])
def test_mlp_full_size_vs_oracle(seats):
    cfg = SimConfig(**scenarios.CFG2)
    n, p = 5632, 2
    rng = np.random.default_rng(7)
    c, h, w = cfg.obs_shape
    obs16 = (rng.random((n, c, h, w)) * (rng.random((n, c, h, w)) < 0.3)).astype(np.float16)
    mm = rng.random((n, p, 5)) < 0.8
    mm[..., 4] = True
    bm = rng.random((n, p, 2)) < 0.7
    bm[..., 0] = True
    params = init_params(cfg.obs_shape, "mlp", seed=3)
    pol = B200Policy(params, cfg.obs_shape, p, seats=seats)
    u = rng.random((len(seats), n, 2)).astype(np.float32)
    logits, acts, logp = pol.forward_logits(_padded(obs16), torch.from_numpy(mm).cuda(),
                                            torch.from_numpy(bm).cuda(), torch.from_numpy(u).cuda())
    lg = logits.cpu().numpy()
    for s, pid in enumerate(seats):
        ml, bl, v = O.mlp_forward(params, obs16.astype(np.float32), pid, p)
        assert _rel(lg[s, :, :5], ml) <= REL_TOL, _rel(lg[s, :, :5], ml)
        assert _rel(lg[s, :, 5:7], bl) <= REL_TOL
        assert _rel(lg[s, :, 7], v) <= REL_TOL
        a, lp, _, _, _ = O.mlp_act(params, obs16.astype(np.float32), mm[:, pid], bm[:, pid], pid,
                                   p, u[s, :, 0], u[s, :, 1])
        mismatch = int((acts[s].cpu().numpy() != a).any(-1).sum())
        assert mismatch == 0, f"{mismatch} sampled actions differ"
        assert np.abs(logp[s].cpu().numpy() - lp).max() <= 1e-3


def test_mlp_ragged_tail_and_small_batch():
    cfg = SimConfig(**scenarios.CFG2)
    p = 2
    params = init_params(cfg.obs_shape, "mlp", seed=5)
    pol = B200Policy(params, cfg.obs_shape, p, seats=(0,))
    rng = np.random.default_rng(11)
    for n in (1, 37, 129, 300):
        obs16 = rng.random((n,) + cfg.obs_shape).astype(np.float16)
        mm = np.ones((n, p, 5), bool)
        bm = np.ones((n, p, 2), bool)
        logits, _, _ = pol.forward_logits(_padded(obs16), torch.from_numpy(mm).cuda(),
                                          torch.from_numpy(bm).cuda())
        ml, _, v = O.mlp_forward(params, obs16.astype(np.float32), 0, p)
        assert _rel(logits[0, :, :5].cpu().numpy(), ml) <= REL_TOL
        assert _rel(logits[0, :, 7].cpu().numpy(), v) <= REL_TOL


@pytest.mark.parametrize("n,seats", [(2100, (0, 1)), (2200, (0, 1)), (2433, (0, 1)),
                                     (2100, (0,))])
def test_mlp_pair_batches_with_ragged_pairs(n, seats):
    # two-seat batches above 16 row tiles run on SM pairs: an odd tile count
    # leaves the last pair's second CTA past the end, a ragged count cuts a
    # tile (one seat: the single-CTA kernel at the same sizes)
    cfg = SimConfig(**scenarios.CFG2)
    p = 2
    rng = np.random.default_rng(n)
    obs16 = (rng.random((n,) + cfg.obs_shape) * (rng.random((n,) + cfg.obs_shape) < 0.3)
             ).astype(np.float16)
    mm = rng.random((n, p, 5)) < 0.8
    mm[..., 4] = True
    bm = rng.random((n, p, 2)) < 0.7
    bm[..., 0] = True
    params = init_params(cfg.obs_shape, "mlp", seed=9)
    pol = B200Policy(params, cfg.obs_shape, p, seats=seats)
    u = rng.random((len(seats), n, 2)).astype(np.float32)
    logits, acts, logp = pol.forward_logits(_padded(obs16), torch.from_numpy(mm).cuda(),
                                            torch.from_numpy(bm).cuda(), torch.from_numpy(u).cuda())
    lg = logits.cpu().numpy()
    for s, pid in enumerate(seats):
        ml, bl, v = O.mlp_forward(params, obs16.astype(np.float32), pid, p)
        assert _rel(lg[s, :, :5], ml) <= REL_TOL and _rel(lg[s, :, 5:7], bl) <= REL_TOL
        assert _rel(lg[s, :, 7], v) <= REL_TOL
        a, lp, _, _, _ = O.mlp_act(params, obs16.astype(np.float32), mm[:, pid], bm[:, pid], pid,
                                   p, u[s, :, 0], u[s, :, 1])
        assert int((acts[s].cpu().numpy() != a).any(-1).sum()) == 0
        assert np.abs(logp[s].cpu().numpy() - lp).max() <= 1e-3


@pytest.mark.parametrize("n,seats", [(5632, (0,)), (300, (0,)), (2100, (0, 1)), (2433, (0, 1)),
                                     (1000, (0, 1))])
def test_mlp_zero_tile_skip_is_bit_identical(n, seats):
    # rows with whole 64-entry K tiles zero in some 128-row tiles (and in
    # single rows): with the rows' K-tile flags the first layer skips the
    # tiles that are zero in every row of a row tile (one CTA, the split-K
    # cluster at 300 rows and 1000 two-seat rows, SM pairs at 2100 / 2433);
    # outputs must equal the unflagged pass bit for bit.  Over-reported
    # flags (all set) change nothing either.
    from qqt_b200.sim import tile_flags
    cfg = SimConfig(**scenarios.CFG2)
    p = 2
    rng = np.random.default_rng(n + len(seats))
    c, h, w = cfg.obs_shape
    k = c * h * w
    kt = (k + 63) // 64
    obs16 = (rng.random((n, k)) * (rng.random((n, k)) < 0.3)).astype(np.float16)
    for r0 in range(0, n, 128):
        for t in np.flatnonzero(rng.random(kt) < 0.45):
            obs16[r0:r0 + 128, 64 * t:64 * t + 64] = 0
    for i in rng.choice(n, size=n // 10, replace=False):
        obs16[i, 64 * rng.integers(kt):][:64] = 0
    obs = _padded(obs16.reshape((n,) + cfg.obs_shape))
    flags = tile_flags(torch.as_strided(obs, (n, obs.stride(0)), (obs.stride(0), 1)))
    mm = rng.random((n, p, 5)) < 0.8
    mm[..., 4] = True
    bm = rng.random((n, p, 2)) < 0.7
    bm[..., 0] = True
    mm, bm = torch.from_numpy(mm).cuda(), torch.from_numpy(bm).cuda()
    params = init_params(cfg.obs_shape, "mlp", seed=13)
    pol = B200Policy(params, cfg.obs_shape, p, seats=seats)
    u = torch.from_numpy(rng.random((len(seats), n, 2)).astype(np.float32)).cuda()
    base = pol.forward_logits(obs, mm, bm, u)
    for fl in (flags, torch.full_like(flags, -1)):
        got = pol.forward_logits(obs, mm, bm, u, obs_tiles=fl)
        assert torch.equal(got[0], base[0]), "logits differ with K-tile flags"
        for a, b in zip(got[1], base[1]):
            assert torch.equal(a, b)
        assert torch.equal(got[2], base[2])
    ml, _, v = O.mlp_forward(params, obs16.reshape((n,) + cfg.obs_shape).astype(np.float32),
                             seats[0], p)
    assert _rel(base[0][0, :, :5].cpu().numpy(), ml) <= REL_TOL
    assert _rel(base[0][0, :, 7].cpu().numpy(), v) <= REL_TOL


def test_mlp_all_zero_rows_with_clear_flags():
    # every flag clear (rows all zero): the first K tile still runs, so the
    # layer-1 accumulators are written and the output is the bias path's
    cfg = SimConfig(**scenarios.CFG2)
    n, p = 300, 2
    obs = _padded(np.zeros((n,) + cfg.obs_shape, np.float16))
    mm = torch.ones((n, p, 5), dtype=torch.bool, device="cuda")
    bm = torch.ones((n, p, 2), dtype=torch.bool, device="cuda")
    pol = B200Policy(init_params(cfg.obs_shape, "mlp", seed=4), cfg.obs_shape, p, seats=(0,))
    u = torch.rand((1, n, 2), device="cuda")
    base = pol.forward_logits(obs, mm, bm, u)
    got = pol.forward_logits(obs, mm, bm, u,
                             obs_tiles=torch.zeros((n, 4), dtype=torch.int32, device="cuda"))
    assert torch.equal(got[0], base[0]) and torch.equal(got[2], base[2])


def test_cnn_logits_vs_reference_goldens():
    g = G.load("traj_cfg5")
    cfg = SimConfig(**scenarios.CFG2)
    params = init_params(cfg.obs_shape, "cnn", seed=3)
    pol = B200Policy(params, cfg.obs_shape, 2, seats=(0,), arch="cnn")
    for i, t in enumerate(g["obs_ticks"]):
        obs = _padded(g["obs"][i])
        mm = torch.from_numpy(g["mm"][t]).cuda()
        bm = torch.from_numpy(g["bm"][t]).cuda()
        u = torch.from_numpy(g["u_net"][t][:, 0].astype(np.float32)).cuda().view(1, -1, 2)
        logits, acts, logp = pol.forward_logits(obs, mm, bm, u)
        lg = logits[0].cpu().numpy()
        assert _rel(lg[:, :5], g["logits_m"][t][:, 0]) <= REL_TOL
        assert _rel(lg[:, 5:7], g["logits_b"][t][:, 0]) <= REL_TOL
        assert _rel(lg[:, 7], g["value"][t][:, 0]) <= REL_TOL
        assert np.array_equal(acts[0].cpu().numpy(), g["actions"][t][:, 0])


@pytest.mark.parametrize("seats", [(0,), (0, 1)])
def test_cnn_vs_oracle(seats):
    cfg = SimConfig(**scenarios.CFG2)
    n, p = 300, 2
    rng = np.random.default_rng(17)
    shp = (n,) + tuple(cfg.obs_shape)
    obs16 = (rng.random(shp) * (rng.random(shp) < 0.3)).astype(np.float16)
    mm = np.ones((n, p, 5), bool)
    bm = np.ones((n, p, 2), bool)
    params = init_params(cfg.obs_shape, "cnn", seed=4)
    pol = B200Policy(params, cfg.obs_shape, p, seats=seats, arch="cnn")
    logits, _, _ = pol.forward_logits(_padded(obs16), torch.from_numpy(mm).cuda(),
                                      torch.from_numpy(bm).cuda())
    lg = logits.cpu().numpy()
    for s, pid in enumerate(seats):
        ml, bl, v = O.cnn_forward(params, obs16.astype(np.float32), pid, p)
        assert _rel(lg[s, :, :5], ml) <= REL_TOL
        assert _rel(lg[s, :, 5:7], bl) <= REL_TOL
        assert _rel(lg[s, :, 7], v) <= REL_TOL
