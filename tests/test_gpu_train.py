"""The PPO update's first-layer kernels (csrc/train_mlp.cu) against float64
references of the same products (train/model.py:121-153, train/ppo.py:364-437).

qqt_gather_rows is compared bit for bit with torch indexing; qqt_l1_forward
and qqt_l1_wgrad (through the autograd function the update uses) with the
float64 product of the same float16 rows and float32 weights, for both seats'
view permutations, ragged row counts (a partial last tile, several tiles per
persistent CTA) and gradients spread over twelve decades.  The whole
MLPActorCritic.evaluate on the device is compared with its CPU restatement.
"""

from __future__ import annotations

import pytest
import torch

from qqt_b200.ppo import MLPActorCritic, _Layer1, gather_rows, inv_cols, obs_rows

pytestmark = pytest.mark.gpu

SHAPE = (14, 13, 13)
K_IN = 14 * 169


def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _rows(n, seed, stride=2368):
    g = torch.Generator().manual_seed(seed)
    x = torch.rand((n, K_IN), generator=g)
    x = torch.where(torch.rand((n, K_IN), generator=g) < 0.3, x, torch.zeros(()))
    rows = torch.zeros((n, stride), dtype=torch.float16)
    rows[:, :K_IN] = x.half()
    return rows.cuda()


def _weights(seed):
    g = torch.Generator().manual_seed(seed)
    w0 = (torch.randn((128, K_IN), generator=g) * 0.02).cuda()
    b0 = (torch.randn(128, generator=g) * 0.1).cuda()
    return w0, b0


def test_gather_rows_bit_exact():
    _need_cuda()
    from qqt_b200 import _capi
    src = _rows(1000, 1)
    idx = torch.randint(0, 1000, (777,), device="cuda")
    idx[5] = 999
    idx[6] = 0
    out = gather_rows(src, idx)
    torch.cuda.synchronize()
    assert torch.equal(out, src[idx])
    assert _capi.device_error() == 0


@pytest.mark.parametrize("row_bytes", [16, 48, 112, 4736])
def test_gather_rows_small_rows_bit_exact(row_bytes):
    """Several rows per warp for short rows (the packed per-row side data)."""
    _need_cuda()
    from qqt_b200 import _capi
    src = torch.randint(0, 256, (3001, row_bytes), dtype=torch.uint8, device="cuda")
    idx = torch.randint(0, 3001, (2049,), device="cuda")
    out = gather_rows(src, idx)
    torch.cuda.synchronize()
    assert torch.equal(out, src[idx])
    assert _capi.device_error() == 0


def test_gather_rows_bad_index_flags_and_zero_fills():
    _need_cuda()
    from qqt_b200 import _capi
    src = _rows(64, 2)
    idx = torch.tensor([3, 64, -1, 7], device="cuda")
    out = gather_rows(src, idx)
    torch.cuda.synchronize()
    assert _capi.device_error() == 1 << 4   # QQT_DEV_BAD_INDEX
    assert torch.equal(out[0], src[3]) and torch.equal(out[3], src[7])
    assert not out[1].any() and not out[2].any()


@pytest.mark.parametrize("n", [1, 300, 37965])
@pytest.mark.parametrize("pid", [0, 1])
def test_l1_forward_and_wgrad_match_float64(n, pid):
    _need_cuda()
    from qqt_b200 import _capi
    rows = _rows(n, 10 + n)
    w0, b0 = _weights(3 + pid)
    w0p = w0[:, inv_cols(2, 14, 13, 13, pid).cuda()]
    w0.requires_grad_(True)
    b0.requires_grad_(True)
    h1 = _Layer1.apply(rows, w0, b0, K_IN, (2, 14, 169, pid))
    x64 = rows[:, :K_IN].double()
    ref = x64 @ w0p.detach().double().T + b0.detach().double()
    err = (h1.double() - ref).abs().max().item()
    assert err <= 1e-5 * max(1.0, ref.abs().max().item()), err
    # gradients over twelve decades of magnitude
    g = torch.Generator().manual_seed(7 + n)
    dh = torch.randn((n, 128), generator=g) * torch.pow(10.0, -12 * torch.rand((n, 128), generator=g))
    dh = (dh * 1e-3).cuda()
    h1.backward(dh)
    torch.cuda.synchronize()
    assert _capi.device_error() == 0
    gp = dh.double().T @ x64                                   # gradient of the permuted W0
    ref_w = torch.zeros_like(gp)
    ref_w[:, inv_cols(2, 14, 13, 13, pid).cuda()] = gp
    scale = ref_w.abs().max().item()
    err_w = (w0.grad.double() - ref_w).abs().max().item()
    assert err_w <= 1e-5 * scale, (err_w, scale)
    # db0 is torch's float32 column sum (as in the reference's autograd)
    db_err = (b0.grad.double() - dh.double().sum(0)).abs().max().item()
    assert db_err <= 1e-5 * dh.double().abs().sum(0).max().item()


def test_zero_gradient_is_exact_zero():
    _need_cuda()
    rows = _rows(200, 4)
    w0, b0 = _weights(5)
    w0.requires_grad_(True)
    h1 = _Layer1.apply(rows, w0, b0, K_IN, (2, 14, 169, 0))
    h1.backward(torch.zeros_like(h1))
    torch.cuda.synchronize()
    assert not w0.grad.any()


def _away_from_kinks(m, obs4, pid, rel=1e-4):
    """Rows whose ReLU inputs (after LN1, LN2 and in the head hidden layers)
    all lie farther than rel x their layer's scale from zero, in float64: a
    pre-activation within rounding of zero may take the other side of the
    kink in a float32 implementation, which changes that row's gradient by
    a finite amount.  The loss weights the remaining rows only."""
    with torch.no_grad():
        p = {k: v.double() for k, v in m.state_dict().items()}
        x = obs4.reshape(obs4.shape[0], -1).double()
        w0 = p["shared.0.weight"][:, getattr(m, f"inv_cols_{pid}")]
        h = x @ w0.T + p["shared.0.bias"]
        a1 = torch.nn.functional.layer_norm(h, (128,), p["shared.1.weight"], p["shared.1.bias"])
        h = a1.clamp(min=0) @ p["shared.3.weight"].T + p["shared.3.bias"]
        a2 = torch.nn.functional.layer_norm(h, (128,), p["shared.4.weight"], p["shared.4.bias"])
        r2 = a2.clamp(min=0)
        gs = [r2 @ p[f"{hd}.0.weight"].T + p[f"{hd}.0.bias"]
              for hd in ("move_head", "bomb_head", "critic")]
        keep = torch.ones(x.shape[0], dtype=torch.bool)
        for t in [a1, a2] + gs:
            keep &= (t.abs() > rel * t.abs().max()).all(1)
        return keep


@pytest.mark.parametrize("n", [1, 520, 20000, 40000])
def test_evaluate_on_device_matches_cpu_restatement(n):
    """The fused training forward, the two tail backward kernels and the
    first layer's weight gradient against torch autograd on the CPU."""
    _need_cuda()
    from qqt_b200 import _capi
    torch.manual_seed(0)
    m_cpu = MLPActorCritic(SHAPE, 2)
    with torch.no_grad():
        for p in m_cpu.parameters():      # LayerNorm affine and biases away from 1 / 0
            p.add_(torch.randn_like(p) * 0.05)
    m_gpu = MLPActorCritic(SHAPE, 2).cuda()
    m_gpu.load_state_dict(m_cpu.state_dict())
    rows = _rows(n, 11)
    obs4 = rows[:, :K_IN].cpu().view(n, *SHAPE)
    mm = torch.rand((n, 5)) < 0.8
    mm[:, 4] = True
    bm = torch.rand((n, 2)) < 0.7
    bm[:, 0] = True
    act = torch.stack([torch.multinomial(mm.float(), 1)[:, 0],
                       torch.multinomial(bm.float(), 1)[:, 0]], -1)
    for pid in (0, 1):
        keep = _away_from_kinks(m_cpu, obs4, pid)
        assert keep.float().mean() > 0.5
        wl = torch.linspace(-1, 1, n) * keep
        outs = []
        for m, dev, ob in ((m_cpu, "cpu", obs4), (m_gpu, "cuda", rows)):
            m.zero_grad()
            logp, ent, v = m.evaluate(ob, mm.to(dev), bm.to(dev), act.to(dev), pid)
            k = keep.to(dev).float()
            loss = -(logp * wl.to(dev)).mean() + 0.5 * (v * v * k).mean() - 0.03 * (ent * k).mean()
            loss.backward()
            outs.append({"logp": logp.detach().cpu(), "v": v.detach().cpu(),
                         "ent": ent.detach().cpu(),
                         **{k: p.grad.detach().cpu() for k, p in m.named_parameters()}})
        torch.cuda.synchronize()
        assert _capi.device_error() == 0
        for k in outs[0]:
            a, b = outs[0][k].double(), outs[1][k].double()
            # outputs to 1e-5 of their largest entry, but never tighter than
            # 1e-6 absolute (float32 sums of O(1) terms in different orders:
            # one row's value can be ~5e-3 itself); gradients (float32 sums
            # over the batch, in different orders on the two devices) to 5e-5
            # of their largest entry
            out = k in ("logp", "v", "ent")
            tol = (1e-5 if out else 5e-5) * max(1e-30, a.abs().max().item())
            tol = max(tol, 1e-6 if out else 1e-12)
            assert (a - b).abs().max().item() <= tol, (k, (a - b).abs().max().item(), tol)


def test_obs_rows_pads_four_dimensional_batches():
    x = (torch.rand((3,) + SHAPE) < 0.5).half()
    r = obs_rows(x, K_IN)
    assert r.shape == (3, 2368) and torch.equal(r[:, :K_IN], x.reshape(3, -1))
    assert not r[:, K_IN:].any()
    with pytest.raises(TypeError):
        obs_rows(x.float(), K_IN)


@pytest.mark.parametrize("n", [77, 3000])
def test_gathered_rows_read_in_place_equal_pre_gathered(n):
    """rows_idx: the training forward and the weight-gradient GEMM read the
    minibatch's rows of the row buffer in place (TMA gather4); outputs and
    every gradient equal the pre-gathered path bit for bit.  Invalid ids read
    row 0 and raise QQT_DEV_BAD_INDEX."""
    _need_cuda()
    from qqt_b200 import _capi
    torch.manual_seed(1)
    m = MLPActorCritic(SHAPE, 2).cuda()
    src = _rows(5000, 21)
    idx = torch.randint(0, 5000, (n,), device="cuda")
    mm = torch.rand((n, 5), device="cuda") < 0.8
    mm[:, 4] = True
    bm = torch.rand((n, 2), device="cuda") < 0.7
    bm[:, 0] = True
    act = torch.stack([torch.multinomial(mm.float(), 1)[:, 0],
                       torch.multinomial(bm.float(), 1)[:, 0]], -1)
    w = torch.linspace(-1, 1, n, device="cuda")

    def run(x, rows_idx):
        m.zero_grad()
        logp, ent, v = m.evaluate(x, mm, bm, act, 1, rows_idx=rows_idx)
        (-(logp * w).mean() + 0.5 * (v * v).mean() - 0.03 * ent.mean()).backward()
        return [logp.detach(), ent.detach(), v.detach()] + [p.grad.clone() for p in m.parameters()]

    ref = run(src[idx], None)
    got = run(src, idx)
    torch.cuda.synchronize()
    assert _capi.device_error() == 0
    for a, b in zip(ref, got):
        assert torch.equal(a, b)
    bad = idx.clone()
    bad[0], bad[-1] = -1, 5000
    fixed = bad.clamp(0, 4999)
    fixed[0] = fixed[-1] = 0
    ref = run(src[fixed], None)
    got = run(src, bad)
    torch.cuda.synchronize()
    assert _capi.device_error() == 1 << 4
    for a, b in zip(ref, got):
        assert torch.equal(a, b)
