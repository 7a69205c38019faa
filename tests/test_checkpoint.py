"""Checkpoint format and first-layer migration (train/train.py:92-158,
243-260, 307-331).

CPU: the migration against the reference's adapt_first_conv outputs
(tests/golden/ckpt_adapt.npz, bit-exact), a checkpoint written by the
reference's own save_ckpt (tests/golden/ref_ckpt_mlp.pt) read back, and the
round trip of this package's writer.  GPU: a saved checkpoint loads into the
B200 policy and acts like the float64 oracle on the same parameters.
"""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from qqt_b200 import checkpoint as C
from qqt_b200.policy_init import init_params, mlp_param_shapes

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")
REF_KEYS = {"format_version", "model", "obs_shape", "n_players", "arch", "opt", "pool",
            "fixed_elo", "curriculum", "global_step", "elo", "args", "torch_rng", "py_rng"}


def _golden():
    return np.load(os.path.join(GOLD, "ckpt_adapt.npz"))


@pytest.mark.parametrize("arch", ["mlp", "cnn"])
@pytest.mark.parametrize("p_old,p_new", [(2, 3), (3, 2)])
def test_adapt_first_layer_matches_reference(arch, p_old, p_new):
    g = _golden()
    tag = f"{arch}_{p_old}to{p_new}"
    first = C.FIRST_LAYER[arch]
    old_shape = (2 * p_old + 3 + C.obs_extra(p_old), 3, 3)
    new_shape = (2 * p_new + 3 + C.obs_extra(p_new), 3, 3)
    old = {first: torch.from_numpy(g[f"{tag}__old"])}
    out = C.adapt_first_layer(old, old_shape, new_shape, arch, p_old, p_new)
    assert np.array_equal(out[first].numpy(), g[f"{tag}__new"])
    assert out[first].dtype == torch.float32


def test_adapt_keeps_other_keys_and_same_shape():
    params = {k: torch.randn(v) for k, v in mlp_param_shapes((14, 3, 3)).items()}
    same = C.adapt_first_layer(params, (14, 3, 3), (14, 3, 3), "mlp")
    assert all(torch.equal(same[k], params[k]) for k in params)
    new = {k: torch.zeros(v) for k, v in mlp_param_shapes((19, 3, 3)).items()}
    out = C.adapt_first_layer(params, (14, 3, 3), (19, 3, 3), "mlp", new_state=new)
    g = _golden()
    assert sorted(out.keys()) == list(g["mlp_2to3__keys"])
    for k in params:
        if k != "shared.0.weight":
            assert torch.equal(out[k], params[k])


def test_reference_written_checkpoint_loads():
    ck = C.load_ckpt(os.path.join(GOLD, "ref_ckpt_mlp.pt"))
    assert set(ck) == REF_KEYS
    assert ck["arch"] == "mlp" and tuple(ck["obs_shape"]) == (14, 3, 3) and ck["n_players"] == 2
    shapes = mlp_param_shapes((14, 3, 3))
    assert set(ck["model"]) == set(shapes)
    for k, v in ck["model"].items():
        assert tuple(v.shape) == shapes[k] and v.dtype == torch.float32
    assert ck["curriculum"] == {"stage_idx": 2, "episodes_in_stage": 37,
                                "recent_wins": [1.0, 0.0, 0.5]}
    assert ck["global_step"] == 12345 and ck["elo"] == 1012.5


def test_save_round_trip_and_reference_keys(tmp_path):
    ref = C.load_ckpt(os.path.join(GOLD, "ref_ckpt_mlp.pt"))
    params = init_params((14, 13, 13), "mlp", seed=2)
    path = str(tmp_path / "sub" / "ck.pt")
    C.save_ckpt(path, model=params, obs_shape=(14, 13, 13), n_players=2, arch="mlp",
                global_step=77, elo=1003.0, fixed_elo={"astar": 1001.0},
                curriculum={"stage_idx": 1, "episodes_in_stage": 5, "recent_wins": [0.5]},
                args={"arch": "mlp"})
    assert not os.path.exists(path + ".tmp")
    ck = C.load_ckpt(path)
    assert set(ck) == set(ref)
    for k in ref:
        assert type(ck[k]) is type(ref[k]) or k == "model", k
    assert set(ck["pool"]) == set(ref["pool"]) and set(ck["curriculum"]) == set(ref["curriculum"])
    for k, v in params.items():
        assert np.array_equal(ck["model"][k].numpy(), v)
    assert ck["global_step"] == 77 and ck["fixed_elo"] == {"astar": 1001.0}


def test_old_format_rejected(tmp_path):
    path = str(tmp_path / "old.pt")
    torch.save({"format_version": 1, "model": {}}, path)
    with pytest.raises(ValueError):
        C.load_ckpt(path)


def test_infer_players():
    assert C.infer_players(14) == 2 and C.infer_players(19) == 3 and C.infer_players(7) == 2


@pytest.mark.gpu
def test_checkpoint_policy_acts_like_oracle(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from oracle import qqt_oracle as O
    from qqt_b200 import _capi
    shape = (14, 13, 13)
    params = init_params(shape, "mlp", seed=9)
    path = str(tmp_path / "ck.pt")
    C.save_ckpt(path, model=params, obs_shape=shape, n_players=2, arch="mlp")
    pol = C.load_policy(path, device="cuda", seats=(1,))
    n = 300
    rng = np.random.default_rng(3)
    obs16 = (rng.random((n,) + shape) * (rng.random((n,) + shape) < 0.3)).astype(np.float16)
    rows = torch.zeros((n, 2368), dtype=torch.float16, device="cuda")
    rows[:, :2366] = torch.from_numpy(obs16.reshape(n, -1)).cuda()
    obs = rows[:, :2366].view((n,) + shape)
    mm = torch.ones((n, 2, 5), dtype=torch.bool, device="cuda")
    bm = torch.ones((n, 2, 2), dtype=torch.bool, device="cuda")
    logits, _, _ = pol.forward_logits(obs, mm, bm)
    torch.cuda.synchronize()
    assert _capi.device_error() == 0
    ml, bl, v = O.mlp_forward(params, obs16.astype(np.float32), 1, 2)
    lg = logits[0].cpu().numpy()
    for got, want in ((lg[:, :5], ml), (lg[:, 5:7], bl), (lg[:, 7], v)):
        assert np.abs(got - want).max() / np.abs(want).max() <= 2e-3


@pytest.mark.parametrize("p_old,p_new", [(2, 3), (3, 2)])
def test_adapt_first_layer_lstm_matches_reference(p_old, p_new):
    """The LSTM's local CNN takes the observation channels in view order:
    l_conv1.weight migrates like conv0 (train/train.py:140-147), bit-exact
    to the reference's adapt_first_conv (tests/golden/ckpt_adapt_lstm.npz)."""
    g = np.load(os.path.join(GOLD, "ckpt_adapt_lstm.npz"))
    tag = f"lstm_{p_old}to{p_new}"
    old_shape = (2 * p_old + 3 + C.obs_extra(p_old), 13, 13)
    new_shape = (2 * p_new + 3 + C.obs_extra(p_new), 13, 13)
    old = {"l_conv1.weight": torch.from_numpy(g[f"{tag}__old"])}
    out = C.adapt_first_layer(old, old_shape, new_shape, "lstm", p_old, p_new)
    assert np.array_equal(out["l_conv1.weight"].numpy(), g[f"{tag}__new"])


def test_unsupported_arch_errors(tmp_path):
    with pytest.raises(ValueError, match="unsupported arch"):
        C.adapt_first_layer({}, (14, 3, 3), (19, 3, 3), "transformer")
    path = str(tmp_path / "lstm.pt")
    C.save_ckpt(path, model={"l_conv1.weight": torch.zeros(32, 14, 3, 3)}, obs_shape=(14, 13, 13),
                n_players=2, arch="lstm")
    assert C.load_ckpt(path)["arch"] == "lstm"
    with pytest.raises(ValueError, match="B200Policy runs"):
        C.load_policy(path, device="cpu")
