"""The allocation-free step entry point (qqt_step_noalloc).

It serves callers that cannot allocate device memory -- code running inside
another runtime's stream capture, or embeddings that hand this library only
pre-placed buffers -- by keeping the step's scratch in a static device array.
This test calls it through the C ABI and checks its results against the
regular qqt_step (which takes a caller-allocated scratch buffer) on
identical states, for two calls in a row that both use the scratch
(first_step = 1).  Collected last on purpose: it must pass both alone in a
fresh process and after every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _pair(n):
    from qqt_b200 import scenarios
    from qqt_b200.config import SimConfig
    from qqt_b200.sim import B200Sim
    import __graft_entry__ as ge
    cfg = SimConfig(**scenarios.CFG2)
    tm = ge._template_state(cfg, n, 3)
    a = B200Sim(cfg, n, device="cuda", seed=3, template=tm)
    b = B200Sim(cfg, n, device="cuda", seed=3, template=tm)
    return cfg, a, b


def _call(sim, fn, acts, rb):
    from qqt_b200 import _capi as capi
    args = [ctypes.byref(sim._ccfg), ctypes.byref(sim._cstate), acts.data_ptr(),
            rb[0].data_ptr(), rb[1].data_ptr(), sim._tiers.data_ptr(), 1,
            ctypes.byref(sim._cout), None]
    if fn == "qqt_step":
        rc = capi.lib().qqt_step(*args, sim._step_scratch.data_ptr(), sim._stream())
    else:
        rc = capi.lib().qqt_step_noalloc(*args, sim._stream())
    capi.check(rc, fn)


def test_step_noalloc_matches_step_twice():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from qqt_b200 import _capi as capi
    n = 1000
    cfg, a, b = _pair(n)
    p = cfg.n_players
    g = torch.Generator(device="cuda").manual_seed(5)
    for call in range(2):
        acts = torch.stack([torch.randint(0, 5, (n, p), device="cuda", generator=g),
                            torch.randint(0, 2, (n, p), device="cuda", generator=g)], -1)
        rb = (torch.rand((n, p), device="cuda", generator=g),
              torch.rand((n, p), device="cuda", generator=g))
        _call(a, "qqt_step", acts, rb)
        ra = a._reward.clone()
        da = a._done.clone()
        _call(b, "qqt_step_noalloc", acts, rb)
        torch.cuda.synchronize()
        assert torch.allclose(ra, b._reward, atol=1e-6, rtol=0), f"call {call}: rewards"
        assert torch.equal(da, b._done), f"call {call}: done"
        sa, sb = a.numpy_state(), b.numpy_state()
        for k in sa:
            assert np.array_equal(sa[k], sb[k]), f"call {call}: state {k}"
        assert int(a._tiers.item()) == int(b._tiers.item())
    assert capi.device_error() == 0


def test_step_noalloc_rejects_oversize():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from qqt_b200 import _capi as capi
    from qqt_b200.sim import make_ccfg
    from qqt_b200 import scenarios
    from qqt_b200.config import SimConfig
    c = make_ccfg(SimConfig(**scenarios.CFG2), 200000, 1.0)   # 400000 > 262144
    st = capi.QqtState()
    rc = capi.lib().qqt_step_noalloc(ctypes.byref(c), ctypes.byref(st), None, None, None, None,
                                     1, None, None, None)
    assert rc == 3   # QQT_E_LIMIT, before touching any pointer
