"""Failure detection without a GPU fault (host side, CPU only).

* The C-ABI entry points reject bad arguments on the host before any CUDA
  call: null pointers and impossible sizes (QQT_E_ARG), grids or player
  counts above the compiled limits (QQT_E_LIMIT), misaligned pointers or
  strides (QQT_E_ALIGN); `_capi.check` turns a non-zero status into an
  exception naming the call.  The pointers given here are never
  dereferenced: every case returns at validation.
* The PPO update's one collective (the gradient all-reduce over every
  rank's shard) ends with an error, not a hang, when a peer rank dies
  between steps: two gloo ranks with a short process-group timeout, rank 1
  exits, rank 0's all-reduce raises.
"""

from __future__ import annotations

import ctypes
import os

import pytest

from qqt_b200 import _capi
from qqt_b200.config import SimConfig
from qqt_b200 import scenarios

E_ARG, E_ALIGN, E_LIMIT = 1, 2, 3
FAKE = 0x100000            # a 256-byte aligned address that is never dereferenced


def _cfg(**kw):
    from qqt_b200.sim import make_ccfg
    cfg = SimConfig(**{**scenarios.CFG2, **kw})
    return make_ccfg(cfg, 64, 1.0)


def test_config_validation_codes():
    L = _capi.lib()
    state = _capi.QqtState()
    assert L.qqt_observe(None, ctypes.byref(state), None, None, None, None, None) == E_ARG
    c = _cfg()
    c.n_envs = 0
    assert L.qqt_observe(ctypes.byref(c), ctypes.byref(state), None, None, None, None,
                         None) == E_ARG
    c = _cfg()
    c.height = 99
    assert L.qqt_observe(ctypes.byref(c), ctypes.byref(state), None, None, None, None,
                         None) == E_LIMIT
    c = _cfg()
    c.n_players = 9
    assert L.qqt_observe(ctypes.byref(c), ctypes.byref(state), None, None, None, None,
                         None) == E_LIMIT
    # a valid config with a missing state pointer, actions or scratch
    c = _cfg()
    assert L.qqt_step(ctypes.byref(c), None, FAKE, FAKE, FAKE, FAKE, 0, None, None, FAKE,
                      None) == E_ARG
    assert L.qqt_step(ctypes.byref(c), ctypes.byref(state), None, FAKE, FAKE, FAKE, 0, None,
                      None, FAKE, None) == E_ARG
    assert L.qqt_local_view(ctypes.byref(c), ctypes.byref(state), FAKE, 0, 0, FAKE, FAKE, FAKE,
                            None) == E_ARG


def test_training_entry_points_reject_bad_arguments():
    L = _capi.lib()
    # row gather: null, misaligned source, row longer than the stride
    assert L.qqt_gather_rows(None, 10, 4736, FAKE, 5, FAKE, 4736, 4736, None) == E_ARG
    assert L.qqt_gather_rows(FAKE + 8, 10, 4736, FAKE, 5, FAKE, 4736, 4736, None) == E_ALIGN
    assert L.qqt_gather_rows(FAKE, 10, 4736, FAKE, 5, FAKE, 4736, 9472, None) == E_ARG
    # first layer: empty batch, stride not a multiple of 8, misaligned output
    assert L.qqt_l1_forward(FAKE, FAKE, 0, 2368, 2366, FAKE, FAKE, None) == E_ARG
    assert L.qqt_l1_forward(FAKE, FAKE, 10, 2367, 2366, FAKE, FAKE, None) == E_ALIGN
    assert L.qqt_l1_forward(FAKE, FAKE, 10, 2368, 2366, FAKE, FAKE + 4, None) == E_ALIGN
    # weight gradient: k_in inconsistent with channels x cells, then a bad seat
    assert L.qqt_l1_wgrad(FAKE, 10, 2368, 2366, None, 0, FAKE, 2, 14, 170, 0, FAKE, FAKE,
                          None) == E_ARG
    assert L.qqt_l1_wgrad(FAKE, 10, 2368, 2366, None, 0, FAKE, 2, 14, 169, 5, FAKE, FAKE,
                          None) == E_ARG
    # fused training forward / tail backward: missing outputs, too-short mask rows
    assert L.qqt_mlp_train_forward(FAKE, FAKE, 10, 2368, 2366, None, 0, FAKE, 5, FAKE, 2, FAKE,
                                   2, FAKE, FAKE, FAKE, None, FAKE, None) == E_ARG
    assert L.qqt_mlp_train_forward(FAKE, FAKE, 10, 2368, 2366, None, 0, FAKE, 4, FAKE, 2, FAKE,
                                   2, FAKE, FAKE, FAKE, FAKE, FAKE, None) == E_ARG
    grads = (ctypes.c_void_p * 20)(*([FAKE] * 20))
    grads[7] = None
    assert L.qqt_mlp_train_backward(FAKE, 10, 2366, FAKE, FAKE, FAKE, 5, FAKE, 2, FAKE, 2,
                                    FAKE, grads, FAKE, FAKE, None) == E_ARG


def test_check_names_the_failed_call():
    with pytest.raises(RuntimeError, match="qqt_demo failed: misaligned"):
        _capi.check(E_ALIGN, "qqt_demo")
    _capi.check(0, "qqt_demo")


def _dying_peer(rank, port, q):
    import datetime
    import torch
    import torch.distributed as dist
    from qqt_b200.ppo import _all_reduce
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)        # the rank leaves between steps, with nothing in flight
    try:
        _all_reduce(torch.ones(345_288))
        q.put("no error")
    except Exception as e:   # noqa: BLE001 - any error is the expected outcome
        q.put("error: " + type(e).__name__)


def test_gradient_all_reduce_fails_fast_when_a_rank_dies():
    import multiprocessing as mp
    import socket
    import time
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dying_peer, args=(r, port, q)) for r in range(2)]
    t0 = time.time()
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert got.startswith("error"), got
    assert time.time() - t0 < 120
