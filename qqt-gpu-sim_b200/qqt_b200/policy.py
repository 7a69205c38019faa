"""B200Policy: the reference ActorCritic(arch="mlp") forward/act on the
tcgen05 kernels (train/model.py:54-259).

Parameters use the reference's state_dict keys, so a reference checkpoint's
`model` dict loads directly.  The first layer's per-seat view permutation is
folded into a packed weight copy (column gather + fp16 hi/lo split) built on
the device by `qqt_mlp_pack`; call `repack()` after any parameter update.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _capi as capi
from .sim import check_tile_flags

PARAM_NAMES = ("shared.0.weight shared.0.bias shared.1.weight shared.1.bias shared.3.weight "
               "shared.3.bias shared.4.weight shared.4.bias move_head.0.weight "
               "move_head.0.bias move_head.2.weight move_head.2.bias bomb_head.0.weight "
               "bomb_head.0.bias bomb_head.2.weight bomb_head.2.bias critic.0.weight "
               "critic.0.bias critic.2.weight critic.2.bias").split()


CNN_PARAM_NAMES = ("conv0.weight conv0.bias conv.0.weight conv.0.bias conv.2.weight conv.2.bias "
                   "conv.3.weight conv.3.bias conv.5.weight conv.5.bias conv.6.weight conv.6.bias "
                   "conv.8.weight conv.8.bias conv.9.weight conv.9.bias").split() + PARAM_NAMES


def _rows(t: torch.Tensor, width: int):
    if t.dtype == torch.bool:
        t = t.view(torch.uint8)
    if t.dim() != 2 or t.shape[1] != width or t.stride(1) != 1:
        t = t.reshape(-1, width).contiguous()
    return t


class B200Policy:
    """Actor-critic (arch "mlp" or "cnn") for one or two seats sharing one
    observation.

    params: name -> tensor/ndarray (reference state_dict keys).
    seats: the pids this pack serves; for the MLP two seats run as one
    N=256 tensor-core GEMM.
    """

    def __init__(self, params: dict, obs_shape, n_players: int = 2, seats=(0,),
                 device="cuda", arch: str = "mlp") -> None:
        if arch not in ("mlp", "cnn"):
            raise ValueError(f"unsupported arch {arch}")
        self.arch = arch
        self.names = PARAM_NAMES if arch == "mlp" else CNN_PARAM_NAMES
        self.device = torch.device(device)
        self.obs_shape = tuple(obs_shape)
        c, h, w = self.obs_shape
        self.k_in = c * h * w
        self.n_players = n_players
        self.seats = tuple(int(s) for s in seats)
        if not 1 <= len(self.seats) <= 2:
            raise ValueError("one or two seats per pack")
        self.params = {k: torch.as_tensor(np.asarray(params[k]) if not torch.is_tensor(params[k])
                                          else params[k]).to(self.device, torch.float32)
                       .contiguous() for k in self.names}
        L = capi.lib()
        if arch == "mlp":
            nbytes = int(L.qqt_mlp_pack_bytes(self.k_in, len(self.seats)))
        else:
            nbytes = int(L.qqt_cnn_pack_bytes(c, h * w, len(self.seats)))
        self.pack = torch.zeros((nbytes,), dtype=torch.uint8, device=self.device)
        self._work = {}
        self.repack()

    def repack(self) -> None:
        L = capi.lib()
        ptrs = (ctypes.c_void_p * len(self.names))(*[self.params[k].data_ptr() for k in self.names])
        pids = (ctypes.c_int32 * 2)(*(list(self.seats) + [0] * (2 - len(self.seats))))
        c, h, w = self.obs_shape
        if self.arch == "mlp":
            rc = L.qqt_mlp_pack(ptrs, self.k_in, self.n_players, c, h * w, len(self.seats), pids,
                                self.pack.data_ptr(), capi.stream_ptr(self.device))
        else:
            rc = L.qqt_cnn_pack(ptrs, self.n_players, c, h * w, len(self.seats), pids,
                                self.pack.data_ptr(), capi.stream_ptr(self.device))
        capi.check(rc, "qqt_%s_pack" % self.arch)

    def load_state_dict(self, sd: dict) -> None:
        for k in self.names:
            self.params[k].copy_(torch.as_tensor(sd[k]))
        self.repack()

    def _work_buf(self, n):
        buf = self._work.get(n)
        if buf is None:
            fn = capi.lib().qqt_mlp_work_bytes if self.arch == "mlp" else capi.lib().qqt_cnn_work_bytes
            nb = int(fn(n, len(self.seats)))
            buf = torch.empty((nb // 4,), dtype=torch.float32, device=self.device)
            self._work[n] = buf
        return buf

    @staticmethod
    def _obs_rows(obs: torch.Tensor):
        """(pointer, row stride in elements) of an fp16 obs whose rows are equally
        spaced with a 16-byte multiple stride (the engine's padded buffer)."""
        if obs.dtype != torch.float16:
            obs = obs.half()
        n = obs.shape[0]
        stride = obs.stride(0)
        inner_ok = obs[0].is_contiguous() if obs.dim() > 1 else True
        if not inner_ok or stride % 8 or obs.data_ptr() % 16:
            k = obs[0].numel()
            pad = (k + 7) // 8 * 8
            buf = torch.zeros((n, pad), dtype=torch.float16, device=obs.device)
            buf[:, :k] = obs.reshape(n, -1)
            return buf, pad
        return obs, stride

    def act_seats(self, obs, mmasks, bmasks, u, acts, logp=None, value=None, logits=None,
                  obs_tiles=None):
        """Act for every seat of the pack in one call.

        obs (N, C, H, W) fp16; mmasks/bmasks: per seat (N,5)/(N,2) views;
        u (S, N, 2) uniforms; acts: per seat (N, 2) int64 views to fill.
        obs_tiles: optional (N, 4) int32 nonzero-K-tile flags of the obs rows
        (as the step's fused observation writes them); the MLP then skips the
        first-layer K tiles that are zero in all rows of a row tile (exact).
        The CNN ignores them.
        """
        n = obs.shape[0]
        S = len(self.seats)
        # (a repacked copy keeps every entry at its index, so the flags hold)
        ob, stride = self._obs_rows(obs)
        if obs_tiles is not None:
            check_tile_flags(obs_tiles, n)
        mms = [_rows(m, 5) for m in mmasks]
        bms = [_rows(b, 2) for b in bmasks]
        for a in acts:
            if a.stride(1) != 1 or a.dtype != torch.int64:
                raise ValueError("action rows must be int64 with unit inner stride")
        if any(m.stride(0) != mms[0].stride(0) for m in mms) or \
                any(b.stride(0) != bms[0].stride(0) for b in bms) or \
                any(a.stride(0) != acts[0].stride(0) for a in acts):
            raise ValueError("seats must share row strides")
        uu = u.to(self.device, torch.float32).contiguous()
        mp = (ctypes.c_void_p * 2)(*([m.data_ptr() for m in mms] + [0] * (2 - S)))
        bp = (ctypes.c_void_p * 2)(*([b.data_ptr() for b in bms] + [0] * (2 - S)))
        ap = (ctypes.c_void_p * 2)(*([a.data_ptr() for a in acts] + [0] * (2 - S)))
        if self.arch == "mlp":
            rc = capi.lib().qqt_mlp_act(self.pack.data_ptr(), ob.data_ptr(), capi.ptr(obs_tiles),
                                        n, stride, self.k_in,
                                        S, mp, mms[0].stride(0), bp, bms[0].stride(0),
                                        uu.data_ptr(), ap, acts[0].stride(0), capi.ptr(logp),
                                        capi.ptr(value), capi.ptr(logits),
                                        self._work_buf(n).data_ptr(), capi.stream_ptr(self.device))
        else:
            c, h, w = self.obs_shape
            rc = capi.lib().qqt_cnn_act(self.pack.data_ptr(), ob.data_ptr(), n, stride, h, w, c, S,
                                        mp, mms[0].stride(0), bp, bms[0].stride(0),
                                        uu.data_ptr(), ap, acts[0].stride(0), capi.ptr(logp),
                                        capi.ptr(value), capi.ptr(logits),
                                        self._work_buf(n).data_ptr(), capi.stream_ptr(self.device))
        capi.check(rc, "qqt_%s_act" % self.arch)

    def act(self, obs, move_mask, bomb_mask, pid: int = 0, u=None):
        """ActorCritic.act: (actions (B,2), logp (B,), value (B,)) for seat pid."""
        if pid not in self.seats:
            raise ValueError(f"pack built for seats {self.seats}, not {pid}")
        if len(self.seats) != 1:
            raise ValueError("act() serves single-seat packs; use act_seats()")
        n = obs.shape[0]
        if u is None:
            u = torch.rand((1, n, 2), device=self.device)
        acts = torch.empty((n, 2), dtype=torch.int64, device=self.device)
        logp = torch.empty((1, n), dtype=torch.float32, device=self.device)
        value = torch.empty((1, n), dtype=torch.float32, device=self.device)
        self.act_seats(obs, [move_mask], [bomb_mask], u.reshape(1, n, 2), [acts], logp, value)
        return acts, logp[0], value[0]

    def forward_logits(self, obs, move_mask, bomb_mask, u=None, obs_tiles=None):
        """(logits (S,N,8): 5 move, 2 bomb, value; actions per seat; logp (S,N)).
        obs_tiles: optional K-tile flags of the rows (see act_seats)."""
        n = obs.shape[0]
        S = len(self.seats)
        if u is None:
            u = torch.rand((S, n, 2), device=self.device)
        logits = torch.empty((S, n, 8), dtype=torch.float32, device=self.device)
        logp = torch.empty((S, n), dtype=torch.float32, device=self.device)
        acts = [torch.empty((n, 2), dtype=torch.int64, device=self.device) for _ in range(S)]
        mm = [move_mask[:, p] for p in self.seats]
        bm = [bomb_mask[:, p] for p in self.seats]
        self.act_seats(obs, mm, bm, u, acts, logp, None, logits, obs_tiles=obs_tiles)
        return logits, acts, logp
