"""ctypes binding of libqqt_b200.so (the C ABI declared in include/qqt_b200.h).

The library is built in-tree (qqt_b200/_lib/libqqt_b200.so, see build.py).
Loading fails loudly when it is missing: there is no CPU fallback.
"""

from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libqqt_b200.so")

c_i32, c_i64, c_u64, c_f32, c_p = (ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64,
                                   ctypes.c_float, ctypes.c_void_p)

_CFG_INTS = ("n_envs height width n_players fuse blast max_steps invuln_ticks max_hp "
             "resolve_rounds danger_rounds corridor hit_attr_penalty growth_bombs_max "
             "growth_blast_max place_dist_cooldown crate_speed_only timeout_draw "
             "win_hp_scaled combo_on obs_extra obs_channels obs_stride obs_fp32").split()
_CFG_FLOATS = ("radius step_len move_eps2 step_penalty hit_reward brick_reward "
               "danger_penalty explore_coef place_cover_reward place_chain_reward "
               "place_dist_reward place_dist_radius chain_time_factor chain_time_rest "
               "growth_speed_step growth_speed_max pen_speed recycle_crate_prob "
               "combo_reward combo_gap_factor win_bonus win_bonus_per_hp chain_blast_bonus "
               "obs_growth_bombs_max fuse_f max_steps_f h_minus_rad w_minus_rad").split()


_CFG_HAZARD = ([(n, c_i32) for n in ("hazard_on hazard_wave_ticks hazard_bombs_min "
                                       "hazard_bombs_max hazard_blast_min "
                                       "hazard_blast_max").split()]
               + [("hazard_ramp_ticks", c_f32), ("hazard_seed_lo", ctypes.c_uint32),
                  ("hazard_seed_hi", ctypes.c_uint32)])


class QqtCfg(ctypes.Structure):
    _fields_ = [(n, c_i32) for n in _CFG_INTS] + [(n, c_f32) for n in _CFG_FLOATS] + _CFG_HAZARD


STATE_FIELDS = ("wall brick crate recycle fuse owner bomb_blast pos alive hp since_bomb t "
                "bombs_cap blast_cap spd_g invuln pending_lost combo last_hit lo_bombs "
                "lo_blast lo_spd crate_prob hazard").split()


class QqtState(ctypes.Structure):
    _fields_ = [(n, c_p) for n in STATE_FIELDS]


class QqtTemplate(ctypes.Structure):
    _fields_ = [("wall", c_p), ("brick", c_p), ("crate", c_p), ("spawn", c_p),
                ("bombs_cap", c_p), ("blast_cap", c_p), ("spd", c_p), ("crate_prob", c_p),
                ("seed", c_u64), ("swap_spawns", c_i32), ("since_bomb0", c_i32),
                ("episode", c_p)]


MG_WORDS = 14


class QqtMapGen(ctypes.Structure):
    _fields_ = [("seed", c_u64), ("episode", c_p), ("opp_boost", c_p), ("is_open", c_p),
                ("map_kind", c_p), ("corridor_mode", c_i32), ("cut_pure", c_f32),
                ("cut_open", c_f32), ("cut_ring", c_f32), ("obst_max", c_i32),
                ("random_wall_rows", c_i32), ("top_wall_rows", c_i32), ("corr_c0", c_i32),
                ("corr_c1", c_i32), ("n_edge", c_i32), ("edge_cols", c_i32 * 4),
                ("wall_density", c_f32), ("ring_density", c_f32), ("hazard_fraction", c_f32),
                ("ring_r0", c_i32), ("ring_r1", c_i32), ("ring_c0", c_i32), ("ring_c1", c_i32),
                ("open_cross", c_i32), ("start_bombs", c_i64 * 3), ("start_blast", c_i64 * 3),
                ("start_spd", c_f32 * 3), ("crate_prob_kind", c_f32 * 3),
                ("opp_bombs2", c_i64), ("opp_blast2", c_i64), ("opp_spd2", c_f32),
                ("opp_mult", c_f32), ("bombs_max", c_i64), ("blast_max", c_i64),
                ("spd_max", c_f32), ("spawn", ((c_f32 * 2) * 4) * 3),
                ("clear_spawn", ctypes.c_uint32 * MG_WORDS),
                ("clear_ring", ctypes.c_uint32 * MG_WORDS),
                ("cross", ctypes.c_uint32 * MG_WORDS)]


class QqtStepOut(ctypes.Structure):
    _fields_ = [("reward", c_p), ("done", c_p), ("died", c_p), ("winner", c_p),
                ("n_alive", c_p), ("covered", c_p), ("triggered", c_p), ("reset_mask", c_p),
                ("hit", c_p)]


_lib = None


def lib():
    """Load libqqt_b200.so once; raises if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"qqt_b200: CUDA library not built ({LIB_PATH}); run "
                "`python -c 'import __graft_entry__ as g; g.build()'` or "
                "`python qqt-gpu-sim_b200/build.py`")
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.POINTER
        sig = {
            "qqt_step": (c_i32, [P(QqtCfg), P(QqtState), c_p, c_p, c_p, c_p, c_i32,
                                 P(QqtStepOut), P(QqtTemplate), c_p, c_p]),
            "qqt_step_observe": (c_i32, [P(QqtCfg), P(QqtState), c_p, c_p, c_p, c_p, c_i32,
                                 P(QqtStepOut), P(QqtTemplate), c_p, c_p, c_p, c_p, c_p,
                                 c_p]),
            "qqt_step_scratch_bytes": (c_u64, [P(QqtCfg)]),
            "qqt_step_noalloc": (c_i32, [P(QqtCfg), P(QqtState), c_p, c_p, c_p, c_p, c_i32,
                                         P(QqtStepOut), P(QqtTemplate), c_p]),
            "qqt_observe": (c_i32, [P(QqtCfg), P(QqtState), c_p, c_p, c_p, c_p, c_p]),
            "qqt_legal_mask": (c_i32, [P(QqtCfg), P(QqtState), c_p, c_p, c_p]),
            "qqt_astar_act": (c_i32, [P(QqtCfg), P(QqtState), c_p, c_p, c_i32, c_p, c_i32,
                                      c_i32, c_p, c_p, c_p, c_i32, c_p, c_p, c_p, c_i32,
                                      c_p, c_p, c_p, c_p]),
            "qqt_hunter_act": (c_i32, [P(QqtCfg), P(QqtState), c_p, c_p, c_i32, c_p, c_i32,
                                       c_i32, c_p, c_p, c_i32, c_p, c_p, c_p, c_p, c_p]),
            "qqt_random_act": (c_i32, [P(QqtCfg), P(QqtState), c_p, c_i32, c_p, c_i32, c_i32,
                                       c_p, c_p, c_f32, c_p, c_i32, c_p]),
            "qqt_greedy_act": (c_i32, [P(QqtCfg), P(QqtState), c_p, c_p, c_i32, c_p, c_i32,
                                       c_i32, c_p, c_p, c_i32, c_p]),
            "qqt_flush_recycle": (c_i32, [P(QqtCfg), P(QqtState), c_p, c_u64, c_u64, c_p]),
            "qqt_map_reset": (c_i32, [P(QqtCfg), P(QqtState), P(QqtMapGen), c_p, c_p, c_p, c_p,
                                      c_p, c_p]),
            "qqt_gae": (c_i32, [c_p, c_i32, c_p, c_p, c_i32, c_p, c_i32, c_i32, ctypes.c_double,
                                ctypes.c_double, c_p, c_p, c_p]),
            "qqt_local_view": (c_i32, [P(QqtCfg), P(QqtState), c_p, c_i32, c_i32, c_p, c_p, c_p,
                                       c_p]),
            "qqt_gather_rows": (c_i32, [c_p, c_i64, c_i64, c_p, c_i64, c_p, c_i64, c_i64, c_p]),
            "qqt_l1_pack": (c_i32, [c_p, c_i32, c_i32, c_i32, c_i32, c_i32, c_p, c_p]),
            "qqt_l1_pack_bytes": (c_u64, [c_i32]),
            "qqt_l1_forward": (c_i32, [c_p, c_p, c_i64, c_i32, c_i32, c_p, c_p, c_p]),
            "qqt_l1_wgrad": (c_i32, [c_p, c_i64, c_i32, c_i32, c_p, c_i64, c_p, c_i32, c_i32,
                                     c_i32, c_i32, c_p, c_p, c_p]),
            "qqt_l1_wgrad_work_bytes": (c_u64, [c_i64, c_i32]),
            "qqt_mlp_train_forward": (c_i32, [c_p, c_p, c_i32, c_i32, c_i32, c_p, c_i64, c_p,
                                              c_i32, c_p, c_i32, c_p, c_i32, c_p, c_p, c_p, c_p,
                                              c_p, c_p]),
            "qqt_mlp_train_backward": (c_i32, [c_p, c_i32, c_i32, c_p, c_p, c_p, c_i32, c_p,
                                               c_i32, c_p, c_i32, c_p, c_p, c_p, c_p, c_p]),
            "qqt_mlp_train_work_bytes": (c_u64, [c_i32]),
            "qqt_get_error": (c_i32, [P(ctypes.c_uint32)]),
            "qqt_phase_read": (c_i32, [c_p, ctypes.c_uint32, P(ctypes.c_uint32)]),
            "qqt_phase_reset": (c_i32, []),
            "qqt_version": (ctypes.c_char_p, []),
        }
        optional = {
            "qqt_mlp_act": (c_i32, [c_p, c_p, c_p, c_i32, c_i32, c_i32, c_i32, c_p, c_i32, c_p,
                                    c_i32, c_p, c_p, c_i32, c_p, c_p, c_p, c_p, c_p]),
            "qqt_mlp_pack": (c_i32, [c_p, c_i32, c_i32, c_i32, c_i32, c_i32, c_p, c_p, c_p]),
            "qqt_mlp_pack_bytes": (c_u64, [c_i32, c_i32]),
            "qqt_mlp_work_bytes": (c_u64, [c_i32, c_i32]),
            "qqt_mlp_param_names": (ctypes.c_char_p, []),
            "qqt_test_set_wait_polls": (c_i32, [ctypes.c_uint32]),
            "qqt_cnn_act": (c_i32, [c_p, c_p, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32, c_p,
                                    c_i32, c_p, c_i32, c_p, c_p, c_i32, c_p, c_p, c_p, c_p,
                                    c_p]),
            "qqt_cnn_pack": (c_i32, [c_p, c_i32, c_i32, c_i32, c_i32, c_p, c_p, c_p]),
            "qqt_cnn_pack_bytes": (c_u64, [c_i32, c_i32, c_i32]),
            "qqt_cnn_work_bytes": (c_u64, [c_i32, c_i32]),
            "qqt_cnn_param_names": (ctypes.c_char_p, []),
        }
        for name, (res, args) in list(sig.items()) + list(optional.items()):
            if name in optional and not hasattr(L, name):
                continue
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


ERRORS = {1: "bad argument", 2: "misaligned pointer or stride", 3: "size above limit",
          4: "CUDA launch error", 5: "unsupported device"}


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed: {ERRORS.get(rc, rc)}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_error() -> int:
    """Read and clear the device error word (synchronises)."""
    v = ctypes.c_uint32(0)
    check(lib().qqt_get_error(ctypes.byref(v)), "qqt_get_error")
    return int(v.value)
