"""ctypes bindings of libzealot_rl.so (declared in include/zealot_rl.h).

There is no fallback: if the shared library is missing or cannot be
loaded, ``lib()`` raises.  ``ZEALOT_RL_LIB`` may point at another build.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("ZEALOT_RL_LIB", os.path.join(HERE, "libzealot_rl.so"))

MAX_LAYERS = 8

OK, INVALID_ARG, CUDA_ERROR, NCCL_ERROR, TIMEOUT, NOT_SUPPORTED, OUT_OF_MEMORY, IO_ERROR = range(8)
STATUS_NAMES = ["OK", "INVALID_ARG", "CUDA_ERROR", "NCCL_ERROR", "TIMEOUT",
                "NOT_SUPPORTED", "OUT_OF_MEMORY", "IO_ERROR"]
PRECISIONS = {"tf32": 0, "fp32": 1, "bf16": 2}


class ZrlError(RuntimeError):
    def __init__(self, status: int, msg: str):
        name = STATUS_NAMES[status] if 0 <= status < len(STATUS_NAMES) else str(status)
        super().__init__(f"{name}: {msg}")
        self.status = status


class ModelConfig(C.Structure):
    _fields_ = [("n_actor_dims", C.c_int32),
                ("actor_dims", C.c_int32 * (MAX_LAYERS + 1)),
                ("n_critic_dims", C.c_int32),
                ("critic_dims", C.c_int32 * (MAX_LAYERS + 1)),
                ("max_samples", C.c_int64),
                ("precision", C.c_int32)]


class PpoConfigC(C.Structure):
    _fields_ = [("gamma", C.c_float), ("lam", C.c_float), ("clip", C.c_float),
                ("entropy_coef", C.c_float), ("value_coef", C.c_float),
                ("epochs", C.c_int32), ("minibatches", C.c_int32),
                ("max_grad_norm", C.c_float), ("desired_kl", C.c_float),
                ("lr_min", C.c_float), ("lr_max", C.c_float),
                ("adaptive_lr", C.c_int32)]


class StatsC(C.Structure):
    _fields_ = [("kl", C.c_float), ("surrogate", C.c_float),
                ("value_loss", C.c_float), ("entropy", C.c_float), ("lr", C.c_float)]


class CommC(C.Structure):
    _fields_ = [("rank", C.c_int32), ("world_size", C.c_int32),
                ("nccl_id", C.c_uint8 * 128), ("timeout_ms", C.c_int32)]


class BatchC(C.Structure):
    _fields_ = [("obs", C.c_void_p), ("critic_obs", C.c_void_p),
                ("action", C.c_void_p), ("mean_old", C.c_void_p),
                ("logp_old", C.c_void_p), ("value_old", C.c_void_p),
                ("adv", C.c_void_p), ("ret", C.c_void_p),
                ("n", C.c_int64), ("n_global", C.c_int64), ("row_offset", C.c_int64),
                ("on_device", C.c_int32), ("write_back_adv", C.c_int32)]


class RolloutC(C.Structure):
    _fields_ = [("rewards", C.c_void_p), ("values", C.c_void_p),
                ("dones", C.c_void_p), ("last_values", C.c_void_p),
                ("n_envs", C.c_int64), ("T", C.c_int64)]


# name -> (restype, argtypes); every symbol declared in include/zealot_rl.h
_P = C.c_void_p
_SIGS = {
    "zrl_abi_version": (C.c_int32, []),
    "zrl_nccl_unique_id": (C.c_int, [_P]),
    "zrl_create": (C.c_int, [C.POINTER(ModelConfig), C.c_int, C.POINTER(CommC), C.POINTER(_P)]),
    "zrl_destroy": (C.c_int, [_P]),
    "zrl_last_error": (C.c_char_p, [_P]),
    "zrl_synchronize": (C.c_int, [_P]),
    "zrl_stream": (_P, [_P]),
    "zrl_param_count": (C.c_int64, [_P]),
    "zrl_init_reference": (C.c_int, [_P, C.c_float, C.c_float, C.POINTER(C.c_uint64)]),
    "zrl_set_params": (C.c_int, [_P, _P, C.c_int64]),
    "zrl_get_params": (C.c_int, [_P, _P, C.c_int64]),
    "zrl_set_adam_state": (C.c_int, [_P, _P, _P, _P, C.c_int64]),
    "zrl_get_adam_state": (C.c_int, [_P, _P, _P, _P, C.c_int64]),
    "zrl_set_normalizers": (C.c_int, [_P, _P, _P, C.c_float, _P, _P, C.c_float]),
    "zrl_get_normalizers": (C.c_int, [_P, _P, _P, _P, _P, _P, _P]),
    "zrl_record_obs": (C.c_int, [_P, _P, _P, C.c_int64]),
    "zrl_record_obs_ex": (C.c_int, [_P, _P, _P, C.c_int64, C.c_int32, C.c_int32]),
    "zrl_pending_push": (C.c_int, [_P, _P, _P, C.c_int64, C.c_int32, C.c_int32]),
    "zrl_commit_pending": (C.c_int, [_P]),
    "zrl_get_pending": (C.c_int, [_P, _P, _P, C.POINTER(C.c_float), _P, _P,
                                  C.POINTER(C.c_float)]),
    "zrl_set_lr": (C.c_int, [_P, C.c_float]),
    "zrl_get_lr": (C.c_int, [_P, C.POINTER(C.c_float)]),
    "zrl_gae": (C.c_int, [_P, _P, _P, _P, _P, C.c_int64, C.c_int64, C.c_float,
                          C.c_float, _P, _P, C.c_int32]),
    "zrl_update": (C.c_int, [_P, C.POINTER(PpoConfigC), C.POINTER(BatchC), C.POINTER(StatsC)]),
    "zrl_gae_update": (C.c_int, [_P, C.POINTER(PpoConfigC), C.POINTER(RolloutC),
                                 C.POINTER(BatchC), C.POINTER(StatsC)]),
    "zrl_forward": (C.c_int, [_P, _P, _P, C.c_int64, _P, _P, C.c_int32]),
    "zrl_policy_step": (C.c_int, [_P, _P, _P, C.c_int64, C.c_uint64, C.c_uint64,
                                  _P, _P, _P, _P, C.c_int32]),
    "zrl_policy_step_lcg": (C.c_int, [_P, _P, _P, C.c_int64, C.POINTER(C.c_uint64), _P, _P,
                                      _P, _P, C.c_int32]),
    "zrl_minibatch_grads": (C.c_int, [_P, C.POINTER(PpoConfigC), C.POINTER(BatchC), _P,
                                      C.c_int64, _P, _P]),
    "zrl_apply_grads": (C.c_int, [_P, C.POINTER(PpoConfigC), _P, C.c_float]),
    "zrl_gemm": (C.c_int, [_P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _P, C.c_int32,
                           _P, C.c_int32, _P, C.c_int32, C.c_int32]),
    "zrl_gae_normalize_noalloc": (C.c_int, [_P, _P, _P, _P, C.c_int64, C.c_int64,
                                            C.c_float, C.c_float, _P, _P, _P, _P]),
    "zrl_save": (C.c_int, [_P, C.c_char_p]),
    "zrl_load": (C.c_int, [_P, C.c_char_p]),
    "zrl_load_from_bytes": (C.c_int, [_P, _P, C.c_size_t]),
    "zrl_lcg_new": (C.c_uint64, [C.c_uint64]),
    "zrl_lcg_unit": (C.c_float, [C.POINTER(C.c_uint64)]),
    "zrl_lcg_gauss": (C.c_float, [C.POINTER(C.c_uint64)]),
    "zrl_shuffle": (None, [C.c_uint64, C.c_int64, _P]),
    "zrl_shuffle_device": (C.c_int, [_P, C.c_uint64, C.c_int64, _P]),
    "zrl_rank_orders": (C.c_int64, [C.c_uint64, C.c_int64, C.c_int64, C.c_int64, C.c_int32,
                                    _P, _P]),
    "zrl_rank_orders_device": (C.c_int64, [_P, C.c_uint64, C.c_int64, C.c_int64, C.c_int64,
                                           C.c_int32, _P, _P]),
    "zrl_kernel_launches": (C.c_int64, [_P]),
    "zrl_set_mirror": (C.c_int, [_P, _P, _P, _P, _P, _P, _P]),
    "zrl_set_wait_limit": (C.c_int, [_P, C.c_uint64]),
    "zrl_test_stall_next_gemm": (C.c_int, [_P]),
    "zrl_test_comm_wait": (C.c_int, [C.c_int32, C.c_int32, C.POINTER(C.c_int32)]),
    "zrl_set_profiling": (C.c_int, [_P, C.c_int32]),
    "zrl_get_profile": (C.c_int, [_P, C.POINTER(C.c_float), C.POINTER(C.c_float),
                                  C.POINTER(C.c_int64)]),
    "zrl_profile_site": (C.c_int32, [_P, C.c_int32, C.POINTER(C.c_char_p),
                                     C.POINTER(C.c_float), C.POINTER(C.c_int64)]),
}

_lib = None


def lib():
    """Load libzealot_rl.so (raises if it is missing: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m zealot_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def exported_symbols():
    return list(_SIGS)


def ptr(a) -> int:
    """Address of a numpy array or a torch tensor (device or host)."""
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        assert a.flags["C_CONTIGUOUS"]
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        assert a.is_contiguous()
        return a.data_ptr()
    raise TypeError(type(a))


def check(status: int, ctx=None):
    if status != OK:
        msg = lib().zrl_last_error(ctx).decode() if ctx else ""
        raise ZrlError(status, msg)
