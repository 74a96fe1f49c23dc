"""ctypes front end of the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: this package is the checker that the CUDA library
is compared against.  It may be imported by tests/, by
``__graft_entry__.smoke()`` and by ``bench.py``'s CPU-baseline leg -- never by
the product package ``zealot_b200``.

The C code restates zealot-rl (``zealot-rl/src/{rng,net,ppo}.rs``); see
``zrl_oracle.h`` for the function-by-function map to the reference lines.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import warnings
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")


def build(force: bool = False) -> str:
    """Compile liboracle.so from the C restatement (make -C oracle): make
    rebuilds it whenever the C sources are newer than the library, and
    force rebuilds it unconditionally.  Where make or the compiler cannot
    run and a library is already there (a copy of the tree on another
    machine), that library is used, with a warning."""
    try:
        subprocess.run(["make", "-s", "-C", _HERE] + (["-B"] if force else []), check=True)
    except (OSError, subprocess.CalledProcessError) as e:
        if force or not os.path.exists(_LIB_PATH):
            raise
        warnings.warn(f"oracle: make failed ({e}); using the existing {_LIB_PATH}")
    return _LIB_PATH


class PpoConfigC(C.Structure):
    _fields_ = [
        ("gamma", C.c_float), ("lam", C.c_float), ("clip", C.c_float),
        ("entropy_coef", C.c_float), ("value_coef", C.c_float),
        ("epochs", C.c_int32), ("minibatches", C.c_int32),
        ("max_grad_norm", C.c_float), ("desired_kl", C.c_float),
        ("lr_min", C.c_float), ("lr_max", C.c_float),
        ("adaptive_lr", C.c_int32),
    ]


class StatsC(C.Structure):
    _fields_ = [("kl", C.c_float), ("surrogate", C.c_float),
                ("value_loss", C.c_float), ("entropy", C.c_float),
                ("lr", C.c_float)]


class BatchC(C.Structure):
    _fields_ = [("obs", C.c_void_p), ("critic_obs", C.c_void_p),
                ("action", C.c_void_p), ("mean_old", C.c_void_p),
                ("logp_old", C.c_void_p), ("value_old", C.c_void_p),
                ("adv", C.c_void_p), ("ret", C.c_void_p), ("n", C.c_int64)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(_LIB_PATH)
        L.orc_lcg_new.restype = C.c_uint64
        L.orc_lcg_new.argtypes = [C.c_uint64]
        L.orc_lcg_unit.restype = C.c_float
        L.orc_lcg_unit.argtypes = [C.POINTER(C.c_uint64)]
        L.orc_lcg_gauss.restype = C.c_float
        L.orc_lcg_gauss.argtypes = [C.POINTER(C.c_uint64)]
        L.orc_lcg_fill_unit.argtypes = [C.POINTER(C.c_uint64), _f32p, C.c_int64]
        L.orc_lcg_fill_gauss.argtypes = [C.POINTER(C.c_uint64), _f32p, C.c_int64]
        L.orc_shuffle.argtypes = [C.c_uint64, C.c_int64, _i64p]
        L.orc_gae.argtypes = [_f32p, _f32p, _u8p, C.c_float, C.c_int64,
                              C.c_float, C.c_float, _f32p, _f32p]
        L.orc_gae_batch.argtypes = [_f32p, _f32p, _u8p, _f32p, C.c_int64,
                                    C.c_int64, C.c_float, C.c_float, _f32p, _f32p]
        L.orc_mlp_param_count.restype = C.c_int64
        L.orc_mlp_param_count.argtypes = [_i32p, C.c_int32]
        L.orc_mlp_act_count.restype = C.c_int64
        L.orc_mlp_act_count.argtypes = [_i32p, C.c_int32]
        L.orc_mlp_init.argtypes = [_i32p, C.c_int32, C.c_float,
                                   C.POINTER(C.c_uint64), _f32p]
        L.orc_mlp_forward.argtypes = [_i32p, C.c_int32, _f32p, _f32p, _f32p]
        L.orc_mlp_backward.argtypes = [_i32p, C.c_int32, _f32p, _f32p, _f32p,
                                       _f32p, C.c_void_p]
        L.orc_grad_l2_norm.restype = C.c_float
        L.orc_grad_l2_norm.argtypes = [_f32p, C.c_int64]
        L.orc_grad_clip.argtypes = [_f32p, C.c_int64, C.c_float]
        L.orc_adam_step.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_int64,
                                    C.POINTER(C.c_int32), C.c_float]
        L.orc_powi.restype = C.c_float
        L.orc_powi.argtypes = [C.c_float, C.c_int32]
        L.orc_norm_normalize.argtypes = [_f32p, _f32p, C.c_float, _f32p,
                                         C.c_int64, _f32p]
        L.orc_norm_update.argtypes = [_f32p, _f32p, C.POINTER(C.c_float),
                                      _f32p, C.c_int64]
        L.orc_norm_commit.argtypes = [_f32p, _f32p, C.POINTER(C.c_float), _f32p, _f32p,
                                      C.POINTER(C.c_float), C.c_int64]
        L.orc_ac_new.restype = C.c_void_p
        L.orc_ac_new.argtypes = [_i32p, C.c_int32, _i32p, C.c_int32]
        L.orc_ac_free.argtypes = [C.c_void_p]
        L.orc_ac_init_reference.argtypes = [C.c_void_p, C.c_float, C.c_float,
                                            C.POINTER(C.c_uint64)]
        L.orc_ac_param_count.restype = C.c_int64
        L.orc_ac_param_count.argtypes = [C.c_void_p]
        L.orc_ac_set_params.argtypes = [C.c_void_p, _f32p]
        L.orc_ac_get_params.argtypes = [C.c_void_p, _f32p]
        L.orc_ac_set_normalizers.argtypes = [C.c_void_p, _f32p, _f32p, C.c_float,
                                             _f32p, _f32p, C.c_float]
        L.orc_ac_set_lr.argtypes = [C.c_void_p, C.c_float]
        L.orc_ac_set_operand_rounding.argtypes = [C.c_void_p, C.c_int32]
        L.orc_ac_get_lr.restype = C.c_float
        L.orc_ac_get_lr.argtypes = [C.c_void_p]
        L.orc_ac_get_adam.argtypes = [C.c_void_p, _i32p, _f32p, _f32p]
        L.orc_ac_set_adam.argtypes = [C.c_void_p, _i32p, _f32p, _f32p]
        L.orc_ac_forward.argtypes = [C.c_void_p, _f32p, _f32p, C.c_int64,
                                     _f32p, _f32p]
        L.orc_ac_logp.restype = C.c_float
        L.orc_ac_logp.argtypes = [C.c_void_p, _f32p, _f32p]
        L.orc_ac_entropy.restype = C.c_float
        L.orc_ac_entropy.argtypes = [C.c_void_p]
        L.orc_ac_minibatch_grads.argtypes = [C.c_void_p, C.POINTER(BatchC), _i64p,
                                             C.c_int64, C.POINTER(PpoConfigC),
                                             _f32p, _f32p, C.c_int32]
        L.orc_ac_apply.argtypes = [C.c_void_p, C.POINTER(PpoConfigC), _f32p,
                                   C.c_float]
        L.orc_ac_update.restype = C.c_int
        L.orc_ac_update.argtypes = [C.c_void_p, C.POINTER(BatchC),
                                    C.POINTER(PpoConfigC), C.POINTER(StatsC),
                                    C.c_int32]
        _lib = L
    return _lib


# ----------------------------------------------------------------- wrappers

def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


class Lcg:
    """rng.rs:9-33."""

    def __init__(self, seed: int):
        self.state = C.c_uint64(lib().orc_lcg_new(seed))

    def unit(self) -> float:
        return lib().orc_lcg_unit(C.byref(self.state))

    def gauss(self) -> float:
        return lib().orc_lcg_gauss(C.byref(self.state))

    def units(self, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        lib().orc_lcg_fill_unit(C.byref(self.state), out, n)
        return out

    def gausses(self, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        lib().orc_lcg_fill_gauss(C.byref(self.state), out, n)
        return out


def shuffle(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.int64)
    lib().orc_shuffle(seed, n, out)
    return out


def gae(rewards, values, dones, last_value, gamma, lam):
    r, v = _f32(rewards), _f32(values)
    d = np.ascontiguousarray(dones, dtype=np.uint8)
    adv = np.empty_like(r)
    ret = np.empty_like(r)
    lib().orc_gae(r, v, d, float(last_value), len(r), gamma, lam, adv, ret)
    return adv, ret


def gae_batch(rewards, values, dones, last_values, gamma, lam):
    """rewards/values/dones: [n_envs, T] env-major; returns adv, ret [n_envs, T]."""
    r, v = _f32(rewards), _f32(values)
    d = np.ascontiguousarray(dones, dtype=np.uint8)
    lv = _f32(last_values)
    n_envs, T = r.shape
    adv = np.empty_like(r)
    ret = np.empty_like(r)
    lib().orc_gae_batch(r, v, d, lv, n_envs, T, gamma, lam, adv, ret)
    return adv, ret


class Mlp:
    """net.rs Mlp over a flat [w_0, b_0, w_1, b_1, ...] buffer."""

    def __init__(self, dims, params=None):
        self.dims = np.asarray(dims, np.int32)
        n = lib().orc_mlp_param_count(self.dims, len(self.dims))
        self.params = np.zeros(n, np.float32) if params is None else _f32(params).copy()

    @classmethod
    def new(cls, dims, out_scale, rng: Lcg):
        m = cls(dims)
        lib().orc_mlp_init(m.dims, len(m.dims), out_scale, C.byref(rng.state), m.params)
        return m

    def forward(self, x):
        acts = np.empty(lib().orc_mlp_act_count(self.dims, len(self.dims)), np.float32)
        lib().orc_mlp_forward(self.dims, len(self.dims), self.params, _f32(x), acts)
        return acts

    def output(self, acts):
        return acts[-int(self.dims[-1]):]

    def backward(self, acts, g_out, grads):
        g_in = np.empty(int(self.dims[0]), np.float32)
        lib().orc_mlp_backward(self.dims, len(self.dims), self.params, acts,
                               _f32(g_out), grads, g_in.ctypes.data)
        return g_in

    def tensors(self, flat=None):
        """Split a flat buffer into [(w, b), ...] views."""
        flat = self.params if flat is None else flat
        out, off = [], 0
        for l in range(len(self.dims) - 1):
            fi, fo = int(self.dims[l]), int(self.dims[l + 1])
            w = flat[off:off + fo * fi].reshape(fo, fi)
            off += fo * fi
            b = flat[off:off + fo]
            off += fo
            out.append((w, b))
        return out


def adam_step(p, g, m, v, t: int, lr: float) -> int:
    tt = C.c_int32(t)
    lib().orc_adam_step(p, _f32(g), m, v, len(p), C.byref(tt), lr)
    return tt.value


def grad_l2_norm(g) -> float:
    return lib().orc_grad_l2_norm(_f32(g), len(g))


def grad_clip(g, max_norm):
    lib().orc_grad_clip(g, len(g), max_norm)


def powi(a: float, b: int) -> float:
    return lib().orc_powi(a, b)


@dataclass
class PpoConfig:
    """ppo.rs:22-65 with its defaults."""
    gamma: float = 0.99
    lam: float = 0.95
    clip: float = 0.2
    entropy_coef: float = 0.01
    value_coef: float = 1.0
    epochs: int = 5
    minibatches: int = 4
    max_grad_norm: float = 1.0
    desired_kl: float = 0.01
    lr_bounds: tuple = (1e-5, 1e-2)
    adaptive_lr: bool = True

    def c(self) -> PpoConfigC:
        return PpoConfigC(self.gamma, self.lam, self.clip, self.entropy_coef,
                          self.value_coef, self.epochs, self.minibatches,
                          self.max_grad_norm, self.desired_kl,
                          self.lr_bounds[0], self.lr_bounds[1],
                          1 if self.adaptive_lr else 0)


class SoaBatch:
    """Structure-of-arrays batch: one row per zealot-rl Sample."""

    FIELDS = ("obs", "critic_obs", "action", "mean_old", "logp_old",
              "value_old", "adv", "ret")

    def __init__(self, **arrays):
        for f in self.FIELDS:
            setattr(self, f, _f32(arrays[f]).copy())
        self.n = self.logp_old.shape[0]

    def c(self) -> BatchC:
        return BatchC(*(getattr(self, f).ctypes.data for f in self.FIELDS), self.n)

    def copy(self):
        return SoaBatch(**{f: getattr(self, f) for f in self.FIELDS})


class ActorCritic:
    """ppo.rs ActorCritic (CPU oracle)."""

    def __init__(self, actor_dims, critic_dims):
        self.adims = np.asarray(actor_dims, np.int32)
        self.cdims = np.asarray(critic_dims, np.int32)
        self.h = lib().orc_ac_new(self.adims, len(self.adims), self.cdims, len(self.cdims))
        if not self.h:
            raise ValueError("invalid dims")
        self.np = lib().orc_ac_param_count(self.h)

    def __del__(self):
        h = getattr(self, "h", None)
        if h and _lib is not None:
            _lib.orc_ac_free(h)
            self.h = None

    @classmethod
    def new(cls, actor_dims, critic_dims, init_noise_std, init_lr, rng: Lcg):
        ac = cls(actor_dims, critic_dims)
        lib().orc_ac_init_reference(ac.h, init_noise_std, init_lr, C.byref(rng.state))
        return ac

    @property
    def params(self) -> np.ndarray:
        out = np.empty(self.np, np.float32)
        lib().orc_ac_get_params(self.h, out)
        return out

    @params.setter
    def params(self, flat):
        flat = _f32(flat)
        assert flat.shape == (self.np,)
        lib().orc_ac_set_params(self.h, flat)

    def set_normalizers(self, om, om2, oc, cm, cm2, cc):
        lib().orc_ac_set_normalizers(self.h, _f32(om), _f32(om2), oc, _f32(cm), _f32(cm2), cc)

    @property
    def lr(self) -> float:
        return lib().orc_ac_get_lr(self.h)

    @lr.setter
    def lr(self, v):
        lib().orc_ac_set_lr(self.h, v)

    def set_tf32_operands(self, on: bool = True):
        """Emulate a tf32 tensor-core backend's operand rounding (inputs,
        weights, hidden activations and deltas rounded to tf32, f32
        accumulation) on top of the reference arithmetic."""
        lib().orc_ac_set_operand_rounding(self.h, 1 if on else 0)

    def set_bf16_operands(self, on: bool = True):
        """The same with bf16 operands (nearest, ties to even)."""
        lib().orc_ac_set_operand_rounding(self.h, 2 if on else 0)

    def adam_state(self):
        t3 = np.zeros(3, np.int32)
        m = np.empty(self.np, np.float32)
        v = np.empty(self.np, np.float32)
        lib().orc_ac_get_adam(self.h, t3, m, v)
        return t3, m, v

    def set_adam_state(self, t3, m, v):
        lib().orc_ac_set_adam(self.h, np.asarray(t3, np.int32), _f32(m), _f32(v))

    def forward(self, obs, cobs):
        obs, cobs = _f32(obs), _f32(cobs)
        n = obs.shape[0]
        mean = np.empty((n, int(self.adims[-1])), np.float32)
        val = np.empty(n, np.float32)
        lib().orc_ac_forward(self.h, obs, cobs, n, mean, val)
        return mean, val

    def logp(self, action, mean) -> float:
        return lib().orc_ac_logp(self.h, _f32(action), _f32(mean))

    def entropy(self) -> float:
        return lib().orc_ac_entropy(self.h)

    def minibatch_grads(self, batch: SoaBatch, idx, cfg: PpoConfig, n_threads=1):
        idx = np.ascontiguousarray(idx, np.int64)
        g = np.empty(self.np, np.float32)
        sums = np.empty(3, np.float32)
        bc = batch.c()
        cc = cfg.c()
        lib().orc_ac_minibatch_grads(self.h, C.byref(bc), idx, len(idx), C.byref(cc),
                                     g, sums, n_threads)
        return g, sums

    def apply(self, cfg: PpoConfig, grads, kl: float):
        cc = cfg.c()
        lib().orc_ac_apply(self.h, C.byref(cc), _f32(grads), kl)

    def update(self, batch: SoaBatch, cfg: PpoConfig, n_threads=1):
        bc = batch.c()
        cc = cfg.c()
        st = StatsC()
        rc = lib().orc_ac_update(self.h, C.byref(bc), C.byref(cc), C.byref(st), n_threads)
        if rc != 0:
            raise ValueError("fewer samples than minibatches")
        return {"kl": st.kl, "surrogate": st.surrogate, "value_loss": st.value_loss,
                "entropy": st.entropy, "lr": st.lr}
