"""zealot-rl's public API (zealot-rl/src/lib.rs:27-28) on the B200 backend.

Names, argument meaning and defaults follow the Rust crate:

* ``PpoConfig``  -- ppo.rs:22-65 (``lr_bounds`` is a tuple as in Rust)
* ``PpoStats``   -- ppo.rs:89-102
* ``Sample``     -- ppo.rs:67-87 (an update also accepts a ``SoaBatch``)
* ``Lcg``        -- rng.rs:9-33
* ``gae``        -- ppo.rs:681-703
* ``ActorCritic``-- ppo.rs:208-651: ``new``, ``update``, ``mean``, ``value``,
  ``logp``, ``entropy``, ``sample``, ``record_obs``, ``save``, ``load``,
  ``load_from_bytes`` and the ``lr`` / ``log_std`` attributes.

Everything runs in libzealot_rl.so on the GPU; errors raise
``native.ZrlError`` (the Rust API panics on ``n < minibatches``,
ppo.rs:340; this raises ``ZrlError(INVALID_ARG)``).
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

from . import native as N

LOG_SQRT_2PI = np.float32(0.9189385)


@dataclass
class PpoConfig:
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

    def c(self) -> N.PpoConfigC:
        return N.PpoConfigC(self.gamma, self.lam, self.clip, self.entropy_coef,
                            self.value_coef, self.epochs, self.minibatches,
                            self.max_grad_norm, self.desired_kl, self.lr_bounds[0],
                            self.lr_bounds[1], 1 if self.adaptive_lr else 0)


@dataclass
class PpoStats:
    kl: float = 0.0
    surrogate: float = 0.0
    value_loss: float = 0.0
    entropy: float = 0.0
    lr: float = 0.0


@dataclass
class Sample:
    obs: Sequence[float] = field(default_factory=list)
    critic_obs: Sequence[float] = field(default_factory=list)
    action: Sequence[float] = field(default_factory=list)
    mean_old: Sequence[float] = field(default_factory=list)
    logp_old: float = 0.0
    value_old: float = 0.0
    adv: float = 0.0
    ret: float = 0.0


class SoaBatch:
    """Structure-of-arrays batch: numpy (host) or torch CUDA tensors."""

    FIELDS = ("obs", "critic_obs", "action", "mean_old", "logp_old",
              "value_old", "adv", "ret")

    def __init__(self, **arrays):
        for f in self.FIELDS:
            a = arrays[f]
            if isinstance(a, np.ndarray) or not hasattr(a, "data_ptr"):
                a = np.ascontiguousarray(a, dtype=np.float32)
            setattr(self, f, a)
        self.n = int(self.logp_old.shape[0])
        self.on_device = hasattr(self.obs, "data_ptr") and getattr(self.obs, "is_cuda", False)

    @classmethod
    def from_samples(cls, batch: Sequence[Sample]):
        return cls(**{f: np.array([getattr(s, f) for s in batch], np.float32)
                      for f in cls.FIELDS})

    def c(self, n_global=0, row_offset=0, write_back_adv=False) -> N.BatchC:
        return N.BatchC(*(N.ptr(getattr(self, f)) for f in self.FIELDS), self.n,
                        n_global, row_offset, 1 if self.on_device else 0,
                        1 if write_back_adv else 0)


class Lcg:
    """rng.rs Lcg (64-bit LCG, Box-Muller gauss)."""

    def __init__(self, seed: int):
        self.state = C.c_uint64(N.lib().zrl_lcg_new(seed))

    new = classmethod(lambda cls, seed: cls(seed))

    def unit(self) -> float:
        return N.lib().zrl_lcg_unit(C.byref(self.state))

    def gauss(self) -> float:
        return N.lib().zrl_lcg_gauss(C.byref(self.state))


def shuffle(seed: int, n: int) -> np.ndarray:
    """The epoch permutation of ppo.rs:357-363."""
    out = np.empty(n, np.int64)
    N.lib().zrl_shuffle(seed, n, out.ctypes.data)
    return out


def _model_config(actor_dims, critic_dims, max_samples, precision) -> N.ModelConfig:
    mc = N.ModelConfig()
    mc.n_actor_dims = len(actor_dims)
    mc.n_critic_dims = len(critic_dims)
    for i, d in enumerate(actor_dims):
        mc.actor_dims[i] = d
    for i, d in enumerate(critic_dims):
        mc.critic_dims[i] = d
    mc.max_samples = max_samples
    mc.precision = N.PRECISIONS[precision] if isinstance(precision, str) else precision
    return mc


class Context:
    """Owns one zrl_ctx (one device, one stream)."""

    def __init__(self, actor_dims, critic_dims, precision="tf32", device=0,
                 max_samples=0, comm: N.CommC | None = None):
        self.actor_dims = tuple(int(d) for d in actor_dims)
        self.critic_dims = tuple(int(d) for d in critic_dims)
        mc = _model_config(self.actor_dims, self.critic_dims, max_samples, precision)
        h = C.c_void_p()
        st = N.lib().zrl_create(C.byref(mc), device, C.byref(comm) if comm else None,
                                C.byref(h))
        if st != N.OK:
            raise N.ZrlError(st, f"zrl_create(actor={self.actor_dims}, "
                                 f"critic={self.critic_dims}, precision={precision})")
        self.h = h
        self.np = N.lib().zrl_param_count(h)

    def close(self):
        if getattr(self, "h", None):
            N.lib().zrl_destroy(self.h)
            self.h = None

    __del__ = close

    def call(self, name, *args):
        N.check(getattr(N.lib(), name)(self.h, *args), self.h)


_gae_ctx = None


def gae(rewards, values, dones, last_value, gamma, lam):
    """ppo.rs:681-703 for one trajectory (runs on the GPU)."""
    global _gae_ctx
    if _gae_ctx is None:
        _gae_ctx = Context((1, 1), (1, 1), precision="fp32")
    r = np.ascontiguousarray(rewards, np.float32)
    v = np.ascontiguousarray(values, np.float32)
    d = np.ascontiguousarray(dones, np.uint8)
    lv = np.array([last_value], np.float32)
    adv = np.empty_like(r)
    ret = np.empty_like(r)
    _gae_ctx.call("zrl_gae", N.ptr(r), N.ptr(v), N.ptr(d), N.ptr(lv), 1, len(r),
                  gamma, lam, N.ptr(adv), N.ptr(ret), 0)
    return adv, ret


class ActorCritic:
    """Gaussian actor-critic (ppo.rs:208-651) backed by libzealot_rl.so."""

    def __init__(self, actor_dims, critic_dims, precision="tf32", device=0,
                 comm: N.CommC | None = None):
        self.ctx = Context(actor_dims, critic_dims, precision, device, comm=comm)
        self.actor_dims = self.ctx.actor_dims
        self.critic_dims = self.ctx.critic_dims

    # -- construction ---------------------------------------------------
    @classmethod
    def new(cls, actor_dims, critic_dims, init_noise_std, init_lr, rng: Lcg,
            precision="tf32", device=0):
        """ActorCritic::new (ppo.rs:235-266), advancing rng like the reference."""
        ac = cls(actor_dims, critic_dims, precision, device)
        ac.ctx.call("zrl_init_reference", init_noise_std, init_lr, C.byref(rng.state))
        return ac

    @classmethod
    def load(cls, path: str, precision="tf32", device=0):
        dims = _safetensors_dims(open(path, "rb").read())
        ac = cls(*dims, precision=precision, device=device)
        ac.ctx.call("zrl_load", path.encode())
        return ac

    @classmethod
    def load_from_bytes(cls, data: bytes, precision="tf32", device=0):
        dims = _safetensors_dims(data)
        ac = cls(*dims, precision=precision, device=device)
        buf = np.frombuffer(data, np.uint8).copy()
        ac.ctx.call("zrl_load_from_bytes", N.ptr(buf), len(data))
        return ac

    def save(self, path: str):
        self.ctx.call("zrl_save", path.encode())

    # -- state ----------------------------------------------------------
    @property
    def action_dim(self) -> int:
        return self.actor_dims[-1]

    @property
    def params(self) -> np.ndarray:
        out = np.empty(self.ctx.np, np.float32)
        self.ctx.call("zrl_get_params", N.ptr(out), self.ctx.np)
        return out

    @params.setter
    def params(self, flat):
        flat = np.ascontiguousarray(flat, np.float32)
        self.ctx.call("zrl_set_params", N.ptr(flat), len(flat))

    @property
    def log_std(self) -> np.ndarray:
        return self.params[-self.action_dim:]

    @property
    def lr(self) -> float:
        v = C.c_float()
        self.ctx.call("zrl_get_lr", C.byref(v))
        return v.value

    @lr.setter
    def lr(self, v: float):
        self.ctx.call("zrl_set_lr", float(v))

    def adam_state(self):
        t3 = np.zeros(3, np.int32)
        m = np.empty(self.ctx.np, np.float32)
        v = np.empty(self.ctx.np, np.float32)
        self.ctx.call("zrl_get_adam_state", N.ptr(t3), N.ptr(m), N.ptr(v), self.ctx.np)
        return t3, m, v

    def set_adam_state(self, t3, m, v):
        t3 = np.ascontiguousarray(t3, np.int32)
        m = np.ascontiguousarray(m, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        self.ctx.call("zrl_set_adam_state", N.ptr(t3), N.ptr(m), N.ptr(v), self.ctx.np)

    def set_normalizers(self, om, om2, oc, cm, cm2, cc):
        a = [np.ascontiguousarray(x, np.float32) for x in (om, om2, cm, cm2)]
        self.ctx.call("zrl_set_normalizers", N.ptr(a[0]), N.ptr(a[1]), float(oc),
                      N.ptr(a[2]), N.ptr(a[3]), float(cc))

    def normalizers(self):
        od, cd = self.actor_dims[0], self.critic_dims[0]
        om, om2 = np.empty(od, np.float32), np.empty(od, np.float32)
        cm, cm2 = np.empty(cd, np.float32), np.empty(cd, np.float32)
        oc, cc = C.c_float(), C.c_float()
        self.ctx.call("zrl_get_normalizers", N.ptr(om), N.ptr(om2), C.byref(oc),
                      N.ptr(cm), N.ptr(cm2), C.byref(cc))
        return om, om2, oc.value, cm, cm2, cc.value

    def record_obs(self, obs, critic_obs):
        """ActorCritic::record_obs (ppo.rs:276-279); rows are folded in order."""
        o = np.ascontiguousarray(obs, np.float32).reshape(-1, self.actor_dims[0])
        c = np.ascontiguousarray(critic_obs, np.float32).reshape(-1, self.critic_dims[0])
        self.ctx.call("zrl_record_obs", N.ptr(o), N.ptr(c), o.shape[0])

    def record_obs_rows(self, obs, critic_obs, parallel=False):
        """record_obs of many rows, numpy or torch CUDA tensors; parallel
        folds 256-row chunks and merges them with Normalizer::commit's
        formula (the same statistics up to f32 rounding)."""
        o, c, n, dev = self._obs_rows(obs, critic_obs)
        self.ctx.call("zrl_record_obs_ex", N.ptr(o), N.ptr(c), n, dev, 1 if parallel else 0)

    def set_mirror(self, obs, critic_obs=None, action=None):
        """The L/R mirror augmentation (biped_train_gpu.rs:89-185, 988-1003):
        each argument a (perm, sign) pair of a signed permutation
        (P x)[i] = sign[i] * x[perm[i]]; obs=None turns it off.  Updates then
        train on the mirrored copies of the batch followed by the batch."""
        if obs is None:
            self.ctx.call("zrl_set_mirror", None, None, None, None, None, None)
            self._mirror = None
            return
        arrs = []
        for perm, sign in (obs, critic_obs, action):
            arrs += [np.ascontiguousarray(perm, np.int32), np.ascontiguousarray(sign, np.float32)]
        self.ctx.call("zrl_set_mirror", *[N.ptr(a) for a in arrs])
        self._mirror = arrs

    # -- the trainer's frozen-normalizer flow (PendingNorm, ppo.rs:118-195)
    def pending_push(self, obs, critic_obs, parallel=False):
        """PendingNorm::push (ppo.rs:126-136) of rows into the pending
        statistics of both normalizers (pn_obs / pn_cobs)."""
        o, c, n, dev = self._obs_rows(obs, critic_obs)
        self.ctx.call("zrl_pending_push", N.ptr(o), N.ptr(c), n, dev, 1 if parallel else 0)

    def commit_pending(self):
        """Normalizer::commit (ppo.rs:179-195) of both pending states."""
        self.ctx.call("zrl_commit_pending")

    def pending(self):
        od, cd = self.actor_dims[0], self.critic_dims[0]
        om, om2 = np.empty(od, np.float32), np.empty(od, np.float32)
        cm, cm2 = np.empty(cd, np.float32), np.empty(cd, np.float32)
        oc, cc = C.c_float(), C.c_float()
        self.ctx.call("zrl_get_pending", N.ptr(om), N.ptr(om2), C.byref(oc),
                      N.ptr(cm), N.ptr(cm2), C.byref(cc))
        return om, om2, oc.value, cm, cm2, cc.value

    def _obs_rows(self, obs, critic_obs):
        if hasattr(obs, "data_ptr"):
            o = obs.contiguous()
            c = critic_obs.contiguous()
            return o, c, o.shape[0], 1
        o = np.ascontiguousarray(obs, np.float32).reshape(-1, self.actor_dims[0])
        c = np.ascontiguousarray(critic_obs, np.float32).reshape(-1, self.critic_dims[0])
        return o, c, o.shape[0], 0

    # -- inference -------------------------------------------------------
    def forward(self, obs=None, critic_obs=None, n=None):
        """Batched ActorCritic::mean / value; either input may be None."""
        on_dev = 0
        if obs is not None:
            n = obs.shape[0]
        elif critic_obs is not None:
            n = critic_obs.shape[0]
        src = obs if obs is not None else critic_obs
        if hasattr(src, "data_ptr"):
            import torch
            on_dev = 1
            mean = torch.empty((n, self.action_dim), dtype=torch.float32, device=src.device) if obs is not None else None
            val = torch.empty(n, dtype=torch.float32, device=src.device) if critic_obs is not None else None
        else:
            obs = None if obs is None else np.ascontiguousarray(obs, np.float32)
            critic_obs = None if critic_obs is None else np.ascontiguousarray(critic_obs, np.float32)
            mean = np.empty((n, self.action_dim), np.float32) if obs is not None else None
            val = np.empty(n, np.float32) if critic_obs is not None else None
        self.ctx.call("zrl_forward", N.ptr(obs), N.ptr(critic_obs), n, N.ptr(mean),
                      N.ptr(val), on_dev)
        return mean, val

    def mean(self, obs):
        m, _ = self.forward(obs=np.asarray(obs, np.float32).reshape(1, -1))
        return m[0]

    def value(self, critic_obs) -> float:
        _, v = self.forward(critic_obs=np.asarray(critic_obs, np.float32).reshape(1, -1))
        return float(v[0])

    def logp(self, action, mean) -> float:
        ls = self.log_std
        lp = np.float32(0.0)
        for k in range(self.action_dim):
            d = (np.float32(action[k]) - np.float32(mean[k])) / np.exp(ls[k])
            lp = np.float32(lp + (np.float32(-0.5) * d * d - ls[k] - LOG_SQRT_2PI))
        return float(lp)

    def entropy(self) -> float:
        c = np.float32(0.5) + LOG_SQRT_2PI
        s = np.float32(0.0)
        for ls in self.log_std:
            s = np.float32(s + (ls + c))
        return float(s)

    def sample(self, obs, rng: Lcg):
        """ActorCritic::sample (ppo.rs:313-323) with the host Lcg stream."""
        mean = self.mean(obs)
        ls = self.log_std
        action = np.array([mean[k] + np.float32(math.exp(ls[k])) * np.float32(rng.gauss())
                           for k in range(self.action_dim)], np.float32)
        return action, self.logp(action, mean), mean

    def policy_step(self, obs, critic_obs, seed: int, counter: int):
        """Batched rollout step on the GPU: (action, logp, mean, value) with
        Philox4x32-10 normal draws keyed by (seed, counter)."""
        obs = np.ascontiguousarray(obs, np.float32)
        critic_obs = np.ascontiguousarray(critic_obs, np.float32)
        n = obs.shape[0]
        act = np.empty((n, self.action_dim), np.float32)
        lp = np.empty(n, np.float32)
        mean = np.empty((n, self.action_dim), np.float32)
        val = np.empty(n, np.float32)
        self.ctx.call("zrl_policy_step", N.ptr(obs), N.ptr(critic_obs), n, seed, counter,
                      N.ptr(act), N.ptr(lp), N.ptr(mean), N.ptr(val), 0)
        return act, lp, mean, val

    def sample_rows(self, obs, critic_obs, rng: "Lcg"):
        """ActorCritic::sample (ppo.rs:313-323) for every row in order from
        one Lcg stream, on the GPU: (action, logp, mean, value); rng
        advances past the draws used, as n sequential sample calls would."""
        obs = np.ascontiguousarray(obs, np.float32)
        critic_obs = np.ascontiguousarray(critic_obs, np.float32)
        n = obs.shape[0]
        act = np.empty((n, self.action_dim), np.float32)
        lp = np.empty(n, np.float32)
        mean = np.empty((n, self.action_dim), np.float32)
        val = np.empty(n, np.float32)
        self.ctx.call("zrl_policy_step_lcg", N.ptr(obs), N.ptr(critic_obs), n,
                      C.byref(rng.state), N.ptr(act), N.ptr(lp), N.ptr(mean), N.ptr(val), 0)
        return act, lp, mean, val

    # -- training --------------------------------------------------------
    def update(self, batch, cfg: PpoConfig, n_global=0, row_offset=0,
               write_back_adv=False) -> PpoStats:
        """ActorCritic::update (ppo.rs:338-384).  A list of Samples has its
        advantages normalized in place, as in the reference; a SoaBatch
        does when write_back_adv is set."""
        samples = None
        if isinstance(batch, (list, tuple)):
            samples = batch
            batch = SoaBatch.from_samples(batch)
        st = N.StatsC()
        bc = batch.c(n_global, row_offset,
                     write_back_adv=samples is not None or write_back_adv)
        cc = cfg.c()
        self.ctx.call("zrl_update", C.byref(cc), C.byref(bc), C.byref(st))
        if samples is not None:
            for s, a in zip(samples, batch.adv):
                s.adv = float(a)
        return PpoStats(st.kl, st.surrogate, st.value_loss, st.entropy, st.lr)

    def gae_update(self, rewards, values, dones, last_values, batch: SoaBatch,
                   cfg: PpoConfig, n_global=0, row_offset=0) -> PpoStats:
        """gae over env-major [n_envs, T] arrays, then update() in one call."""
        n_envs, T = rewards.shape
        ro = N.RolloutC(N.ptr(rewards), N.ptr(values), N.ptr(dones), N.ptr(last_values),
                        n_envs, T)
        st = N.StatsC()
        bc = batch.c(n_global, row_offset)
        cc = cfg.c()
        self.ctx.call("zrl_gae_update", C.byref(cc), C.byref(ro), C.byref(bc), C.byref(st))
        return PpoStats(st.kl, st.surrogate, st.value_loss, st.entropy, st.lr)

    # -- parity hooks ----------------------------------------------------
    def minibatch_grads(self, batch: SoaBatch, idx, cfg: PpoConfig):
        idx = np.ascontiguousarray(idx, np.int64)
        g = np.empty(self.ctx.np, np.float32)
        sums = np.empty(3, np.float32)
        bc = batch.c()
        cc = cfg.c()
        self.ctx.call("zrl_minibatch_grads", C.byref(cc), C.byref(bc), N.ptr(idx),
                      len(idx), N.ptr(g), N.ptr(sums))
        return g, sums

    def apply_grads(self, cfg: PpoConfig, grads, kl: float):
        g = np.ascontiguousarray(grads, np.float32)
        cc = cfg.c()
        self.ctx.call("zrl_apply_grads", C.byref(cc), N.ptr(g), float(kl))

    def kernel_launches(self) -> int:
        return N.lib().zrl_kernel_launches(self.ctx.h)

    def close(self):
        self.ctx.close()


def _safetensors_dims(data: bytes):
    """Rebuild (actor_dims, critic_dims) from a checkpoint header the way
    load_from_bytes scans contiguous w_{l} (ppo.rs:590-614)."""
    import json
    import struct
    (hlen,) = struct.unpack("<Q", data[:8])
    hdr = json.loads(data[8:8 + hlen])
    out = []
    for prefix in ("actor", "critic"):
        dims = []
        l = 0
        while f"{prefix}.w_{l}" in hdr:
            sh = hdr[f"{prefix}.w_{l}"]["shape"]
            if l == 0:
                dims.append(sh[1])
            dims.append(sh[0])
            l += 1
        if not dims:
            raise ValueError(f"no layers under prefix `{prefix}`")
        out.append(tuple(dims))
    return out
