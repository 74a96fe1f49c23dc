"""Shared builders for the parity tests: seeded rollouts fed identically to
the CUDA library and to the CPU oracle."""
from __future__ import annotations

import numpy as np

import oracle as O
from zealot_b200 import synth
from zealot_b200 import zealot_rl as Z

SMALL_A = (12, 64, 32, 5)
SMALL_C = (10, 64, 32, 1)
C_A = synth.C_ACTOR
C_C = synth.C_CRITIC


def oracle_forward(adims, cdims):
    def fwd(params, obs, cobs):
        ac = O.ActorCritic(adims, cdims)
        ac.params = params
        return ac.forward(obs, cobs)
    return fwd


class Case:
    """A rollout, its GAE (oracle), an oracle ActorCritic and the params the
    update starts from (optionally moved away from the rollout policy so
    that ratios differ from 1 and the clipped branches are exercised)."""

    def __init__(self, adims=SMALL_A, cdims=SMALL_C, n_envs=8, T=12, seed=0,
                 perturb=0.0, norm_stats=False, dones_p=None):
        self.adims, self.cdims = tuple(adims), tuple(cdims)
        self.ro = synth.make_rollout(seed, n_envs, T, adims, cdims,
                                     oracle_forward(adims, cdims))
        if dones_p is not None:
            rng = np.random.default_rng(seed + 99)
            self.ro.dones = (rng.random(self.ro.dones.shape) < dones_p).astype(np.uint8)
        adv, ret = O.gae_batch(self.ro.rewards, self.ro.value_old.reshape(n_envs, T),
                               self.ro.dones, self.ro.last_values, 0.99, 0.95)
        self.adv = adv.reshape(-1).astype(np.float32)
        self.ret = ret.reshape(-1).astype(np.float32)
        rng = np.random.default_rng(seed + 1)
        self.params = self.ro.params.copy()
        if perturb:
            self.params += (perturb * rng.standard_normal(self.params.shape)).astype(np.float32)
            self.params[-adims[-1]:] = (0.05 * rng.standard_normal(adims[-1])).astype(np.float32)
        self.norm = None
        if norm_stats:
            od, cd = adims[0], cdims[0]
            self.norm = (
                (0.3 * rng.standard_normal(od)).astype(np.float32),
                (1.0 + rng.random(od)).astype(np.float32) * 40.0, np.float32(41.0),
                (0.3 * rng.standard_normal(cd)).astype(np.float32),
                (1.0 + rng.random(cd)).astype(np.float32) * 40.0, np.float32(41.0))

    def soa(self):
        ro = self.ro
        return Z.SoaBatch(obs=ro.obs, critic_obs=ro.critic_obs, action=ro.action,
                          mean_old=ro.mean_old, logp_old=ro.logp_old,
                          value_old=ro.value_old, adv=self.adv.copy(), ret=self.ret)

    def oracle_batch(self):
        ro = self.ro
        return O.SoaBatch(obs=ro.obs, critic_obs=ro.critic_obs, action=ro.action,
                          mean_old=ro.mean_old, logp_old=ro.logp_old,
                          value_old=ro.value_old, adv=self.adv.copy(), ret=self.ret)

    def oracle_ac(self, lr=1e-3):
        ac = O.ActorCritic(self.adims, self.cdims)
        ac.params = self.params
        ac.lr = lr
        if self.norm:
            ac.set_normalizers(*self.norm)
        return ac

    def gpu_ac(self, precision="fp32", lr=1e-3):
        ac = Z.ActorCritic(self.adims, self.cdims, precision=precision)
        ac.params = self.params
        ac.lr = lr
        if self.norm:
            ac.set_normalizers(*self.norm)
        return ac


def rel(a, b) -> float:
    """Norm-wise relative error: max|a-b| / max|b|."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def split_tensors(flat, adims, cdims):
    """Yield (name, view) per tensor of a flat save-order buffer."""
    off = 0
    for prefix, dims in (("actor", adims), ("critic", cdims)):
        for l in range(len(dims) - 1):
            fi, fo = dims[l], dims[l + 1]
            yield f"{prefix}.w_{l}", flat[off:off + fo * fi]
            off += fo * fi
            yield f"{prefix}.b_{l}", flat[off:off + fo]
            off += fo
    yield "log_std", flat[off:]


def tensor_rel(a, b, adims, cdims):
    out = {}
    for (name, x), (_, y) in zip(split_tensors(a, adims, cdims), split_tensors(b, adims, cdims)):
        out[name] = rel(x, y)
    return out
