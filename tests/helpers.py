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


def oracle_update_with_drift(case: Case, ocfg, threads=(3, 7)):
    """Run the oracle update single-threaded (the reference order) and with
    other thread counts.  The reference reduces per-thread gradients in a
    rayon-dependent order (ppo.rs:406-462), so its own result moves with the
    thread count; Adam amplifies such summation-order differences wherever
    first moments nearly cancel.  Returns (delta params, stats, per-tensor
    drift = the largest relative change of the delta across thread counts)."""
    orc = case.oracle_ac()
    st = orc.update(case.oracle_batch(), ocfg, n_threads=1)
    dp = orc.params - case.params
    drift = {}
    for nt in threads:
        o2 = case.oracle_ac()
        o2.update(case.oracle_batch(), ocfg, n_threads=nt)
        for k, v in tensor_l2(o2.params - case.params, dp, case.adims, case.cdims).items():
            drift[k] = max(drift.get(k, 0.0), v)
    return dp, st, orc, drift


def tensor_l2(a, b, adims, cdims):
    out = {}
    for (name, x), (_, y) in zip(split_tensors(a, adims, cdims), split_tensors(b, adims, cdims)):
        x = np.asarray(x, np.float64)
        y = np.asarray(y, np.float64)
        out[name] = float(np.linalg.norm(x - y) / max(np.linalg.norm(y), 1e-30))
    return out


def assert_update_close(gpu_dp, ref_dp, drift, adims, cdims, l2_floor=1e-2):
    """Parameter change of a whole update, per tensor.

    Adam's step is lr * m_hat / (sqrt(v_hat) + eps), at t=1 about
    lr * sign(g): an element whose gradient sits at the rounding-noise floor
    may step either way in any two implementations (the oracle against
    itself with another thread count included), so a max-norm is
    ill-conditioned.  The check is: relative L2 error <= max(l2_floor,
    3 x the oracle's own thread-count drift), and at most 0.1% of the
    elements (at least one) differing by more than 5% of the largest step."""
    l2 = tensor_l2(gpu_dp, ref_dp, adims, cdims)
    bad = {}
    for (name, x), (_, y) in zip(split_tensors(gpu_dp, adims, cdims),
                                 split_tensors(ref_dp, adims, cdims)):
        lim = max(l2_floor, 3.0 * drift.get(name, 0.0))
        big = int(np.sum(np.abs(np.asarray(x, np.float64) - y) > 0.05 * np.abs(y).max()))
        if l2[name] > lim or big > max(1, int(0.001 * y.size)):
            bad[name] = (l2[name], lim, big, y.size)
    assert not bad, bad


def with_own_rollout_policy(case: Case, gpu_ac, batch):
    """mean_old/logp_old recomputed by the GPU's own forward, as a GPU
    rollout would record them (ppo.rs:313-323): the first minibatch's KL is
    then exactly 0 in both implementations, so the adaptive-LR branch
    (kl > 0, ppo.rs:479) is taken alike."""
    from zealot_b200 import synth
    mean, _ = gpu_ac.forward(case.ro.obs)
    batch.mean_old = np.ascontiguousarray(mean, np.float32)
    ls = gpu_ac.log_std
    batch.logp_old = synth.logp_rows(case.ro.action, mean, ls)
    return batch
