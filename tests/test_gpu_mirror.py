"""The L/R mirror augmentation (biped_train_gpu.rs:89-185, 988-1003) fused
into the epoch gather, against the batch doubled explicitly.

mirror_sample restated: obs, critic_obs, action and mean_old mapped by
signed permutations (P x)[i] = sign[i] * x[perm[i]]; logp_old, value_old,
adv and ret kept; the mirrored copies first, then the samples.
* the GPU update with the mirror on equals the GPU update of the explicitly
  doubled batch (the same rows, in the same virtual order, through the same
  kernels): parameters bit for bit, statistics exactly;
* it follows the oracle's update of the doubled batch (ppo.rs:338-510) as
  any fp32 update does: relative L2 of the parameter change per tensor
  within max(1e-2, 3 x the oracle's own thread-count drift).
"""
import numpy as np
import pytest

import oracle as O
from helpers import SMALL_A, SMALL_C, Case, assert_update_close, tensor_l2
from zealot_b200 import native as N
from zealot_b200 import zealot_rl as Z

pytestmark = pytest.mark.gpu


def _sperm(d, seed):
    """An involutive signed permutation: adjacent pairs swapped, signs fixed
    per pair (the structure of the reference's joint mirrors)."""
    rng = np.random.default_rng(seed)
    perm = np.arange(d, dtype=np.int32)
    for k in range(0, d - 1, 2):
        perm[k], perm[k + 1] = k + 1, k
    sign = np.where(rng.random(d) < 0.4, -1.0, 1.0).astype(np.float32)
    for k in range(0, d - 1, 2):
        sign[k + 1] = sign[k]
    return perm, sign


def _apply(x, sp):
    perm, sign = sp
    return (x[:, perm] * sign).astype(np.float32)


def _doubled(case, sps):
    b = case.soa()
    mir = dict(obs=_apply(b.obs, sps[0]), critic_obs=_apply(b.critic_obs, sps[1]),
               action=_apply(b.action, sps[2]), mean_old=_apply(b.mean_old, sps[2]))
    cat = {}
    for f in Z.SoaBatch.FIELDS:
        base = getattr(b, f)
        cat[f] = np.ascontiguousarray(np.concatenate([mir.get(f, base), base]))
    return cat


@pytest.mark.parametrize("precision", ["fp32", "tf32"])
def test_mirror_equals_the_explicitly_doubled_batch(precision):
    case = Case(SMALL_A, SMALL_C, n_envs=10, T=12, seed=41, perturb=0.03, norm_stats=True)
    sps = (_sperm(SMALL_A[0], 1), _sperm(SMALL_C[0], 2), _sperm(SMALL_A[-1], 3))
    cfg = Z.PpoConfig(epochs=2, minibatches=4)
    a = case.gpu_ac(precision)
    a.set_mirror(*sps)
    st_a = a.update(case.soa(), cfg)
    b = case.gpu_ac(precision)
    st_b = b.update(Z.SoaBatch(**_doubled(case, sps)), cfg)
    assert np.array_equal(a.params, b.params)
    assert st_a == st_b
    # off again: the plain update
    a2 = case.gpu_ac(precision)
    a2.set_mirror(None)
    a3 = case.gpu_ac(precision)
    a2.update(case.soa(), cfg)
    a3.update(case.soa(), cfg)
    assert np.array_equal(a2.params, a3.params)


def test_mirror_update_follows_the_oracle():
    case = Case(SMALL_A, SMALL_C, n_envs=10, T=12, seed=42, perturb=0.03, norm_stats=True)
    sps = (_sperm(SMALL_A[0], 4), _sperm(SMALL_C[0], 5), _sperm(SMALL_A[-1], 6))
    cfg = Z.PpoConfig(epochs=2, minibatches=4)
    ocfg = O.PpoConfig(epochs=2, minibatches=4)
    gpu = case.gpu_ac("fp32")
    gpu.set_mirror(*sps)
    st = gpu.update(case.soa(), cfg)
    d = _doubled(case, sps)
    orc = case.oracle_ac()
    st2 = orc.update(O.SoaBatch(**d), ocfg, n_threads=1)
    dp = orc.params - case.params
    o2 = case.oracle_ac()
    o2.update(O.SoaBatch(**_doubled(case, sps)), ocfg, n_threads=7)
    drift = tensor_l2(o2.params - case.params, dp, case.adims, case.cdims)
    assert_update_close(gpu.params - case.params, dp, drift, case.adims, case.cdims)
    for k in ("kl", "surrogate", "value_loss", "entropy"):
        assert abs(getattr(st, k) - st2[k]) <= 1e-4 * max(abs(st2[k]), 1e-3), (k, st, st2)


def test_mirror_rejects_what_is_not_a_signed_permutation():
    ac = Z.ActorCritic(SMALL_A, SMALL_C, precision="fp32")
    good = (_sperm(SMALL_A[0], 1), _sperm(SMALL_C[0], 2), _sperm(SMALL_A[-1], 3))
    bad_perm = (np.zeros(SMALL_A[0], np.int32), good[0][1])
    with pytest.raises(N.ZrlError):
        ac.set_mirror(bad_perm, good[1], good[2])
    bad_sign = (good[0][0], np.full(SMALL_A[0], 0.5, np.float32))
    with pytest.raises(N.ZrlError):
        ac.set_mirror(bad_sign, good[1], good[2])
