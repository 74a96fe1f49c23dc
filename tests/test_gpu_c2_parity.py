"""Parity at the benchmark's size: the C2 workload runs minibatches of
24,576 rows, and at that size the update takes code paths that toy sizes
never reach -- grouped launches of both nets, CTA-pair (256-row) tiles
running several rounds per persistent CTA, double-buffered accumulators,
the split-K counts chosen for the weight gradients (at C2: 10 for layer 1's
and 8 for layer 0's, whose tiles move 3/4 of the bytes, 24 for the flat group) and the
column-sum rows the segment reduce folds.  These tests run those paths.

Inputs: a seeded rollout with the C2 dims (96->512->256->128->29 actor,
96->512->256->128->1 critic), its policy outputs recorded by the GPU
forward (both sides then see identical bytes), the parameters perturbed so
that ratios differ from 1 and the clipped branches are taken, non-trivial
observation normalizers.

Two oracles: the reference's f32 arithmetic, and the same with every GEMM
operand rounded to tf32 where this library stores it (inputs, weights,
hidden activations, deltas; O.ActorCritic.set_tf32_operands).  The second
separates what tf32 itself does to the result (the rounding, measured at
up to 3.2e-3 on these gradients) from what this implementation adds.

Tolerances (tf32 tensor-core mode, the default), norm-wise relative per
tensor:
* one minibatch gradient against the tf32-rounding oracle: critic tensors
  2e-4 (summation order only), actor tensors and log_std 1.5e-3 -- the
  actor's gradient is a strongly cancelling sum over rows (normalized
  advantages times likelihood-ratio terms), so row-level differences of a
  few tf32 ulps (the tensor core's accumulation order, ELU's exp on the
  special-function unit) are magnified relative to the result;
* the same gradient against the f32 reference: 5e-3 (tf32 rounding plus the
  above); the three loss sums: 2e-3, the bar for tf32 losses;
* the update's Adam step applied by the oracle to the GPU's own gradient:
  parameters within 1e-5 (the composition check of the C1 test);
* a whole C2 update (5 epochs x 4 minibatches of 24,576): statistics within
  2e-2 of the f32 reference; the parameter change within max(5e-2, 3 x the
  oracle's own thread-count drift) relative L2 of the tf32-rounding oracle
  (at most 0.1 % of elements off by more than 5 % of the largest step) and
  within 1e-1 of the f32 reference -- twenty Adam steps, each about
  lr * sign(m / sqrt(v)), amplify any difference wherever a gradient
  element sits near zero (the two oracles differ by 5.2e-2 after them).
"""
import os

import numpy as np
import pytest

import oracle as O
from helpers import C_A, C_C, assert_update_close, rel, tensor_l2, tensor_rel
from zealot_b200 import synth
from zealot_b200 import zealot_rl as Z

pytestmark = pytest.mark.gpu

MB = 24_576          # the C2 minibatch (4096 x 24 / 4)
THREADS = os.cpu_count() or 1


class BigCase:
    """A C2-dims rollout whose policy outputs come from the GPU forward."""

    def __init__(self, n_envs, T, seed, perturb=0.02):
        self.adims, self.cdims = C_A, C_C
        rng = np.random.default_rng(seed + 1)
        params = synth.xavier_params(np.random.default_rng(seed), C_A, C_C)
        fw = Z.ActorCritic(C_A, C_C, precision="tf32")
        fw.params = params

        def forward(p, obs, cobs):
            return fw.forward(obs, cobs)

        self.ro = synth.make_rollout(seed, n_envs, T, C_A, C_C, forward, params=params)
        fw.close()
        adv, ret = O.gae_batch(self.ro.rewards, self.ro.value_old.reshape(n_envs, T),
                               self.ro.dones, self.ro.last_values, 0.99, 0.95)
        self.adv = adv.reshape(-1).astype(np.float32)
        self.ret = ret.reshape(-1).astype(np.float32)
        self.params = params + (perturb * rng.standard_normal(params.shape)).astype(np.float32)
        self.params[-C_A[-1]:] = (0.05 * rng.standard_normal(C_A[-1])).astype(np.float32)
        od, cd = C_A[0], C_C[0]
        self.norm = ((0.3 * rng.standard_normal(od)).astype(np.float32),
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

    def gpu_ac(self, lr=1e-3):
        ac = Z.ActorCritic(self.adims, self.cdims, precision="tf32")
        ac.params = self.params
        ac.lr = lr
        ac.set_normalizers(*self.norm)
        return ac

    def oracle_ac(self, lr=1e-3):
        ac = O.ActorCritic(self.adims, self.cdims)
        ac.params = self.params
        ac.lr = lr
        ac.set_normalizers(*self.norm)
        return ac


@pytest.fixture(scope="module")
def mb_case():
    return BigCase(n_envs=MB // 24, T=24, seed=21)


ACTOR_TOL = 1.5e-3   # against the tf32-rounding oracle, actor and log_std
CRITIC_TOL = 2e-4


def _check_against_tf32_oracle(g, g_tf):
    errs = tensor_rel(g, g_tf, C_A, C_C)
    bad = {k: v for k, v in errs.items()
           if v > (CRITIC_TOL if k.startswith("critic") else ACTOR_TOL)}
    assert not bad, bad


def test_c2_minibatch_gradient_matches_oracle(mb_case):
    """One C2 minibatch (24,576 rows in a Fisher-Yates order) through the
    update's own forward/loss/backward/reduce path."""
    case = mb_case
    idx = O.shuffle(5, case.ro.n)
    assert len(idx) == MB
    g, s = case.gpu_ac().minibatch_grads(case.soa(), idx, Z.PpoConfig())
    g2, s2 = case.oracle_ac().minibatch_grads(case.oracle_batch(), idx, O.PpoConfig(),
                                               n_threads=THREADS)
    ot = case.oracle_ac()
    ot.set_tf32_operands()
    gt, _ = ot.minibatch_grads(case.oracle_batch(), idx, O.PpoConfig(), n_threads=THREADS)
    _check_against_tf32_oracle(g, gt)
    errs = tensor_rel(g, g2, case.adims, case.cdims)
    bad = {k: v for k, v in errs.items() if v > 5e-3}
    assert not bad, bad
    for a, b in zip(s, s2):
        assert abs(a - b) <= 2e-3 * max(abs(b), 1e-3), (s, s2)


@pytest.mark.parametrize("adaptive", [False, True])
def test_c2_minibatch_update_composition(mb_case, adaptive):
    """zrl_update on one 24,576-row minibatch (1 epoch x 1 minibatch):
    its statistics, its gradient (recomputed on the advantages it wrote
    back, in the epoch's order) and the oracle's clip + Adam step on that
    gradient, which must reproduce the GPU's parameters."""
    case = mb_case
    cfg = Z.PpoConfig(epochs=1, minibatches=1, adaptive_lr=adaptive)
    ocfg = O.PpoConfig(epochs=1, minibatches=1, adaptive_lr=adaptive)
    gpu = case.gpu_ac()
    batch = case.soa()
    st = gpu.update(batch, cfg, write_back_adv=True)
    st2 = case.oracle_ac().update(case.oracle_batch(), ocfg, n_threads=THREADS)
    assert st.lr == pytest.approx(st2["lr"], rel=1e-6)
    for k in ("kl", "surrogate", "value_loss", "entropy"):
        assert abs(getattr(st, k) - st2[k]) <= 2e-3 * max(abs(st2[k]), 1e-3), (k, st, st2)
    idx = O.shuffle(1, case.ro.n)  # epoch 0: t_logstd (0) + 1
    g = case.gpu_ac().minibatch_grads(batch, idx, cfg)[0]
    ob = case.oracle_batch()
    ob.adv[:] = batch.adv
    ot = case.oracle_ac()
    ot.set_tf32_operands()
    g_tf, _ = ot.minibatch_grads(ob, idx, ocfg, n_threads=THREADS)
    _check_against_tf32_oracle(g, g_tf)
    # the step the GPU took used its own minibatch KL (the update's statistic
    # with one minibatch) for the adaptive learning rate
    o3 = case.oracle_ac()
    o3.apply(ocfg, g, st.kl)
    assert rel(gpu.params, o3.params) < 1e-5
    assert rel(gpu.params - case.params, o3.params - case.params) < 1e-4


def test_c2_whole_update_matches_oracle():
    """A whole C2 update: 4096 envs x 24, 5 epochs x 4 minibatches of 24,576,
    adaptive LR on (the C2 workload)."""
    case = BigCase(n_envs=4096, T=24, seed=22)
    cfg = Z.PpoConfig(epochs=5, minibatches=4, adaptive_lr=True)
    ocfg = O.PpoConfig(epochs=5, minibatches=4, adaptive_lr=True)
    gpu = case.gpu_ac()
    st = gpu.update(case.soa(), cfg)
    dg = gpu.params - case.params
    assert gpu.adam_state()[0].tolist() == [20, 20, 20]
    # the f32 reference: statistics, and the parameter change within 1e-1
    orc = case.oracle_ac()
    st2 = orc.update(case.oracle_batch(), ocfg, n_threads=THREADS)
    for k in ("kl", "surrogate", "value_loss", "entropy", "lr"):
        assert abs(getattr(st, k) - st2[k]) <= 2e-2 * max(abs(st2[k]), 1e-3), (k, st, st2)
    l2 = tensor_l2(dg, orc.params - case.params, case.adims, case.cdims)
    assert max(l2.values()) < 1e-1, l2
    # the tf32-rounding oracle, with its own thread-count drift
    ot = case.oracle_ac()
    ot.set_tf32_operands()
    ot.update(case.oracle_batch(), ocfg, n_threads=THREADS)
    dp = ot.params - case.params
    o2 = case.oracle_ac()
    o2.set_tf32_operands()
    o2.update(case.oracle_batch(), ocfg, n_threads=max(1, THREADS // 2 - 1))
    drift = tensor_l2(o2.params - case.params, dp, case.adims, case.cdims)
    assert_update_close(dg, dp, drift, case.adims, case.cdims, l2_floor=5e-2)
