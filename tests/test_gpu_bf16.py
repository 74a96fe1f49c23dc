"""The bf16 tensor-core path (the C5 workload: bf16 GEMM inputs,
fp32 master weights and Adam) against the fp32 CPU oracle.

In a bf16 context every GEMM operand is stored in bf16 (round to nearest
even: normalized observations, the weight copy Adam writes, hidden
activations, deltas) and accumulated in fp32; everything else (the loss,
bias gradients as column sums of the unrounded deltas, GAE, Adam on the
fp32 master) is the fp32 path.  bf16 keeps 8 significant bits (unit
roundoff 2^-9 = 2e-3), so values that pass through three or four bf16
GEMM layers differ from the fp32 oracle by about 1e-2 relative: the bar
for the forward outputs is 3e-2.  The gradient carries that error through
the PPO ratio exp(logp - logp_old), where logp sums 29 squared
standardized action residuals (ppo.rs:297-305, 410-433): every actor
tensor then moves by the same ~3 % (measured 3.0-3.3 % on the C5 dims),
so the gradient bar is 5e-2 per tensor (norm-wise), and a whole update
must move the parameters in the oracle's direction (cosine > 0.97).

Those bars measure bf16 itself.  The second oracle rounds every GEMM
operand to bf16 where this library stores it (O.ActorCritic.
set_bf16_operands: inputs, weights, hidden activations, deltas; products
exact in f32), so against it only the summation order and the ELU's
exponential differ.  Measured on the C5 dims: forward 2.6e-4, gradient
tensors at most 6.1e-4, loss sums 3e-5, a whole update 9.8e-3 relative L2
per tensor (the oracle against itself with another thread count: 1.2e-3),
cosine 0.99997.  Bars: forward and gradient 2e-3 per tensor, loss sums
1e-3, update 2e-2 per tensor and cosine > 0.999 -- a sign error in any one
tensor fails them.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from tests.helpers import Case, tensor_l2
from zealot_b200 import zealot_rl as Z

pytestmark = pytest.mark.gpu

C5_A = (96, 1024, 512, 256, 29)
C5_C = (256, 1024, 512, 256, 1)
TOL = 3e-2
TOL_GRAD = 5e-2


@pytest.fixture(scope="module")
def case():
    return Case(C5_A, C5_C, n_envs=16, T=12, seed=21, perturb=0.03, norm_stats=True)


def test_bf16_forward(case):
    gpu = case.gpu_ac("bf16")
    orc = case.oracle_ac()
    mean, value = gpu.forward(case.ro.obs, case.ro.critic_obs)
    m2, v2 = orc.forward(case.ro.obs, case.ro.critic_obs)
    em = np.linalg.norm(mean - m2) / np.linalg.norm(m2)
    ev = np.linalg.norm(value - v2) / np.linalg.norm(v2)
    assert em < TOL and ev < TOL, (em, ev)


def test_bf16_gradient(case):
    gpu = case.gpu_ac("bf16")
    orc = case.oracle_ac()
    idx = O.shuffle(3, case.ro.n)
    g, s = gpu.minibatch_grads(case.soa(), idx, Z.PpoConfig())
    g2, s2 = orc.minibatch_grads(case.oracle_batch(), idx, O.PpoConfig(), n_threads=8)
    errs = tensor_l2(g, g2, case.adims, case.cdims)
    bad = {k: v for k, v in errs.items() if v > TOL_GRAD}
    assert not bad, bad
    np.testing.assert_allclose(s, s2, rtol=TOL_GRAD, atol=1e-4)


def test_bf16_update_moves_like_the_oracle(case):
    gpu = case.gpu_ac("bf16", lr=1e-3)
    orc = case.oracle_ac(lr=1e-3)
    cfg = Z.PpoConfig(epochs=2, minibatches=4, adaptive_lr=False)
    st = gpu.update(case.soa(), cfg)
    st2 = orc.update(case.oracle_batch(), O.PpoConfig(epochs=2, minibatches=4, adaptive_lr=False))
    d_gpu = gpu.params - case.params
    d_orc = orc.params - case.params
    # Adam's early steps are about lr * sign(g): the direction of the whole
    # parameter change is what must agree
    cos = float(d_gpu @ d_orc / (np.linalg.norm(d_gpu) * np.linalg.norm(d_orc)))
    assert cos > 0.97, cos
    assert abs(st.value_loss - st2["value_loss"]) <= TOL * abs(st2["value_loss"])


TOL_BF = 2e-3


def _bf16_oracle(case, lr=None):
    orc = case.oracle_ac() if lr is None else case.oracle_ac(lr=lr)
    orc.set_bf16_operands()
    return orc


def test_bf16_forward_matches_the_bf16_oracle(case):
    gpu = case.gpu_ac("bf16")
    mean, value = gpu.forward(case.ro.obs, case.ro.critic_obs)
    m2, v2 = _bf16_oracle(case).forward(case.ro.obs, case.ro.critic_obs)
    em = np.linalg.norm(mean - m2) / np.linalg.norm(m2)
    ev = np.linalg.norm(value - v2) / np.linalg.norm(v2)
    assert em < TOL_BF and ev < TOL_BF, (em, ev)


def test_bf16_gradient_matches_the_bf16_oracle(case):
    gpu = case.gpu_ac("bf16")
    idx = O.shuffle(3, case.ro.n)
    g, s = gpu.minibatch_grads(case.soa(), idx, Z.PpoConfig())
    g2, s2 = _bf16_oracle(case).minibatch_grads(case.oracle_batch(), idx, O.PpoConfig(),
                                                n_threads=8)
    errs = tensor_l2(g, g2, case.adims, case.cdims)
    bad = {k: v for k, v in errs.items() if v > TOL_BF}
    assert not bad, bad
    np.testing.assert_allclose(s, s2, rtol=1e-3, atol=1e-5)


def test_bf16_update_matches_the_bf16_oracle(case):
    cfg = Z.PpoConfig(epochs=2, minibatches=4, adaptive_lr=False)
    gpu = case.gpu_ac("bf16", lr=1e-3)
    st = gpu.update(case.soa(), cfg)
    orc = _bf16_oracle(case, lr=1e-3)
    st2 = orc.update(case.oracle_batch(), O.PpoConfig(epochs=2, minibatches=4, adaptive_lr=False))
    d_gpu = gpu.params - case.params
    d_orc = orc.params - case.params
    l2 = tensor_l2(d_gpu, d_orc, case.adims, case.cdims)
    bad = {k: v for k, v in l2.items() if v > 2e-2}
    assert not bad, bad
    cos = float(d_gpu @ d_orc / (np.linalg.norm(d_gpu) * np.linalg.norm(d_orc)))
    assert cos > 0.999, cos
    for k in ("kl", "surrogate", "value_loss", "entropy"):
        assert abs(getattr(st, k) - st2[k]) <= 2e-3 * max(abs(st2[k]), 1e-3), (k, st, st2)
