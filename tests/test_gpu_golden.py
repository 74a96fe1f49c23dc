"""The CUDA library on the C1 golden fixture (tests/golden/c1_golden.npz):
GAE and the epoch permutation bit-exact, the fp32-mode minibatch gradient
and one whole update close to the oracle's stored results."""
from __future__ import annotations

import os

import numpy as np
import pytest

from tests.golden import make_golden as G

pytestmark = pytest.mark.gpu

PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "c1_golden.npz")


@pytest.fixture(scope="module")
def case():
    g = dict(np.load(PATH))
    params, obs, cobs, rewards, dones, eps = G.inputs()
    o = np.ascontiguousarray(obs[:, :G.T].reshape(-1, G.ADIMS[0]), np.float32)
    c = np.ascontiguousarray(cobs[:, :G.T].reshape(-1, G.CDIMS[0]), np.float32)
    return g, params, o, c, rewards, dones


def _batch(Z, g, o, c, adv):
    return Z.SoaBatch(obs=o, critic_obs=c, action=g["action"], mean_old=g["mean_old"],
                      logp_old=g["logp_old"], value_old=g["value_old"], adv=adv, ret=g["ret"])


def test_gae_and_permutation_bit_exact(case):
    from zealot_b200 import zealot_rl as Z
    g, params, o, c, rewards, dones = case
    from zealot_b200 import native as N
    ac = Z.ActorCritic(G.ADIMS, G.CDIMS, precision="tf32")
    r = np.ascontiguousarray(rewards, np.float32)
    v = np.ascontiguousarray(g["value_old"], np.float32)
    d = np.ascontiguousarray(dones, np.uint8)
    lv = np.ascontiguousarray(g["last_values"], np.float32)
    adv = np.empty(G.N_ENVS * G.T, np.float32)
    ret = np.empty_like(adv)
    ac.ctx.call("zrl_gae", N.ptr(r), N.ptr(v), N.ptr(d), N.ptr(lv), G.N_ENVS, G.T,
                0.99, 0.95, N.ptr(adv), N.ptr(ret), 0)
    np.testing.assert_array_equal(adv, g["adv"])
    np.testing.assert_array_equal(ret, g["ret"])
    np.testing.assert_array_equal(Z.shuffle(1, G.N_ENVS * G.T), g["perm"])
    ac.close()


def test_fp32_gradient_and_update(case):
    from zealot_b200 import zealot_rl as Z
    g, params, o, c, rewards, dones = case
    ac = Z.ActorCritic(G.ADIMS, G.CDIMS, precision="fp32")
    ac.params = params
    ac.lr = 1e-3
    cfg = Z.PpoConfig(epochs=1, minibatches=1, adaptive_lr=False)
    grads, sums = ac.minibatch_grads(_batch(Z, g, o, c, g["adv"].copy()), g["perm"], cfg)
    sample = np.asarray(grads, np.float32)[::G.STRIDE]
    err = np.abs(sample - g["grads_sample"]).max() / np.abs(g["grads_sample"]).max()
    assert err < 1e-4, err
    np.testing.assert_allclose(sums, g["sums3"], rtol=1e-4, atol=1e-7)
    ac.params = params
    st = ac.update(_batch(Z, g, o, c, g["adv"].copy()), cfg)
    d_gpu = (ac.params - params)[::G.STRIDE]
    d_ref = g["new_params_sample"] - params[::G.STRIDE]
    rel = np.linalg.norm(d_gpu - d_ref) / np.linalg.norm(d_ref)
    assert rel < 1e-3, rel
    np.testing.assert_allclose([st.kl, st.surrogate, st.value_loss], g["stats"][:3],
                               rtol=1e-3, atol=1e-6)
    ac.close()
