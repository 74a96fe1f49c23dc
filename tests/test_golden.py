"""The C1 golden fixture (tests/golden/c1_golden.npz, made by
tests/golden/make_golden.py): its inputs regenerate bit-exactly from the
reference Lcg, and the CPU oracle reproduces every stored output exactly
(single-threaded, the reference's sequential order) -- a pin of the oracle
against drift, next to the known-answer tests of test_oracle.py."""
from __future__ import annotations

import os

import numpy as np
import pytest

from tests.golden import make_golden as G

PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "c1_golden.npz")


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(PATH))


@pytest.fixture(scope="module")
def fresh():
    return G.compute()


def test_inputs_regenerate(golden):
    params, obs, cobs, rewards, dones, eps = G.inputs()
    np.testing.assert_array_equal(G.summary(params)[0], golden["params_summary"])
    np.testing.assert_array_equal(G.summary(params)[1], golden["params_sample"])
    o = obs[:, :G.T].reshape(-1, G.ADIMS[0])
    np.testing.assert_array_equal(G.summary(o)[0], golden["obs_summary"])


@pytest.mark.parametrize("key", ["mean_old", "value_old", "logp_old", "last_values", "action",
                                 "adv", "ret", "perm", "grads_summary", "grads_sample", "sums3",
                                 "new_params_summary", "new_params_sample", "adv_normalized",
                                 "stats"])
def test_oracle_reproduces(golden, fresh, key):
    np.testing.assert_array_equal(fresh[key], golden[key])
