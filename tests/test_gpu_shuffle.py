"""The device epoch permutation (zrl_shuffle_device) against the host
Fisher-Yates loop of ppo.rs:357-363 (zrl_shuffle, itself pinned to the
oracle's Lcg): bit-exact, from tiny n to the 8-GPU C4 sample count."""
import ctypes as C

import numpy as np
import pytest

from zealot_b200 import native as N
from zealot_b200 import zealot_rl as Z

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,seed", [(1, 1), (2, 5), (3, 2), (17, 3), (1000, 7), (98304, 13),
                                    (786432, 21), (1572864, 9), (98304, 2), (98304, 3)])
def test_device_shuffle_matches_host(n, seed):
    import torch
    ctx = Z.Context((4, 4), (4, 1), precision="tf32")
    host = np.empty(n, np.int64)
    N.lib().zrl_shuffle(seed, n, host.ctypes.data)
    dev = torch.full((n,), -7, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    ctx.call("zrl_shuffle_device", seed, n, dev.data_ptr())
    got = dev.cpu().numpy().astype(np.int64)
    np.testing.assert_array_equal(got, host)


def test_device_shuffle_empty():
    ctx = Z.Context((4, 4), (4, 1), precision="tf32")
    ctx.call("zrl_shuffle_device", 1, 0, None)
