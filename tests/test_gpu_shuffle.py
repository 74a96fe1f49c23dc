"""The device epoch permutation (zrl_shuffle_device) against the host
Fisher-Yates loop of ppo.rs:357-363 (zrl_shuffle, itself pinned to the
oracle's Lcg): bit-exact, from tiny n to the 8-GPU C4 sample count."""
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


@pytest.mark.parametrize("n_global,world,mbs,seed", [(96, 2, 4, 1), (1536, 4, 4, 7),
                                                     (1000, 3, 7, 21), (98, 8, 5, 2),
                                                     (786432, 8, 4, 13), (1572864, 8, 4, 5)])
def test_device_rank_orders_match_host(n_global, world, mbs, seed):
    """zrl_rank_orders_device (device permutation + order-keeping
    compaction) equals the host zrl_rank_orders for every rank."""
    import torch
    ctx = Z.Context((4, 4), (4, 1), precision="tf32")
    n_local = n_global // world
    for r in range(world):
        off = r * n_local
        order = np.full(n_local + 1, -9, np.int32)
        counts = np.zeros(mbs, np.int64)
        n = N.lib().zrl_rank_orders(seed, n_global, n_local, off, mbs, order.ctypes.data,
                                    counts.ctypes.data)
        dev = torch.full((n_local + 1,), -9, dtype=torch.int32, device="cuda")
        dcounts = np.zeros(mbs, np.int64)
        torch.cuda.synchronize()
        nd = N.lib().zrl_rank_orders_device(ctx.h, seed, n_global, n_local, off, mbs,
                                            dev.data_ptr(), dcounts.ctypes.data)
        assert nd == n
        np.testing.assert_array_equal(dcounts, counts)
        np.testing.assert_array_equal(dev.cpu().numpy(), order)
