"""The several-rank minibatch orders (zrl_rank_orders, the host code the
data-parallel update runs) against a restatement on the oracle's shuffle:
rank r of a world holds rows [r * n_local, (r + 1) * n_local); per global
minibatch slice of the epoch permutation (ppo.rs:356-367) it keeps the
positions it holds, as local rows, in permutation order.  Runs on CPU."""
import numpy as np
import pytest

import oracle as O
from zealot_b200 import native as N


def _reference(seed, n_global, n_local, row_offset, mbs):
    perm = np.asarray(O.shuffle(seed, n_global), np.int64)
    mb = n_global // mbs
    order, counts = [], []
    for m in range(mbs):
        sel = perm[m * mb:(m + 1) * mb] - row_offset
        sel = sel[(sel >= 0) & (sel < n_local)]
        order.append(sel)
        counts.append(len(sel))
    return np.concatenate(order).astype(np.int32), np.asarray(counts, np.int64)


@pytest.mark.parametrize("n_global,world,mbs,seed", [(96, 2, 4, 1), (1536, 4, 4, 7),
                                                     (1000, 3, 7, 21), (98, 8, 5, 2),
                                                     (24576, 8, 4, 13)])
def test_rank_orders_match_reference(n_global, world, mbs, seed):
    n_local = n_global // world
    seen = np.zeros(n_global, np.int64)
    for r in range(world):
        off = r * n_local
        order = np.full(n_local + 1, -9, np.int32)
        counts = np.zeros(mbs, np.int64)
        n = N.lib().zrl_rank_orders(seed, n_global, n_local, off, mbs, order.ctypes.data,
                                    counts.ctypes.data)
        want_o, want_c = _reference(seed, n_global, n_local, off, mbs)
        assert n == len(want_o)
        np.testing.assert_array_equal(order[:n], want_o)
        np.testing.assert_array_equal(counts, want_c)
        assert order[n] == -9  # nothing past the rank's rows
        seen[order[:n].astype(np.int64) + off] += 1
    # every sample of the used slices lands on exactly one rank
    mb = n_global // mbs
    used = np.asarray(O.shuffle(seed, n_global), np.int64)[:mb * mbs]
    held = used[used < world * n_local]
    assert seen[held].tolist() == [1] * len(held)


def test_rank_orders_rejects_bad_arguments():
    order = np.zeros(4, np.int32)
    counts = np.zeros(2, np.int64)
    assert N.lib().zrl_rank_orders(1, 0, 4, 0, 2, order.ctypes.data, counts.ctypes.data) == -1
    assert N.lib().zrl_rank_orders(1, 8, 4, 0, 0, order.ctypes.data, counts.ctypes.data) == -1
