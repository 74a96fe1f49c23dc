"""The normalizers' statistics on the device against the oracle
(ppo.rs:104-195): PendingNorm::push, Normalizer::commit and
Normalizer::update (record_obs).

* the sequential fold (mode 0) and commit: bit-exact;
* the parallel fold (mode 1, 256-row chunks merged with the commit formula):
  within 1e-5 relative of the exact statistics, up to a C2 rollout's 98,304
  rows and on ragged row counts (the sequential f32 fold itself drifts by
  2e-5 over that many rows).
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from helpers import SMALL_A, SMALL_C
from zealot_b200 import zealot_rl as Z

pytestmark = pytest.mark.gpu


def _oracle_fold(mean, m2, count, rows):
    mean, m2 = mean.copy(), m2.copy()
    c = C.c_float(count)
    for r in rows:
        O.lib().orc_norm_update(mean, m2, C.byref(c), np.ascontiguousarray(r), len(r))
    return mean, m2, c.value


def _rows(seed, n):
    g = np.random.default_rng(seed)
    obs = (g.standard_normal((n, SMALL_A[0])) * 3 + 1).astype(np.float32)
    cobs = (g.standard_normal((n, SMALL_C[0])) * 0.5 - 2).astype(np.float32)
    return obs, cobs


def test_pending_push_and_commit_bit_exact():
    ac = Z.ActorCritic(SMALL_A, SMALL_C, precision="fp32")
    # live statistics first (record_obs), then a pending batch in two pushes
    live_o, live_c = _rows(1, 50)
    ac.record_obs(live_o, live_c)
    p1, p2 = _rows(2, 300), _rows(3, 123)
    ac.pending_push(*p1)
    ac.pending_push(*p2)
    om, om2, oc, cm, cm2, cc = ac.pending()
    zo, zc = np.zeros(SMALL_A[0], np.float32), np.zeros(SMALL_C[0], np.float32)
    eo = _oracle_fold(zo, zo, 0.0, np.concatenate([p1[0], p2[0]]))
    ec = _oracle_fold(zc, zc, 0.0, np.concatenate([p1[1], p2[1]]))
    assert np.array_equal(om, eo[0]) and np.array_equal(om2, eo[1]) and oc == eo[2] == 423
    assert np.array_equal(cm, ec[0]) and np.array_equal(cm2, ec[1]) and cc == ec[2]
    # the live normalizers are untouched until commit
    lo = _oracle_fold(zo, np.ones_like(zo), 1.0, live_o)
    lc = _oracle_fold(zc, np.ones_like(zc), 1.0, live_c)
    got = ac.normalizers()
    assert np.array_equal(got[0], lo[0]) and np.array_equal(got[1], lo[1]) and got[2] == lo[2]
    ac.commit_pending()
    want = []
    for live, pend in ((lo, eo), (lc, ec)):
        m, s, c = live[0].copy(), live[1].copy(), C.c_float(live[2])
        pm, ps, pc = pend[0].copy(), pend[1].copy(), C.c_float(pend[2])
        O.lib().orc_norm_commit(m, s, C.byref(c), pm, ps, C.byref(pc), len(m))
        want.append((m, s, c.value))
    got = ac.normalizers()
    assert np.array_equal(got[0], want[0][0]) and np.array_equal(got[1], want[0][1])
    assert got[2] == want[0][2]
    assert np.array_equal(got[3], want[1][0]) and np.array_equal(got[4], want[1][1])
    assert got[5] == want[1][2]
    # the pending state is empty again; an empty commit changes nothing
    assert ac.pending()[2] == 0.0 and not ac.pending()[0].any()
    ac.commit_pending()
    again = ac.normalizers()
    assert all(np.array_equal(a, b) for a, b in zip(again, got))


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def _stats64(rows):
    x = rows.astype(np.float64)
    mu = x.mean(0)
    return float(len(x)), mu, ((x - mu) ** 2).sum(0)


def _merge64(a, b):
    n1, m1, s1 = a
    n2, m2, s2 = b
    tot = n1 + n2
    d = m2 - m1
    return tot, m1 + d * n2 / tot, s1 + s2 + d * d * n1 * n2 / tot


@pytest.mark.parametrize("n", [1, 255, 257, 5000, 98_304])
def test_parallel_fold_matches_exact_statistics(n):
    """The parallel fold against the exact (float64) statistics of the same
    rows: within 1e-5 relative.  The sequential fold (the reference's f32
    recurrence) is held to 1e-4 of the same truth: over 10^5 rows its own
    rounding reaches 2e-5 of m2."""
    rows = _rows(10 + n, n)
    seq = Z.ActorCritic(SMALL_A, SMALL_C, precision="fp32")
    par = Z.ActorCritic(SMALL_A, SMALL_C, precision="fp32")
    seq.pending_push(*rows)
    par.pending_push(*rows, parallel=True)
    a, b = seq.pending(), par.pending()
    assert a[2] == b[2] == n and a[5] == b[5] == n
    for k, (im, is2) in enumerate(((0, 1), (3, 4))):
        _, mu, m2 = _stats64(rows[k])
        assert _rel(b[im], mu) < 1e-5 and _rel(b[is2], m2) < 1e-5, (k, _rel(b[is2], m2))
        assert _rel(a[im], mu) < 1e-4 and _rel(a[is2], m2) < 1e-4
    # the live update (record_obs) in parallel on top of existing statistics
    prior = _rows(7, 40)
    seq.record_obs(*prior)
    par.record_obs(*prior)
    start = seq.normalizers()
    seq.record_obs_rows(*rows)
    par.record_obs_rows(*rows, parallel=True)
    a, b = seq.normalizers(), par.normalizers()
    assert a[2] == b[2] == 41 + n
    for k, (im, is2, ic) in enumerate(((0, 1, 2), (3, 4, 5))):
        s0 = (float(start[ic]), start[im].astype(np.float64), start[is2].astype(np.float64))
        _, mu, m2 = _merge64(s0, _stats64(rows[k]))
        assert _rel(b[im], mu) < 1e-5 and _rel(b[is2], m2) < 1e-5, (k, _rel(b[is2], m2))
        assert _rel(a[im], mu) < 1e-4 and _rel(a[is2], m2) < 1e-4


def test_device_rows():
    import torch
    rows = _rows(21, 777)
    host = Z.ActorCritic(SMALL_A, SMALL_C, precision="fp32")
    dev = Z.ActorCritic(SMALL_A, SMALL_C, precision="fp32")
    host.pending_push(*rows)
    dev.pending_push(torch.from_numpy(rows[0]).cuda(), torch.from_numpy(rows[1]).cuda())
    assert all(np.array_equal(np.asarray(x), np.asarray(y))
               for x, y in zip(host.pending(), dev.pending()))
