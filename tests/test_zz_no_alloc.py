"""zrl_gae_normalize_noalloc against the allocating entry points.

The no-allocation entry point exists for callers that cannot call cudaMalloc
where they need advantages (their GPU memory belongs to another runtime's
pool, or their loop forbids allocation).  It must give what the allocating path gives: GAE advantages and
returns bit-identical to zrl_gae's, and normalized advantages within 1e-5
(the tolerance of the advantage tests) of those zrl_update writes back.
Two calls in a row with different sizes check that the scratch array it
shares between calls carries nothing over.  This file is collected last so
that a stopping run has executed every other test first; it also passes on
its own in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

from zealot_b200 import native as N
from zealot_b200 import zealot_rl as Z

pytestmark = pytest.mark.gpu

MAX_ENVS = 262_144


def _rollout(seed, n_envs, T):
    rng = np.random.default_rng(seed)
    r = (0.1 * rng.standard_normal((n_envs, T))).astype(np.float32)
    v = rng.standard_normal((n_envs, T)).astype(np.float32)
    d = (rng.random((n_envs, T)) < 0.05).astype(np.uint8)
    lv = rng.standard_normal(n_envs).astype(np.float32)
    return r, v, d, lv


def _reference(ctx, r, v, d, lv, gamma, lam):
    """The allocating path: zrl_gae, then zrl_update with no epochs (only the
    advantage normalization, written back)."""
    n_envs, T = r.shape
    adv = np.empty_like(r)
    ret = np.empty_like(r)
    ctx.call("zrl_gae", N.ptr(r), N.ptr(v), N.ptr(d), N.ptr(lv), n_envs, T, gamma, lam,
             N.ptr(adv), N.ptr(ret), 0)
    n = n_envs * T
    z4 = np.zeros((n, 4), np.float32)
    z1 = np.zeros(n, np.float32)
    batch = Z.SoaBatch(obs=z4, critic_obs=z4, action=np.zeros((n, 2), np.float32),
                       mean_old=np.zeros((n, 2), np.float32), logp_old=z1, value_old=z1,
                       adv=adv.reshape(-1).copy(), ret=ret.reshape(-1))
    st = N.StatsC()
    cfg = Z.PpoConfig(epochs=0, minibatches=1).c()
    bc = batch.c(write_back_adv=True)
    ctx.call("zrl_update", C.byref(cfg), C.byref(bc), C.byref(st))
    return adv, ret, batch.adv


def _noalloc(torch, r, v, d, lv, gamma, lam):
    dev = torch.device("cuda")
    t = [torch.from_numpy(x).to(dev) for x in (r, v, d, lv)]
    adv = torch.full(r.shape, float("nan"), device=dev)
    ret = torch.full(r.shape, float("nan"), device=dev)
    norm = torch.full(r.shape, float("nan"), device=dev)
    st = N.lib().zrl_gae_normalize_noalloc(
        t[0].data_ptr(), t[1].data_ptr(), t[2].data_ptr(), t[3].data_ptr(),
        r.shape[0], r.shape[1], gamma, lam, adv.data_ptr(), ret.data_ptr(),
        norm.data_ptr(), None)
    assert st == N.OK
    torch.cuda.synchronize()
    return adv.cpu().numpy(), ret.cpu().numpy(), norm.cpu().numpy().reshape(-1)


def test_noalloc_matches_allocating_path_twice():
    import torch
    ctx = Z.Context((4, 8, 2), (4, 8, 1), precision="fp32")
    # first a large call, then a smaller one: stale partial sums of the first
    # call sit in the shared scratch and must not leak into the second
    for seed, n_envs, T in ((1, 3000, 24), (2, 57, 48)):
        r, v, d, lv = _rollout(seed, n_envs, T)
        a_ref, r_ref, n_ref = _reference(ctx, r, v, d, lv, 0.99, 0.95)
        a, rt, nrm = _noalloc(torch, r, v, d, lv, 0.99, 0.95)
        assert np.array_equal(a, a_ref) and np.array_equal(rt, r_ref)
        err = np.abs(nrm - n_ref).max() / np.abs(n_ref).max()
        assert err <= 1e-5, err
        assert abs(float(nrm.mean())) < 1e-4 and abs(float(nrm.std()) - 1.0) < 1e-4


def test_noalloc_rejects_sizes_beyond_its_scratch():
    import torch
    x = torch.zeros(16, device="cuda")
    p = x.data_ptr()
    st = N.lib().zrl_gae_normalize_noalloc(p, p, p, p, MAX_ENVS + 1, 1, 0.99, 0.95,
                                           p, p, p, None)
    assert st == N.INVALID_ARG
    assert bool(torch.all(x == 0))  # nothing was written
