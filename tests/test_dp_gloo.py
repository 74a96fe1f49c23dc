"""Data-parallel decomposition of the update, on CPU with two gloo ranks.

The library shards the batch by rows: rank r holds rows
[r * n_local, (r + 1) * n_local), every rank draws the same global epoch
permutation (Lcg seed = step + epoch * minibatches + 1, the order of
ppo.rs:360-366), keeps per minibatch the positions whose rows it holds, and
sums per-rank gradients scaled by 1 / (global minibatch size) with one
allreduce per minibatch.  These tests run that decomposition with the CPU
oracle as the per-rank gradient and torch.distributed (gloo, world size 2)
as the allreduce, and check it against the single-process gradient of each
global minibatch -- the property the multi-GPU path relies on -- with two,
three and four ranks (rank shares of a global minibatch are uneven and may
be empty).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

import oracle as O
from tests.helpers import Case, SMALL_A, SMALL_C

MINIBATCHES = 4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case():
    return Case(SMALL_A, SMALL_C, n_envs=8, T=12, seed=7, perturb=0.05)


def _rank_rows(perm, m, mb, row_off, n_local):
    """Positions of global minibatch m owned by this rank, as local rows (in
    permutation order) -- the per-rank order the library builds."""
    sel = perm[m * mb:(m + 1) * mb] - row_off
    return sel[(sel >= 0) & (sel < n_local)]


def _local_batch(case, lo, hi):
    full = case.soa()
    return O.SoaBatch(**{k: np.ascontiguousarray(getattr(full, k)[lo:hi])
                         for k in ("obs", "critic_obs", "action", "mean_old", "logp_old",
                                   "value_old", "adv", "ret")})


def _worker(rank, world, port, step, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = _case()
        n = case.ro.n
        n_local = n // world
        row_off = rank * n_local
        mb = n // MINIBATCHES
        ac = O.ActorCritic(case.adims, case.cdims)
        ac.params = case.params
        cfg = O.PpoConfig()
        local = _local_batch(case, row_off, row_off + n_local)
        out = []
        for e in range(2):
            perm = O.shuffle(step + e * MINIBATCHES + 1, n)
            for m in range(MINIBATCHES):
                idx = _rank_rows(perm, m, mb, row_off, n_local)
                g = np.zeros(ac.np, np.float32)
                s = np.zeros(3, np.float32)
                if len(idx):
                    g, s = ac.minibatch_grads(local, idx, cfg)
                    # the oracle scales by 1 / len(idx); the library by
                    # 1 / (global minibatch size)
                    g = g * np.float32(len(idx) / mb)
                    s = s * np.float32(len(idx) / mb)
                t = torch.from_numpy(np.concatenate([g, s]).astype(np.float64))
                dist.all_reduce(t)
                out.append((len(idx), t.numpy().astype(np.float32)))
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,step", [(2, 0), (2, 13), (3, 5), (4, 13)])
def test_rank_gradients_sum_to_global_minibatch(world, step):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, step, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    case = _case()
    n = case.ro.n
    mb = n // MINIBATCHES
    ac = O.ActorCritic(case.adims, case.cdims)
    ac.params = case.params
    cfg = O.PpoConfig()
    full = case.soa()
    full = O.SoaBatch(**{k: getattr(full, k) for k in ("obs", "critic_obs", "action", "mean_old",
                                                      "logp_old", "value_old", "adv", "ret")})
    i = 0
    for e in range(2):
        perm = O.shuffle(step + e * MINIBATCHES + 1, n)
        for m in range(MINIBATCHES):
            g, s = ac.minibatch_grads(full, perm[m * mb:(m + 1) * mb], cfg)
            want = np.concatenate([g, s])
            # every global position went to exactly one rank
            assert sum(res[r][i][0] for r in range(world)) == mb
            # every rank holds the same allreduced sum
            for r in range(1, world):
                np.testing.assert_array_equal(res[0][i][1], res[r][i][1])
            got = res[0][i][1]
            err = np.abs(got - want).max() / max(np.abs(want).max(), 1e-30)
            assert err < 1e-5, (e, m, err)
            i += 1
