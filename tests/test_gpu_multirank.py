"""Two ranks on two GPUs through the C ABI: the data-parallel update (rows
sharded by rank, NCCL allreduce of each minibatch gradient, ppo.rs:350-383
per rank) against one GPU running the whole batch.  Skipped with fewer
than two GPUs.

Both runs use the fp32 CUDA-core mode, so they differ only in the order the
per-row gradient terms are summed (per rank, then across ranks); the
parameter change of the update must agree to 1e-4 relative L2.
"""
from __future__ import annotations

import numpy as np
import pytest

from tests.helpers import Case, SMALL_A, SMALL_C

pytestmark = pytest.mark.gpu

WORLD = 2


def _case():
    return Case(SMALL_A, SMALL_C, n_envs=16, T=12, seed=3, perturb=0.05)


def _rank(rank, q_id, q_out):
    import ctypes
    from zealot_b200 import native as N
    from zealot_b200 import zealot_rl as Z
    if rank == 0:
        buf = (ctypes.c_uint8 * 128)()
        N.check(N.lib().zrl_nccl_unique_id(buf))
        for _ in range(WORLD - 1):
            q_id.put(bytes(buf))
        uid = bytes(buf)
    else:
        uid = q_id.get(timeout=120)
    comm = N.CommC()
    comm.rank, comm.world_size, comm.timeout_ms = rank, WORLD, 60000
    for i, v in enumerate(uid):
        comm.nccl_id[i] = v
    case = _case()
    n = case.ro.n
    n_local = n // WORLD
    lo = rank * n_local
    full = case.soa()
    part = Z.SoaBatch(**{f: np.ascontiguousarray(getattr(full, f)[lo:lo + n_local])
                         for f in ("obs", "critic_obs", "action", "mean_old", "logp_old",
                                   "value_old", "adv", "ret")})
    ac = Z.ActorCritic(case.adims, case.cdims, precision="fp32", device=rank, comm=comm)
    ac.params = case.params
    cfg = Z.PpoConfig(epochs=2, minibatches=4)
    st = ac.update(part, cfg, n_global=n, row_offset=lo)
    q_out.put((rank, ac.params.copy(), (st.kl, st.surrogate, st.value_loss)))
    ac.close()


def test_two_gpu_update_matches_one_gpu():
    import torch
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q_id, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, q_id, q_out)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = dict((r, (p, s)) for r, p, s in (q_out.get(timeout=300) for _ in range(WORLD)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # both ranks end with the same parameters
    np.testing.assert_array_equal(res[0][0], res[1][0])

    from zealot_b200 import zealot_rl as Z
    case = _case()
    ac = Z.ActorCritic(case.adims, case.cdims, precision="fp32", device=0)
    ac.params = case.params
    cfg = Z.PpoConfig(epochs=2, minibatches=4)
    st = ac.update(case.soa(), cfg)
    one = ac.params.copy()
    ac.close()
    d_dp = res[0][0] - case.params
    d_one = one - case.params
    rel = np.linalg.norm(d_dp - d_one) / np.linalg.norm(d_one)
    assert rel < 1e-4, rel
    np.testing.assert_allclose(res[0][1], (st.kl, st.surrogate, st.value_loss),
                               rtol=1e-3, atol=1e-6)
