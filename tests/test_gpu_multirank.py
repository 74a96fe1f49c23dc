"""Two ranks on two GPUs through the C ABI: the data-parallel update (rows
sharded by rank, NCCL allreduce of each minibatch gradient, ppo.rs:350-383
per rank) against one GPU running the whole batch.  Skipped with fewer
than two GPUs.

Each rank runs three updates in a row, so the path a trainer takes runs
too: the second and third updates use the epoch orders that the update
before queued on the device at its end (their per-minibatch counts arrive
with that update's closing synchronization).  After every update the
parameters of the two ranks must be identical and the parameter change
must agree with the one-GPU run:

* fp32 CUDA-core mode (toy dims): the two runs differ only in the order the
  per-row gradient terms are summed (per rank, then across ranks): 1e-4
  relative L2 on the change since the start;
* tf32 tensor-core mode with the C2 dims and 6,144 rows per rank: forward
  and input gradients are row-local, only the weight-gradient sums are
  split differently; after three updates (30 Adam steps, which amplify
  summation noise where a gradient element is near zero) 1e-3 relative L2.
Statistics agree within 1e-3 (fp32) and 1e-2 (tf32) relative.
"""
from __future__ import annotations

import numpy as np
import pytest

from tests.helpers import C_A, C_C, SMALL_A, SMALL_C, Case

pytestmark = pytest.mark.gpu

WORLD = 2
UPDATES = 3

CONFIGS = {
    "fp32_small": dict(dims=(SMALL_A, SMALL_C), n_envs=16, T=12, precision="fp32",
                       epochs=2, minibatches=4, tol=1e-4, stats_tol=1e-3),
    "tf32_c2dims": dict(dims=(C_A, C_C), n_envs=512, T=24, precision="tf32",
                        epochs=2, minibatches=2, tol=1e-3, stats_tol=1e-2),
}


def _case(name):
    c = CONFIGS[name]
    return Case(*c["dims"], n_envs=c["n_envs"], T=c["T"], seed=3, perturb=0.05)


def _cfg(name):
    from zealot_b200 import zealot_rl as Z
    c = CONFIGS[name]
    return Z.PpoConfig(epochs=c["epochs"], minibatches=c["minibatches"])


def _rank(name, rank, q_id, q_out):
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
    case = _case(name)
    n = case.ro.n
    n_local = n // WORLD
    lo = rank * n_local
    full = case.soa()
    ac = Z.ActorCritic(case.adims, case.cdims, precision=CONFIGS[name]["precision"],
                       device=rank, comm=comm)
    ac.params = case.params
    out = []
    for _ in range(UPDATES):
        part = Z.SoaBatch(**{f: np.ascontiguousarray(getattr(full, f)[lo:lo + n_local])
                             for f in ("obs", "critic_obs", "action", "mean_old", "logp_old",
                                       "value_old", "adv", "ret")})
        st = ac.update(part, _cfg(name), n_global=n, row_offset=lo)
        out.append((ac.params.copy(), (st.kl, st.surrogate, st.value_loss)))
    q_out.put((rank, out))
    ac.close()


@pytest.mark.parametrize("name", list(CONFIGS))
def test_two_gpu_updates_match_one_gpu(name):
    import torch
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q_id, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(name, r, q_id, q_out)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = dict(q_out.get(timeout=600) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0

    from zealot_b200 import zealot_rl as Z
    case = _case(name)
    ac = Z.ActorCritic(case.adims, case.cdims, precision=CONFIGS[name]["precision"], device=0)
    ac.params = case.params
    tol = CONFIGS[name]["tol"]
    for u in range(UPDATES):
        st = ac.update(case.soa(), _cfg(name))
        one = ac.params.copy()
        p0, s0 = res[0][u]
        p1, _ = res[1][u]
        # both ranks end every update with the same parameters
        np.testing.assert_array_equal(p0, p1)
        d_dp = p0 - case.params
        d_one = one - case.params
        err = np.linalg.norm(d_dp - d_one) / np.linalg.norm(d_one)
        assert err < tol, (u, err)
        np.testing.assert_allclose(s0, (st.kl, st.surrogate, st.value_loss),
                                   rtol=CONFIGS[name]["stats_tol"], atol=1e-6)
    ac.close()
