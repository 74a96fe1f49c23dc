"""Failure detection without a GPU fault.

CPU (fakes): the bounded stream wait of the several-rank path -- the poll of
the stream and of NCCL's asynchronous error that aborts the communicator on
a timeout or an error (zrl_comm.cpp) -- driven through zrl_test_comm_wait.

GPU: a tensor-core pipeline wait made to run out (zrl_test_stall_next_gemm:
the MMA issuer waits on a barrier nothing completes) under a 5 ms wait
limit; the update returns ZRL_TIMEOUT, the kernel's other roles give up in
turn, and the context then runs a correct update again.
"""
import ctypes as C
import time

import numpy as np
import pytest

from zealot_b200 import native as N


@pytest.mark.parametrize("scenario,status,aborted", [
    (0, N.OK, 0),           # the stream completes
    (1, N.TIMEOUT, 1),      # a peer never arrives: timeout, communicator aborted
    (2, N.NCCL_ERROR, 1),   # NCCL reports an asynchronous error: aborted
    (3, N.CUDA_ERROR, 0),   # a kernel failed on the stream
])
def test_comm_wait_failure_paths(scenario, status, aborted):
    ab = C.c_int32(-1)
    t0 = time.time()
    st = N.lib().zrl_test_comm_wait(scenario, 200, C.byref(ab))
    dt = time.time() - t0
    assert st == status and ab.value == aborted
    if scenario == 1:
        assert 0.2 <= dt < 5.0   # bounded by the timeout, not longer
    else:
        assert dt < 1.0


def test_comm_wait_rejects_bad_arguments():
    ab = C.c_int32(0)
    assert N.lib().zrl_test_comm_wait(9, 10, C.byref(ab)) == N.INVALID_ARG


@pytest.mark.gpu
def test_gemm_wait_runs_out_and_the_context_recovers():
    from helpers import C_A, C_C, Case
    from zealot_b200 import zealot_rl as Z
    case = Case(C_A, C_C, n_envs=16, T=24, seed=31, perturb=0.02)
    cfg = Z.PpoConfig(epochs=1, minibatches=2)
    ref = case.gpu_ac("tf32")
    ref.update(case.soa(), cfg)
    want = ref.params.copy()

    ac = case.gpu_ac("tf32")
    N.check(N.lib().zrl_set_wait_limit(ac.ctx.h, 5_000_000), ac.ctx.h)   # 5 ms
    N.check(N.lib().zrl_test_stall_next_gemm(ac.ctx.h), ac.ctx.h)
    t0 = time.time()
    with pytest.raises(N.ZrlError) as e:
        ac.update(case.soa(), cfg)
    assert e.value.status == N.TIMEOUT
    assert "timed out" in str(e.value)
    assert time.time() - t0 < 10.0
    # usable again: same starting point, same result as a fresh context
    ac.params = case.params
    # (the arrays must outlive the call: an address taken from a temporary
    # points at freed memory by the time the library reads it)
    t3 = np.zeros(3, np.int32)
    m0 = np.zeros(ac.ctx.np, np.float32)
    v0 = np.zeros(ac.ctx.np, np.float32)
    N.check(N.lib().zrl_set_adam_state(ac.ctx.h, t3.ctypes.data, m0.ctypes.data,
                                       v0.ctypes.data, ac.ctx.np), ac.ctx.h)
    ac.lr = ref_lr = 1e-3
    ref2 = case.gpu_ac("tf32", lr=ref_lr)
    ref2.update(case.soa(), cfg)
    ac.update(case.soa(), cfg)
    assert np.array_equal(ac.params, ref2.params)
