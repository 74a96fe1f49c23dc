"""Generate the C1 golden fixture (tests/golden/c1_golden.npz).

Workload C1 (the CPU-runnable case): 64 envs x 24 steps, actor
96-512-256-128-29, critic 96-512-256-128-1, 1 epoch x 1 minibatch, Adam lr
1e-3, adaptive LR off, seed 0.  Every input comes from the reference Lcg
(rng.rs), so it is regenerated bit-exactly from the seed:

  params   Xavier-uniform, U(+-sqrt(6/(fan_in+fan_out))) = (2u-1)*a with
           u = Lcg.unit(), layer by layer (actor first), biases 0, log_std 0
  obs      gauss(), [envs][T+1][96], then critic obs the same way
  rewards  0.1 * gauss(), [envs][T];  dones  unit() < 0.005, [envs][T]
  eps      gauss(), [envs*T][29]

The rollout policy outputs (mean_old, value_old, last_values), logp_old and
every expected output come from the CPU oracle (oracle/zrl_oracle.c, the C
restatement of zealot-rl): GAE advantages/returns (ppo.rs:681-703), the
epoch permutation (ppo.rs:356-363), the minibatch gradient and statistics
(ppo.rs:388-462, single-threaded: the reference's sequential order) and the
parameters after one update (ppo.rs:338-384).  Large vectors are stored as
per-tensor sums, L2 norms and every 97th element, which keeps the file
small and still pins them.

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle as O  # noqa: E402

ADIMS = (96, 512, 256, 128, 29)
CDIMS = (96, 512, 256, 128, 1)
N_ENVS, T, SEED = 64, 24, 0
STRIDE = 97


def inputs(seed: int = SEED):
    rng = O.Lcg(seed)
    parts = []
    for dims in (ADIMS, CDIMS):
        for l in range(len(dims) - 1):
            fi, fo = dims[l], dims[l + 1]
            a = np.float32(np.sqrt(6.0 / (fi + fo)))
            u = rng.units(fo * fi)
            parts.append(((np.float32(2.0) * u - np.float32(1.0)) * a).astype(np.float32))
            parts.append(np.zeros(fo, np.float32))
    parts.append(np.zeros(ADIMS[-1], np.float32))
    params = np.concatenate(parts)
    obs = rng.gausses(N_ENVS * (T + 1) * ADIMS[0]).reshape(N_ENVS, T + 1, ADIMS[0])
    cobs = rng.gausses(N_ENVS * (T + 1) * CDIMS[0]).reshape(N_ENVS, T + 1, CDIMS[0])
    rewards = (np.float32(0.1) * rng.gausses(N_ENVS * T)).astype(np.float32).reshape(N_ENVS, T)
    dones = (rng.units(N_ENVS * T) < np.float32(0.005)).astype(np.uint8).reshape(N_ENVS, T)
    eps = rng.gausses(N_ENVS * T * ADIMS[-1]).reshape(N_ENVS * T, ADIMS[-1])
    return params, obs, cobs, rewards, dones, eps


def rollout(params, obs, cobs, eps):
    ac = O.ActorCritic(ADIMS, CDIMS)
    ac.params = params
    o = np.ascontiguousarray(obs[:, :T].reshape(-1, ADIMS[0]), np.float32)
    c = np.ascontiguousarray(cobs[:, :T].reshape(-1, CDIMS[0]), np.float32)
    mean_old, value_old = ac.forward(o, c)
    log_std = params[-ADIMS[-1]:]
    action = (mean_old + np.exp(log_std)[None, :] * eps).astype(np.float32)
    logp_old = np.array([ac.logp(action[i], mean_old[i]) for i in range(len(action))],
                        np.float32)
    _, last_values = ac.forward(np.ascontiguousarray(obs[:, T], np.float32),
                                np.ascontiguousarray(cobs[:, T], np.float32))
    return o, c, action, np.asarray(mean_old, np.float32), logp_old, \
        np.asarray(value_old, np.float32), np.asarray(last_values, np.float32)


def summary(v):
    v = np.asarray(v, np.float64)
    return np.array([v.sum(), np.sqrt((v * v).sum())]), np.asarray(v[::STRIDE], np.float32)


def compute():
    params, obs, cobs, rewards, dones, eps = inputs()
    o, c, action, mean_old, logp_old, value_old, last_values = rollout(params, obs, cobs, eps)
    adv, ret = O.gae_batch(rewards, value_old.reshape(N_ENVS, T), dones, last_values, 0.99, 0.95)
    adv = adv.reshape(-1).astype(np.float32)
    ret = ret.reshape(-1).astype(np.float32)
    batch = O.SoaBatch(obs=o, critic_obs=c, action=action, mean_old=mean_old,
                       logp_old=logp_old, value_old=value_old, adv=adv, ret=ret)
    cfg = O.PpoConfig(epochs=1, minibatches=1, adaptive_lr=False)
    ac = O.ActorCritic(ADIMS, CDIMS)
    ac.params = params
    ac.lr = 1e-3
    perm = O.shuffle(1, N_ENVS * T)  # step 0, epoch 0: Lcg seed 0 + 0 + 1
    grads, sums = ac.minibatch_grads(batch, perm, cfg)
    upd = batch.copy()
    stats = ac.update(upd, cfg)
    out = dict(
        params_summary=summary(params)[0], params_sample=summary(params)[1],
        obs_summary=summary(o)[0], cobs_summary=summary(c)[0],
        mean_old=mean_old, value_old=value_old, logp_old=logp_old, last_values=last_values,
        action=action, adv=adv, ret=ret, perm=np.asarray(perm, np.int32),
        grads_summary=summary(grads)[0], grads_sample=summary(grads)[1], sums3=sums,
        new_params_summary=summary(ac.params)[0], new_params_sample=summary(ac.params)[1],
        adv_normalized=upd.adv,
        stats=np.array([stats["kl"], stats["surrogate"], stats["value_loss"], stats["entropy"],
                        stats["lr"]], np.float32))
    return out


if __name__ == "__main__":
    out = compute()
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "c1_golden.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path), "bytes")
