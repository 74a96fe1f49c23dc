"""Seeded synthetic rollouts for the PPO-update workloads.

There is no environment on this path (physics is out of scope), so every
workload is generated from a seed with numpy's PCG64 generator.  The value
distributions follow the benchmark configurations:

* weights: Xavier-uniform ``U(+-sqrt(6/(fan_in+fan_out)))`` per layer, actor
  first then critic, biases 0, ``log_std`` 0;
* observations and critic observations ~ N(0, 1), T+1 steps per env (the
  last step only feeds the bootstrap value);
* rewards ~ N(0, 0.1^2); dones ~ Bernoulli(0.005);
* actions ``a = mean_old + exp(log_std) * eps`` with eps ~ N(0, 1), and
  ``logp_old`` the diagonal-Gaussian log-prob of ``a`` (ppo.rs:297-305).

``mean_old``/``value_old``/``last_value`` come from a caller-supplied forward
function so that the same generator serves the GPU library (bench) and the
CPU oracle (tests).  Arrays are env-major: sample index ``e*T + t``, as the
reference trainer flattens its rollout (biped_train_gpu.rs:982-987).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

LOG_SQRT_2PI = np.float32(0.9189385)


@dataclass
class Workload:
    name: str
    n_envs: int
    T: int
    actor_dims: tuple
    critic_dims: tuple
    epochs: int
    minibatches: int
    precision: str = "tf32"
    lr: float = 1e-3
    extra: dict = field(default_factory=dict)

    @property
    def n(self) -> int:
        return self.n_envs * self.T


C_ACTOR = (96, 512, 256, 128, 29)
C_CRITIC = (96, 512, 256, 128, 1)

WORKLOADS = {
    # C1: the CPU-runnable reference update.
    "c1": Workload("c1", 64, 24, C_ACTOR, C_CRITIC, 1, 1),
    # single-B200 full update.
    "c2": Workload("c2", 4096, 24, C_ACTOR, C_CRITIC, 5, 4),
    # data-parallel scaling config (whole job).
    "c4": Workload("c4", 65536, 24, C_ACTOR, C_CRITIC, 5, 4),
    # wide asymmetric actor-critic, bf16 GEMM inputs.
    "c5": Workload("c5", 16384, 48, (96, 1024, 512, 256, 29),
                   (256, 1024, 512, 256, 1), 5, 8, precision="bf16"),
}


def xavier_params(rng: np.random.Generator, actor_dims, critic_dims) -> np.ndarray:
    """Flat parameters in ActorCritic::save order (ppo.rs:539-571)."""
    parts = []
    for dims in (actor_dims, critic_dims):
        for l in range(len(dims) - 1):
            fi, fo = dims[l], dims[l + 1]
            a = np.sqrt(6.0 / (fi + fo))
            parts.append(rng.uniform(-a, a, size=fo * fi).astype(np.float32))
            parts.append(np.zeros(fo, np.float32))
    parts.append(np.zeros(actor_dims[-1], np.float32))  # log_std = ln(1)
    return np.concatenate(parts)


def logp_rows(action: np.ndarray, mean: np.ndarray, log_std: np.ndarray) -> np.ndarray:
    """Row-wise ActorCritic::logp in f32 (sequential over k like ppo.rs:297-305)."""
    std = np.exp(log_std.astype(np.float32))
    lp = np.zeros(action.shape[0], np.float32)
    for k in range(action.shape[1]):
        d = (action[:, k] - mean[:, k]) / std[k]
        lp = lp + (np.float32(-0.5) * d * d - log_std[k] - LOG_SQRT_2PI)
    return lp.astype(np.float32)


@dataclass
class Rollout:
    params: np.ndarray
    obs: np.ndarray          # [n, obs_dim]
    critic_obs: np.ndarray   # [n, cobs_dim]
    action: np.ndarray       # [n, act]
    mean_old: np.ndarray     # [n, act]
    logp_old: np.ndarray     # [n]
    value_old: np.ndarray    # [n]
    rewards: np.ndarray      # [n_envs, T]
    dones: np.ndarray        # [n_envs, T] uint8
    last_values: np.ndarray  # [n_envs]
    n_envs: int
    T: int

    @property
    def n(self) -> int:
        return self.n_envs * self.T

    def nbytes(self) -> int:
        return sum(getattr(self, f).nbytes for f in
                   ("obs", "critic_obs", "action", "mean_old", "logp_old",
                    "value_old", "rewards", "dones", "last_values"))


def make_rollout(seed: int, n_envs: int, T: int, actor_dims, critic_dims,
                 forward, params: np.ndarray | None = None) -> Rollout:
    """Generate one seeded rollout.

    ``forward(params, obs, critic_obs) -> (mean [n, act], value [n])`` is the
    policy used to produce ``mean_old``/``value_old``/``last_values``.
    """
    rng = np.random.default_rng(seed)
    if params is None:
        params = xavier_params(rng, actor_dims, critic_dims)
    od, cd, A = actor_dims[0], critic_dims[0], actor_dims[-1]
    obs = rng.standard_normal((n_envs, T + 1, od), dtype=np.float32)
    cobs = rng.standard_normal((n_envs, T + 1, cd), dtype=np.float32)
    rewards = (np.float32(0.1) * rng.standard_normal((n_envs, T), dtype=np.float32)).astype(np.float32)
    dones = (rng.random((n_envs, T)) < 0.005).astype(np.uint8)
    eps = rng.standard_normal((n_envs * T, A), dtype=np.float32)

    o = np.ascontiguousarray(obs[:, :T].reshape(-1, od))
    c = np.ascontiguousarray(cobs[:, :T].reshape(-1, cd))
    mean_old, value_old = forward(params, o, c)
    log_std = params[-A:]
    action = (mean_old + np.exp(log_std)[None, :] * eps).astype(np.float32)
    logp_old = logp_rows(action, mean_old, log_std)
    _, last_values = forward(params, np.ascontiguousarray(obs[:, T]),
                             np.ascontiguousarray(cobs[:, T]))
    return Rollout(params=params, obs=o, critic_obs=c, action=action,
                   mean_old=np.ascontiguousarray(mean_old, np.float32),
                   logp_old=logp_old, value_old=np.ascontiguousarray(value_old, np.float32),
                   rewards=rewards, dones=dones,
                   last_values=np.ascontiguousarray(last_values, np.float32),
                   n_envs=n_envs, T=T)
