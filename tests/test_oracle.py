"""The CPU oracle against the reference's own known-answer tests.

Each test restates one unit test of zealot-rl (file:line given) and runs it
on the C restatement, which pins the oracle before it is used as the
checker for the CUDA library.  Further checks follow: a float64
finite-difference check of the whole PPO gradient, the multi-threaded fold
against the sequential one, and bit-for-bit comparisons of GAE, the Welford
normalizer, Adam, the gradient clip and the operand roundings with numpy
float32 restatements in the reference's operation order.
"""
import math

import numpy as np
import pytest

import oracle as O
from zealot_b200 import synth


def test_lcg_deterministic_unit():
    # rng.rs:39-46
    a, b = O.Lcg(9), O.Lcg(9)
    for _ in range(100):
        assert a.unit() == b.unit()


def test_lcg_first_values_match_definition():
    # rng.rs:14-26 restated with Python integers: x = x*a + c mod 2^64,
    # unit = (x >> 40) / 2^24 in f32.
    x = 9 | 1
    lcg = O.Lcg(9)
    for _ in range(50):
        x = (x * 6364136223846793005 + 1442695040888963407) % (1 << 64)
        want = np.float32(np.float32(x >> 40) / np.float32(1 << 24))
        assert np.float32(lcg.unit()) == want


def test_lcg_seed_or_one_collision():
    # Lcg::new(s) ORs 1 (rng.rs:14-16): seeds 2 and 3 give one stream.
    a, b = O.Lcg(2), O.Lcg(3)
    assert [a.unit() for _ in range(8)] == [b.unit() for _ in range(8)]


def test_gauss_moments():
    g = O.Lcg(5).gausses(200_000)
    assert abs(float(g.mean())) < 0.01
    assert abs(float(g.std()) - 1.0) < 0.01


def test_shuffle_is_permutation_and_matches_python():
    n = 1000
    order = O.shuffle(7, n)
    assert sorted(order.tolist()) == list(range(n))
    # ppo.rs:357-363 in pure Python (f32 product, truncation, min(j, i)).
    x = 7 | 1
    ref = list(range(n))
    for i in range(n - 1, 0, -1):
        x = (x * 6364136223846793005 + 1442695040888963407) % (1 << 64)
        u = np.float32(np.float32(x >> 40) / np.float32(1 << 24))
        j = int(np.float32(u * np.float32(i + 1)))
        j = min(j, i)
        ref[i], ref[j] = ref[j], ref[i]
    assert order.tolist() == ref


def test_gae_matches_hand_computation():
    # ppo.rs:709-721
    adv, ret = O.gae([1.0, 2.0], [0.0, 0.0], [0, 0], 0.0, 1.0, 1.0)
    assert abs(ret[1] - 2.0) < 1e-6 and abs(ret[0] - 3.0) < 1e-6
    assert abs(adv[0] - 3.0) < 1e-6 and abs(adv[1] - 2.0) < 1e-6


def test_gae_respects_done_boundary():
    # ppo.rs:760-768
    adv, _ = O.gae([1.0, 1.0], [5.0, 5.0], [1, 0], 0.0, 0.99, 0.95)
    assert abs(adv[0] - (-4.0)) < 1e-6


def test_elu_and_grad():
    # net.rs:258-265 through a [1,1,1] net: hidden ELU with w=1, b=0, linear
    # output with w=1, b=0, so the output is elu(x) and the input gradient
    # of a unit output gradient is elu'(x).
    m = O.Mlp([1, 1, 1], np.array([1, 0, 1, 0], np.float32))
    for x, want in [(2.0, 2.0), (0.0, 0.0), (-1.0, math.exp(-1.0) - 1.0)]:
        acts = m.forward([x])
        assert abs(float(m.output(acts)[0]) - want) < 1e-6
    acts = m.forward([2.0])
    g = np.zeros(4, np.float32)
    assert m.backward(acts, [1.0], g)[0] == 1.0
    acts = m.forward([-1.0])
    g = np.zeros(4, np.float32)
    assert abs(float(m.backward(acts, [1.0], g)[0]) - math.exp(-1.0)) < 1e-6


def test_backward_matches_finite_difference():
    # net.rs:267-307
    rng = O.Lcg(123)
    dims = [4, 6, 5, 3]
    net = O.Mlp.new(dims, 1.0, rng)
    x = np.array([0.3, -0.7, 0.1, 0.9], np.float32)
    target = np.array([0.2, -0.4, 0.6], np.float32)

    def loss():
        o = net.output(net.forward(x))
        return 0.5 * float(np.sum((o - target) ** 2, dtype=np.float32))

    acts = net.forward(x)
    g = np.zeros_like(net.params)
    net.backward(acts, net.output(acts) - target, g)
    eps = 1e-3
    off = 0
    for l in range(len(dims) - 1):
        nw = dims[l + 1] * dims[l]
        for idx in (0, nw // 2, nw - 1):
            k = off + idx
            orig = net.params[k]
            net.params[k] = orig + eps
            lp = loss()
            net.params[k] = orig - eps
            lm = loss()
            net.params[k] = orig
            fd = (lp - lm) / (2 * eps)
            assert abs(fd - g[k]) < 1e-2, (l, idx, fd, g[k])
        off += nw + dims[l + 1]


def test_adam_minimizes_quadratic():
    # net.rs:309-328
    rng = O.Lcg(7)
    net = O.Mlp.new([2, 1], 1.0, rng)
    m = np.zeros_like(net.params)
    v = np.zeros_like(net.params)
    x = np.array([1.0, -2.0], np.float32)
    target = 0.5

    def loss():
        return float((net.output(net.forward(x))[0] - target) ** 2)

    l0 = loss()
    t = 0
    for _ in range(500):
        acts = net.forward(x)
        g = np.zeros_like(net.params)
        net.backward(acts, [2.0 * (net.output(acts)[0] - target)], g)
        t = O.adam_step(net.params, g, m, v, t, 1e-2)
    assert loss() < l0 * 1e-3


def test_grad_clip_caps_norm():
    # net.rs:330-338
    net = O.Mlp.new([3, 4, 2], 1.0, O.Lcg(1))
    g = np.zeros_like(net.params)
    g[3 * 4] = 100.0  # b_0[0]
    O.grad_clip(g, 1.0)
    assert abs(O.grad_l2_norm(g) - 1.0) < 1e-4


def test_powi_is_square_and_multiply():
    for t in range(1, 60):
        r = np.float32(1.0)
        a = np.float32(0.999)
        b = t
        while True:
            if b & 1:
                r = np.float32(r * a)
            b //= 2
            if b == 0:
                break
            a = np.float32(a * a)
        assert np.float32(O.powi(0.999, t)) == r
        assert abs(O.powi(0.9, t) - 0.9 ** t) < 1e-6


def _bandit_sample(ac: O.ActorCritic, obs, rng: O.Lcg):
    mean, _ = ac.forward(obs[None, :], obs[None, :])
    mean = mean[0]
    ls = ac.params[-len(mean):]
    action = np.array([mean[k] + np.float32(math.exp(ls[k])) * np.float32(rng.gauss())
                       for k in range(len(mean))], np.float32)
    return action, ac.logp(action, mean), mean


@pytest.mark.slow
def test_ppo_improves_on_bandit():
    # ppo.rs:770-845
    rng = O.Lcg(2024)
    target = np.array([0.7, -0.4], np.float32)
    ac = O.ActorCritic.new([3, 32, 2], [3, 32, 1], 0.6, 3e-3, rng)
    cfg = O.PpoConfig(entropy_coef=0.0, minibatches=4, epochs=4)
    obs = np.array([0.5, -0.2, 0.1], np.float32)

    def mean_reward():
        m, _ = ac.forward(obs[None, :], obs[None, :])
        return -float(np.sum((m[0] - target) ** 2))

    r0 = mean_reward()
    n = 256
    for _ in range(120):
        rows = {f: [] for f in O.SoaBatch.FIELDS}
        for _ in range(n):
            action, logp, mean_old = _bandit_sample(ac, obs, rng)
            r = -float(np.sum((action - target) ** 2, dtype=np.float32))
            _, v = ac.forward(obs[None, :], obs[None, :])
            adv, ret = O.gae([r], [v[0]], [1], 0.0, cfg.gamma, cfg.lam)
            for f, val in (("obs", obs), ("critic_obs", obs), ("action", action),
                           ("mean_old", mean_old), ("logp_old", logp),
                           ("value_old", v[0]), ("adv", adv[0]), ("ret", ret[0])):
                rows[f].append(val)
        batch = O.SoaBatch(**{f: np.array(v, np.float32) for f, v in rows.items()})
        ac.update(batch, cfg)
    r1 = mean_reward()
    assert r1 > r0 + 0.2, (r0, r1)
    m, _ = ac.forward(obs[None, :], obs[None, :])
    assert abs(m[0][0] - target[0]) < 0.25 and abs(m[0][1] - target[1]) < 0.25


# ------------------------------------------------------------------ extras

def _small_rollout(seed=3, n_envs=6, T=8, adims=(7, 16, 12, 3), cdims=(5, 16, 12, 1),
                   fresh=True):
    def fwd(params, obs, cobs):
        ac = O.ActorCritic(adims, cdims)
        ac.params = params
        return ac.forward(obs, cobs)

    ro = synth.make_rollout(seed, n_envs, T, adims, cdims, fwd)
    adv, ret = O.gae_batch(ro.rewards, ro.value_old.reshape(n_envs, T), ro.dones,
                           ro.last_values, 0.99, 0.95)
    batch = O.SoaBatch(obs=ro.obs, critic_obs=ro.critic_obs, action=ro.action,
                       mean_old=ro.mean_old, logp_old=ro.logp_old,
                       value_old=ro.value_old, adv=adv.reshape(-1),
                       ret=ret.reshape(-1))
    return ro, batch


def _ppo_loss64(params, adims, cdims, batch, idx, cfg):
    """float64 PPO objective whose gradient minibatch_step accumulates
    (unclipped regime): mean(-ratio*A + value_coef*(v-R)^2) - ent*entropy."""
    A = adims[-1]

    def mlp(dims, p, x):
        off = 0
        a = x
        for l in range(len(dims) - 1):
            fi, fo = dims[l], dims[l + 1]
            w = p[off:off + fo * fi].reshape(fo, fi)
            off += fo * fi
            b = p[off:off + fo]
            off += fo
            z = a @ w.T + b
            a = z if l == len(dims) - 2 else np.where(z > 0, z, np.exp(z) - 1)
        return a, off

    na = O.lib().orc_mlp_param_count(np.asarray(adims, np.int32), len(adims))
    mean, _ = mlp(adims, params[:na], batch.obs[idx].astype(np.float64))
    v, nc = mlp(cdims, params[na:], batch.critic_obs[idx].astype(np.float64))
    ls = params[na + nc:]
    d = (batch.action[idx] - mean) / np.exp(ls)
    logp = np.sum(-0.5 * d * d - ls - 0.9189385, axis=1)
    ratio = np.exp(logp - batch.logp_old[idx])
    surr = ratio * batch.adv[idx]
    vl = (v[:, 0] - batch.ret[idx]) ** 2
    ent = np.sum(ls + 0.5 + 0.9189385)
    return np.mean(-surr + cfg.value_coef * vl) - cfg.entropy_coef * ent


def test_minibatch_grads_match_float64_finite_difference():
    adims, cdims = (7, 16, 12, 3), (5, 16, 12, 1)
    ro, batch = _small_rollout(adims=adims, cdims=cdims)
    ac = O.ActorCritic(adims, cdims)
    ac.params = ro.params
    cfg = O.PpoConfig()
    idx = np.arange(0, batch.n, 2)
    # identity normalizers: the oracle whitens with mean 0 / var 1 and
    # clamps to +-5, which N(0,1) inputs essentially never reach.
    assert np.abs(batch.obs).max() < 5 and np.abs(batch.critic_obs).max() < 5
    g, sums = ac.minibatch_grads(batch, idx, cfg)
    p64 = ro.params.astype(np.float64)
    rng = np.random.default_rng(0)
    picks = rng.choice(len(p64), size=60, replace=False)
    # fresh rollout: mean_old == current mean, v_old == current v -> ratio 1,
    # nothing clipped, so the f64 objective is exactly what is differentiated
    h = 1e-5
    for k in picks:
        pp = p64.copy()
        pp[k] += h
        lp = _ppo_loss64(pp, adims, cdims, batch, idx, cfg)
        pp[k] -= 2 * h
        lm = _ppo_loss64(pp, adims, cdims, batch, idx, cfg)
        fd = (lp - lm) / (2 * h)
        assert abs(fd - g[k]) < 2e-4 + 2e-3 * abs(fd), (k, fd, g[k])
    assert abs(sums[2]) < 1e-6  # KL of a fresh rollout is 0


def test_parallel_fold_matches_sequential():
    ro, batch = _small_rollout()
    ac = O.ActorCritic((7, 16, 12, 3), (5, 16, 12, 1))
    ac.params = ro.params
    cfg = O.PpoConfig()
    idx = O.shuffle(1, batch.n)
    g1, s1 = ac.minibatch_grads(batch, idx, cfg, n_threads=1)
    g4, s4 = ac.minibatch_grads(batch, idx, cfg, n_threads=4)
    scale = np.abs(g1).max()
    assert np.abs(g1 - g4).max() <= 1e-5 * scale
    assert np.allclose(s1, s4, rtol=1e-5, atol=1e-7)


def test_update_is_deterministic_and_moves_params():
    ro, batch = _small_rollout()
    cfg = O.PpoConfig(epochs=2, minibatches=3)
    outs = []
    for _ in range(2):
        ac = O.ActorCritic((7, 16, 12, 3), (5, 16, 12, 1))
        ac.params = ro.params
        st = ac.update(batch.copy(), cfg)
        outs.append((ac.params, st, ac.adam_state()[0]))
    assert np.array_equal(outs[0][0], outs[1][0])
    assert outs[0][1] == outs[1][1]
    assert outs[0][2].tolist() == [6, 6, 6]
    assert not np.array_equal(outs[0][0], ro.params)


def _tf32(x):
    """Round f32 to the tf32 grid, nearest, ties away from zero."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = ((u + 0x1000) & 0xFFFFE000).astype(np.uint32)
    return u.view(np.float32)


def test_tf32_operand_mode_matches_a_python_restatement():
    """The oracle's tf32 operand-rounding mode (the checker for the tensor-core
    path): input, weights and hidden activations rounded to tf32, products
    summed in f32 in the reference's order, output layer kept f32."""
    assert _tf32(np.float32(1.0 + 2 ** -11)) == np.float32(1.0 + 2 ** -10)  # tie: away
    assert _tf32(np.float32(1.0 + 2 ** -12)) == np.float32(1.0)
    assert _tf32(np.float32(-(1.0 + 2 ** -11))) == np.float32(-(1.0 + 2 ** -10))
    adims, cdims = (5, 7, 3), (4, 6, 1)
    rng = np.random.default_rng(0)
    ac = O.ActorCritic(adims, cdims)
    params = rng.standard_normal(ac.np).astype(np.float32)
    ac.params = params
    obs = rng.standard_normal((3, 5)).astype(np.float32)
    cobs = rng.standard_normal((3, 4)).astype(np.float32)
    m32, _ = ac.forward(obs, cobs)
    ac.set_tf32_operands()
    mt, vt = ac.forward(obs, cobs)
    assert not np.array_equal(m32, mt)

    def fwd(dims, p, x):
        a = _tf32(x)
        off = 0
        for l in range(len(dims) - 1):
            fi, fo = dims[l], dims[l + 1]
            w = p[off:off + fo * fi].reshape(fo, fi)
            b = p[off + fo * fi:off + fo * fi + fo]
            off += fo * fi + fo
            out = np.empty(fo, np.float32)
            for o in range(fo):
                z = np.float32(b[o])
                for i in range(fi):
                    z = np.float32(z + np.float32(_tf32(w[o, i]) * a[i]))
                if l < len(dims) - 2:
                    z = np.float32(z if z > 0 else np.float32(np.exp(z)) - np.float32(1))
                    z = _tf32(z)
                out[o] = z
            a = out
        return a

    npa = sum(adims[l + 1] * adims[l] + adims[l + 1] for l in range(len(adims) - 1))
    for r in range(3):
        np.testing.assert_allclose(fwd(adims, params, obs[r]), mt[r], rtol=2e-7, atol=0)
        np.testing.assert_allclose(fwd(cdims, params[npa:], cobs[r]), vt[r:r + 1],
                                   rtol=2e-7, atol=0)


def _bf16(x):
    """Round f32 to bf16, nearest, ties to even (kept as f32)."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def test_bf16_operand_mode_matches_a_python_restatement():
    """The oracle's bf16 operand-rounding mode (the checker for the bf16
    tensor-core path), against the same restatement as the tf32 mode."""
    assert _bf16(np.float32(1.0 + 2 ** -8)) == np.float32(1.0)          # tie: even
    assert _bf16(np.float32(1.0 + 3 * 2 ** -8)) == np.float32(1.0 + 2 ** -6)
    assert _bf16(np.float32(1.0 + 2 ** -8 + 2 ** -20)) == np.float32(1.0 + 2 ** -7)
    adims, cdims = (5, 7, 3), (4, 6, 1)
    rng = np.random.default_rng(1)
    ac = O.ActorCritic(adims, cdims)
    params = rng.standard_normal(ac.np).astype(np.float32)
    ac.params = params
    obs = rng.standard_normal((3, 5)).astype(np.float32)
    cobs = rng.standard_normal((3, 4)).astype(np.float32)
    ac.set_bf16_operands()
    mb, vb = ac.forward(obs, cobs)

    def fwd(dims, p, x):
        a = _bf16(x)
        off = 0
        for l in range(len(dims) - 1):
            fi, fo = dims[l], dims[l + 1]
            w = p[off:off + fo * fi].reshape(fo, fi)
            b = p[off + fo * fi:off + fo * fi + fo]
            off += fo * fi + fo
            out = np.empty(fo, np.float32)
            for o in range(fo):
                z = np.float32(b[o])
                for i in range(fi):
                    z = np.float32(z + np.float32(_bf16(w[o, i]) * a[i]))
                if l < len(dims) - 2:
                    z = np.float32(z if z > 0 else np.float32(np.exp(z)) - np.float32(1))
                    z = _bf16(z)
                out[o] = z
            a = out
        return a

    npa = sum(adims[l + 1] * adims[l] + adims[l + 1] for l in range(len(adims) - 1))
    for r in range(3):
        np.testing.assert_allclose(fwd(adims, params, obs[r]), mb[r], rtol=2e-7, atol=0)
        np.testing.assert_allclose(fwd(cdims, params[npa:], cobs[r]), vb[r:r + 1],
                                   rtol=2e-7, atol=0)


def test_norm_commit_matches_python_restatement():
    """orc_norm_commit against ppo.rs:179-195 restated with numpy float32
    scalars (every operation rounded to f32, left to right)."""
    import ctypes as C
    rng = np.random.default_rng(3)
    dim = 7
    mean = rng.standard_normal(dim).astype(np.float32)
    m2 = (rng.random(dim) * 9 + 1).astype(np.float32)
    pm = rng.standard_normal(dim).astype(np.float32)
    pm2 = (rng.random(dim) * 5).astype(np.float32)
    n1, n2 = np.float32(1234.0), np.float32(77.0)
    tot = np.float32(n1 + n2)
    want_m, want_s = mean.copy(), m2.copy()
    for i in range(dim):
        d = np.float32(pm[i] - mean[i])
        want_m[i] = np.float32(want_m[i] + np.float32(np.float32(d * n2) / tot))
        t = np.float32(np.float32(np.float32(np.float32(d * d) * n1) * n2) / tot)
        want_s[i] = np.float32(want_s[i] + np.float32(pm2[i] + t))
    c, pc = C.c_float(float(n1)), C.c_float(float(n2))
    m, s, p, ps = mean.copy(), m2.copy(), pm.copy(), pm2.copy()
    O.lib().orc_norm_commit(m, s, C.byref(c), p, ps, C.byref(pc), dim)
    assert np.array_equal(m, want_m) and np.array_equal(s, want_s)
    assert c.value == tot and pc.value == 0.0 and not p.any() and not ps.any()
    # an empty pending state leaves everything as it is
    c2, pc2 = C.c_float(5.0), C.c_float(0.0)
    m3 = mean.copy()
    O.lib().orc_norm_commit(m3, m2.copy(), C.byref(c2), pm.copy(), pm2.copy(), C.byref(pc2), dim)
    assert np.array_equal(m3, mean) and c2.value == 5.0


def test_gae_random_cases_match_python_restatement():
    """orc_gae against ppo.rs:681-703 restated with numpy float32 scalars
    (each operation rounded to f32, left to right, as the Rust expression
    evaluates), bit for bit: ragged lengths, episode ends anywhere (the
    first and the last step included), several gamma/lambda pairs."""
    rng = np.random.default_rng(11)
    f = np.float32
    for case in range(40):
        T = int(rng.integers(1, 60))
        r = (rng.standard_normal(T) * rng.choice([0.01, 1.0, 100.0])).astype(np.float32)
        v = rng.standard_normal(T).astype(np.float32)
        d = rng.random(T) < rng.choice([0.0, 0.1, 0.5])
        if case % 5 == 0:
            d[0] = d[-1] = True
        lv = f(rng.standard_normal())
        gamma, lam = [(0.99, 0.95), (0.9, 1.0), (1.0, 0.0), (0.5, 0.5)][case % 4]
        g32, l32 = f(gamma), f(lam)
        want_a = np.empty(T, np.float32)
        want_r = np.empty(T, np.float32)
        acc, nv = f(0.0), lv
        for i in reversed(range(T)):
            nt = f(0.0) if d[i] else f(1.0)
            delta = f(f(r[i] + f(f(g32 * nv) * nt)) - v[i])
            acc = f(delta + f(f(f(g32 * l32) * nt) * acc))
            want_a[i] = acc
            want_r[i] = f(acc + v[i])
            nv = v[i]
        adv, ret = O.gae(r, v, d, lv, gamma, lam)
        assert np.array_equal(adv, want_a), case
        assert np.array_equal(ret, want_r), case


def test_norm_update_and_normalize_match_python_restatement():
    """orc_norm_update (Normalizer::update, ppo.rs:160-167, and the
    PendingNorm::push recurrence) and orc_norm_normalize (ppo.rs:197-205)
    against numpy float32 restatements, bit for bit, from the identity prior
    (mean 0, m2 1, count 1) through observations of mixed scales; normalize
    then hits both clamps and the 1e-8 variance floor."""
    import ctypes as C
    rng = np.random.default_rng(5)
    f = np.float32
    dim = 9
    mean = np.zeros(dim, np.float32)
    m2 = np.ones(dim, np.float32)
    cnt = C.c_float(1.0)
    w_mean, w_m2, w_cnt = mean.copy(), m2.copy(), f(1.0)
    for k in range(200):
        x = (rng.standard_normal(dim) * [1e-3, 0.1, 1, 10, 1e3, 1, 1, 5, 0.5]
             + [0, 3, -2, 0, 50, 0, 0, 0, 1]).astype(np.float32)
        x[5] = f(0.25)  # a constant feature: its variance decays toward the floor
        O.lib().orc_norm_update(mean, m2, C.byref(cnt), x, dim)
        w_cnt = f(w_cnt + f(1.0))
        for i in range(dim):
            dd = f(x[i] - w_mean[i])
            w_mean[i] = f(w_mean[i] + f(dd / w_cnt))
            w_m2[i] = f(w_m2[i] + f(dd * f(x[i] - w_mean[i])))
        assert f(cnt.value) == w_cnt
        assert np.array_equal(mean, w_mean) and np.array_equal(m2, w_m2), k
    for scale in (1.0, 100.0):
        x = (rng.standard_normal(dim) * scale).astype(np.float32)
        out = np.empty(dim, np.float32)
        O.lib().orc_norm_normalize(mean, m2, cnt.value, x, dim, out)
        want = np.empty(dim, np.float32)
        for i in range(dim):
            var = max(f(m2[i] / f(cnt.value)), f(1e-8))
            want[i] = min(max(f(f(x[i] - mean[i]) / np.sqrt(var)), f(-5.0)), f(5.0))
        assert np.array_equal(out, want), scale
    # zero variance: the floor, then the clamp
    z = np.zeros(dim, np.float32)
    out = np.empty(dim, np.float32)
    O.lib().orc_norm_normalize(z, z, 7.0, np.full(dim, 1e-5, np.float32), dim, out)
    assert np.array_equal(out, np.full(dim, f(f(1e-5) / np.sqrt(f(1e-8))), np.float32))
    O.lib().orc_norm_normalize(z, z, 7.0, np.full(dim, 1.0, np.float32), dim, out)
    assert np.array_equal(out, np.full(dim, 5.0, np.float32))


def test_adam_and_clip_match_python_restatement():
    """orc_adam_step (Adam::step, net.rs:233-251) and orc_grad_l2_norm /
    orc_grad_clip (MlpGrad::l2_norm / clip, net.rs:180-202) against numpy
    float32 restatements in the reference's operation order, bit for bit,
    over several steps with gradients of mixed scale (zeros included)."""
    rng = np.random.default_rng(9)
    f = np.float32
    n = 257
    p = rng.standard_normal(n).astype(np.float32)
    m = np.zeros(n, np.float32)
    v = np.zeros(n, np.float32)
    wp, wm, wv = p.copy(), m.copy(), v.copy()
    b1, b2, eps = f(0.9), f(0.999), f(1e-8)
    t = 0
    for step in range(6):
        g = (rng.standard_normal(n) * rng.choice([1e-6, 1e-2, 1.0, 30.0])).astype(np.float32)
        g[::17] = 0.0
        lr = [1e-3, 3e-4, 1e-2][step % 3]
        t = O.adam_step(p, g, m, v, t, lr)
        bc1 = f(f(1.0) - f(O.powi(0.9, t)))
        bc2 = f(f(1.0) - f(O.powi(0.999, t)))
        for i in range(n):
            wm[i] = f(f(b1 * wm[i]) + f(f(f(1.0) - b1) * g[i]))
            wv[i] = f(f(b2 * wv[i]) + f(f(f(f(1.0) - b2) * g[i]) * g[i]))
            upd = f(f(f(lr) * f(wm[i] / bc1)) / f(np.sqrt(f(wv[i] / bc2)) + eps))
            wp[i] = f(wp[i] - upd)
        assert t == step + 1
        assert np.array_equal(m, wm) and np.array_equal(v, wv), step
        assert np.array_equal(p, wp), step
    for scale in (1e-3, 1.0, 1e3):
        g = (rng.standard_normal(n) * scale).astype(np.float32)
        s = f(0.0)
        for x in g:
            s = f(s + f(x * x))
        norm = np.sqrt(s)
        assert f(O.grad_l2_norm(g)) == norm
        for max_norm in (0.5, 1.0, 1e6):
            got = g.copy()
            O.grad_clip(got, max_norm)
            want = g.copy()
            if norm > f(max_norm) and norm > 0:
                want = (want * f(f(max_norm) / norm)).astype(np.float32)
            assert np.array_equal(got, want), (scale, max_norm)


def test_minibatch_losses_match_a_float64_restatement():
    """The oracle's minibatch statistics (surrogate, value loss, KL) and its
    log_std gradient against ppo.rs:408-452 (with logp and kl,
    ppo.rs:297-334) restated in float64 on the oracle's own forward outputs:
    the clipped surrogate and its clip mask, the clipped value loss, the
    entropy term of the log_std gradient and the KL of shared-std
    Gaussians.  The finite-difference test checks the gradient against the
    oracle's loss; this one checks the loss formulas themselves."""
    from tests.helpers import Case, SMALL_A, SMALL_C
    case = Case(SMALL_A, SMALL_C, n_envs=8, T=12, seed=4, perturb=0.08, norm_stats=True)
    ac = O.ActorCritic(case.adims, case.cdims)
    ac.params = case.params
    ac.set_normalizers(*case.norm)
    batch = case.oracle_batch()
    cfg = O.PpoConfig()
    idx = np.random.default_rng(2).permutation(batch.n)[:48]
    g, sums = ac.minibatch_grads(batch, idx, cfg)

    A = case.adims[-1]
    ls = case.params[-A:].astype(np.float64)
    mean, value = ac.forward(batch.obs[idx], batch.critic_obs[idx])
    mean, value = mean.astype(np.float64), value.astype(np.float64)
    act = batch.action[idx].astype(np.float64)
    mo = batch.mean_old[idx].astype(np.float64)
    lpo = batch.logp_old[idx].astype(np.float64)
    vo = batch.value_old[idx].astype(np.float64)
    adv = batch.adv[idx].astype(np.float64)
    ret = batch.ret[idx].astype(np.float64)
    scale = 1.0 / len(idx)
    c = cfg.clip
    log_sqrt_2pi = 0.5 * math.log(2.0 * math.pi)
    logp = np.sum(-0.5 * ((act - mean) / np.exp(ls)) ** 2 - ls - log_sqrt_2pi, axis=1)
    ratio = np.exp(logp - lpo)
    surr = np.minimum(ratio * adv, np.clip(ratio, 1 - c, 1 + c) * adv)
    clipped = ((adv >= 0) & (ratio > 1 + c)) | ((adv < 0) & (ratio < 1 - c))
    assert clipped.any() and (~clipped).any()  # both branches exercised
    d = act - mean
    inv_var = np.exp(-2.0 * ls)
    dls = adv[:, None] * ratio[:, None] * (d * d * inv_var - 1.0)
    g_ls = np.sum(np.where(clipped[:, None], 0.0, -dls), axis=0) * scale
    g_ls += -cfg.entropy_coef * scale * len(idx)
    v_cl = vo + np.clip(value - vo, -c, c)
    l_un, l_cl = (value - ret) ** 2, (v_cl - ret) ** 2
    vloss = np.where(l_cl > l_un, l_cl, l_un)
    assert (l_cl > l_un).any()  # the clipped value branch is taken somewhere
    kl = np.sum(0.5 * ((mean - mo) * np.exp(-ls)) ** 2, axis=1)
    want = np.array([surr.sum(), vloss.sum(), kl.sum()]) * scale
    np.testing.assert_allclose(sums, want, rtol=1e-4, atol=1e-7)
    err = np.max(np.abs(g[-A:] - g_ls)) / np.max(np.abs(g_ls))
    assert err < 1e-4, err
