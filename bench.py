"""PPO-update benchmark (metric: PPO-update samples/s).

One step = one full zealot-rl update of a synthetic rollout: GAE over every
env, advantage normalization, then epochs x minibatches of shuffled
minibatch steps (forward and backward of actor and critic, PPO losses,
per-net gradient clip, adaptive LR, Adam).  At N=1 the workload is
The C2 workload (N=4096 envs x T=24, 5 epochs x 4 minibatches, tf32
GEMMs); with --gpus N every rank runs that per-GPU workload on its own envs
(weak scaling; the global minibatch is N times larger) and the gradient is
allreduced over NCCL once per minibatch.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--config c2|c4|c5] [--precision tf32|fp32|bf16]

Timing: CUDA events on the library's stream around each update; an L2
flush (a 512 MiB write) runs between timed updates, outside the events;
ms_per_step is the max over ranks of the mean.  `e2e` times the same
update through the host-pointer API (pinned host buffers, H2D copies of the
whole rollout and the D2H of the statistics inside the timed region).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "PPO-update samples/s (fwd+bwd+GAE+Adam)"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--config", default=None, choices=["c1", "c2", "c3", "c4", "c5"])
    p.add_argument("--precision", default=None, choices=["tf32", "fp32", "bf16"])
    p.add_argument("--envs-per-gpu", type=int, default=None)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-other-configs", action="store_true",
                   help="skip the C3 rollout-step and C5 wide-update measurements")
    p.add_argument("--profile-only", action="store_true",
                   help="run warmup+steps without clocks/baselines (for ncu)")
    p.add_argument("--traffic-csv", default=None,
                   help="ncu raw CSV with dram__bytes_{read,write}.sum of the GEMM launches "
                        "(roofline.traffic); without it traffic is null")
    return p.parse_args()


def workload(args, world):
    from zealot_b200 import synth
    name = args.config or "c2"
    w = synth.WORKLOADS[name]
    if name == "c4":
        n_envs_local = w.n_envs // world  # the 65,536-env job split over ranks
        scaling = "strong"
    else:
        n_envs_local = args.envs_per_gpu or w.n_envs
        scaling = "weak"
    precision = args.precision or w.precision
    return w, n_envs_local, precision, scaling


def flops_per_sample_pass(adims, cdims):
    """Algorithmic GEMM FLOPs per sample per epoch: forward, weight gradient
    (every layer) and input gradient (every layer but the first)."""
    f = 0
    for d in (adims, cdims):
        macs = [d[l] * d[l + 1] for l in range(len(d) - 1)]
        f += 2 * sum(macs) * 2 + 2 * sum(macs[1:])
    return f


def bytes_per_sample_pass(adims, cdims, elem):
    """Algorithmic HBM bytes of the GEMMs per sample per epoch: every
    activation and delta row read or written once per GEMM that uses it --
    forward (read a_l, write a_l+1), input gradient (read delta_l and the
    stored a_l for ELU', write delta_l-1; every layer but the first) and
    weight gradient (read delta_l and a_l).  Weights (L2-resident) and
    split-K partials are left out."""
    f = 0
    for d in (adims, cdims):
        L = len(d) - 1
        f += sum(d[l] + d[l + 1] for l in range(L))            # forward
        f += sum(d[l + 1] + 2 * d[l] for l in range(1, L))     # dgrad
        f += sum(d[l + 1] + d[l] for l in range(L))            # wgrad
    return f * elem


class Clocks:
    """nvidia-smi sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first(self, timeout=5.0):
        """Block until nvidia-smi has printed its first sample (it takes a
        few hundred ms to start), so the timed region is sampled."""
        t0 = time.time()
        while self.proc and not self.lines and time.time() - t0 < timeout:
            time.sleep(0.02)

    def mark(self):
        self.i0 = len(self.lines)

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        # the samples taken during the timed region (from the mark on); if
        # the region was shorter than the sampling period, the sample just
        # before it and the one after it (both under load)
        lines = self.lines[getattr(self, "i0", 0):]
        if len(lines) < 2:
            lines = self.lines[max(getattr(self, "i0", 0) - 1, 0):]
        for ln in lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except OSError:
        return {}


def tf32_peak(torch, dev):
    """cuBLAS tf32 GEMM (8192^3) throughput, the tensor-core denominator for
    a tf32 kernel (MEASURED_PEAKS has bf16 only).  Best of 10, burst."""
    torch.backends.cuda.matmul.allow_tf32 = True
    a = torch.randn(8192, 8192, device=dev)
    b = torch.randn(8192, 8192, device=dev)
    for _ in range(3):
        a @ b
    torch.cuda.synchronize()
    best = 1e9
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        a @ b
        e1.record()
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    torch.backends.cuda.matmul.allow_tf32 = False
    del a, b
    return 2 * 8192 ** 3 / (best * 1e-3) / 1e12


def ncu_traffic(path):
    """Mean DRAM bytes (read + write) per launch of the tensor-core GEMM
    kernel from an ncu raw CSV (``--metrics dram__bytes_read.sum,
    dram__bytes_write.sum --csv``), or None without one."""
    if not path or not os.path.exists(path):
        return None
    import csv
    per = {}
    with open(path) as f:
        rows = [r for r in csv.reader(ln for ln in f if not ln.startswith("=="))]
    if not rows:
        return None
    h = rows[0]
    try:
        iid, ik, im, iv = (h.index("ID"), h.index("Kernel Name"), h.index("Metric Name"),
                           h.index("Metric Value"))
    except ValueError:
        return None
    for r in rows[1:]:
        if len(r) <= iv or "tc_gemm_kernel" not in r[ik]:
            continue
        if r[im] in ("dram__bytes_read.sum", "dram__bytes_write.sum"):
            unit = r[h.index("Metric Unit")] if "Metric Unit" in h else "byte"
            scale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}.get(unit, 1)
            per[r[iid]] = per.get(r[iid], 0.0) + float(r[iv].replace(",", "")) * scale
    return sum(per.values()) / len(per) if per else None


# ------------------------------------------------------------- CPU legs

def cpu_model():
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_rollout(w, seed=0, n_envs=None):
    """A synthetic rollout with the workload's shapes and value
    distributions for the CPU legs (the oracle port of zealot-rl's CPU
    update): obs / critic obs ~ N(0,1), actions around a zero mean with
    log_std 0, rewards ~ N(0, 0.1^2), dones ~ Bernoulli(0.005), values ~ N(0,1)."""
    import oracle as O
    from zealot_b200 import synth
    n_envs = n_envs or w.n_envs
    rng = np.random.default_rng(seed)
    params = synth.xavier_params(rng, w.actor_dims, w.critic_dims)
    n = n_envs * w.T
    od, cd, A = w.actor_dims[0], w.critic_dims[0], w.actor_dims[-1]
    action = rng.standard_normal((n, A), dtype=np.float32)
    b = O.SoaBatch(obs=rng.standard_normal((n, od), dtype=np.float32),
                   critic_obs=rng.standard_normal((n, cd), dtype=np.float32),
                   action=action, mean_old=np.zeros((n, A), np.float32),
                   logp_old=synth.logp_rows(action, np.zeros((n, A), np.float32),
                                            np.zeros(A, np.float32)),
                   value_old=rng.standard_normal(n, dtype=np.float32),
                   adv=np.zeros(n, np.float32), ret=np.zeros(n, np.float32))
    rew = (0.1 * rng.standard_normal((n_envs, w.T))).astype(np.float32)
    dones = (rng.random((n_envs, w.T)) < 0.005).astype(np.uint8)
    lv = rng.standard_normal(n_envs).astype(np.float32)
    return params, b, rew, dones, lv


def cpu_update(w, params, b, rew, dones, lv, epochs, threads):
    """GAE + ActorCritic::update (the oracle port, ppo.rs:338-510) over the
    rollout: `epochs` epochs of w.minibatches minibatch steps.  Seconds."""
    import oracle as O
    n_envs = rew.shape[0]
    ac = O.ActorCritic(w.actor_dims, w.critic_dims)
    ac.params = params
    ac.lr = w.lr
    cfg = O.PpoConfig(epochs=epochs, minibatches=w.minibatches)
    t0 = time.perf_counter()
    adv, ret = O.gae_batch(rew, b.value_old.reshape(n_envs, w.T), dones, lv, 0.99, 0.95)
    b.adv[:] = adv.reshape(-1)
    b.ret[:] = ret.reshape(-1)
    ac.update(b, cfg, n_threads=threads)
    return time.perf_counter() - t0


def cpu_baseline(w):
    """The reference's CPU update (oracle port) timed on this host: one whole
    update of the workload on every core, and one thread on a bounded
    sample (one minibatch step of an eighth of the rows)."""
    import oracle as O
    threads = os.cpu_count() or 1
    params, b, rew, dones, lv = cpu_rollout(w)
    dt = cpu_update(w, params, b, rew, dones, lv, w.epochs, threads)
    value = w.n / dt
    # one thread: a minibatch step of n/8 rows (the per-sample cost is what
    # the single thread measures), scaled to the update's sample passes
    rows = max(1, w.n // w.minibatches // 8)
    ac = O.ActorCritic(w.actor_dims, w.critic_dims)
    ac.params = params
    idx = np.arange(rows, dtype=np.int64)
    t0 = time.perf_counter()
    ac.minibatch_grads(b, idx, O.PpoConfig(), n_threads=1)
    t1 = time.perf_counter() - t0
    one = w.n / (t1 * (w.n * w.epochs / rows))
    return {"value": value, "unit": "samples/s", "cores": threads, "kind": "port",
            "cpu_model": cpu_model(),
            "sample": f"one whole {w.name} update (GAE + {w.epochs} epochs x {w.minibatches} "
                      f"minibatch steps over {w.n} samples: forward, backward, clip, Adam) "
                      f"on {threads} threads, {dt:.2f} s",
            "one_thread": {"value": one, "unit": "samples/s", "cores": 1,
                           "sample": f"the forward/backward of {rows} rows ({t1:.2f} s), "
                                     f"scaled to the update's {w.n * w.epochs} sample passes"}}


def run_reference(args):
    """The reference's CPU path (zealot-rl's update restated in C, the oracle
    port) on every host core: each step is one epoch of the update (its
    minibatch steps over every sample; the epochs of an update do identical
    work), and samples/s is the update's samples over epochs x that time."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    w, _, precision, scaling = workload(args, 1)
    threads = os.cpu_count() or 1
    params, b, rew, dones, lv = cpu_rollout(w)
    vals = []
    for i in range(args.warmup + args.steps):
        dt = cpu_update(w, params, b, rew, dones, lv, 1, threads)
        if i >= args.warmup:
            vals.append(dt)
    dt = statistics.median(vals)
    value = w.n / (dt * w.epochs)
    line = {"metric": METRIC, "value": value, "unit": "samples/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": w.name, "n_envs_per_gpu": w.n_envs, "n_envs_total": w.n_envs,
                       "T": w.T, "samples_per_update": w.n, "epochs": w.epochs,
                       "minibatches": w.minibatches,
                       "minibatch_size": w.n // w.minibatches,
                       "actor": list(w.actor_dims), "critic": list(w.critic_dims),
                       "parallelism": "cpu"},
            "cpu_baseline": {"value": value, "unit": "samples/s", "cores": threads,
                             "kind": "port", "cpu_model": cpu_model(),
                             "sample": f"per step one epoch of the {w.name} update (GAE + "
                                       f"{w.minibatches} minibatch steps over all {w.n} "
                                       f"samples), {dt:.2f} s median; update = "
                                       f"{w.epochs} epochs"},
            "e2e": {"value": value, "unit": "samples/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- GPU leg

def bench_c3(args):
    """The C3 workload: the rollout step -- batch 4096 x obs 96
    through the actor and critic, Gaussian action sampling with seeded
    Philox draws and the log-prob (zrl_policy_step on device buffers),
    repeated for the T = 24 steps of a rollout.  Latency per step and
    samples/s; one GPU (other ranks exit)."""
    import torch
    if int(os.environ.get("RANK", "0")) != 0:
        return
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    line = measure_c3(args.steps, args.warmup, args.precision or "tf32", local)
    print(json.dumps(line), flush=True)


def measure_c3(steps, warmup, precision, local):
    import torch
    from zealot_b200 import native as N
    from zealot_b200 import synth
    from zealot_b200 import zealot_rl as Z
    dev = torch.device("cuda", local)
    n, T = 4096, 24
    adims, cdims = synth.WORKLOADS["c2"].actor_dims, synth.WORKLOADS["c2"].critic_dims
    ac = Z.ActorCritic(adims, cdims, precision=precision, device=local)
    ac.params = synth.xavier_params(np.random.default_rng(1234), adims, cdims)
    g = torch.Generator(device="cpu").manual_seed(7)
    obs = torch.randn(T, n, adims[0], generator=g).to(dev)
    cobs = torch.randn(T, n, cdims[0], generator=g).to(dev)
    act = torch.empty(n, adims[-1], device=dev)
    mean = torch.empty(n, adims[-1], device=dev)
    lp = torch.empty(n, device=dev)
    val = torch.empty(n, device=dev)
    stream = torch.cuda.ExternalStream(N.lib().zrl_stream(ac.ctx.h), device=dev)
    torch.cuda.synchronize()

    def rollout(seed):
        for t in range(T):
            ac.ctx.call("zrl_policy_step", obs[t].data_ptr(), cobs[t].data_ptr(), n, seed, t,
                        act.data_ptr(), lp.data_ptr(), mean.data_ptr(), val.data_ptr(), 1)

    for i in range(warmup):
        rollout(i)
    times = []
    l0 = ac.kernel_launches()
    for i in range(steps):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        rollout(100 + i)
        e1.record(stream)
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    ms = sum(times) / len(times)
    launches = (ac.kernel_launches() - l0) // steps
    line = {"metric": "rollout-step samples/s (policy forward + Gaussian sampling + logp)",
            "value": n * T / (ms * 1e-3), "unit": "samples/s", "n_gpus": 1,
            "steps": steps, "warmup": warmup, "ms_per_step": ms,
            "ms_per_rollout_step": ms / T, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": precision,
            "data": "synthetic obs ~N(0,1), Xavier-uniform init",
            "config": {"workload": "c3", "batch": n, "T": T, "actor": list(adims),
                       "critic": list(cdims),
                       "note": "one step = a T-step rollout of policy steps; each policy "
                               "step returns when its outputs are on the device"},
            "gpu_launches": int(launches)}
    ac.close()
    return line


def measure_update(name, steps, warmup, local):
    """Device-resident update throughput of another workload on this GPU
    (CUDA events on the library's stream, 512 MiB L2 flush between timed
    updates), with its GEMMs' tensor-core throughput from a profiled
    update."""
    import ctypes as C

    import torch
    from zealot_b200 import native as N
    from zealot_b200 import synth
    from zealot_b200 import zealot_rl as Z
    dev = torch.device("cuda", local)
    w = synth.WORKLOADS[name]
    ac = Z.ActorCritic(w.actor_dims, w.critic_dims, precision=w.precision, device=local)
    params = synth.xavier_params(np.random.default_rng(1234), w.actor_dims, w.critic_dims)
    ac.params = params
    ac.lr = w.lr
    ro = synth.make_rollout(1000, w.n_envs, w.T, w.actor_dims, w.critic_dims,
                            lambda p, o, c: ac.forward(o, c), params=params)

    def dt_(a, dtype=torch.float32):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev, dtype)

    d = {f: dt_(getattr(ro, f)) for f in ("obs", "critic_obs", "action", "mean_old",
                                          "logp_old", "value_old")}
    b = Z.SoaBatch(adv=torch.zeros(ro.n, device=dev), ret=torch.zeros(ro.n, device=dev), **d)
    rew, val = dt_(ro.rewards), dt_(ro.value_old.reshape(ro.n_envs, ro.T))
    done, lv = dt_(ro.dones, torch.uint8), dt_(ro.last_values)
    cfg = Z.PpoConfig(epochs=w.epochs, minibatches=w.minibatches, adaptive_lr=True)
    stream = torch.cuda.ExternalStream(N.lib().zrl_stream(ac.ctx.h), device=dev)
    flush = torch.empty(512 * 1024 * 1024 // 4, device=dev)
    for _ in range(warmup):
        ac.gae_update(rew, val, done, lv, b, cfg, ro.n, 0)
    times = []
    for _ in range(steps):
        with torch.cuda.stream(stream):
            flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        ac.gae_update(rew, val, done, lv, b, cfg, ro.n, 0)
        e1.record(stream)
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    ms = sum(times) / len(times)
    N.check(N.lib().zrl_set_profiling(ac.ctx.h, 1), ac.ctx.h)
    ac.gae_update(rew, val, done, lv, b, cfg, ro.n, 0)
    g_ms, u_ms, g_n = C.c_float(), C.c_float(), C.c_int64()
    N.lib().zrl_get_profile(ac.ctx.h, C.byref(g_ms), C.byref(u_ms), C.byref(g_n))
    fl = flops_per_sample_pass(w.actor_dims, w.critic_dims) * ro.n * w.epochs
    ac.close()
    del flush
    return {"workload": name, "samples_per_update": ro.n, "epochs": w.epochs,
            "minibatches": w.minibatches, "actor": list(w.actor_dims),
            "critic": list(w.critic_dims), "dtype": w.precision, "steps": steps,
            "warmup": warmup, "ms_per_update": ms, "samples_per_s": ro.n / (ms * 1e-3),
            "gemm_ms_per_update": g_ms.value,
            "gemm_tflops": fl / (g_ms.value * 1e-3) / 1e12 if g_ms.value > 0 else None,
            "algorithmic_gflop_per_update": fl / 1e9}


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.config == "c3":
        return bench_c3(args)

    import torch
    import torch.distributed as dist
    from zealot_b200 import native as N
    from zealot_b200 import synth
    from zealot_b200 import zealot_rl as Z

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("gloo", timeout=timedelta(seconds=120))

    w, n_envs, precision, scaling = workload(args, world)
    comm = None
    if world > 1:
        idb = torch.zeros(128, dtype=torch.uint8)
        if rank == 0:
            import ctypes
            buf = (ctypes.c_uint8 * 128)()
            N.check(N.lib().zrl_nccl_unique_id(buf))
            idb = torch.tensor(list(buf), dtype=torch.uint8)
        dist.broadcast(idb, 0)
        comm = N.CommC()
        comm.rank, comm.world_size, comm.timeout_ms = rank, world, 120000
        for i, v in enumerate(idb.tolist()):
            comm.nccl_id[i] = v

    ac = Z.ActorCritic(w.actor_dims, w.critic_dims, precision=precision, device=local,
                       comm=comm)
    # identical parameters on every rank; per-rank rollouts of its own envs
    params = synth.xavier_params(np.random.default_rng(1234), w.actor_dims, w.critic_dims)
    ac.params = params
    ac.lr = w.lr

    def gpu_forward(p, obs, cobs):
        return ac.forward(obs, cobs)

    ro = synth.make_rollout(1000 + rank, n_envs, w.T, w.actor_dims, w.critic_dims,
                            gpu_forward, params=params)
    n_local = ro.n
    n_global = n_local * world
    row_off = rank * n_local
    cfg = Z.PpoConfig(epochs=w.epochs, minibatches=w.minibatches, adaptive_lr=True)

    # device-resident copies
    def dt_(a, dtype=torch.float32):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev, dtype)

    d = {f: dt_(getattr(ro, f)) for f in ("obs", "critic_obs", "action", "mean_old",
                                          "logp_old", "value_old")}
    d_rew = dt_(ro.rewards)
    d_val = dt_(ro.value_old.reshape(ro.n_envs, ro.T))
    d_done = dt_(ro.dones, torch.uint8)
    d_lv = dt_(ro.last_values)
    d_adv = torch.zeros(n_local, device=dev)
    d_ret = torch.zeros(n_local, device=dev)
    dbatch = Z.SoaBatch(adv=d_adv, ret=d_ret, **d)
    # pinned host copies for the e2e leg
    def pin(a, dtype=torch.float32):
        t = torch.from_numpy(np.ascontiguousarray(a)).to(dtype).pin_memory()
        return t.numpy()

    h = {f: pin(getattr(ro, f)) for f in ("obs", "critic_obs", "action", "mean_old",
                                          "logp_old", "value_old")}
    h_rew, h_val = pin(ro.rewards), pin(ro.value_old.reshape(ro.n_envs, ro.T))
    h_done = pin(ro.dones, torch.uint8)
    h_lv = pin(ro.last_values)
    hbatch = Z.SoaBatch(adv=pin(np.zeros(n_local, np.float32)),
                        ret=pin(np.zeros(n_local, np.float32)), **h)
    h2d_bytes = sum(a.nbytes for a in h.values()) + h_rew.nbytes + h_val.nbytes + \
        h_done.nbytes + h_lv.nbytes
    d2h_bytes = 5 * 4  # PpoStats

    stream = torch.cuda.ExternalStream(N.lib().zrl_stream(ac.ctx.h), device=dev)
    flush = torch.empty(512 * 1024 * 1024 // 4, device=dev)

    def step_device():
        return ac.gae_update(d_rew, d_val, d_done, d_lv, dbatch, cfg, n_global, row_off)

    def step_host():
        return ac.gae_update(h_rew, h_val, h_done, h_lv, hbatch, cfg, n_global, row_off)

    def barrier():
        if world > 1:
            dist.barrier()

    def timed(fn, k):
        times = []
        for _ in range(k):
            with torch.cuda.stream(stream):
                flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            st = fn()
            e1.record(stream)
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
        return times, st

    for _ in range(args.warmup):
        step_device()
    barrier()
    torch.cuda.synchronize()
    if args.profile_only:
        for _ in range(args.steps):
            step_device()
        torch.cuda.synchronize()
        return

    clocks = Clocks(local)
    clocks.start()
    clocks.wait_first()
    step_device()  # keep the GPU under load while the sampler settles
    l0 = ac.kernel_launches()
    barrier()
    torch.cuda.synchronize()
    clocks.mark()
    times, st = timed(step_device, args.steps)
    torch.cuda.synchronize()
    barrier()
    launches = (ac.kernel_launches() - l0) // args.steps
    clk = clocks.stop()
    ms = sum(times) / len(times)
    # e2e through the host-pointer API
    for _ in range(max(1, args.warmup // 2)):
        step_host()
    e2e_times, _ = timed(step_host, max(3, args.steps // 2))
    e2e_ms = sum(e2e_times) / len(e2e_times)
    # profiling pass: GEMM device time via events around each GEMM launch
    N.check(N.lib().zrl_set_profiling(ac.ctx.h, 1), ac.ctx.h)
    step_device()
    import ctypes as C
    g_ms, u_ms, g_n = C.c_float(), C.c_float(), C.c_int64()
    N.lib().zrl_get_profile(ac.ctx.h, C.byref(g_ms), C.byref(u_ms), C.byref(g_n))
    breakdown = {}
    i = 0
    while True:
        nm, t, k = C.c_char_p(), C.c_float(), C.c_int64()
        if not N.lib().zrl_profile_site(ac.ctx.h, i, C.byref(nm), C.byref(t), C.byref(k)):
            break
        breakdown[nm.value.decode()] = {"ms": round(t.value, 4), "launches": int(k.value)}
        i += 1
    N.lib().zrl_set_profiling(ac.ctx.h, 0)

    if world > 1:
        t = torch.tensor([ms, e2e_ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = t.tolist()

    value = n_global / (ms * 1e-3)
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        ac.close()
        return
    peaks = measured_peaks()
    fl = flops_per_sample_pass(w.actor_dims, w.critic_dims) * n_local * w.epochs
    if precision == "bf16":
        peak, peak_src = peaks.get("bf16_tflops", 1590.0), (
            "MEASURED_PEAKS bf16_tflops (burst)" if "bf16_tflops" in peaks else "fallback 1.59 PF")
    elif precision == "tf32":
        peak, peak_src = tf32_peak(torch, dev), "cuBLAS tf32 8192^3 measured in this run (burst)"
    else:
        peak, peak_src = 75.0, "nominal fp32 CUDA-core peak (no measured figure)"
    hbm = peaks.get("hbm_gbs", 6650.0)
    hbm_src = "MEASURED_PEAKS.json hbm_gbs (copy)" if "hbm_gbs" in peaks else "fallback 6.65 TB/s"
    # The MLP GEMMs are the update's one dense contraction: tensor-core
    # bound by the workload's own arithmetic (algorithmic FLOPs: forward,
    # weight and input gradients of both nets).  achieved = FLOPs of one
    # launch on average / its average duration (CUDA events around every
    # GEMM launch in a profiled update) = FLOPs of the update's GEMMs / their
    # summed time.
    achieved = fl / (g_ms.value * 1e-3) / 1e12 if g_ms.value > 0 else None
    # the layer-by-layer design's own bytes: every activation and delta row
    # once per GEMM that reads or writes it (what the GEMMs cannot avoid
    # moving as designed); weights (L2-resident) and split-K partials left out
    by = bytes_per_sample_pass(w.actor_dims, w.critic_dims,
                               2 if precision == "bf16" else 4) * n_local * w.epochs
    ach_gbs = by / (g_ms.value * 1e-3) / 1e9 if g_ms.value > 0 else None
    # the whole update against its floor: algorithmic GEMM FLOPs at the
    # tensor peak plus the update's algorithmic HBM bytes at the copy
    # bandwidth (per sample pass: obs, critic obs, action, mean_old and four
    # scalars of the epoch's minibatch, 1016 B; per parameter and minibatch
    # step: 28 B of Adam and 12 B of weight/gradient traffic; GAE and the
    # advantage moments), all on n_local samples of this rank
    A = w.actor_dims[-1]
    row_bytes = 4 * (w.actor_dims[0] + w.critic_dims[0] + 2 * A + 4)
    n_par = sum(d[l] * d[l + 1] + d[l + 1] for d in (w.actor_dims, w.critic_dims)
                for l in range(len(d) - 1)) + A
    steps = w.epochs * w.minibatches
    upd_bytes = row_bytes * n_local * w.epochs + 40 * n_par * steps + 17 * n_local + \
        12 * n_local
    floor_ms = (fl / (peak * 1e12) + upd_bytes / (hbm * 1e9)) * 1e3
    gn = max(int(g_n.value), 1)
    roof = {"bound": "tensor", "kernel": "tc_gemm_kernel (every MLP GEMM launch of one update)",
            "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": (achieved / peak) if achieved else None,
            "traffic": ncu_traffic(args.traffic_csv),
            "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum per GEMM "
                               f"launch, {args.traffic_csv}") if args.traffic_csv else
                              "null: no ncu capture passed (--traffic-csv)",
            "peak_source": peak_src + "; MEASURED_PEAKS has no tf32 figure" if precision == "tf32"
                           else peak_src,
            "algorithmic_flop_per_launch": fl / gn,
            "algorithmic_gflop_per_update": fl / 1e9,
            "gemm_ms_per_update": g_ms.value, "gemm_launches_per_update": g_n.value,
            "avg_launch_us": 1e3 * g_ms.value / gn,
            "gemm_share_of_update": g_ms.value / u_ms.value if u_ms.value else None,
            "profiled_update_ms": u_ms.value, "breakdown_ms_per_update": breakdown,
            "hbm_view": {"achieved": ach_gbs, "peak": hbm, "unit": "GB/s",
                         "frac": (ach_gbs / hbm) if ach_gbs else None, "peak_source": hbm_src,
                         "bytes": "every activation/delta row once per GEMM that uses it",
                         "gb_per_update": by / 1e9},
            "update_floor": {"floor_ms": floor_ms, "measured_ms": ms,
                             "frac": floor_ms / ms,
                             "algorithmic_gb_per_update": upd_bytes / 1e9,
                             "how": "GEMM FLOPs / tensor peak + update bytes / HBM copy bandwidth"}}
    cpu = None if args.no_cpu_baseline or world > 1 else cpu_baseline(w)
    # the other single-GPU configurations, timed on this GPU in the same run
    # (C3: the rollout step; C5: the wide bf16 actor-critic)
    others = None
    if world == 1 and not args.no_other_configs and (args.config or "c2") == "c2":
        others = {"c3": measure_c3(10, 3, "tf32", local),
                  "c5": measure_update("c5", 3, 2, local)}
    line = {"metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": precision, "data": "synthetic (seeded rollouts, Xavier-uniform init)",
            "config": {"workload": w.name, "n_envs_per_gpu": n_envs, "n_envs_total": n_envs * world,
                       "T": w.T, "samples_per_update": n_global, "epochs": w.epochs,
                       "minibatches": w.minibatches,
                       "minibatch_size": n_global // w.minibatches,
                       "actor": list(w.actor_dims), "critic": list(w.critic_dims),
                       "parallelism": f"dp{world}", "l2": "512 MiB flush between timed updates"},
            "e2e": {"value": n_global / (e2e_ms * 1e-3), "unit": "samples/s",
                    "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes},
            "gpu_launches": int(launches),
            "roofline": roof, "clocks": clk, "cpu_baseline": cpu, "other_configs": others,
            "stats_last": {"kl": st.kl, "surrogate": st.surrogate,
                           "value_loss": st.value_loss, "entropy": st.entropy, "lr": st.lr}}
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    ac.close()


if __name__ == "__main__":
    main()
