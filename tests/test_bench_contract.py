"""bench.py's reference arm on CPU: the JSON line a benchmark driver parses.

`bench.py --impl reference` times zealot-rl's CPU update (the oracle port)
on the host cores and prints one JSON line with the same metric, unit and
config keys as the GPU arm, plus `impl`, `cpu_baseline` and an `e2e` object
whose copy counts are zero.  Under torchrun only rank 0 prints; the other
ranks exit 0 without work.  Run here on the small C1 workload; the parser
that fills roofline.traffic from an ncu CSV is checked on a synthetic one."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(extra_env=None):
    env = dict(os.environ)
    env.update(extra_env or {})
    p = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", "c1",
                        "--steps", "2", "--warmup", "1"], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-2000:]
    return [ln for ln in p.stdout.splitlines() if ln.strip()]


def test_reference_arm_prints_one_complete_line():
    lines = _run()
    assert len(lines) == 1, lines
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
              "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference"
    assert d["unit"] == "samples/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert (d["steps"], d["warmup"], d["n_gpus"]) == (2, 1, 1)
    assert d["config"]["workload"] == "c1"
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert cb["unit"] == d["unit"] and cb["sample"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["unit"] == d["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0


def test_reference_arm_is_silent_on_other_ranks():
    assert _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}) == []


def test_traffic_is_read_from_an_ncu_csv(tmp_path):
    """roofline.traffic from `--traffic-csv`: the mean over the captured
    tc_gemm_kernel launches of dram__bytes_read.sum + dram__bytes_write.sum,
    whatever unit ncu printed, other kernels ignored; None without a usable
    capture."""
    sys.path.insert(0, ROOT)
    import bench
    hdr = ('"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream",'
           '"Block Size","Grid Size","Device","CC","Section Name","Metric Name",'
           '"Metric Unit","Metric Value"\n')

    def row(i, kernel, metric, unit, value):
        return (f'"{i}","1","python","h","{kernel}","1","7","(320, 1, 1)","(148, 1, 1)",'
                f'"0","10.0","Command line profiler metrics","{metric}","{unit}","{value}"\n')

    k = "void zrl::tc_gemm_kernel<256, false, false, 2, 5, 2, false, 1>(TcMaps, TcGroup)"
    csv = tmp_path / "gemm.csv"
    csv.write_text("==PROF== Connected to process 1\n" + hdr
                   + row(0, k, "dram__bytes_read.sum", "Mbyte", "101.80")
                   + row(0, k, "dram__bytes_write.sum", "Kbyte", "6,500.00")
                   + row(0, k, "gpu__time_duration.sum", "usecond", "34.8")
                   + row(1, "head_kernel(HeadParams)", "dram__bytes_read.sum", "Mbyte", "31.4")
                   + row(2, k, "dram__bytes_read.sum", "Gbyte", "0.2")
                   + row(2, k, "dram__bytes_write.sum", "byte", "100000000"))
    want = ((101.8e6 + 6.5e6) + (0.2e9 + 1e8)) / 2
    assert abs(bench.ncu_traffic(str(csv)) - want) < 1.0
    assert bench.ncu_traffic(str(tmp_path / "missing.csv")) is None
    bad = tmp_path / "bad.csv"
    bad.write_text('"a","b"\n"1","2"\n')
    assert bench.ncu_traffic(str(bad)) is None


def test_roofline_flop_count_is_the_documented_one():
    """The numerator of roofline.achieved: GEMM FLOPs per sample pass of the
    C1-C4 nets (actor 96-512-256-128-29, critic 96-512-256-128-1): forward
    859,648, weight gradient 859,648, input gradient 663,040 -- 2,382,336 in
    all, so a C2 update (98,304 samples x 5 epochs) is 1.171 TFLOP."""
    sys.path.insert(0, ROOT)
    import bench
    a, c = (96, 512, 256, 128, 29), (96, 512, 256, 128, 1)
    assert bench.flops_per_sample_pass(a, c) == 2_382_336
    fwd = sum(2 * d[i] * d[i + 1] for d in (a, c) for i in range(4))
    assert fwd == 859_648
    assert abs(bench.flops_per_sample_pass(a, c) * 98_304 * 5 / 1e12 - 1.171) < 5e-4
