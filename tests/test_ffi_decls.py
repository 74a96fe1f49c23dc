"""include/zealot_rl_ffi.rs (the Rust binding a zealot-rl maintainer adds as
zealot-rl-cuda/src/ffi.rs) declares every entry point of include/zealot_rl.h
and nothing else."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_rust_declarations_cover_the_header():
    header = open(os.path.join(ROOT, "include", "zealot_rl.h")).read()
    header = re.sub(r"/\*.*?\*/", "", header, flags=re.S)  # declarations, not comments
    declared = set(re.findall(r"\b(zrl_[a-z0-9_]+)\s*\(", header))
    rs = open(os.path.join(ROOT, "include", "zealot_rl_ffi.rs")).read()
    bound = set(re.findall(r"pub fn (zrl_[a-z0-9_]+)", rs))
    assert declared == bound, (sorted(declared - bound), sorted(bound - declared))
