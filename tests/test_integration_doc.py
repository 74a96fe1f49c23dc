"""INTEGRATION.md's Rust FFI block declares every entry point of
include/zealot_rl.h (and nothing else), so the binding a maintainer copies
stays complete."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_ffi_block_covers_the_header():
    header = open(os.path.join(ROOT, "include", "zealot_rl.h")).read()
    header = re.sub(r"/\*.*?\*/", "", header, flags=re.S)  # declarations, not comments
    declared = set(re.findall(r"\b(zrl_[a-z0-9_]+)\s*\(", header))
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    bound = set(re.findall(r"pub fn (zrl_[a-z0-9_]+)", doc))
    assert declared == bound, (sorted(declared - bound), sorted(bound - declared))
