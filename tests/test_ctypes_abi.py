"""The ctypes binding table (zealot_b200/native.py) against the C header it
binds (include/zealot_rl.h), on CPU.

ctypes trusts its argtypes: a missing argument, an int32 declared where the
prototype takes an int64, or a struct whose field offsets drift from the
header's is not reported by anything -- the library simply reads the wrong
bytes.  These tests catch that class of mistake without a GPU:

* every prototype in the header has the same return kind and the same
  number and kinds of arguments as its ctypes entry (pointers, and for
  pointer-to-struct or pointer-to-scalar arguments the same pointee; scalar
  sizes, signedness and float-ness);
* the header's structs, compiled by gcc, have the size and field offsets of
  the ctypes Structures the Python side fills in.
"""
from __future__ import annotations

import ctypes as C
import os
import re
import shutil
import subprocess

import pytest

from zealot_b200 import native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "zealot_rl.h")

# header struct type -> ctypes Structure of the binding
STRUCTS = {
    "zrl_model_config": N.ModelConfig,
    "zrl_ppo_config": N.PpoConfigC,
    "zrl_stats": N.StatsC,
    "zrl_comm": N.CommC,
    "zrl_batch": N.BatchC,
    "zrl_rollout": N.RolloutC,
}

# scalar C types -> (kind, bytes, signed)
C_SCALARS = {
    "zrl_status": ("int", 4, True),
    "int": ("int", 4, True),
    "int32_t": ("int", 4, True),
    "uint32_t": ("int", 4, False),
    "int64_t": ("int", 8, True),
    "uint64_t": ("int", 8, False),
    "size_t": ("int", 8, False),
    "uint8_t": ("int", 1, False),
    "char": ("int", 1, True),
    "float": ("float", 4, True),
    "double": ("float", 8, True),
}

CT_SCALARS = {
    C.c_int: ("int", 4, True),
    C.c_int32: ("int", 4, True),
    C.c_uint32: ("int", 4, False),
    C.c_int64: ("int", 8, True),
    C.c_uint64: ("int", 8, False),
    C.c_size_t: ("int", 8, False),
    C.c_uint8: ("int", 1, False),
    C.c_float: ("float", 4, True),
    C.c_double: ("float", 8, True),
}


def _header_text() -> str:
    with open(HEADER) as f:
        s = f.read()
    s = re.sub(r"/\*.*?\*/", " ", s, flags=re.S)
    s = re.sub(r"//[^\n]*", " ", s)
    return s


def _prototypes():
    """name -> (return type, [parameter types]) of every zrl_* function."""
    s = _header_text()
    out = {}
    for m in re.finditer(r"([A-Za-z_][\w\s\*]*?)\b(zrl_\w+)\s*\(([^;{}]*?)\)\s*;", s):
        ret, name, params = m.group(1), m.group(2), m.group(3)
        ret = " ".join(ret.split()[-2:]) if ret.strip().endswith("*") else ret.split()[-1]
        ps = []
        if params.strip() not in ("", "void"):
            for p in params.split(","):
                p = " ".join(p.replace("*", " * ").split())
                # drop the parameter name: the last identifier after the type
                toks = p.split()
                if len(toks) >= 2 and re.match(r"^[A-Za-z_]\w*$", toks[-1]):
                    toks = toks[:-1]
                ps.append(" ".join(t for t in toks if t != "const"))
        out[name] = (ret.replace("const", "").strip(), ps)
    return out


def _c_kind(t: str):
    t = " ".join(t.split())
    if t.endswith("*"):
        return ("ptr", t[:-1].strip())
    if t == "void":
        return ("void",)
    assert t in C_SCALARS, f"unmapped C type {t!r}"
    return ("scalar", C_SCALARS[t])


def _ct_kind(ct):
    if ct is None:
        return ("void",)
    if ct in (C.c_void_p, C.c_char_p):
        return ("ptr", None)
    if isinstance(ct, type) and issubclass(ct, C._Pointer):
        return ("ptr", ct._type_)
    assert ct in CT_SCALARS, f"unmapped ctypes type {ct!r}"
    return ("scalar", CT_SCALARS[ct])


def _same(c_type: str, ct) -> bool:
    ck, tk = _c_kind(c_type), _ct_kind(ct)
    if ck[0] != tk[0]:
        return False
    if ck[0] != "ptr":
        return ck == tk
    pointee_c, pointee_ct = ck[1], tk[1]
    if pointee_ct is None:  # c_void_p / c_char_p: any pointer, but not a struct
        return pointee_c not in STRUCTS
    if isinstance(pointee_ct, type) and issubclass(pointee_ct, C.Structure):
        return STRUCTS.get(pointee_c) is pointee_ct
    return _same(pointee_c, pointee_ct)  # a pointer to a scalar or to a pointer


def test_every_prototype_has_its_ctypes_signature():
    protos = _prototypes()
    assert set(protos) == set(N._SIGS), (set(protos) ^ set(N._SIGS))
    bad = []
    for name, (ret, params) in sorted(protos.items()):
        cres, cargs = N._SIGS[name]
        if not _same(ret, cres) and not (ret == "void" and cres is None):
            bad.append(f"{name}: returns {ret}, bound as {cres}")
        if len(params) != len(cargs):
            bad.append(f"{name}: {len(params)} parameters, bound with {len(cargs)}")
            continue
        for i, (p, ca) in enumerate(zip(params, cargs)):
            if not _same(p, ca):
                bad.append(f"{name} argument {i}: {p} bound as {ca}")
    assert not bad, "\n".join(bad)


def test_struct_layouts_match_the_header(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"',
             'int main(void) {']
    for cname, st in STRUCTS.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in st._fields_:
            lines.append(f'  printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ['  return 0;', '}']
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-std=c11", "-o", str(exe), str(src)], check=True)
    got = {}
    for ln in subprocess.run([str(exe)], check=True, capture_output=True,
                             text=True).stdout.splitlines():
        s, f, v = ln.split()
        got[(s, f)] = int(v)
    for cname, st in STRUCTS.items():
        assert got[(cname, "size")] == C.sizeof(st), cname
        for field, _ in st._fields_:
            assert got[(cname, field)] == getattr(st, field).offset, (cname, field)


def test_the_checker_reports_planted_mismatches():
    # the comparisons above would pass vacuously if _same accepted anything
    assert not _same("int64_t", C.c_int32)
    assert not _same("uint64_t", C.c_int64)
    assert not _same("float", C.c_double)
    assert not _same("float *", C.c_float)
    assert not _same("zrl_batch *", C.POINTER(N.StatsC))
    assert not _same("zrl_batch *", C.c_void_p)
    assert not _same("uint64_t *", C.POINTER(C.c_uint32))
    assert _same("zrl_ctx * *", C.POINTER(C.c_void_p))
    assert _same("zrl_batch *", C.POINTER(N.BatchC))
