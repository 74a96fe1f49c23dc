"""include/zealot_rl_ffi.rs (the Rust binding a zealot-rl maintainer adds as
zealot-rl-cuda/src/ffi.rs) declares every entry point of include/zealot_rl.h
and nothing else, with the header's types.

No Rust toolchain is in this image, so the binding is checked here at the
type level instead of by rustc: every argument and return type of every
`pub fn` equals the header prototype's (scalar widths, pointer levels and
the constness of each pointee: `*const T` for `const T *`, `*mut T` for
`T *`), and every `#[repr(C)]` struct has the header struct's field types
in the header's order (array lengths included)."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "zealot_rl.h")
RUST = os.path.join(ROOT, "include", "zealot_rl_ffi.rs")

MACROS = {"ZRL_MAX_LAYERS": "8"}

# canonical scalar names (Rust spelling) of the header's C types
C_BASE = {
    "float": "f32", "double": "f64", "int": "i32", "int32_t": "i32",
    "uint32_t": "u32", "int64_t": "i64", "uint64_t": "u64", "size_t": "usize",
    "uint8_t": "u8", "char": "c_char", "void": "void", "zrl_status": "i32",
    "zrl_ctx": "ZrlCtx", "zrl_model_config": "ZrlModelConfig",
    "zrl_ppo_config": "ZrlPpoConfig", "zrl_stats": "ZrlStats", "zrl_comm": "ZrlComm",
    "zrl_batch": "ZrlBatch", "zrl_rollout": "ZrlRollout",
}
RUST_BASE = {"c_int": "i32", "c_void": "void"}


def _strip_c_comments(s):
    s = re.sub(r"/\*.*?\*/", " ", s, flags=re.S)
    return re.sub(r"//[^\n]*", " ", s)


def _c_type(decl: str, named: bool):
    """('ptr', pointee_is_const, inner) / ('base', name) of a C declaration
    such as 'const float *rewards' or 'const char **name'."""
    toks = decl.replace("*", " * ").split()
    if named:
        assert re.match(r"^[A-Za-z_]\w*$", toks[-1]) and len(toks) >= 2, decl
        toks = toks[:-1]
    first = toks.index("*") if "*" in toks else len(toks)
    base = [t for t in toks[:first] if t != "const"]
    assert len(base) == 1, decl
    t = ("base", C_BASE[base[0]])
    pointee_const = "const" in toks[:first]
    rest = toks[first:]
    while rest:
        assert rest[0] == "*", decl
        t = ("ptr", pointee_const, t)
        rest = rest[1:]
        pointee_const = bool(rest) and rest[0] == "const"
        if pointee_const:
            rest = rest[1:]
    return t


def _rust_type(s: str):
    s = s.strip()
    m = re.match(r"^\*(const|mut)\s+(.+)$", s)
    if m:
        return ("ptr", m.group(1) == "const", _rust_type(m.group(2)))
    m = re.match(r"^\[\s*(\w+)\s*;\s*(\d+)\s*\]$", s)
    if m:
        return ("array", _rust_type(m.group(1)), int(m.group(2)))
    assert re.match(r"^[A-Za-z_]\w*$", s), s
    return ("base", RUST_BASE.get(s, s))


def _header_prototypes():
    s = _strip_c_comments(open(HEADER).read())
    out = {}
    for m in re.finditer(r"([A-Za-z_][\w\s\*]*?)\b(zrl_\w+)\s*\(([^;{}]*?)\)\s*;", s):
        ret, name, params = m.group(1), m.group(2), m.group(3).strip()
        args = [] if params in ("", "void") else [_c_type(p, True) for p in params.split(",")]
        out[name] = (_c_type(ret.split("typedef")[-1].strip(), False), args)
    return out


def _rust_functions():
    s = re.sub(r"//[^\n]*", " ", open(RUST).read())
    out = {}
    for m in re.finditer(r"pub fn (zrl_\w+)\s*\(([^)]*)\)\s*(?:->\s*([^;]+))?;", s):
        name, params, ret = m.group(1), m.group(2).strip(), m.group(3)
        args = []
        if params:
            for p in params.split(","):
                if p.strip():
                    args.append(_rust_type(p.split(":", 1)[1]))
        out[name] = (_rust_type(ret) if ret else ("base", "void"), args)
    return out


def _header_structs():
    """struct name (Rust spelling) -> [field types] in declaration order."""
    s = _strip_c_comments(open(HEADER).read())
    for k, v in MACROS.items():
        s = s.replace(k, v)
    out = {}
    for m in re.finditer(r"typedef\s+struct\s*\{(.*?)\}\s*(\w+)\s*;", s, flags=re.S):
        body, cname = m.group(1), m.group(2)
        fields = []
        for decl in body.split(";"):
            decl = decl.strip()
            if not decl:
                continue
            head, *more = [d.strip() for d in decl.split(",")]
            # 'float gamma, lam' -> base 'float', declarators 'gamma', 'lam'
            hm = re.match(r"^((?:const\s+)?\w+)\s+(.*)$", head)
            base, decls = hm.group(1), [hm.group(2)] + more
            for d in decls:
                am = re.match(r"^(\**)\s*(\w+)\s*(?:\[([^\]]+)\])?$", d)
                stars, n = am.group(1), am.group(3)
                t = _c_type(f"{base} {stars}{am.group(2)}", True)
                if n is not None:
                    t = ("array", t, int(eval(n, {"__builtins__": {}})))
                fields.append(t)
        out[C_BASE[cname]] = fields
    return out


def _rust_structs():
    s = re.sub(r"//[^\n]*", " ", open(RUST).read())
    out = {}
    for m in re.finditer(r"pub struct (\w+)\s*\{(.*?)\}", s, flags=re.S):
        name, body = m.group(1), m.group(2)
        fields = []
        for f in re.split(r",(?![^\[]*\])", body):
            f = f.strip()
            if not f or f.startswith("_p"):
                continue
            fields.append(_rust_type(f.split(":", 1)[1]))
        out[name] = fields
    return out


def test_rust_declarations_cover_the_header():
    assert set(_header_prototypes()) == set(_rust_functions()), (
        sorted(set(_header_prototypes()) ^ set(_rust_functions())))


def test_rust_signatures_match_the_header():
    h, r = _header_prototypes(), _rust_functions()
    bad = []
    for name in sorted(h):
        hret, hargs = h[name]
        rret, rargs = r[name]
        if hret != rret:
            bad.append(f"{name}: returns {hret} in C, {rret} in Rust")
        if len(hargs) != len(rargs):
            bad.append(f"{name}: {len(hargs)} arguments in C, {len(rargs)} in Rust")
            continue
        for i, (a, b) in enumerate(zip(hargs, rargs)):
            if a != b:
                bad.append(f"{name} argument {i}: {a} in C, {b} in Rust")
    assert not bad, "\n".join(bad)


def test_rust_structs_match_the_header():
    h, r = _header_structs(), _rust_structs()
    assert set(h) <= set(r), sorted(set(h) - set(r))
    for name, fields in h.items():
        assert r[name] == fields, (name, fields, r[name])


def test_the_type_parsers_tell_constness_and_width_apart():
    assert _c_type("const float *x", True) == _rust_type("*const f32")
    assert _c_type("float *x", True) != _rust_type("*const f32")
    assert _c_type("const char **name", True) == _rust_type("*mut *const c_char")
    assert _c_type("zrl_ctx **out", True) == _rust_type("*mut *mut ZrlCtx")
    assert _c_type("int64_t n", True) != _rust_type("i32")
    assert _c_type("size_t n", True) == _rust_type("usize")
