"""The Rust binding (crates/strata-backend-cuda/src/ffi.rs) against the C
headers it binds (include/strata_cuda.h, include/strata_gguf.h): the same
functions, each with the same arity, pointer depth, pointee constness and
integer widths; the same struct layouts (field order and types); the same
status codes. No Rust toolchain is needed: both sides are parsed as text."""
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
HEADERS = [ROOT / "include" / "strata_cuda.h", ROOT / "include" / "strata_gguf.h"]
FFI = ROOT / "crates" / "strata-backend-cuda" / "src" / "ffi.rs"
CRATE = ROOT / "crates" / "strata-backend-cuda"

# C base type -> the Rust name ffi.rs must use for it
C_TO_RUST = {
    "int": "c_int", "char": "c_char", "void": "c_void", "float": "f32", "double": "f64",
    "int64_t": "i64", "uint64_t": "u64", "int32_t": "i32", "uint32_t": "u32", "uint16_t": "u16",
    "uint8_t": "u8", "size_t": "usize",
    "strata_ctx": "StrataCtx", "strata_weight": "StrataWeight", "strata_moe": "StrataMoe",
    "strata_gguf": "StrataGguf", "strata_upload": "strata_upload", "strata_moe_desc": "strata_moe_desc",
    "strata_gguf_shard": "strata_gguf_shard", "strata_gguf_tensor": "strata_gguf_tensor",
    "strata_gguf_value": "strata_gguf_value",
}


def _c_text(directives=False):
    """The headers without comments (and without preprocessor lines unless asked)."""
    out = []
    for h in HEADERS:
        t = re.sub(r"/\*.*?\*/", " ", h.read_text(), flags=re.S)
        t = re.sub(r"//[^\n]*", " ", t)
        if not directives:
            t = "\n".join(line for line in t.splitlines() if not line.lstrip().startswith("#"))
        out.append(t)
    return "\n".join(out)


def _c_type(decl):
    """'const uint8_t **data' -> (('u8', True, 2), 'data'); the name may be absent."""
    decl = " ".join(decl.replace("*", " * ").split())
    toks = decl.split()
    stars = toks.count("*")
    words = [w for w in toks if w != "*"]
    const = "const" in words
    words = [w for w in words if w not in ("const", "struct")]
    # the declarator name is the last word when there are two (type + name)
    name = words[-1] if len(words) > 1 else None
    base = words[0]
    assert base in C_TO_RUST, f"unmapped C type {base!r} in {decl!r}"
    return (C_TO_RUST[base], const and stars > 0, stars), name


def _rust_type(t):
    """'*mut *const u8' -> ('u8', True, 2); intermediate levels must be *mut (C has no `* const`)."""
    t = t.strip()
    quals = re.findall(r"\*(mut|const)\s*", t)
    base = re.sub(r"\*(mut|const)\s*", "", t).strip()
    assert all(q == "mut" for q in quals[:-1]), f"{t}: a const pointer to a pointer has no C counterpart here"
    return (base, bool(quals) and quals[-1] == "const", len(quals))


def c_functions():
    fns = {}
    for m in re.finditer(r"([A-Za-z_][\w\s\*]*?)\b(strata_cuda_\w+)\s*\(([^;{]*?)\)\s*;", _c_text()):
        ret = _c_type(m.group(1))[0]
        args = m.group(3).strip()
        params = [] if args in ("", "void") else [_c_type(a)[0] for a in args.split(",")]
        fns[m.group(2)] = (ret, params)
    return fns


def _rust_src():
    return re.sub(r"//[^\n]*", "", FFI.read_text())


def rust_functions():
    fns = {}
    src = _rust_src()
    blocks = re.findall(r'extern\s+"C"\s*\{(.*?)\n\}', src, flags=re.S)
    assert blocks, "no extern \"C\" block in ffi.rs"
    for block in blocks:
        for m in re.finditer(r"pub(?:\(crate\))?\s+fn\s+(\w+)\s*\((.*?)\)\s*(?:->\s*([^;]+))?;", block, flags=re.S):
            params = []
            for p in [p for p in (s.strip() for s in m.group(2).split(",")) if p]:
                params.append(_rust_type(p.split(":", 1)[1]))
            ret = _rust_type(m.group(3)) if m.group(3) else ("c_void", False, 0)
            fns[m.group(1)] = (ret, params)
    return fns


def c_structs():
    out = {}
    for m in re.finditer(r"typedef\s+struct\s*\{(.*?)\}\s*(\w+)\s*;", _c_text(), flags=re.S):
        fields = []
        for decl in [d.strip() for d in m.group(1).split(";") if d.strip()]:
            # 'int64_t n_expert, rows, cols' declares three fields of one type
            head, *more = [s.strip() for s in decl.split(",")]
            ty, name = _c_type(head)
            for n in [name] + more:
                a = re.match(r"(\w+)\[(\d+)\]$", n)  # an array field: name[count]
                fields.append((a.group(1) if a else n, ty, int(a.group(2)) if a else 1))
        out[m.group(2)] = fields
    return out


def rust_structs():
    out = {}
    for m in re.finditer(r"#\[repr\(C\)\][^\n]*\n(?:#\[[^\n]*\n)*pub\(crate\)\s+struct\s+(\w+)\s*\{(.*?)\}", _rust_src(),
                         flags=re.S):
        fields = []
        for f in re.finditer(r"pub\(crate\)\s+(\w+)\s*:\s*([^,]+),", m.group(2)):
            ty = f.group(2).strip()
            a = re.match(r"\[(.+);\s*(\d+)\]$", ty)
            # type_ / str_ stand for the C fields `type` / `str` (Rust keywords or prelude names)
            fields.append((f.group(1).rstrip("_"), _rust_type(a.group(1) if a else ty), int(a.group(2)) if a else 1))
        out[m.group(1)] = fields
    return out


def c_constants():
    text = _c_text(directives=True)
    consts = {k: int(v) for k, v in re.findall(r"#define\s+(STRATA_\w+)\s+(\d+)", text)}
    for body in re.findall(r"enum\s*\{(.*?)\}", text, flags=re.S):
        for k, v in re.findall(r"(STRATA_\w+)\s*=\s*(\d+)", body):
            consts[k] = int(v)
    return consts


def rust_constants():
    return {k: int(v) for k, v in re.findall(r"pub\(crate\)\s+const\s+(STRATA_\w+)\s*:\s*\w+\s*=\s*(\d+)\s*;", _rust_src())}


def test_crate_files_exist():
    for f in ["Cargo.toml", "build.rs", "src/ffi.rs", "src/lib.rs"]:
        assert (CRATE / f).is_file(), f


def test_same_functions():
    c, r = c_functions(), rust_functions()
    assert len(c) > 60
    assert sorted(set(c) - set(r)) == [], "declared in the headers, not bound in ffi.rs"
    assert sorted(set(r) - set(c)) == [], "bound in ffi.rs, not declared in the headers"


def test_same_signatures():
    c, r = c_functions(), rust_functions()
    bad = []
    for name, (cret, cparams) in c.items():
        rret, rparams = r[name]
        if len(cparams) != len(rparams):
            bad.append(f"{name}: {len(cparams)} arguments in C, {len(rparams)} in Rust")
            continue
        if cret != rret:
            bad.append(f"{name}: returns {cret} in C, {rret} in Rust")
        for i, (a, b) in enumerate(zip(cparams, rparams)):
            if a != b:
                bad.append(f"{name} argument {i}: {a} in C, {b} in Rust")
    assert not bad, "\n".join(bad)


def test_same_struct_layouts():
    c, r = c_structs(), rust_structs()
    assert set(c) == {"strata_upload", "strata_moe_desc", "strata_gguf_shard", "strata_gguf_tensor",
                      "strata_gguf_value"}
    for name, fields in c.items():
        assert name in r, f"struct {name} not in ffi.rs"
        assert r[name] == fields, f"{name}: C {fields}\n Rust {r[name]}"


def test_same_status_codes():
    c, r = c_constants(), rust_constants()
    for k, v in r.items():
        assert c.get(k) == v, f"{k} = {v} in Rust, {c.get(k)} in C"
    for k in c:
        if k == "STRATA_OK" or k.startswith("STRATA_ERR_"):
            assert k in r, f"status {k} not in ffi.rs"


def test_crate_has_no_cpu_fallback():
    lib = (CRATE / "src" / "lib.rs").read_text()
    assert "strata_backend_cpu" not in lib and "CpuBackend" not in lib
    assert "strata-backend-cpu" not in (CRATE / "Cargo.toml").read_text()
    assert "UnsupportedQuant" in lib
    # every binding lib.rs calls exists in ffi.rs
    called = set(re.findall(r"ffi::(strata_cuda_\w+)\s*\(", lib))
    assert called and called <= set(rust_functions())
