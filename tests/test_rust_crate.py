"""The Rust binding crate (qwen3-image21_b200/rust/b200-attn) against the C header it binds.

No Rust toolchain exists here, so the crate is checked as text: the #[repr(C)] structs
must list the header's fields in the same order with the same widths, and the extern
block must declare every function of include/b200_attn.h with matching parameter types
and return type.  A mismatch here is an ABI break for the engine's call sites."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "b200_attn.h")
CRATE = os.path.join(ROOT, "qwen3-image21_b200", "rust", "b200-attn")

# C type -> the Rust type the binding must use for it
C_TO_RUST = {
    "int32_t": "i32", "int64_t": "i64", "uint32_t": "u32", "size_t": "usize", "float": "f32",
    "int": "c_int", "void*": "*mut c_void", "const void*": "*const c_void",
    "const float*": "*const f32", "float*": "*mut f32", "int32_t*": "*mut i32",
    "const int32_t*": "*const i32", "const int64_t*": "*const i64", "int64_t*": "*mut i64",
    "const uint8_t*": "*const u8", "uint8_t*": "*mut u8", "const b200_kv_desc*": "*const KvDesc",
    "b200_kv_desc*": "*mut KvDesc", "const b200_attn_args*": "*const AttnArgs",
    "size_t*": "*mut usize", "b200_stream_t": "*mut c_void", "const char*": "*const c_char",
}


def _strip_c_comments(s):
    s = re.sub(r"/\*.*?\*/", " ", s, flags=re.S)
    return re.sub(r"//[^\n]*", " ", s)


def _c_decl(decl):
    """'const void* prefix_k' -> ('prefix_k', 'const void*'); an array parameter
    ('const int32_t axes[3]') decays to a pointer."""
    decl = " ".join(decl.split())
    arr = re.match(r"(.*\w)\s*\[\w*\]$", decl)
    if arr:
        decl = arr.group(1)
        name = re.match(r"(.*?)\s*(\w+)$", decl)
        return name.group(2), _norm_c_type(name.group(1) + "*")
    m = re.match(r"(.*?)\s*(\w+)$", decl)
    return m.group(2), _norm_c_type(m.group(1))


def _norm_c_type(t):
    """'const void *' / 'const void*' -> 'const void*'."""
    return " ".join(t.replace("*", " * ").split()).replace(" *", "*")


def header_struct(name):
    src = _strip_c_comments(open(HEADER).read())
    m = re.search(r"typedef struct \{([^{}]*)\}\s*" + name + r";", src, re.S)
    assert m, name
    fields = []
    for stmt in m.group(1).split(";"):
        stmt = stmt.strip()
        if not stmt:
            continue
        n, t = _c_decl(stmt)
        fields.append((n, _norm_c_type(t)))
    return fields


def header_functions():
    src = _strip_c_comments(open(HEADER).read())
    out = {}
    for m in re.finditer(r"^(int|const char\*)\s+(b200_\w+)\(([^)]*)\);", src, re.M | re.S):
        ret, name, params = m.group(1), m.group(2), m.group(3)
        ps = [] if params.strip() in ("", "void") else [_c_decl(p.strip()) for p in params.split(",")]
        out[name] = (ret, [(n, _norm_c_type(t)) for n, t in ps])
    return out


def rust_source():
    return open(os.path.join(CRATE, "src", "lib.rs")).read()


def rust_struct(name):
    src = rust_source()
    m = re.search(r"pub struct " + name + r"\s*\{(.*?)\n\s*\}", src, re.S)
    assert m, name
    return [(n, " ".join(t.split())) for n, t in re.findall(r"pub (\w+):\s*([^,]+),", m.group(1))]


def rust_functions():
    src = rust_source()
    block = re.search(r'extern "C" \{(.*?)\n    \}', src, re.S).group(1)
    out = {}
    for m in re.finditer(r"pub fn (b200_\w+)\((.*?)\)\s*(->\s*([^;]+))?;", block, re.S):
        params = [p.strip() for p in m.group(2).split(",") if p.strip()]
        ps = []
        for p in params:
            n, t = p.split(":", 1)
            ps.append((n.strip(), " ".join(t.split())))
        out[m.group(1)] = (" ".join((m.group(4) or "()").split()), ps)
    return out


def test_crate_files_exist():
    for f in ("Cargo.toml", "build.rs", os.path.join("src", "lib.rs")):
        assert os.path.exists(os.path.join(CRATE, f)), f
    build = open(os.path.join(CRATE, "build.rs")).read()
    assert "arch=compute_100a,code=sm_100a" in build
    for src in ("attn_fwd.cu", "block_ops.cu", "dequant.cu", "gemm.cu", "host_layout.cpp", "tp.cpp"):
        assert src in build  # every library source is compiled
        assert os.path.exists(os.path.join(ROOT, "qwen3-image21_b200", "csrc", src))


def test_attn_args_matches_header():
    c = header_struct("b200_attn_args")
    r = rust_struct("AttnArgs")
    assert [n for n, _ in c] == [n for n, _ in r]
    for (n, ct), (_, rt) in zip(c, r):
        assert C_TO_RUST[ct] == rt, (n, ct, rt)


def test_kv_desc_matches_header():
    c = header_struct("b200_kv_desc")
    r = rust_struct("KvDesc")
    assert [(n, C_TO_RUST[t]) for n, t in c] == r


def test_extern_block_matches_header():
    c = header_functions()
    r = rust_functions()
    assert set(c) == set(r), set(c) ^ set(r)
    for name, (cret, cps) in c.items():
        rret, rps = r[name]
        assert C_TO_RUST[cret] == rret, (name, cret, rret)
        assert len(cps) == len(rps), name
        for (cn, ct), (rn, rt) in zip(cps, rps):
            assert C_TO_RUST[ct] == rt, (name, cn, ct, rt)


def test_constants_match_header():
    h = open(HEADER).read()
    src = rust_source()
    for cname, rname in (("B200_ATTN_HEAD_DIM", "B200_ATTN_HEAD_DIM"),
                         ("B200_ATTN_ABI_VERSION", "B200_ATTN_ABI_VERSION"),
                         ("B200_ATTN_SPLIT_WORKSPACE_BYTES", "B200_ATTN_SPLIT_WORKSPACE_BYTES")):
        cv = int(re.search(r"#define " + cname + r"\s+(\d+)", h).group(1))
        rv = int(re.search(r"pub const " + rname + r": \w+ = (\d+);", src).group(1))
        assert cv == rv, cname
    codes = dict(re.findall(r"(B200_(?:OK|ERR_\w+))\s*=\s*(-?\d+)", h))
    for k, v in codes.items():
        assert re.search(r"pub const " + k + r": c_int = " + v + ";", src), k
