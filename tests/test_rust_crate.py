"""The Rust binding crate (crates/llm-cuda) against the C header (no GPU, no rustc).

Neither this container nor the GPU box has a Rust toolchain, so the crate
cannot be compiled here.  What can be checked is that its declarations say
what the header says: every function of include/llmhost_kv.h is declared in
src/ffi.rs with the same number of parameters, the same parameter types
(C type -> Rust type) and the same return type, and the three #[repr(C)]
structs list the header's fields in the header's order with matching types.
"""
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "llmhost_kv.h"
CRATE = ROOT / "crates" / "llm-cuda"
FFI = CRATE / "src" / "ffi.rs"

C_TO_RUST = {
    "int": "i32", "int32_t": "i32", "uint32_t": "u32", "int64_t": "i64", "uint64_t": "u64", "float": "f32",
    "double": "f64", "kv_sched": "kv_sched",
    "size_t": "usize", "void": "c_void", "char": "c_char",
    "kv_pool": "kv_pool", "kv_state": "kv_state", "kv_pool_config": "kv_pool_config",
    "kv_token_move": "kv_token_move", "kv_tree_error": "kv_tree_error",
}


def _strip_c_comments(s: str) -> str:
    s = re.sub(r"/\*.*?\*/", " ", s, flags=re.S)
    return re.sub(r"//[^\n]*", " ", s)


def _c_type(decl: str) -> str:
    """'const uint32_t *block_tables' -> '*const u32'; 'int32_t n' -> 'i32'."""
    decl = decl.strip()
    stars = decl.count("*")
    toks = decl.replace("*", " * ").split()
    const_ptr = toks[0] == "const" and stars > 0
    toks = [t for t in toks if t not in ("const", "*")]
    if stars:  # the last token is the name
        base = toks[0]
    else:
        base = toks[0] if len(toks) == 1 else toks[0]
    rust = C_TO_RUST[base]
    if stars == 0:
        return rust
    if stars == 1:
        return ("*const " if const_ptr else "*mut ") + rust
    assert stars == 2
    return "*mut *mut " + rust  # kv_pool **out


def header_functions():
    text = _strip_c_comments(HEADER.read_text())
    text = re.sub(r"#[^\n]*", " ", text)
    funcs = {}
    for m in re.finditer(r"\b(int|size_t|void\s*\*|const\s+char\s*\*)\s*(kv_\w+)\s*\(([^)]*)\)\s*;", text):
        ret, name, args = m.group(1), m.group(2), m.group(3)
        params = [] if args.strip() in ("", "void") else [_c_type(a) for a in args.split(",")]
        ret = {"int": "i32", "size_t": "usize"}.get(ret.strip(), None) or (
            "*const c_char" if "char" in ret else "*mut c_void")
        funcs[name] = (params, ret)
    return funcs


def _norm_rust(t: str) -> str:
    return re.sub(r"\s+", " ", t.strip())


def rust_functions():
    text = FFI.read_text()
    text = re.sub(r"//[^\n]*", " ", text)
    body = text[text.index('#[link(name = "llmhost_kv")]'):]
    body = body[body.index("{") + 1:]
    depth, end = 1, 0
    for i, ch in enumerate(body):
        depth += ch == "{"
        depth -= ch == "}"
        if depth == 0:
            end = i
            break
    body = body[:end]
    funcs = {}
    for m in re.finditer(r"pub fn (\w+)\s*\(([^)]*)\)\s*(?:->\s*([^;]+))?;", body, flags=re.S):
        name, args, ret = m.group(1), m.group(2), (m.group(3) or "()").strip()
        params = []
        for a in args.split(","):
            a = a.strip()
            if a:
                params.append(_norm_rust(a.split(":", 1)[1]))
        funcs[name] = (params, _norm_rust(ret))
    return funcs


def test_every_header_function_is_bound_with_the_same_signature():
    h, r = header_functions(), rust_functions()
    assert len(h) >= 40, sorted(h)
    assert set(h) == set(r), (sorted(set(h) - set(r)), sorted(set(r) - set(h)))
    for name, (params, ret) in h.items():
        rp, rr = r[name]
        assert len(rp) == len(params), (name, len(rp), len(params))
        assert rp == params, (name, rp, params)
        assert rr == ret, (name, rr, ret)


def _c_struct_fields(name):
    text = _strip_c_comments(HEADER.read_text())
    m = re.search(r"typedef struct \{([^}]*)\}\s*" + name + r"\s*;", text)
    assert m, name
    out = []
    for ln in m.group(1).split(";"):
        ln = ln.strip()
        if ln:
            ty, field = ln.rsplit(None, 1)
            out.append((field, C_TO_RUST[ty]))
    return out


def _rust_struct_fields(name):
    text = FFI.read_text()
    m = re.search(r"pub struct " + name + r"\s*\{([^}]*)\}", text)
    assert m, name
    out = []
    for ln in m.group(1).split(","):
        ln = ln.strip()
        if ln:
            field, ty = ln.replace("pub ", "").split(":")
            out.append((field.strip(), ty.strip()))
    return out


def test_repr_c_structs_match_the_header():
    for name in ("kv_pool_config", "kv_token_move", "kv_tree_error"):
        assert _rust_struct_fields(name) == _c_struct_fields(name), name


def test_constants_match_the_header():
    h = _strip_c_comments(HEADER.read_text())
    rs = FFI.read_text()
    for m in re.finditer(r"\b(KV_(?:OK|ERR_\w+|DTYPE_\w+|TREE_\w+))\s*=\s*(\d+)", h):
        name, val = m.group(1), int(m.group(2))
        rm = re.search(r"pub const " + name + r": i32 = (\d+);", rs)
        assert rm and int(rm.group(1)) == val, name
    assert "pub const KV_PAGE_NONE: u32 = 0xFFFF_FFFF;" in rs
    assert "pub const KV_API_VERSION: i32 = 1;" in rs and "#define KV_API_VERSION 1" in HEADER.read_text()


def test_crate_files_present_and_backend_implemented():
    cargo = (CRATE / "Cargo.toml").read_text()
    assert 'name = "llm-cuda"' in cargo and 'links = "llmhost_kv"' in cargo and "llm-core" in cargo
    build = (CRATE / "build.rs").read_text()
    assert "llmhost_b200.build" in build and "rustc-link-lib=dylib=llmhost_kv" in build
    lib = (CRATE / "src" / "lib.rs").read_text()
    # llm_core::Backend (crates/llm-core/src/backend.rs:4-13): Buffer, name(), alloc(len)
    assert "impl llm_core::Backend for CudaBackend" in lib
    assert "type Buffer = DeviceBuffer;" in lib
    assert 'fn name(&self) -> &\'static str' in lib and "fn alloc(&self, len: usize) -> DeviceBuffer" in lib
    # every unsafe block in the crate states why it is sound
    for f in (CRATE / "src").glob("*.rs"):
        lines = f.read_text().splitlines()
        for i, ln in enumerate(lines):
            if re.search(r"\bunsafe \{", ln) and "unsafe impl" not in ln:
                ctx = "\n".join(lines[max(0, i - 3):i + 1])
                assert "SAFETY" in ctx or "# Safety" in "\n".join(lines[max(0, i - 30):i]), (f.name, i + 1)
