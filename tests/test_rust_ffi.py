"""The Rust FFI crate (rust/src/cuda_ffi.rs) against the C header it binds (include/arctic_cuda.h):
the same functions in the same order, each parameter and return type the Rust equivalent of the C
one, and the same #[repr(C)] struct fields. No Rust toolchain exists in this image, so the crate is
checked as text; the function list is found with the same pattern as tests/test_abi.py."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "arctic_cuda.h")
RUST = os.path.join(ROOT, "rust", "src", "cuda_ffi.rs")

BASE = {"int": "c_int", "uint32_t": "u32", "int32_t": "i32", "uint16_t": "u16", "int8_t": "i8", "uint64_t": "u64",
        "float": "f32", "double": "f64", "size_t": "usize", "char": "c_char", "void": "c_void",
        "ae_ctx": "ae_ctx", "ae_tokenizer": "ae_tokenizer", "ae_model_desc": "ae_model_desc",
        "ae_linear_desc": "ae_linear_desc", "ae_layer_desc": "ae_layer_desc"}


def c_type(decl: str) -> str:
    """Rust spelling of a C type ('const uint16_t*' -> '*const u16', 'ae_ctx* const*' -> '*const *mut ae_ctx')."""
    toks = re.findall(r"\w+|\*", decl)
    const_base = False
    if toks and toks[0] == "const":
        const_base = True
        toks = toks[1:]
    base = BASE[toks[0]]
    if len(toks) > 1 and toks[1] == "const":  # 'char const'
        const_base = True
        toks = toks[:1] + toks[2:]
    out, pointee_const = base, const_base
    for i, t in enumerate(toks[1:], 1):
        if t == "*":
            out = ("*const " if pointee_const else "*mut ") + out
            pointee_const = False
        elif t == "const":
            pointee_const = True
    return out


def c_functions():
    txt = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = []
    for ret, name, params in re.findall(r"([\w\s\*]+?)\b(ae_[a-z_0-9]+)\s*\(([^)]*)\)\s*;", txt):
        args = []
        for p in [x.strip() for x in params.split(",") if x.strip() and x.strip() != "void"]:
            m = re.match(r"(.*?)(\w+)$", p)
            args.append(c_type(m.group(1)))
        out.append((name, c_type(ret.strip()), args))
    return out


def rust_functions():
    txt = open(RUST).read()
    block = txt[txt.index('extern "C" {'):]
    out = []
    for name, params, ret in re.findall(r"pub fn (\w+)\((.*?)\)\s*(?:->\s*([^;]+?))?\s*;", block, flags=re.S):
        args = [re.sub(r"\s+", " ", a.split(":", 1)[1]).strip() for a in params.split(",") if a.strip()]
        out.append((name, (ret or "()").strip(), args))
    return out


def c_structs():
    txt = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for body, name in re.findall(r"typedef struct \{(.*?)\}\s*(\w+);", txt, flags=re.S):
        fields = []
        for f in [x.strip() for x in body.split(";") if x.strip()]:
            m = re.match(r"(.*?)(\w+)(\[(\d+)\])?$", f)
            t = c_type(m.group(1))
            fields.append((m.group(2), f"[{t}; {m.group(4)}]" if m.group(3) else t))
        out[name] = fields
    return out


def rust_structs():
    txt = open(RUST).read()
    out = {}
    for name, body in re.findall(r"pub struct (ae_\w+) \{(.*?)\n\}", txt, flags=re.S):
        fields = re.findall(r"pub (\w+): ([^,\n]+),", body)
        if fields:
            out[name] = [(n, t.strip()) for n, t in fields]
    return out


def test_functions_match_header():
    c, r = c_functions(), rust_functions()
    assert [f[0] for f in r] == [f[0] for f in c]
    for (name, cret, cargs), (_, rret, rargs) in zip(c, r):
        assert rret == cret, (name, rret, cret)
        assert rargs == cargs, (name, rargs, cargs)


def test_function_set_is_the_abi_test_set():
    from test_abi import declared

    assert sorted(f[0] for f in rust_functions()) == declared()


def test_structs_match_header():
    c, r = c_structs(), rust_structs()
    assert set(c) == {"ae_linear_desc", "ae_layer_desc", "ae_model_desc"}
    for name, fields in c.items():
        assert r[name] == fields, name


def test_type_mapping_examples():
    assert c_type("const uint16_t*") == "*const u16"
    assert c_type("ae_ctx* const*") == "*const *mut ae_ctx"
    assert c_type("const char* const*") == "*const *const c_char"
    assert c_type("ae_tokenizer**") == "*mut *mut ae_tokenizer"
    assert c_type("int") == "c_int"
