"""The Rust binding (ane-infer_b200/rust/src/lib.rs) against the C header it declares, read
as text (this image has no Rust toolchain): every extern function exists in include/ab2.h with
the same parameter count and parameter types, and the #[repr(C)] structs list the header's fields
in the same order with the same types."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = open(os.path.join(ROOT, "include", "ab2.h")).read()
RUST = open(os.path.join(ROOT, "ane-infer_b200", "rust", "src", "lib.rs")).read()

C_TO_RUST = {"int": "c_int", "int32_t": "i32", "int64_t": "i64", "uint64_t": "u64", "uint32_t": "u32",
             "float": "f32", "double": "f64", "uint8_t": "u8", "char": "c_char", "void": "c_void"}


def _strip_comments(s):
    return re.sub(r"/\*.*?\*/", "", s, flags=re.S)


def _split_params(p):
    p = " ".join(p.split())
    return [] if p in ("", "void") else [x.strip() for x in p.split(",")]


def c_functions():
    h = _strip_comments(HEADER)
    out = {}
    for m in re.finditer(r"([A-Za-z_][\w \*]*?)\b(ab2_\w+)\s*\(([^;{]*?)\)\s*;", h, flags=re.S):
        ret = " ".join(m.group(1).split()[-3:])  # the return type ends the text before the name
        ret = re.sub(r"^.*?\b(const char ?\*|int|void)\s*$", r"\1", ret)
        out[m.group(2)] = (_split_params(m.group(3)), ret.replace(" ", ""))
    return out


def c_param_type(p):
    """'const float* x' -> ('f32', '*const'); 'ab2_ctx** out' -> ('ab2_ctx', '*mut *mut')."""
    p = p.replace("*", " * ")
    toks = p.split()
    const = "const" in toks
    toks = [t for t in toks if t != "const"]
    stars = toks.count("*")
    base = [t for t in toks if t != "*"][0]
    base = C_TO_RUST.get(base, base)
    if stars == 0:
        return base, ""
    # the innermost pointee keeps the const, outer levels are mutable
    ptr = ("*const" if const else "*mut") + " *mut" * (stars - 1)
    return base, ptr


def rust_functions():
    block = RUST[RUST.index('extern "C" {'):]
    block = block[: block.index("\n    }\n")]
    out = {}
    for m in re.finditer(r"pub fn (ab2_\w+)\(([^)]*)\)\s*(->\s*([^;]+))?;", block, flags=re.S):
        out[m.group(1)] = (_split_params(m.group(2)), (m.group(4) or "").strip())
    return out


def rust_param_type(p):
    ty = p.split(":", 1)[1].strip()
    ptr = " ".join(re.findall(r"\*(?:const|mut)", ty))
    base = re.sub(r"\*(?:const|mut)\s*", "", ty).strip()
    return base, ptr


def test_every_rust_extern_matches_the_header():
    cf, rf = c_functions(), rust_functions()
    assert len(rf) >= 15
    rets = {"int": "c_int", "void": "", "constchar*": "*const c_char"}
    for name, (rparams, rret) in rf.items():
        assert name in cf, f"{name} is not declared in include/ab2.h"
        cparams, cret = cf[name]
        assert rets[cret] == rret, (name, cret, rret)
        assert len(rparams) == len(cparams), (name, rparams, cparams)
        for rp, cp in zip(rparams, cparams):
            assert rust_param_type(rp) == c_param_type(cp), (name, rp, cp)


def _c_struct_fields(name):
    h = _strip_comments(HEADER)
    body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (name, name), h, flags=re.S).group(1)
    fields = []
    for decl in body.split(";"):
        decl = " ".join(decl.split())
        if not decl:
            continue
        ctype, rest = decl.split(" ", 1)
        for f in rest.split(","):
            f = f.strip()
            m = re.match(r"(\w+)\[(\d+)\]", f)
            if m:
                fields.append((m.group(1), f"[{C_TO_RUST[ctype]}; {m.group(2)}]"))
            else:
                fields.append((f, C_TO_RUST[ctype]))
    return fields


def _rust_struct_fields(name):
    body = re.search(r"pub struct %s \{(.*?)\}" % name, RUST, flags=re.S).group(1)
    return [(n, t.strip()) for n, t in re.findall(r"pub (\w+): ([^,\n]+),", body)]


def test_repr_c_structs_match_the_header():
    for name in ("ab2_options", "ab2_config"):
        assert _rust_struct_fields(name) == _c_struct_fields(name), name
