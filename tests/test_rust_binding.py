"""The committed Rust binding (qwen3-tts-hip_b200/rust/src/lib.rs) against the
C header: every entry point of include/qtts_b200.h is declared in the
binding's extern block with the same parameter and return types, and the
#[repr(C)] structs have the header's fields in the header's order. No Rust
toolchain is present, so this is a textual check of the signatures."""
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "qtts_b200.h"
BINDING = ROOT / "qwen3-tts-hip_b200" / "rust" / "src" / "lib.rs"

SCALARS = {"int32_t": "i32", "uint32_t": "u32", "size_t": "usize", "uint64_t": "u64",
           "float": "f32", "double": "f64", "char": "c_char", "void": "()"}


def strip_comments(text):
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.sub(r"//[^\n]*", "", text)


def c_type_to_rust(ctype):
    t = ctype.strip()
    const = t.startswith("const ")
    t = t.replace("const ", "").strip()
    stars = t.count("*")
    base = t.replace("*", "").strip()
    r = SCALARS.get(base, base)
    if stars == 0:
        return r
    out = ("*const " if const else "*mut ") + r
    for _ in range(stars - 1):
        out = "*mut " + out
    return out


def header_functions():
    text = strip_comments(HEADER.read_text())
    funcs = {}
    for m in re.finditer(r"\b(int32_t|void|const char\*)\s+(qtts_\w+)\s*\(([^)]*)\)\s*;", text):
        ret, name, params = m.groups()
        args = []
        if params.strip() != "void":
            for p in params.split(","):
                p = " ".join(p.split())
                pm = re.match(r"(.*?)(\w+)$", p)
                args.append(c_type_to_rust(pm.group(1)))
        funcs[name] = (None if ret == "void" else c_type_to_rust(ret), args)
    return funcs


def binding_functions():
    text = BINDING.read_text()
    block = text[text.index('extern "C" {'):]
    block = block[: block.index("\n    }\n")]
    funcs = {}
    for m in re.finditer(r"pub fn (qtts_\w+)\((.*?)\)\s*(->\s*([^;]+))?;", block, re.S):
        name, params, _, ret = m.groups()
        args = []
        for p in params.split(","):
            p = " ".join(p.split())
            if not p:
                continue
            args.append(p.split(":", 1)[1].strip())
        funcs[name] = (ret.strip() if ret else None, args)
    return funcs


def test_every_entry_point_bound_with_the_same_signature():
    h, b = header_functions(), binding_functions()
    assert len(h) >= 30
    assert set(h) == set(b), (set(h) ^ set(b))
    for name, sig in h.items():
        assert b[name] == sig, (name, sig, b[name])


def _c_struct_fields(name):
    text = strip_comments(HEADER.read_text())
    m = next(m for m in re.finditer(r"typedef struct \{([^{}]*)\}\s*(\w+)\s*;", text)
             if m.group(2) == name)
    fields = []
    for line in m.group(1).split(";"):
        line = " ".join(line.split())
        if not line:
            continue
        fm = re.match(r"(.*?)(\w+)(\[(\d+)\])?$", line)
        ty = c_type_to_rust(fm.group(1))
        if fm.group(4):
            ty = f"[{ty}; {fm.group(4)}]"
        fields.append((fm.group(2), ty))
    return fields


def _rust_struct_fields(name):
    text = BINDING.read_text()
    m = re.search(r"pub struct " + name + r" \{(.*?)\n    \}", text, re.S)
    out = []
    for line in m.group(1).split(","):
        line = " ".join(line.split())
        if line.startswith("pub "):
            f, ty = line[4:].split(":", 1)
            out.append((f.strip(), ty.strip()))
    return out


def test_structs_match_the_header():
    for name in ("qtts_generate_options", "qtts_stream_options", "qtts_text_stream_options",
                 "qtts_codes_chunk", "qtts_engine_info"):
        assert _c_struct_fields(name) == _rust_struct_fields(name), name


def test_error_mapping_keeps_cuda_apart_from_invalid_input():
    text = BINDING.read_text()
    body = text[text.index("pub fn check("):]
    body = body[: body.index("\n}\n")]
    assert "QTTS_ERR_INVALID_INPUT | ffi::QTTS_ERR_CACHE_FULL => {" in body
    assert "QTTS_ERR_CUDA | ffi::QTTS_ERR_DEVICE_STATE => {" in body
    assert "Error::Cuda { call, status, message: last_error() }" in body
    assert "QTTS_ERR_IO => Err(Error::Io(" in body
