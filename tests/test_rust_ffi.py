"""The Rust binding crate (rust/qwen-cuda-sys) against the C header, without a Rust toolchain.

There is no cargo/rustc here, so the crate cannot be compiled; instead this checks, by parsing
both sources, that every `#[repr(C)]` struct has the header's fields in the same order with the
same types (so the same offsets and size, computed with ctypes) and that every function the
header declares is declared in the crate's `extern "C"` block with the same parameter types.
It also checks that the `--device cuda` patch for the reference crate applies to it (when the
reference checkout is present)."""
import ctypes as C
import re
import shutil
import subprocess

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "qwen_cuda.h"
LIB_RS = ROOT / "rust" / "qwen-cuda-sys" / "src" / "lib.rs"
PATCH = ROOT / "rust" / "qwen-rust-cuda" / "device-cuda.patch"
REFERENCE = ROOT.parent / "reference"

SCALARS = {  # canonical name: (C spellings, Rust spellings, ctypes type)
    "u8": (("uint8_t",), ("u8",), C.c_uint8),
    "u32": (("uint32_t",), ("u32",), C.c_uint32),
    "u64": (("uint64_t",), ("u64",), C.c_uint64),
    "usize": (("size_t",), ("usize",), C.c_size_t),
    "int": (("int",), ("c_int", "i32"), C.c_int),
    "f32": (("float",), ("f32", "c_float"), C.c_float),
    "f64": (("double",), ("f64",), C.c_double),
    "char": (("char",), ("c_char",), C.c_char),
    "void": (("void",), ("c_void",), None),
}
OPAQUE = ("qc_engine", "qc_matrix", "qc_sampler", "qc_batch", "qc_config", "qc_tensor_desc", "qc_stats",
          "qc_phase_times")


def _canon_scalar(tok: str, lang: int) -> str:
    for k, v in SCALARS.items():
        if tok in v[lang]:
            return k
    if tok in OPAQUE:
        return tok
    raise AssertionError(f"unknown type {tok!r}")


def c_type(decl: str):
    """'const qc_engine* e' / 'qc_engine** out' / 'qc_sampler* const* s' / 'uint32_t n' -> canonical
    nested tuple.  A const before the base type, or after the k-th '*', makes the next pointer level
    point to const data (Rust *const)."""
    toks = re.findall(r"\*|\w+", decl)
    const_next = False
    if toks[0] == "const":
        const_next = True
        toks = toks[1:]
    t = _canon_scalar(toks[0], 0)
    rest = toks[1:]
    if rest and rest[-1] not in ("*", "const"):
        rest = rest[:-1]  # the parameter name
    for tok in rest:
        if tok == "*":
            t = ("ptr", "const" if const_next else "mut", t)
            const_next = False
        else:
            assert tok == "const", decl
            const_next = True
    return t


def rust_type(s: str):
    s = s.strip()
    if s.startswith("*const ") or s.startswith("*mut "):
        kind, rest = s[1:].split(" ", 1)
        return ("ptr", kind, rust_type(rest))
    m = re.match(r"^\[(\w+);\s*(\d+)\]$", s)
    if m:
        return ("arr", _canon_scalar(m.group(1), 1), int(m.group(2)))
    return _canon_scalar(s, 1)


def header_structs() -> dict:
    text = HEADER.read_text()
    out = {}
    for body, name in re.findall(r"typedef struct \w+ \{(.*?)\} (\w+);", text, re.S):
        fields = []
        for line in re.sub(r"/\*.*?\*/", "", body, flags=re.S).split(";"):
            line = line.strip()
            if not line:
                continue
            m = re.match(r"^(const\s+)?(\w+)\s*(\*?)\s*(.+)$", line)
            const, base, star, names = m.groups()
            for nm in names.split(","):
                nm = nm.strip()
                arr = re.match(r"^(\w+)\[(\d+)\]$", nm)
                t = _canon_scalar(base, 0)
                if star:
                    t = ("ptr", "const" if const else "mut", t)
                if arr:
                    fields.append((arr.group(1), ("arr", t, int(arr.group(2)))))
                else:
                    fields.append((nm, t))
        out[name] = fields
    return out


def rust_structs() -> dict:
    text = LIB_RS.read_text()
    out = {}
    for name, body in re.findall(r"#\[repr\(C\)\]\s*(?:#\[derive[^\]]*\]\s*)?pub struct (\w+) \{(.*?)\n    \}", text, re.S):
        fields = re.findall(r"pub (\w+): ([^,\n]+),", body)
        if fields:
            out[name] = [(n, rust_type(t)) for n, t in fields]
    return out


def header_functions() -> dict:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for ret, name, params in re.findall(r"^(int|void|const char\*)\s+(qc_\w+)\((.*?)\);", text, re.S | re.M):
        ps = [p for p in (x.strip() for x in params.replace("\n", " ").split(",")) if p and p != "void"]
        out[name] = ([c_type(p) for p in ps], ret.replace(" ", ""))
    return out


def rust_functions() -> dict:
    text = LIB_RS.read_text()
    block = text[text.index('extern "C" {'):text.index("pub mod safe")]
    out = {}
    for name, params, ret in re.findall(r"pub fn (qc_\w+)\((.*?)\)\s*(?:->\s*([^;]+))?;", block, re.S):
        ps = [p.strip() for p in params.replace("\n", " ").split(",") if p.strip()]
        out[name] = ([rust_type(p.split(":", 1)[1]) for p in ps], (ret or "").strip())
    return out


def _ctype(t):
    if isinstance(t, tuple) and t[0] == "ptr":
        return C.c_void_p
    if isinstance(t, tuple) and t[0] == "arr":
        return SCALARS[t[1]][2] * t[2]
    return SCALARS[t][2]


def _layout(fields):
    S = type("S", (C.Structure,), {"_fields_": [(n, _ctype(t)) for n, t in fields]})
    return C.sizeof(S), [getattr(S, n).offset for n, _ in fields]


def test_repr_c_structs_match_the_header():
    h, r = header_structs(), rust_structs()
    assert set(h) == {"qc_config", "qc_tensor_desc", "qc_stats", "qc_phase_times"}
    for name, fields in h.items():
        assert name in r, f"{name} missing from lib.rs"
        assert r[name] == fields, (name, r[name], fields)
        assert _layout(r[name]) == _layout(fields)
    assert _layout(h["qc_tensor_desc"])[0] == 56 and _layout(h["qc_config"])[0] == 48


def test_every_header_function_is_bound_with_the_same_signature():
    h, r = header_functions(), rust_functions()
    assert len(h) >= 47
    missing = sorted(set(h) - set(r))
    assert not missing, f"not declared in lib.rs: {missing}"
    ret_map = {"int": "c_int", "void": "", "constchar*": "*const c_char"}
    for name, (params, ret) in h.items():
        rp, rret = r[name]
        assert rp == params, (name, rp, params)
        assert rret == ret_map[ret], (name, rret, ret)
    assert not set(r) - set(h), "lib.rs declares functions the header does not"


def test_exports_cover_the_header(cuda_engine):
    """Every function the header (and so the Rust crate) declares is in the export list that
    tests/test_capi.py checks against the built library."""
    assert set(header_functions()) <= set(cuda_engine.EXPORTS)


@pytest.mark.skipif(not REFERENCE.exists() or shutil.which("git") is None, reason="reference checkout absent")
def test_device_cuda_patch_applies_to_the_reference(tmp_path):
    work = tmp_path / "qwen-rust"
    shutil.copytree(REFERENCE, work, ignore=shutil.ignore_patterns(".git", "target"))
    r = subprocess.run(["git", "apply", "--unidiff-zero", str(PATCH)], cwd=work, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    main = (work / "src" / "main.rs").read_text()
    assert "Device::Cuda => Box::new(qwen_rust::cuda::CudaBackend::new(self.cuda_device)?)" in main
    assert "fn forward_token(" in (work / "src" / "backend.rs").read_text()
    assert "backend.forward_token(" in (work / "src" / "model.rs").read_text()
    assert 'cuda = ["dep:qwen-cuda-sys"]' in (work / "Cargo.toml").read_text()
