"""The Rust binding (rust/src/gpu_gemm/ffi.rs) against the C header and the
library, on CPU. The image has no Rust toolchain, so the binding is checked
as text: every constant equals the header's value, every #[repr(C)] struct
lists the header's fields in the header's order (the same order the ctypes
mirror uses), and every declared function is one the library exports."""
import os
import re

import pytest

from momiru_b200 import _abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
def _read(*parts):
    with open(os.path.join(ROOT, *parts)) as f:
        return f.read()


FFI = _read("rust", "src", "gpu_gemm", "ffi.rs")
HEADER = _read("include", "momiru_gemm.h")


def header_constants():
    consts = {}
    for name, value in re.findall(r"\b(MMR_[A-Z0-9_]+)\s*=\s*(\d+)", HEADER):
        consts[name] = int(value)
    m = re.search(r"#define MMR_MAX_RANK (\d+)", HEADER)
    consts["MMR_MAX_RANK"] = int(m.group(1))
    return consts


def rust_struct_fields(name):
    m = re.search(r"pub struct %s \{(.*?)\n\}" % name, FFI, re.S)
    assert m, name
    return re.findall(r"pub (\w+):", m.group(1))


def test_constants_match_the_header():
    hc = header_constants()
    rust = dict((n, int(v)) for n, v in re.findall(r"pub const (MMR_\w+): (?:i32|usize) = (\d+);", FFI))
    assert rust, "no constants parsed"
    for name, value in rust.items():
        assert hc.get(name) == value, (name, value, hc.get(name))
    # every status code of the header is bound
    for name in hc:
        if name.startswith("MMR_ERR_") or name == "MMR_OK":
            assert name in rust, name


@pytest.mark.parametrize("rust_name,ctype", [
    ("mmr_view", _abi.MmrView), ("mmr_matmul_desc", _abi.MmrMatmulDesc), ("mmr_gemm_info", _abi.MmrGemmInfo),
    ("mmr_launch_record", _abi.MmrLaunchRecord), ("mmr_ipc_handle", _abi.MmrIpcHandle),
    ("mmr_sharded_desc", _abi.MmrShardedDesc),
])
def test_structs_follow_the_header_layout(rust_name, ctype):
    assert rust_struct_fields(rust_name) == [f for f, _ in ctype._fields_]
    # and the header declares the same field names in the same order
    m = re.search(r"typedef struct %s \{(.*?)\} %s;" % (rust_name, rust_name), HEADER, re.S)
    assert m, rust_name
    body = re.sub(r"/\*.*?\*/", "", m.group(1), flags=re.S)
    names = []
    for decl in body.split(";"):
        decl = decl.strip()
        if not decl:
            continue
        for part in decl.split(","):
            tok = re.findall(r"\*?\s*(\w+)\s*(?:\[[^\]]*\])?\s*$", part.strip())
            names.append(tok[0])
    assert names == rust_struct_fields(rust_name)


def test_declared_functions_are_exported():
    fns = re.findall(r"pub fn (mmr_\w+)\(", FFI)
    assert len(fns) >= 18
    for fn in fns:
        assert fn in _abi.EXPORTED, fn
        assert re.search(r"MMR_API\s+(?:int32_t|const char \*)\s*%s\s*\(" % fn, HEADER), fn
