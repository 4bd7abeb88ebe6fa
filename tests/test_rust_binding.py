"""CPU checks of the Rust drop-in crate (nodestor-cuda/) against the C ABI.

No Rust toolchain exists here, so the crate is checked as text: every
function include/nsq.h declares appears in nodestor-cuda/src/ffi.rs under the
same name with the same number of arguments, ffi.rs declares nothing the
header lacks, and the status, type and layout constants have the header's
values.  The engine wrapper (src/lib.rs) must map every status onto a
NodeStorError variant and keep the reference operator's matmul signature
(crates/nodestor-vulkan/src/lib.rs:117-122).
"""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _strip_c_comments(s):
    return re.sub(r"/\*.*?\*/", "", s, flags=re.S)


def _count_args(arglist: str) -> int:
    a = arglist.strip()
    if a in ("", "void"):
        return 0
    return len([p for p in a.split(",") if p.strip()])


def header_functions():
    src = _strip_c_comments(open(os.path.join(ROOT, "include", "nsq.h")).read())
    out = {}
    for m in re.finditer(r"\b(nsq_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", src, flags=re.S):
        out[m.group(1)] = _count_args(m.group(2))
    return out


def header_constants():
    src = _strip_c_comments(open(os.path.join(ROOT, "include", "nsq.h")).read())
    return {m.group(1): int(m.group(2)) for m in re.finditer(r"#define\s+(NSQ_[A-Z0-9_]+)\s+(-?\d+)\b", src)}


def rust_source(name):
    return open(os.path.join(ROOT, "nodestor-cuda", "src", name)).read()


def rust_functions():
    src = re.sub(r"//[^\n]*", "", rust_source("ffi.rs"))
    block = src[src.index('extern "C" {'):src.index("pub mod cudart")]
    out = {}
    for m in re.finditer(r"pub fn (nsq_[a-z0-9_]+)\s*\(([^)]*)\)", block, flags=re.S):
        out[m.group(1)] = _count_args(m.group(2))
    return out


def test_crate_files_exist():
    for f in ("Cargo.toml", "build.rs", "src/ffi.rs", "src/lib.rs"):
        assert os.path.exists(os.path.join(ROOT, "nodestor-cuda", f)), f


def test_ffi_declares_every_header_function_with_its_arity():
    h, r = header_functions(), rust_functions()
    assert len(h) >= 25
    assert set(h) == set(r), (sorted(set(h) - set(r)), sorted(set(r) - set(h)))
    for name, n in h.items():
        assert r[name] == n, (name, n, r[name])


def test_ffi_constants_match_header():
    hc = header_constants()
    src = rust_source("ffi.rs")
    consts = {m.group(1): int(m.group(2)) for m in re.finditer(r"pub const (NSQ_[A-Z0-9_]+): \w+ = (-?\d+);", src)}
    assert len(consts) >= 20
    for name, v in consts.items():
        assert name in hc, name
        assert hc[name] == v, (name, v, hc[name])
    assert "NSQ_OK" in consts


def test_struct_fields_match_header():
    src = _strip_c_comments(open(os.path.join(ROOT, "include", "nsq.h")).read())
    rs = rust_source("ffi.rs")
    for c_name, r_name in (("nsq_segment", "NsqSegment"), ("nsq_xsegment", "NsqXSegment")):
        body = re.search(r"typedef struct " + c_name + r"\s*\{(.*?)\}", src, flags=re.S).group(1)
        c_fields = [f.strip().split()[-1].lstrip("*") for f in body.split(";") if f.strip()]
        rbody = re.search(r"pub struct " + r_name + r"\s*\{(.*?)\}", rs, flags=re.S).group(1)
        r_fields = re.findall(r"pub (\w+):", rbody)
        assert [f.lower() for f in c_fields] == [f.lower() for f in r_fields], (c_name, c_fields, r_fields)


def test_engine_keeps_the_reference_signature_and_maps_every_status():
    lib = rust_source("lib.rs")
    assert re.search(r"pub fn matmul\(&self, a: &CudaBuffer, b: &CudaBuffer, m: u32, k: u32, n: u32\)\s*->\s*"
                     r"Result<CudaBuffer, NodeStorError>", lib)
    for code in ("NSQ_ERR_TYPE", "NSQ_ERR_SHAPE", "NSQ_ERR_ALIGN", "NSQ_ERR_NULL", "NSQ_ERR_WORKSPACE",
                 "NSQ_ERR_FORMAT", "NSQ_ERR_TIMEOUT"):
        assert f"ffi::{code}" in lib, code
    for variant in ("NotSupported", "ConfigError", "InvalidModelFormat", "Timeout", "VulkanError"):
        assert f"NodeStorError::{variant}" in lib, variant
    build = open(os.path.join(ROOT, "nodestor-cuda", "build.rs")).read()
    assert "cargo:rustc-link-lib=dylib=nsq" in build and "planejaja_b200" in build
