"""The C ABI seen from C and from the Rust bindings (no GPU).

* `c_abi_check.c`, compiled with the system C compiler against
  include/lfm_cuda.h and linked with liblfm2_b200.so, prints the struct
  layouts and calls the entry points that need no device.
* The Rust FFI crate (lfm2-w9100-rust_b200/rust/lfm2-cuda-sys/src/lib.rs) is
  not compiled here (no Rust toolchain): its `#[repr(C)]` structs are laid out
  by the C rules in Python and compared with the C compiler's offsets, and its
  `extern "C"` block is compared with the header (same functions, same
  argument counts).
"""

import os
import re
import shutil
import subprocess

import pytest

from conftest import PKG, ROOT

LIB_RS = os.path.join(PKG, "rust", "lfm2-cuda-sys", "src", "lib.rs")
HEADER = os.path.join(ROOT, "include", "lfm_cuda.h")
RUST_TYPES = {"u32": (4, 4), "f32": (4, 4), "u64": (8, 8), "i32": (4, 4), "i64": (8, 8)}


@pytest.fixture(scope="module")
def c_report(tmp_path_factory):
    import lfm2_b200
    lfm2_b200.lib()  # the library exists (built)
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    exe = str(tmp_path_factory.mktemp("cabi") / "c_abi_check")
    subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "c_abi_check.c"), "-o", exe, "-L", PKG, "-llfm2_b200",
                    f"-Wl,-rpath,{PKG}"], check=True)
    out = subprocess.run([exe, "/nonexistent/model.gguf"], check=True, capture_output=True, text=True).stdout
    return out.splitlines()


def rust_struct(name):
    src = open(LIB_RS).read()
    body = re.search(r"pub struct " + name + r"\s*\{(.*?)\}", src, re.S).group(1)
    fields = re.findall(r"pub (\w+):\s*([^,]+),", body)
    off, out, align_max = 0, {}, 1
    for f, ty in fields:
        ty = ty.strip()
        m = re.fullmatch(r"\[(\w+);\s*(\d+)\]", ty)
        size, align = (RUST_TYPES[m.group(1)][0] * int(m.group(2)), RUST_TYPES[m.group(1)][1]) if m else RUST_TYPES[ty]
        off = (off + align - 1) // align * align
        out[f] = (off, size)
        off += size
        align_max = max(align_max, align)
    return out, (off + align_max - 1) // align_max * align_max


@pytest.mark.parametrize("name", ["lfm_hparams", "lfm_counters"])
def test_rust_repr_c_layout_matches_c(c_report, name):
    fields, size = rust_struct(name)
    c_fields = {}
    for ln in c_report:
        p = ln.split()
        if p[0] == name:
            c_fields[p[1]] = (int(p[2]), int(p[3]))
        if p[:2] == ["size", name]:
            c_size = int(p[2])
    assert fields == c_fields
    assert size == c_size


def test_c_caller_gets_status_and_message(c_report):
    line = next(ln for ln in c_report if ln.startswith("inspect "))
    assert line.startswith("inspect 2 "), line  # LFM_ERR_MODEL
    assert "open model file" in line
    assert "q6k_device_bytes 3440640" in c_report  # 2048 rows x 8 blocks x 210 B


def _header_functions():
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for m in re.finditer(r"^[A-Za-z_][\w \*]*?\b(lfm_\w+)\s*\((.*?)\);", src, flags=re.M | re.S):
        args = m.group(2).strip()
        out[m.group(1)] = 0 if args in ("", "void") else args.count(",") + 1
    return out


def _rust_functions():
    src = open(LIB_RS).read()
    block = "\n".join(re.findall(r'extern "C" \{(.*?)\n\}', src, re.S))
    out = {}
    for m in re.finditer(r"pub fn (lfm_\w+)\((.*?)\)", block, re.S):
        args = m.group(2).strip()
        out[m.group(1)] = 0 if not args else args.rstrip(",").count(",") + 1
    return out


def test_rust_bindings_cover_the_header():
    assert _rust_functions() == _header_functions()
