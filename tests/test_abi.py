"""The C-ABI library loads on a CPU host and exports every symbol that
include/lfm_cuda.h declares (no compute calls without a GPU)."""

import os
import re

from conftest import ROOT


def _declared():
    names = []
    inc = os.path.join(ROOT, "include")
    for f in sorted(os.listdir(inc)):
        if f.endswith(".h"):
            src = open(os.path.join(inc, f)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names += re.findall(r"^[A-Za-z_][\w \*]*?\b(lfm_\w+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = _declared()
    assert "lfm_engine_create" in names and "lfm_forward_token" in names and "lfm_q6k_matmul" in names


def test_library_exports_every_declared_symbol():
    import lfm2_b200
    lib = lfm2_b200.lib()
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing
    assert sorted(lfm2_b200.EXPORTS) == _declared()


def test_engine_create_fails_cleanly_without_model():
    import ctypes

    import lfm2_b200
    lib = lfm2_b200.lib()
    h = ctypes.c_void_p()
    st = lib.lfm_engine_create(b"/nonexistent/model.gguf", 0, ctypes.byref(h))
    assert st != 0 and not h.value
    assert lib.lfm_global_error().decode()


def test_device_bytes_matches_gguf_size():
    import lfm2_b200
    lib = lfm2_b200.lib()
    assert lib.lfm_q6k_device_bytes(2048, 128000) == 128000 * 8 * 210
    assert lib.lfm_q6k_device_bytes(1792, 2048 * 32) == 2048 * 32 * 7 * 210
    assert lib.lfm_q6k_device_bytes(100, 4) == 0
