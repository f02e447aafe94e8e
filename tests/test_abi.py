"""C ABI checks that need no GPU: the library loads and exports every symbol
include/mbr_b200.h declares."""
import os
import re
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "mbr_b200.h")).read()
    return sorted(set(re.findall(r"MBR_API\s+[\w\s\*]+?\b(mbr_\w+)\s*\(", src)))


def test_header_and_binding_agree():
    import cudasep

    assert declared_symbols() == sorted(cudasep.EXPORTS)


def test_library_exports_declared_symbols():
    import cudasep

    lib = cudasep.lib()  # raises if libmbr_b200.so is missing
    out = subprocess.run(["nm", "-D", "--defined-only", cudasep.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r" T (mbr_\w+)$", out, flags=re.M))
    for s in declared_symbols():
        assert s in exported, s
        assert hasattr(lib, s)
    assert lib.mbr_version() >= 100


def test_errors_surface_without_gpu_calls():
    import ctypes

    import cudasep

    lib = cudasep.lib()
    h = ctypes.c_void_p()
    rc = lib.mbr_create(b"/nonexistent/model.csm", 0, 1, ctypes.byref(h))
    assert rc != 0 and not h
    assert len(lib.mbr_last_error()) > 0
    rc = lib.mbr_get_info(None, 0, None)
    assert rc == 1 and b"null" in lib.mbr_last_error()
