"""CPU-side checks of the C ABI: the library builds, loads and exports every
entry point include/xvec_gpu.h declares (no compute without a GPU)."""
import os
import re
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    text = open(os.path.join(ROOT, "include", "xvec_gpu.h")).read()
    return sorted(set(re.findall(r"\b(xvec_gpu_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from xvec_b200 import LIB_PATH
    out = subprocess.run(["nm", "-D", "--defined-only", LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (xvec_gpu_\w+)", out))
    missing = [s for s in _declared_symbols() if s not in exported]
    assert not missing, missing


def test_python_binding_lists_every_declared_symbol():
    import xvec_b200
    assert sorted(xvec_b200.EXPORTED_SYMBOLS) == _declared_symbols()


def test_abi_version_and_errors_without_gpu():
    import ctypes
    import xvec_b200
    lib = xvec_b200.library()
    assert lib.xvec_gpu_abi_version() == 2
    # Invalid descriptors fail before any device work.
    desc = xvec_b200.IndexDesc(xvec_b200.INDEX_FLAT, 0, 1, 1, 0)
    h = ctypes.c_void_p()
    st = lib.xvec_gpu_index_create(ctypes.byref(desc), ctypes.byref(h))
    assert st == xvec_b200.INVALID_ARGUMENT
    assert "dimension" in xvec_b200.last_error()


def test_library_is_built_for_sm100a():
    from xvec_b200 import LIB_PATH
    out = subprocess.run(["cuobjdump", "--list-elf", LIB_PATH], capture_output=True, text=True)
    if out.returncode == 0:
        assert "sm_100a" in out.stdout
