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
    assert lib.xvec_gpu_abi_version() == 4
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


def test_communicator_entry_points_without_gpu():
    """The NCCL ids and the argument checks of the multi-GPU entry points
    need no device: ids are 128 bytes and distinct; nil or out-of-range
    arguments fail before any device work."""
    import ctypes
    import xvec_b200
    lib = xvec_b200.library()
    a, b = xvec_b200.Comm.unique_id(), xvec_b200.Comm.unique_id()
    assert len(a) == len(b) == xvec_b200.COMM_ID_BYTES and a != b
    h = ctypes.c_void_p()
    uid = (ctypes.c_uint8 * 128).from_buffer_copy(a)
    assert lib.xvec_gpu_comm_init_rank(0, uid, 2, 2, 1000, ctypes.byref(h)) == \
        xvec_b200.INVALID_ARGUMENT
    assert "out of range" in xvec_b200.last_error()
    assert lib.xvec_gpu_comm_init_rank(0, None, 1, 0, 1000, ctypes.byref(h)) == \
        xvec_b200.INVALID_ARGUMENT
    opts = xvec_b200.SearchOpts()
    opts.top_k = 1
    assert lib.xvec_gpu_sharded_search_device(None, None, None, 1, ctypes.byref(opts), None,
                                              None, None) == xvec_b200.INVALID_ARGUMENT
    assert lib.xvec_gpu_sharded_search(None, None, 0, None, 1, ctypes.byref(opts), None, None,
                                       None) == xvec_b200.INVALID_ARGUMENT
    assert lib.xvec_gpu_comm_size(None) == 0 and lib.xvec_gpu_comm_rank(None) == -1
    assert lib.xvec_gpu_comm_destroy(None) == 0


def test_wait_limit_setter_round_trip():
    import xvec_b200
    assert xvec_b200.set_wait_limit_ns(5_000) == 2_000_000_000
    assert xvec_b200.set_wait_limit_ns(0) == 5_000
    assert xvec_b200.set_wait_limit_ns(0) == 2_000_000_000
