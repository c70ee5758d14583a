"""The C-ABI library loads and exports every function include/mcpm.h declares (no GPU needed)."""
import os
import re

from conftest import REPO


def declared_symbols():
    src = open(os.path.join(REPO, "include", "mcpm.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mcpm_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    import ctypes
    from mcpm import engine as E
    lib = E.load_library()
    names = declared_symbols()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) == set(E.SIGNATURES), set(names) ^ set(E.SIGNATURES)
    assert isinstance(ctypes.CDLL(E.lib_path()), ctypes.CDLL)


def test_status_strings():
    from mcpm import engine as E
    lib = E.load_library()
    for s in range(11):
        assert lib.mcpm_status_string(s)


def test_engine_create_rejects_bad_config():
    from mcpm import engine as E
    lib = E.load_library()
    import ctypes as C
    h = C.c_void_p()
    cfg = E.mcpm_config(0, 1 << 20, 0)      # max_seq beyond the supported 16384
    assert lib.mcpm_engine_create(C.byref(cfg), C.byref(h)) == E.BAD_ARG
    assert lib.mcpm_engine_create(None, C.byref(h)) == E.BAD_ARG


def test_ops_reject_bad_arguments_without_touching_memory():
    from mcpm import engine as E
    lib = E.load_library()
    assert lib.mcpm_quantize_q8k(None, None, 256, 0, None) == E.BAD_ARG
    assert lib.mcpm_gemv_q8k(12, 16, 16, 16, 4, 100, None) == E.BAD_ARG        # cols not a multiple of 256
    assert lib.mcpm_gemv_q8k(8, 16, 16, 16, 4, 2048, None) == E.UNSUPPORTED_TYPE
    assert lib.mcpm_rmsnorm_q8k(16, 16, 16, 1024, 1e-6, None) == E.BAD_ARG


def facade_build(out_dir, name="facade_driver"):
    """Compiles tests/cpp/<name>.cpp against include/minicpm5_engine.hpp and links it with the
    in-tree libmcpm.so; returns the binary path."""
    import subprocess
    from mcpm import engine as E
    lib = E.lib_path()
    exe = os.path.join(str(out_dir), name)
    cmd = ["g++", "-std=c++17", "-O1", "-I", os.path.join(REPO, "include"), os.path.join(REPO, "tests", "cpp", name + ".cpp"),
           "-o", exe, lib, "-L/usr/local/cuda/lib64", "-lcudart", "-Wl,-rpath," + os.path.dirname(lib) + ":/usr/local/cuda/lib64"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_cpp_facade_compiles_and_links(tmp_path):
    """The reference-shaped C++ facades (MiniCPM5Engine, Sampler) build against the C ABI."""
    assert os.path.exists(facade_build(tmp_path))
    assert os.path.exists(facade_build(tmp_path, "sampler_driver"))
