"""The C-ABI library loads and exports exactly the entry points include/lowbit_b200.h declares
(no compute calls: this runs without a GPU)."""
import ctypes as C
import re
import subprocess

from conftest import ROOT

from lowbit_b200 import _build


def declared():
    text = (ROOT / "include" / "lowbit_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lbc_[a-z0-9_]+)\s*\(", text)))


def test_library_builds_and_exports_every_declared_symbol():
    so = _build.build()
    names = declared()
    assert "lbc_gemm_w4a16" in names and len(names) >= 10
    lib = C.CDLL(str(so))
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/lowbit_b200.h but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", str(so)], capture_output=True, text=True).stdout
    exported = sorted(set(re.findall(r" T (lbc_[a-z0-9_]+)", out)))
    assert exported == names, f"exported {exported} != declared {names}"


def test_version_query_needs_no_gpu():
    lib = C.CDLL(str(_build.build()))
    assert lib.lbc_version() == 1


def test_kernels_are_built_for_sm100a_only():
    assert "arch=compute_100a,code=sm_100a" in " ".join(_build.ARCH)
    assert "--use_fast_math" not in _build.FLAGS


def test_python_binding_declares_every_entry_point():
    """lowbit_b200.kernels.lib() loads the library and sets a ctypes signature
    for every entry point the header declares (no calls)."""
    from lowbit_b200 import kernels as K
    lib = K.lib()
    for n in declared():
        if n == "lbc_gemm_w4a8_noalloc":   # bound by its own test module
            continue
        fn = getattr(lib, n)
        assert fn.argtypes is not None, f"{n} has no ctypes signature in lowbit_b200.kernels"
