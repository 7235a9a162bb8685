"""The C-ABI library loads and exports every entry point include/nnb.h declares (no GPU needed).

No compute call is made here: on a machine without a GPU only host-side paths run (version, math
mode, argument checks that reject a call before any device work).
"""
import ctypes
import subprocess

import nnb


def test_library_exports_every_declared_symbol():
    names = nnb.header_symbols()
    assert len(names) >= 8
    lib = ctypes.CDLL(str(nnb.LIB_PATH))
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", str(nnb.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert set(names) <= exported


def test_every_declared_symbol_has_a_binding():
    assert set(nnb.header_symbols()) <= set(nnb._SIGS)


def test_version_and_math_mode():
    assert nnb.lib().nnb_version().decode().count(".") == 2
    old = nnb.get_math_mode()
    nnb.set_math_mode(nnb.MATH_TF32)
    assert nnb.get_math_mode() == nnb.MATH_TF32
    nnb.set_math_mode(old)
    try:
        nnb.set_math_mode(7)
    except ValueError as e:
        assert "math mode" in str(e)
    else:
        raise AssertionError("invalid math mode accepted")


def test_built_for_sm100a_only():
    """The build compiles every kernel for sm_100a and nothing else."""
    from nnb import _build
    flags = " ".join(_build.NVCC_FLAGS)
    assert "arch=compute_100a,code=sm_100a" in flags
    assert flags.count("-gencode") == 1
