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


def test_flash_attention_host_checks():
    """Head sizes other than 64 and bad shapes are rejected on the host, before any device work."""
    lib = nnb.lib()
    assert lib.nnb_flash_attention_supported(512, 8) == 1
    assert lib.nnb_flash_attention_supported(48, 1) == 0
    assert lib.nnb_flash_attention_supported(30, 4) == 0
    st = lib.nnb_flash_attention_fwd(None, 2, 8, 8, 96, 2, None, None, None, None, 0, None, None)
    assert st == 3 and "head size 48" in lib.nnb_last_error().decode()         # NNB_ERR_UNSUPPORTED
    st = lib.nnb_flash_attention_fwd(None, 2, 8, 9, 128, 2, None, None, None, None, 1, None, None)
    assert st == 5                                                              # causal needs Tq == Tk
    st = lib.nnb_flash_attention_bwd(None, 1, 4, 4, 64, 3, *([None] * 7), 0, None, 1, None, 1, None, 1)
    assert st == 5                                                              # heads does not divide D


def test_sgemm_host_release_without_calls():
    """Releasing the host-buffer GEMM's device buffers before any call is a no-op (no CUDA work)."""
    nnb.sgemm_host_release()


def test_linear_pack_bytes():
    """The kept input pack's size (host arithmetic only): panels of round_up(M, 256) rows x
    round_up(K, 32) depths, hi and lo in 3xTF32 (hi only in TF32), rounded to 1 KB, then one flag per
    padded row and the any-flag; 0 for an unknown math mode."""
    lib = nnb.lib()
    panels = 512 * 96 * 2 * 4                       # M = 300 -> 512 rows, K = 70 -> 96 depths
    assert lib.nnb_linear_pack_bytes(300, 70, nnb.MATH_FP32X3) == panels + (512 + 1) * 4
    assert lib.nnb_linear_pack_bytes(300, 70, nnb.MATH_TF32) == panels // 2 + (512 + 1) * 4
    assert lib.nnb_linear_pack_bytes(32768, 512, nnb.MATH_FP32X3) == 32768 * 512 * 8 + (32768 + 1) * 4
    assert lib.nnb_linear_pack_bytes(16, 16, 7) == 0


def test_linear_ex_host_checks():
    """nnb_linear_fwd_ex / nnb_linear_bwd_ex reject bad arguments before any device work."""
    lib = nnb.lib()
    p = ctypes.c_void_p(16)                          # never dereferenced: the checks come first
    assert lib.nnb_linear_fwd_ex(None, 1, 4, 0, 4, p, p, 0, p, 0, p, 0, None, None) == 5     # K == 0: shape
    assert lib.nnb_linear_fwd_ex(None, 2, 4, 4, 4, p, p, 0, p, 0, p, 0, p, None) == 1       # GELU form, 2 weights
    assert lib.nnb_linear_fwd_ex(None, 2, 4, 4, 4, p, p, 15, p, 4, p, 16, None, None) == 1  # weights overlap
    assert lib.nnb_linear_fwd_ex(None, 1, 4, 4, 4, None, p, 0, p, 0, p, 0, None, None) == 1  # null input
    assert lib.nnb_linear_bwd_ex(None, 6, 4, 4, 4, p, p, None, 0, p, *([None, 0] * 2), 0, None, 0, 0) == 5
