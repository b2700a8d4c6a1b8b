"""The C-ABI library loads and exports every function include/*.h declares (CPU only)."""

import glob
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for header in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(header).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        for m in re.finditer(r"\b(tmc_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_every_declared_symbol_is_exported():
    import tmc_cuda
    names = declared_functions()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(tmc_cuda.lib, n)]
    assert not missing, missing


def test_library_reports_errors_without_a_gpu_call():
    import tmc_cuda
    assert tmc_cuda.lib.tmc_cuda_abi_version() >= 1
    # A null-pointer kernel call is rejected on the host before any launch.
    code = tmc_cuda.lib.tmc_k_rmsnorm_gemv_f32(None, None, None, None, 1, 8, 8, 1e-5, None)
    assert code == tmc_cuda.ERR_INVALID
    assert "null" in tmc_cuda.last_error()


def test_rmsnorm_and_tuners_validate_arguments_on_the_host():
    import ctypes
    import tmc_cuda
    assert tmc_cuda.lib.tmc_k_rmsnorm(None, None, None, 1, 8, 1e-5, 0, 256, None) == tmc_cuda.ERR_INVALID
    sel = tmc_cuda.GemvSelection()
    assert tmc_cuda.lib.tmc_tune_decode_gemv(1, 8, 8, None, None, 1, 0, ctypes.byref(sel), None, 0) == \
        tmc_cuda.ERR_INVALID
    rsel = tmc_cuda.RMSNormSelection()
    assert tmc_cuda.lib.tmc_tune_rmsnorm(1, 8, 1e-5, 0, None, None, None, 0, ctypes.byref(rsel), None, None,
                                         0) == tmc_cuda.ERR_INVALID
