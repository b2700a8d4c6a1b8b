"""The C-ABI library loads and exports every function include/*.h declares, and
refuses bad arguments on the host before any launch (CPU only)."""

import glob
import os
import re

import pytest

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


# Host-side rejections of the graph-path operators: non-null placeholder
# pointers (never dereferenced), so the size and value checks are what refuse.
P = 0x1000
REJECTIONS = [
    ("rmsnorm rows", lambda l: l.tmc_k_rmsnorm(P, P, P, 0, 8, 1e-5, 0, 256, None), "INVALID", "rows >= 1"),
    ("rmsnorm eps", lambda l: l.tmc_k_rmsnorm(P, P, P, 1, 8, 0.0, 0, 256, None), "INVALID", "eps"),
    ("rmsnorm threads", lambda l: l.tmc_k_rmsnorm(P, P, P, 1, 8, 1e-5, 0, 48, None), "UNSUPPORTED", "power of two"),
    ("add-norm b_rows", lambda l: l.tmc_k_fused_add_norm(P, P, P, P, P, 3, 8, 2, 1e-5, 0, 0, None), "INVALID",
     "b_rows"),
    ("layer-norm bias", lambda l: l.tmc_k_fused_add_norm(P, P, P, None, P, 1, 8, 1, 1e-5, 1, 0, None), "INVALID",
     "null"),
    ("add-norm eps", lambda l: l.tmc_k_fused_add_norm(P, P, P, P, P, 1, 8, 1, -1.0, 0, 1, None), "INVALID", "eps"),
    ("silu-mul width", lambda l: l.tmc_k_fused_silu_mul(P, P, P, 1, 0, 1, 0, None), "INVALID", "width"),
    ("linear-relu n", lambda l: l.tmc_k_fused_linear_relu(P, P, P, P, 2, 3, 0, 0, None), "INVALID", "m, k, n"),
]


@pytest.mark.parametrize("name,call,code,fragment", REJECTIONS, ids=[r[0] for r in REJECTIONS])
def test_graph_operators_reject_bad_arguments_on_the_host(name, call, code, fragment):
    import tmc_cuda
    assert call(tmc_cuda.lib) == getattr(tmc_cuda, "ERR_" + code)
    assert fragment in tmc_cuda.last_error()


def test_noalloc_attention_refuses_requests_beyond_its_fixed_scratch():
    # The limit is checked on the host before the scratch array is looked up or
    # anything is launched: partials rows*hq*splits*(d+2)*4 (rounded up to 256)
    # plus rows*hkv*4 bytes of tickets must fit in 8 MiB.
    from ctypes import c_int, c_void_p
    import tmc_cuda
    fn = tmc_cuda.lib.tmc_k_paged_attention_f16_noalloc
    fn.restype = c_int
    fn.argtypes = [c_void_p] * 5 + [c_int] + [c_void_p] * 2 + [c_int] * 9 + [c_void_p] * 2
    limit = 8 << 20
    rows, hq, hkv, d, splits = 64, 32, 8, 128, 8
    need = (tmc_cuda.attention_workspace_bytes(rows, hq, hkv, d, splits) + 255) // 256 * 256 + rows * hkv * 4
    assert need == (rows * hq * splits * (d + 2) * 4 + 255) // 256 * 256 + rows * hkv * 4 > limit
    code = fn(P, P, P, P, P, 1, P, P, rows, hq, hkv, d, 16, 64, 1024, splits, 64, None, None)
    assert code == tmc_cuda.ERR_UNSUPPORTED
    assert f"needs {need} bytes" in tmc_cuda.last_error() and str(limit) in tmc_cuda.last_error()
    assert fn(P, P, P, P, P, 1, P, P, 0, hq, hkv, d, 16, 64, 1024, 1, 64, None, None) == tmc_cuda.ERR_INVALID


def test_builtin_kernel_catalog_is_listed_on_the_host():
    # tmc_kernel_count / tmc_kernel_at / tmc_kernel_lookup / tmc_kernel_describe
    # need no GPU: the catalog is this library's own table.
    import tmc_cuda
    cat = tmc_cuda.kernels()
    for name, counts in {"rmsnorm": (2, 1, 3), "rmsnorm_gemv_f32": (3, 1, 4), "gemv_f16": (2, 1, 3),
                         "batched_gemm_f16": (2, 1, 3), "fused_add_rmsnorm": (3, 1, 4),
                         "fused_add_layernorm": (4, 1, 4), "fused_silu_mul": (2, 1, 3),
                         "fused_linear_relu": (3, 1, 3), "paged_attention_f16": (6, 1, 10)}.items():
        assert cat[name][:3] == counts, name
        assert cat[name][3]
    import ctypes
    h = ctypes.c_void_p()
    assert tmc_cuda.lib.tmc_kernel_lookup(b"missing", ctypes.byref(h)) == tmc_cuda.ERR_UNSUPPORTED
    assert "no built-in kernel" in tmc_cuda.last_error()
    assert tmc_cuda.float_bits(1.0) == 0x3F800000
