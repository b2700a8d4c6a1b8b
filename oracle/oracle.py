"""CPU oracle bindings -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this
module, as the checker; the product path (aicompiler-test_b200/) never does.

- ``liboracle.so`` (oracle/graph_ref.c): a plain-C restatement of the
  reference's fp64 GraphReference / Validator path and of its serving paged
  attention (citations in graph_ref.c).
- ``_ref/libtmcref.so`` (oracle/ref_driver.cpp): the reference's OWN
  ``evaluateGraph`` compiled from its sources (oracle/Makefile); present when
  the reference was available at build time. Used to pin the restatement.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_double, c_float, c_int, c_int32, c_long, c_uint16

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libtmcref.so")


def _load(path):
    if not os.path.exists(path):
        return None
    return ctypes.CDLL(path)


_lib = _load(ORACLE_LIB)
_ref = _load(REF_LIB)

_F = POINTER(c_float)
_D = POINTER(c_double)
_I = POINTER(c_int32)

if _lib is not None:
    _lib.oracle_store.restype = c_float
    _lib.oracle_store.argtypes = [c_double, c_int]
    _lib.oracle_round_f16.argtypes = [_F, _F, c_long]
    _lib.oracle_f32_to_f16_bits.argtypes = [_F, POINTER(c_uint16), c_long]
    _lib.oracle_f16_bits_to_f32.argtypes = [POINTER(c_uint16), _F, c_long]
    _lib.oracle_rmsnorm.argtypes = [_F, _F, c_long, c_long, c_double, _D]
    _lib.oracle_rmsnorm_matmul.argtypes = [_F, _F, _F, c_long, c_long, c_long, c_double, _D]
    _lib.oracle_gemv.argtypes = [_F, _F, c_long, c_long, c_long, _D]
    _lib.oracle_compare.restype = c_long
    _lib.oracle_compare.argtypes = [_F, _D, c_long, c_double, c_double, _D, POINTER(c_long)]
    _lib.oracle_paged_attention.restype = c_int
    _lib.oracle_paged_attention.argtypes = [_F, _F, _F, _I, c_long, _I, _I, c_long, c_long, c_long,
                                            c_long, c_long, _D]

    _lib.oracle_fusion.restype = c_int
    _lib.oracle_fusion.argtypes = [c_int, _F, _F, _F, _F, c_long, c_long, c_long, c_long, c_double, c_int, _D]

if _ref is not None:
    _ref.ref_last_error.restype = c_char_p
    _ref.ref_rmsnorm_matmul.restype = c_int
    _ref.ref_rmsnorm_matmul.argtypes = [_F, _F, _F, c_long, c_long, c_long, c_float, _D]
    _ref.ref_fusion.restype = c_int
    _ref.ref_fusion.argtypes = [c_int, _F, _F, _F, _F, c_long, c_long, c_long, c_long, c_float, c_int, _D]
    _ref.ref_rmsnorm.restype = c_int
    _ref.ref_rmsnorm.argtypes = [_F, _F, c_long, c_long, c_float, c_int, _D]
    if hasattr(_ref, "ref_form_regions"):
        _I32P = POINTER(c_int)
        _ref.ref_form_regions.restype = c_long
        _ref.ref_form_regions.argtypes = [c_long, c_long, c_long, _I32P, c_long, _I32P, c_long, _I32P, _I32P,
                                          _I32P, c_long]
    if hasattr(_ref, "ref_plan_buffers"):
        _I32P = POINTER(c_int)
        _ref.ref_plan_buffers.restype = c_long
        _ref.ref_plan_buffers.argtypes = [c_long, c_long, c_long, _I32P, c_long, _I32P, c_long, _I32P, _I32P,
                                          _I32P]


def available() -> bool:
    return _lib is not None


def reference_available() -> bool:
    return _ref is not None


def _need():
    if _lib is None:
        raise RuntimeError(f"oracle not built: {ORACLE_LIB} (run `make -C oracle`)")


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a, t):
    return a.ctypes.data_as(t)


def round_f16(values) -> np.ndarray:
    """fp32 -> fp16 (RNE) -> fp32, the reference's storeValue for fp16."""
    _need()
    v = _f32(values)
    out = np.empty_like(v)
    _lib.oracle_round_f16(_p(v, _F), _p(out, _F), v.size)
    return out


def f32_to_f16_bits(values) -> np.ndarray:
    _need()
    v = _f32(values)
    out = np.empty(v.shape, dtype=np.uint16)
    _lib.oracle_f32_to_f16_bits(_p(v, _F), out.ctypes.data_as(POINTER(c_uint16)), v.size)
    return out


def rmsnorm(x, w, eps=1e-5) -> np.ndarray:
    _need()
    x = _f32(x)
    w = _f32(w)
    rows, width = x.shape
    out = np.empty((rows, width), dtype=np.float64)
    _lib.oracle_rmsnorm(_p(x, _F), _p(w, _F), rows, width, eps, _p(out, _D))
    return out


def rmsnorm_matmul(x, gamma, w, eps=1e-5) -> np.ndarray:
    """C1: y = W . rmsnorm(x) with the reference's fp32-stored RMSNorm (fp64 sums)."""
    _need()
    x = _f32(x)
    gamma = _f32(gamma)
    w = _f32(w)
    rows, k = x.shape
    n = w.shape[0]
    y = np.empty((rows, n), dtype=np.float64)
    _lib.oracle_rmsnorm_matmul(_p(x, _F), _p(gamma, _F), _p(w, _F), rows, k, n, eps, _p(y, _D))
    return y


def gemv(x, w) -> np.ndarray:
    _need()
    x = _f32(x)
    w = _f32(w)
    rows, k = x.shape
    n = w.shape[0]
    y = np.empty((rows, n), dtype=np.float64)
    _lib.oracle_gemv(_p(x, _F), _p(w, _F), rows, k, n, _p(y, _D))
    return y


def compare(actual, reference, atol, rtol):
    """Validator::compare: (passed, max_abs_error, mismatches, first_mismatch)."""
    _need()
    a = _f32(actual).reshape(-1)
    r = np.ascontiguousarray(reference, dtype=np.float64).reshape(-1)
    worst = c_double(0.0)
    first = c_long(-1)
    bad = _lib.oracle_compare(_p(a, _F), _p(r, _D), a.size, atol, rtol, ctypes.byref(worst),
                              ctypes.byref(first))
    return bad == 0, worst.value, int(bad), int(first.value)


def paged_attention(q, k_pool, v_pool, table, table_rows, positions, hkv, page_size) -> np.ndarray:
    """Serving paged decode attention with the GQA head map (fp64 context)."""
    _need()
    q = _f32(q)
    rows, hq, d = q.shape
    k_pool = _f32(k_pool)
    v_pool = _f32(v_pool)
    table = np.ascontiguousarray(table, dtype=np.int32)
    table_rows = np.ascontiguousarray(table_rows, dtype=np.int32)
    positions = np.ascontiguousarray(positions, dtype=np.int32)
    out = np.empty((rows, hq, d), dtype=np.float64)
    rc = _lib.oracle_paged_attention(_p(q, _F), _p(k_pool, _F), _p(v_pool, _F), _p(table, _I),
                                     table.shape[1], _p(table_rows, _I), _p(positions, _I), rows,
                                     hq, hkv, d, page_size, _p(out, _D))
    if rc != 0:
        raise ValueError("oracle paged attention: missing page")
    return out


# ---- the reference's own evaluateGraph (oracle/_ref) --------------------------------

def ref_rmsnorm_matmul(x, gamma, w, eps=1e-5) -> np.ndarray:
    if _ref is None:
        raise RuntimeError("oracle/_ref not built (reference sources absent at build time)")
    x = _f32(x)
    gamma = _f32(gamma)
    w = _f32(w)
    rows, k = x.shape
    n = w.shape[0]
    y = np.empty((rows, n), dtype=np.float64)
    if _ref.ref_rmsnorm_matmul(_p(x, _F), _p(gamma, _F), _p(w, _F), rows, k, n, eps, _p(y, _D)) != 0:
        raise RuntimeError(_ref.ref_last_error().decode())
    return y


def ref_rmsnorm(x, gamma, eps=1e-5, dtype=1) -> np.ndarray:
    if _ref is None:
        raise RuntimeError("oracle/_ref not built (reference sources absent at build time)")
    x = _f32(x)
    gamma = _f32(gamma)
    rows, width = x.shape
    y = np.empty((rows, width), dtype=np.float64)
    if _ref.ref_rmsnorm(_p(x, _F), _p(gamma, _F), rows, width, eps, dtype, _p(y, _D)) != 0:
        raise RuntimeError(_ref.ref_last_error().decode())
    return y


FUSION_KINDS = {"add_rmsnorm": 0, "add_layernorm": 1, "silu_mul": 2, "linear_relu": 3}


def _fusion_args(kind, x, b, w, c, n):
    x = _f32(x)
    rows, width = x.shape
    b = _f32(b)
    b_rows = 1 if (kind != "linear_relu" and b.ndim == 1) else (b.shape[0] if kind != "linear_relu" else width)
    w = _f32(w if w is not None else np.zeros(1, np.float32))
    c = _f32(c if c is not None else np.zeros(1, np.float32))
    out_cols = n if kind == "linear_relu" else width
    return x, b, w, c, rows, width, b_rows, out_cols


def fusion(kind, x, b, w=None, c=None, eps=1e-5, fp16=False, n=0) -> np.ndarray:
    """The graph suite's fused regions in fp64 (graph_ref.c oracle_fusion);
    inputs must already hold storage values (round_f16 for fp16 graphs)."""
    _need()
    x, b, w, c, rows, width, b_rows, out_cols = _fusion_args(kind, x, b, w, c, n)
    out = np.empty((rows, out_cols), dtype=np.float64)
    code = _lib.oracle_fusion(FUSION_KINDS[kind], _p(x, _F), _p(b, _F), _p(w, _F), _p(c, _F), rows, width,
                              b_rows, n, eps, 0 if fp16 else 1, _p(out, _D))
    if code != 0:
        raise ValueError(kind)
    return out


def ref_fusion(kind, x, b, w=None, c=None, eps=1e-5, fp16=False, n=0) -> np.ndarray:
    """The same graph through the reference's own evaluateGraph (oracle/_ref)."""
    if _ref is None:
        raise RuntimeError("oracle/_ref not built")
    x, b, w, c, rows, width, b_rows, out_cols = _fusion_args(kind, x, b, w, c, n)
    out = np.empty((rows, out_cols), dtype=np.float64)
    if _ref.ref_fusion(FUSION_KINDS[kind], _p(x, _F), _p(b, _F), _p(w, _F), _p(c, _F), rows, width, b_rows, n,
                       eps, 0 if fp16 else 1, _p(out, _D)) != 0:
        raise RuntimeError(_ref.ref_last_error().decode())
    return out


def encode_graph(nodes):
    """Flat node encoding shared with oracle/_ref and the planner tests:
    per node (op number, operands...) -> {op, operand count, operands...}."""
    flat = []
    for op, *operands in nodes:
        flat += [int(op), len(operands)] + [int(v) for v in operands]
    return np.asarray(flat, dtype=np.int32)


def decode_regions(flat):
    """{fusion, #nodes, nodes..., #inputs, inputs..., #outputs, outputs...} ->
    [(fusion, nodes, inputs, outputs)]."""
    out, i = [], 0
    while i < len(flat):
        kind = int(flat[i])
        i += 1
        parts = []
        for _ in range(3):
            k = int(flat[i])
            parts.append([int(x) for x in flat[i + 1:i + 1 + k]])
            i += 1 + k
        out.append((kind, *parts))
    return out


def ref_form_regions(n, squares, vectors, nodes, outputs):
    """The reference's own analyze + formRegions (oracle/_ref) on a graph of fp32
    [n, n] inputs (`squares`), [n] inputs (`vectors`) and `nodes` as
    (op number, operands...), node i defining value squares + vectors + i.
    Returns (order, contiguity per value, regions), or raises ValueError with
    the reference's message when it rejects the graph."""
    if _ref is None or not hasattr(_ref, "ref_form_regions"):
        raise RuntimeError("oracle/_ref not built with region formation")
    flat = encode_graph(nodes)
    outs = np.asarray(outputs, dtype=np.int32)
    order = np.zeros(len(nodes), np.int32)
    values = squares + vectors + len(nodes)
    contiguous = np.zeros(values, np.int32)
    cap = 64 * (len(nodes) + 1) + 16
    regions = np.zeros(cap, np.int32)
    P = POINTER(c_int)
    w = _ref.ref_form_regions(n, squares, vectors, flat.ctypes.data_as(P), len(nodes), outs.ctypes.data_as(P),
                              len(outs), order.ctypes.data_as(P), contiguous.ctypes.data_as(P),
                              regions.ctypes.data_as(P), cap)
    if w < 0:
        raise ValueError(_ref.ref_last_error().decode())
    return order.tolist(), contiguous.tolist(), decode_regions(regions[:w])


def ref_plan_buffers(n, squares, vectors, nodes, outputs):
    """The reference's own planGraph (oracle/_ref) on the ref_form_regions graph
    encoding: (roles per value: 0 input, 1 intermediate, 2 output; alias per
    value, -1 for none; launched node indices in plan order)."""
    if _ref is None or not hasattr(_ref, "ref_plan_buffers"):
        raise RuntimeError("oracle/_ref not built with graph planning")
    flat = encode_graph(nodes)
    outs = np.asarray(outputs, dtype=np.int32)
    values = squares + vectors + len(nodes)
    roles = np.zeros(values, np.int32)
    alias = np.zeros(values, np.int32)
    launches = np.zeros(max(len(nodes), 1), np.int32)
    P = POINTER(c_int)
    k = _ref.ref_plan_buffers(n, squares, vectors, flat.ctypes.data_as(P), len(nodes), outs.ctypes.data_as(P),
                              len(outs), roles.ctypes.data_as(P), alias.ctypes.data_as(P), launches.ctypes.data_as(P))
    if k < 0:
        raise ValueError(_ref.ref_last_error().decode())
    return roles.tolist(), alias.tolist(), launches[:k].tolist()


def ref_evaluate_graph(inputs, nodes, outputs, values):
    """The reference's own evaluateGraph (oracle/_ref) on a typed graph in the
    tmc_graph encoding: inputs [(dtype 0 fp16 / 1 fp32, shape)], nodes [(op
    name or number, operands, attributes)], values = one array per input.
    Returns the declared outputs (fp64, flat)."""
    if _ref is None:
        raise RuntimeError("oracle/_ref not built (reference sources absent at build time)")
    import sys as _sys
    _sys.path.insert(0, __import__("os").path.join(__import__("os").path.dirname(__file__), "..",
                                                   "aicompiler-test_b200"))
    from tmc_cuda import encode_typed_graph
    types, flat = encode_typed_graph(inputs, nodes)
    data = np.concatenate([np.asarray(v, np.float32).reshape(-1) for v in values]).astype(np.float32)
    outs = np.asarray(outputs, np.int32)
    cap = 1 << 24
    out = np.empty(cap, dtype=np.float64)
    P = POINTER(c_int32)
    fn = _ref.ref_evaluate_graph
    fn.restype = c_long
    fn.argtypes = [c_int, P, c_int, P, c_int, P, _F, _D, c_long]
    n = fn(len(inputs), types.ctypes.data_as(P), len(nodes), flat.ctypes.data_as(P), len(outputs),
           outs.ctypes.data_as(P), _p(data, _F), _p(out, _D), cap)
    if n < 0:
        raise RuntimeError(_ref.ref_last_error().decode())
    return out[:n].copy()
