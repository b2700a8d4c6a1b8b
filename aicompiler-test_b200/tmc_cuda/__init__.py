"""ctypes binding of the B200 decode backend's C ABI (include/tmc_cuda.h).

This module is the Python host mirror used by the tests and the benchmark. It
loads the in-tree ``lib/libtmc_cuda.so`` and fails loudly when it is missing:
there is no CPU or PyTorch fallback behind any call here.

Naming follows the reference's C++ surface (tensor::metal::MetalRuntime,
reference src/backend/metal/MetalRuntime.hpp:149-208): ``Runtime`` is one
device + stream, ``Buffer`` is a typed device allocation created from logical
host floats.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import (POINTER, c_char_p, c_float, c_int, c_int32, c_size_t, c_uint32, c_uint64,
                    c_void_p)

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "lib", "libtmc_cuda.so")

F16, F32, BF16, I32 = 0, 1, 2, 3
OK = 0
ERR_INVALID, ERR_CUDA, ERR_OOM, ERR_DEVICE_STATUS, ERR_UNSUPPORTED, ERR_UNAVAILABLE = 1, 2, 3, 4, 5, 6

_NP_BY_DTYPE = {F16: np.float16, F32: np.float32, I32: np.int32}


class TmcError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[tmc status {code}] {message}")
        self.code = code
        self.message = message


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"libtmc_cuda.so not built at {LIB_PATH}; run `make -C aicompiler-test_b200` "
            "(the CUDA extension is required, there is no fallback)")
    return ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)


lib = _load()


def _sig(name, restype, *argtypes):
    fn = getattr(lib, name)
    fn.restype = restype
    fn.argtypes = list(argtypes)
    return fn


class DeviceInfo(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char * 256),
        ("compute_major", c_int),
        ("compute_minor", c_int),
        ("multiprocessor_count", c_int),
        ("max_threads_per_block", c_size_t),
        ("max_shared_per_block", c_size_t),
        ("total_global_mem", c_size_t),
        ("l2_cache_bytes", c_size_t),
        ("supports_bf16", c_int),
    ]


_sig("tmc_cuda_last_error", c_char_p)
_sig("tmc_cuda_abi_version", c_int)
_sig("tmc_cuda_device_count", c_int, POINTER(c_int))
_sig("tmc_cuda_device_info", c_int, c_int, POINTER(DeviceInfo))
_sig("tmc_runtime_create", c_int, c_int, POINTER(c_void_p))
_sig("tmc_runtime_destroy", None, c_void_p)
_sig("tmc_runtime_stream", c_void_p, c_void_p)
_sig("tmc_runtime_synchronize", c_int, c_void_p)
_sig("tmc_runtime_status_ptr", c_void_p, c_void_p)
_sig("tmc_buffer_create", c_int, c_void_p, c_size_t, c_int, POINTER(c_float), POINTER(c_void_p))
_sig("tmc_buffer_destroy", None, c_void_p)
_sig("tmc_buffer_write", c_int, c_void_p, POINTER(c_float), c_size_t, c_size_t)
_sig("tmc_buffer_read", c_int, c_void_p, POINTER(c_float), c_size_t)
_sig("tmc_buffer_write_bytes", c_int, c_void_p, c_void_p, c_size_t, c_size_t)
_sig("tmc_buffer_read_bytes", c_int, c_void_p, c_void_p, c_size_t, c_size_t)
_sig("tmc_buffer_device_ptr", c_void_p, c_void_p)
_sig("tmc_buffer_count", c_size_t, c_void_p)
_sig("tmc_buffer_dtype", c_int, c_void_p)
_sig("tmc_k_rmsnorm_gemv_f32", c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
     c_float, c_void_p)
_sig("tmc_k_gemv_f16", c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p)
_sig("tmc_k_gemv_f16_f32out", c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p)
_sig("tmc_k_attention_workspace_bytes", c_size_t, c_int, c_int, c_int, c_int, c_int)
_sig("tmc_k_paged_attention_f16", c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
     c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p,
     c_void_p, c_void_p, c_void_p)
_sig("tmc_k_fill_normal_f16", c_int, c_void_p, c_size_t, c_uint64, c_float, c_float, c_void_p)


def last_error() -> str:
    return lib.tmc_cuda_last_error().decode()


def check(code: int):
    if code != OK:
        raise TmcError(code, last_error())


def device_count() -> int:
    n = c_int(0)
    code = lib.tmc_cuda_device_count(ctypes.byref(n))
    return n.value if code == OK else 0


def device_info(device: int = 0) -> DeviceInfo:
    info = DeviceInfo()
    check(lib.tmc_cuda_device_info(device, ctypes.byref(info)))
    return info


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(POINTER(c_float))


class Runtime:
    """One device and its stream (reference MetalRuntime)."""

    def __init__(self, device: int = 0):
        h = c_void_p()
        check(lib.tmc_runtime_create(device, ctypes.byref(h)))
        self.handle = h
        self.device = device

    def close(self):
        if self.handle:
            lib.tmc_runtime_destroy(self.handle)
            self.handle = c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self):
        return lib.tmc_runtime_stream(self.handle)

    @property
    def status_ptr(self):
        return lib.tmc_runtime_status_ptr(self.handle)

    def synchronize(self):
        check(lib.tmc_runtime_synchronize(self.handle))

    def buffer(self, count: int, dtype: int = F32, init=None) -> "Buffer":
        return Buffer(self, count, dtype, init)

    def upload(self, array: np.ndarray, dtype: int | None = None) -> "Buffer":
        """Raw upload of an fp16/fp32/int32 numpy array (bit pattern preserved)."""
        array = np.ascontiguousarray(array)
        if dtype is None:
            dtype = {np.dtype(np.float16): F16, np.dtype(np.float32): F32,
                     np.dtype(np.int32): I32}[array.dtype]
        buf = Buffer(self, array.size, dtype, None)
        check(lib.tmc_buffer_write_bytes(buf.handle, array.ctypes.data_as(c_void_p), array.nbytes, 0))
        return buf


class Buffer:
    """Typed device buffer (reference MetalBuffer / BufferHandle)."""

    def __init__(self, runtime: Runtime, count: int, dtype: int, init=None):
        self.runtime = runtime
        self.count = int(count)
        self.dtype = dtype
        h = c_void_p()
        if init is not None:
            init = np.ascontiguousarray(init, dtype=np.float32).reshape(-1)
            assert init.size == count
            check(lib.tmc_buffer_create(runtime.handle, count, dtype, _fptr(init), ctypes.byref(h)))
        else:
            check(lib.tmc_buffer_create(runtime.handle, count, dtype, None, ctypes.byref(h)))
        self.handle = h

    def __del__(self):
        try:
            if self.handle:
                lib.tmc_buffer_destroy(self.handle)
                self.handle = c_void_p()
        except Exception:
            pass

    @property
    def ptr(self) -> int:
        return lib.tmc_buffer_device_ptr(self.handle)

    def read(self) -> np.ndarray:
        """Logical float values."""
        out = np.empty(self.count, dtype=np.float32)
        check(lib.tmc_buffer_read(self.handle, _fptr(out), self.count))
        return out

    def read_raw(self) -> np.ndarray:
        out = np.empty(self.count, dtype=_NP_BY_DTYPE[self.dtype])
        check(lib.tmc_buffer_read_bytes(self.handle, out.ctypes.data_as(c_void_p), out.nbytes, 0))
        return out

    def write(self, values, offset: int = 0):
        values = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
        check(lib.tmc_buffer_write(self.handle, _fptr(values), values.size, offset))

    def write_raw(self, array: np.ndarray, byte_offset: int = 0):
        array = np.ascontiguousarray(array)
        check(lib.tmc_buffer_write_bytes(self.handle, array.ctypes.data_as(c_void_p), array.nbytes,
                                         byte_offset))


# ---- kernel wrappers (device pointers) ------------------------------------------------

def rmsnorm_gemv_f32(rt: Runtime, x: Buffer, gamma: Buffer, w: Buffer, y: Buffer, rows: int, k: int,
                     n: int, eps: float):
    check(lib.tmc_k_rmsnorm_gemv_f32(x.ptr, gamma.ptr, w.ptr, y.ptr, rows, k, n, eps, rt.stream))


def gemv_f16(rt: Runtime, x: Buffer, w: Buffer, y: Buffer, rows: int, k: int, n: int):
    if y.dtype == F16:
        check(lib.tmc_k_gemv_f16(x.ptr, w.ptr, y.ptr, rows, k, n, rt.stream))
    else:
        check(lib.tmc_k_gemv_f16_f32out(x.ptr, w.ptr, y.ptr, rows, k, n, rt.stream))


def attention_workspace_bytes(rows, hq, hkv, d, max_splits) -> int:
    return int(lib.tmc_k_attention_workspace_bytes(rows, hq, hkv, d, max_splits))


def paged_attention_f16(rt: Runtime, q: Buffer, out: Buffer, k_pool: Buffer, v_pool: Buffer,
                        block_table: Buffer, table_stride: int, table_rows: Buffer,
                        positions: Buffer, rows: int, hq: int, hkv: int, d: int, page_size: int,
                        pool_pages: int, capacity: int, max_splits: int, min_chunk: int,
                        workspace: Buffer | None, counters: Buffer):
    check(lib.tmc_k_paged_attention_f16(
        q.ptr, out.ptr, k_pool.ptr, v_pool.ptr, block_table.ptr, table_stride, table_rows.ptr,
        positions.ptr, rows, hq, hkv, d, page_size, pool_pages, capacity, max_splits, min_chunk,
        workspace.ptr if workspace is not None else None, counters.ptr, rt.status_ptr, rt.stream))


def fill_normal_f16(rt: Runtime, buf: Buffer, seed: int, mean: float, std: float):
    check(lib.tmc_k_fill_normal_f16(buf.ptr, buf.count, seed, mean, std, rt.stream))
