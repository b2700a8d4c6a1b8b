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
_sig("tmc_k_fused_add_norm", c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_float,
     c_int, c_int, c_void_p)
_sig("tmc_k_fused_silu_mul", c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p)
_sig("tmc_k_fused_linear_relu", c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p)
_sig("tmc_k_rmsnorm", c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_int, c_int, c_void_p)
_sig("tmc_k_gemv_f16", c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p)
_sig("tmc_k_gemv_f16_f32out", c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p)
_sig("tmc_k_batched_gemm_workspace_bytes", c_size_t, c_int, c_int, c_int)
_sig("tmc_k_batched_gemm_f16_f32out", c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p,
     c_void_p, c_void_p)
_sig("tmc_k_attention_workspace_bytes", c_size_t, c_int, c_int, c_int, c_int, c_int)
_sig("tmc_k_paged_attention_f16", c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
     c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p,
     c_void_p, c_void_p, c_void_p)
_sig("tmc_k_paged_attention_f16_ex", c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
     c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p,
     c_void_p, c_int, c_int, c_void_p, c_void_p)
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

    def read_raw_range(self, byte_offset: int, count: int) -> np.ndarray:
        """`count` elements of the raw storage starting at `byte_offset`."""
        out = np.empty(count, dtype=_NP_BY_DTYPE[self.dtype])
        check(lib.tmc_buffer_read_bytes(self.handle, out.ctypes.data_as(c_void_p), out.nbytes, byte_offset))
        return out

    def write(self, values, offset: int = 0):
        values = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
        check(lib.tmc_buffer_write(self.handle, _fptr(values), values.size, offset))

    def write_raw(self, array: np.ndarray, byte_offset: int = 0):
        array = np.ascontiguousarray(array)
        check(lib.tmc_buffer_write_bytes(self.handle, array.ctypes.data_as(c_void_p), array.nbytes,
                                         byte_offset))


# ---- prepared executions and sequences (prepareBuffers / prepareSequence) --------------

_sig("tmc_kernel_count", c_int)
_sig("tmc_kernel_at", c_int, c_int, POINTER(c_void_p))
_sig("tmc_kernel_lookup", c_int, c_char_p, POINTER(c_void_p))
_sig("tmc_kernel_describe", c_int, c_void_p, POINTER(c_char_p), POINTER(c_int), POINTER(c_int), POINTER(c_int),
     POINTER(c_char_p))
_sig("tmc_prepare", c_int, c_void_p, c_void_p, POINTER(c_void_p), c_int, POINTER(c_void_p), c_int, c_size_t,
     c_size_t, POINTER(ctypes.c_uint32), c_int, POINTER(c_void_p))
_sig("tmc_prepared_destroy", None, c_void_p)
_sig("tmc_prepared_run", c_int, c_void_p, POINTER(c_float), c_size_t, POINTER(ctypes.c_double),
     POINTER(ctypes.c_double))
_sig("tmc_prepared_execute", c_int, c_void_p, POINTER(ctypes.c_double), POINTER(ctypes.c_double))
_sig("tmc_sequence_create", c_int, c_void_p, POINTER(c_void_p), c_int, POINTER(c_void_p))
_sig("tmc_sequence_destroy", None, c_void_p)
_sig("tmc_sequence_execute", c_int, c_void_p, POINTER(ctypes.c_double), POINTER(ctypes.c_double))
_sig("tmc_sequence_launch", c_int, c_void_p, c_int)


def float_bits(value: float) -> int:
    """The uint32 bit pattern of an fp32 value (floating constants of tmc_prepare)."""
    return int(np.array([value], np.float32).view(np.uint32)[0])


def kernels() -> dict:
    """Built-in kernels: name -> (inputs, outputs, constants, signature)."""
    out = {}
    for i in range(lib.tmc_kernel_count()):
        h = c_void_p()
        check(lib.tmc_kernel_at(i, ctypes.byref(h)))
        name, sig = c_char_p(), c_char_p()
        ni, no, nc = c_int(), c_int(), c_int()
        check(lib.tmc_kernel_describe(h, ctypes.byref(name), ctypes.byref(ni), ctypes.byref(no), ctypes.byref(nc),
                                      ctypes.byref(sig)))
        out[name.value.decode()] = (ni.value, no.value, nc.value, sig.value.decode())
    return out


class Prepared:
    """A built-in kernel bound to buffers and constants (reference
    MetalRuntime::prepareBuffers -> PreparedExecution)."""

    def __init__(self, rt: "Runtime", kernel: str, inputs, outputs, constants=(), groups=1, threads=256):
        k = c_void_p()
        check(lib.tmc_kernel_lookup(kernel.encode(), ctypes.byref(k)))
        ins = (c_void_p * max(1, len(inputs)))(*[b.handle for b in inputs])
        outs = (c_void_p * max(1, len(outputs)))(*[b.handle for b in outputs])
        consts = (ctypes.c_uint32 * max(1, len(constants)))(*[int(c) & 0xFFFFFFFF for c in constants])
        h = c_void_p()
        check(lib.tmc_prepare(rt.handle, k, ins, len(inputs), outs, len(outputs), groups, threads, consts,
                              len(constants), ctypes.byref(h)))
        self.handle = h
        self.first_output_count = outputs[0].count if outputs else 0

    def run(self):
        """NaN sentinels, execute, read the first output: (values, gpu_us, cpu_us)."""
        out = np.empty(self.first_output_count, np.float32)
        g, c = ctypes.c_double(), ctypes.c_double()
        check(lib.tmc_prepared_run(self.handle, _fptr(out), out.size, ctypes.byref(g), ctypes.byref(c)))
        return out, g.value, c.value

    def execute(self):
        g, c = ctypes.c_double(), ctypes.c_double()
        check(lib.tmc_prepared_execute(self.handle, ctypes.byref(g), ctypes.byref(c)))
        return g.value, c.value

    def close(self):
        if getattr(self, "handle", None):
            lib.tmc_prepared_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()


class Sequence:
    """Prepared executions in order, captured once as a CUDA graph (reference
    MetalRuntime::prepareSequence)."""

    def __init__(self, rt: "Runtime", steps):
        arr = (c_void_p * len(steps))(*[s.handle for s in steps])
        h = c_void_p()
        check(lib.tmc_sequence_create(rt.handle, arr, len(steps), ctypes.byref(h)))
        self.handle = h
        self.steps = list(steps)

    def execute(self):
        g, c = ctypes.c_double(), ctypes.c_double()
        check(lib.tmc_sequence_execute(self.handle, ctypes.byref(g), ctypes.byref(c)))
        return g.value, c.value

    def launch(self, replays: int = 1):
        """Enqueue `replays` replays on the runtime stream (no synchronisation)."""
        check(lib.tmc_sequence_launch(self.handle, replays))

    def close(self):
        if getattr(self, "handle", None):
            lib.tmc_sequence_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()


# ---- kernel wrappers (device pointers) ------------------------------------------------

def rmsnorm_gemv_f32(rt: Runtime, x: Buffer, gamma: Buffer, w: Buffer, y: Buffer, rows: int, k: int,
                     n: int, eps: float):
    check(lib.tmc_k_rmsnorm_gemv_f32(x.ptr, gamma.ptr, w.ptr, y.ptr, rows, k, n, eps, rt.stream))


def rmsnorm(rt: Runtime, x: Buffer, gamma: Buffer, y: Buffer, rows: int, width: int, eps: float,
            threads: int = 256):
    """RMSNormOp over [rows, width]; all three buffers fp32 or all fp16; threads 0 = baseline."""
    check(lib.tmc_k_rmsnorm(x.ptr, gamma.ptr, y.ptr, rows, width, eps, int(x.dtype == F16), threads, rt.stream))


def fused_add_norm(rt: Runtime, x: Buffer, b: Buffer, w: Buffer, y: Buffer, rows: int, width: int, b_rows: int,
                   eps: float = 1e-5, c: Buffer = None):
    """Add -> RMSNorm, or Add -> LayerNorm when the bias `c` is given (emitFusion)."""
    check(lib.tmc_k_fused_add_norm(x.ptr, b.ptr, w.ptr, c.ptr if c is not None else None, y.ptr, rows, width,
                                   b_rows, eps, int(c is not None), int(x.dtype == F16), rt.stream))


def fused_silu_mul(rt: Runtime, x: Buffer, b: Buffer, y: Buffer, rows: int, width: int, b_rows: int):
    check(lib.tmc_k_fused_silu_mul(x.ptr, b.ptr, y.ptr, rows, width, b_rows, int(x.dtype == F16), rt.stream))


def fused_linear_relu(rt: Runtime, a: Buffer, w: Buffer, bias: Buffer, y: Buffer, m: int, k: int, n: int):
    check(lib.tmc_k_fused_linear_relu(a.ptr, w.ptr, bias.ptr, y.ptr, m, k, n, int(a.dtype == F16), rt.stream))


def gemv_f16(rt: Runtime, x: Buffer, w: Buffer, y: Buffer, rows: int, k: int, n: int):
    if y.dtype == F16:
        check(lib.tmc_k_gemv_f16(x.ptr, w.ptr, y.ptr, rows, k, n, rt.stream))
    else:
        check(lib.tmc_k_gemv_f16_f32out(x.ptr, w.ptr, y.ptr, rows, k, n, rt.stream))


def batched_gemm_workspace_bytes(n: int, k: int, rows: int) -> int:
    return int(lib.tmc_k_batched_gemm_workspace_bytes(n, k, rows))


def batched_gemm_f16(rt: Runtime, x: Buffer, w: Buffer, y: Buffer, rows: int, k: int, n: int,
                     workspace: Buffer):
    """y [rows, n] fp32 = x [rows, k] . W [n, k]^T on the tcgen05 tensor cores."""
    check(lib.tmc_k_batched_gemm_f16_f32out(x.ptr, w.ptr, y.ptr, rows, k, n, workspace.ptr,
                                            rt.status_ptr, rt.stream))


def attention_workspace_bytes(rows, hq, hkv, d, max_splits) -> int:
    return int(lib.tmc_k_attention_workspace_bytes(rows, hq, hkv, d, max_splits))


def paged_attention_f16(rt: Runtime, q: Buffer, out: Buffer, k_pool: Buffer, v_pool: Buffer,
                        block_table: Buffer, table_stride: int, table_rows: Buffer,
                        positions: Buffer, rows: int, hq: int, hkv: int, d: int, page_size: int,
                        pool_pages: int, capacity: int, max_splits: int, min_chunk: int,
                        workspace: Buffer | None, counters: Buffer, schedule: int = 0, row_group: int = 1):
    """schedule: 0 automatic, 1 split-K with cluster merges, 2 streaming (persistent CTAs);
    row_group 2: prefill rows of one sequence served in groups (streaming schedule)."""
    check(lib.tmc_k_paged_attention_f16_ex(
        q.ptr, out.ptr, k_pool.ptr, v_pool.ptr, block_table.ptr, table_stride, table_rows.ptr,
        positions.ptr, rows, hq, hkv, d, page_size, pool_pages, capacity, max_splits, min_chunk,
        workspace.ptr if workspace is not None else None, counters.ptr, schedule, row_group, rt.status_ptr,
        rt.stream))


def fill_normal_f16(rt: Runtime, buf: Buffer, seed: int, mean: float, std: float):
    check(lib.tmc_k_fill_normal_f16(buf.ptr, buf.count, seed, mean, std, rt.stream))


# ---- decoder executor (tmc_decoder_*) ------------------------------------------------

class DecoderConfig(ctypes.Structure):
    _fields_ = [
        ("hidden_size", c_int), ("heads", c_int), ("kv_heads", c_int), ("head_dim", c_int),
        ("intermediate_size", c_int), ("vocab_size", c_int), ("layers", c_int),
        ("capacity", c_int), ("epsilon", c_float), ("rope_theta", ctypes.c_double),
        ("max_rows", c_int), ("max_slots", c_int), ("page_size", c_int), ("pool_pages", c_int),
        ("tp_rank", c_int), ("tp_size", c_int), ("use_graphs", c_int), ("use_pdl", c_int),
    ]


_I32P = POINTER(c_int32)
_sig("tmc_decoder_create", c_int, c_void_p, POINTER(DecoderConfig), POINTER(c_void_p))
_sig("tmc_decoder_destroy", None, c_void_p)
_sig("tmc_decoder_load_weight", c_int, c_void_p, c_char_p, POINTER(c_float), c_size_t)
_sig("tmc_decoder_load_weight_f16", c_int, c_void_p, c_char_p, c_void_p, c_size_t)
_sig("tmc_decoder_read_weight", c_int, c_void_p, c_char_p, POINTER(c_float), c_size_t)
_sig("tmc_decoder_init_random", c_int, c_void_p, c_uint64, c_float)
_sig("tmc_decoder_prefill", c_int, c_void_p, c_int, _I32P, c_int, POINTER(c_float), _I32P)
_sig("tmc_decoder_prefill_timing", c_int, c_void_p, POINTER(ctypes.c_double), POINTER(ctypes.c_double))
_sig("tmc_decoder_decode", c_int, c_void_p, _I32P, _I32P, c_int, POINTER(c_float), _I32P)
_sig("tmc_decoder_generate", c_int, c_void_p, _I32P, _I32P, c_int, c_int, _I32P,
     POINTER(ctypes.c_double))
_sig("tmc_decoder_current_length", c_size_t, c_void_p, c_int)
_sig("tmc_decoder_read_kv", c_int, c_void_p, c_int, c_int, POINTER(c_float), POINTER(c_float), c_size_t)
_sig("tmc_decoder_restore_kv", c_int, c_void_p, c_int, c_size_t, POINTER(c_float), POINTER(c_float))
_sig("tmc_decoder_block_table", c_int, c_void_p, c_int, _I32P, c_size_t, POINTER(c_size_t))
_sig("tmc_decoder_stage_length", c_int, c_void_p, c_int, c_size_t)
_sig("tmc_decoder_commit_length", c_int, c_void_p, c_int, c_size_t)
_sig("tmc_decoder_rollback_length", c_int, c_void_p, c_int, c_size_t)
_sig("tmc_decoder_release", c_int, c_void_p, c_int)
_sig("tmc_decoder_storage", c_int, c_void_p, POINTER(c_size_t), POINTER(c_size_t), POINTER(c_size_t))
_sig("tmc_decoder_local_dims", c_int, c_void_p, POINTER(c_int), POINTER(c_int), POINTER(c_int),
     POINTER(c_int), POINTER(c_int))
_sig("tmc_decoder_pool_stats", c_int, c_void_p, POINTER(c_size_t), POINTER(c_size_t),
     POINTER(c_size_t), POINTER(c_size_t), POINTER(c_size_t))
_sig("tmc_decoder_inject_page_failures", c_int, c_void_p, c_size_t)
_sig("tmc_decoder_kernels_per_step", c_int, c_void_p, c_int)
_sig("tmc_decoder_step_bytes", ctypes.c_double, c_void_p, c_int, _I32P)
_sig("tmc_decoder_profile_kernel", c_int, c_void_p, c_int, c_int, c_int, POINTER(ctypes.c_double),
     POINTER(ctypes.c_double), POINTER(c_int))
_sig("tmc_decoder_set_trace", c_int, c_void_p, c_size_t)
_sig("tmc_decoder_read_trace", c_int, c_void_p, POINTER(ctypes.c_uint64), c_size_t, POINTER(c_size_t))
_sig("tmc_nccl_unique_id", c_int, ctypes.c_char_p, c_size_t)
_sig("tmc_decoder_attach_nccl", c_int, c_void_p, ctypes.c_char_p, c_size_t, c_int, c_int)
_sig("tmc_decoder_exchange_handle", c_int, c_void_p, ctypes.c_char_p, c_size_t)
_sig("tmc_decoder_attach_peers", c_int, c_void_p, ctypes.c_char_p, c_size_t, c_int, c_int)
_sig("tmc_decoder_attach_local_peers", c_int, c_void_p, POINTER(c_void_p), c_int, c_int)
_sig("tmc_decoder_set_wait_budgets", c_int, c_void_p, c_uint64, c_uint64)
EXCHANGE_HANDLE_BYTES = 64


class ServingMetrics(ctypes.Structure):
    _fields_ = [(n, ctypes.c_double) for n in (
        "total_time_us", "tokens_per_second", "prefill_gpu_us", "decode_gpu_us", "scheduler_overhead_us",
        "kv_management_overhead_us", "preemption_overhead_us", "average_active_batch")] + \
        [(n, ctypes.c_uint64) for n in (
            "max_active_batch", "preemptions", "resumes", "peak_pages", "page_allocations", "page_releases",
            "decode_submissions", "decoded_tokens", "prefill_tokens", "ticks", "model_bytes", "kv_pool_bytes",
            "activation_bytes")]

    def as_dict(self):
        return {name: getattr(self, name) for name, _ in self._fields_}


_sig("tmc_serving_run", c_int, c_void_p, c_int, _I32P, _I32P, _I32P, _I32P, _I32P,
     POINTER(ctypes.c_double), POINTER(ctypes.c_double), POINTER(c_float), POINTER(c_float),
     POINTER(ServingMetrics), ctypes.c_char_p, c_size_t)


def _i32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32).reshape(-1))


_sig("tmc_plan_regions", c_int, c_int, _I32P, c_size_t, c_int, _I32P, c_int, _I32P, _I32P, _I32P, c_size_t,
     POINTER(c_size_t))

_sig("tmc_plan_buffers", c_int, c_int, _I32P, c_size_t, c_int, _I32P, c_int, _I32P, _I32P, _I32P, POINTER(c_int))

REGION_KINDS = ("Unfused", "Add + RMSNorm", "Residual Add + LayerNorm", "SiLU + Mul", "Linear + ReLU")


def plan_regions(input_count: int, nodes, outputs, contiguous):
    """Fused-kernel regions of a typed tensor graph (tmc_plan_regions; the
    reference's formRegions). nodes: [(op number, operand value ids...)], node i
    defining value input_count + i; contiguous: per value. Returns (topological
    order, [(kind, nodes, inputs, outputs)])."""
    flat = []
    for op, *operands in nodes:
        flat += [int(op), len(operands)] + [int(v) for v in operands]
    flat = np.asarray(flat, np.int32)
    outs = np.asarray(outputs, np.int32)
    cont = np.asarray(contiguous, np.int32)
    if cont.size != input_count + len(nodes):
        raise ValueError("contiguous needs one flag per value")
    order = np.zeros(max(len(nodes), 1), np.int32)
    written = c_size_t(0)
    cap = 64 * (len(nodes) + 1) + 16
    while True:
        regions = np.zeros(cap, np.int32)
        code = lib.tmc_plan_regions(input_count, flat.ctypes.data_as(_I32P), flat.size, len(nodes),
                                    outs.ctypes.data_as(_I32P), outs.size, cont.ctypes.data_as(_I32P),
                                    order.ctypes.data_as(_I32P), regions.ctypes.data_as(_I32P), cap,
                                    ctypes.byref(written))
        if code == OK or written.value <= cap:
            break
        cap = written.value
    check(code)
    out, i = [], 0
    while i < written.value:
        kind = int(regions[i])
        i += 1
        parts = []
        for _ in range(3):
            k = int(regions[i])
            parts.append([int(x) for x in regions[i + 1:i + 1 + k]])
            i += 1 + k
        out.append((kind, *parts))
    return order[:len(nodes)].tolist(), out


def plan_buffers(input_count: int, nodes, outputs):
    """Buffer roles (0 input, 1 intermediate, 2 output), view aliases (-1 for
    none) and launched nodes of a tensor graph (tmc_plan_buffers; the
    reference's planGraph); same graph encoding as plan_regions."""
    flat = []
    for op, *operands in nodes:
        flat += [int(op), len(operands)] + [int(v) for v in operands]
    flat = np.asarray(flat, np.int32)
    outs = np.asarray(outputs, np.int32)
    values = input_count + len(nodes)
    roles = np.zeros(max(values, 1), np.int32)
    alias = np.zeros(max(values, 1), np.int32)
    launches = np.zeros(max(len(nodes), 1), np.int32)
    count = c_int(0)
    check(lib.tmc_plan_buffers(input_count, flat.ctypes.data_as(_I32P), flat.size, len(nodes),
                               outs.ctypes.data_as(_I32P), outs.size, roles.ctypes.data_as(_I32P),
                               alias.ctypes.data_as(_I32P), launches.ctypes.data_as(_I32P), ctypes.byref(count)))
    return roles[:values].tolist(), alias[:values].tolist(), launches[:count.value].tolist()


# ---- graph compilation (tmc_graph_*; the reference's compileGraph) -----------------------

OPS = ("Add", "Mul", "MatMul", "RMSNorm", "LayerNorm", "ReLU", "SiLU", "Softmax", "RoPE", "ReduceSum",
       "ReduceMean", "Reshape", "View", "Transpose", "Contiguous", "MaskedFill", "Slice", "Embedding", "Gather")

_sig("tmc_graph_plan", c_int, c_int, _I32P, c_size_t, _I32P, c_size_t, c_int, _I32P, c_int, c_char_p, c_size_t,
     POINTER(c_size_t))
_sig("tmc_graph_compile", c_int, c_void_p, c_int, _I32P, c_size_t, _I32P, c_size_t, c_int, _I32P, c_int,
     POINTER(c_void_p))
_sig("tmc_graph_destroy", None, c_void_p)
_sig("tmc_graph_describe", c_int, c_void_p, c_char_p, c_size_t, POINTER(c_size_t))
_sig("tmc_graph_value_info", c_int, c_void_p, c_int, POINTER(c_int), POINTER(c_int), POINTER(ctypes.c_int64),
     POINTER(c_size_t))
_sig("tmc_graph_run", c_int, c_void_p, POINTER(POINTER(c_float)), POINTER(POINTER(c_float)),
     POINTER(ctypes.c_double), POINTER(ctypes.c_double))
_sig("tmc_graph_input_buffer", c_int, c_void_p, c_int, POINTER(c_void_p))
_sig("tmc_graph_launch", c_int, c_void_p, c_int)


def encode_typed_graph(inputs, nodes):
    """(input_types, nodes) int32 arrays of the tmc_graph_* encoding.
    inputs: [(dtype F16 / F32, shape)]; nodes: [(op name or number, operands,
    attributes)], attributes a list of ints or floats (floats become their
    fp32 bit patterns: RMSNorm / LayerNorm epsilon)."""
    types = []
    for dtype, shape in inputs:
        types += [int(dtype), len(shape)] + [int(d) for d in shape]
    flat = []
    for op, operands, *rest in nodes:
        attrs = rest[0] if rest else []
        op = OPS.index(op) if isinstance(op, str) else int(op)
        enc = [float_bits(a) if isinstance(a, float) else int(a) for a in attrs]
        enc = [a - (1 << 32) if a >= (1 << 31) else a for a in enc]
        flat += [op, len(operands)] + [int(v) for v in operands] + [len(enc)] + enc
    return np.asarray(types, np.int32), np.asarray(flat, np.int32)


def graph_plan(inputs, nodes, outputs) -> list:
    """Host-only launch plan of a typed graph: one line per kernel launch."""
    types, flat = encode_typed_graph(inputs, nodes)
    outs = _i32(outputs)
    need = c_size_t(0)
    args = (len(inputs), types.ctypes.data_as(_I32P), types.size, flat.ctypes.data_as(_I32P), flat.size, len(nodes),
            outs.ctypes.data_as(_I32P), outs.size)
    check(lib.tmc_graph_plan(*args, None, 0, ctypes.byref(need)))
    buf = ctypes.create_string_buffer(need.value)
    check(lib.tmc_graph_plan(*args, buf, need.value, ctypes.byref(need)))
    return [line for line in buf.value.decode().splitlines() if line]


class Graph:
    """A compiled tensor graph (reference compileGraph -> CompiledGraph)."""

    def __init__(self, rt: "Runtime", inputs, nodes, outputs):
        types, flat = encode_typed_graph(inputs, nodes)
        outs = _i32(outputs)
        h = c_void_p()
        check(lib.tmc_graph_compile(rt.handle, len(inputs), types.ctypes.data_as(_I32P), types.size,
                                    flat.ctypes.data_as(_I32P), flat.size, len(nodes), outs.ctypes.data_as(_I32P),
                                    outs.size, ctypes.byref(h)))
        self.handle = h
        self.runtime = rt
        self.inputs = [(int(d), tuple(int(x) for x in s)) for d, s in inputs]
        self.outputs = [int(o) for o in outputs]

    def value_shape(self, value: int):
        dt, rank = c_int(), c_int()
        dims = (ctypes.c_int64 * 4)()
        n = c_size_t()
        check(lib.tmc_graph_value_info(self.handle, value, ctypes.byref(dt), ctypes.byref(rank), dims, ctypes.byref(n)))
        return tuple(dims[i] for i in range(rank.value))

    def plan(self) -> list:
        need = c_size_t(0)
        check(lib.tmc_graph_describe(self.handle, None, 0, ctypes.byref(need)))
        buf = ctypes.create_string_buffer(need.value)
        check(lib.tmc_graph_describe(self.handle, buf, need.value, ctypes.byref(need)))
        return [line for line in buf.value.decode().splitlines() if line]

    def run(self, *arrays):
        """Logical float outputs (one array per declared output) and the GPU time."""
        ins = [np.ascontiguousarray(a, dtype=np.float32).reshape(-1) for a in arrays]
        assert len(ins) == len(self.inputs)
        outs = [np.empty(self.value_shape(v), np.float32) for v in self.outputs]
        in_ptrs = (POINTER(c_float) * max(1, len(ins)))(*[_fptr(a) for a in ins])
        out_ptrs = (POINTER(c_float) * len(outs))(*[_fptr(o) for o in outs])
        g, c = ctypes.c_double(), ctypes.c_double()
        check(lib.tmc_graph_run(self.handle, in_ptrs, out_ptrs, ctypes.byref(g), ctypes.byref(c)))
        return outs, g.value

    def close(self):
        if getattr(self, "handle", None):
            lib.tmc_graph_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()


class ManifestInfo(ctypes.Structure):
    _fields_ = [("version", c_int), ("batch", c_int), ("hidden_size", c_int), ("heads", c_int), ("head_dim", c_int),
                ("intermediate_size", c_int), ("vocab_size", c_int), ("layers", c_int), ("capacity", c_int),
                ("prefill_length", c_int), ("decode_count", c_int), ("epsilon", c_float),
                ("requested_dtype", ctypes.c_char * 8), ("effective_dtype", ctypes.c_char * 8),
                ("kv_heads", c_int), ("rope_theta", ctypes.c_double)]


_sig("tmc_manifest_open", c_int, c_char_p, POINTER(c_void_p))
_sig("tmc_manifest_close", None, c_void_p)
_sig("tmc_manifest_get_info", c_int, c_void_p, POINTER(ManifestInfo))
_sig("tmc_manifest_tensor", c_int, c_void_p, c_char_p, POINTER(POINTER(c_float)), POINTER(c_size_t))
_sig("tmc_decoder_load_manifest", c_int, c_void_p, c_void_p)


class Manifest:
    """A decoder-only manifest in the reference's export format
    (importDecoderLLMWorkload, DecoderLLMImporter.cpp:154-281)."""

    def __init__(self, path: str):
        self.handle = None
        h = c_void_p()
        check(lib.tmc_manifest_open(str(path).encode(), ctypes.byref(h)))
        self.handle = h
        info = ManifestInfo()
        check(lib.tmc_manifest_get_info(self.handle, ctypes.byref(info)))
        self.info = {f: getattr(info, f) for f, _ in ManifestInfo._fields_}
        for f in ("requested_dtype", "effective_dtype"):
            self.info[f] = self.info[f].decode()

    def tensor(self, name: str) -> np.ndarray:
        ptr, n = POINTER(c_float)(), c_size_t()
        check(lib.tmc_manifest_tensor(self.handle, name.encode(), ctypes.byref(ptr), ctypes.byref(n)))
        return np.ctypeslib.as_array(ptr, shape=(n.value,)).copy()

    def decoder(self, runtime, **kw) -> "Decoder":
        """A decoder with the manifest's dimensions and its weights loaded."""
        i = self.info
        dec = Decoder(runtime, i["hidden_size"], i["heads"], i["intermediate_size"], i["vocab_size"], i["layers"],
                      i["capacity"], kv_heads=i["kv_heads"], epsilon=i["epsilon"], rope_theta=i["rope_theta"], **kw)
        check(lib.tmc_decoder_load_manifest(dec.handle, self.handle))
        return dec

    def close(self):
        if self.handle:
            lib.tmc_manifest_close(self.handle)
            self.handle = None

    def __del__(self):
        self.close()


class Decoder:
    """Decoder executor (reference CompiledDecoderLLM, DecoderLLMExecutor.hpp:46-102)."""

    def __init__(self, runtime: Runtime, hidden, heads, intermediate, vocab, layers, capacity,
                 kv_heads=None, head_dim=None, epsilon=1e-5, rope_theta=10000.0, max_rows=8,
                 max_slots=1, page_size=0, pool_pages=0, tp_rank=0, tp_size=1, use_graphs=True,
                 use_pdl=True):
        self.runtime = runtime
        cfg = DecoderConfig(hidden, heads, kv_heads or heads, head_dim or hidden // heads,
                            intermediate, vocab, layers, capacity, epsilon, rope_theta, max_rows,
                            max_slots, page_size, pool_pages, tp_rank, tp_size, int(use_graphs),
                            int(use_pdl))
        self.cfg = cfg
        h = c_void_p()
        check(lib.tmc_decoder_create(runtime.handle, ctypes.byref(cfg), ctypes.byref(h)))
        self.handle = h
        dims = [c_int() for _ in range(5)]
        check(lib.tmc_decoder_local_dims(h, *[ctypes.byref(d) for d in dims]))
        (self.local_heads, self.local_kv_heads, self.local_intermediate, self.local_vocab,
         self.vocab_offset) = [d.value for d in dims]

    def close(self):
        if self.handle:
            lib.tmc_decoder_destroy(self.handle)
            self.handle = c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # weights
    def load_weight(self, name: str, values):
        values = np.asarray(values)
        if values.dtype == np.float16:
            v = np.ascontiguousarray(values.reshape(-1))
            check(lib.tmc_decoder_load_weight_f16(self.handle, name.encode(), v.ctypes.data_as(c_void_p), v.size))
        else:
            v = np.ascontiguousarray(values.reshape(-1), dtype=np.float32)
            check(lib.tmc_decoder_load_weight(self.handle, name.encode(), _fptr(v), v.size))

    def load_weights(self, weights: dict):
        for name, value in weights.items():
            self.load_weight(name, value)

    def read_weight(self, name: str, count: int) -> np.ndarray:
        out = np.empty(count, dtype=np.float32)
        check(lib.tmc_decoder_read_weight(self.handle, name.encode(), _fptr(out), count))
        return out

    def init_random(self, seed: int, std: float = 0.02):
        check(lib.tmc_decoder_init_random(self.handle, seed, std))

    # execution
    def prefill(self, tokens, slot=0, logits=True):
        t = _i32(tokens)
        out = np.empty((t.size, self.local_vocab), dtype=np.float32) if logits else None
        nxt = np.zeros(1, dtype=np.int32)
        check(lib.tmc_decoder_prefill(self.handle, slot, t.ctypes.data_as(_I32P), t.size,
                                      _fptr(out) if logits else None, nxt.ctypes.data_as(_I32P)))
        return out, int(nxt[0])

    def prefill_timing(self):
        """(gpu_us, cpu_us) of the last prefill call."""
        g, c = ctypes.c_double(0.0), ctypes.c_double(0.0)
        check(lib.tmc_decoder_prefill_timing(self.handle, ctypes.byref(g), ctypes.byref(c)))
        return g.value, c.value

    def decode(self, tokens, slots=None, logits=True):
        t = _i32(tokens)
        s = _i32(slots if slots is not None else range(t.size))
        out = np.empty((t.size, self.local_vocab), dtype=np.float32) if logits else None
        nxt = np.zeros(t.size, dtype=np.int32)
        check(lib.tmc_decoder_decode(self.handle, s.ctypes.data_as(_I32P), t.ctypes.data_as(_I32P), t.size,
                                     _fptr(out) if logits else None, nxt.ctypes.data_as(_I32P)))
        return out, nxt

    def generate(self, tokens, steps, slots=None):
        t = _i32(tokens)
        s = _i32(slots if slots is not None else range(t.size))
        out = np.zeros((steps, t.size), dtype=np.int32)
        us = ctypes.c_double(0.0)
        check(lib.tmc_decoder_generate(self.handle, s.ctypes.data_as(_I32P), t.ctypes.data_as(_I32P), t.size,
                                       steps, out.ctypes.data_as(_I32P), ctypes.byref(us)))
        return out, us.value

    # KV state
    def length(self, slot=0) -> int:
        return int(lib.tmc_decoder_current_length(self.handle, slot))

    def read_kv(self, layer, slot=0):
        n = self.local_kv_heads * self.length(slot) * self.cfg.head_dim
        k = np.empty(n, np.float32)
        v = np.empty(n, np.float32)
        check(lib.tmc_decoder_read_kv(self.handle, layer, slot, _fptr(k), _fptr(v), n))
        shape = (self.local_kv_heads, self.length(slot), self.cfg.head_dim)
        return k.reshape(shape), v.reshape(shape)

    def restore_kv(self, slot, keys, values):
        keys = np.ascontiguousarray(keys, dtype=np.float32)
        values = np.ascontiguousarray(values, dtype=np.float32)
        length = keys.shape[2]
        check(lib.tmc_decoder_restore_kv(self.handle, slot, length, _fptr(keys), _fptr(values)))

    def block_table(self, slot=0):
        n = c_size_t(0)
        check(lib.tmc_decoder_block_table(self.handle, slot, None, 0, ctypes.byref(n)))
        out = np.zeros(n.value, np.int32)
        check(lib.tmc_decoder_block_table(self.handle, slot, out.ctypes.data_as(_I32P), n.value, ctypes.byref(n)))
        return out

    def stage(self, slot, length):
        check(lib.tmc_decoder_stage_length(self.handle, slot, length))

    def commit(self, slot, length):
        check(lib.tmc_decoder_commit_length(self.handle, slot, length))

    def rollback(self, slot, length):
        check(lib.tmc_decoder_rollback_length(self.handle, slot, length))

    def release(self, slot=0):
        check(lib.tmc_decoder_release(self.handle, slot))

    def storage(self):
        a, b, c = c_size_t(), c_size_t(), c_size_t()
        check(lib.tmc_decoder_storage(self.handle, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c)))
        return {"model": a.value, "kv": b.value, "activation": c.value}

    def pool_stats(self):
        vals = [c_size_t() for _ in range(5)]
        check(lib.tmc_decoder_pool_stats(self.handle, *[ctypes.byref(v) for v in vals]))
        return dict(zip(("capacity", "used", "peak", "allocations", "releases"), [v.value for v in vals]))

    def inject_page_failures(self, n):
        check(lib.tmc_decoder_inject_page_failures(self.handle, n))

    def kernels_per_step(self, rows=1) -> int:
        return int(lib.tmc_decoder_kernels_per_step(self.handle, rows))

    def step_bytes(self, context_lengths) -> float:
        c = _i32(context_lengths)
        return float(lib.tmc_decoder_step_bytes(self.handle, c.size, c.ctypes.data_as(_I32P)))

    KERNELS = ("qkv", "attention", "o_proj", "gate_up", "down", "lm_head")

    def profile_kernel(self, kind, rows=1, rounds=4):
        """(mean launch us, algorithmic bytes per launch, launches per step)."""
        k = self.KERNELS.index(kind) if isinstance(kind, str) else int(kind)
        us, b, n = ctypes.c_double(), ctypes.c_double(), c_int()
        check(lib.tmc_decoder_profile_kernel(self.handle, k, rows, rounds, ctypes.byref(us),
                                             ctypes.byref(b), ctypes.byref(n)))
        return us.value, b.value, n.value

    def set_trace(self, capacity: int):
        check(lib.tmc_decoder_set_trace(self.handle, capacity))
        self._trace_cap = capacity

    def read_trace(self) -> np.ndarray:
        """Structured array (layer, kind, cta, t_entry, t_ready, t_exit) in ns."""
        cap = getattr(self, "_trace_cap", 0)
        buf = np.zeros((cap, 4), dtype=np.uint64)
        n = c_size_t(0)
        check(lib.tmc_decoder_read_trace(self.handle, buf.ctypes.data_as(POINTER(ctypes.c_uint64)), cap,
                                         ctypes.byref(n)))
        rec = buf[:min(n.value, cap)]
        out = np.zeros(len(rec), dtype=[("layer", "i4"), ("kind", "i4"), ("cta", "i4"),
                                        ("t_entry", "u8"), ("t_ready", "u8"), ("t_exit", "u8")])
        tag = rec[:, 0] >> np.uint64(32)
        out["layer"] = (tag >> np.uint64(8)).astype(np.int32)
        out["kind"] = (tag & np.uint64(0xff)).astype(np.int32)
        out["cta"] = (rec[:, 0] & np.uint64(0xffffffff)).astype(np.int32)
        out["t_entry"], out["t_ready"], out["t_exit"] = rec[:, 1], rec[:, 2], rec[:, 3]
        return out

    def attach_nccl(self, unique_id: bytes, world: int, rank: int):
        check(lib.tmc_decoder_attach_nccl(self.handle, unique_id, len(unique_id), world, rank))

    def exchange_handle(self) -> bytes:
        """CUDA IPC handle of this rank's peer-exchange window."""
        buf = ctypes.create_string_buffer(EXCHANGE_HANDLE_BYTES)
        check(lib.tmc_decoder_exchange_handle(self.handle, buf, EXCHANGE_HANDLE_BYTES))
        return buf.raw

    def attach_local_peers(self, ranks, rank: int):
        """Attach the windows of decoders driven by this process (ranks[r]
        is rank r's decoder, ranks[rank] is self)."""
        arr = (c_void_p * len(ranks))(*[d.handle for d in ranks])
        check(lib.tmc_decoder_attach_local_peers(self.handle, arr, len(ranks), rank))

    def set_wait_budgets(self, peer_ns: int = 0, local_ns: int = 0):
        """Budgets of the kernels' bounded waits in ns (0: the defaults)."""
        check(lib.tmc_decoder_set_wait_budgets(self.handle, peer_ns, local_ns))

    def attach_peers(self, handles, rank: int):
        """Map every rank's window (handles in rank order) and switch the
        tensor-parallel reductions to the fused peer exchange."""
        blob = b"".join(handles)
        check(lib.tmc_decoder_attach_peers(self.handle, blob, EXCHANGE_HANDLE_BYTES, len(handles), rank))


def serve(decoder: "Decoder", prompts, decode_counts, arrival_ticks=None, logits=False, log=False):
    """Continuous batching over the decoder's slots (tmc_serving_run).

    Returns a dict: tokens (list of int32 arrays, 1 + decode_count each),
    ttft_us, finish_us (arrays), metrics (dict), and when asked prefill_logits /
    decode_logits (lists of [len, local_vocab] arrays) and the scheduler log."""
    n = len(prompts)
    lens = [len(p) for p in prompts]
    offsets = np.zeros(n + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(lens)
    flat = _i32(np.concatenate([np.asarray(p, dtype=np.int32) for p in prompts]))
    counts = _i32(decode_counts)
    arrivals = _i32(arrival_ticks if arrival_ticks is not None else np.zeros(n))
    generated = np.zeros(int(counts.sum()) + n, dtype=np.int32)
    ttft = np.zeros(n, dtype=np.float64)
    finish = np.zeros(n, dtype=np.float64)
    vl = decoder.local_vocab
    pl = np.zeros((int(offsets[-1]), vl), dtype=np.float32) if logits else None
    dl = np.zeros((int(counts.sum()), vl), dtype=np.float32) if logits else None
    metrics = ServingMetrics()
    log_buf = ctypes.create_string_buffer(1 << 20) if log else None
    dptr = lambda a: a.ctypes.data_as(POINTER(ctypes.c_double))
    fptr = lambda a: a.ctypes.data_as(POINTER(c_float)) if a is not None else None
    check(lib.tmc_serving_run(decoder.handle, n, offsets.ctypes.data_as(_I32P), flat.ctypes.data_as(_I32P),
                              counts.ctypes.data_as(_I32P), arrivals.ctypes.data_as(_I32P),
                              generated.ctypes.data_as(_I32P), dptr(ttft), dptr(finish), fptr(pl), fptr(dl),
                              ctypes.byref(metrics), log_buf, (1 << 20) if log else 0))
    out = {"tokens": [], "ttft_us": ttft, "finish_us": finish, "metrics": metrics.as_dict()}
    g = 0
    for c in counts:
        out["tokens"].append(generated[g:g + 1 + int(c)])
        g += 1 + int(c)
    if logits:
        out["prefill_logits"] = [pl[offsets[i]:offsets[i + 1]] for i in range(n)]
        d0 = np.concatenate([[0], np.cumsum(counts)])
        out["decode_logits"] = [dl[d0[i]:d0[i + 1]] for i in range(n)]
    if log:
        out["log"] = log_buf.value.decode()
    return out


_sig("tmc_kernel_contract_json", c_int, c_char_p, c_char_p, c_size_t, POINTER(c_size_t))
_sig("tmc_admit_generated_kernel", c_int, c_char_p, c_char_p, c_int, c_char_p, c_char_p, POINTER(c_int),
     POINTER(ctypes.c_double), c_char_p, c_size_t)
_sig("tmc_registry_create", c_int, POINTER(c_void_p))
_sig("tmc_registry_destroy", None, c_void_p)
_sig("tmc_registry_load", c_int, c_void_p, c_char_p, POINTER(c_int), c_char_p, c_size_t)
_sig("tmc_registry_launch", c_int, c_void_p, c_char_p, POINTER(c_void_p), c_int, ctypes.c_uint, c_void_p)


def kernel_contract(pattern: str) -> dict:
    """The generated-kernel contract of `pattern` (makeKernelContract) as a dict."""
    import json
    need = c_size_t(0)
    check(lib.tmc_kernel_contract_json(pattern.encode(), None, 0, ctypes.byref(need)))
    buf = ctypes.create_string_buffer(need.value)
    check(lib.tmc_kernel_contract_json(pattern.encode(), buf, need.value, None))
    return json.loads(buf.value.decode())


def admit_generated_kernel(pattern: str, source: str, block_size: int, feedback_path: str = "",
                           artifact_path: str = "") -> dict:
    """Validate-then-benchmark admission (admitGeneratedKernel). Returns
    {admitted, speedup, log, feedback (dict or None)}."""
    import json
    admitted, speedup = c_int(0), ctypes.c_double(0.0)
    log = ctypes.create_string_buffer(1 << 16)
    check(lib.tmc_admit_generated_kernel(pattern.encode(), source.encode(), block_size, feedback_path.encode(),
                                         artifact_path.encode(), ctypes.byref(admitted), ctypes.byref(speedup),
                                         log, 1 << 16))
    feedback = None
    if feedback_path:
        with open(feedback_path) as f:
            feedback = json.loads(f.read())
    return {"admitted": bool(admitted.value), "speedup": speedup.value, "log": log.value.decode(),
            "feedback": feedback}


class GemvSelection(ctypes.Structure):
    _fields_ = [("success", c_int), ("use_baseline", c_int), ("ks", c_int), ("dynamic", c_int),
                ("tensor_core", c_int), ("conservative_speedup", ctypes.c_double)]


_sig("tmc_tune_decode_gemv", c_int, c_int, c_int, c_int, POINTER(c_float), POINTER(c_float), c_int, c_int,
     POINTER(GemvSelection), c_char_p, c_size_t)


def tune_decode_gemv(input, weight, fp16_storage: bool = True, prefill: bool = False) -> dict:
    """tuneDecodeGEMV: input [rows, k], weight [n, k], stored as fp16 or fp32."""
    x = np.ascontiguousarray(np.asarray(input, dtype=np.float32))
    w = np.ascontiguousarray(np.asarray(weight, dtype=np.float32))
    rows, k = x.shape
    n = w.shape[0]
    sel = GemvSelection()
    log = ctypes.create_string_buffer(1 << 14)
    check(lib.tmc_tune_decode_gemv(rows, k, n, x.ctypes.data_as(POINTER(c_float)), w.ctypes.data_as(POINTER(c_float)),
                                   int(fp16_storage), int(prefill), ctypes.byref(sel), log, 1 << 14))
    return {"success": bool(sel.success), "use_baseline": bool(sel.use_baseline), "ks": sel.ks,
            "dynamic": bool(sel.dynamic), "tensor_core": bool(sel.tensor_core),
            "speedup": sel.conservative_speedup, "log": log.value.decode()}


class RMSNormSelection(ctypes.Structure):
    _fields_ = [("success", c_int), ("used_baseline", c_int), ("selected_threads", c_int),
                ("speedup", ctypes.c_double), ("max_abs_error", ctypes.c_double)]


_sig("tmc_tune_rmsnorm", c_int, c_int, c_int, c_float, c_int, POINTER(c_float), POINTER(c_float), POINTER(c_int),
     c_int, POINTER(RMSNormSelection), POINTER(c_float), c_char_p, c_size_t)


def tune_rmsnorm(input, weight, eps: float, fp16: bool = False, candidate_threads=(64, 128, 256, 512)) -> dict:
    """tuneRMSNorm: input [rows, width], weight [width]; returns the selection and its validated output."""
    x = np.ascontiguousarray(np.asarray(input, dtype=np.float32))
    w = np.ascontiguousarray(np.asarray(weight, dtype=np.float32))
    rows, width = x.shape
    cands = (c_int * len(candidate_threads))(*candidate_threads)
    sel = RMSNormSelection()
    out = np.zeros((rows, width), dtype=np.float32)
    log = ctypes.create_string_buffer(1 << 14)
    check(lib.tmc_tune_rmsnorm(rows, width, eps, int(fp16), x.ctypes.data_as(POINTER(c_float)),
                               w.ctypes.data_as(POINTER(c_float)), cands, len(candidate_threads), ctypes.byref(sel),
                               out.ctypes.data_as(POINTER(c_float)), log, 1 << 14))
    return {"success": bool(sel.success), "used_baseline": bool(sel.used_baseline),
            "threads": sel.selected_threads, "speedup": sel.speedup, "max_abs_error": sel.max_abs_error,
            "output": out, "log": log.value.decode()}


class KernelRegistry:
    """Admitted generated kernels loaded from a directory of artifacts."""

    def __init__(self):
        h = c_void_p()
        check(lib.tmc_registry_create(ctypes.byref(h)))
        self.handle = h

    def load(self, directory: str):
        n = c_int(0)
        log = ctypes.create_string_buffer(1 << 14)
        check(lib.tmc_registry_load(self.handle, directory.encode(), ctypes.byref(n), log, 1 << 14))
        return n.value, log.value.decode()

    def launch(self, rt: "Runtime", pattern: str, buffers, work_items: int):
        arr = (c_void_p * len(buffers))(*[b.ptr for b in buffers])
        check(lib.tmc_registry_launch(self.handle, pattern.encode(), arr, len(buffers), work_items, rt.stream))

    def __del__(self):
        try:
            lib.tmc_registry_destroy(self.handle)
        except Exception:
            pass


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    check(lib.tmc_nccl_unique_id(buf, 128))
    return buf.raw
