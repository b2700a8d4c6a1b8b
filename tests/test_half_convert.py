"""Host fp16 / bf16 conversion (aicompiler-test_b200/csrc/half_convert.hpp, the
rounding every host float takes on its way into fp16 / bf16 device storage, as
the reference's Metal buffers do, MetalRuntime.mm:42-104,537-556), against
numpy's IEEE binary16 and torch's bfloat16 conversions (both round to nearest,
ties to even): every fp16 value decoded, every fp16 rounding boundary (the
midpoints and their float32 neighbours), random float32 bit patterns, overflow,
subnormals, signed zeros, infinities and NaN."""

import ctypes
import os
import shutil
import subprocess

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "aicompiler-test_b200", "csrc")


@pytest.fixture(scope="module")
def conv(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    out = str(tmp_path_factory.mktemp("halfshim") / "libhalfshim.so")
    subprocess.run(["g++", "-std=c++17", "-O2", "-shared", "-fPIC", "-I", CSRC,
                    os.path.join(ROOT, "tests", "half_shim.cpp"), "-o", out], check=True, capture_output=True)
    lib = ctypes.CDLL(out)
    for name in ("to_half", "from_half", "to_bf16", "from_bf16"):
        getattr(lib, name).restype = None
        getattr(lib, name).argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]

    def run(name, values, out_dtype):
        values = np.ascontiguousarray(values)
        out = np.empty(values.shape, out_dtype)
        getattr(lib, name)(values.ctypes.data, out.ctypes.data, values.size)
        return out
    return run


def f32_bits(bits):
    return np.asarray(bits, np.uint32).view(np.float32)


def boundary_floats():
    # Every finite fp16 value, the midpoint to its successor, and the float32
    # neighbours of that midpoint (where rounding direction and ties are decided).
    h = np.arange(0, 0x7c00, dtype=np.uint16).view(np.float16).astype(np.float64)
    nxt = np.append(h[1:], 65536.0)
    mid = ((h + nxt) / 2).astype(np.float32)
    cands = [h.astype(np.float32), mid, np.nextafter(mid, np.float32(np.inf)), np.nextafter(mid, np.float32(0))]
    v = np.concatenate(cands)
    return np.concatenate([v, -v])


def test_half_decode_is_exact_for_every_pattern(conv):
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    got = conv("from_half", bits, np.float32)
    ref = bits.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))
    assert np.all(np.isnan(got[nan]))


def test_half_encode_rounds_to_nearest_even_at_every_boundary(conv):
    v = boundary_floats()
    got = conv("to_half", v, np.uint16)
    with np.errstate(over="ignore"):  # the top midpoint (65520) rounds to infinity
        ref = v.astype(np.float16)
    assert np.array_equal(got, ref.view(np.uint16))


def test_half_encode_matches_on_random_bit_patterns_and_edges(conv):
    rng = np.random.default_rng(0)
    v = f32_bits(rng.integers(0, 2 ** 32, 1 << 21, dtype=np.uint64))
    edges = np.array([0.0, -0.0, 65504.0, 65519.996, 65520.0, -65520.0, 1e-8, 2.0 ** -24, 2.0 ** -25,
                      2.0 ** -25 * 1.0000001, 2.0 ** -14, 5.9604645e-08, np.inf, -np.inf], np.float32)
    v = np.concatenate([v, edges])
    got = conv("to_half", v, np.uint16)
    with np.errstate(over="ignore"):
        ref = v.astype(np.float16)
    nan = np.isnan(v)
    assert np.array_equal(got[~nan], ref[~nan].view(np.uint16))
    # NaN stays NaN (quiet) with its sign.
    g = got[nan]
    assert np.all((g & 0x7c00) == 0x7c00) and np.all((g & 0x3ff) != 0)
    assert np.array_equal(g >> 15, (v[nan].view(np.uint32) >> 31).astype(np.uint16))


def test_bf16_round_trip_matches_torch(conv):
    rng = np.random.default_rng(1)
    v = f32_bits(rng.integers(0, 2 ** 32, 1 << 21, dtype=np.uint64))
    # Ties: the low 16 bits exactly 0x8000, with even and odd kept halves.
    ties = f32_bits((rng.integers(0, 2 ** 16, 4096, dtype=np.uint64) << 16) | 0x8000)
    v = np.concatenate([v, ties, np.array([0.0, -0.0, np.inf, -np.inf, 3.3895314e38], np.float32)])
    got = conv("to_bf16", v, np.uint16)
    ref = torch.from_numpy(v).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    nan = np.isnan(v)
    assert np.array_equal(got[~nan], ref[~nan])
    assert np.all(np.isnan(conv("from_bf16", got[nan], np.float32)))
    back = conv("from_bf16", got[~nan], np.float32)
    assert np.array_equal(back.view(np.uint32), got[~nan].astype(np.uint32) << 16)
