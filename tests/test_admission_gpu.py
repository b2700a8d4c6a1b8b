"""Generated-kernel admission on the GPU (admitGeneratedKernel,
src/runtime/GeneratedKernelAdmission.cpp:204-318): NVRTC compile for sm_100a,
interface check, numerical validation of all contract cases against fp64,
two paired performance rounds against the template kernel (>= 1.05x each),
feedback and artifact files, and the registry that reloads admitted kernels
(KernelRegistry, src/runtime/KernelRegistry.hpp:25-38)."""

import json
import os

import numpy as np
import pytest

import tmc_cuda

pytestmark = pytest.mark.gpu

FAST_GEMV = r"""
extern "C" __global__ void generated_decoder_gemv_2048_4096(const float *x, const float *w, float *y,
                                                            unsigned work_items) {
  const unsigned j = blockIdx.x;
  const float4 *w4 = reinterpret_cast<const float4 *>(w + (size_t)j * 2048);
  const float4 *x4 = reinterpret_cast<const float4 *>(x);
  float s = 0.0f;
#pragma unroll 4
  for (unsigned i = threadIdx.x; i < 512; i += blockDim.x) {
    const float4 a = x4[i], b = __ldg(w4 + i);
    s += a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ float part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (unsigned i = 0; i < blockDim.x / 32; ++i) t += part[i];
    y[j] = t;
  }
}
"""


def admit(tmp_path, pattern, source, block):
    fb, art = str(tmp_path / "feedback.json"), str(tmp_path / "artifacts" / f"{pattern}.json")
    os.makedirs(tmp_path / "artifacts", exist_ok=True)
    return tmc_cuda.admit_generated_kernel(pattern, source, block, fb, art), art


def values(count, seed, scale=1.0):
    i = np.arange(count)
    return (((i * 17 + seed * 31) % 257) - 128).astype(np.float32) / 128 * np.float32(scale)


def test_fast_candidate_is_admitted_and_registry_runs_it(rt, tmp_path):
    r, art = admit(tmp_path, "decoder_gemv_2048_4096", FAST_GEMV, 128)
    assert r["admitted"], r["log"]
    assert r["feedback"]["status"] == "admitted" and r["speedup"] >= 1.05
    assert os.path.exists(art)
    reg = tmc_cuda.KernelRegistry()
    n, log = reg.load(str(tmp_path / "artifacts"))
    assert n == 1, log
    x, w = values(2048, 2), values(2048 * 4096, 11, 0.125)
    xb, wb = rt.upload(x), rt.upload(w)
    yb = rt.buffer(4096, tmc_cuda.F32)
    reg.launch(rt, "decoder_gemv_2048_4096", [xb, wb, yb], 4096)
    rt.synchronize()
    ref = w.reshape(4096, 2048).astype(np.float64) @ x.astype(np.float64)
    assert np.allclose(yb.read(), ref, atol=2e-4, rtol=2e-3)


@pytest.mark.parametrize("source,block,stage", [
    ("this is not CUDA", 64, "compile"),
    ('extern "C" __global__ void generated_decoder_gemv_64_128(const float *x, const float *w, float *y) {}',
     64, "interface"),
    ('extern "C" __global__ void generated_decoder_gemv_64_128(const float *x, const float *w, float *y, '
     'unsigned n) { if (threadIdx.x == 0) y[blockIdx.x] = 0.0f; }', 64, "numerical_validation"),
    ('extern "C" __global__ void generated_decoder_gemv_64_128(const float *x, const float *w, float *y, '
     'unsigned n) {}', 96, "hardware_filter"),
])
def test_rejections(rt, tmp_path, source, block, stage):
    r, art = admit(tmp_path, "decoder_gemv_64_128", source, block)
    assert not r["admitted"]
    assert r["feedback"]["stage"] == stage, r["log"]
    assert r["feedback"]["status"] == "retry"
    assert not os.path.exists(art)


def test_slow_correct_candidate_fails_performance(rt, tmp_path):
    src = r"""
extern "C" __global__ void generated_decoder_residual_rmsnorm(const float *res, const float *upd, const float *w,
                                                              float *sum, float *norm, unsigned n) {
  __nanosleep(200000);
  __shared__ float sq[64];
  const unsigned i = threadIdx.x;
  const float v = res[i] + upd[i];
  sq[i] = v * v;
  __syncthreads();
  float t = 0.0f;
  for (int j = 0; j < 64; ++j) t += sq[j];
  sum[i] = v;
  norm[i] = v * rsqrtf(t / 64.0f + 1e-5f) * w[i];
}
"""
    r, _ = admit(tmp_path, "decoder_residual_rmsnorm", src, 64)
    assert not r["admitted"]
    assert r["feedback"]["stage"] == "performance", r["log"]
    assert r["feedback"]["speedup"] < 1.05


def test_fp16_gated_mlp_candidate_validates(rt, tmp_path):
    src = r"""
#include <cuda_fp16.h>
extern "C" __global__ void generated_decoder_gated_mlp_fp16(const __half *x, const __half *wg, const __half *wu,
                                                            __half *y, unsigned n) {
  const unsigned j = blockIdx.x, lane = threadIdx.x;
  float g = 0.0f, u = 0.0f;
  for (unsigned i = lane; i < 64; i += 32) {
    g += __half2float(x[i]) * __half2float(wg[j * 64 + i]);
    u += __half2float(x[i]) * __half2float(wu[j * 64 + i]);
  }
  for (int o = 16; o > 0; o >>= 1) {
    g += __shfl_xor_sync(0xffffffffu, g, o);
    u += __shfl_xor_sync(0xffffffffu, u, o);
  }
  if (lane == 0) {
    g = __half2float(__float2half_rn(g));
    u = __half2float(__float2half_rn(u));
    const float a = __half2float(__float2half_rn(g / (1.0f + expf(-g))));
    y[j] = __float2half_rn(a * u);
  }
}
"""
    r, _ = admit(tmp_path, "decoder_gated_mlp_fp16", src, 32)
    assert "all outputs numerical validation: PASS" in r["log"]
    assert r["feedback"]["status"] == "admitted" or r["feedback"]["stage"] == "performance", r["log"]


@pytest.mark.parametrize("rows,k,n", [(1, 4096, 4096), (4, 1024, 2816), (1, 4096, 14336)])
def test_decode_gemv_tuner_selects_an_admitted_config(rt, rows, k, n):
    # tuneDecodeGEMV (DecodeGEMVTuner.cpp:162-304): every candidate validated,
    # selection only with >= 1.05x in two rounds over the generic linear layer.
    rng = np.random.default_rng(rows + k + n)
    x = rng.standard_normal((rows, k)).astype(np.float16).astype(np.float32)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float16).astype(np.float32)
    sel = tmc_cuda.tune_decode_gemv(x, w)
    assert sel["success"], sel["log"]
    assert "numerical: FAIL" not in sel["log"], sel["log"]
    if not sel["use_baseline"]:
        assert sel["speedup"] >= 1.05 and sel["ks"] in (1, 2, 4, 8)
        assert "-> admitted" in sel["log"]
    # At weight-streaming sizes the decode GEMV beats one CTA per output.
    if k * n >= 16 << 20:
        assert not sel["use_baseline"], sel["log"]


def test_decode_gemv_tuner_prefill_admits_the_tensor_core_gemm(rt):
    # The prefill candidate set (DecodeGEMVTuner.cpp:209-213): 64 rows, the
    # tcgen05 GEMM against the generic linear baseline, validated against the
    # baseline's output (64 x 4096 x 4096 > 64M MACs, 9 samples).
    rng = np.random.default_rng(3)
    x = rng.standard_normal((64, 4096)).astype(np.float16).astype(np.float32)
    w = (rng.standard_normal((4096, 4096)) * 0.02).astype(np.float16).astype(np.float32)
    sel = tmc_cuda.tune_decode_gemv(x, w, prefill=True)
    assert sel["success"], sel["log"]
    assert "samples=9" in sel["log"] and "numerical: FAIL" not in sel["log"], sel["log"]
    assert not sel["use_baseline"] and sel["tensor_core"] and sel["speedup"] >= 1.05, sel["log"]


def test_decode_gemv_tuner_fp32_storage_keeps_the_baseline(rt):
    # Every candidate reads fp16 weights: with fp32 storage the hardware filter
    # rejects them and the validated baseline is the selection.
    rng = np.random.default_rng(4)
    x = rng.standard_normal((2, 1024)).astype(np.float32)
    w = (rng.standard_normal((512, 1024)) * 0.02).astype(np.float32)
    sel = tmc_cuda.tune_decode_gemv(x, w, fp16_storage=False)
    assert sel["success"] and sel["use_baseline"], sel["log"]
    assert sel["log"].count("Hardware Filter: FAIL") == 5 and "dtype=fp32" in sel["log"], sel["log"]
