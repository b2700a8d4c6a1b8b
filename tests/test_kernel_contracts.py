"""Generated-kernel contracts on the CPU (no GPU needed): the contract a
generator is given (makeKernelContract / serializeKernelContract,
src/llm/KernelContract.hpp:54-65, DecoderKernelContracts.cpp:129-245) --
patterns, buffer interface and kernel signature, three seeded cases, the fp16
variants' tolerances and input types, the 8M-weight GEMV cap and unknown
patterns."""

import pytest

import tmc_cuda


@pytest.mark.parametrize("pattern,inputs,outputs,work", [
    ("decoder_gemv_64_128", ["input", "weight"], ["output"], 128),
    ("decoder_rope", ["query", "key", "cosine", "sine", "valid_length"], ["rotated_query", "rotated_key"], 32),
    ("decoder_residual_rmsnorm", ["residual", "update", "weight"], ["sum", "normalized"], 1),
    ("decoder_gated_mlp", ["input", "gate_weight", "up_weight"], ["gated"], 128),
])
def test_contract_interface(pattern, inputs, outputs, work):
    c = tmc_cuda.kernel_contract(pattern)
    assert c["function_name"] == "generated_" + pattern
    assert [i["name"] for i in c["inputs"]] == inputs
    assert [o["name"] for o in c["outputs"]] == outputs
    assert len(c["cases"]) == 3 and all(case["work_items"] == work for case in c["cases"])
    assert c["minimum_speedup"] == pytest.approx(1.05)
    assert c["signature"].startswith('extern "C" __global__ void generated_' + pattern + "(")
    assert c["signature"].endswith("unsigned work_items)")
    assert c["group_per_work_item"] == (pattern != "decoder_rope")


def test_fp16_variants():
    c = tmc_cuda.kernel_contract("decoder_rope_fp16")
    assert c["storage"] == "fp16" and c["absolute_tolerance"] == pytest.approx(2e-2)
    # RoPE tables stay fp32, the length stays int32, Q/K become fp16.
    assert [i["type"] for i in c["inputs"]] == ["fp16", "fp16", "fp32", "fp32", "int32"]
    g = tmc_cuda.kernel_contract("decoder_gemv_2048_4096_fp16")
    assert [i["type"] for i in g["inputs"]] == ["fp16", "fp16"] and g["outputs"][0]["type"] == "fp16"


def test_gemv_contract_cap_and_unknown_patterns():
    tmc_cuda.kernel_contract("decoder_gemv_2048_4096")  # 8M weights: allowed
    with pytest.raises(tmc_cuda.TmcError):
        tmc_cuda.kernel_contract("decoder_gemv_4096_4096")
    with pytest.raises(tmc_cuda.TmcError):
        tmc_cuda.kernel_contract("decoder_softmax")
