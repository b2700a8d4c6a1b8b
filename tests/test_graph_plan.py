"""Graph compilation planning on the host (tmc_graph_plan, no GPU): the
kernels a typed tensor graph becomes, region by region, as the reference's
compileGraph prepares one execution per region (GraphExecutor.cpp:346-431),
and the graphs it refuses."""

import pytest

F16, F32 = 0, 1


def plan(inputs, nodes, outputs):
    import tmc_cuda
    return tmc_cuda.graph_plan(inputs, nodes, outputs)


C1_NODES = [("RMSNorm", [0, 1], [1e-5]), ("Transpose", [2], [0, 1]), ("MatMul", [3, 4])]


def test_c1_graph_with_fp16_weight_is_one_fused_gemv():
    steps = plan([(F32, (1, 4096)), (F32, (4096,)), (F16, (4096, 4096))], C1_NODES, [5])
    assert steps == ["rmsnorm_gemv_f32(v0, v1, v2) -> v5 [RMSNorm -> GEMV (norm in the GEMV prologue)]"]


def test_c1_graph_with_fp32_weight_runs_norm_then_matmul():
    steps = plan([(F32, (2, 256)), (F32, (256,)), (F32, (128, 256))], C1_NODES, [5])
    assert steps == ["rmsnorm(v0, v1) -> v3 [Unfused]", "matmul(v3, v2) -> v5 [Unfused]"]


def test_norm_that_is_also_an_output_is_not_folded():
    steps = plan([(F32, (1, 64)), (F32, (64,)), (F16, (32, 64))], C1_NODES, [3, 5])
    assert [s.split("(")[0] for s in steps] == ["rmsnorm", "matmul"]


def test_fused_regions_map_to_their_kernels():
    x = (F32, (4, 64))
    row = (F32, (64,))
    # Add -> RMSNorm, SiLU -> Mul, MatMul -> Add -> ReLU, Add -> LayerNorm.
    assert plan([x, row, row], [("Add", [0, 1]), ("RMSNorm", [3, 2], [1e-5])], [4]) == \
        ["fused_add_rmsnorm(v0, v1, v2) -> v4 [Add + RMSNorm]"]
    assert plan([x, x], [("SiLU", [0]), ("Mul", [1, 2])], [3]) == ["fused_silu_mul(v0, v1) -> v3 [SiLU + Mul]"]
    assert plan([x, (F32, (64, 32)), (F32, (32,))], [("MatMul", [0, 1]), ("Add", [3, 2]), ("ReLU", [4])], [5]) == \
        ["fused_linear_relu(v0, v1, v2) -> v5 [Linear + ReLU]"]
    assert plan([x, x, row, row], [("Add", [0, 1]), ("LayerNorm", [4, 2, 3], [1e-5])], [5]) == \
        ["fused_add_layernorm(v0, v1, v2, v3) -> v5 [Residual Add + LayerNorm]"]


def test_unfused_nodes_views_and_the_decode_gemv():
    x = (F16, (3, 128))
    steps = plan([x, (F16, (128,)), (F16, (96, 128))],
                 [("RMSNorm", [0, 1]), ("Transpose", [2], [0, 1]), ("MatMul", [3, 4]), ("Reshape", [5], [288]),
                  ("ReLU", [6])], [7])
    assert steps == ["rmsnorm(v0, v1) -> v3 [Unfused]", "gemv_f16(v3, v2) -> v5 [Unfused]",
                     "relu(v5) -> v7 [Unfused]"]
    # A row broadcast Add on the smaller operand first, then Mul.
    steps = plan([(F32, (8,)), (F32, (5, 8))], [("Add", [0, 1]), ("Mul", [2, 2])], [3])
    assert steps == ["add(v1, v0) -> v2 [Unfused]", "mul(v2, v2) -> v3 [Unfused]"]


@pytest.mark.parametrize("inputs,nodes,outputs,fragment", [
    ([(F32, (4, 8))], [("Softmax", [0])], [1], "Softmax has no graph kernel"),
    ([(F32, (4, 8)), (F16, (4, 8))], [("Add", [0, 1])], [2], "matching floating-point dtypes"),
    ([(F32, (4, 8)), (F32, (3, 8))], [("Add", [0, 1])], [2], "broadcast"),
    ([(F32, (2, 4, 8)), (F32, (8, 4))], [("MatMul", [0, 1])], [2], "two-dimensional"),
    ([(F32, (4, 8))], [("Transpose", [0], [0, 1])], [1], "strided view"),
    ([(F32, (4, 8))], [("Add", [0, 2]), ("Add", [1, 0])], [2], "dependency cycle"),
    ([(F32, (4, 8)), (F32, (8,))], [("RMSNorm", [0, 1], [0.0])], [2], "epsilon"),
])
def test_refused_graphs(inputs, nodes, outputs, fragment):
    import tmc_cuda
    with pytest.raises(tmc_cuda.TmcError) as err:
        plan(inputs, nodes, outputs)
    assert fragment in err.value.message
