"""Region planning (tmc_plan_regions, aicompiler-test_b200/csrc/RegionPlanner.hpp)
against the reference's own analyze + formRegions
(src/analyzer/GraphAnalyzer.cpp:278-364, PatternAnalyzer.cpp:32-132, compiled
into oracle/_ref): on seeded random tensor graphs built to contain the fusable
chains (MatMul -> Add -> ReLU, Add -> RMSNorm / LayerNorm, SiLU -> Mul) and
the conditions that break them (extra uses, graph outputs, view producers,
non-contiguous operands, the sum as a norm's weight), the planner must give
the same topological order and the same regions (members, fusion kind,
inputs, outputs) as the reference, given the reference's contiguity of each
value."""

import numpy as np
import pytest

from oracle import oracle


# Op numbers of the reference's tensor::OpType (GraphOp keeps them).
ADD, MUL, MATMUL, RMSNORM, LAYERNORM, RELU, SILU, SOFTMAX = 0, 1, 2, 3, 4, 5, 6, 7
RESHAPE, TRANSPOSE, CONTIGUOUS = 11, 13, 14

pytestmark = pytest.mark.skipif(not oracle.reference_available(), reason="oracle/_ref not built")


@pytest.fixture(scope="module")
def planner():
    import tmc_cuda

    def plan(inputs, nodes, outputs, contiguous):
        try:
            return tmc_cuda.plan_regions(inputs, nodes, outputs, contiguous)
        except tmc_cuda.TmcError as e:
            raise ValueError(str(e)) from e
    return plan


def compare(planner, n, squares, vectors, nodes, outputs):
    order, contiguous, ref = oracle.ref_form_regions(n, squares, vectors, nodes, outputs)
    got_order, got = planner(squares + vectors, nodes, outputs, contiguous)
    assert got_order == order
    assert got == ref
    return ref


def random_graph(rng, size):
    """A valid graph of fp32 [n, n] values (and [n] norm parameters): every
    operand choice respects the reference's type rules (norms and reshapes
    need contiguous data; a transpose yields a strided view)."""
    squares, vectors = int(rng.integers(1, 4)), 2
    values = [{"vec": False, "contig": True} for _ in range(squares)] + \
             [{"vec": True, "contig": True} for _ in range(vectors)]
    vec_ids = list(range(squares, squares + vectors))
    nodes = []

    def pick(contig=False, recent=True):
        cands = [i for i, v in enumerate(values) if not v["vec"] and (v["contig"] or not contig)]
        if recent and rng.random() < 0.7:
            cands = cands[-3:]
        return int(rng.choice(cands))

    def emit(op, *operands, contig=True):
        nodes.append((op, *operands))
        values.append({"vec": False, "contig": contig})
        return len(values) - 1

    while len(nodes) < size:
        r = rng.random()
        if r < 0.12:    # MatMul -> Add (bias or matrix) -> ReLU
            mm = emit(MATMUL, pick(), pick(recent=False))
            add = emit(ADD, mm, int(rng.choice(vec_ids)) if rng.random() < 0.5 else pick(recent=False))
            emit(RELU, add)
        elif r < 0.24:  # Add -> RMSNorm / LayerNorm
            s = emit(ADD, pick(), pick())
            if rng.random() < 0.5:
                emit(RMSNORM, s, int(rng.choice(vec_ids)))
            else:
                emit(LAYERNORM, s, vec_ids[0], vec_ids[1])
        elif r < 0.36:  # SiLU -> Mul, the activation on either side
            a = emit(SILU, pick())
            other = pick()
            emit(MUL, *((a, other) if rng.random() < 0.5 else (other, a)))
        elif r < 0.46:
            emit(TRANSPOSE, pick(), contig=False)
        elif r < 0.52:
            emit(RESHAPE, pick(contig=True))
        elif r < 0.57:
            emit(CONTIGUOUS, pick())
        elif r < 0.62:
            emit(SOFTMAX, pick())
        elif r < 0.70:
            v = pick()
            emit(ADD if rng.random() < 0.5 else MUL, v, v if rng.random() < 0.3 else pick())
        elif r < 0.78:
            emit(RELU if rng.random() < 0.5 else SILU, pick())
        elif r < 0.86:
            emit(MATMUL, pick(), pick())
        elif r < 0.93:
            emit(RMSNORM, pick(contig=True), int(rng.choice(vec_ids)))
        else:
            emit(LAYERNORM, pick(contig=True), vec_ids[0], vec_ids[1])
    first = squares + vectors
    last = first + len(nodes) - 1
    outputs = [last] + [v for v in range(first, last) if rng.random() < 0.12]
    return squares, vectors, nodes, outputs


def test_random_graphs_get_the_reference_buffer_plan():
    # planGraph (KernelPlan.cpp:11-59): buffer roles, view aliases, launched nodes.
    import tmc_cuda
    rng = np.random.default_rng(77)
    aliased = 0
    for _ in range(300):
        squares, vectors, nodes, outputs = random_graph(rng, int(rng.integers(2, 24)))
        if rng.random() < 0.2:
            outputs = outputs + [0]                  # an input that is also an output stays an input
        ref = oracle.ref_plan_buffers(4, squares, vectors, nodes, outputs)
        assert tmc_cuda.plan_buffers(squares + vectors, nodes, outputs) == ref
        aliased += sum(1 for a in ref[1] if a >= 0)
    assert aliased > 0


def test_random_graphs_split_into_the_reference_regions(planner):
    rng = np.random.default_rng(2024)
    kinds, checked = set(), 0
    for _ in range(400):
        squares, vectors, nodes, outputs = random_graph(rng, int(rng.integers(2, 24)))
        ref = compare(planner, 4, squares, vectors, nodes, outputs)
        kinds.update(k for k, *_ in ref)
        checked += 1
    assert checked == 400
    assert kinds == {0, 1, 2, 3, 4}, kinds  # every fusion kind occurred, and unfused regions


@pytest.mark.parametrize("case", ["fused", "sum_is_output", "sum_is_weight", "transposed_operand",
                                  "silu_used_twice", "read_twice", "view_producer", "chain_broken"])
def test_fusion_boundaries_match_the_reference(planner, case):
    # Values: 0, 1 [4, 4] inputs; 2, 3 [4] parameters; node i defines 4 + i.
    graphs = {
        # Add->RMSNorm, SiLU->Mul, MatMul->Add->ReLU all fuse.
        "fused": ([(ADD, 0, 1), (RMSNORM, 4, 2), (SILU, 5), (MUL, 1, 6), (MATMUL, 7, 0), (ADD, 8, 3),
                   (RELU, 9)], [10]),
        # The sum is also a graph output: it cannot stay inside a region.
        "sum_is_output": ([(ADD, 0, 1), (RMSNORM, 4, 2)], [4, 5]),
        # The sum reaches the norm as its weight, not its data.
        "sum_is_weight": ([(ADD, 2, 3), (RMSNORM, 0, 4)], [5]),
        # A fused MatMul operand is a transpose view (non-contiguous).
        "transposed_operand": ([(TRANSPOSE, 1), (MATMUL, 0, 4), (ADD, 5, 2), (RELU, 6)], [7]),
        # The activation has a second use.
        "silu_used_twice": ([(SILU, 0), (MUL, 4, 1), (ADD, 4, 5)], [6]),
        # The Mul reads the activation twice: two uses of one value.
        "read_twice": ([(SILU, 0), (MUL, 4, 4)], [5]),
        # A view produces the ReLU input of a would-be chain.
        "view_producer": ([(MATMUL, 0, 1), (ADD, 4, 2), (RESHAPE, 5), (RELU, 6)], [7]),
        # Add -> Softmax is not a fusion; MatMul -> Add with two uses of the sum.
        "chain_broken": ([(MATMUL, 0, 1), (ADD, 4, 0), (RELU, 5), (SOFTMAX, 5)], [6, 7]),
    }
    nodes, outputs = graphs[case]
    ref = compare(planner, 4, 2, 2, nodes, outputs)
    fused = [k for k, *_ in ref if k != 0]
    expected = {"fused": [1, 3, 4]}.get(case, [])
    assert sorted(fused) == expected, ref


def test_planner_reports_a_cycle(planner):
    # Node 0 reads node 1's result and node 1 reads node 0's.
    with pytest.raises(ValueError, match="cycle"):
        planner(1, [(ADD, 0, 2), (RELU, 1)], [2], [1, 1, 1])


def test_malformed_graphs_are_refused():
    import tmc_cuda
    with pytest.raises(tmc_cuda.TmcError, match="unknown op"):
        tmc_cuda.plan_regions(1, [(99, 0)], [1], [1, 1])
    with pytest.raises(tmc_cuda.TmcError, match="not a graph value"):
        tmc_cuda.plan_regions(1, [(RELU, 5)], [1], [1, 1])
    with pytest.raises(tmc_cuda.TmcError, match="graph output"):
        tmc_cuda.plan_regions(1, [(RELU, 0)], [7], [1, 1])
