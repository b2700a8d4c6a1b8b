// oracle/ref_driver.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A thin extern "C" driver around the reference's own CPU oracle
// (tensor::validation::evaluateGraph, reference src/validation/GraphReference.cpp:98,
// with analyze(), src/analyzer/GraphAnalyzer.cpp:278), compiled from the
// reference sources where they lie (oracle/Makefile) into oracle/_ref/.
// It is used to pin the C restatement in oracle/graph_ref.c and to time the
// reference's CPU path; the product never links it.
#include <cstdint>
#include <cstring>
#include <exception>
#include <stdexcept>
#include <string>
#include <vector>

#include "analyzer/GraphAnalyzer.hpp"
#include "analyzer/PatternAnalyzer.hpp"
#include "planner/KernelPlan.hpp"
#include "validation/GraphReference.hpp"

using namespace tensor;

namespace {
thread_local std::string g_error;
}

extern "C" {

const char *ref_last_error() { return g_error.c_str(); }

// The C1 graph of the scope table: RMSNorm(x, gamma) -> MatMul with a
// Transpose(W) view, everything fp32 (W holds fp16-rounded values because
// TensorIR MatMul requires matching dtypes, GraphAnalyzer.cpp:74).
// y receives the fp64 "precise" outputs of evaluateGraph.
int ref_rmsnorm_matmul(const float *x, const float *gamma, const float *w, long rows, long k,
                       long n, float eps, double *y) {
  try {
    TensorGraph graph;
    const auto xi = graph.addInput("x", TensorType{{std::size_t(rows), std::size_t(k)}, DType::Float32});
    const auto gi = graph.addInput("gamma", TensorType{{std::size_t(k)}, DType::Float32});
    const auto wi = graph.addInput("weight", TensorType{{std::size_t(n), std::size_t(k)}, DType::Float32});
    const auto normed = graph.addNode(OpType::RMSNorm, {xi, gi}, RMSNormAttributes{eps, -1});
    const auto wt = graph.addNode(OpType::Transpose, {wi}, TransposeAttributes{0, 1});
    const auto out = graph.addNode(OpType::MatMul, {normed, wt});
    graph.outputs = {out};
    const auto analyzed = analyzer::analyze(graph);
    GraphInputs inputs;
    inputs[xi] = std::vector<float>(x, x + rows * k);
    inputs[gi] = std::vector<float>(gamma, gamma + k);
    inputs[wi] = std::vector<float>(w, w + n * k);
    const auto result = validation::evaluateGraph(analyzed, inputs);
    const auto &o = result.outputs.at(0);
    std::memcpy(y, o.data(), o.size() * sizeof(double));
    return 0;
  } catch (const std::exception &e) {
    g_error = e.what();
    return 1;
  }
}

// RMSNorm graph alone (the graph-suite RMSNorm cases, tensor_graph_examples.cpp:79-123),
// dtype 0 = fp16 storage, 1 = fp32.
int ref_rmsnorm(const float *x, const float *gamma, long rows, long width, float eps, int dtype,
                double *y) {
  try {
    const DType dt = dtype == 0 ? DType::Float16 : DType::Float32;
    TensorGraph graph;
    const auto xi = graph.addInput("x", TensorType{{std::size_t(rows), std::size_t(width)}, dt});
    const auto gi = graph.addInput("gamma", TensorType{{std::size_t(width)}, dt});
    const auto out = graph.addNode(OpType::RMSNorm, {xi, gi}, RMSNormAttributes{eps, -1});
    graph.outputs = {out};
    const auto analyzed = analyzer::analyze(graph);
    GraphInputs inputs;
    inputs[xi] = std::vector<float>(x, x + rows * width);
    inputs[gi] = std::vector<float>(gamma, gamma + width);
    const auto result = validation::evaluateGraph(analyzed, inputs);
    const auto &o = result.outputs.at(0);
    std::memcpy(y, o.data(), o.size() * sizeof(double));
    return 0;
  } catch (const std::exception &e) {
    g_error = e.what();
    return 1;
  }
}

// The graph suite's fused regions (tensor_graph_examples.cpp:115-143,210-225),
// formed by formRegions (PatternAnalyzer.cpp:32-132) and emitted by emitFusion
// (FusionMetalEmitter.cpp:81-214): kind 0 Add -> RMSNorm, 1 Add -> LayerNorm,
// 2 SiLU -> Mul, 3 MatMul -> Add(bias) -> ReLU. x [rows, width]; b is the
// second operand of the Add / Mul ([b_rows, width], b_rows 1 or rows) or the
// MatMul weight [width, n]; w / c the norm weight / bias (or the ReLU bias
// [n]). dtype 0 = fp16 storage, 1 = fp32. y: fp64 precise outputs.
int ref_fusion(int kind, const float *x, const float *b, const float *w, const float *c, long rows, long width,
               long b_rows, long n, float eps, int dtype, double *y) {
  try {
    const DType dt = dtype == 0 ? DType::Float16 : DType::Float32;
    const auto R = std::size_t(rows), W = std::size_t(width), BR = std::size_t(b_rows), N = std::size_t(n);
    TensorGraph graph;
    GraphInputs inputs;
    const auto xi = graph.addInput("x", TensorType{{R, W}, dt});
    inputs[xi] = std::vector<float>(x, x + R * W);
    if (kind == 3) {
      const auto wi = graph.addInput("weight", TensorType{{W, N}, dt});
      const auto bi = graph.addInput("bias", TensorType{{N}, dt});
      inputs[wi] = std::vector<float>(b, b + W * N);
      inputs[bi] = std::vector<float>(c, c + N);
      const auto linear = graph.addNode(OpType::MatMul, {xi, wi});
      const auto biased = graph.addNode(OpType::Add, {linear, bi});
      graph.outputs = {graph.addNode(OpType::ReLU, {biased})};
    } else {
      const TensorType bt = BR == 1 ? TensorType{{W}, dt} : TensorType{{R, W}, dt};
      const auto bi = graph.addInput("b", bt);
      inputs[bi] = std::vector<float>(b, b + BR * W);
      if (kind == 2) {
        const auto act = graph.addNode(OpType::SiLU, {xi});
        graph.outputs = {graph.addNode(OpType::Mul, {act, bi})};
      } else {
        const auto wi = graph.addInput("weight", TensorType{{W}, dt});
        inputs[wi] = std::vector<float>(w, w + W);
        const auto added = graph.addNode(OpType::Add, {xi, bi});
        if (kind == 0) {
          graph.outputs = {graph.addNode(OpType::RMSNorm, {added, wi}, RMSNormAttributes{eps, -1})};
        } else {
          const auto ci = graph.addInput("bias", TensorType{{W}, dt});
          inputs[ci] = std::vector<float>(c, c + W);
          LayerNormAttributes attributes;
          attributes.epsilon = eps;
          graph.outputs = {graph.addNode(OpType::LayerNorm, {added, wi, ci}, attributes)};
        }
      }
    }
    const auto analyzed = analyzer::analyze(graph);
    const auto result = validation::evaluateGraph(analyzed, inputs);
    const auto &o = result.outputs.at(0);
    std::memcpy(y, o.data(), o.size() * sizeof(double));
    return 0;
  } catch (const std::exception &e) {
    g_error = e.what();
    return 1;
  }
}

// The graph encoding of ref_form_regions / ref_plan_buffers (see below).
static TensorGraph build_square_graph(long n, long squares, long vectors, const int *nodes, long node_count,
                               const int *outputs, long output_count) {
  const auto N = std::size_t(n);
  TensorGraph graph;
  for (long i = 0; i < squares; ++i) graph.addInput("m" + std::to_string(i), TensorType{{N, N}, DType::Float32});
  for (long i = 0; i < vectors; ++i) graph.addInput("v" + std::to_string(i), TensorType{{N}, DType::Float32});
  const int *p = nodes;
  for (long i = 0; i < node_count; ++i) {
    const auto op = static_cast<OpType>(*p++);
    const int arity = *p++;
    std::vector<ValueId> operands(p, p + arity);
    p += arity;
    OpAttributes attributes;
    if (op == OpType::Transpose) attributes = TransposeAttributes{0, 1};
    if (op == OpType::Reshape || op == OpType::View) attributes = ReshapeAttributes{{N, N}};
    graph.addNode(op, operands, attributes);
  }
  graph.outputs.assign(outputs, outputs + output_count);
  return graph;
}

// The reference's own region formation (analyze + formRegions,
// src/analyzer/PatternAnalyzer.cpp:32-132) on a graph given as:
//   n: every tensor is fp32 [n, n] except `vectors` inputs of shape [n];
//   `squares` [n, n] inputs (value ids 0..squares-1), then the vectors;
//   nodes: per node {op (OpType number), operand count, operands...}; node i
//   defines value squares + vectors + i (Transpose swaps axes 0 and 1, Reshape /
//   View keep [n, n]);
//   outputs: declared graph outputs.
// Writes order[node_count], contiguous[value_count] (0/1) and the regions as
// {fusion, #nodes, nodes..., #inputs, inputs..., #outputs, outputs...} into
// regions (capacity `cap` ints); returns the number of ints written, or -1
// with ref_last_error() set when the reference rejects the graph.
long ref_form_regions(long n, long squares, long vectors, const int *nodes, long node_count, const int *outputs,
                      long output_count, int *order, int *contiguous, int *regions, long cap) {
  try {
    const auto graph = build_square_graph(n, squares, vectors, nodes, node_count, outputs, output_count);
    const auto planned = analyzer::formRegions(analyzer::analyze(graph));
    for (std::size_t i = 0; i < planned.analyzed.order.size(); ++i) order[i] = int(planned.analyzed.order[i]);
    for (std::size_t v = 0; v < planned.analyzed.types.size(); ++v)
      contiguous[v] = planned.analyzed.types[v].isContiguous() ? 1 : 0;
    long w = 0;
    auto put = [&](long value) {
      if (w >= cap) throw std::runtime_error("region output buffer too small");
      regions[w++] = int(value);
    };
    for (const auto &r : planned.regions) {
      put(long(r.fusion));
      put(long(r.nodes.size()));
      for (auto x : r.nodes) put(long(x));
      put(long(r.inputs.size()));
      for (auto x : r.inputs) put(long(x));
      put(long(r.outputs.size()));
      for (auto x : r.outputs) put(long(x));
    }
    return w;
  } catch (const std::exception &e) {
    g_error = e.what();
    return -1;
  }
}

// The reference's planGraph (src/planner/KernelPlan.cpp:11-59) on the same
// encoding: roles[value] (0 input, 1 intermediate, 2 output), alias_of[value]
// (-1 when the value owns storage) and the launched nodes in plan order;
// returns their count, or -1 with ref_last_error() set.
long ref_plan_buffers(long n, long squares, long vectors, const int *nodes, long node_count, const int *outputs,
                      long output_count, int *roles, int *alias_of, int *launches) {
  try {
    const auto graph = build_square_graph(n, squares, vectors, nodes, node_count, outputs, output_count);
    const auto plan = planner::planGraph(analyzer::analyze(graph));
    for (const auto &b : plan.buffers) {
      roles[b.value] = b.role == planner::BufferRole::Input ? 0 : b.role == planner::BufferRole::Intermediate ? 1 : 2;
      alias_of[b.value] = b.aliasOf ? int(*b.aliasOf) : -1;
    }
    long k = 0;
    for (const auto &kernel : plan.kernels) launches[k++] = int(kernel.nodeIndex);
    return k;
  } catch (const std::exception &e) {
    g_error = e.what();
    return -1;
  }
}

// The reference's own evaluateGraph on a typed graph in the encoding of
// tmc_graph_compile (include/tmc_cuda.h): input types {dtype 0 fp16 / 1 fp32,
// rank, dims...}, nodes {op, #operands, operands..., #attributes,
// attributes...} (RMSNorm / LayerNorm: epsilon bits; Transpose: first,
// second; Reshape / View: dims). `inputs` holds every input's logical values
// back to back; each declared output's fp64 values are written back to back
// into `out` (capacity `out_len`). Returns the number written, or -1 with
// ref_last_error() set.
long ref_evaluate_graph(int input_count, const int *input_types, int node_count, const int *nodes, int output_count,
                        const int *outputs, const float *inputs, double *out, long out_len) {
  try {
    TensorGraph graph;
    GraphInputs values;
    long at = 0, data = 0;
    for (int i = 0; i < input_count; ++i) {
      const DType dt = input_types[at] == 0 ? DType::Float16 : DType::Float32;
      const int rank = input_types[at + 1];
      at += 2;
      std::vector<std::size_t> shape;
      std::size_t count = 1;
      for (int d = 0; d < rank; ++d) {
        shape.push_back(std::size_t(input_types[at + d]));
        count *= std::size_t(input_types[at + d]);
      }
      at += rank;
      const auto id = graph.addInput("in" + std::to_string(i), TensorType{shape, dt});
      values[id] = std::vector<float>(inputs + data, inputs + data + count);
      data += long(count);
    }
    at = 0;
    for (int i = 0; i < node_count; ++i) {
      const auto op = static_cast<OpType>(nodes[at]);
      const int arity = nodes[at + 1];
      at += 2;
      std::vector<ValueId> operands;
      for (int k = 0; k < arity; ++k) operands.push_back(ValueId(nodes[at + k]));
      at += arity;
      const int nattr = nodes[at++];
      std::vector<int> attrs(nodes + at, nodes + at + nattr);
      at += nattr;
      OpAttributes attributes;
      float eps = 1e-5f;
      if (!attrs.empty() && (op == OpType::RMSNorm || op == OpType::LayerNorm))
        std::memcpy(&eps, &attrs[0], 4);
      if (op == OpType::RMSNorm) attributes = RMSNormAttributes{eps, -1};
      if (op == OpType::LayerNorm) {
        LayerNormAttributes a;
        a.epsilon = eps;
        attributes = a;
      }
      if (op == OpType::Transpose)
        attributes = TransposeAttributes{attrs.size() >= 2 ? attrs[0] : 0, attrs.size() >= 2 ? attrs[1] : 1};
      if (op == OpType::Reshape || op == OpType::View) {
        ReshapeAttributes a;
        for (int d : attrs) a.shape.push_back(std::size_t(d));
        attributes = a;
      }
      graph.addNode(op, operands, attributes);
    }
    for (int i = 0; i < output_count; ++i) graph.outputs.push_back(ValueId(outputs[i]));
    const auto analyzed = analyzer::analyze(graph);
    const auto result = validation::evaluateGraph(analyzed, values);
    long w = 0;
    for (const auto &o : result.outputs) {
      if (w + long(o.size()) > out_len) throw std::runtime_error("output buffer too small");
      std::memcpy(out + w, o.data(), o.size() * sizeof(double));
      w += long(o.size());
    }
    return w;
  } catch (const std::exception &e) {
    g_error = e.what();
    return -1;
  }
}

}  // extern "C"
