// extern "C" graph compilation (GraphCompiler.hpp): a typed tensor graph in,
// its planned regions prepared as catalog kernels and replayed as one CUDA
// graph (declarations and reference citations in include/tmc_cuda.h).
#include <chrono>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "GraphCompiler.hpp"
#include "KernelCatalog.hpp"
#include "api_util.hpp"
#include "tmc_cuda.h"

using namespace tensor::planner;
using tensor::cuda::BufferHandle;
using tensor::cuda::ElementType;
using tensor::cuda::PreparedExecution;
using tensor::cuda::PreparedSequence;

struct tmc_graph {
  tensor::cuda::CudaRuntime *rt = nullptr;
  CompilePlan plan;
  std::size_t inputCount = 0;
  std::vector<std::size_t> outputs;
  std::vector<BufferHandle> buffers;  // per value; aliases share their owner's
  std::vector<std::shared_ptr<PreparedExecution>> steps;
  std::unique_ptr<PreparedSequence> sequence;
};

using namespace tmc_api;

namespace {

std::string parse(int input_count, const int32_t *input_types, size_t input_types_len, const int32_t *nodes,
                  size_t nodes_len, int node_count, const int32_t *outputs, int output_count, CompileGraph *g) {
  if (input_count < 0 || node_count < 0 || output_count <= 0) return "counts must be non-negative, outputs positive";
  if ((input_count > 0 && !input_types) || (node_count > 0 && !nodes) || !outputs) return "null pointer";
  std::size_t at = 0;
  for (int i = 0; i < input_count; ++i) {
    if (at + 2 > input_types_len) return "input type encoding is shorter than input_count types";
    ValueType t;
    t.dtype = input_types[at];
    const int rank = input_types[at + 1];
    at += 2;
    if (rank < 1 || rank > 4 || at + std::size_t(rank) > input_types_len) return "input rank must be 1..4";
    for (int d = 0; d < rank; ++d) {
      if (input_types[at + d] <= 0) return "input dimensions must be positive";
      t.shape.push_back(std::size_t(input_types[at + d]));
    }
    at += std::size_t(rank);
    g->inputTypes.push_back(std::move(t));
  }
  const std::size_t values = std::size_t(input_count) + std::size_t(node_count);
  at = 0;
  for (int i = 0; i < node_count; ++i) {
    if (at + 2 > nodes_len) return "node encoding is shorter than node_count nodes";
    const int op = nodes[at], arity = nodes[at + 1];
    at += 2;
    if (op < 0 || op > static_cast<int>(GraphOp::Gather)) return "unknown op number";
    if (arity < 0 || at + std::size_t(arity) + 1 > nodes_len) return "node encoding is shorter than its operands";
    CompileNode n;
    n.op = static_cast<GraphOp>(op);
    for (int k = 0; k < arity; ++k) {
      const int v = nodes[at + std::size_t(k)];
      if (v < 0 || std::size_t(v) >= values) return "operand is not a graph value";
      n.inputs.push_back(std::size_t(v));
    }
    at += std::size_t(arity);
    const int nattr = nodes[at++];
    if (nattr < 0 || at + std::size_t(nattr) > nodes_len) return "node encoding is shorter than its attributes";
    n.attrs.assign(nodes + at, nodes + at + nattr);
    at += std::size_t(nattr);
    g->nodes.push_back(std::move(n));
  }
  for (int i = 0; i < output_count; ++i) {
    if (outputs[i] < 0 || std::size_t(outputs[i]) >= values) return "graph output is not a graph value";
    g->outputs.push_back(std::size_t(outputs[i]));
  }
  return {};
}

std::string describe(const CompilePlan &plan) {
  std::ostringstream o;
  for (const auto &s : plan.steps) {
    o << s.kernel << "(";
    for (std::size_t i = 0; i < s.inputs.size(); ++i) o << (i ? ", " : "") << "v" << s.inputs[i];
    o << ") -> v" << s.output << " [" << s.region << "]\n";
  }
  return o.str();
}

}  // namespace

extern "C" {

int tmc_graph_plan(int input_count, const int32_t *input_types, size_t input_types_len, const int32_t *nodes,
                   size_t nodes_len, int node_count, const int32_t *outputs, int output_count, char *text,
                   size_t size, size_t *needed) {
  CompileGraph g;
  const std::string bad =
      parse(input_count, input_types, input_types_len, nodes, nodes_len, node_count, outputs, output_count, &g);
  if (!bad.empty()) return fail(TMC_ERR_INVALID, bad);
  const CompilePlan plan = planCompile(g);
  if (!plan.error.empty()) return fail(TMC_ERR_UNSUPPORTED, plan.error);
  const std::string d = describe(plan);
  if (needed) *needed = d.size() + 1;
  if (text && size > 0) {
    const std::size_t n = d.size() < size - 1 ? d.size() : size - 1;
    d.copy(text, n);
    text[n] = '\0';
  }
  return ok();
}

int tmc_graph_compile(tmc_runtime *rt, int input_count, const int32_t *input_types, size_t input_types_len,
                      const int32_t *nodes, size_t nodes_len, int node_count, const int32_t *outputs,
                      int output_count, tmc_graph **out) {
  if (!rt || !out) return fail(TMC_ERR_INVALID, "null runtime or out");
  *out = nullptr;
  CompileGraph g;
  const std::string bad =
      parse(input_count, input_types, input_types_len, nodes, nodes_len, node_count, outputs, output_count, &g);
  if (!bad.empty()) return fail(TMC_ERR_INVALID, bad);
  auto cg = std::make_unique<tmc_graph>();
  cg->rt = rt->rt.get();
  cg->plan = planCompile(g);
  if (!cg->plan.error.empty()) return fail(TMC_ERR_UNSUPPORTED, cg->plan.error);
  cg->inputCount = std::size_t(input_count);
  cg->outputs = g.outputs;
  const auto &types = cg->plan.types;
  cg->buffers.resize(types.size());
  for (std::size_t v = 0; v < types.size(); ++v) {
    if (types[v].owner != v) continue;
    auto r = cg->rt->createBuffer(types[v].elements(), nullptr,
                                  types[v].dtype == kGraphF16 ? ElementType::Float16 : ElementType::Float32);
    if (!r.buffer) return fail(TMC_ERR_OUT_OF_MEMORY, r.errorMessage);
    cg->buffers[v] = r.buffer;
  }
  for (std::size_t v = 0; v < types.size(); ++v) cg->buffers[v] = cg->buffers[types[v].owner];
  std::vector<const PreparedExecution *> raw;
  for (const auto &s : cg->plan.steps) {
    const auto *k = tensor::cuda::findKernel(s.kernel);
    if (!k) return fail(TMC_ERR_UNSUPPORTED, "no catalog kernel " + s.kernel);
    std::vector<BufferHandle> ins;
    for (auto v : s.inputs) ins.push_back(cg->buffers[v]);
    auto r = tensor::cuda::prepareKernel(*cg->rt, *k, ins, {cg->buffers[s.output]},
                                         tensor::cuda::DispatchSize{s.groups, s.threads}, s.constants);
    if (!r.execution) return fail(TMC_ERR_INVALID, s.kernel + ": " + r.errorMessage);
    cg->steps.emplace_back(std::move(r.execution));
    raw.push_back(cg->steps.back().get());
  }
  if (!raw.empty()) {
    auto seq = cg->rt->prepareSequence(raw);
    if (!seq.execution) return fail(TMC_ERR_CUDA, seq.errorMessage);
    cg->sequence = std::move(seq.execution);
  }
  *out = cg.release();
  return ok();
}

void tmc_graph_destroy(tmc_graph *graph) { delete graph; }

int tmc_graph_describe(const tmc_graph *graph, char *text, size_t size, size_t *needed) {
  if (!graph) return fail(TMC_ERR_INVALID, "graph is null");
  const std::string d = describe(graph->plan);
  if (needed) *needed = d.size() + 1;
  if (text && size > 0) {
    const std::size_t n = d.size() < size - 1 ? d.size() : size - 1;
    d.copy(text, n);
    text[n] = '\0';
  }
  return ok();
}

int tmc_graph_value_info(const tmc_graph *graph, int value, int *dtype, int *rank, int64_t *dims, size_t *elements) {
  if (!graph) return fail(TMC_ERR_INVALID, "graph is null");
  if (value < 0 || std::size_t(value) >= graph->plan.types.size()) return fail(TMC_ERR_INVALID, "no such value");
  const auto &t = graph->plan.types[std::size_t(value)];
  if (dtype) *dtype = t.dtype;
  if (rank) *rank = int(t.shape.size());
  if (dims)
    for (std::size_t i = 0; i < t.shape.size(); ++i) dims[i] = int64_t(t.shape[i]);
  if (elements) *elements = t.elements();
  return ok();
}

int tmc_graph_run(tmc_graph *graph, const float *const *inputs, float *const *outputs, double *gpu_us,
                  double *cpu_us) {
  if (!graph || (graph->inputCount > 0 && !inputs) || !outputs) return fail(TMC_ERR_INVALID, "null argument");
  const auto c0 = std::chrono::steady_clock::now();
  for (std::size_t i = 0; i < graph->inputCount; ++i) {
    if (!inputs[i]) return fail(TMC_ERR_INVALID, "null input " + std::to_string(i));
    const std::string e = graph->rt->writeBuffer(graph->buffers[i], inputs[i], graph->plan.types[i].elements());
    if (!e.empty()) return fail(TMC_ERR_CUDA, e);
  }
  double gpu = 0.0;
  if (graph->sequence) {
    const auto r = graph->sequence->execute();
    if (!r.executionPassed) {
      const bool device = r.errorMessage.rfind("device status", 0) == 0;
      return fail(device ? TMC_ERR_DEVICE_STATUS : TMC_ERR_CUDA, r.errorMessage);
    }
    gpu = r.gpuExecutionTimeUs ? *r.gpuExecutionTimeUs : 0.0;
  }
  for (std::size_t i = 0; i < graph->outputs.size(); ++i) {
    if (!outputs[i]) return fail(TMC_ERR_INVALID, "null output " + std::to_string(i));
    const std::size_t v = graph->outputs[i];
    const auto values = graph->buffers[v]->read();
    std::copy(values.begin(), values.begin() + graph->plan.types[v].elements(), outputs[i]);
  }
  if (gpu_us) *gpu_us = gpu;
  if (cpu_us) *cpu_us = std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - c0).count();
  return ok();
}

int tmc_graph_input_buffer(tmc_graph *graph, int input, tmc_buffer **out) {
  if (!graph || !out) return fail(TMC_ERR_INVALID, "null argument");
  if (input < 0 || std::size_t(input) >= graph->inputCount) return fail(TMC_ERR_INVALID, "no such input");
  *out = new tmc_buffer{graph->buffers[std::size_t(input)], graph->rt};
  return ok();
}

int tmc_graph_launch(tmc_graph *graph, int replays) {
  if (!graph || replays < 0) return fail(TMC_ERR_INVALID, "null graph or negative replays");
  if (!graph->sequence) return ok();
  cudaSetDevice(graph->rt->device());
  for (int i = 0; i < replays; ++i) {
    const cudaError_t e = cudaGraphLaunch(graph->sequence->graph(), graph->rt->stream());
    if (e != cudaSuccess) return cuda_fail(e, "cudaGraphLaunch");
  }
  return ok();
}

}  // extern "C"
