// C-ABI entry of the region planner (RegionPlanner.hpp): which nodes of a typed
// tensor graph run as one fused kernel.
#include <cstddef>
#include <cstdint>
#include <string>

#include "RegionPlanner.hpp"
#include "api_util.hpp"
#include "tmc_cuda.h"

using namespace tensor::planner;

namespace {

// Parses the flat graph encoding shared by the planner entry points; returns ""
// or why the encoding is refused.
std::string parseGraph(int input_count, const int32_t *nodes, size_t nodes_len, int node_count,
                       const int32_t *outputs, int output_count, PlanGraph *g) {
  if (input_count < 0 || node_count < 0 || output_count < 0) return "negative count";
  if ((node_count > 0 && !nodes) || (output_count > 0 && !outputs)) return "null pointer";
  g->valueCount = std::size_t(input_count) + std::size_t(node_count);
  for (int i = 0; i < input_count; ++i) g->inputs.push_back(std::size_t(i));
  std::size_t at = 0;
  for (int i = 0; i < node_count; ++i) {
    if (at + 2 > nodes_len) return "node encoding is shorter than node_count nodes";
    const int op = nodes[at], arity = nodes[at + 1];
    at += 2;
    if (op < 0 || op > static_cast<int>(GraphOp::Gather)) return "unknown op number";
    if (arity < 0 || at + std::size_t(arity) > nodes_len) return "node encoding is shorter than its operand counts";
    PlanNode n;
    n.op = static_cast<GraphOp>(op);
    for (int k = 0; k < arity; ++k) {
      const int v = nodes[at + std::size_t(k)];
      if (v < 0 || std::size_t(v) >= g->valueCount) return "operand is not a graph value";
      n.inputs.push_back(std::size_t(v));
    }
    at += std::size_t(arity);
    n.outputs.push_back(std::size_t(input_count) + std::size_t(i));
    g->nodes.push_back(std::move(n));
  }
  for (int i = 0; i < output_count; ++i) {
    if (outputs[i] < 0 || std::size_t(outputs[i]) >= g->valueCount) return "graph output is not a graph value";
    g->outputs.push_back(std::size_t(outputs[i]));
  }
  return {};
}

}  // namespace

extern "C" int tmc_plan_regions(int input_count, const int32_t *nodes, size_t nodes_len, int node_count,
                                const int32_t *outputs, int output_count, const int32_t *contiguous,
                                int32_t *order, int32_t *regions, size_t capacity, size_t *written) {
  using namespace tmc_api;
  if ((node_count > 0 && !order) || !contiguous || !written || (capacity > 0 && !regions))
    return fail(TMC_ERR_INVALID, "null pointer");
  PlanGraph g;
  const std::string bad = parseGraph(input_count, nodes, nodes_len, node_count, outputs, output_count, &g);
  if (!bad.empty()) return fail(TMC_ERR_INVALID, bad);
  for (std::size_t v = 0; v < g.valueCount; ++v) g.contiguous.push_back(contiguous[v] != 0);
  const RegionPlan plan = planRegions(g);
  if (!plan.error.empty()) return fail(TMC_ERR_INVALID, plan.error);
  for (std::size_t i = 0; i < plan.order.size(); ++i) order[i] = int32_t(plan.order[i]);
  std::size_t w = 0;
  auto put = [&](std::size_t value) {
    if (w < capacity) regions[w] = int32_t(value);
    ++w;
  };
  for (const auto &r : plan.regions) {
    put(std::size_t(r.kind));
    put(r.nodes.size());
    for (auto x : r.nodes) put(x);
    put(r.inputs.size());
    for (auto x : r.inputs) put(x);
    put(r.outputs.size());
    for (auto x : r.outputs) put(x);
  }
  *written = w;
  if (w > capacity) return fail(TMC_ERR_INVALID, "regions buffer too small: " + std::to_string(w) + " ints needed");
  return ok();
}

extern "C" int tmc_plan_buffers(int input_count, const int32_t *nodes, size_t nodes_len, int node_count,
                                const int32_t *outputs, int output_count, int32_t *roles, int32_t *alias_of,
                                int32_t *launches, int *launch_count) {
  using namespace tmc_api;
  const std::size_t values = std::size_t(input_count < 0 ? 0 : input_count) + std::size_t(node_count < 0 ? 0 : node_count);
  if ((values > 0 && (!roles || !alias_of)) || (node_count > 0 && !launches) || !launch_count)
    return fail(TMC_ERR_INVALID, "null pointer");
  PlanGraph g;
  const std::string bad = parseGraph(input_count, nodes, nodes_len, node_count, outputs, output_count, &g);
  if (!bad.empty()) return fail(TMC_ERR_INVALID, bad);
  const BufferPlan plan = planBuffers(g);
  if (!plan.error.empty()) return fail(TMC_ERR_INVALID, plan.error);
  for (std::size_t v = 0; v < g.valueCount; ++v) {
    roles[v] = int32_t(plan.roles[v]);
    alias_of[v] = plan.aliasOf[v] == region_detail::kNone ? -1 : int32_t(plan.aliasOf[v]);
  }
  for (std::size_t i = 0; i < plan.launches.size(); ++i) launches[i] = int32_t(plan.launches[i]);
  *launch_count = int(plan.launches.size());
  return ok();
}
