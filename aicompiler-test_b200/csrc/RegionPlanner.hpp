// Region planning for tensor graphs: which nodes run as one fused kernel.
// The counterpart of the reference's formRegions (src/analyzer/PatternAnalyzer.cpp:32-132)
// and of the topological order analyze() computes (src/analyzer/GraphAnalyzer.cpp:278-364),
// written against an already-typed graph: the caller supplies, per value,
// whether its storage is contiguous (views such as Transpose are not).
//
// Fusions, tried in this order at each node not yet placed (node order is the
// topological order; ready nodes leave in FIFO order, node index breaking
// ties):
//   * Linear + ReLU:      MatMul -> Add -> ReLU
//   * Add + RMSNorm / Add + LayerNorm: Add -> norm, the sum being the norm's data
//     (first) operand
//   * SiLU + Mul:         SiLU -> Mul, the activation on either side of the Mul.
// An edge inside a fusion must be exclusive: the producer's result has exactly
// that one use (a node reading a value twice counts twice), it is not a graph
// output, and the producer is not a view. Every operand of every fused node
// must be contiguous, or the seed node stays alone. A region's inputs are the
// operands produced outside it; its outputs are the results used outside it or
// declared graph outputs (at least the last node's result); a fused region
// must have exactly one output. These rules are the reference's, so a graph
// splits into the same regions, and each fused region maps onto one kernel of
// this library (tmc_k_fused_add_norm, tmc_k_fused_silu_mul,
// tmc_k_fused_linear_relu).
#pragma once

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <deque>
#include <limits>
#include <string>
#include <vector>

namespace tensor::planner {

// Operation kinds, numbered as the reference's tensor::OpType.
enum class GraphOp : int {
  Add, Mul, MatMul, RMSNorm, LayerNorm, ReLU, SiLU, Softmax, RoPE,
  ReduceSum, ReduceMean, Reshape, View, Transpose, Contiguous,
  MaskedFill, Slice, Embedding, Gather
};

inline bool isViewOp(GraphOp op) {
  return op == GraphOp::Reshape || op == GraphOp::View || op == GraphOp::Transpose;
}

struct PlanNode {
  GraphOp op = GraphOp::Add;
  std::vector<std::size_t> inputs;   // value ids
  std::vector<std::size_t> outputs;  // value ids
};

struct PlanGraph {
  std::size_t valueCount = 0;
  std::vector<std::size_t> inputs;   // graph inputs (value ids)
  std::vector<PlanNode> nodes;
  std::vector<std::size_t> outputs;  // declared graph outputs
  std::vector<bool> contiguous;      // per value
};

enum class RegionKind : int { Single = 0, AddRMSNorm, AddLayerNorm, SiLUMul, LinearReLU };

struct PlannedRegion {
  RegionKind kind = RegionKind::Single;
  std::vector<std::size_t> nodes;    // node indices, producer first
  std::vector<std::size_t> inputs;   // value ids entering the region
  std::vector<std::size_t> outputs;  // value ids leaving it
};

struct RegionPlan {
  std::vector<std::size_t> order;    // topological node order
  std::vector<PlannedRegion> regions;
  std::string error;                 // empty when the plan is valid
};

namespace region_detail {

constexpr std::size_t kNone = std::numeric_limits<std::size_t>::max();

template <class T>
bool has(const std::vector<T> &v, const T &x) {
  return std::find(v.begin(), v.end(), x) != v.end();
}

template <class T>
void addOnce(std::vector<T> &v, const T &x) {
  if (!has(v, x)) v.push_back(x);
}

struct Tables {
  std::vector<std::size_t> producer;               // value -> node (kNone for graph inputs)
  std::vector<std::vector<std::size_t>> uses;      // value -> consuming node, once per operand slot
};

inline Tables buildTables(const PlanGraph &g) {
  Tables t;
  t.producer.assign(g.valueCount, kNone);
  t.uses.assign(g.valueCount, {});
  for (std::size_t n = 0; n < g.nodes.size(); ++n) {
    for (auto v : g.nodes[n].outputs) t.producer[v] = n;
    for (auto v : g.nodes[n].inputs) t.uses[v].push_back(n);
  }
  return t;
}

// Kahn's algorithm: a node is ready when every operand produced by a node has
// been produced (an operand read twice is waited for twice); ready nodes leave
// in FIFO order, the initial ones by index.
inline std::vector<std::size_t> topologicalOrder(const PlanGraph &g, const Tables &t, std::string *error) {
  const std::size_t n = g.nodes.size();
  std::vector<std::size_t> pending(n, 0);
  std::vector<std::vector<std::size_t>> wakes(n);
  for (std::size_t i = 0; i < n; ++i)
    for (auto v : g.nodes[i].inputs)
      if (t.producer[v] != kNone) {
        ++pending[i];
        wakes[t.producer[v]].push_back(i);
      }
  std::deque<std::size_t> ready;
  for (std::size_t i = 0; i < n; ++i)
    if (pending[i] == 0) ready.push_back(i);
  std::vector<std::size_t> order;
  while (!ready.empty()) {
    const auto i = ready.front();
    ready.pop_front();
    order.push_back(i);
    for (auto next : wakes[i])
      if (--pending[next] == 0) ready.push_back(next);
  }
  if (order.size() != n) *error = "Tensor graph contains a dependency cycle.";
  return order;
}

}  // namespace region_detail

inline RegionPlan planRegions(const PlanGraph &g) {
  using namespace region_detail;
  RegionPlan plan;
  if (g.contiguous.size() != g.valueCount) {
    plan.error = "Region planning needs the contiguity of every value.";
    return plan;
  }
  for (const auto &node : g.nodes) {
    if (node.outputs.empty()) {
      plan.error = "Graph node has no results.";
      return plan;
    }
    for (auto v : node.inputs)
      if (v >= g.valueCount) plan.error = "Invalid graph ValueId.";
    for (auto v : node.outputs)
      if (v >= g.valueCount) plan.error = "Invalid graph ValueId.";
  }
  if (!plan.error.empty()) return plan;
  const Tables t = buildTables(g);
  plan.order = topologicalOrder(g, t, &plan.error);
  if (!plan.error.empty()) return plan;

  std::vector<bool> placed(g.nodes.size(), false);
  // The single result of `node`, if it has exactly one result with one use.
  auto soleUse = [&](std::size_t node) -> std::size_t {
    const auto &outs = g.nodes[node].outputs;
    if (outs.size() != 1 || t.uses[outs[0]].size() != 1) return kNone;
    return t.uses[outs[0]].front();
  };
  // `value` may stay inside a region that also holds its only consumer `into`.
  auto internal = [&](std::size_t value, std::size_t into) {
    return t.uses[value].size() == 1 && t.uses[value].front() == into && !has(g.outputs, value) &&
           !isViewOp(g.nodes[t.producer[value]].op);
  };
  auto free = [&](std::size_t node) { return node != kNone && !placed[node]; };

  // Each matcher returns the fused chain starting at `seed`, or nothing.
  auto linearRelu = [&](std::size_t seed) -> std::vector<std::size_t> {
    if (g.nodes[seed].op != GraphOp::MatMul) return {};
    const auto add = soleUse(seed);
    if (!free(add) || g.nodes[add].op != GraphOp::Add || !internal(g.nodes[seed].outputs[0], add)) return {};
    const auto relu = soleUse(add);
    if (!free(relu) || g.nodes[relu].op != GraphOp::ReLU || !internal(g.nodes[add].outputs[0], relu)) return {};
    return {seed, add, relu};
  };
  auto addNorm = [&](std::size_t seed, RegionKind *kind) -> std::vector<std::size_t> {
    if (g.nodes[seed].op != GraphOp::Add) return {};
    const auto norm = soleUse(seed);
    if (!free(norm)) return {};
    const auto &nn = g.nodes[norm];
    if (nn.op != GraphOp::RMSNorm && nn.op != GraphOp::LayerNorm) return {};
    const auto sum = g.nodes[seed].outputs[0];
    if (!internal(sum, norm) || nn.inputs.empty() || nn.inputs.front() != sum) return {};
    *kind = nn.op == GraphOp::RMSNorm ? RegionKind::AddRMSNorm : RegionKind::AddLayerNorm;
    return {seed, norm};
  };
  auto siluMul = [&](std::size_t seed) -> std::vector<std::size_t> {
    if (g.nodes[seed].op != GraphOp::SiLU) return {};
    const auto mul = soleUse(seed);
    if (!free(mul) || g.nodes[mul].op != GraphOp::Mul || !internal(g.nodes[seed].outputs[0], mul)) return {};
    return {seed, mul};
  };

  for (auto seed : plan.order) {
    if (placed[seed]) continue;
    PlannedRegion r;
    RegionKind kind = RegionKind::Single;
    std::vector<std::size_t> chain = linearRelu(seed);
    if (!chain.empty()) kind = RegionKind::LinearReLU;
    if (chain.empty()) chain = addNorm(seed, &kind);
    if (chain.empty() && !(chain = siluMul(seed)).empty()) kind = RegionKind::SiLUMul;
    bool contiguousOperands = true;
    for (auto node : chain)
      for (auto v : g.nodes[node].inputs) contiguousOperands = contiguousOperands && g.contiguous[v];
    if (chain.empty() || !contiguousOperands) {
      chain.assign(1, seed);
      kind = RegionKind::Single;
    }
    r.kind = kind;
    r.nodes = chain;
    for (auto node : chain) placed[node] = true;
    for (auto node : chain)
      for (auto v : g.nodes[node].inputs)
        if (t.producer[v] == kNone || !has(chain, t.producer[v])) addOnce(r.inputs, v);
    for (auto node : chain)
      for (auto v : g.nodes[node].outputs) {
        bool leaves = has(g.outputs, v);
        for (auto user : t.uses[v]) leaves = leaves || !has(chain, user);
        if (leaves) addOnce(r.outputs, v);
      }
    if (r.outputs.empty()) r.outputs.push_back(g.nodes[chain.back()].outputs.front());
    if (kind != RegionKind::Single && r.outputs.size() != 1) {
      plan.error = "A fused region must have one external result.";
      return plan;
    }
    plan.regions.push_back(std::move(r));
  }
  return plan;
}

// Buffers and launches of a graph, as the reference's planGraph decides them
// (src/planner/KernelPlan.cpp:11-59): every value is a graph input, a declared
// output or an intermediate (an input that is also an output stays an input); a
// view's result aliases the view's data operand; every node that is not a view
// launches a kernel, in topological order. (The reference's per-launch
// threadgroup sizes are Metal dispatch geometry; this library's launchers choose
// their own grids.)
enum class BufferRole : int { Input = 0, Intermediate, Output };

struct BufferPlan {
  std::vector<BufferRole> roles;        // per value
  std::vector<std::size_t> aliasOf;     // per value; region_detail::kNone when it owns storage
  std::vector<std::size_t> launches;    // node indices, topological order
  std::string error;
};

inline BufferPlan planBuffers(const PlanGraph &g) {
  using namespace region_detail;
  BufferPlan plan;
  for (const auto &node : g.nodes) {
    if (node.outputs.empty()) plan.error = "Graph node has no results.";
    for (auto v : node.inputs)
      if (v >= g.valueCount) plan.error = "Invalid graph ValueId.";
    for (auto v : node.outputs)
      if (v >= g.valueCount) plan.error = "Invalid graph ValueId.";
  }
  if (!plan.error.empty()) return plan;
  const Tables t = buildTables(g);
  const auto order = topologicalOrder(g, t, &plan.error);
  if (!plan.error.empty()) return plan;
  plan.roles.assign(g.valueCount, BufferRole::Intermediate);
  plan.aliasOf.assign(g.valueCount, kNone);
  for (std::size_t v = 0; v < g.valueCount; ++v) {
    if (has(g.inputs, v)) plan.roles[v] = BufferRole::Input;
    else if (has(g.outputs, v)) plan.roles[v] = BufferRole::Output;
  }
  for (auto n : order) {
    const auto &node = g.nodes[n];
    if (isViewOp(node.op)) {
      if (!node.inputs.empty()) plan.aliasOf[node.outputs.front()] = node.inputs.front();
    } else {
      plan.launches.push_back(n);
    }
  }
  return plan;
}

inline const char *regionKindName(RegionKind kind) {
  switch (kind) {
    case RegionKind::Single: return "Unfused";
    case RegionKind::AddRMSNorm: return "Add + RMSNorm";
    case RegionKind::AddLayerNorm: return "Residual Add + LayerNorm";
    case RegionKind::SiLUMul: return "SiLU + Mul";
    case RegionKind::LinearReLU: return "Linear + ReLU";
  }
  return "?";
}

}  // namespace tensor::planner
