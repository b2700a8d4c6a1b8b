// Graph compilation for the TensorGraph path: the counterpart of the
// reference's compileGraph (src/runtime/GraphExecutor.cpp:346-431), which
// analyzes a typed graph (analyze, src/analyzer/GraphAnalyzer.cpp:278-364),
// plans its buffers and regions (planGraph / planRegions, KernelPlan.cpp:11-59,
// RegionPlan.cpp:8-29) and prepares one execution per region.
//
// planCompile is host-only: it infers every value's type (shape, storage
// type, contiguity; views alias their data operand), forms the fused regions
// exactly as formRegions does (RegionPlanner.hpp), and picks one kernel of
// this library's catalog (KernelCatalog.hpp) per region:
//   Add + RMSNorm / Add + LayerNorm  -> fused_add_rmsnorm / fused_add_layernorm
//   SiLU + Mul                        -> fused_silu_mul
//   MatMul + Add + ReLU               -> fused_linear_relu
//   RMSNorm feeding only a MatMul with a Transpose view of an fp16 [N, K]
//     weight, fp32 rows <= 4          -> rmsnorm_gemv_f32 (the norm runs in the
//                                        GEMV's prologue; no intermediate)
//   RMSNorm                           -> rmsnorm
//   MatMul, fp16 rows <= 8 against a Transpose view of an fp16 [N, K] weight
//                                     -> gemv_f16
//   MatMul otherwise                  -> matmul
//   Add / Mul / ReLU / SiLU           -> add / mul / relu / silu
//   Transpose / Reshape / View        -> no launch (an alias)
// The remaining reference ops (Softmax, RoPE, reductions, Contiguous,
// MaskedFill, Slice, Embedding, Gather) have no graph kernel here and are
// refused with a message naming the op. Storage types are the reference's
// (all operands of a node share one floating type, GraphAnalyzer.cpp:74),
// with one extension: a MatMul's right-hand operand may be fp16 under an fp32
// left-hand side, so weights can stay in fp16 (the C1 graph with an fp16 W).
#pragma once

#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "RegionPlanner.hpp"

namespace tensor::planner {

enum GraphDType : int { kGraphF16 = 0, kGraphF32 = 1 };  // TMC_F16 / TMC_F32

struct ValueType {
  int dtype = kGraphF32;
  std::vector<std::size_t> shape;
  std::vector<std::size_t> strides;  // elements
  std::size_t owner = 0;             // value whose storage this one uses
  bool transposed2d = false;         // a 2-D Transpose view of its owner
  std::size_t elements() const {
    std::size_t n = 1;
    for (auto d : shape) n *= d;
    return n;
  }
  bool contiguous() const {
    std::size_t expect = 1;
    for (std::size_t i = shape.size(); i-- > 0;) {
      if (shape[i] != 1 && strides[i] != expect) return false;
      expect *= shape[i];
    }
    return true;
  }
};

struct CompileNode {
  GraphOp op = GraphOp::Add;
  std::vector<std::size_t> inputs;
  std::vector<std::int32_t> attrs;  // RMSNorm / LayerNorm: [eps bits]; Transpose: [first, second]; Reshape / View: dims
};

struct CompileGraph {
  std::vector<ValueType> inputTypes;  // shape + dtype of each graph input
  std::vector<CompileNode> nodes;     // node i defines value inputs + i
  std::vector<std::size_t> outputs;
};

struct LaunchStep {
  std::string kernel;                  // catalog name
  std::vector<std::size_t> inputs;     // storage-owning values, binding order
  std::size_t output = 0;              // storage-owning value
  std::vector<std::uint32_t> constants;
  std::size_t groups = 1, threads = 256;
  std::string region;                  // which region (kind name) it implements
  std::vector<std::size_t> nodes;      // graph nodes it covers
};

struct CompilePlan {
  std::vector<ValueType> types;        // every value
  std::vector<LaunchStep> steps;       // in execution order
  std::string error;
};

namespace compile_detail {

inline std::uint32_t floatBits(float f) {
  std::uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
}

inline ValueType dense(std::vector<std::size_t> shape, int dtype, std::size_t owner) {
  ValueType t;
  t.dtype = dtype;
  t.shape = std::move(shape);
  t.strides.assign(t.shape.size(), 1);
  for (std::size_t i = t.shape.size(); i-- > 1;) t.strides[i - 1] = t.strides[i] * t.shape[i];
  t.owner = owner;
  return t;
}

inline const char *opName(GraphOp op) {
  static const char *names[] = {"Add", "Mul", "MatMul", "RMSNorm", "LayerNorm", "ReLU", "SiLU", "Softmax", "RoPE",
                                "ReduceSum", "ReduceMean", "Reshape", "View", "Transpose", "Contiguous",
                                "MaskedFill", "Slice", "Embedding", "Gather"};
  return names[static_cast<int>(op)];
}

// [rows, width] view of a tensor whose last axis is the width.
inline void rowsWidth(const ValueType &t, std::size_t *rows, std::size_t *width) {
  *width = t.shape.empty() ? 1 : t.shape.back();
  *rows = *width == 0 ? 0 : t.elements() / *width;
}

// b broadcast over rows of x: b has x's shape, or is [width] / [1, width].
inline bool rowBroadcast(const ValueType &x, const ValueType &b, std::size_t *bRows) {
  std::size_t rows, width, br, bw;
  rowsWidth(x, &rows, &width);
  rowsWidth(b, &br, &bw);
  if (bw != width) return false;
  if (b.shape == x.shape) {
    *bRows = rows;
    return true;
  }
  if (br == 1) {
    *bRows = 1;
    return true;
  }
  return false;
}

inline float attrEps(const CompileNode &n) {
  if (n.attrs.empty()) return 1e-5f;
  float f;
  const std::uint32_t u = static_cast<std::uint32_t>(n.attrs[0]);
  std::memcpy(&f, &u, 4);
  return f;
}

// Type of node n's result (value id `self`), or an error.
inline std::string infer(const CompileNode &n, const std::vector<ValueType> &types, std::size_t self, ValueType *out) {
  auto arity = [&](std::size_t k) -> std::string {
    if (n.inputs.size() != k) return std::string(opName(n.op)) + ": invalid input count.";
    return {};
  };
  std::string e;
  const ValueType &a = types.at(n.inputs.empty() ? 0 : n.inputs[0]);
  switch (n.op) {
    case GraphOp::Add:
    case GraphOp::Mul: {
      if (!(e = arity(2)).empty()) return e;
      const ValueType &b = types[n.inputs[1]];
      if (a.dtype != b.dtype) return std::string(opName(n.op)) + " requires matching floating-point dtypes.";
      std::size_t br;
      const ValueType &big = a.elements() >= b.elements() ? a : b;
      const ValueType &small = a.elements() >= b.elements() ? b : a;
      if (!rowBroadcast(big, small, &br))
        return std::string(opName(n.op)) + ": only equal shapes or a broadcast last-axis row are supported.";
      *out = dense(big.shape, a.dtype, self);
      return {};
    }
    case GraphOp::ReLU:
    case GraphOp::SiLU:
      if (!(e = arity(1)).empty()) return e;
      *out = dense(a.shape, a.dtype, self);
      return {};
    case GraphOp::MatMul: {
      if (!(e = arity(2)).empty()) return e;
      const ValueType &b = types[n.inputs[1]];
      if (a.dtype != b.dtype && !(a.dtype == kGraphF32 && b.dtype == kGraphF16))
        return "MatMul requires matching floating-point dtypes (or an fp16 right-hand operand under fp32).";
      if (a.shape.size() != 2 || b.shape.size() != 2 || a.shape[1] != b.shape[0])
        return "MatMul requires [M, K] and [K, N] (two-dimensional operands here).";
      *out = dense({a.shape[0], b.shape[1]}, a.dtype, self);
      return {};
    }
    case GraphOp::RMSNorm: {
      if (!(e = arity(2)).empty()) return e;
      const ValueType &w = types[n.inputs[1]];
      if (a.shape.empty() || w.shape.size() != 1 || w.shape[0] != a.shape.back() || w.dtype != a.dtype)
        return "RMSNorm weight must match the normalized (last) axis and dtype.";
      if (!(attrEps(n) > 0.0f)) return "RMSNorm epsilon must be finite and positive.";
      *out = dense(a.shape, a.dtype, self);
      return {};
    }
    case GraphOp::LayerNorm: {
      if (!(e = arity(3)).empty()) return e;
      const ValueType &w = types[n.inputs[1]], &c = types[n.inputs[2]];
      if (a.shape.empty() || w.shape.size() != 1 || c.shape.size() != 1 || w.shape[0] != a.shape.back() ||
          c.shape[0] != a.shape.back() || w.dtype != a.dtype || c.dtype != a.dtype)
        return "LayerNorm weight and bias must match normalized axes.";
      if (!(attrEps(n) > 0.0f)) return "LayerNorm epsilon must be finite and positive.";
      *out = dense(a.shape, a.dtype, self);
      return {};
    }
    case GraphOp::Transpose: {
      if (!(e = arity(1)).empty()) return e;
      const int first = n.attrs.size() >= 2 ? n.attrs[0] : 0, second = n.attrs.size() >= 2 ? n.attrs[1] : 1;
      if (a.shape.size() != 2 || !((first == 0 && second == 1) || (first == 1 && second == 0)) || !a.contiguous())
        return "Transpose: only the 2-D swap of a contiguous tensor is supported.";
      ValueType t = a;
      std::swap(t.shape[0], t.shape[1]);
      std::swap(t.strides[0], t.strides[1]);
      t.transposed2d = true;
      *out = t;  // aliases a's storage (owner unchanged)
      return {};
    }
    case GraphOp::Reshape:
    case GraphOp::View: {
      if (!(e = arity(1)).empty()) return e;
      std::vector<std::size_t> shape;
      for (auto d : n.attrs) {
        if (d <= 0) return std::string(opName(n.op)) + ": dimensions must be positive.";
        shape.push_back(static_cast<std::size_t>(d));
      }
      ValueType t = dense(shape, a.dtype, a.owner);
      if (t.elements() != a.elements()) return std::string(opName(n.op)) + " must preserve the element count.";
      if (!a.contiguous()) return std::string(opName(n.op)) + " of a non-contiguous view is not supported.";
      *out = t;
      return {};
    }
    default:
      return std::string(opName(n.op)) + " has no graph kernel in this backend.";
  }
}

}  // namespace compile_detail

inline CompilePlan planCompile(const CompileGraph &cg) {
  using namespace compile_detail;
  CompilePlan plan;
  const std::size_t nin = cg.inputTypes.size();
  const std::size_t values = nin + cg.nodes.size();
  // Structure first (cycles, operand ids), with the reference planner's rules.
  PlanGraph g;
  g.valueCount = values;
  for (std::size_t i = 0; i < nin; ++i) g.inputs.push_back(i);
  for (std::size_t i = 0; i < cg.nodes.size(); ++i) {
    PlanNode pn;
    pn.op = cg.nodes[i].op;
    pn.inputs = cg.nodes[i].inputs;
    for (auto v : pn.inputs)
      if (v >= values) {
        plan.error = "Invalid graph ValueId.";
        return plan;
      }
    pn.outputs = {nin + i};
    g.nodes.push_back(std::move(pn));
  }
  g.outputs = cg.outputs;
  for (auto v : g.outputs)
    if (v >= values) {
      plan.error = "Invalid graph ValueId.";
      return plan;
    }
  region_detail::Tables tables = region_detail::buildTables(g);
  const auto order = region_detail::topologicalOrder(g, tables, &plan.error);
  if (!plan.error.empty()) return plan;
  // Types in topological order.
  plan.types.resize(values);
  for (std::size_t i = 0; i < nin; ++i) {
    const ValueType &t = cg.inputTypes[i];
    if (t.dtype != kGraphF16 && t.dtype != kGraphF32) {
      plan.error = "Graph inputs must be fp16 or fp32 (the graph kernels' storage types).";
      return plan;
    }
    plan.types[i] = dense(t.shape, t.dtype, i);
    if (plan.types[i].elements() == 0) {
      plan.error = "Graph inputs must have a positive element count.";
      return plan;
    }
  }
  for (auto n : order) {
    const std::string e = infer(cg.nodes[n], plan.types, nin + n, &plan.types[nin + n]);
    if (!e.empty()) {
      plan.error = e;
      return plan;
    }
  }
  for (auto v : cg.outputs)
    if (!plan.types[v].contiguous()) {
      plan.error = "A graph output must not be a strided view (read it through a kernel first).";
      return plan;
    }
  g.contiguous.resize(values);
  for (std::size_t v = 0; v < values; ++v) g.contiguous[v] = plan.types[v].contiguous();
  const RegionPlan regions = planRegions(g);
  if (!regions.error.empty()) {
    plan.error = regions.error;
    return plan;
  }
  auto own = [&](std::size_t v) { return plan.types[v].owner; };
  auto isOutput = [&](std::size_t v) { return region_detail::has(cg.outputs, v); };
  std::vector<bool> covered(cg.nodes.size(), false);
  auto rw = [&](std::size_t v, std::size_t *rows, std::size_t *width) { rowsWidth(plan.types[v], rows, width); };

  for (const auto &r : regions.regions) {
    const CompileNode &head = cg.nodes[r.nodes.front()];
    const std::size_t out = nin + r.nodes.back();
    LaunchStep s;
    s.region = regionKindName(r.kind);
    s.nodes = r.nodes;
    if (r.kind == RegionKind::AddRMSNorm || r.kind == RegionKind::AddLayerNorm) {
      const CompileNode &norm = cg.nodes[r.nodes[1]];
      std::size_t x = head.inputs[0], b = head.inputs[1];
      if (plan.types[x].elements() < plan.types[b].elements()) std::swap(x, b);
      std::size_t rows, width, brows = 1;
      rw(x, &rows, &width);
      rowBroadcast(plan.types[x], plan.types[b], &brows);
      s.kernel = r.kind == RegionKind::AddRMSNorm ? "fused_add_rmsnorm" : "fused_add_layernorm";
      s.inputs = {own(x), own(b), own(norm.inputs[1])};
      if (r.kind == RegionKind::AddLayerNorm) s.inputs.push_back(own(norm.inputs[2]));
      s.constants = {(std::uint32_t)rows, (std::uint32_t)width, (std::uint32_t)brows, floatBits(attrEps(norm))};
    } else if (r.kind == RegionKind::SiLUMul) {
      const CompileNode &mul = cg.nodes[r.nodes[1]];
      const std::size_t act = nin + r.nodes[0];
      const std::size_t x = head.inputs[0];
      const std::size_t b = mul.inputs[0] == act ? mul.inputs[1] : mul.inputs[0];
      std::size_t rows, width, brows = 1;
      rw(out, &rows, &width);
      if (!rowBroadcast(plan.types[out], plan.types[b], &brows) || plan.types[x].elements() != rows * width) {
        plan.error = "SiLU + Mul: the activation must have the product's shape.";
        return plan;
      }
      s.kernel = "fused_silu_mul";
      s.inputs = {own(x), own(b)};
      s.constants = {(std::uint32_t)rows, (std::uint32_t)width, (std::uint32_t)brows};
    } else if (r.kind == RegionKind::LinearReLU) {
      const CompileNode &add = cg.nodes[r.nodes[1]];
      const std::size_t lin = nin + r.nodes[0];
      const std::size_t bias = add.inputs[0] == lin ? add.inputs[1] : add.inputs[0];
      const ValueType &a = plan.types[head.inputs[0]], &w = plan.types[head.inputs[1]];
      if (a.dtype != w.dtype || plan.types[bias].shape.size() != 1 || plan.types[bias].shape[0] != w.shape[1]) {
        plan.error = "Linear + ReLU: the bias must be one row of the output width, all operands one dtype.";
        return plan;
      }
      s.kernel = "fused_linear_relu";
      s.inputs = {own(head.inputs[0]), own(head.inputs[1]), own(bias)};
      s.constants = {(std::uint32_t)a.shape[0], (std::uint32_t)a.shape[1], (std::uint32_t)w.shape[1]};
    } else {
      const std::size_t node = r.nodes.front();
      switch (head.op) {
        case GraphOp::Transpose:
        case GraphOp::Reshape:
        case GraphOp::View:
          continue;  // an alias: no launch
        case GraphOp::RMSNorm: {
          // Fold into the next GEMV when that is its only use (and it is not
          // a graph output): the B200 decode kernel's RMSNorm prologue.
          const auto &uses = tables.uses[out];
          if (!isOutput(out) && uses.size() == 1 && cg.nodes[uses[0]].op == GraphOp::MatMul &&
              cg.nodes[uses[0]].inputs[0] == out) {
            const std::size_t rhs = cg.nodes[uses[0]].inputs[1];
            const ValueType &x = plan.types[head.inputs[0]], &w = plan.types[rhs];
            if (x.dtype == kGraphF32 && x.shape.size() == 2 && x.shape[0] <= 4 && x.shape[1] % 8 == 0 &&
                w.transposed2d && plan.types[own(rhs)].dtype == kGraphF16 &&
                plan.types[head.inputs[1]].dtype == kGraphF32) {
              covered[node] = true;  // emitted with the MatMul below
              continue;
            }
          }
          std::size_t rows, width;
          rw(out, &rows, &width);
          s.kernel = "rmsnorm";
          s.inputs = {own(head.inputs[0]), own(head.inputs[1])};
          s.constants = {(std::uint32_t)rows, (std::uint32_t)width, floatBits(attrEps(head))};
          s.groups = rows;
          s.threads = 256;
          break;
        }
        case GraphOp::MatMul: {
          const std::size_t lhs = head.inputs[0], rhs = head.inputs[1];
          const ValueType &a = plan.types[lhs], &w = plan.types[rhs];
          const std::size_t m = a.shape[0], k = a.shape[1], n = w.shape[1];
          if (!a.contiguous()) {
            plan.error = "MatMul: the left-hand operand must be contiguous.";
            return plan;
          }
          const bool lhsFolded = lhs >= nin && covered[lhs - nin];
          if (lhsFolded) {
            const CompileNode &norm = cg.nodes[lhs - nin];
            s.kernel = "rmsnorm_gemv_f32";
            s.inputs = {own(norm.inputs[0]), own(norm.inputs[1]), own(rhs)};
            s.constants = {(std::uint32_t)m, (std::uint32_t)k, (std::uint32_t)n, floatBits(attrEps(norm))};
            s.region = "RMSNorm -> GEMV (norm in the GEMV prologue)";
            s.nodes = {lhs - nin, node};
          } else if (a.dtype == kGraphF16 && w.transposed2d && m <= 8 && k % 8 == 0) {
            s.kernel = "gemv_f16";
            s.inputs = {own(lhs), own(rhs)};
            s.constants = {(std::uint32_t)m, (std::uint32_t)k, (std::uint32_t)n};
          } else {
            if (!w.contiguous() && !w.transposed2d) {
              plan.error = "MatMul: the right-hand operand must be contiguous or a Transpose view.";
              return plan;
            }
            s.kernel = "matmul";
            s.inputs = {own(lhs), own(rhs)};
            s.constants = {(std::uint32_t)m, (std::uint32_t)k, (std::uint32_t)n, w.transposed2d ? 1u : 0u};
          }
          break;
        }
        case GraphOp::Add:
        case GraphOp::Mul: {
          std::size_t x = head.inputs[0], b = head.inputs[1];
          if (plan.types[x].elements() < plan.types[b].elements()) std::swap(x, b);
          if (!plan.types[x].contiguous() || !plan.types[b].contiguous()) {
            plan.error = std::string(opName(head.op)) + ": operands must be contiguous.";
            return plan;
          }
          std::size_t rows, width, brows = 1;
          rw(x, &rows, &width);
          rowBroadcast(plan.types[x], plan.types[b], &brows);
          s.kernel = head.op == GraphOp::Add ? "add" : "mul";
          s.inputs = {own(x), own(b)};
          s.constants = {(std::uint32_t)rows, (std::uint32_t)width, (std::uint32_t)brows};
          break;
        }
        case GraphOp::ReLU:
        case GraphOp::SiLU:
          if (!plan.types[head.inputs[0]].contiguous()) {
            plan.error = std::string(opName(head.op)) + ": the operand must be contiguous.";
            return plan;
          }
          s.kernel = head.op == GraphOp::ReLU ? "relu" : "silu";
          s.inputs = {own(head.inputs[0])};
          s.constants = {(std::uint32_t)plan.types[out].elements()};
          break;
        case GraphOp::LayerNorm: {
          // LayerNorm outside a fused region: the fused kernel with a zero
          // residual is not the reference's node; refuse instead.
          plan.error = "LayerNorm runs here only fused behind its residual Add.";
          return plan;
        }
        default:
          plan.error = std::string(opName(head.op)) + " has no graph kernel in this backend.";
          return plan;
      }
    }
    s.output = own(out);
    plan.steps.push_back(std::move(s));
  }
  return plan;
}

}  // namespace tensor::planner
