// Built-in kernel catalog (see KernelCatalog.hpp).
#include "KernelCatalog.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>

#include "attention.cuh"
#include "fusion.cuh"
#include "gemm.cuh"
#include "gemv.cuh"
#include "graph_ops.cuh"
#include "rmsnorm.cuh"

namespace tensor::cuda {
namespace {

float bitsToFloat(std::uint32_t bits) {
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// Every buffer of the binding has element type `t` (inputs then outputs, in
// binding order); `types` lists them when they differ.
std::string requireTypes(const KernelBinding &b, const std::vector<ElementType> &types, const char *name) {
  std::size_t i = 0;
  for (const auto *group : {&b.inputs, &b.outputs})
    for (const auto &buf : *group) {
      if (buf->elementType() != types[i])
        return std::string(name) + ": buffer " + std::to_string(i) + " must be " + elementName(types[i]) +
               ", not " + elementName(buf->elementType()) + ".";
      ++i;
    }
  return {};
}

std::string requireCount(const BufferHandle &buf, std::size_t need, const char *name, const char *what) {
  if (buf->elementCount() < need)
    return std::string(name) + ": " + what + " holds " + std::to_string(buf->elementCount()) + " elements, needs " +
           std::to_string(need) + ".";
  return {};
}

// Same floating type (fp32 or fp16) for every buffer.
std::string uniformFloat(const KernelBinding &b, const char *name) {
  const ElementType t = b.inputs[0]->elementType();
  if (t != ElementType::Float32 && t != ElementType::Float16)
    return std::string(name) + ": buffers must be fp32 or fp16.";
  std::vector<ElementType> types(b.inputs.size() + b.outputs.size(), t);
  return requireTypes(b, types, name);
}

#define TMC_CHECK(expr)              \
  do {                               \
    std::string e_ = (expr);         \
    if (!e_.empty()) return e_;      \
  } while (0)

// ---- rmsnorm / rmsnorm_baseline: x [rows, width], gamma [width] -> y ----
// constants {rows, width, eps bits}; threads per CTA from the dispatch
// (rmsnorm: a power of two in [32, 1024]; the baseline always runs 256).
std::string bindRmsnorm(CudaRuntime &, KernelBinding &b) {
  TMC_CHECK(uniformFloat(b, "rmsnorm"));
  const std::size_t rows = b.constants[0], width = b.constants[1];
  const float eps = bitsToFloat(b.constants[2]);
  if (rows == 0 || width == 0 || !(eps > 0.0f)) return "rmsnorm: rows, width and eps must be positive.";
  TMC_CHECK(requireCount(b.inputs[0], rows * width, "rmsnorm", "x"));
  TMC_CHECK(requireCount(b.inputs[1], width, "rmsnorm", "gamma"));
  TMC_CHECK(requireCount(b.outputs[0], rows * width, "rmsnorm", "y"));
  const std::size_t t = b.dispatch.threadsPerThreadgroup;
  if (t < 32 || (t & (t - 1)) != 0) return "rmsnorm: threads per CTA must be a power of two >= 32.";
  return {};
}
cudaError_t launchRmsnorm(const KernelBinding &b, cudaStream_t s) {
  return tmc::launch_rmsnorm(b.inputs[0]->data(), b.inputs[1]->data(), b.outputs[0]->data(), (int)b.constants[0],
                             (int)b.constants[1], bitsToFloat(b.constants[2]),
                             b.inputs[0]->elementType() == ElementType::Float16,
                             (int)b.dispatch.threadsPerThreadgroup, s);
}
cudaError_t launchRmsnormBaseline(const KernelBinding &b, cudaStream_t s) {
  return tmc::launch_rmsnorm_baseline(b.inputs[0]->data(), b.inputs[1]->data(), b.outputs[0]->data(),
                                      (int)b.constants[0], (int)b.constants[1], bitsToFloat(b.constants[2]),
                                      b.inputs[0]->elementType() == ElementType::Float16, s);
}

// ---- rmsnorm_gemv_f32: x f32 [rows, k], gamma f32 [k], W f16 [n, k] -> y f32 [rows, n] ----
// constants {rows (1..4), k (% 8 == 0), n, eps bits}
std::string bindRmsnormGemv(CudaRuntime &, KernelBinding &b) {
  TMC_CHECK(requireTypes(b, {ElementType::Float32, ElementType::Float32, ElementType::Float16, ElementType::Float32},
                         "rmsnorm_gemv_f32"));
  const std::size_t rows = b.constants[0], k = b.constants[1], n = b.constants[2];
  if (rows < 1 || rows > 4 || k < 8 || k % 8 != 0 || n < 1 || !(bitsToFloat(b.constants[3]) > 0.0f))
    return "rmsnorm_gemv_f32: need 1 <= rows <= 4, k % 8 == 0, n >= 1, eps > 0.";
  TMC_CHECK(requireCount(b.inputs[0], rows * k, "rmsnorm_gemv_f32", "x"));
  TMC_CHECK(requireCount(b.inputs[1], k, "rmsnorm_gemv_f32", "gamma"));
  TMC_CHECK(requireCount(b.inputs[2], n * k, "rmsnorm_gemv_f32", "W"));
  TMC_CHECK(requireCount(b.outputs[0], rows * n, "rmsnorm_gemv_f32", "y"));
  return {};
}
cudaError_t launchRmsnormGemvImpl(const KernelBinding &b, cudaStream_t s, bool pdl) {
  tmc::GemvParams p{};
  p.W = static_cast<const __half *>(b.inputs[2]->data());
  p.M = (int)b.constants[0];
  p.K = (int)b.constants[1];
  p.N = (int)b.constants[2];
  p.prologue = tmc::kProF32Norm;
  p.x = b.inputs[0]->data();
  p.x_stride = p.K;
  p.gamma = b.inputs[1]->data();
  p.eps = bitsToFloat(b.constants[3]);
  p.epilogue = tmc::kEpiF32;
  p.y_f32 = static_cast<float *>(b.outputs[0]->data());
  p.y_stride = p.N;
  return tmc::launch_gemv(p, s, pdl, b.numSms);
}
cudaError_t launchRmsnormGemv(const KernelBinding &b, cudaStream_t s) { return launchRmsnormGemvImpl(b, s, false); }
cudaError_t launchRmsnormGemvPdl(const KernelBinding &b, cudaStream_t s) { return launchRmsnormGemvImpl(b, s, true); }

// ---- gemv_f16: x f16 [rows, k], W f16 [n, k] -> y f16 or f32 [rows, n] ----
// constants {rows (1..8), k (% 8 == 0), n}
std::string bindGemv(CudaRuntime &, KernelBinding &b) {
  const ElementType yt = b.outputs[0]->elementType();
  if (yt != ElementType::Float16 && yt != ElementType::Float32) return "gemv_f16: y must be fp16 or fp32.";
  TMC_CHECK(requireTypes(b, {ElementType::Float16, ElementType::Float16, yt}, "gemv_f16"));
  const std::size_t rows = b.constants[0], k = b.constants[1], n = b.constants[2];
  if (rows < 1 || rows > 8 || k < 8 || k % 8 != 0 || n < 1) return "gemv_f16: need 1 <= rows <= 8, k % 8 == 0.";
  TMC_CHECK(requireCount(b.inputs[0], rows * k, "gemv_f16", "x"));
  TMC_CHECK(requireCount(b.inputs[1], n * k, "gemv_f16", "W"));
  TMC_CHECK(requireCount(b.outputs[0], rows * n, "gemv_f16", "y"));
  return {};
}
cudaError_t launchGemvImpl(const KernelBinding &b, cudaStream_t s, bool pdl) {
  tmc::GemvParams p{};
  p.W = static_cast<const __half *>(b.inputs[1]->data());
  p.M = (int)b.constants[0];
  p.K = (int)b.constants[1];
  p.N = (int)b.constants[2];
  p.prologue = tmc::kProF16;
  p.x = b.inputs[0]->data();
  p.x_stride = p.K;
  if (b.outputs[0]->elementType() == ElementType::Float16) {
    p.epilogue = tmc::kEpiF16;
    p.y_f16 = static_cast<__half *>(b.outputs[0]->data());
  } else {
    p.epilogue = tmc::kEpiF32;
    p.y_f32 = static_cast<float *>(b.outputs[0]->data());
  }
  p.y_stride = p.N;
  return tmc::launch_gemv(p, s, pdl, b.numSms);
}
cudaError_t launchGemv(const KernelBinding &b, cudaStream_t s) { return launchGemvImpl(b, s, false); }
cudaError_t launchGemvPdl(const KernelBinding &b, cudaStream_t s) { return launchGemvImpl(b, s, true); }

// ---- batched_gemm_f16: x f16 [rows, k], W f16 [n, k] -> y f32 [rows, n] (tcgen05) ----
// constants {rows (1..256), k (% 8 == 0), n}; the split-K workspace and tile
// tickets are allocated here and retained by the prepared execution.
std::string bindBatchedGemm(CudaRuntime &rt, KernelBinding &b) {
  TMC_CHECK(requireTypes(b, {ElementType::Float16, ElementType::Float16, ElementType::Float32}, "batched_gemm_f16"));
  const std::size_t rows = b.constants[0], k = b.constants[1], n = b.constants[2];
  if (rows < 1 || rows > 256 || k < 8 || k % 8 != 0 || n < 1)
    return "batched_gemm_f16: need 1 <= rows <= 256, k % 8 == 0.";
  TMC_CHECK(requireCount(b.inputs[0], rows * k, "batched_gemm_f16", "x"));
  TMC_CHECK(requireCount(b.inputs[1], n * k, "batched_gemm_f16", "W"));
  TMC_CHECK(requireCount(b.outputs[0], rows * n, "batched_gemm_f16", "y"));
  const tmc::GemmPlan plan = tmc::plan_gemm((int)n, (int)k, (int)rows, b.numSms);
  const std::size_t partial = (tmc::gemm_workspace_floats(plan) * 4 + 255) / 256 * 256;
  auto ws = rt.createBuffer(partial / 4 + 1, nullptr, ElementType::Float32);
  if (!ws.buffer) return ws.errorMessage;
  auto tickets = rt.createBuffer((std::size_t)plan.tiles * 2, nullptr, ElementType::Int32);  // zeroed
  if (!tickets.buffer) return tickets.errorMessage;
  b.workspace = ws.buffer;
  b.counters = tickets.buffer;
  return {};
}
cudaError_t launchBatchedGemm(const KernelBinding &b, cudaStream_t s) {
  const int rows = (int)b.constants[0], k = (int)b.constants[1], n = (int)b.constants[2];
  const tmc::GemmPlan plan = tmc::plan_gemm(n, k, rows, b.numSms);
  CUtensorMap wm, xm;
  cudaError_t e;
  if ((e = tmc::make_tensor_map_f16(&wm, b.inputs[1]->data(), n, k, tmc::kGemmTileRows)) != cudaSuccess) return e;
  if ((e = tmc::make_tensor_map_f16(&xm, b.inputs[0]->data(), rows, k, plan.tn)) != cudaSuccess) return e;
  tmc::GemvParams p{};
  p.W = static_cast<const __half *>(b.inputs[1]->data());
  p.N = n;
  p.K = k;
  p.M = rows;
  p.prologue = tmc::kProF16;
  p.x = b.inputs[0]->data();
  p.x_stride = k;
  p.epilogue = tmc::kEpiF32;
  p.y_f32 = static_cast<float *>(b.outputs[0]->data());
  p.y_stride = n;
  p.status = b.status;
  // The kernel leaves its tile tickets at zero, so a retained workspace can be replayed.
  return tmc::launch_gemm(p, wm, xm, plan, static_cast<float *>(b.workspace->data()),
                          static_cast<unsigned int *>(b.counters->data()), s, false);
}

// ---- fused regions (formRegions / emitFusion) ----
// fused_add_rmsnorm:   x [rows, width], b [b_rows, width], w [width] -> y
// fused_add_layernorm: x, b, w, c [width] -> y
//   constants {rows, width, b_rows (1 or rows), eps bits}
std::string bindAddNorm(const KernelBinding &b, const char *name) {
  TMC_CHECK(uniformFloat(b, name));
  const std::size_t rows = b.constants[0], width = b.constants[1], brows = b.constants[2];
  if (rows < 1 || width < 1 || (brows != 1 && brows != rows) || !(bitsToFloat(b.constants[3]) > 0.0f))
    return std::string(name) + ": rows, width >= 1, b_rows 1 or rows, eps > 0.";
  TMC_CHECK(requireCount(b.inputs[0], rows * width, name, "x"));
  TMC_CHECK(requireCount(b.inputs[1], brows * width, name, "b"));
  for (std::size_t i = 2; i < b.inputs.size(); ++i) TMC_CHECK(requireCount(b.inputs[i], width, name, "w / c"));
  TMC_CHECK(requireCount(b.outputs[0], rows * width, name, "y"));
  return {};
}
std::string bindAddRmsnorm(CudaRuntime &, KernelBinding &b) { return bindAddNorm(b, "fused_add_rmsnorm"); }
std::string bindAddLayernorm(CudaRuntime &, KernelBinding &b) { return bindAddNorm(b, "fused_add_layernorm"); }
cudaError_t launchAddNorm(const KernelBinding &b, cudaStream_t s) {
  const bool ln = b.inputs.size() == 4;
  return tmc::launch_fused_add_norm(b.inputs[0]->data(), b.inputs[1]->data(), b.inputs[2]->data(),
                                    ln ? b.inputs[3]->data() : nullptr, b.outputs[0]->data(), (int)b.constants[0],
                                    (int)b.constants[1], (int)b.constants[2], bitsToFloat(b.constants[3]), ln,
                                    b.inputs[0]->elementType() == ElementType::Float16, s);
}

// fused_silu_mul: x [rows, width], b [b_rows, width] -> y; constants {rows, width, b_rows}
std::string bindSiluMul(CudaRuntime &, KernelBinding &b) {
  TMC_CHECK(uniformFloat(b, "fused_silu_mul"));
  const std::size_t rows = b.constants[0], width = b.constants[1], brows = b.constants[2];
  if (rows < 1 || width < 1 || (brows != 1 && brows != rows)) return "fused_silu_mul: b_rows must be 1 or rows.";
  TMC_CHECK(requireCount(b.inputs[0], rows * width, "fused_silu_mul", "x"));
  TMC_CHECK(requireCount(b.inputs[1], brows * width, "fused_silu_mul", "b"));
  TMC_CHECK(requireCount(b.outputs[0], rows * width, "fused_silu_mul", "y"));
  return {};
}
cudaError_t launchSiluMul(const KernelBinding &b, cudaStream_t s) {
  return tmc::launch_fused_silu_mul(b.inputs[0]->data(), b.inputs[1]->data(), b.outputs[0]->data(),
                                    (int)b.constants[0], (int)b.constants[1], (int)b.constants[2],
                                    b.inputs[0]->elementType() == ElementType::Float16, s);
}

// fused_linear_relu: a [m, k], w [k, n], bias [n] -> y [m, n]; constants {m, k, n}
std::string bindLinearRelu(CudaRuntime &, KernelBinding &b) {
  TMC_CHECK(uniformFloat(b, "fused_linear_relu"));
  const std::size_t m = b.constants[0], k = b.constants[1], n = b.constants[2];
  if (m < 1 || k < 1 || n < 1) return "fused_linear_relu: m, k, n must be positive.";
  TMC_CHECK(requireCount(b.inputs[0], m * k, "fused_linear_relu", "a"));
  TMC_CHECK(requireCount(b.inputs[1], k * n, "fused_linear_relu", "w"));
  TMC_CHECK(requireCount(b.inputs[2], n, "fused_linear_relu", "bias"));
  TMC_CHECK(requireCount(b.outputs[0], m * n, "fused_linear_relu", "y"));
  return {};
}
cudaError_t launchLinearRelu(const KernelBinding &b, cudaStream_t s) {
  return tmc::launch_fused_linear_relu(b.inputs[0]->data(), b.inputs[1]->data(), b.inputs[2]->data(),
                                       b.outputs[0]->data(), (int)b.constants[0], (int)b.constants[1],
                                       (int)b.constants[2], b.inputs[0]->elementType() == ElementType::Float16, s);
}

// ---- generic graph nodes (graph_ops.cuh) ----
// add / mul: x [rows, width], b [b_rows, width] -> y; constants {rows, width, b_rows}
std::string bindBinary(const KernelBinding &b, const char *name) {
  TMC_CHECK(uniformFloat(b, name));
  const std::size_t rows = b.constants[0], width = b.constants[1], brows = b.constants[2];
  if (rows < 1 || width < 1 || (brows != 1 && brows != rows)) return std::string(name) + ": b_rows must be 1 or rows.";
  TMC_CHECK(requireCount(b.inputs[0], rows * width, name, "x"));
  TMC_CHECK(requireCount(b.inputs[1], brows * width, name, "b"));
  TMC_CHECK(requireCount(b.outputs[0], rows * width, name, "y"));
  return {};
}
std::string bindAdd(CudaRuntime &, KernelBinding &b) { return bindBinary(b, "add"); }
std::string bindMul(CudaRuntime &, KernelBinding &b) { return bindBinary(b, "mul"); }
cudaError_t launchBinary(const KernelBinding &b, cudaStream_t s, bool mul) {
  return tmc::launch_graph_binary(b.inputs[0]->data(), b.inputs[1]->data(), b.outputs[0]->data(), (int)b.constants[0],
                                  (int)b.constants[1], (int)b.constants[2], mul,
                                  b.inputs[0]->elementType() == ElementType::Float16, s);
}
cudaError_t launchAdd(const KernelBinding &b, cudaStream_t s) { return launchBinary(b, s, false); }
cudaError_t launchMul(const KernelBinding &b, cudaStream_t s) { return launchBinary(b, s, true); }

// relu / silu: x -> y; constants {count}
std::string bindUnary(const KernelBinding &b, const char *name) {
  TMC_CHECK(uniformFloat(b, name));
  const std::size_t count = b.constants[0];
  if (count < 1) return std::string(name) + ": count must be positive.";
  TMC_CHECK(requireCount(b.inputs[0], count, name, "x"));
  TMC_CHECK(requireCount(b.outputs[0], count, name, "y"));
  return {};
}
std::string bindRelu(CudaRuntime &, KernelBinding &b) { return bindUnary(b, "relu"); }
std::string bindSilu(CudaRuntime &, KernelBinding &b) { return bindUnary(b, "silu"); }
cudaError_t launchRelu(const KernelBinding &b, cudaStream_t s) {
  return tmc::launch_graph_unary(b.inputs[0]->data(), b.outputs[0]->data(), b.constants[0], false,
                                 b.inputs[0]->elementType() == ElementType::Float16, s);
}
cudaError_t launchSilu(const KernelBinding &b, cudaStream_t s) {
  return tmc::launch_graph_unary(b.inputs[0]->data(), b.outputs[0]->data(), b.constants[0], true,
                                 b.inputs[0]->elementType() == ElementType::Float16, s);
}

// matmul: a [m, k], W ([k, n], or [n, k] read transposed) -> y [m, n];
// constants {m, k, n, w_transposed}; a and y fp32 or fp16, W as a or fp16.
std::string bindMatmul(CudaRuntime &, KernelBinding &b) {
  const ElementType at = b.inputs[0]->elementType(), wt = b.inputs[1]->elementType();
  if ((at != ElementType::Float32 && at != ElementType::Float16) || (wt != at && wt != ElementType::Float16))
    return "matmul: a and y fp32 or fp16, W the same type or fp16.";
  TMC_CHECK(requireTypes(b, {at, wt, at}, "matmul"));
  const std::size_t m = b.constants[0], k = b.constants[1], n = b.constants[2];
  if (m < 1 || k < 1 || n < 1 || b.constants[3] > 1) return "matmul: m, k, n positive, w_transposed 0 or 1.";
  TMC_CHECK(requireCount(b.inputs[0], m * k, "matmul", "a"));
  TMC_CHECK(requireCount(b.inputs[1], k * n, "matmul", "W"));
  TMC_CHECK(requireCount(b.outputs[0], m * n, "matmul", "y"));
  return {};
}
cudaError_t launchMatmul(const KernelBinding &b, cudaStream_t s) {
  return tmc::launch_graph_matmul(b.inputs[0]->data(), b.inputs[1]->data(), b.outputs[0]->data(), (int)b.constants[0],
                                  (int)b.constants[1], (int)b.constants[2], b.constants[3] != 0,
                                  b.inputs[0]->elementType() == ElementType::Float16,
                                  b.inputs[1]->elementType() == ElementType::Float16, s);
}

// ---- paged_attention_f16 (emitServingPagedKVAttention) ----
// q f16 [rows, hq, d], k_pool, v_pool f16 [pool_pages, hkv, page, d],
// block_table i32 [*, table_stride], table_rows i32 [rows], positions i32 [rows]
// -> out f16 [rows, hq, d]; constants {rows, hq, hkv, d, page_size,
// pool_pages, capacity, table_stride, max_splits, min_chunk}. The split
// workspace and tickets are allocated here and retained.
std::string bindAttention(CudaRuntime &rt, KernelBinding &b) {
  const auto F16 = ElementType::Float16, I32 = ElementType::Int32;
  TMC_CHECK(requireTypes(b, {F16, F16, F16, I32, I32, I32, F16}, "paged_attention_f16"));
  const std::size_t rows = b.constants[0], hq = b.constants[1], hkv = b.constants[2], d = b.constants[3],
                    page = b.constants[4], pool = b.constants[5], stride = b.constants[7];
  const std::size_t splits = b.constants[8], chunk = b.constants[9];
  if (rows < 1 || hkv < 1 || hq % hkv != 0 || page < 1 || pool < 1 || stride < 1 || splits < 1 || chunk < 1)
    return "paged_attention_f16: invalid dimensions.";
  TMC_CHECK(requireCount(b.inputs[0], rows * hq * d, "paged_attention_f16", "q"));
  TMC_CHECK(requireCount(b.inputs[1], pool * hkv * page * d, "paged_attention_f16", "k_pool"));
  TMC_CHECK(requireCount(b.inputs[2], pool * hkv * page * d, "paged_attention_f16", "v_pool"));
  TMC_CHECK(requireCount(b.inputs[4], rows, "paged_attention_f16", "table_rows"));
  TMC_CHECK(requireCount(b.inputs[5], rows, "paged_attention_f16", "positions"));
  TMC_CHECK(requireCount(b.outputs[0], rows * hq * d, "paged_attention_f16", "out"));
  const std::size_t capped = splits < (std::size_t)tmc::kAttentionMaxSplits ? splits : tmc::kAttentionMaxSplits;
  auto ws = rt.createBuffer(tmc::attention_workspace_bytes((int)rows, (int)hq, (int)hkv, (int)d, (int)capped) / 4 + 1,
                            nullptr, ElementType::Float32);
  if (!ws.buffer) return ws.errorMessage;
  auto counters = rt.createBuffer(rows * hkv, nullptr, ElementType::Int32);  // zeroed
  if (!counters.buffer) return counters.errorMessage;
  b.workspace = ws.buffer;
  b.counters = counters.buffer;
  b.constants[8] = (std::uint32_t)capped;
  return {};
}
cudaError_t launchAttention(const KernelBinding &b, cudaStream_t s) {
  const auto &c = b.constants;
  tmc::AttentionParams p{};
  p.q = static_cast<const __half *>(b.inputs[0]->data());
  p.q_stride = (long long)c[1] * c[3];
  p.out = static_cast<__half *>(b.outputs[0]->data());
  p.out_stride = p.q_stride;
  p.k_pool = static_cast<const __half *>(b.inputs[1]->data());
  p.v_pool = static_cast<const __half *>(b.inputs[2]->data());
  p.block_table = static_cast<const int *>(b.inputs[3]->data());
  p.table_stride = (int)c[7];
  p.table_rows = static_cast<const int *>(b.inputs[4]->data());
  p.positions = static_cast<const int *>(b.inputs[5]->data());
  p.rows = (int)c[0];
  p.hq = (int)c[1];
  p.hkv = (int)c[2];
  p.head_dim = (int)c[3];
  p.page_size = (int)c[4];
  p.pool_pages = (int)c[5];
  p.capacity = (int)c[6];
  p.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(c[3])));
  p.max_splits = (int)c[8];
  p.min_chunk = (int)c[9];
  p.early_mode = 2;
  p.ws_acc = static_cast<float *>(b.workspace->data());
  p.ws_ml = p.ws_acc + (size_t)c[0] * c[1] * c[8] * c[3];
  p.counters = static_cast<unsigned int *>(b.counters->data());
  p.status = b.status;
  CUtensorMap km, vm;
  const uint64_t poolRows = (uint64_t)c[5] * c[2] * c[4];
  if ((c[3] == 64 || c[3] == 128) && c[4] % 16 == 0 &&
      tmc::make_tensor_map_f16(&km, p.k_pool, poolRows, c[3], 16) == cudaSuccess &&
      tmc::make_tensor_map_f16(&vm, p.v_pool, poolRows, c[3], 16) == cudaSuccess) {
    p.k_map = &km;
    p.v_map = &vm;
  }
  return tmc::launch_attention(p, s, false);
}

#undef TMC_CHECK

}  // namespace

const std::vector<KernelEntry> &kernelCatalog() {
  static const std::vector<KernelEntry> catalog = {
      {"rmsnorm", 2, 1, 3,
       "x [rows, width], gamma [width] -> y [rows, width], all fp32 or all fp16; constants {rows, width, eps as "
       "float bits}; dispatch: threads per CTA (power of two >= 32)",
       bindRmsnorm, launchRmsnorm},
      {"rmsnorm_baseline", 2, 1, 3,
       "the frozen 256-thread scalar RMSNorm; same interface as rmsnorm", bindRmsnorm, launchRmsnormBaseline},
      {"rmsnorm_gemv_f32", 3, 1, 4,
       "x fp32 [rows, k], gamma fp32 [k], W fp16 [n, k] -> y fp32 [rows, n]; constants {rows (1..4), k (% 8), n, "
       "eps bits}",
       bindRmsnormGemv, launchRmsnormGemv, launchRmsnormGemvPdl, 1u << 2},
      {"gemv_f16", 2, 1, 3,
       "x fp16 [rows, k], W fp16 [n, k] -> y fp16 or fp32 [rows, n]; constants {rows (1..8), k (% 8), n}",
       bindGemv, launchGemv, launchGemvPdl, 1u << 1},
      {"batched_gemm_f16", 2, 1, 3,
       "x fp16 [rows, k], W fp16 [n, k] -> y fp32 [rows, n] on tcgen05 tensor cores; constants {rows (1..256), "
       "k (% 8), n}",
       bindBatchedGemm, launchBatchedGemm},
      {"fused_add_rmsnorm", 3, 1, 4,
       "x [rows, width], b [b_rows, width], w [width] -> y = RMSNorm(x + b) * w; constants {rows, width, b_rows, "
       "eps bits}",
       bindAddRmsnorm, launchAddNorm},
      {"fused_add_layernorm", 4, 1, 4,
       "x [rows, width], b [b_rows, width], w, c [width] -> y = LayerNorm(x + b) * w + c; constants {rows, width, "
       "b_rows, eps bits}",
       bindAddLayernorm, launchAddNorm},
      {"fused_silu_mul", 2, 1, 3,
       "x [rows, width], b [b_rows, width] -> y = silu(x) * b; constants {rows, width, b_rows}", bindSiluMul,
       launchSiluMul},
      {"fused_linear_relu", 3, 1, 3,
       "a [m, k], w [k, n], bias [n] -> y = relu(a . w + bias) [m, n]; constants {m, k, n}", bindLinearRelu,
       launchLinearRelu},
      {"add", 2, 1, 3, "x [rows, width], b [b_rows, width] -> y = x + b; constants {rows, width, b_rows}", bindAdd,
       launchAdd},
      {"mul", 2, 1, 3, "x [rows, width], b [b_rows, width] -> y = x * b; constants {rows, width, b_rows}", bindMul,
       launchMul},
      {"relu", 1, 1, 1, "x -> y = max(x, 0); constants {count}", bindRelu, launchRelu},
      {"silu", 1, 1, 1, "x -> y = x * sigmoid(x); constants {count}", bindSilu, launchSilu},
      {"matmul", 2, 1, 4,
       "a [m, k], W [k, n] (or [n, k] read transposed) -> y [m, n]; a, y fp32 or fp16, W as a or fp16; constants "
       "{m, k, n, w_transposed}",
       bindMatmul, launchMatmul},
      {"paged_attention_f16", 6, 1, 10,
       "q fp16 [rows, hq, d], k_pool, v_pool fp16 [pool_pages, hkv, page, d], block_table i32, table_rows i32 "
       "[rows], positions i32 [rows] -> out fp16 [rows, hq, d]; constants {rows, hq, hkv, d, page_size, "
       "pool_pages, capacity, table_stride, max_splits, min_chunk}",
       bindAttention, launchAttention},
  };
  return catalog;
}

const KernelEntry *findKernel(const std::string &name) {
  for (const auto &k : kernelCatalog())
    if (name == k.name) return &k;
  return nullptr;
}

PreparationResult prepareKernel(CudaRuntime &runtime, const KernelEntry &kernel, std::vector<BufferHandle> inputs,
                                std::vector<BufferHandle> outputs, DispatchSize dispatch,
                                std::vector<std::uint32_t> constants) {
  PreparationResult result;
  if (!runtime.isAvailable()) {
    result.errorMessage = runtime.initializationError();
    return result;
  }
  // Binding count and dispatch limits as prepareBuffers checks them
  // (MetalRuntime.mm:608-620), then the kernel's own interface.
  const std::size_t bindingCount = inputs.size() + outputs.size() + !constants.empty();
  if (inputs.empty() || outputs.empty() || bindingCount > 31 || constants.size() > 1024) {
    result.errorMessage = "Invalid buffer binding count or oversized inline constants.";
    return result;
  }
  const HardwareInfo hw = runtime.hardwareInfo();
  if (dispatch.threadgroupCount == 0 || dispatch.threadgroupCount > std::numeric_limits<std::uint32_t>::max() ||
      dispatch.threadsPerThreadgroup == 0 || dispatch.threadsPerThreadgroup > hw.maxThreadsPerThreadgroup) {
    result.errorMessage = "Kernel dispatch exceeds device or pipeline limits.";
    return result;
  }
  for (std::size_t i = 0; i < outputs.size(); ++i) {
    if (!outputs[i] || std::find(outputs.begin(), outputs.begin() + i, outputs[i]) != outputs.begin() + i) {
      result.errorMessage = "Outputs must be distinct buffers on the current device.";
      return result;
    }
  }
  for (const auto &input : inputs) {
    if (!input || std::find(outputs.begin(), outputs.end(), input) != outputs.end()) {
      result.errorMessage = "Input is missing, on another device, or aliases an output.";
      return result;
    }
  }
  if ((int)inputs.size() != kernel.inputs || (int)outputs.size() != kernel.outputs ||
      (int)constants.size() != kernel.constants) {
    result.errorMessage = std::string(kernel.name) + " binds " + std::to_string(kernel.inputs) + " inputs, " +
                          std::to_string(kernel.outputs) + " outputs and " + std::to_string(kernel.constants) +
                          " constants: " + kernel.signature;
    return result;
  }
  KernelBinding binding;
  binding.inputs = inputs;
  binding.outputs = outputs;
  binding.constants = std::move(constants);
  binding.dispatch = dispatch;
  binding.status = runtime.deviceStatus();
  binding.numSms = hw.multiprocessorCount > 0 ? hw.multiprocessorCount : 148;
  std::string error = kernel.bind(runtime, binding);
  if (!error.empty()) {
    result.errorMessage = error;
    return result;
  }
  auto launch = kernel.launch;
  std::vector<BufferHandle> early;
  for (std::size_t i = 0; i < inputs.size(); ++i)
    if (kernel.earlyInputs & (1u << i)) early.push_back(inputs[i]);
  result = runtime.prepare([binding, launch](cudaStream_t s) { return launch(binding, s); }, std::move(inputs),
                           std::move(outputs), kernel.name);
  if (result.execution && kernel.launchOverlapped) {
    auto overlapped = kernel.launchOverlapped;
    result.execution->allowOverlap([binding, overlapped](cudaStream_t s) { return overlapped(binding, s); },
                                   std::move(early));
  }
  return result;
}

}  // namespace tensor::cuda
