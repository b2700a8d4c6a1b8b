/*
 * oracle/graph_ref.c -- TEST INFRASTRUCTURE ONLY (the CPU checker, never the
 * product path). Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it.
 *
 * A plain-C restatement of the reference's CPU oracle for the ops on the decode
 * hot path, in fp64 with the reference's storage rounding:
 *   - storeValue(): fp64 -> float -> storage dtype, GraphReference.cpp:82-87.
 *     The reference's CPU floatToHalf (GraphReference.cpp:38-59) rounds a
 *     float's dropped mantissa bits to nearest with ties AWAY from zero (it
 *     adds half an fp16 ulp and truncates, normals and subnormals alike), so
 *     oracle_store does the same; a tie is common when two fp16 values are
 *     added. oracle_round_f16 / oracle_f32_to_f16_bits convert inputs with IEEE
 *     round-to-nearest-even, the conversion of the GPU (and of Metal).
 *   - rmsNormReference(): Validator.cpp:40-66;
 *   - MatMul: GraphReference.cpp:150-167 (fp64 sums of stored operands);
 *   - Transpose (materialised view): GraphReference.cpp:269-287;
 *   - compare(): atol + rtol*|ref| with first-mismatch index, Validator.cpp:11-38;
 *   - the decode GEMV fp64 reference of DecodeGEMVTuner.cpp:98-118;
 *   - serving paged decode attention, KVCacheMetalEmitter.cpp:312-406
 *     (scale 1/sqrt(D), softmax, fp32-stored context), extended with the GQA
 *     head map h -> h / (Hq/Hkv) that the reference lacks.
 */
#include <math.h>
#include <stdlib.h>
#include <stdint.h>
#include <string.h>

/* ---- storage rounding (GraphReference.cpp:82-87) --------------------------- */

static uint16_t f32_to_f16_bits(float value) {
  uint32_t f;
  memcpy(&f, &value, 4);
  const uint32_t sign = (f >> 16) & 0x8000u;
  const uint32_t absf = f & 0x7fffffffu;
  if (absf >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (absf > 0x7f800000u ? 0x200u : 0u));
  if (absf >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
  const int e = (int)(absf >> 23);
  if (e < 113) {
    if (e < 102) return (uint16_t)sign;
    const uint32_t mant = (absf & 0x7fffffu) | 0x800000u;
    const int shift = 126 - e;
    uint32_t h = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1u), mid = 1u << (shift - 1);
    if (rem > mid || (rem == mid && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
  }
  uint32_t h = ((uint32_t)(e - 112) << 10) | ((absf >> 13) & 0x3ffu);
  const uint32_t rem = absf & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  return (uint16_t)(sign | h);
}

static float f16_bits_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  uint32_t f;
  float out;
  if (e == 0) {
    out = (float)m * (1.0f / 16777216.0f);
    if (sign) out = -out;
    return out;
  }
  if (e == 31) f = sign | 0x7f800000u | (m << 13);
  else f = sign | ((e + 112) << 23) | (m << 13);
  memcpy(&out, &f, 4);
  return out;
}

/* fp32 -> fp16 bits rounding the magnitude to nearest, ties away from zero
 * (the storage rounding of the reference's CPU graph evaluator). */
static uint16_t f32_to_f16_bits_ties_away(float value) {
  uint32_t f;
  memcpy(&f, &value, 4);
  const uint32_t sign = (f >> 16) & 0x8000u;
  const int e = (int)((f >> 23) & 0xffu);
  const uint32_t m = f & 0x7fffffu;
  if (e == 0xff) return (uint16_t)(sign | (m != 0u ? 0x7e00u : 0x7c00u));
  const int he = e - 112; /* fp16 biased exponent */
  if (he >= 31) return (uint16_t)(sign | 0x7c00u);
  if (he <= 0) { /* fp16 subnormal (or zero) */
    if (he < -10) return (uint16_t)sign;
    const int drop = 14 - he; /* bits of the 24-bit significand below fp16's last */
    const uint32_t significand = m | 0x800000u;
    return (uint16_t)(sign | ((significand + (1u << (drop - 1))) >> drop));
  }
  const uint32_t up = m + (1u << 12); /* half of fp16's last mantissa bit */
  if (up & 0x800000u) return (uint16_t)(he + 1 >= 31 ? (sign | 0x7c00u) : (sign | ((uint32_t)(he + 1) << 10)));
  return (uint16_t)(sign | ((uint32_t)he << 10) | (up >> 13));
}

/* dtype: 0 = fp16, 1 = fp32 (the TMC_F16 / TMC_F32 codes) */
float oracle_store(double value, int dtype) {
  const float as_float = (float)value;
  if (dtype == 0) return f16_bits_to_f32(f32_to_f16_bits_ties_away(as_float));
  return as_float;
}

void oracle_round_f16(const float *in, float *out, long n) {
  for (long i = 0; i < n; ++i) out[i] = f16_bits_to_f32(f32_to_f16_bits(in[i]));
}

void oracle_f32_to_f16_bits(const float *in, uint16_t *out, long n) {
  for (long i = 0; i < n; ++i) out[i] = f32_to_f16_bits(in[i]);
}

void oracle_f16_bits_to_f32(const uint16_t *in, float *out, long n) {
  for (long i = 0; i < n; ++i) out[i] = f16_bits_to_f32(in[i]);
}

/* ---- RMSNorm (Validator.cpp:40-66) ----------------------------------------- */
void oracle_rmsnorm(const float *x, const float *w, long rows, long width, double eps,
                    double *out) {
  for (long r = 0; r < rows; ++r) {
    double ss = 0.0;
    for (long c = 0; c < width; ++c) {
      const double v = x[r * width + c];
      ss += v * v;
    }
    /* RMSNormAttributes::epsilon is a float (TensorIR.hpp:40): widen the float. */
    const double inv = 1.0 / sqrt(ss / (double)width + (double)(float)eps);
    for (long c = 0; c < width; ++c) out[r * width + c] = (double)x[r * width + c] * inv * (double)w[c];
  }
}

/* ---- C1 graph: RMSNorm -> Transpose(W) view -> MatMul ----------------------
 * x [rows, k] fp32, gamma [k] fp32, w [n, k] (values already fp16-rounded;
 * TensorIR forbids fp32 x fp16 MatMul, GraphAnalyzer.cpp:74, so the graph
 * declares W fp32 holding fp16 values, which is exact). The RMSNorm result is
 * stored as fp32 (storeValue), then MatMul sums in fp64; y is the fp64
 * "precise" output the reference compares against (GraphReference.cpp:338). */
void oracle_rmsnorm_matmul(const float *x, const float *gamma, const float *w, long rows, long k,
                           long n, double eps, double *y) {
  for (long r = 0; r < rows; ++r) {
    double ss = 0.0;
    for (long c = 0; c < k; ++c) ss += (double)x[r * k + c] * (double)x[r * k + c];
    const double inv = 1.0 / sqrt(ss / (double)k + (double)(float)eps);
    /* stored RMSNorm value (fp32) */
    float *normed = (float *)malloc((size_t)k * sizeof(float));
    if (normed == NULL) return;
    for (long c = 0; c < k; ++c) normed[c] = (float)((double)x[r * k + c] * inv * (double)gamma[c]);
    for (long j = 0; j < n; ++j) {
      double s = 0.0;
      const float *wr = w + j * k;
      for (long c = 0; c < k; ++c) s += (double)normed[c] * (double)wr[c];
      y[r * n + j] = s;
    }
    free(normed);
  }
}

/* ---- decode GEMV fp64 reference (DecodeGEMVTuner.cpp:98-118) --------------- */
void oracle_gemv(const float *x, const float *w, long rows, long k, long n, double *y) {
  for (long r = 0; r < rows; ++r)
    for (long j = 0; j < n; ++j) {
      double s = 0.0;
      for (long c = 0; c < k; ++c) s += (double)x[r * k + c] * (double)w[j * k + c];
      y[r * n + j] = s;
    }
}

/* ---- compare (Validator.cpp:11-38) -----------------------------------------
 * Returns the mismatch count; writes the max abs error and the first mismatch
 * index (-1 if none). */
long oracle_compare(const float *actual, const double *reference, long n, double atol, double rtol,
                    double *max_abs_error, long *first_mismatch) {
  long mismatches = 0;
  double worst = 0.0;
  *first_mismatch = -1;
  for (long i = 0; i < n; ++i) {
    const double e = reference[i], v = actual[i];
    const int finite = isfinite(v) && isfinite(e);
    const double err = finite ? fabs(v - e) : INFINITY;
    if (err > worst) worst = err;
    if (!finite || err > atol + rtol * fabs(e)) {
      if (mismatches == 0) *first_mismatch = i;
      ++mismatches;
    }
  }
  *max_abs_error = worst;
  return mismatches;
}

/* ---- serving paged decode attention (KVCacheMetalEmitter.cpp:312-406) ------
 * q [rows, hq, d] (fp16 values as float), pools [pages, hkv, page, d],
 * table [*, stride], table_rows[rows], positions[rows]; out [rows, hq, d] as
 * fp64 (the reference context before storage rounding). Returns -1 on a
 * missing page (the reference kernel returns without writing). */
int oracle_paged_attention(const float *q, const float *k_pool, const float *v_pool,
                           const int32_t *table, long stride, const int32_t *table_rows,
                           const int32_t *positions, long rows, long hq, long hkv, long d,
                           long page_size, double *out) {
  const long group = hq / hkv;
  const double scale = 1.0 / sqrt((double)d);
  for (long r = 0; r < rows; ++r) {
    const long len = (long)positions[r] + 1;
    const int32_t *t = table + (long)table_rows[r] * stride;
    for (long h = 0; h < hq; ++h) {
      const long kvh = h / group;
      const float *qh = q + (r * hq + h) * d;
      double mx = -INFINITY;
      /* two passes: max, then exp-sum and weighted values (exact softmax) */
      for (long p = 0; p < len; ++p) {
        const int32_t page = t[p / page_size];
        if (page < 0) return -1;
        const float *kr = k_pool + (((long)page * hkv + kvh) * page_size + p % page_size) * d;
        double s = 0.0;
        for (long i = 0; i < d; ++i) s += (double)qh[i] * (double)kr[i];
        s *= scale;
        if (s > mx) mx = s;
      }
      double den = 0.0;
      double *o = out + (r * hq + h) * d;
      for (long i = 0; i < d; ++i) o[i] = 0.0;
      for (long p = 0; p < len; ++p) {
        const int32_t page = t[p / page_size];
        const long base = (((long)page * hkv + kvh) * page_size + p % page_size) * d;
        double s = 0.0;
        for (long i = 0; i < d; ++i) s += (double)qh[i] * (double)k_pool[base + i];
        const double e = exp(s * scale - mx);
        den += e;
        for (long i = 0; i < d; ++i) o[i] += e * (double)v_pool[base + i];
      }
      for (long i = 0; i < d; ++i) o[i] /= den;
    }
  }
  return 0;
}

/* ---- fused graph regions (GraphReference.cpp:129-199, node by node) --------
 * The graph suite's fused regions (tensor_graph_examples.cpp:115-143,210-225):
 * kind 0 Add -> RMSNorm, 1 Add -> LayerNorm, 2 SiLU -> Mul,
 * 3 MatMul -> Add(bias) -> ReLU. Inputs hold storage values. x [rows, width];
 * b: the Add / Mul operand [b_rows, width] (b_rows 1 broadcasts over rows) or
 * the MatMul weight [width, n]; w, c: the norm weight / LayerNorm bias [width],
 * or (kind 3) c the ReLU bias [n]. Every intermediate node is stored in the
 * graph's dtype (oracle_store) before the next node reads it; y receives the
 * last node's fp64 value, the reference's "precise" output. Returns 0, or 1
 * for an unknown kind. */
int oracle_fusion(int kind, const float *x, const float *b, const float *w, const float *c, long rows,
                  long width, long b_rows, long n, double eps, int dtype, double *y) {
  const double e = (double)(float)eps; /* the attributes hold a float */
  if (kind == 3) {
    for (long r = 0; r < rows; ++r)
      for (long j = 0; j < n; ++j) {
        double s = 0.0;
        for (long k = 0; k < width; ++k) s += (double)x[r * width + k] * (double)b[k * n + j];
        const float linear = oracle_store(s, dtype);
        const float biased = oracle_store((double)linear + (double)c[j], dtype);
        y[r * n + j] = biased > 0.0f ? (double)biased : 0.0;
      }
    return 0;
  }
  if (kind == 2) {
    for (long r = 0; r < rows; ++r)
      for (long i = 0; i < width; ++i) {
        const double v = x[r * width + i];
        const double ex = exp(v >= 0.0 ? -v : v);
        const float act = oracle_store(v >= 0.0 ? v / (1.0 + ex) : v * ex / (1.0 + ex), dtype);
        y[r * width + i] = (double)act * (double)b[(b_rows == 1 ? 0 : r) * width + i];
      }
    return 0;
  }
  if (kind != 0 && kind != 1) return 1;
  float *added = (float *)malloc((size_t)width * sizeof(float));
  if (added == NULL) return 1;
  for (long r = 0; r < rows; ++r) {
    double sum = 0.0, squares = 0.0;
    for (long i = 0; i < width; ++i) {
      added[i] = oracle_store((double)x[r * width + i] + (double)b[(b_rows == 1 ? 0 : r) * width + i], dtype);
      sum += added[i];
      squares += (double)added[i] * (double)added[i];
    }
    if (kind == 0) {
      const double inv = 1.0 / sqrt(squares / (double)width + e);
      for (long i = 0; i < width; ++i) y[r * width + i] = (double)added[i] * inv * (double)w[i];
    } else {
      const double mean = sum / (double)width;
      double variance = squares / (double)width - mean * mean;
      if (variance < 0.0) variance = 0.0;
      const double inv = 1.0 / sqrt(variance + e);
      for (long i = 0; i < width; ++i) y[r * width + i] = ((double)added[i] - mean) * inv * (double)w[i] + (double)c[i];
    }
  }
  free(added);
  return 0;
}
