// faber_oracle.cpp — TEST INFRASTRUCTURE ONLY.
//
// CPU restatement of faber-runtime's Q4_K decoder oracle, made
// shape-parametric. It is the checker for the CUDA path: only tests/,
// __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs load
// it. Nothing in faber_runtime_b200 links, imports or calls it.
//
// Every function below names the reference function it restates
// (file:line inside faber-runtime). The arithmetic keeps the reference's
// operation order and rounding points:
//   * all f32 ops are separate IEEE round-to-nearest operations: this file is
//     compiled with -ffp-contract=off and without fast-math, matching Rust,
//     which never contracts a*b+c into an FMA;
//   * every reduction is a strictly sequential left-to-right sum (OpenMP is
//     used only ACROSS independent output rows / heads, never inside a sum,
//     so results are bit-identical for any thread count);
//   * libm: powf/cosf/sinf/expf/logf/sqrtf are glibc's, which is what Rust's
//     f32::{powf,cos,sin,exp,ln,sqrt} call on Linux.
//
// Deviations from the reference, all value-preserving:
//   * shapes are run-time parameters instead of the pinned-row constants
//     (src/decoder_ops.rs:60-79, src/cpu_oracle.rs:128-154);
//   * weights are dequantized row by row on the fly instead of materialized
//     whole (src/cpu_oracle.rs:302-345); the f16 weight rounding
//     (src/cpu_oracle.rs:356-360) is applied to the same values, so the
//     products and sums see identical operands;
//   * the attention scale is 1/sqrtf(head_dim) (0.125 for head_dim 64, the
//     reference's hard-coded ATTENTION_SCALE, src/decoder_ops.rs:79).

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <new>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API extern "C" __attribute__((visibility("default")))

namespace {

// GGUF dtype ids of the admitted block types (src/gguf.rs:135-144).
enum : int32_t { T_F32 = 0, T_Q5_0 = 6, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14 };

inline float from_bits(uint32_t b) { float f; std::memcpy(&f, &b, 4); return f; }
inline uint32_t to_bits(float f) { uint32_t b; std::memcpy(&b, &f, 4); return b; }
inline uint16_t le16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

int g_threads = 1;

}  // namespace

// ---------------------------------------------------------------------------
// Half <-> f32
// ---------------------------------------------------------------------------

// half_to_f32 — src/dequant.rs:122-144. Exact binary16 -> binary32 bit
// expansion, subnormals normalized by the leading-bit position.
ORC_API float orc_half_to_f32(uint16_t bits) {
  const uint32_t sign = (bits >> 15) & 1u;
  const uint32_t exp = (bits >> 10) & 0x1fu;
  const uint32_t frac = bits & 0x3ffu;
  uint32_t b32;
  if (exp == 0) {
    if (frac == 0) {
      b32 = sign << 31;
    } else {
      const uint32_t p = 32u - (uint32_t)__builtin_clz(frac);
      b32 = (sign << 31) | ((p + 102u) << 23) | ((frac << (24u - p)) - (1u << 23));
    }
  } else if (exp == 0x1f) {
    b32 = (sign << 31) | (0xffu << 23) | (frac << 13);
  } else {
    b32 = (sign << 31) | ((exp + 112u) << 23) | (frac << 13);
  }
  return from_bits(b32);
}

// round_half_to_even — src/cpu_oracle.rs:275-289.
static uint32_t round_half_to_even(float v) {
  const float f = std::floor(v);
  const float frac = v - f;
  if (frac < 0.5f) return (uint32_t)f;
  if (frac > 0.5f) return (uint32_t)(f + 1.0f);
  const uint32_t fi = (uint32_t)f;
  return (fi % 2 == 0) ? fi : fi + 1;
}

// f32_to_f16_rn — src/cpu_oracle.rs:225-271. Round-to-nearest-even, with the
// reference's NaN payload rule (zero high payload -> 0x7c01).
ORC_API uint16_t orc_f32_to_f16_rn(float x) {
  const uint32_t bits = to_bits(x);
  const uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
  const uint32_t m = bits & 0x7fffffffu;
  if (m >= 0x7f800000u) {
    if (m == 0x7f800000u) return sign | 0x7c00u;
    const uint16_t mant = (uint16_t)((m >> 13) & 0x3ffu);
    if (mant == 0) return sign | 0x7c01u;
    return sign | 0x7c00u | mant;
  }
  if (m >= 0x477ff000u) return sign | 0x7c00u;
  if (m >= 0x38800000u) {
    const uint32_t unexp = (m >> 23) & 0xffu;
    const uint32_t mant = m & 0x7fffffu;
    uint32_t word = ((unexp - 112u) << 10) | (mant >> 13);
    const uint32_t rest = mant & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (word & 1u) != 0)) word += 1;
    return sign | (uint16_t)word;
  }
  const float scaled = from_bits(m) * 16777216.0f;
  const uint32_t m10 = round_half_to_even(scaled);
  return sign | (uint16_t)m10;
}

// kv_f16_round / metal_f16_round_weights element op — src/cpu_oracle.rs:292-294,356-360.
ORC_API float orc_f16_round(float x) { return orc_half_to_f32(orc_f32_to_f16_rn(x)); }

ORC_API void orc_half_to_f32_array(const uint16_t* h, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = orc_half_to_f32(h[i]);
}

ORC_API void orc_f32_to_f16_array(const float* x, uint16_t* h, int64_t n) {
  for (int64_t i = 0; i < n; ++i) h[i] = orc_f32_to_f16_rn(x[i]);
}

ORC_API void orc_f16_round_array(const float* x, float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) y[i] = orc_f16_round(x[i]);
}

// ---------------------------------------------------------------------------
// Block dequant — src/dequant.rs:151-260
// ---------------------------------------------------------------------------

// dequant_q8_0 — src/dequant.rs:151-154.
static void dq_q8_0(const uint8_t* b, float* y) {
  const float d = orc_half_to_f32(le16(b));
  for (int j = 0; j < 32; ++j) y[j] = (float)(int8_t)b[2 + j] * d;
}

// dequant_q5_0 — src/dequant.rs:160-174.
static void dq_q5_0(const uint8_t* b, float* y) {
  const float d = orc_half_to_f32(le16(b));
  const uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) |
                      ((uint32_t)b[5] << 24);
  const uint8_t* qs = b + 6;
  for (uint32_t j = 0; j < 16; ++j) {
    const uint32_t xh0 = ((qh >> (j + 0)) << 4) & 0x10u;
    const uint32_t xh1 = (qh >> (j + 12)) & 0x10u;
    const int32_t x0 = (int32_t)((qs[j] & 0x0fu) | xh0) - 16;
    const int32_t x1 = (int32_t)((qs[j] >> 4) | xh1) - 16;
    y[j] = (float)x0 * d;
    y[j + 16] = (float)x1 * d;
  }
}

// get_scale_min_k4 — src/dequant.rs:178-187.
static inline void scale_min_k4(int index, const uint8_t* s, uint8_t* sc, uint8_t* m) {
  if (index < 4) {
    *sc = s[index] & 63;
    *m = s[index + 4] & 63;
  } else {
    *sc = (uint8_t)((s[index + 4] & 0x0f) | ((s[index - 4] >> 6) << 4));
    *m = (uint8_t)((s[index + 4] >> 4) | ((s[index] >> 6) << 4));
  }
}

// dequant_q4_k — src/dequant.rs:194-217. d1 = d*sc, m1 = dmin*m and
// y = d1*q - m1 are three separately rounded f32 operations.
static void dq_q4_k(const uint8_t* b, float* y) {
  const float d = orc_half_to_f32(le16(b));
  const float mn = orc_half_to_f32(le16(b + 2));
  const uint8_t* scales = b + 4;
  const uint8_t* qs = b + 16;
  int is = 0, qoff = 0;
  for (int chunk = 0; chunk < 256; chunk += 64) {
    uint8_t sc, m;
    scale_min_k4(is, scales, &sc, &m);
    const float d1 = d * (float)sc;
    const float m1 = mn * (float)m;
    scale_min_k4(is + 1, scales, &sc, &m);
    const float d2 = d * (float)sc;
    const float m2 = mn * (float)m;
    for (int l = 0; l < 32; ++l) {
      y[chunk + l] = d1 * (float)(qs[qoff + l] & 0x0f) - m1;
      y[chunk + 32 + l] = d2 * (float)(qs[qoff + l] >> 4) - m2;
    }
    qoff += 32;
    is += 2;
  }
}

// dequant_q6_k — src/dequant.rs:224-255, (d*sc)*q order.
static void dq_q6_k(const uint8_t* b, float* y) {
  const float d = orc_half_to_f32(le16(b + 208));
  const uint8_t* ql = b;
  const uint8_t* qh = b + 128;
  const uint8_t* sc = b + 192;
  for (int n = 0; n < 256; n += 128) {
    const int sc_base = n / 16, ql_off = n / 2, qh_off = n / 4;
    for (int l = 0; l < 32; ++l) {
      const int is = l / 16;
      const int q1 = (int)((ql[ql_off + l] & 0x0f) | (((qh[qh_off + l] >> 0) & 3) << 4)) - 32;
      const int q2 = (int)((ql[ql_off + l + 32] & 0x0f) | (((qh[qh_off + l] >> 2) & 3) << 4)) - 32;
      const int q3 = (int)((ql[ql_off + l] >> 4) | (((qh[qh_off + l] >> 4) & 3) << 4)) - 32;
      const int q4 = (int)((ql[ql_off + l + 32] >> 4) | (((qh[qh_off + l] >> 6) & 3) << 4)) - 32;
      const float s0 = (float)(int8_t)sc[sc_base + is + 0];
      const float s2 = (float)(int8_t)sc[sc_base + is + 2];
      const float s4 = (float)(int8_t)sc[sc_base + is + 4];
      const float s6 = (float)(int8_t)sc[sc_base + is + 6];
      y[n + l] = d * s0 * (float)q1;
      y[n + l + 32] = d * s2 * (float)q2;
      y[n + l + 64] = d * s4 * (float)q3;
      y[n + l + 96] = d * s6 * (float)q4;
    }
  }
}

// Block geometry of the admitted types (src/quantized_tensor_layout.rs:184,515-521).
ORC_API int orc_block_geometry(int32_t type, int64_t* elems, int64_t* bytes) {
  switch (type) {
    case T_F32: *elems = 1; *bytes = 4; return 0;
    case T_Q5_0: *elems = 32; *bytes = 22; return 0;
    case T_Q8_0: *elems = 32; *bytes = 34; return 0;
    case T_Q4_K: *elems = 256; *bytes = 144; return 0;
    case T_Q6_K: *elems = 256; *bytes = 210; return 0;
    default: return -1;
  }
}

// dequant_block — src/dequant.rs:282-305 (type dispatch; F32 passthrough is
// dequant_f32, src/dequant.rs:258-260). Returns the element count or -1.
ORC_API int orc_dequant_block(int32_t type, const uint8_t* block, float* out) {
  switch (type) {
    case T_F32: std::memcpy(out, block, 4); return 1;
    case T_Q5_0: dq_q5_0(block, out); return 32;
    case T_Q8_0: dq_q8_0(block, out); return 32;
    case T_Q4_K: dq_q4_k(block, out); return 256;
    case T_Q6_K: dq_q6_k(block, out); return 256;
    default: return -1;
  }
}

// dequant_row — src/dequant.rs:323-340: n_blocks concatenated blocks in GGUF
// block order.
ORC_API int orc_dequant_row(int32_t type, const uint8_t* packed, int64_t n_blocks, float* out) {
  int64_t be, bb;
  if (orc_block_geometry(type, &be, &bb) != 0) return -1;
  for (int64_t i = 0; i < n_blocks; ++i) orc_dequant_block(type, packed + i * bb, out + i * be);
  return 0;
}

// Flat element range [start, start+count) of a block-packed tensor — the
// slice the reference takes from its materialized f32 tensor
// (src/decoder_ops.rs:402 after src/dequant.rs:360). Rows may straddle blocks.
ORC_API int orc_dequant_range(int32_t type, const uint8_t* data, int64_t start, int64_t count,
                              float* out) {
  int64_t be, bb;
  if (orc_block_geometry(type, &be, &bb) != 0) return -1;
  if (count <= 0) return 0;
  float tmp[256];
  const int64_t first = start / be, last = (start + count - 1) / be;
  for (int64_t b = first; b <= last; ++b) {
    orc_dequant_block(type, data + b * bb, tmp);
    const int64_t b0 = b * be;
    const int64_t lo = std::max(start, b0), hi = std::min(start + count, b0 + be);
    for (int64_t e = lo; e < hi; ++e) out[e - start] = tmp[e - b0];
  }
  return 0;
}

// ---------------------------------------------------------------------------
// Decoder ops — src/decoder_ops.rs
// ---------------------------------------------------------------------------

// Sequential f32 sum of products. Rust's `Iterator::sum` for f32 folds from
// -0.0 (the additive identity that keeps the sign of an all-(-0.0) sum).
static inline float dot_seq(const float* a, const float* b, int64_t n) {
  float s = -0.0f;
  for (int64_t i = 0; i < n; ++i) s = s + a[i] * b[i];
  return s;
}

// rms_norm — src/decoder_ops.rs:126-144: f64 sum of squares, mean cast to
// f32, scale = 1/sqrt(mean+eps), y = x*scale*w.
ORC_API void orc_rms_norm(const float* x, const float* w, int64_t n, float eps, float* y) {
  double sum = -0.0;
  for (int64_t i = 0; i < n; ++i) sum = sum + (double)x[i] * (double)x[i];
  const float mean = (float)(sum / (double)n);
  const float scale = 1.0f / std::sqrt(mean + eps);
  for (int64_t i = 0; i < n; ++i) y[i] = x[i] * scale * w[i];
}

// rope_norm — src/decoder_ops.rs:166-188: consecutive pairs,
// theta = pos * base^(-(2k)/dim).
ORC_API void orc_rope_norm(const float* x, uint32_t pos, float base, int64_t dim, float* y) {
  if (y != x) std::memcpy(y, x, sizeof(float) * (size_t)dim);
  for (int64_t k = 0; k < dim / 2; ++k) {
    const float theta = (float)pos * powf(base, -(2.0f * (float)k) / (float)dim);
    const float c = cosf(theta), s = sinf(theta);
    const float x0 = y[2 * k], x1 = y[2 * k + 1];
    y[2 * k] = x0 * c - x1 * s;
    y[2 * k + 1] = x0 * s + x1 * c;
  }
}

// rope_all_heads — src/cpu_oracle.rs:658-669 (head_dim == rope dim).
ORC_API void orc_rope_all_heads(const float* x, int64_t n_heads, int64_t head_dim, uint32_t pos,
                                float base, float* y) {
  for (int64_t h = 0; h < n_heads; ++h)
    orc_rope_norm(x + h * head_dim, pos, base, head_dim, y + h * head_dim);
}

// The cos/sin pair rope_norm uses for (pos, k) — exported so the host-side
// table builder can be checked against the oracle bit for bit.
ORC_API void orc_rope_cos_sin(uint32_t pos, int64_t k, float base, int64_t dim, float* c,
                              float* s) {
  const float theta = (float)pos * powf(base, -(2.0f * (float)k) / (float)dim);
  *c = cosf(theta);
  *s = sinf(theta);
}

// silu — src/decoder_ops.rs:196-198.
ORC_API float orc_silu(float x) { return x / (1.0f + expf(-x)); }

// softmax_row — src/decoder_ops.rs:207-229.
ORC_API void orc_softmax_row(const float* s, int64_t n, float* p) {
  float mx = -INFINITY;
  for (int64_t i = 0; i < n; ++i)
    if (std::isfinite(s[i]) && s[i] > mx) mx = s[i];
  if (!std::isfinite(mx)) {
    for (int64_t i = 0; i < n; ++i) p[i] = 0.0f;
    return;
  }
  float sum = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    p[i] = expf(s[i] - mx);
    sum += p[i];
  }
  if (sum == 0.0f || !std::isfinite(sum)) {
    for (int64_t i = 0; i < n; ++i) p[i] = 0.0f;
    return;
  }
  const float inv = 1.0f / sum;
  for (int64_t i = 0; i < n; ++i) p[i] = p[i] * inv;
}

// Shared body of attention_gqa (src/cpu_oracle.rs:711-792) and the superseded
// attention_causal (src/decoder_ops.rs:258-335); they differ only in the
// head grouping (h / ratio vs h % n_kv_heads).
static int attention_impl(const float* q, const float* k, const float* v, int64_t n_q,
                          int64_t n_kv, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                          float scale, float* ctx, bool modulo_grouping) {
  if (n_q > n_kv || n_kv_heads <= 0 || n_heads % n_kv_heads != 0) return -1;
  const int64_t q_span = n_heads * head_dim, kv_span = n_kv_heads * head_dim;
  const int64_t ratio = n_heads / n_kv_heads;
  int rc = 0;
#pragma omp parallel for collapse(2) num_threads(g_threads) schedule(static)
  for (int64_t i = 0; i < n_q; ++i) {
    for (int64_t h = 0; h < n_heads; ++h) {
      const int64_t gpos = n_kv - n_q + i;
      const int64_t row = i * q_span;
      const int64_t kh = modulo_grouping ? (h % n_kv_heads) : (h / ratio);
      const float* qh = q + row + h * head_dim;
      std::vector<float> scores((size_t)(gpos + 1)), probs((size_t)(gpos + 1));
      for (int64_t j = 0; j <= gpos; ++j) {
        const float* kj = k + j * kv_span + kh * head_dim;
        float dot = 0.0f;
        for (int64_t d = 0; d < head_dim; ++d) dot += qh[d] * kj[d];
        scores[(size_t)j] = dot * scale;
      }
      orc_softmax_row(scores.data(), gpos + 1, probs.data());
      float* out = ctx + row + h * head_dim;
      for (int64_t d = 0; d < head_dim; ++d) {
        float acc = 0.0f;
        for (int64_t j = 0; j <= gpos; ++j) acc += probs[(size_t)j] * v[j * kv_span + kh * head_dim + d];
        out[d] = acc;
      }
    }
  }
  return rc;
}

// attention_gqa — src/cpu_oracle.rs:711-792 (verified grouping h / ratio).
ORC_API int orc_attention_gqa(const float* q, const float* k, const float* v, int64_t n_q,
                              int64_t n_kv, int64_t n_heads, int64_t n_kv_heads, int64_t head_dim,
                              float scale, float* ctx) {
  return attention_impl(q, k, v, n_q, n_kv, n_heads, n_kv_heads, head_dim, scale, ctx, false);
}

// attention_causal — src/decoder_ops.rs:258-335 (superseded grouping h % n_kv).
ORC_API int orc_attention_causal(const float* q, const float* k, const float* v, int64_t n_q,
                                 int64_t n_kv, int64_t n_heads, int64_t n_kv_heads,
                                 int64_t head_dim, float scale, float* ctx) {
  return attention_impl(q, k, v, n_q, n_kv, n_heads, n_kv_heads, head_dim, scale, ctx, true);
}

// swiglu — src/decoder_ops.rs:351-362.
ORC_API void orc_swiglu(const float* g, const float* u, int64_t n, float* y) {
  for (int64_t i = 0; i < n; ++i) y[i] = orc_silu(g[i]) * u[i];
}

// dense — src/decoder_ops.rs:378-406, f32 weights, K-major rows.
ORC_API void orc_dense(const float* w, const float* x, int64_t in, int64_t out, float* y) {
#pragma omp parallel for num_threads(g_threads) schedule(static)
  for (int64_t j = 0; j < out; ++j) y[j] = dot_seq(x, w + j * in, in);
}

// dense over a block-packed tensor with the weights dequantized row by row
// (and f16-rounded when f16_round != 0, src/cpu_oracle.rs:356-360) — the same
// operands the reference's materialized dense sees.
ORC_API int orc_dense_q(int32_t type, const uint8_t* data, int64_t in, int64_t out,
                        const float* x, float* y, int f16_round) {
  int64_t be, bb;
  if (orc_block_geometry(type, &be, &bb) != 0) return -1;
#pragma omp parallel num_threads(g_threads)
  {
    std::vector<float> row((size_t)in);
#pragma omp for schedule(static)
    for (int64_t j = 0; j < out; ++j) {
      orc_dequant_range(type, data, j * in, in, row.data());
      if (f16_round)
        for (int64_t i = 0; i < in; ++i) row[(size_t)i] = orc_f16_round(row[(size_t)i]);
      y[j] = dot_seq(x, row.data(), in);
    }
  }
  return 0;
}

// residual_add — src/decoder_ops.rs:420-427.
ORC_API void orc_residual_add(const float* a, const float* b, int64_t n, float* y) {
  for (int64_t i = 0; i < n; ++i) y[i] = a[i] + b[i];
}

// log_softmax — src/cpu_oracle.rs:942-968. Returns 0, or -1 when the finite
// gate fails (empty input, non-finite logit, bad denominator).
ORC_API int orc_log_softmax(const float* x, int64_t n, float* out) {
  if (n <= 0) return -1;
  float mx = -INFINITY;
  for (int64_t i = 0; i < n; ++i) {
    if (!std::isfinite(x[i])) return -1;
    if (x[i] > mx) mx = x[i];
  }
  float sum = 0.0f;
  for (int64_t i = 0; i < n; ++i) sum += expf(x[i] - mx);
  if (!std::isfinite(sum) || sum == 0.0f) return -1;
  const float ln_sum = logf(sum);
  for (int64_t i = 0; i < n; ++i) out[i] = (x[i] - mx) - ln_sum;
  return 0;
}

// top1_non_eog — src/cpu_oracle.rs:979-995: strict '>' so the lowest index
// wins ties; EOG ids skipped; all-masked -> 0.
ORC_API int64_t orc_top1_non_eog(const float* logits, int64_t n, const int64_t* eog,
                                 int64_t n_eog) {
  int64_t best = -1;
  float best_val = -INFINITY;
  for (int64_t t = 0; t < n; ++t) {
    bool skip = false;
    for (int64_t e = 0; e < n_eog; ++e) skip = skip || (eog[e] == t);
    if (skip) continue;
    if (logits[t] > best_val) {
      best_val = logits[t];
      best = t;
    }
  }
  return best < 0 ? 0 : best;
}

ORC_API void orc_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
ORC_API int orc_get_threads(void) { return g_threads; }

// ---------------------------------------------------------------------------
// Model + incremental runner — src/cpu_oracle.rs:409-445, 808-926
// ---------------------------------------------------------------------------

namespace {

struct TensorRef {
  int32_t type = -1;
  const uint8_t* data = nullptr;
  int64_t rows = 0, cols = 0;  // rows = out_features, cols = in_features
};

enum Slot : int {
  S_ATTN_NORM = 0, S_Q = 1, S_K = 2, S_V = 3, S_O = 4, S_FFN_NORM = 5,
  S_GATE = 6, S_UP = 7, S_DOWN = 8, N_SLOTS = 9
};
enum GSlot : int { G_TOKEN_EMBD = 0, G_OUTPUT_NORM = 1, G_OUTPUT = 2, N_GSLOTS = 3 };

struct Model {
  int32_t n_layers, d, n_heads, n_kv_heads, head_dim, ffn, vocab, tied;
  float eps, theta;
  std::vector<TensorRef> layer;  // n_layers * N_SLOTS
  TensorRef global[N_GSLOTS];
};

// Layer intermediates of the last push_token, kept for layer-level parity.
enum Trace : int {
  TR_ATTN_IN = 0, TR_Q_ROT = 1, TR_K_ROT = 2, TR_V = 3, TR_CTX = 4, TR_H2 = 5,
  TR_HH = 6, TR_H_OUT = 7, N_TRACE = 8
};

struct Run {
  const Model* m;
  int64_t n = 0;
  int64_t max_ctx;
  std::vector<float> h_last;
  std::vector<std::vector<float>> k_cache, v_cache;  // per layer [n][Hkv*hd]
  bool trace = false;
  std::vector<std::vector<float>> tr;  // n_layers * N_TRACE
};

// Dense through a TensorRef with the reference's f16 weight rounding
// (metal_f16_round_weights is applied to every materialized weight except
// output_norm, src/cpu_oracle.rs:323-331,420-421,434).
void dense_ref(const TensorRef& t, const float* x, float* y) {
  if (t.type == T_F32) {
    // f32 tensor (e.g. the tied token_embd head): rounded through f16 on use.
    const float* w = reinterpret_cast<const float*>(t.data);
#pragma omp parallel num_threads(g_threads)
    {
      std::vector<float> row((size_t)t.cols);
#pragma omp for schedule(static)
      for (int64_t j = 0; j < t.rows; ++j) {
        for (int64_t i = 0; i < t.cols; ++i) row[(size_t)i] = orc_f16_round(w[j * t.cols + i]);
        y[j] = dot_seq(x, row.data(), t.cols);
      }
    }
  } else {
    orc_dense_q(t.type, t.data, t.cols, t.rows, x, y, 1);
  }
}

void norm_weight(const TensorRef& t, int64_t n, bool round, std::vector<float>& out) {
  out.resize((size_t)n);
  if (t.type == T_F32) {
    const float* w = reinterpret_cast<const float*>(t.data);
    for (int64_t i = 0; i < n; ++i) out[(size_t)i] = round ? orc_f16_round(w[i]) : w[i];
  } else {
    orc_dequant_range(t.type, t.data, 0, n, out.data());
    if (round)
      for (auto& v : out) v = orc_f16_round(v);
  }
}

}  // namespace

// cfg_i = {n_layers, d_model, n_heads, n_kv_heads, head_dim, ffn, vocab, tied_head}
// cfg_f = {rms_eps, rope_theta}
ORC_API void* orc_model_new(const int32_t* cfg_i, const float* cfg_f) {
  Model* m = new (std::nothrow) Model();
  if (!m) return nullptr;
  m->n_layers = cfg_i[0]; m->d = cfg_i[1]; m->n_heads = cfg_i[2]; m->n_kv_heads = cfg_i[3];
  m->head_dim = cfg_i[4]; m->ffn = cfg_i[5]; m->vocab = cfg_i[6]; m->tied = cfg_i[7];
  m->eps = cfg_f[0]; m->theta = cfg_f[1];
  m->layer.assign((size_t)m->n_layers * N_SLOTS, TensorRef());
  return m;
}

ORC_API void orc_model_free(void* p) { delete static_cast<Model*>(p); }

// Register one tensor (the caller keeps the bytes alive). layer = -1 selects
// the global slots (token_embd, output_norm, output).
ORC_API int orc_model_set(void* p, int32_t layer, int32_t slot, int32_t type, const void* data,
                          int64_t rows, int64_t cols) {
  Model* m = static_cast<Model*>(p);
  TensorRef t;
  t.type = type; t.data = static_cast<const uint8_t*>(data); t.rows = rows; t.cols = cols;
  if (layer < 0) {
    if (slot < 0 || slot >= N_GSLOTS) return -1;
    m->global[slot] = t;
  } else {
    if (layer >= m->n_layers || slot < 0 || slot >= N_SLOTS) return -1;
    m->layer[(size_t)layer * N_SLOTS + slot] = t;
  }
  return 0;
}

ORC_API void* orc_run_new(void* model, int64_t max_ctx, int trace) {
  const Model* m = static_cast<const Model*>(model);
  Run* r = new (std::nothrow) Run();
  if (!r) return nullptr;
  r->m = m;
  r->max_ctx = max_ctx;
  r->h_last.assign((size_t)m->d, 0.0f);
  r->k_cache.assign((size_t)m->n_layers, {});
  r->v_cache.assign((size_t)m->n_layers, {});
  r->trace = trace != 0;
  if (r->trace) r->tr.assign((size_t)m->n_layers * N_TRACE, {});
  return r;
}

ORC_API void orc_run_free(void* p) { delete static_cast<Run*>(p); }
ORC_API int64_t orc_run_len(void* p) { return static_cast<Run*>(p)->n; }

// Install an f32 K/V prefix of n positions for every layer (values are
// rounded through f16 like every cached K/V). Lets a long-context decode be
// checked without running the prefix through this oracle.
ORC_API int orc_run_set_prefix(void* p, int32_t layer, const float* k, const float* v,
                               int64_t n) {
  Run* r = static_cast<Run*>(p);
  const Model* m = r->m;
  if (layer < 0 || layer >= m->n_layers) return -1;
  const int64_t span = (int64_t)m->n_kv_heads * m->head_dim;
  auto& kc = r->k_cache[(size_t)layer];
  auto& vc = r->v_cache[(size_t)layer];
  kc.resize((size_t)(n * span));
  vc.resize((size_t)(n * span));
  for (int64_t i = 0; i < n * span; ++i) {
    kc[(size_t)i] = orc_f16_round(k[i]);
    vc[(size_t)i] = orc_f16_round(v[i]);
  }
  r->n = n;
  return 0;
}

// ForwardRun::push_token — src/cpu_oracle.rs:859-912.
// Returns 0, -1 token out of range, -2 context full.
ORC_API int orc_run_push(void* p, int64_t token) {
  Run* r = static_cast<Run*>(p);
  const Model* m = r->m;
  if (token < 0 || token >= m->vocab) return -1;
  if (r->n >= r->max_ctx) return -2;
  const int64_t d = m->d, H = m->n_heads, Hkv = m->n_kv_heads, hd = m->head_dim, F = m->ffn;
  const int64_t qspan = H * hd, kvspan = Hkv * hd;
  const uint32_t pos = (uint32_t)r->n;
  const float scale = 1.0f / sqrtf((float)hd);

  // embed_rows — src/cpu_oracle.rs:538-545, token_embd already f16-rounded
  // at build (src/cpu_oracle.rs:420-421).
  std::vector<float> h((size_t)d);
  {
    const TensorRef& e = m->global[G_TOKEN_EMBD];
    if (e.type == T_F32) {
      const float* w = reinterpret_cast<const float*>(e.data) + token * d;
      for (int64_t i = 0; i < d; ++i) h[(size_t)i] = orc_f16_round(w[i]);
    } else {
      orc_dequant_range(e.type, e.data, token * d, d, h.data());
      for (auto& v : h) v = orc_f16_round(v);
    }
  }
  std::vector<float> a((size_t)d), q((size_t)qspan), k((size_t)kvspan), v((size_t)kvspan);
  std::vector<float> qr((size_t)qspan), kr((size_t)kvspan), ctx((size_t)qspan), o((size_t)d);
  std::vector<float> h2((size_t)d), f((size_t)d), g((size_t)F), u((size_t)F), hh((size_t)F),
      dn((size_t)d), wn;
  for (int64_t il = 0; il < m->n_layers; ++il) {
    const TensorRef* L = &m->layer[(size_t)il * N_SLOTS];
    norm_weight(L[S_ATTN_NORM], d, true, wn);
    orc_rms_norm(h.data(), wn.data(), d, m->eps, a.data());
    dense_ref(L[S_Q], a.data(), q.data());
    dense_ref(L[S_K], a.data(), k.data());
    dense_ref(L[S_V], a.data(), v.data());
    orc_rope_all_heads(q.data(), H, hd, pos, m->theta, qr.data());
    orc_rope_all_heads(k.data(), Hkv, hd, pos, m->theta, kr.data());
    auto& kc = r->k_cache[(size_t)il];
    auto& vc = r->v_cache[(size_t)il];
    for (int64_t i = 0; i < kvspan; ++i) kc.push_back(orc_f16_round(kr[(size_t)i]));
    for (int64_t i = 0; i < kvspan; ++i) vc.push_back(orc_f16_round(v[(size_t)i]));
    orc_attention_gqa(qr.data(), kc.data(), vc.data(), 1, r->n + 1, H, Hkv, hd, scale, ctx.data());
    dense_ref(L[S_O], ctx.data(), o.data());
    orc_residual_add(h.data(), o.data(), d, h2.data());
    norm_weight(L[S_FFN_NORM], d, true, wn);
    orc_rms_norm(h2.data(), wn.data(), d, m->eps, f.data());
    dense_ref(L[S_GATE], f.data(), g.data());
    dense_ref(L[S_UP], f.data(), u.data());
    orc_swiglu(g.data(), u.data(), F, hh.data());
    dense_ref(L[S_DOWN], hh.data(), dn.data());
    std::vector<float> hin;
    if (r->trace) hin = h;
    orc_residual_add(h2.data(), dn.data(), d, h.data());
    if (r->trace) {
      auto* T = &r->tr[(size_t)il * N_TRACE];
      T[TR_ATTN_IN] = a; T[TR_Q_ROT] = qr; T[TR_K_ROT] = kr; T[TR_V] = v; T[TR_CTX] = ctx;
      T[TR_H2] = h2; T[TR_HH] = hh; T[TR_H_OUT] = h;
    }
  }
  r->n += 1;
  r->h_last = h;
  return 0;
}

// Layer intermediates of the last push (trace mode); returns the element
// count copied, or -1.
ORC_API int64_t orc_run_trace(void* p, int32_t layer, int32_t which, float* out) {
  Run* r = static_cast<Run*>(p);
  if (!r->trace || layer < 0 || layer >= r->m->n_layers || which < 0 || which >= N_TRACE)
    return -1;
  const auto& t = r->tr[(size_t)layer * N_TRACE + which];
  std::memcpy(out, t.data(), t.size() * sizeof(float));
  return (int64_t)t.size();
}

ORC_API int orc_run_hidden(void* p, float* out) {
  Run* r = static_cast<Run*>(p);
  std::memcpy(out, r->h_last.data(), r->h_last.size() * sizeof(float));
  return 0;
}

// ForwardRun::position_logits — src/cpu_oracle.rs:920-926 (output_norm is
// NOT f16-rounded, src/cpu_oracle.rs:434; the head is the tied token_embd or
// a separate output tensor).
ORC_API int orc_run_logits(void* p, float* logits) {
  Run* r = static_cast<Run*>(p);
  const Model* m = r->m;
  if (r->n == 0) return -1;
  std::vector<float> wn, normed((size_t)m->d);
  norm_weight(m->global[G_OUTPUT_NORM], m->d, false, wn);
  orc_rms_norm(r->h_last.data(), wn.data(), m->d, m->eps, normed.data());
  TensorRef head = m->tied ? m->global[G_TOKEN_EMBD] : m->global[G_OUTPUT];
  head.rows = m->vocab;
  head.cols = m->d;
  dense_ref(head, normed.data(), logits);
  return 0;
}

// run_greedy — src/greedy_run.rs:186-248: prompt through ForwardRun, then at
// each step logits -> finite gate -> top1_non_eog -> feed back. Returns 0,
// -1 bad token, -2 context full, -3 empty prompt; *all_finite receives the
// finite gate. logits_out (optional) receives n_gen x vocab logits.
ORC_API int orc_run_greedy(void* model, const int64_t* prompt, int64_t n_prompt, int64_t n_gen,
                           const int64_t* eog, int64_t n_eog, int64_t* out_tokens,
                           float* logits_out, int32_t* all_finite) {
  const Model* m = static_cast<const Model*>(model);
  if (n_prompt <= 0) return -3;
  Run* r = static_cast<Run*>(orc_run_new(model, n_prompt + n_gen, 0));
  int rc = 0;
  for (int64_t i = 0; i < n_prompt && rc == 0; ++i) rc = orc_run_push(r, prompt[i]);
  std::vector<float> logits((size_t)m->vocab), logp((size_t)m->vocab);
  int32_t finite = 1;
  for (int64_t i = 0; i < n_gen && rc == 0; ++i) {
    orc_run_logits(r, logits.data());
    if (orc_log_softmax(logits.data(), m->vocab, logp.data()) != 0) finite = 0;
    const int64_t tok = orc_top1_non_eog(logits.data(), m->vocab, eog, n_eog);
    out_tokens[i] = tok;
    if (logits_out) std::memcpy(logits_out + i * m->vocab, logits.data(), sizeof(float) * (size_t)m->vocab);
    if (i + 1 < n_gen) rc = orc_run_push(r, tok);
  }
  if (all_finite) *all_finite = finite;
  orc_run_free(r);
  return rc;
}
