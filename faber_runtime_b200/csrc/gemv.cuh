// gemv.cuh — fused Q4_K dequant-GEMV for batch-1 decode (sm_100a).
//
// y[j] = sum_i w[j][i] * x[i] with w[j][i] = f16(f32(d*sc*q - dmin*m)), the
// reference's dense (src/decoder_ops.rs:378-406) over dequant_q4_k
// (src/dequant.rs:194-217) after metal_f16_round_weights
// (src/cpu_oracle.rs:356-360).
//
// Data path per warp and 16-row tile:
//   * 16-byte streaming loads of the Q4_K tile (headers + quants); each lane
//     owns one 32-byte quant chunk (two sub-blocks) of two rows;
//   * per weight: a mask-or against the 2^23 magic turns a nibble into an
//     exact float, then one packed f32x2 FMA computes d1*q - m1 with a single
//     rounding (d1*q is exact, so this equals the reference's separately
//     rounded multiply then subtract), and one cvt.rn.f16x2 rounds two
//     weights to f16 exactly as the reference does — the packed result is
//     already the tensor-core A operand;
//   * x is staged once per CTA in shared memory as an exact two-term f16
//     split (x*2^-s = hi + lo, s a power-of-two scale from max|x|), and
//     mma.sync m16n8k16 (f16 x f16 -> f32) multiplies the 16x16 weight tile
//     by [hi, lo]: column 0 and 1 of the accumulator sum to y*2^-s. The
//     tensor core is the reduction engine (no shuffles);
//   * warps split K (super-blocks) and the CTA reduces the 8 partial tiles
//     in shared memory in a fixed order (deterministic), then runs a fused
//     epilogue (store / residual add / RoPE + KV-cache append / SwiGLU /
//     logits + argmax).
#pragma once

#include "common.cuh"

namespace faber {

// PRO_NORM_RES: x = x + x2 (the residual add deferred from a tensor-parallel
// all-reduce), written back by CTA 0, then rms_norm as PRO_NORM.
enum GemvPrologue : int { PRO_PLAIN = 0, PRO_NORM = 1, PRO_NORM_RES = 2 };
enum GemvEpilogue : int { EPI_STORE = 0, EPI_RESID = 1, EPI_QKV = 2, EPI_SWIGLU = 3, EPI_LOGITS = 4 };
enum GemvLayout : int { WL_TILED = 0, WL_NATIVE = 1, WL_F16 = 2 };

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kXPad = 256;  // zero halo (elements) in front of x for row offsets
constexpr int kMaxEog = 8;

struct GemvArgs {
  const uint8_t* w;          // weights (layout per template parameter)
  int32_t n_tiles;           // 16-row tiles
  int32_t nb;                // 256-element super-block columns per row
  int32_t n_rows;            // true output rows
  int32_t n_cols;            // true input length
  const int32_t* tile_xoff;  // per-tile element offset of x (tiled layout), or null
  const int32_t* row_map;    // [n_tiles*16] output row of each tile row (-1 pad), or null
  const float* x;            // input (PRO_PLAIN: the vector; PRO_NORM: the residual stream)
  const float* x2;           // PRO_NORM_RES: second residual term
  float* x_sum_out;          // PRO_NORM_RES: x + x2 (CTA 0 writes)
  const float* norm_w;       // PRO_NORM weight
  float eps;
  float* x_norm_out;         // optional copy of the normalized input (CTA 0 writes)
  float* out;
  const float* res;          // EPI_RESID: out = res + y (may alias out)
  // EPI_QKV
  float* q_out;
  __half* k_cache;           // this layer's K cache [ctx][kv_stride]
  __half* v_cache;
  const float2* rope;        // [ctx][head_dim/2] (cos, sin)
  const int32_t* pos_ptr;    // current position
  int32_t nq, nk, head_dim;
  float* k_trace;            // optional f32 copies of k_rot / v (tracing)
  float* v_trace;
  // EPI_LOGITS
  unsigned long long* argmax_key;
  int32_t* finite_flag;
  int32_t n_eog;
  int32_t row_offset;        // global index of local row 0 (vocab shard)
  int64_t eog[kMaxEog];
};

// Padded shared-memory index of virtual x element v (8 halves of padding
// every 64 keeps the B-fragment reads of the four lane groups on distinct
// banks).
__device__ __forceinline__ int xs_index(int v) { return v + ((v >> 6) << 3); }

__host__ __device__ inline int gemv_xs_halves(int nb) {
  const int n = kXPad + nb * 256;
  const int base = n + ((n >> 6) << 3);
  // tail so that the lo array starts 64 bytes off the hi array's bank phase
  return ((base * 2) % 128 == 64) ? base + 64 : base + 32;
}

// ---------------------------------------------------------------------------
// Block reductions (fixed order: deterministic and identical in every CTA)
// ---------------------------------------------------------------------------
__device__ __forceinline__ double block_sum_f64(double v, double* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double s = 0.0;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[w];
  return s;
}

__device__ __forceinline__ float block_max_f32(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = 0.0f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
  return m;
}

// Power-of-two scale that brings max|x| into [2^13, 2^14).
__device__ __forceinline__ int split_shift(float bound) {
  if (!(bound > 0.0f) || !isfinite(bound)) return 0;
  int e;
  frexpf(bound, &e);
  int s = e - 14;
  return max(-100, min(100, s));
}

// Stage x (or rms_norm(x) * w) into shared memory as the hi/lo f16 split.
// Returns the output scale 2^s.
template <int PRO>
__device__ float stage_x(const GemvArgs& a, __half* xh, __half* xl, double* redd, float* redf) {
  const int n = a.n_cols;
  double ss = 0.0;
  float mx = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = (PRO == PRO_NORM_RES) ? a.x[i] + a.x2[i] : a.x[i];
    if (PRO != PRO_PLAIN) {
      ss += (double)v * (double)v;
      mx = fmaxf(mx, fabsf(v * a.norm_w[i]));
    } else {
      mx = fmaxf(mx, fabsf(v));
    }
  }
  float scale = 1.0f;
  float bound;
  if (PRO != PRO_PLAIN) {
    // rms_norm (src/decoder_ops.rs:126-144): f64 sum, mean cast to f32,
    // scale = 1/sqrt(mean + eps).
    const double tot = block_sum_f64(ss, redd);
    const float mean = (float)(tot / (double)n);
    scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
    bound = block_max_f32(mx, redf) * scale * 1.001f;
  } else {
    bound = block_max_f32(mx, redf);
  }
  const int s = split_shift(bound);
  const float in_s = ldexpf(1.0f, -s);
  const int total = kXPad + a.nb * 256;
  for (int p = threadIdx.x; p < total / 2; p += blockDim.x) {
    const int v0 = 2 * p - kXPad;
    float val[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int v = v0 + k;
      float x = 0.0f;
      if (v >= 0 && v < n) {
        x = a.x[v];
        if (PRO == PRO_NORM_RES) {
          x = x + a.x2[v];
          if (blockIdx.x == 0) a.x_sum_out[v] = x;
        }
        if (PRO != PRO_PLAIN) {
          x = __fmul_rn(__fmul_rn(x, scale), a.norm_w[v]);
          if (a.x_norm_out && blockIdx.x == 0) a.x_norm_out[v] = x;
        }
      }
      val[k] = x * in_s;
    }
    const __half2 hi = __floats2half2_rn(val[0], val[1]);
    const float2 hf = __half22float2(hi);
    const __half2 lo = __floats2half2_rn(val[0] - hf.x, val[1] - hf.y);
    const int idx = xs_index(2 * p);
    *reinterpret_cast<__half2*>(xh + idx) = hi;
    *reinterpret_cast<__half2*>(xl + idx) = lo;
  }
  __syncthreads();
  return ldexpf(1.0f, s);
}

// ---------------------------------------------------------------------------
// Weight item: one 16-row tile x one 256-element super-block column
// ---------------------------------------------------------------------------
struct Q4Regs {
  uint4 hA, hB;        // headers of rows g and g+8
  uint4 qA0, qA1;      // quant chunk t (32 bytes) of row g
  uint4 qB0, qB1;      // ... of row g+8
};

template <int WL>
__device__ __forceinline__ void q4_load(const GemvArgs& a, int tile, int b, int g, int t,
                                        Q4Regs& r) {
  if (WL == WL_TILED) {
    const uint8_t* base = a.w + ((size_t)tile * a.nb + b) * kTileItemBytes;
    r.hA = ldg_stream(base + 16 * g);
    r.hB = ldg_stream(base + 16 * (g + 8));
    const uint8_t* qa = base + 256 + 128 * g + 32 * t;
    const uint8_t* qb = qa + 128 * 8;
    r.qA0 = ldg_stream(qa);
    r.qA1 = ldg_stream(qa + 16);
    r.qB0 = ldg_stream(qb);
    r.qB1 = ldg_stream(qb + 16);
  } else {
    const int ra = tile * kTileRows + g, rb = ra + 8;
    const uint4 z = make_uint4(0, 0, 0, 0);
    r.hA = r.hB = r.qA0 = r.qA1 = r.qB0 = r.qB1 = z;
    if (ra < a.n_rows) {
      const uint8_t* p = a.w + ((size_t)ra * a.nb + b) * kQ4kBlockBytes;
      r.hA = ldg_stream(p);
      r.qA0 = ldg_stream(p + 16 + 32 * t);
      r.qA1 = ldg_stream(p + 32 + 32 * t);
    }
    if (rb < a.n_rows) {
      const uint8_t* p = a.w + ((size_t)rb * a.nb + b) * kQ4kBlockBytes;
      r.hB = ldg_stream(p);
      r.qB0 = ldg_stream(p + 16 + 32 * t);
      r.qB1 = ldg_stream(p + 32 + 32 * t);
    }
  }
}

// Per-row scale constants for this lane's two sub-blocks (2t low nibbles,
// 2t+1 high nibbles): get_scale_min_k4 (src/dequant.rs:178-187) for all
// eight sub-blocks at once as packed bytes, then d1 = d*sc, m1 = dmin*m.
struct RowScales {
  float2 lo01, lo23, hi01, hi23;  // d1 and d2 pre-scaled per nibble position
  float2 nm1, nm2;                // (-m1, -m1), (-m2, -m2)
};

__device__ __forceinline__ RowScales row_scales(const uint4 h, int t) {
  const float d = __half2float(__ushort_as_half((unsigned short)(h.x & 0xffffu)));
  const float dmin = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
  const uint32_t s0 = h.y, s1 = h.z, s2 = h.w;
  uint32_t sc, mm;
  if (t < 2) {
    sc = s0 & 0x3f3f3f3fu;
    mm = s1 & 0x3f3f3f3fu;
  } else {
    sc = (s2 & 0x0f0f0f0fu) | ((s0 >> 2) & 0x30303030u);
    mm = ((s2 >> 4) & 0x0f0f0f0fu) | ((s1 >> 2) & 0x30303030u);
  }
  const int sh = (t & 1) * 16;
  const float sc_lo = (float)((sc >> sh) & 0xffu), sc_hi = (float)((sc >> (sh + 8)) & 0xffu);
  const float m_lo = (float)((mm >> sh) & 0xffu), m_hi = (float)((mm >> (sh + 8)) & 0xffu);
  const float d1 = __fmul_rn(d, sc_lo), d2 = __fmul_rn(d, sc_hi);
  const float m1 = __fmul_rn(dmin, m_lo), m2 = __fmul_rn(dmin, m_hi);
  RowScales r;
  r.lo01 = make_float2(d1, d1 * 0x1p-8f);
  r.lo23 = make_float2(d1 * 0x1p-16f, d1 * 0x1p-12f);
  r.hi01 = make_float2(d2 * 0x1p-4f, d2 * 0x1p-12f);
  r.hi23 = make_float2(d2 * 0x1p-8f, d2 * 0x1p-16f);
  r.nm1 = make_float2(-m1, -m1);
  r.nm2 = make_float2(-m2, -m2);
  return r;
}

// Dequantize the 8 nibbles of one quant word into four f16x2 A-operand
// registers: lo = (e, e+1), (e+2, e+3) of the low sub-block; hi = the same
// slots of the high sub-block.
__device__ __forceinline__ void dequant_word(uint32_t w, const RowScales& s, uint32_t& lo0,
                                             uint32_t& lo2, uint32_t& hi0, uint32_t& hi2) {
  constexpr uint32_t M = 0x4b000000u;  // 2^23
  const float2 negM = make_float2(-8388608.0f, -8388608.0f);
  const uint32_t u = w >> 12;
  float2 f01 = make_float2(u2f((w & 0x0000000fu) | M), u2f((w & 0x00000f00u) | M));
  float2 f23 = make_float2(u2f((w & 0x000f0000u) | M), u2f((u & 0x0000f000u) | M));
  float2 h01 = make_float2(u2f((w & 0x000000f0u) | M), u2f((w & 0x0000f000u) | M));
  float2 h23 = make_float2(u2f((u & 0x00000f00u) | M), u2f((u & 0x000f0000u) | M));
  f01 = __ffma2_rn(__fadd2_rn(f01, negM), s.lo01, s.nm1);
  f23 = __ffma2_rn(__fadd2_rn(f23, negM), s.lo23, s.nm1);
  h01 = __ffma2_rn(__fadd2_rn(h01, negM), s.hi01, s.nm2);
  h23 = __ffma2_rn(__fadd2_rn(h23, negM), s.hi23, s.nm2);
  lo0 = pack_half2(f01.x, f01.y);
  lo2 = pack_half2(f23.x, f23.y);
  hi0 = pack_half2(h01.x, h01.y);
  hi2 = pack_half2(h23.x, h23.y);
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// 16 MMAs of one Q4_K item into the warp accumulators.
__device__ __forceinline__ void q4_compute(const Q4Regs& r, int t, int g, const __half* xsrc,
                                           int xbase, float acc[4]) {
  const RowScales sA = row_scales(r.hA, t);
  const RowScales sB = row_scales(r.hB, t);
#pragma unroll
  for (int pp = 0; pp < 2; ++pp) {
    const uint4 qa = pp ? r.qA1 : r.qA0;
    const uint4 qb = pp ? r.qB1 : r.qB0;
    // B fragments: elements e = 64t + 32n + 16pp + 4i of this super-block.
    uint4 xb_lo0 = make_uint4(0, 0, 0, 0), xb_lo1 = xb_lo0, xb_hi0 = xb_lo0, xb_hi1 = xb_lo0;
    if (g < 2) {
      const int e0 = xbase + 64 * t + 16 * pp;
      xb_lo0 = *reinterpret_cast<const uint4*>(xsrc + xs_index(e0));
      xb_lo1 = *reinterpret_cast<const uint4*>(xsrc + xs_index(e0 + 8));
      xb_hi0 = *reinterpret_cast<const uint4*>(xsrc + xs_index(e0 + 32));
      xb_hi1 = *reinterpret_cast<const uint4*>(xsrc + xs_index(e0 + 40));
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t aL0, aL2, aH0, aH2, bL0, bL2, bH0, bH2;
      dequant_word(word_of(qa, i), sA, aL0, aL2, aH0, aH2);
      dequant_word(word_of(qb, i), sB, bL0, bL2, bH0, bH2);
      const uint4& xl = (i < 2) ? xb_lo0 : xb_lo1;
      const uint4& xh = (i < 2) ? xb_hi0 : xb_hi1;
      const uint32_t xl0 = (i & 1) ? xl.z : xl.x, xl1 = (i & 1) ? xl.w : xl.y;
      const uint32_t xh0 = (i & 1) ? xh.z : xh.x, xh1 = (i & 1) ? xh.w : xh.y;
      mma_16816(acc[0], acc[1], acc[2], acc[3], aL0, bL0, aL2, bL2, xl0, xl1);
      mma_16816(acc[0], acc[1], acc[2], acc[3], aH0, bH0, aH2, bH2, xh0, xh1);
    }
  }
}

// F16 weights (the tied token_embd head): row-major [rows][cols] halves.
struct F16Regs {
  uint4 a[8], b[8];  // 64 halves of rows g and g+8 (this lane's chunk)
};

__device__ __forceinline__ void f16_load(const GemvArgs& a, int tile, int b, int g, int t,
                                         F16Regs& r) {
  const int ra = tile * kTileRows + g, rb = ra + 8;
  const __half* w = reinterpret_cast<const __half*>(a.w);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    r.a[k] = make_uint4(0, 0, 0, 0);
    r.b[k] = make_uint4(0, 0, 0, 0);
  }
  if (ra < a.n_rows) {
    const __half* p = w + (size_t)ra * a.n_cols + b * 256 + 64 * t;
#pragma unroll
    for (int k = 0; k < 8; ++k) r.a[k] = ldg_stream(p + 8 * k);
  }
  if (rb < a.n_rows) {
    const __half* p = w + (size_t)rb * a.n_cols + b * 256 + 64 * t;
#pragma unroll
    for (int k = 0; k < 8; ++k) r.b[k] = ldg_stream(p + 8 * k);
  }
}

__device__ __forceinline__ void f16_compute(const F16Regs& r, int t, int g, const __half* xsrc,
                                            int xbase, float acc[4]) {
#pragma unroll
  for (int n = 0; n < 2; ++n) {
#pragma unroll
    for (int pp = 0; pp < 2; ++pp) {
      uint4 x0 = make_uint4(0, 0, 0, 0), x1 = x0;
      if (g < 2) {
        const int e0 = xbase + 64 * t + 32 * n + 16 * pp;
        x0 = *reinterpret_cast<const uint4*>(xsrc + xs_index(e0));
        x1 = *reinterpret_cast<const uint4*>(xsrc + xs_index(e0 + 8));
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        // offset 32n + 16pp + 4i inside the lane's 64-half chunk
        const int k = 4 * n + 2 * pp + (i >> 1);
        const uint4 va = r.a[k], vb = r.b[k];
        const uint32_t a0 = (i & 1) ? va.z : va.x, a2 = (i & 1) ? va.w : va.y;
        const uint32_t a1 = (i & 1) ? vb.z : vb.x, a3 = (i & 1) ? vb.w : vb.y;
        const uint4& xv = (i < 2) ? x0 : x1;
        const uint32_t b0 = (i & 1) ? xv.z : xv.x, b1 = (i & 1) ? xv.w : xv.y;
        mma_16816(acc[0], acc[1], acc[2], acc[3], a0, a1, a2, a3, b0, b1);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Epilogue: one thread per row pair of the finished tile
// ---------------------------------------------------------------------------
template <int EPI>
__device__ __forceinline__ void gemv_epilogue(const GemvArgs& a, int tile, int pair, float y0,
                                              float y1) {
  const int i0 = 2 * pair, i1 = i0 + 1;
  int r0 = tile * kTileRows + i0, r1 = tile * kTileRows + i1;
  if (a.row_map) {
    r0 = a.row_map[tile * kTileRows + i0];
    r1 = a.row_map[tile * kTileRows + i1];
  }
  const bool v0 = r0 >= 0 && r0 < a.n_rows, v1 = r1 >= 0 && r1 < a.n_rows;
  if (EPI == EPI_STORE) {
    if (v0) a.out[r0] = y0;
    if (v1) a.out[r1] = y1;
  } else if (EPI == EPI_RESID) {
    // residual_add (src/decoder_ops.rs:420-427)
    if (v0) a.out[r0] = a.res[r0] + y0;
    if (v1) a.out[r1] = a.res[r1] + y1;
  } else if (EPI == EPI_QKV) {
    if (!v0) return;
    const int pos = *a.pos_ptr;
    const int kv_stride = a.nk;
    if (r0 < a.nq + a.nk) {
      // rope_norm consecutive pair (src/decoder_ops.rs:166-188) with the
      // host-computed (cos, sin) of theta = pos * base^(-2k/dim).
      const int kk = (r0 % a.head_dim) >> 1;
      const float2 cs = a.rope[(size_t)pos * (a.head_dim >> 1) + kk];
      const float o0 = __fsub_rn(__fmul_rn(y0, cs.x), __fmul_rn(y1, cs.y));
      const float o1 = __fadd_rn(__fmul_rn(y0, cs.y), __fmul_rn(y1, cs.x));
      if (r0 < a.nq) {
        a.q_out[r0] = o0;
        a.q_out[r1] = o1;
      } else {
        // K stored f16-rounded (kv_f16_round, src/cpu_oracle.rs:878-883)
        const int c = r0 - a.nq;
        __half* kp = a.k_cache + (size_t)pos * kv_stride + c;
        *reinterpret_cast<__half2*>(kp) = __floats2half2_rn(o0, o1);
        if (a.k_trace) {
          a.k_trace[c] = o0;
          a.k_trace[c + 1] = o1;
        }
      }
    } else {
      const int c = r0 - a.nq - a.nk;
      __half* vp = a.v_cache + (size_t)pos * kv_stride + c;
      *reinterpret_cast<__half2*>(vp) = __floats2half2_rn(y0, y1);
      if (a.v_trace) {
        a.v_trace[c] = y0;
        a.v_trace[c + 1] = y1;
      }
    }
  } else if (EPI == EPI_SWIGLU) {
    // rows interleaved gate/up; swiglu = silu(g)*u, silu(g) = g/(1+e^-g)
    // (src/decoder_ops.rs:196-198, 351-362)
    if (!v0) return;
    const float s = __fdiv_rn(y0, __fadd_rn(1.0f, expf(-y0)));
    a.out[r0 >> 1] = __fmul_rn(s, y1);
  } else if (EPI == EPI_LOGITS) {
    unsigned long long best = 0ull;
    bool finite = true;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int r = k ? r1 : r0;
      const float y = k ? y1 : y0;
      if (!(k ? v1 : v0)) continue;
      a.out[r] = y;
      if (!isfinite(y)) finite = false;
      const int64_t gr = (int64_t)r + a.row_offset;
      bool eog = false;
      for (int e = 0; e < a.n_eog; ++e) eog |= (a.eog[e] == gr);
      // top1_non_eog (src/cpu_oracle.rs:979-995): strict '>' from -inf, so
      // NaN and -inf never win and the lowest id wins ties.
      if (!eog && y > -INFINITY) {
        const unsigned long long key =
            ((unsigned long long)ordered_bits(y) << 32) | (0xffffffffu - (uint32_t)gr);
        best = key > best ? key : best;
      }
    }
    for (int o = 4; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0x000000ffu, best, o);
      best = other > best ? other : best;
    }
    if (!finite) atomicAnd(a.finite_flag, 0);
    if (pair == 0 && best) atomicMax(a.argmax_key, best);
  }
}

// ---------------------------------------------------------------------------
// The kernel: persistent CTAs over 16-row tiles, 8 warps split K.
// ---------------------------------------------------------------------------
template <int WL, int PRO, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int xs_halves = gemv_xs_halves(a.nb);
  __half* xh = reinterpret_cast<__half*>(smem_raw);
  __half* xl = xh + xs_halves;
  float* part = reinterpret_cast<float*>(xl + xs_halves);  // [2][8][16]
  double* redd = reinterpret_cast<double*>(part + 2 * kGemvWarps * kTileRows);
  float* redf = reinterpret_cast<float*>(redd + kGemvWarps);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  // Weights do not depend on the previous kernel: start the first loads
  // before waiting on the producer of x.
  int tile = blockIdx.x;
  const bool have0 = tile < a.n_tiles && warp < a.nb;
  Q4Regs q4c, q4n;
  F16Regs f16c;
  if (have0) {
    if (WL == WL_F16) f16_load(a, tile, warp, g, t, f16c);
    else q4_load<WL>(a, tile, warp, g, t, q4c);
  }
  pdl_wait();
  const float out_scale = stage_x<PRO>(a, xh, xl, redd, redf);
  pdl_launch_dependents();
  const __half* xsrc = (g == 0) ? xh : xl;

  int it = 0;
  for (; tile < a.n_tiles; tile += gridDim.x, ++it) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const int xoff = a.tile_xoff ? a.tile_xoff[tile] : 0;
    for (int b = warp; b < a.nb; b += kGemvWarps) {
      int nbb = b + kGemvWarps, nt = tile;
      if (nbb >= a.nb) {
        nbb = warp;
        nt = tile + gridDim.x;
      }
      const bool has_next = nt < a.n_tiles && nbb < a.nb;
      const int xbase = kXPad + b * 256 - xoff;
      if (WL == WL_F16) {
        // 64 registers per item: no double buffering, occupancy hides latency
        if (b != warp || tile != (int)blockIdx.x) f16_load(a, tile, b, g, t, f16c);
        f16_compute(f16c, t, g, xsrc, xbase, acc);
      } else {
        if (has_next) q4_load<WL>(a, nt, nbb, g, t, q4n);
        q4_compute(q4c, t, g, xsrc, xbase, acc);
        q4c = q4n;
      }
    }
    float* pb = part + (it & 1) * kGemvWarps * kTileRows;
    if (t == 0) {
      pb[warp * kTileRows + g] = acc[0] + acc[1];
      pb[warp * kTileRows + g + 8] = acc[2] + acc[3];
    }
    __syncthreads();
    if (threadIdx.x < 8) {
      const int p = threadIdx.x;
      float y0 = 0.f, y1 = 0.f;
#pragma unroll
      for (int w = 0; w < kGemvWarps; ++w) {
        y0 += pb[w * kTileRows + 2 * p];
        y1 += pb[w * kTileRows + 2 * p + 1];
      }
      gemv_epilogue<EPI>(a, tile, p, y0 * out_scale, y1 * out_scale);
    }
  }
}

inline size_t gemv_smem_bytes(int nb) {
  return (size_t)2 * gemv_xs_halves(nb) * sizeof(__half) +
         (size_t)2 * kGemvWarps * kTileRows * sizeof(float) + kGemvWarps * sizeof(double) +
         kGemvWarps * sizeof(float) + 16;
}

}  // namespace faber
