// gemv.cuh — fused Q4_K dequant-GEMV for batch-1 decode (sm_100a).
//
// y[j] = sum_i w[j][i] * x[i] with w[j][i] = f16(f32(d*sc*q - dmin*m)), the
// reference's dense (src/decoder_ops.rs:378-406) over dequant_q4_k
// (src/dequant.rs:194-217) after metal_f16_round_weights
// (src/cpu_oracle.rs:356-360).
//
// Data path (a producer warp, 8 consumer warps and an epilogue warp per CTA,
// 2 CTAs per SM):
//   * the producer streams 2304-byte tile items (16 rows x one super-block:
//     16 headers, then 16 x 128 quant bytes) with bulk TMA copies into a
//     3-4 stage shared-memory ring guarded by mbarriers (no multicast);
//   * each consumer lane owns one 32-byte quant chunk (two sub-blocks) of
//     two rows; per 32-bit quant word it forms exact weights with
//       (w & 0x000F000F) | 0x64006400  -> (1024 + q, 1024 + q') as f16x2,
//       fma.f16x2(1024 + q, sc, -1024 sc) -> sc*q exactly (<= 945),
//       fma.rn.f32.f16(d, sc*q, -m1)   -> RN32(d1*q - m1), the reference's
//                                          separately rounded value,
//       cvt.rn.f16x2.f32               -> the f16-rounded weight pair,
//     which is already the tensor-core A operand;
//   * x is staged once per CTA in shared memory as an exact two-term f16
//     split (x*2^-s = hi + lo, s a power-of-two scale from max|x|), and
//     mma.sync m16n8k16 (f16 x f16 -> f32) multiplies the 16x16 weight tile
//     by [hi, lo]: accumulator columns 0 and 1 sum to y*2^-s. The tensor
//     core is the reduction engine;
//   * warps split K (super-blocks); each hands its partial tile over through
//     an mbarrier to a dedicated epilogue warp, which sums the 8 partials in
//     a fixed order (deterministic) and runs the fused epilogue (store /
//     residual add / RoPE + KV-cache append / SwiGLU / logits + argmax).
#pragma once

#include "common.cuh"

namespace faber {

// PRO_NORM_RES: x = x + x2 (the residual add deferred from a tensor-parallel
// all-reduce), written back by CTA 0, then rms_norm as PRO_NORM.
// PRO_NORM_PEERS: x_sum_out = x + (sum over ranks of the exchange buffer, in
// rank order), each CTA summing one slice, then a grid barrier, then rms_norm
// of x_sum_out. EPI_PEERS: the row-parallel output rows go to this rank's
// slot in every rank's exchange buffer over NVLink. Each value travels with
// its exchange epoch in one 8-byte store (single-copy atomic), so a reader
// spins on the element itself: no fence, ticket or flag.
enum GemvPrologue : int { PRO_PLAIN = 0, PRO_NORM = 1, PRO_NORM_RES = 2, PRO_NORM_PEERS = 3 };
enum GemvEpilogue : int {
  EPI_STORE = 0,
  EPI_RESID = 1,
  EPI_QKV = 2,
  EPI_SWIGLU = 3,
  EPI_LOGITS = 4,
  EPI_PEERS = 5
};
enum GemvLayout : int { WL_TILED = 0, WL_NATIVE = 1, WL_F16 = 2 };

constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kXPad = 256;  // zero halo (elements) in front of x for row offsets
constexpr int kMaxEog = 8;
constexpr int kMaxTp = 8;

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
  float* x_sum_out;          // PRO_NORM_RES (CTA 0 writes) / PRO_NORM_PEERS (each CTA a slice): the summed input
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
  // tensor-parallel exchange over peer memory
  int32_t tp;                          // ranks in the group
  int32_t tp_stage;                    // this exchange within a step (2 * layer + 0 O / 1 down)
  int32_t tp_stages;                   // exchanges per step
  const uint32_t* epoch_ptr;           // steps taken (StepState), the epoch base
  unsigned long long* peer_dst[kMaxTp];  // EPI_PEERS: this rank's slot in rank r's buffer
  const unsigned long long* red;       // PRO_NORM_PEERS: local buffer [tp][n_cols]
  unsigned int* grid_bar;              // PRO_NORM_PEERS: {arrived, generation} (local)
  uint32_t peer_wait_limit;            // polls before a peer / grid-barrier wait gives up (0: default)
};

// Epoch of one exchange: unique per (step, exchange) and identical on every
// rank (each rank's embed kernel counts the same steps).
__device__ __forceinline__ uint32_t tp_epoch(const GemvArgs& a) {
  return *a.epoch_ptr * (uint32_t)a.tp_stages + (uint32_t)a.tp_stage + 1u;
}

__device__ __forceinline__ void st_peer(unsigned long long* p, float v, uint32_t epoch) {
  const unsigned long long w = ((unsigned long long)epoch << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ unsigned long long ld_peer(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

// Set by a kernel whose bounded wait expired (never in a correct run):
// 1 = a pipeline stage, 2 = a tensor-parallel peer, 3 = a grid barrier. The
// host reads and clears it after each step.
__device__ int g_pipe_error;

// One exchanged value once its epoch has arrived. Bounded: by default 2^20
// polls (well under a second; a session can set a shorter limit), and no
// wait at all once an earlier wait has expired.
constexpr uint32_t kPeerSpinLimit = 1u << 20;
__device__ __forceinline__ uint32_t peer_limit(const GemvArgs& a) {
  return a.peer_wait_limit ? a.peer_wait_limit : kPeerSpinLimit;
}
__device__ __forceinline__ float peer_value(const unsigned long long* p, uint32_t epoch, uint32_t limit) {
  unsigned long long w = ld_peer(p);
  for (uint32_t n = 0; (uint32_t)(w >> 32) != epoch; w = ld_peer(p)) {
    if (++n >= limit || ((n & 1023u) == 0 && *(volatile int*)&g_pipe_error)) {
      atomicExch(&g_pipe_error, 2);
      break;
    }
  }
  return __uint_as_float((uint32_t)w);
}

// Sum of the ranks' partials of element i, in rank order. All ranks' words
// are requested before any is checked (one round trip when they have
// arrived); a word still carrying an older epoch is then waited for.
__device__ __forceinline__ float peer_sum1(const GemvArgs& a, int i, uint32_t e) {
  unsigned long long w[kMaxTp];
#pragma unroll
  for (int p = 0; p < kMaxTp; ++p)
    if (p < a.tp) w[p] = ld_peer(a.red + (size_t)p * a.n_cols + i);
  float s = 0.0f;
#pragma unroll
  for (int p = 0; p < kMaxTp; ++p) {
    if (p >= a.tp) break;
    const float v = (uint32_t)(w[p] >> 32) == e
                        ? __uint_as_float((uint32_t)w[p])
                        : peer_value(a.red + (size_t)p * a.n_cols + i, e, peer_limit(a));
    s = p == 0 ? v : s + v;
  }
  return s;
}

// Tensor-parallel groups up to this size form the whole summed input in
// every CTA (tp x n peer words read per CTA, no grid barrier); larger groups
// sum one slice per CTA and publish it through a grid barrier.
constexpr int kTpFullSum = 4;

__device__ __forceinline__ ulonglong2 ld_peer2(const unsigned long long* p) {
  ulonglong2 w;
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(w.x), "=l"(w.y) : "l"(p) : "memory");
  return w;
}

// x + the ranks' partials (rank order, as peer_sum1) of every element, into
// xsum[n] in shared memory: 256 threads, element pairs, the words of 4
// pairs per thread requested before any is checked.
__device__ __forceinline__ void peer_full_sum(const GemvArgs& a, float* xsum, uint32_t e) {
  constexpr int NT = kGemvThreads, kB = 4;
  const int n = a.n_cols, n2 = n / 2, tid = threadIdx.x;
  const uint32_t lim = peer_limit(a);
  for (int base = 0; base < n2; base += kB * NT) {
    ulonglong2 w[kB][kTpFullSum];
    float2 xv[kB];
#pragma unroll
    for (int k = 0; k < kB; ++k) {
      const int j = base + k * NT + tid;
      if (j < n2) {
        xv[k] = reinterpret_cast<const float2*>(a.x)[j];
#pragma unroll
        for (int p = 0; p < kTpFullSum; ++p)
          if (p < a.tp) w[k][p] = ld_peer2(a.red + (size_t)p * n + 2 * j);
      }
    }
#pragma unroll
    for (int k = 0; k < kB; ++k) {
      const int j = base + k * NT + tid;
      if (j >= n2) break;
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int p = 0; p < kTpFullSum; ++p) {
        if (p >= a.tp) break;
        const unsigned long long* wp = a.red + (size_t)p * n + 2 * j;
        const float v0 = (uint32_t)(w[k][p].x >> 32) == e ? __uint_as_float((uint32_t)w[k][p].x)
                                                           : peer_value(wp, e, lim);
        const float v1 = (uint32_t)(w[k][p].y >> 32) == e ? __uint_as_float((uint32_t)w[k][p].y)
                                                           : peer_value(wp + 1, e, lim);
        s0 = p == 0 ? v0 : s0 + v0;
        s1 = p == 0 ? v1 : s1 + v1;
      }
      xsum[2 * j] = xv[k].x + s0;
      xsum[2 * j + 1] = xv[k].y + s1;
    }
  }
}

// Grid-wide barrier of a persistent grid (every CTA resident), thread 0 of
// each CTA; sense-reversing, so the same two words serve every launch.
// Bounded like the peer waits.
__device__ __forceinline__ void grid_barrier(unsigned int* bar, uint32_t limit) {
  volatile unsigned int* gen = bar + 1;
  const unsigned int my_gen = *gen;
  __threadfence();
  if (atomicAdd(bar, 1u) == gridDim.x - 1) {
    bar[0] = 0u;
    __threadfence();
    atomicAdd(bar + 1, 1u);
    return;
  }
  for (uint32_t n = 0; *gen == my_gen; ++n) {
    if (n >= limit) {
      atomicExch(&g_pipe_error, 3);
      break;
    }
    __nanosleep(32);
  }
  __threadfence();
}

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
// The 256 threads that stage x and compute: the whole CTA (register kernel)
// or the 8 consumer warps of the pipelined kernel (named barrier 1, so the
// producer warp never takes part).
template <bool NAMED>
__device__ __forceinline__ void cbar() {
  if (NAMED) asm volatile("bar.sync 1, 256;" ::: "memory");
  else __syncthreads();
}

template <bool NAMED>
__device__ __forceinline__ void block_sum_max(double& v, float& m, double* redd, float* redf) {
  for (int o = 16; o > 0; o >>= 1) {
    v += __shfl_xor_sync(0xffffffffu, v, o);
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  cbar<NAMED>();
  if (lane == 0) {
    redd[warp] = v;
    redf[warp] = m;
  }
  cbar<NAMED>();
  double s = 0.0;
  float mm = 0.0f;
#pragma unroll
  for (int w = 0; w < kGemvWarps; ++w) {
    s += redd[w];
    mm = fmaxf(mm, redf[w]);
  }
  v = s;
  m = mm;
}

__device__ __forceinline__ bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Power-of-two scale that brings max|x| into [2^13, 2^14).
__device__ __forceinline__ int split_shift(float bound) {
  if (!(bound > 0.0f) || !isfinite(bound)) return 0;
  int e;
  frexpf(bound, &e);
  int s = e - 14;
  return max(-100, min(100, s));
}

// Element i of the GEMV input before normalization (x, or x + x2).
template <int PRO>
__device__ __forceinline__ float4 load_x4(const GemvArgs& a, int i4, const float* xsum) {
  if (PRO == PRO_NORM_PEERS)
    return xsum ? reinterpret_cast<const float4*>(xsum)[i4]
                : __ldcg(reinterpret_cast<const float4*>(a.x_sum_out) + i4);
  float4 v = reinterpret_cast<const float4*>(a.x)[i4];
  if (PRO == PRO_NORM_RES) {
    const float4 u = reinterpret_cast<const float4*>(a.x2)[i4];
    v = make_float4(v.x + u.x, v.y + u.y, v.z + u.z, v.w + u.w);
  }
  return v;
}

template <int PRO>
__device__ __forceinline__ float load_x1(const GemvArgs& a, int i, const float* xsum) {
  if (PRO == PRO_NORM_RES) return a.x[i] + a.x2[i];
  if (PRO == PRO_NORM_PEERS) return xsum ? xsum[i] : __ldcg(a.x_sum_out + i);
  return a.x[i];
}

// Normalized value: rms_norm's x*scale*w with two rounded products
// (src/decoder_ops.rs:140-143).
template <int PRO>
__device__ __forceinline__ float norm1(float x, float scale, float w) {
  return PRO == PRO_PLAIN ? x : __fmul_rn(__fmul_rn(x, scale), w);
}

__device__ __forceinline__ void split_store(float v0, float v1, float v2, float v3, float in_s,
                                            __half* xh, __half* xl, int idx) {
  const __half2 h01 = __floats2half2_rn(v0 * in_s, v1 * in_s);
  const __half2 h23 = __floats2half2_rn(v2 * in_s, v3 * in_s);
  const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
  const __half2 l01 = __floats2half2_rn(v0 * in_s - f01.x, v1 * in_s - f01.y);
  const __half2 l23 = __floats2half2_rn(v2 * in_s - f23.x, v3 * in_s - f23.y);
  uint2 hv, lv;
  hv.x = *reinterpret_cast<const uint32_t*>(&h01);
  hv.y = *reinterpret_cast<const uint32_t*>(&h23);
  lv.x = *reinterpret_cast<const uint32_t*>(&l01);
  lv.y = *reinterpret_cast<const uint32_t*>(&l23);
  *reinterpret_cast<uint2*>(xh + idx) = hv;
  *reinterpret_cast<uint2*>(xl + idx) = lv;
}

// Stage x (or rms_norm(x) * w) into shared memory as the hi/lo f16 split,
// 256 threads. Pass 1 reduces sum of squares (f64) and a max bound; pass 2
// writes the split. Returns the output scale 2^s.
// PERM stores each group of four elements as (0, 2, 1, 3): the order in which
// the f16-magic dequant (two nibbles per mask, bytes 0/2 then 1/3) fills the
// tensor-core A fragments.
template <int PRO, bool NAMED, bool PERM>
__device__ float stage_x(const GemvArgs& a, __half* xh, __half* xl, double* redd, float* redf) {
  constexpr int NT = kGemvThreads;
  const int n = a.n_cols;
  const int tid = threadIdx.x;
  // PRO_NORM_PEERS, small groups: the whole summed input in shared memory
  // (the x staging area, free until the split below; CTA 0 publishes it)
  float* xsum = nullptr;
  if (PRO == PRO_NORM_PEERS) {
    const uint32_t e = tp_epoch(a);
    // (only where the staging below takes its vectorized one-batch path,
    // which keeps every value in registers before the split overwrites xsum)
    if (a.tp <= kTpFullSum && n % 4 == 0 && n / 4 <= NT * 8 && aligned16(a.x) && aligned16(a.norm_w)) {
      xsum = reinterpret_cast<float*>(xh);
      peer_full_sum(a, xsum, e);
      cbar<NAMED>();
    } else {
      // this CTA's slice of x + sum of the ranks' partials, then every slice
      const int per = (n + (int)gridDim.x - 1) / (int)gridDim.x;
      const int i1 = min(n, ((int)blockIdx.x + 1) * per);
      for (int i = (int)blockIdx.x * per + tid; i < i1; i += NT)
        a.x_sum_out[i] = a.x[i] + peer_sum1(a, i, e);
      cbar<NAMED>();
      if (tid == 0) grid_barrier(a.grid_bar, peer_limit(a));
      cbar<NAMED>();
    }
  }
  const bool vec = (n % 4 == 0) && aligned16(a.x) &&
                   (PRO == PRO_PLAIN || aligned16(a.norm_w)) &&
                   (PRO != PRO_NORM_RES || aligned16(a.x2));
  double ss = 0.0;
  float mx = 0.0f;
  // kXB float4 per thread per batch, every load of a batch issued before any
  // use (one L2 round trip per batch); each thread still sums its elements
  // in increasing index order
  // (norm weights double the registers of a batch); when one batch covers
  // the row the values stay in registers for the second pass
  constexpr int kXB = PRO == PRO_PLAIN ? 12 : 8;
  const int n4 = n / 4;
  const bool one_batch = n4 <= NT * kXB;
  float4 v[kXB], w[kXB];
  if (vec) {
    for (int base = 0; base < n4; base += NT * kXB) {
#pragma unroll
      for (int k = 0; k < kXB; ++k) {
        const int i4 = base + tid + k * NT;
        if (i4 < n4) {
          v[k] = load_x4<PRO>(a, i4, xsum);
          if (PRO != PRO_PLAIN) w[k] = reinterpret_cast<const float4*>(a.norm_w)[i4];
        }
      }
#pragma unroll
      for (int k = 0; k < kXB; ++k) {
        if (base + tid + k * NT >= n4) break;
        if (PRO != PRO_PLAIN) {
          ss += (double)v[k].x * (double)v[k].x;
          ss += (double)v[k].y * (double)v[k].y;
          ss += (double)v[k].z * (double)v[k].z;
          ss += (double)v[k].w * (double)v[k].w;
          mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[k].x * w[k].x), fabsf(v[k].y * w[k].y)),
                               fmaxf(fabsf(v[k].z * w[k].z), fabsf(v[k].w * w[k].w))));
        } else {
          mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[k].x), fabsf(v[k].y)), fmaxf(fabsf(v[k].z), fabsf(v[k].w))));
        }
      }
    }
  } else {
    for (int i = tid; i < n; i += NT) {
      const float v = load_x1<PRO>(a, i, xsum);
      if (PRO != PRO_PLAIN) {
        ss += (double)v * (double)v;
        mx = fmaxf(mx, fabsf(v * a.norm_w[i]));
      } else {
        mx = fmaxf(mx, fabsf(v));
      }
    }
  }
  block_sum_max<NAMED>(ss, mx, redd, redf);
  float scale = 1.0f, bound = mx;
  if (PRO != PRO_PLAIN) {
    // rms_norm (src/decoder_ops.rs:126-144): f64 sum, mean cast to f32,
    // scale = 1/sqrt(mean + eps).
    const float mean = (float)(ss / (double)n);
    scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
    bound = mx * scale * 1.001f;
  }
  const int s = split_shift(bound);
  const float in_s = ldexpf(1.0f, -s);
  const bool cta0 = blockIdx.x == 0;
  // zero halo in front of x and the tail after it
  const int total = kXPad + a.nb * 256;
  for (int p = tid; p < kXPad; p += NT) {
    xh[xs_index(p)] = __float2half(0.0f);
    xl[xs_index(p)] = __float2half(0.0f);
  }
  for (int p = kXPad + n + tid; p < total; p += NT) {
    xh[xs_index(p)] = __float2half(0.0f);
    xl[xs_index(p)] = __float2half(0.0f);
  }
  if (vec) {
    for (int base = 0; base < n4; base += NT * kXB) {
      if (!one_batch) {
#pragma unroll
        for (int k = 0; k < kXB; ++k) {
          const int i4 = base + tid + k * NT;
          if (i4 < n4) {
            v[k] = load_x4<PRO>(a, i4, xsum);
            if (PRO != PRO_PLAIN) w[k] = reinterpret_cast<const float4*>(a.norm_w)[i4];
          }
        }
      }
#pragma unroll
      for (int k = 0; k < kXB; ++k) {
        const int i4 = base + tid + k * NT;
        if (i4 >= n4) break;
        float4 y = v[k];
        if (PRO != PRO_PLAIN)
          y = make_float4(norm1<PRO>(v[k].x, scale, w[k].x), norm1<PRO>(v[k].y, scale, w[k].y),
                          norm1<PRO>(v[k].z, scale, w[k].z), norm1<PRO>(v[k].w, scale, w[k].w));
        if (cta0) {
          if (PRO == PRO_NORM_RES || (PRO == PRO_NORM_PEERS && xsum))
            reinterpret_cast<float4*>(a.x_sum_out)[i4] = v[k];
          if (PRO != PRO_PLAIN && a.x_norm_out) reinterpret_cast<float4*>(a.x_norm_out)[i4] = y;
        }
        if (PERM) split_store(y.x, y.z, y.y, y.w, in_s, xh, xl, xs_index(kXPad + 4 * i4));
        else split_store(y.x, y.y, y.z, y.w, in_s, xh, xl, xs_index(kXPad + 4 * i4));
      }
    }
  } else {
    for (int i = tid; i < n; i += NT) {
      const float v = load_x1<PRO>(a, i, xsum);
      const float y = PRO == PRO_PLAIN ? v : norm1<PRO>(v, scale, a.norm_w[i]);
      if (cta0) {
        if (PRO == PRO_NORM_RES || (PRO == PRO_NORM_PEERS && xsum)) a.x_sum_out[i] = v;
        if (PRO != PRO_PLAIN && a.x_norm_out) a.x_norm_out[i] = y;
      }
      const float sv = y * in_s;
      const __half hi = __float2half_rn(sv);
      const int r = i & 3;
      const int pos = PERM ? ((i & ~3) | (r == 1 ? 2 : (r == 2 ? 1 : r))) : i;
      xh[xs_index(kXPad + pos)] = hi;
      xl[xs_index(kXPad + pos)] = __float2half_rn(sv - __half2float(hi));
    }
  }
  cbar<NAMED>();
  return ldexpf(1.0f, s);
}

// ---------------------------------------------------------------------------
// Weight item: one 16-row tile x one 256-element super-block column
// ---------------------------------------------------------------------------
// One-instruction (w & MASK) | magic, with the magic in a register operand.
template <uint32_t MASK>
__device__ __forceinline__ uint32_t and_or(uint32_t w, uint32_t magic) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(w), "n"(MASK), "r"(magic));
  return d;
}

template <uint32_t SEL>
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "n"(SEL));
  return d;
}

// ---------------------------------------------------------------------------
// Weight formation: two nibbles per mask via f16 magics, exact sc*q in f16, and a
// mixed-precision FMA for RN32(d*(sc*q) - m1).
//   (w & 0x000F000F) | 0x64006400 = (1024 + q, 1024 + q') as f16x2;
//   (w & 0x00F000F0) | 0x54005400 = (64 + q, 64 + q') (high nibbles);
//   fma.f16x2((K + q), sc, -K*sc) = sc*q exactly (<= 945 < 2048);
//   fma.rn.f32.f16(d, sc*q, -m1) = RN32(d*sc*q - m1): d*sc*q is exact in
//   f32 (22 bits) and equals d1*q of the reference, so one rounding here is
//   the reference's d1*q - m1 (src/dequant.rs:204-211).
// A word yields pairs (e, e+2) from bytes 0/2 and (e+1, e+3) from bytes 1/3.
// ---------------------------------------------------------------------------
struct LaneConst {
  uint32_t sel;    // byte permute that gathers this lane's two scale bytes
  uint32_t m1024;  // 0x64006400
  uint32_t m64;    // 0x54005400
};

struct RowScales3 {
  uint32_t sclo2, clo2, schi2, chi2;  // f16x2 (sc, sc), (-K sc, -K sc) per sub-block
  float nm1, nm2;                     // -m1, -m2
  uint32_t dword;                     // header word 0: d (f16) in the low half
};

__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t hmul2_u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t prmt_r(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// RN32(lo16(dword) * q16 + c) for both halves q16 of `q2`.
__device__ __forceinline__ float2 mixed_fma_pair(uint32_t q2, uint32_t dword, float c) {
  float x, y;
  asm("{\n .reg .b16 q0, q1, d0, d1;\n mov.b32 {q0, q1}, %2;\n mov.b32 {d0, d1}, %3;\n"
      " fma.rn.f32.f16 %0, d0, q0, %4;\n fma.rn.f32.f16 %1, d0, q1, %4;\n}"
      : "=f"(x), "=f"(y)
      : "r"(q2), "r"(dword), "f"(c));
  return make_float2(x, y);
}

// RN32(hi16(dword) * q16_lo) and RN32(hi16(dword) * q16_hi): dmin * m (exact).
__device__ __forceinline__ float2 mixed_mul_hi_pair(uint32_t q2, uint32_t dword) {
  float x, y;
  asm("{\n .reg .b16 q0, q1, d0, d1;\n mov.b32 {q0, q1}, %2;\n mov.b32 {d0, d1}, %3;\n"
      " fma.rn.f32.f16 %0, d1, q0, 0f80000000;\n fma.rn.f32.f16 %1, d1, q1, 0f80000000;\n}"
      : "=f"(x), "=f"(y)
      : "r"(q2), "r"(dword));
  return make_float2(x, y);
}

__device__ __forceinline__ RowScales3 row_scales3(const uint4 h, int t, const LaneConst& lc) {
  const uint32_t s0 = h.y, s1 = h.z, s2 = h.w;
  uint32_t sc, mm;  // get_scale_min_k4 for this lane's 4-index half, as packed bytes
  if (t < 2) {
    sc = s0 & 0x3f3f3f3fu;
    mm = s1 & 0x3f3f3f3fu;
  } else {
    sc = (s2 & 0x0f0f0f0fu) | ((s0 >> 2) & 0x30303030u);
    mm = ((s2 >> 4) & 0x0f0f0f0fu) | ((s1 >> 2) & 0x30303030u);
  }
  // (1024 + v_lo, 1024 + v_hi) as f16x2, then minus 1024: exact small ints
  const uint32_t k1024 = 0x64006400u;
  const uint32_t scp = hsub2_u(prmt_r(sc, lc.m1024, lc.sel), k1024);
  const uint32_t mp = hsub2_u(prmt_r(mm, lc.m1024, lc.sel), k1024);
  RowScales3 r;
  r.sclo2 = prmt<0x1010>(scp, 0);  // (sc_lo, sc_lo)
  r.schi2 = prmt<0x3232>(scp, 0);  // (sc_hi, sc_hi)
  r.clo2 = hmul2_u(r.sclo2, 0xe400e400u);  // * -1024
  r.chi2 = hmul2_u(r.schi2, 0xd400d400u);  // * -64
  const float2 m12 = mixed_mul_hi_pair(mp, h.x);
  r.nm1 = -m12.x;
  r.nm2 = -m12.y;
  r.dword = h.x;
  return r;
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// ---------------------------------------------------------------------------
// Decode GEMV item: lane (g, t) of a consumer warp forms rows g and g+8 of
// its 32-byte quant chunk t (sub-blocks 2t, 2t+1) of one 16-row item.
// Instruction budget per 8 weights (one quant word): 4 mask-or (ALU), one
// high multiply for the byte shift (FMA pipe, so the ALU pipe, which issues
// at half rate, only carries the mask-or and the f16 pack), 4 f16x2 FMAs,
// 8 mixed FMAs and 4 packs.
// ---------------------------------------------------------------------------
struct ItemConst {
  uint32_t m1024;     // 0x64006400
  uint32_t m64;       // 0x54005400
  uint32_t sh24;      // 2^24: (w >> 8) as mul.hi (kept opaque in a register)
  uint32_t sel;       // byte selector of this lane's scale / min source bytes
  uint32_t mlo, mhi;  // masks of the 6- or 4-bit low part and the 2-bit high part
  uint32_t msh;       // right shift of the min's low part (0 or 4)
};

__device__ __forceinline__ ItemConst item_const(int t) {
  ItemConst c;
  asm("mov.b32 %0, 0x64006400;" : "=r"(c.m1024));
  asm("mov.b32 %0, 0x54005400;" : "=r"(c.m64));
  asm("mov.b32 %0, 0x01000000;" : "=r"(c.sh24));
  const uint32_t k = 2u * (uint32_t)(t & 1);
  if (t < 2) {
    c.sel = k | ((k + 1u) << 4) | (k << 8) | ((k + 1u) << 12);
    c.mlo = 0x3f3fu;
    c.mhi = 0u;
    c.msh = 0u;
  } else {
    c.sel = (4u + k) | ((5u + k) << 4) | (k << 8) | ((k + 1u) << 12);
    c.mlo = 0x0f0fu;
    c.mhi = 0x3030u;
    c.msh = 4u;
  }
  return c;
}

// Per (row, lane): the formation constants of sub-blocks a = 2t and b = 2t+1.
struct RowScales {
  uint32_t scp;     // (sc_a, sc_b) f16x2
  uint32_t ca, cb;  // (-1024 sc_a) x2 and (-64 sc_b) x2: the magic offsets
  float nma, nmb;   // -(dmin * m_a), -(dmin * m_b)
  uint32_t dword;   // header word 0: d in the low half, dmin in the high half
};

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t m, uint32_t c) {
  uint32_t d;  // (a & m) | c
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(m), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t mulhi_u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.hi.u32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// (lo(b), lo(b)) * c and (hi(b), hi(b)) * c, the broadcast as an operand swizzle.
__device__ __forceinline__ uint32_t hmul2_lo(uint32_t bpair, uint32_t c) {
  uint32_t d;
  asm("{\n .reg .b16 l, h;\n .reg .b32 bb;\n mov.b32 {l, h}, %1;\n mov.b32 bb, {l, l};\n"
      " mul.rn.f16x2 %0, bb, %2;\n}"
      : "=r"(d) : "r"(bpair), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t hmul2_hi(uint32_t bpair, uint32_t c) {
  uint32_t d;
  asm("{\n .reg .b16 l, h;\n .reg .b32 bb;\n mov.b32 {l, h}, %1;\n mov.b32 bb, {h, h};\n"
      " mul.rn.f16x2 %0, bb, %2;\n}"
      : "=r"(d) : "r"(bpair), "r"(c));
  return d;
}
// a * (lo(b), lo(b)) + c and a * (hi(b), hi(b)) + c
__device__ __forceinline__ uint32_t hfma2_lo(uint32_t a, uint32_t bpair, uint32_t c) {
  uint32_t d;
  asm("{\n .reg .b16 l, h;\n .reg .b32 bb;\n mov.b32 {l, h}, %2;\n mov.b32 bb, {l, l};\n"
      " fma.rn.f16x2 %0, %1, bb, %3;\n}"
      : "=r"(d) : "r"(a), "r"(bpair), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t hfma2_hi(uint32_t a, uint32_t bpair, uint32_t c) {
  uint32_t d;
  asm("{\n .reg .b16 l, h;\n .reg .b32 bb;\n mov.b32 {l, h}, %2;\n mov.b32 bb, {h, h};\n"
      " fma.rn.f16x2 %0, %1, bb, %3;\n}"
      : "=r"(d) : "r"(a), "r"(bpair), "r"(c));
  return d;
}

// get_scale_min_k4 (src/dequant.rs:178-187) for this lane's two sub-blocks,
// branch-free. Bytes s[0..11] are header words y, z, w:
//   t < 2  (j = 2t, 2t+1):   sc = s[j] & 63,                     m = s[j+4] & 63
//   t >= 2 (j = 2t, 2t+1):   sc = (s[j+4] & 15) | (s[j-4] >> 6) << 4,
//                            m  = (s[j+4] >> 4) | (s[j] >> 6) << 4
// One byte permute gathers [low-part bytes, high-part bytes] per field.
__device__ __forceinline__ RowScales row_scales(const uint4 h, const ItemConst& ic) {
  const uint32_t X = prmt_r(h.y, h.w, ic.sel);
  const uint32_t Y = prmt_r(h.z, h.w, ic.sel);
  const uint32_t sc16 = lop3_and_or(X, ic.mlo, (X >> 18) & ic.mhi);
  const uint32_t m16 = lop3_and_or(Y >> ic.msh, ic.mlo, (Y >> 18) & ic.mhi);
  // (1024 + v_a, 1024 + v_b) as f16x2, minus 1024: exact small integers
  const uint32_t k1024 = ic.m1024;
  const uint32_t scp = hsub2_u(prmt<0x7150>(sc16, k1024), k1024);
  const uint32_t mp = hsub2_u(prmt<0x7150>(m16, k1024), k1024);
  RowScales r;
  r.scp = scp;
  r.ca = hmul2_lo(scp, 0xe400e400u);  // * -1024
  r.cb = hmul2_hi(scp, 0xd400d400u);  // * -64
  // m1 = dmin * m exactly; its negation keeps the reference's d1*q - m1
  // (sign of zero included)
  const float2 m12 = mixed_mul_hi_pair(mp, h.x);
  r.nma = -m12.x;
  r.nmb = -m12.y;
  r.dword = h.x;
  return r;
}

// Eight exact f16-rounded weights of one quant word: pairs (e, e+2) and
// (e+1, e+3) of sub-block a (low nibbles) and of sub-block b (high nibbles).
__device__ __forceinline__ void dequant_word(uint32_t w, const RowScales& s, const ItemConst& ic,
                                             uint32_t& lo0, uint32_t& lo2, uint32_t& hi0,
                                             uint32_t& hi2) {
  const uint32_t u = mulhi_u(w, ic.sh24);  // w >> 8
  const uint32_t l02 = hfma2_lo(and_or<0x000f000fu>(w, ic.m1024), s.scp, s.ca);
  const uint32_t l13 = hfma2_lo(and_or<0x000f000fu>(u, ic.m1024), s.scp, s.ca);
  const uint32_t h02 = hfma2_hi(and_or<0x00f000f0u>(w, ic.m64), s.scp, s.cb);
  const uint32_t h13 = hfma2_hi(and_or<0x00f000f0u>(u, ic.m64), s.scp, s.cb);
  const float2 a = mixed_fma_pair(l02, s.dword, s.nma);
  const float2 b = mixed_fma_pair(l13, s.dword, s.nma);
  const float2 c = mixed_fma_pair(h02, s.dword, s.nmb);
  const float2 d = mixed_fma_pair(h13, s.dword, s.nmb);
  lo0 = pack_half2(a.x, a.y);  // (e, e+2)
  lo2 = pack_half2(b.x, b.y);  // (e+1, e+3)
  hi0 = pack_half2(c.x, c.y);
  hi2 = pack_half2(d.x, d.y);
}

// Byte offsets inside one staged item (shared memory): tiled = 16 headers
// then 16 x 128 quant bytes; native = 16 consecutive 144-byte blocks.
template <int WL>
struct ItemGeom {
  static constexpr int kHead = WL == WL_TILED ? 16 : kQ4kBlockBytes;       // header of row g
  static constexpr int kQuant0 = WL == WL_TILED ? 256 : 16;                // quants of row 0
  static constexpr int kQuantRow = WL == WL_TILED ? 128 : kQ4kBlockBytes;  // quant row stride
};

// One item: 16 MMAs into four independent accumulator chains (MMA m goes to
// chain m & 3). B fragments come from lane groups 0 (x hi) and 1 (x lo); the
// other groups load the same rows (a shared-memory broadcast) and feed
// accumulator columns 2..7, which are never read. xlo / xhi point at the
// padded x elements 64t + {0..15} and 64t + 32 + {0..15} of the item.
template <int WL>
__device__ __forceinline__ void q4_item(const uint8_t* hdr, const uint8_t* qnt, const __half* xlo,
                                        const __half* xhi, float (&acc)[4][4], const ItemConst& ic) {
  using G = ItemGeom<WL>;
  const uint4 hA = *reinterpret_cast<const uint4*>(hdr);
  const uint4 hB = *reinterpret_cast<const uint4*>(hdr + 8 * G::kHead);
  const RowScales sA = row_scales(hA, ic);
  const RowScales sB = row_scales(hB, ic);
#pragma unroll
  for (int pp = 0; pp < 2; ++pp) {
    const uint4 qa = *reinterpret_cast<const uint4*>(qnt + 16 * pp);
    const uint4 qb = *reinterpret_cast<const uint4*>(qnt + 16 * pp + 8 * G::kQuantRow);
    const uint4 xb_lo0 = *reinterpret_cast<const uint4*>(xlo + 16 * pp);
    const uint4 xb_lo1 = *reinterpret_cast<const uint4*>(xlo + 16 * pp + 8);
    const uint4 xb_hi0 = *reinterpret_cast<const uint4*>(xhi + 16 * pp);
    const uint4 xb_hi1 = *reinterpret_cast<const uint4*>(xhi + 16 * pp + 8);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t aL0, aL2, aH0, aH2, bL0, bL2, bH0, bH2;
      dequant_word(word_of(qa, i), sA, ic, aL0, aL2, aH0, aH2);
      dequant_word(word_of(qb, i), sB, ic, bL0, bL2, bH0, bH2);
      const uint4& xl = (i < 2) ? xb_lo0 : xb_lo1;
      const uint4& xh = (i < 2) ? xb_hi0 : xb_hi1;
      const uint32_t xl0 = (i & 1) ? xl.z : xl.x, xl1 = (i & 1) ? xl.w : xl.y;
      const uint32_t xh0 = (i & 1) ? xh.z : xh.x, xh1 = (i & 1) ? xh.w : xh.y;
      float* cl = acc[(2 * i) & 3];
      float* ch = acc[(2 * i + 1) & 3];
      mma_16816(cl[0], cl[1], cl[2], cl[3], aL0, bL0, aL2, bL2, xl0, xl1);
      mma_16816(ch[0], ch[1], ch[2], ch[3], aH0, bH0, aH2, bH2, xh0, xh1);
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
  } else if (EPI == EPI_PEERS) {
    const uint32_t e = tp_epoch(a);
    for (int p = 0; p < a.tp; ++p) {
      if (v0) st_peer(a.peer_dst[p] + r0, y0, e);
      if (v1) st_peer(a.peer_dst[p] + r1, y1, e);
    }
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
  static_assert(WL == WL_F16, "the register-path kernel serves the f16 head only");
  int tile = blockIdx.x;
  const bool have0 = tile < a.n_tiles && warp < a.nb;
  F16Regs f16c;
  if (have0) f16_load(a, tile, warp, g, t, f16c);
  pdl_wait();
  const float out_scale = stage_x<PRO, false, false>(a, xh, xl, redd, redf);
  pdl_launch_dependents();
  const __half* xsrc = (g == 0) ? xh : xl;

  int it = 0;
  for (; tile < a.n_tiles; tile += gridDim.x, ++it) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const int xoff = a.tile_xoff ? a.tile_xoff[tile] : 0;
    for (int b = warp; b < a.nb; b += kGemvWarps) {
      const int xbase = kXPad + b * 256 - xoff;
      // 64 registers per item: no double buffering, occupancy hides latency
      if (b != warp || tile != (int)blockIdx.x) f16_load(a, tile, b, g, t, f16c);
      f16_compute(f16c, t, g, xsrc, xbase, acc);
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

// ---------------------------------------------------------------------------
// Pipelined Q4_K kernel: one producer warp streams tile items with bulk TMA
// copies (cp.async.bulk, no multicast) into a shared-memory ring guarded by
// mbarriers; 8 consumer warps dequantize from shared memory. Two CTAs per SM
// (one where the staged x needs more than half the shared memory),
// persistent over tiles; under programmatic dependent launch the producer
// starts streaming before the previous kernel has finished.
// ---------------------------------------------------------------------------
constexpr int kConsumerWarps = kGemvWarps;
constexpr int kProducerWarp = kConsumerWarps;      // streams the ring
constexpr int kEpilogueWarp = kConsumerWarps + 1;  // sums partial tiles, runs the epilogue
constexpr int kPipeThreads = (kConsumerWarps + 2) * 32;
constexpr int kStageBytes = kConsumerWarps * kTileItemBytes;  // 18 KB
constexpr int kMaxStages = 4;
constexpr uint32_t kSpinLimit = 1u << 20;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(b)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(b)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(b)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(b)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: after kSpinLimit polls the error word is set and the caller
// proceeds (every barrier stays balanced, so no other warp can block).
__device__ __forceinline__ void mbar_wait(uint64_t* b, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(b, parity)) return;
  atomicExch(&g_pipe_error, 1);
}

// Streaming bulk copy global -> own CTA's shared memory, completing on an
// mbarrier; weights are read once, so L2 may evict them first.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Partial tiles in flight between the consumer warps and the epilogue warp:
// each consumer hands its 16 partial rows of a tile over through an
// mbarrier and goes on; a dedicated epilogue warp sums them and runs the
// epilogue, so neither a barrier nor the epilogue's memory round trips sit
// between a consumer's tiles (it waits only when kParts tiles ahead).
constexpr int kParts = 4;

struct PipeLayout {
  int stages;
  size_t ring, xs, part, redd, redf, bars, total;
};

__host__ __device__ inline PipeLayout pipe_layout(int nb) {
  PipeLayout L;
  L.stages = nb > 24 ? 3 : kMaxStages;
  L.ring = 0;
  L.xs = (size_t)L.stages * kStageBytes;
  L.part = L.xs + (size_t)2 * gemv_xs_halves(nb) * 2;
  L.redd = L.part + (size_t)kParts * kConsumerWarps * kTileRows * 4;
  L.redf = L.redd + (size_t)kConsumerWarps * 8;
  L.bars = (L.redf + (size_t)kConsumerWarps * 4 + 8 + 7) & ~(size_t)7;  // + out_scale
  L.total = L.bars + (size_t)(2 * kMaxStages + 2 * kParts) * 8;
  return L;
}

template <int WL, int PRO, int EPI>
__global__ void __launch_bounds__(kPipeThreads, 2) gemv_pipe_kernel(const GemvArgs a) {
  static_assert(WL == WL_TILED || WL == WL_NATIVE, "Q4_K layouts only");
  extern __shared__ __align__(128) unsigned char smem[];
  const PipeLayout L = pipe_layout(a.nb);
  uint8_t* ring = smem + L.ring;
  const int xs_halves = gemv_xs_halves(a.nb);
  __half* xh = reinterpret_cast<__half*>(smem + L.xs);
  __half* xl = xh + xs_halves;
  float* part = reinterpret_cast<float*>(smem + L.part);
  double* redd = reinterpret_cast<double*>(smem + L.redd);
  float* redf = reinterpret_cast<float*>(smem + L.redf);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + kMaxStages;
  uint64_t* pfull = empty + kMaxStages;  // a tile's partials written by all consumer warps
  uint64_t* pfree = pfull + kParts;      // ... and summed by its epilogue warp

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = L.stages;
  const int R = (a.nb + kConsumerWarps - 1) / kConsumerWarps;  // rounds per tile
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    for (int p = 0; p < kParts; ++p) {
      mbar_init(&pfull[p], kConsumerWarps);
      mbar_init(&pfree[p], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == kProducerWarp) {
    // producer: weights never depend on the previous kernel, so no wait here
    if (lane == 0) {
      uint64_t policy;
      asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
      int q = 0, s = 0;
      uint32_t ph = 0;  // parity of the slot's previous use
      for (int tile = blockIdx.x; tile < a.n_tiles; tile += gridDim.x) {
        for (int r = 0; r < R; ++r, ++q) {
          if (q >= S) mbar_wait(&empty[s], ph);
          const int b0 = r * kConsumerWarps;
          const int cnt = min(kConsumerWarps, a.nb - b0);
          uint8_t* dst = ring + (size_t)s * kStageBytes;
          if (WL == WL_TILED) {
            // the cnt items of one tile round are contiguous: one copy
            mbar_arrive_expect_tx(&full[s], (uint32_t)(cnt * kTileItemBytes));
            bulk_g2s(dst, a.w + ((size_t)tile * a.nb + b0) * kTileItemBytes,
                     (uint32_t)(cnt * kTileItemBytes), &full[s], policy);
          } else {
            const int rows = min(kTileRows, a.n_rows - tile * kTileRows);
            mbar_arrive_expect_tx(&full[s], (uint32_t)(cnt * rows * kQ4kBlockBytes));
            for (int w = 0; w < cnt; ++w)
              for (int i = 0; i < rows; ++i)
                bulk_g2s(dst + w * kTileItemBytes + i * kQ4kBlockBytes,
                         a.w + ((size_t)(tile * kTileRows + i) * a.nb + b0 + w) * kQ4kBlockBytes,
                         kQ4kBlockBytes, &full[s], policy);
          }
          if (++s == S) {
            s = 0;
            if (q >= S) ph ^= 1u;
          }
        }
      }
    }
    return;
  }

  if (warp == kEpilogueWarp) {
    // epilogue: tile by tile in order, the 8 partial tiles summed in warp
    // order (deterministic), then the fused epilogue on lanes 0-7
    pdl_wait();
    float out_scale = 0.f;
    int it = 0;
    for (int tile = blockIdx.x; tile < a.n_tiles; tile += gridDim.x, ++it) {
      const int pi = it % kParts;
      mbar_wait(&pfull[pi], (uint32_t)((it / kParts) & 1));
      if (it == 0) out_scale = *reinterpret_cast<volatile float*>(redf + kConsumerWarps);
      const float* pb = part + pi * kConsumerWarps * kTileRows;
      if (lane < 8) {
        const int p = lane;
        float y0 = 0.f, y1 = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          y0 += pb[w * kTileRows + 2 * p];
          y1 += pb[w * kTileRows + 2 * p + 1];
        }
        gemv_epilogue<EPI>(a, tile, p, y0 * out_scale, y1 * out_scale);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfree[pi]);
    }
    return;
  }

  // consumers
  pdl_wait();
  const float out_scale = stage_x<PRO, true, true>(a, xh, xl, redd, redf);
  pdl_launch_dependents();
  // for the epilogue warp (read after the first tile's hand-over)
  if (threadIdx.x == 0) redf[kConsumerWarps] = out_scale;
  const int g = lane >> 2, t = lane & 3;
  const ItemConst ic = item_const(t);
  const __half* xsrc = (g == 0) ? xh : xl;
  using G = ItemGeom<WL>;
  // this warp's item inside a slot: header of row g, quant chunk t of row g
  const int off_h = warp * kTileItemBytes + G::kHead * g;
  const int off_q = warp * kTileItemBytes + G::kQuant0 + G::kQuantRow * g + 32 * t;
  // consecutive rounds of a warp are 8 super-blocks (2048 elements) apart:
  // 2304 padded halves
  constexpr int kRoundHalves = kConsumerWarps * 256 + ((kConsumerWarps * 256) >> 3);
  int s = 0, it = 0;
  uint32_t ph = 0;
  for (int tile = blockIdx.x; tile < a.n_tiles; tile += gridDim.x, ++it) {
    float acc[4][4];
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[c][0] = acc[c][1] = acc[c][2] = acc[c][3] = 0.f;
    // x elements of this warp's first item: xb0 + {0..15, 32..47} (+16pp);
    // xoff is a multiple of 32, so neither run of 32 crosses a padding gap
    const int xoff = a.tile_xoff ? a.tile_xoff[tile] : 0;
    const int xb0 = kXPad + warp * 256 - xoff + 64 * t;
    const __half* xlo = xsrc + xs_index(xb0);
    const __half* xhi = xsrc + xs_index(xb0 + 32);
    for (int r = 0, b = warp; r < R; ++r, b += kConsumerWarps) {
      mbar_wait(&full[s], ph);
      if (b < a.nb) {
        const uint8_t* slot = ring + (size_t)s * kStageBytes;
        q4_item<WL>(slot + off_h, slot + off_q, xlo, xhi, acc, ic);
      }
      // release the slot once every lane has consumed its bytes
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (++s == S) {
        s = 0;
        ph ^= 1u;
      }
      xlo += kRoundHalves;
      xhi += kRoundHalves;
    }
    // hand this warp's partial rows to the epilogue warp
    const int pi = it % kParts;
    float* pb = part + pi * kConsumerWarps * kTileRows;
    if (it >= kParts) mbar_wait(&pfree[pi], (uint32_t)(((it / kParts) & 1) ^ 1));
    if (t == 0) {
      const float a0 = (acc[0][0] + acc[0][1]) + (acc[1][0] + acc[1][1]) +
                       (acc[2][0] + acc[2][1]) + (acc[3][0] + acc[3][1]);
      const float a1 = (acc[0][2] + acc[0][3]) + (acc[1][2] + acc[1][3]) +
                       (acc[2][2] + acc[2][3]) + (acc[3][2] + acc[3][3]);
      pb[warp * kTileRows + g] = a0;
      pb[warp * kTileRows + g + 8] = a1;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&pfull[pi]);
  }
}

}  // namespace faber
