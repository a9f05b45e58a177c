// attention.cuh — split-K GQA decode attention over the f16 KV cache
// (attention_gqa, src/cpu_oracle.rs:711-792, for one query row).
//
// Grid (kv_heads, splits), splits fixed per session (about six CTAs per SM
// over all kv heads). CTA (kv head kh, split s) covers an equal share of the
// current context, in groups of 32 positions (8 per warp), for the `ratio`
// query heads that share kv head kh (h / ratio == kh, the reference's
// grouping). The kernel is HBM-bound and built around keeping loads in flight:
//   * each warp streams its rows with a two-group register double buffer:
//     the next group's K and V rows (head_dim/32 halves per lane) are
//     requested before the current group is scored;
//   * rows older than the step's own position were written by earlier steps,
//     so the first group is requested before the programmatic-dependency
//     wait and overlaps the tail of the QKV kernel; q and the step's own row
//     are read after it;
//   * scores: per-lane partial dot products of 8 rows, reduced by a
//     transposed butterfly (9 shuffles for 8 rows; lane l ends with row
//     (l >> 2) & 7); score = (q . k) * scale with scale = 1/sqrt(head_dim);
//   * per warp an online softmax (running max, sum of exp, rescaled context);
//     the 4 warps combine in shared memory into the split's partial, and the
//     last CTA of each kv head (atomic ticket) merges the splits in split
//     order, so results do not depend on CTA timing.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "ops.cuh"

namespace faber {

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnRows = 8;                         // rows per warp per group
constexpr int kAttnGroup = kAttnRows * kAttnWarps;   // 32 positions per CTA group
constexpr int kAttnMaxRatio = 8;
constexpr int kAttnMergeBatch = 16;
constexpr int kAttnCtasPerSm = 6;  // splits: ~6 per SM over all kv heads (4 resident by registers; finer shares balance the waves)

struct AttnArgs {
  const float* q;          // [H][hd] post-RoPE queries
  const __half* k;         // this layer's cache [ctx][Hkv*hd]
  const __half* v;
  float* ctx;              // [H][hd]
  float* part;             // scratch [H][max_splits][hd + 2]
  int32_t* counters;       // scratch [Hkv], zero between uses
  const StepState* st;
  int32_t n_heads, n_kv_heads, head_dim, max_splits;
  float scale;
  // batched decode (grid.z = sequence): per-sequence state and this layer's
  // K/V rows; q/ctx, part and counters advance by these strides per sequence
  const SlotRef* slots;
  int32_t slot_q_stride, slot_part_stride, slot_counter_stride;
  int32_t cache_rows;      // rows of k / v (the TMA-streamed kernel's tensor maps)
  // batched launches of the TMA-streamed kernel: this layer's K and V tensor
  // maps of every sequence, [sequence][2], in device memory
  const CUtensorMap* kvmaps;
};

// The arguments of sequence blockIdx.z of a batched launch (identity for a
// single sequence).
__device__ __forceinline__ AttnArgs slot_args(const AttnArgs& a0) {
  AttnArgs a = a0;
  if (a0.slots) {
    const int z = blockIdx.z;
    const SlotRef sl = a0.slots[z];
    a.st = sl.st;
    a.k = sl.k;
    a.v = sl.v;
    a.q = a0.q + (size_t)z * a0.slot_q_stride;
    a.ctx = a0.ctx + (size_t)z * a0.slot_q_stride;
    a.part = a0.part + (size_t)z * a0.slot_part_stride;
    a.counters = a0.counters + (size_t)z * a0.slot_counter_stride;
  }
  return a;
}

// Splits per kv head for a session: about kAttnCtasPerSm CTAs per SM over all
// kv heads, never more than the context has position groups.
inline int attention_splits(int sms, int kv_heads, int max_ctx) {
  const int want = (kAttnCtasPerSm * sms + kv_heads - 1) / kv_heads;
  const int groups = (max_ctx + kAttnGroup - 1) / kAttnGroup;
  return std::max(1, std::min(want, groups));
}

// head_dim/32 halves of one K or V row per lane.
template <int DPL> struct KvVec;
template <> struct KvVec<4> {
  uint2 u;
  __device__ __forceinline__ void zero() { u = make_uint2(0u, 0u); }
  // rows written by earlier kernels: read-only path, no L1 allocation
  __device__ __forceinline__ void load_nc(const __half* p) {
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
                 : "=r"(u.x), "=r"(u.y)
                 : "l"(p));
  }
  // the row the preceding kernel wrote: coherent load after the wait
  __device__ __forceinline__ void load(const __half* p) { u = *reinterpret_cast<const uint2*>(p); }
  __device__ __forceinline__ void load_smem(const void* p) { u = *reinterpret_cast<const uint2*>(p); }
  __device__ __forceinline__ void to_float(float (&f)[4]) const {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    f[0] = a.x;
    f[1] = a.y;
    f[2] = b.x;
    f[3] = b.y;
  }
};
template <> struct KvVec<2> {
  uint32_t u;
  __device__ __forceinline__ void zero() { u = 0u; }
  __device__ __forceinline__ void load_nc(const __half* p) {
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(u) : "l"(p));
  }
  __device__ __forceinline__ void load(const __half* p) { u = *reinterpret_cast<const uint32_t*>(p); }
  __device__ __forceinline__ void load_smem(const void* p) { u = *reinterpret_cast<const uint32_t*>(p); }
  __device__ __forceinline__ void to_float(float (&f)[2]) const {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u));
    f[0] = a.x;
    f[1] = a.y;
  }
};

// Sum over the warp of 8 per-lane values; lane l returns the total of value
// (l >> 2) & 7. Each level halves the values a lane keeps and pairs lanes
// that differ in one bit (4, 3, 2); bits 1 and 0 then sum plainly.
__device__ __forceinline__ float butterfly8(float (&p)[8], int lane) {
#pragma unroll
  for (int level = 0; level < 3; ++level) {
    const int half = 4 >> level;
    const int bit = 16 >> level;
    const bool upper = (lane & bit) != 0;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float keep = upper ? p[i + half] : p[i];
      const float send = upper ? p[i] : p[i + half];
      p[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
    }
  }
  float s = p[0] + __shfl_xor_sync(0xffffffffu, p[0], 2);
  return s + __shfl_xor_sync(0xffffffffu, s, 1);
}

// A warp's 8-row slice of one position group.
template <int DPL>
struct KvGroup {
  KvVec<DPL> k[kAttnRows], v[kAttnRows];
};

// Request rows j0 .. j0+7 (rows >= cur are left zero: the step's own row is
// fetched by load_own after the dependency wait, rows past it are unused).
template <int DPL>
__device__ __forceinline__ void kv_request(KvGroup<DPL>& g, const AttnArgs& a, int j0, int cur,
                                           size_t kvs, size_t col) {
#pragma unroll
  for (int i = 0; i < kAttnRows; ++i) {
    g.k[i].zero();
    g.v[i].zero();
    if (j0 + i < cur) {
      g.k[i].load_nc(a.k + (size_t)(j0 + i) * kvs + col);
      g.v[i].load_nc(a.v + (size_t)(j0 + i) * kvs + col);
    }
  }
}

template <int DPL>
__device__ __forceinline__ void kv_load_own(KvGroup<DPL>& g, const AttnArgs& a, int j0, int cur,
                                            size_t kvs, size_t col) {
#pragma unroll
  for (int i = 0; i < kAttnRows; ++i) {
    if (j0 + i == cur) {
      g.k[i].load(a.k + (size_t)cur * kvs + col);
      g.v[i].load(a.v + (size_t)cur * kvs + col);
    }
  }
}

// Online-softmax update of one warp with one 8-row group (rows j0 .. j0+7,
// valid below n_kv).
template <int DPL, int R>
__device__ __forceinline__ void kv_consume(const KvGroup<DPL>& g, int j0, int n_kv, int ratio,
                                           float scale, const float (&qv)[R][DPL], float (&m)[R],
                                           float (&l)[R], float (&acc)[R][DPL], float (*pw)[kAttnRows],
                                           int lane) {
  const int row = (lane >> 2) & 7;
  const bool valid = j0 + row < n_kv;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (r >= ratio) break;
    float p[kAttnRows];
#pragma unroll
    for (int i = 0; i < kAttnRows; ++i) {
      float kf[DPL];
      g.k[i].to_float(kf);
      float s = 0.0f;
#pragma unroll
      for (int d = 0; d < DPL; ++d) s = fmaf(qv[r][d], kf[d], s);
      p[i] = s;
    }
    // every lane takes part in the shuffles; invalid rows are masked after
    const float dot = butterfly8(p, lane);
    const float s = valid ? dot * scale : -INFINITY;
    float gm = s;
    gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, 4));
    gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, 8));
    gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, 16));
    const float mn = fmaxf(m[r], gm);
    // no valid row yet (mn = -inf): nothing to add or rescale
    const float c = mn == -INFINITY ? 1.0f : expf(m[r] - mn);
    const float e = valid ? expf(s - mn) : 0.0f;
    float es = e;
    es += __shfl_xor_sync(0xffffffffu, es, 4);
    es += __shfl_xor_sync(0xffffffffu, es, 8);
    es += __shfl_xor_sync(0xffffffffu, es, 16);
    l[r] = fmaf(l[r], c, es);
    m[r] = mn;
#pragma unroll
    for (int d = 0; d < DPL; ++d) acc[r][d] *= c;
    if ((lane & 3) == 0) pw[r][row] = e;
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < kAttnRows; ++i) {
    float vf[DPL];
    g.v[i].to_float(vf);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (r >= ratio) break;
      const float e = pw[r][i];
#pragma unroll
      for (int d = 0; d < DPL; ++d) acc[r][d] = fmaf(e, vf[d], acc[r][d]);
    }
  }
  __syncwarp();
}

// Combine the 4 warps' stashed (max, sum, context) into the split's partial,
// and let the last CTA of the kv head (atomic ticket) merge all splits in
// split order. Threads 0-127 take part; sync() is a barrier over them.
template <int HD, int R, class Sync>
__device__ __forceinline__ void attn_merge(const AttnArgs& a, int kh, int split, int active, int ratio,
                                           const float (&wstat)[kAttnWarps][R][2],
                                           const float (&red)[kAttnWarps][R][HD], int* is_last, Sync sync) {
  sync();
  const int stride = HD + 2;
  for (int idx = threadIdx.x; idx < ratio * HD; idx += kAttnThreads) {
    const int r = idx / HD, d = idx % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wstat[w][r][0]);
    float L = 0.0f, s = 0.0f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float f = wstat[w][r][0] == -INFINITY ? 0.0f : expf(wstat[w][r][0] - M);
      L = fmaf(wstat[w][r][1], f, L);
      s = fmaf(red[w][r][d], f, s);
    }
    float* pp = a.part + ((size_t)(kh * ratio + r) * a.max_splits + split) * stride;
    pp[2 + d] = s;
    if (d == 0) {
      pp[0] = M;
      pp[1] = L;
    }
  }
  // the last CTA of this kv head merges all splits in split order
  __threadfence();
  sync();
  if (threadIdx.x == 0) {
    const int ticket = atomicAdd(&a.counters[kh], 1);
    *is_last = (ticket == active - 1);
  }
  sync();
  if (!*is_last) return;
  __threadfence();
  // One pass in split order, kAttnMergeBatch splits' loads in flight at a
  // time: the running (max, sum, context) is rescaled to each batch's max.
  for (int idx = threadIdx.x; idx < ratio * HD; idx += kAttnThreads) {
    const int r = idx / HD, d = idx % HD;
    const float* base = a.part + (size_t)(kh * ratio + r) * a.max_splits * stride;
    float M = -INFINITY, L = 0.0f, acc_d = 0.0f;
    for (int s0 = 0; s0 < active; s0 += kAttnMergeBatch) {
      float ms[kAttnMergeBatch], ls[kAttnMergeBatch], vs[kAttnMergeBatch];
#pragma unroll
      for (int u = 0; u < kAttnMergeBatch; ++u) {
        const bool ok = s0 + u < active;
        const float* p = base + (size_t)(s0 + u) * stride;
        ms[u] = ok ? __ldcg(p) : -INFINITY;
        ls[u] = ok ? __ldcg(p + 1) : 0.0f;
        vs[u] = ok ? __ldcg(p + 2 + d) : 0.0f;
      }
      float mb = M;  // every split holds a valid row, so mb is finite from here
#pragma unroll
      for (int u = 0; u < kAttnMergeBatch; ++u) mb = fmaxf(mb, ms[u]);
      const float c = expf(M - mb);
      L *= c;
      acc_d *= c;
#pragma unroll
      for (int u = 0; u < kAttnMergeBatch; ++u) {
        const float f = expf(ms[u] - mb);  // 0 for the padding entries
        L = fmaf(ls[u], f, L);
        acc_d = fmaf(vs[u], f, acc_d);
      }
      M = mb;
    }
    a.ctx[(size_t)(kh * ratio + r) * HD + d] = acc_d / L;
  }
  if (threadIdx.x == 0) a.counters[kh] = 0;
}

// The end of a split CTA (4 warps, threads 0-127, sync() a barrier over
// them): each warp stashes its (max, sum, context), then attn_merge.
template <int HD, int R, class Sync>
__device__ __forceinline__ void attn_finish(const AttnArgs& a, int kh, int split, int active, int ratio, int warp,
                                            int lane, const float (&m)[R], const float (&l)[R],
                                            const float (&acc)[R][HD / 32], float (&wstat)[kAttnWarps][R][2],
                                            float (&red)[kAttnWarps][R][HD], int* is_last, Sync sync) {
  constexpr int DPL = HD / 32;
  // stash this warp's state
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (r >= ratio) break;
    if (lane == 0) {
      wstat[warp][r][0] = m[r];
      wstat[warp][r][1] = l[r];
    }
#pragma unroll
    for (int d = 0; d < DPL; ++d) red[warp][r][lane * DPL + d] = acc[r][d];
  }
  attn_merge<HD, R>(a, kh, split, active, ratio, wstat, red, is_last, sync);
}

template <int HD, int R>
__global__ void __launch_bounds__(kAttnThreads) attention_decode_kernel(const AttnArgs a0) {
  const AttnArgs a = slot_args(a0);
  constexpr int DPL = HD / 32;
  static_assert(DPL == 2 || DPL == 4, "head_dim 64 or 128");
  __shared__ float pbuf[kAttnWarps][R][kAttnRows];
  __shared__ float wstat[kAttnWarps][R][2];
  __shared__ float red[kAttnWarps][R][HD];
  __shared__ int is_last;

  const int kh = blockIdx.x, split = blockIdx.y;
  // cur_pos was written by this step's embed kernel, which completed before
  // the QKV kernel (whose consumers wait on it) let this grid launch.
  const int cur = a.st->cur_pos;
  const int n_kv = cur + 1;
  const int n_grp = (n_kv + kAttnGroup - 1) / kAttnGroup;
  const int per = (n_grp + gridDim.y - 1) / gridDim.y;  // groups per split
  const int active = (n_grp + per - 1) / per;           // splits with work
  const int g0 = split * per, g1 = min(n_grp, g0 + per);
  if (g0 >= g1) return;
  const int ratio = a.n_heads / a.n_kv_heads;  // <= R
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t kvs = (size_t)a.n_kv_heads * HD;
  const size_t col = (size_t)kh * HD + lane * DPL;
  const int wrow = warp * kAttnRows;  // this warp's row offset inside a group

  KvGroup<DPL> ga, gb;
  kv_request(ga, a, g0 * kAttnGroup + wrow, cur, kvs, col);
  pdl_wait();
  pdl_launch_dependents();
  float qv[R][DPL];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const float* qp = a.q + (size_t)(kh * ratio + r) * HD + lane * DPL;
#pragma unroll
    for (int d = 0; d < DPL; ++d) qv[r][d] = r < ratio ? qp[d] : 0.0f;
  }
  float m[R], l[R], acc[R][DPL];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.0f;
#pragma unroll
    for (int d = 0; d < DPL; ++d) acc[r][d] = 0.0f;
  }
  float(*pw)[kAttnRows] = pbuf[warp];
  // two groups per iteration so that both buffers keep static register names
  for (int g = g0; g < g1; g += 2) {
    const int ja = g * kAttnGroup + wrow, jb = ja + kAttnGroup;
    if (g + 1 < g1) kv_request(gb, a, jb, cur, kvs, col);
    kv_load_own(ga, a, ja, cur, kvs, col);
    kv_consume<DPL, R>(ga, ja, n_kv, ratio, a.scale, qv, m, l, acc, pw, lane);
    if (g + 1 < g1) {
      if (g + 2 < g1) kv_request(ga, a, jb + kAttnGroup, cur, kvs, col);
      kv_load_own(gb, a, jb, cur, kvs, col);
      kv_consume<DPL, R>(gb, jb, n_kv, ratio, a.scale, qv, m, l, acc, pw, lane);
    }
  }
  attn_finish<HD, R>(a, kh, split, active, ratio, warp, lane, m, l, acc, wstat, red, &is_last,
                     [] { __syncthreads(); });
}

}  // namespace faber
