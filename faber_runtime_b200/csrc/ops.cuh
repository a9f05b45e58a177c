// ops.cuh — the other decode kernels: bit-exact Q4_K dequant, f16 rounding,
// embedding gather, split-K GQA decode attention, step bookkeeping.
#pragma once

#include "common.cuh"

namespace faber {

// ---------------------------------------------------------------------------
// Bit-exact Q4_K dequant (validation surface)
// ---------------------------------------------------------------------------

// get_scale_min_k4 — src/dequant.rs:178-187.
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* s, int& sc, int& m) {
  if (j < 4) {
    sc = s[j] & 63;
    m = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
    m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

// dequant_q4_k (src/dequant.rs:194-217) for element e (0..255) of one block:
// d1 = d*sc, m1 = dmin*m, y = d1*q - m1, each rounded separately.
__device__ __forceinline__ float q4k_value(const uint8_t* blk, int e) {
  const float d = __half2float(__ushort_as_half((unsigned short)(blk[0] | (blk[1] << 8))));
  const float dmin = __half2float(__ushort_as_half((unsigned short)(blk[2] | (blk[3] << 8))));
  const int j = e >> 5;          // sub-block
  const int c = j >> 1;          // 32-byte quant chunk
  const int l = e & 31;
  const uint8_t byte = blk[16 + 32 * c + l];
  const int q = (j & 1) ? (byte >> 4) : (byte & 0x0f);
  int sc, m;
  scale_min_k4(j, blk + 4, sc, m);
  const float d1 = __fmul_rn(d, (float)sc);
  const float m1 = __fmul_rn(dmin, (float)m);
  return __fsub_rn(__fmul_rn(d1, (float)q), m1);
}

// One warp per block, lanes stride the 256 elements (coalesced stores).
__global__ void dequant_q4k_native_kernel(const uint8_t* __restrict__ blocks, uint64_t n_blocks,
                                          float* __restrict__ out, int f16r) {
  const uint64_t wid = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= n_blocks) return;
  const uint8_t* blk = blocks + wid * kQ4kBlockBytes;
  float* o = out + wid * kQ4kBlockElems;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int e = k * 32 + lane;
    float v = q4k_value(blk, e);
    if (f16r) v = f16_round(v);
    o[e] = v;
  }
}

// Dequantize a tiled (repacked) weight back to [rows][cols]: one warp per
// (tile, tile row, super-block).
__global__ void dequant_q4k_tiled_kernel(const uint8_t* __restrict__ w, int n_tiles, int nb,
                                         int n_rows, int n_cols, const int32_t* tile_xoff,
                                         const int32_t* row_map, float* __restrict__ out,
                                         int f16r) {
  const uint64_t wid = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const uint64_t total = (uint64_t)n_tiles * kTileRows * nb;
  if (wid >= total) return;
  const int b = (int)(wid % nb);
  const int tr = (int)((wid / nb) % kTileRows);
  const int tile = (int)(wid / ((uint64_t)nb * kTileRows));
  const int row = row_map ? row_map[tile * kTileRows + tr] : tile * kTileRows + tr;
  if (row < 0 || row >= n_rows) return;
  const int xoff = tile_xoff ? tile_xoff[tile] : 0;
  // Reassemble the 144-byte block of this row from the tile item.
  const uint8_t* item = w + ((size_t)tile * nb + b) * kTileItemBytes;
  uint8_t blk[kQ4kBlockBytes];
  for (int i = 0; i < 16; ++i) blk[i] = item[16 * tr + i];
  for (int i = 0; i < 128; ++i) blk[16 + i] = item[256 + 128 * tr + i];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int e = k * 32 + lane;
    const int col = b * 256 + e - xoff;
    if (col < 0 || col >= n_cols) continue;
    float v = q4k_value(blk, e);
    if (f16r) v = f16_round(v);
    out[(size_t)row * n_cols + col] = v;
  }
}

__global__ void f16_round_kernel(const float* __restrict__ x, float* __restrict__ y, uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    y[i] = f16_round(x[i]);
}

// ---------------------------------------------------------------------------
// Decode-step state (device resident; the CUDA graph reads it every step)
// ---------------------------------------------------------------------------
struct StepState {
  int64_t input_token;   // token pushed by the next step
  int32_t n;             // sequence length after the last push
  int32_t cur_pos;       // position being written by the running step
  int32_t gen_count;     // greedy tokens produced
  int32_t finite;        // finite gate over all logits since reset
  int32_t status;        // nonzero: a kernel-side check failed (token out of range)
  int32_t pad;
  unsigned long long argmax_key;
};

// embed_rows (src/cpu_oracle.rs:538-545) with the f16-rounded token_embd
// stored as f16; also opens the step: cur_pos = n, n += 1.
__global__ void embed_kernel(StepState* st, const __half* __restrict__ embd, int d, int vocab,
                             float* __restrict__ h) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t tok = st->input_token;
  const bool ok = tok >= 0 && tok < vocab;
  for (int i = threadIdx.x; i < d; i += blockDim.x)
    h[i] = ok ? __half2float(embd[(size_t)tok * d + i]) : 0.0f;
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!ok) st->status = 1;
    st->cur_pos = st->n;
    st->n = st->n + 1;
    st->argmax_key = 0ull;
  }
}

// After the logits: the argmax becomes the next input token and is recorded.
__global__ void finalize_kernel(StepState* st, int64_t* gen, int32_t gen_cap) {
  pdl_wait();
  pdl_launch_dependents();
  const unsigned long long key = st->argmax_key;
  const int64_t tok = key ? (int64_t)(0xffffffffu - (uint32_t)(key & 0xffffffffull)) : 0;
  st->input_token = tok;
  const int32_t c = st->gen_count;
  if (gen && c >= 0 && c < gen_cap) {
    gen[c] = tok;
    st->gen_count = c + 1;
  }
  st->argmax_key = 0ull;
}

// ---------------------------------------------------------------------------
// Split-K GQA decode attention (attention_gqa, src/cpu_oracle.rs:711-792)
// ---------------------------------------------------------------------------
// Grid (kv_heads, max_splits); CTA (kv head kh, split s) scores positions
// [64 s, 64 s + 64) for the `ratio` query heads sharing kv head kh
// (h / ratio == kh, the verified grouping), keeps (max, sum, acc[hd]) per
// query head, and the last CTA of each kv head merges the splits in split
// order. score = (q.k) * scale; softmax over positions 0..=pos.
constexpr int kAttnChunk = 64;
constexpr int kAttnThreads = 128;
constexpr int kAttnMaxRatio = 8;

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
};

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) attention_decode_kernel(const AttnArgs a) {
  constexpr int DPL = HD / 32;  // dims per lane
  __shared__ float sc[kAttnMaxRatio][kAttnChunk];
  __shared__ float red[kAttnThreads / 32][kAttnMaxRatio][HD];
  __shared__ float stat[kAttnMaxRatio][2];
  __shared__ int is_last;
  pdl_wait();
  pdl_launch_dependents();
  const int kh = blockIdx.x, split = blockIdx.y;
  const int n_kv = a.st->cur_pos + 1;
  const int active = (n_kv + kAttnChunk - 1) / kAttnChunk;
  if (split >= active) return;
  const int ratio = a.n_heads / a.n_kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvs = a.n_kv_heads * HD;
  const int j0 = split * kAttnChunk, j1 = min(n_kv, j0 + kAttnChunk);

  float qv[kAttnMaxRatio][DPL];
#pragma unroll
  for (int r = 0; r < kAttnMaxRatio; ++r)
#pragma unroll
    for (int d = 0; d < DPL; ++d)
      qv[r][d] = r < ratio ? a.q[(size_t)(kh * ratio + r) * HD + lane * DPL + d] : 0.0f;

  // scores: one warp per position, lanes own DPL consecutive dims
  for (int j = j0 + warp; j < j1; j += kAttnThreads / 32) {
    const __half* kp = a.k + (size_t)j * kvs + kh * HD + lane * DPL;
    float kf[DPL];
#pragma unroll
    for (int d = 0; d < DPL; d += 2) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(kp + d));
      kf[d] = f.x;
      kf[d + 1] = f.y;
    }
#pragma unroll
    for (int r = 0; r < kAttnMaxRatio; ++r) {
      if (r >= ratio) break;
      float s = 0.0f;
#pragma unroll
      for (int d = 0; d < DPL; ++d) s = fmaf(qv[r][d], kf[d], s);
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) sc[r][j - j0] = s * a.scale;
    }
  }
  __syncthreads();
  // per query head: chunk max and exp-sum (one warp per head)
  for (int r = warp; r < ratio; r += kAttnThreads / 32) {
    float m = -INFINITY;
    for (int j = lane; j < j1 - j0; j += 32) m = fmaxf(m, sc[r][j]);
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.0f;
    for (int j = lane; j < j1 - j0; j += 32) {
      const float p = expf(sc[r][j] - m);
      sc[r][j] = p;
      l += p;
    }
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) {
      stat[r][0] = m;
      stat[r][1] = l;
    }
  }
  __syncthreads();
  // acc[r][d] = sum_j p_j v_j[d]: warps split positions, lanes own dims
  float acc[kAttnMaxRatio][DPL];
#pragma unroll
  for (int r = 0; r < kAttnMaxRatio; ++r)
#pragma unroll
    for (int d = 0; d < DPL; ++d) acc[r][d] = 0.0f;
  for (int j = j0 + warp; j < j1; j += kAttnThreads / 32) {
    const __half* vp = a.v + (size_t)j * kvs + kh * HD + lane * DPL;
    float vf[DPL];
#pragma unroll
    for (int d = 0; d < DPL; d += 2) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(vp + d));
      vf[d] = f.x;
      vf[d + 1] = f.y;
    }
#pragma unroll
    for (int r = 0; r < kAttnMaxRatio; ++r) {
      if (r >= ratio) break;
      const float p = sc[r][j - j0];
#pragma unroll
      for (int d = 0; d < DPL; ++d) acc[r][d] = fmaf(p, vf[d], acc[r][d]);
    }
  }
#pragma unroll
  for (int r = 0; r < kAttnMaxRatio; ++r) {
    if (r >= ratio) break;
#pragma unroll
    for (int d = 0; d < DPL; ++d) red[warp][r][lane * DPL + d] = acc[r][d];
  }
  __syncthreads();
  const int stride = HD + 2;
  for (int idx = threadIdx.x; idx < ratio * HD; idx += kAttnThreads) {
    const int r = idx / HD, d = idx % HD;
    float s = 0.0f;
    for (int w = 0; w < kAttnThreads / 32; ++w) s += red[w][r][d];
    float* p = a.part + ((size_t)(kh * ratio + r) * a.max_splits + split) * stride;
    p[2 + d] = s;
    if (d == 0) {
      p[0] = stat[r][0];
      p[1] = stat[r][1];
    }
  }
  // the last CTA of this kv head merges all splits in split order
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int ticket = atomicAdd(&a.counters[kh], 1);
    is_last = (ticket == active - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int idx = threadIdx.x; idx < ratio * HD; idx += kAttnThreads) {
    const int r = idx / HD, d = idx % HD;
    const float* base = a.part + (size_t)(kh * ratio + r) * a.max_splits * stride;
    float M = -INFINITY;
    for (int s = 0; s < active; ++s) M = fmaxf(M, __ldcg(base + s * stride));
    float L = 0.0f, acc_d = 0.0f;
    for (int s = 0; s < active; ++s) {
      const float f = expf(__ldcg(base + s * stride) - M);
      L = fmaf(__ldcg(base + s * stride + 1), f, L);
      acc_d = fmaf(__ldcg(base + s * stride + 2 + d), f, acc_d);
    }
    a.ctx[(size_t)(kh * ratio + r) * HD + d] = acc_d / L;
  }
  if (threadIdx.x == 0) a.counters[kh] = 0;
}

}  // namespace faber
