// ops.cuh — the other decode kernels: bit-exact Q4_K dequant, f16 rounding,
// embedding gather, step bookkeeping.
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

// ---------------------------------------------------------------------------
// The other admitted block types, bit-exact (src/dequant.rs:151-174,224-255):
// element e of one block, every product rounded as the reference writes it.
// ---------------------------------------------------------------------------
constexpr uint32_t kGgmlF32 = 0, kGgmlF16 = 1, kGgmlQ5_0 = 6, kGgmlQ8_0 = 8, kGgmlQ4_K = 12,
                   kGgmlQ6_K = 14;

__device__ __forceinline__ float blk_half(const uint8_t* p) {
  return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

// dequant_q8_0 (src/dequant.rs:151-154): (i8) q * d, 32 per 34-byte block.
__device__ __forceinline__ float q8_0_value(const uint8_t* blk, int e) {
  return __fmul_rn((float)(int8_t)blk[2 + e], blk_half(blk));
}

// dequant_q5_0 (src/dequant.rs:160-174): 4 low bits in qs, the fifth from qh;
// elements j and j + 16 share byte qs[j].
__device__ __forceinline__ float q5_0_value(const uint8_t* blk, int e) {
  const uint32_t qh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8) | ((uint32_t)blk[4] << 16) |
                      ((uint32_t)blk[5] << 24);
  const int j = e & 15;
  const uint8_t q = blk[6 + j];
  const int x = e < 16 ? (int)((q & 0x0fu) | (((qh >> j) << 4) & 0x10u)) - 16
                       : (int)((q >> 4) | ((qh >> (j + 12)) & 0x10u)) - 16;
  return __fmul_rn((float)x, blk_half(blk));
}

// dequant_q6_k (src/dequant.rs:224-255): (d * sc) * q, 256 per 210-byte
// block (ql 128 B, qh 64 B, 16 signed scales, d at byte 208).
__device__ __forceinline__ float q6_k_value(const uint8_t* blk, int e) {
  const int n = e & 128, r = e & 127;
  const int g = r >> 5, l = r & 31;  // quarter of the 128-half, position
  const uint8_t* ql = blk + (n >> 1);
  const uint8_t qhb = blk[128 + (n >> 2) + l];
  const uint8_t lo = (g & 1) ? ql[l + 32] : ql[l];
  const int q = (int)(((g & 2) ? (lo >> 4) : (lo & 0x0f)) | (((qhb >> (2 * g)) & 3) << 4)) - 32;
  const float sc = (float)(int8_t)blk[192 + (n >> 4) + (l >> 4) + 2 * g];
  return __fmul_rn(__fmul_rn(blk_half(blk + 208), sc), (float)q);
}

__host__ __device__ inline bool ggml_block_geometry(uint32_t t, int& elems, int& bytes) {
  switch (t) {
    case kGgmlF32: elems = 1; bytes = 4; return true;
    case kGgmlF16: elems = 1; bytes = 2; return true;
    case kGgmlQ5_0: elems = 32; bytes = 22; return true;
    case kGgmlQ8_0: elems = 32; bytes = 34; return true;
    case kGgmlQ4_K: elems = 256; bytes = 144; return true;
    case kGgmlQ6_K: elems = 256; bytes = 210; return true;
    default: return false;
  }
}

// Element e of one block of type t (any admitted type).
__device__ __forceinline__ float block_value(uint32_t t, const uint8_t* blk, int e) {
  switch (t) {
    case kGgmlQ4_K: return q4k_value(blk, e);
    case kGgmlQ6_K: return q6_k_value(blk, e);
    case kGgmlQ8_0: return q8_0_value(blk, e);
    case kGgmlQ5_0: return q5_0_value(blk, e);
    case kGgmlF16: return blk_half(blk);
    default: {
      float v;
      memcpy(&v, blk, 4);
      return v;
    }
  }
}

// Validation surface for every block type: a block per warp, lanes stride its
// elements.
__global__ void dequant_blocks_kernel(uint32_t type, const uint8_t* __restrict__ blocks,
                                      uint64_t n_blocks, float* __restrict__ out, int f16r) {
  int be = 0, bb = 0;
  ggml_block_geometry(type, be, bb);
  const uint64_t wid = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= n_blocks) return;
  const uint8_t* blk = blocks + wid * bb;
  for (int e = lane; e < be; e += 32) {
    float v = block_value(type, blk, e);
    if (f16r) v = f16_round(v);
    out[wid * be + e] = v;
  }
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
  uint32_t tp_epoch;     // steps taken since the session opened (kept by reset):
                         // the epoch base of tensor-parallel exchanges
  unsigned long long argmax_key;
};

// One sequence of a batched decode step: its step state and this layer's
// K/V cache rows ([ctx][Hkv*hd] f16).
struct SlotRef {
  StepState* st;
  __half* k;
  __half* v;
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
    st->tp_epoch = st->tp_epoch + 1u;
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

// Batched decode: embed_kernel for sequence blockIdx.x (its step state,
// row blockIdx.x of h).
__global__ void slots_embed_kernel(const SlotRef* slots, const __half* __restrict__ embd, int d,
                                   int vocab, float* __restrict__ h) {
  pdl_wait();
  pdl_launch_dependents();
  StepState* st = slots[blockIdx.x].st;
  const int64_t tok = st->input_token;
  const bool ok = tok >= 0 && tok < vocab;
  float* hr = h + (size_t)blockIdx.x * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x)
    hr[i] = ok ? __half2float(embd[(size_t)tok * d + i]) : 0.0f;
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!ok) st->status = 1;
    st->cur_pos = st->n;
    st->n = st->n + 1;
    st->argmax_key = 0ull;
  }
}

// Batched decode: finalize_kernel for sequence blockIdx.x; its greedy ids go
// to gen[blockIdx.x * gen_cap ..].
__global__ void slots_finalize_kernel(const SlotRef* slots, int64_t* gen, int32_t gen_cap) {
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x != 0) return;
  StepState* st = slots[blockIdx.x].st;
  const unsigned long long key = st->argmax_key;
  const int64_t tok = key ? (int64_t)(0xffffffffu - (uint32_t)(key & 0xffffffffull)) : 0;
  st->input_token = tok;
  const int32_t c = st->gen_count;
  if (gen && c >= 0 && c < gen_cap) {
    gen[(size_t)blockIdx.x * gen_cap + c] = tok;
    st->gen_count = c + 1;
  }
  st->argmax_key = 0ull;
}

}  // namespace faber
