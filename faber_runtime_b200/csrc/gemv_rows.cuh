// gemv_rows.cuh — dense (src/decoder_ops.rs:378-406) over weights stored as
// rows of native GGML blocks, any admitted type per row (Q4_K, Q6_K, Q5_0,
// Q8_0, F32, F16). This is the path for linears that are not all Q4_K
// (a Q4_K_M file keeps attn_v, ffn_down and the head in Q6_K). Every weight
// is dequantized exactly (src/dequant.rs:151-255) and rounded to f16 like
// the reference's materialized weights (src/cpu_oracle.rs:356-360), then
// multiplied with the f32 input on CUDA cores.
//
// One CTA (8 warps) per 16-row tile, CTAs striding over tiles: warp w
// makes rows 2w and 2w+1 (lanes split the row's blocks), and the 8 lanes of
// warp 0 run the same epilogues as the Q4_K GEMV (QKV + RoPE + KV append,
// residual, SwiGLU, logits + argmax) on the tile's 8 row pairs. Rows are
// stored in the fused order the epilogues expect (Q|K|V, gate/up
// interleaved), so no row map is needed.
#pragma once

#include "gemv.cuh"
#include "ops.cuh"

namespace faber {

constexpr uint32_t kNoRow = 0xffffffffu;  // padding row of the last tile

struct RowsArgs {
  const uint8_t* bytes;     // all rows, back to back
  const uint64_t* row_off;  // [n_tiles * 16] byte offset of each row
  const uint32_t* row_type; // [n_tiles * 16] GGML type of each row (kNoRow: padding)
  int32_t n_tiles;
  int32_t cols;
};

// sum_e f16(w_e) * x_e over one block (fused multiply-add in f32).
__device__ __forceinline__ float dot_block(uint32_t t, const uint8_t* blk, const float* x, float acc) {
  switch (t) {
    case kGgmlQ4_K: {
      const float d = blk_half(blk), dmin = blk_half(blk + 2);
      for (int j = 0; j < 8; ++j) {
        int sc, m;
        scale_min_k4(j, blk + 4, sc, m);
        const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
        const uint8_t* q = blk + 16 + 32 * (j >> 1);
        const int sh = (j & 1) * 4;
#pragma unroll 8
        for (int l = 0; l < 32; ++l) {
          const float w = __fsub_rn(__fmul_rn(d1, (float)((q[l] >> sh) & 0x0f)), m1);
          acc = fmaf(f16_round(w), x[32 * j + l], acc);
        }
      }
      return acc;
    }
    case kGgmlQ6_K: {
      const float d = blk_half(blk + 208);
#pragma unroll 4
      for (int e = 0; e < 256; ++e) {
        const int n = e & 128, r = e & 127, g = r >> 5, l = r & 31;
        const uint8_t lo = (g & 1) ? blk[(n >> 1) + l + 32] : blk[(n >> 1) + l];
        const uint8_t qhb = blk[128 + (n >> 2) + l];
        const int q = (int)(((g & 2) ? (lo >> 4) : (lo & 0x0f)) | (((qhb >> (2 * g)) & 3) << 4)) - 32;
        const float sc = (float)(int8_t)blk[192 + (n >> 4) + (l >> 4) + 2 * g];
        acc = fmaf(f16_round(__fmul_rn(__fmul_rn(d, sc), (float)q)), x[e], acc);
      }
      return acc;
    }
    case kGgmlQ8_0: {
      const float d = blk_half(blk);
#pragma unroll 8
      for (int e = 0; e < 32; ++e)
        acc = fmaf(f16_round(__fmul_rn((float)(int8_t)blk[2 + e], d)), x[e], acc);
      return acc;
    }
    case kGgmlQ5_0: {
#pragma unroll 8
      for (int e = 0; e < 32; ++e) acc = fmaf(f16_round(q5_0_value(blk, e)), x[e], acc);
      return acc;
    }
    case kGgmlF16:
      return fmaf(f16_round(blk_half(blk)), x[0], acc);
    default: {
      float v;
      memcpy(&v, blk, 4);
      return fmaf(f16_round(v), x[0], acc);
    }
  }
}

template <int PRO, int EPI>
__global__ void __launch_bounds__(256) gemv_rows_kernel(const GemvArgs a, const RowsArgs r) {
  static_assert(PRO == PRO_PLAIN || PRO == PRO_NORM, "single-GPU prologues");
  extern __shared__ float xf[];  // [cols] the (normalized) input
  __shared__ double redd[kGemvWarps];
  __shared__ float redf[kGemvWarps];
  __shared__ float yrow[kTileRows];
  const int K = r.cols, tid = threadIdx.x;
  pdl_wait();
  float scale = 1.0f;
  if (PRO == PRO_NORM) {
    // rms_norm (src/decoder_ops.rs:126-144): f64 sum, mean cast to f32,
    // scale = 1/sqrt(mean + eps), y = x * scale * w with two rounded products
    double ss = 0.0;
    float mx = 0.0f;
    for (int i = tid; i < K; i += 256) ss += (double)a.x[i] * (double)a.x[i];
    block_sum_max<false>(ss, mx, redd, redf);
    const float mean = (float)(ss / (double)K);
    scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
  }
  for (int i = tid; i < K; i += 256) {
    const float y = PRO == PRO_NORM ? __fmul_rn(__fmul_rn(a.x[i], scale), a.norm_w[i]) : a.x[i];
    xf[i] = y;
    if (PRO == PRO_NORM && blockIdx.x == 0 && a.x_norm_out) a.x_norm_out[i] = y;
  }
  __syncthreads();
  pdl_launch_dependents();
  const int warp = tid >> 5, lane = tid & 31;
  for (int tile = blockIdx.x; tile < r.n_tiles; tile += gridDim.x) {
    float ys[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int sr = tile * kTileRows + 2 * warp + k;
      const uint32_t ty = r.row_type[sr];
      float acc = 0.0f;
      if (ty != kNoRow) {
        int be = 1, bb = 4;
        ggml_block_geometry(ty, be, bb);
        const uint8_t* row = r.bytes + r.row_off[sr];
        const int nbk = K / be;
        for (int b = lane; b < nbk; b += 32) acc = dot_block(ty, row + (size_t)b * bb, xf + b * be, acc);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      ys[k] = acc;
    }
    if (lane == 0) {
      yrow[2 * warp] = ys[0];
      yrow[2 * warp + 1] = ys[1];
    }
    __syncthreads();
    if (tid < kTileRows / 2) gemv_epilogue<EPI>(a, tile, tid, yrow[2 * tid], yrow[2 * tid + 1]);
    __syncthreads();
  }
}

}  // namespace faber
