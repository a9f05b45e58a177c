// prefill.cuh — batched Q4_K GEMM for prompt processing on the 5th-generation
// tensor cores (tcgen05 + TMEM), sm_100a.
//
//   Y[t][m] = sum_k W[m][k] X[t][k],  t = 0..n-1 tokens, W Q4_K (tile layout)
//
// the reference's dense (src/decoder_ops.rs:378-406) applied to every prompt
// row at once, with the f16-rounded dequantized weights of
// src/cpu_oracle.rs:356-360. The activations keep about f32 accuracy: each
// row of X is split exactly into two f16 rows (x * 2^-s = hi + lo, s a
// per-row power of two), so the MMA's N dimension carries (hi, lo) pairs and
// the epilogue adds the two accumulator columns and rescales.
//
// One CTA computes a 128 x 256 tile of D = W * Xs^T (128 weight rows x 128
// tokens as 256 hi/lo columns) over K in steps of 64:
//   * warp 0, lane 0: TMA loads of the Xs tile (128-byte swizzle, no
//     multicast) into a 3-stage ring, and bulk copies of the raw Q4_K tile
//     items (one super-block column at a time) into a double buffer;
//   * warp 1: allocates 256 TMEM columns, and lane 0 issues
//     tcgen05.mma.cta_group::1.kind::f16 (M 128, N 256, K 16) from the two
//     shared-memory descriptors, committing each stage back to its mbarrier;
//   * warps 2-9 (two per TMEM lane quadrant): dequantize 128 rows x 64
//     weights per stage (a thread makes one row's low- or high-nibble half)
//     with the GEMV's exact f16 formation, write them in the 128-byte-swizzled
//     K-major layout the A descriptor reads, and finally read the
//     accumulators (tcgen05.ld) for the epilogue.
// Every wait is bounded (g_pipe_error = 1 on expiry, then the CTA proceeds;
// barriers stay balanced).
#pragma once

#include <cudaTypedefs.h>

#include "common.cuh"
#include "gemv.cuh"

namespace faber {

constexpr int kPgBM = 128;
constexpr int kPgBN = 256;
constexpr int kPgBK = 64;
constexpr int kPgStages = 3;
constexpr int kPgThreads = 320;  // warp 0 loads, warp 1 MMA, warps 2-9 dequant + epilogue
constexpr int kPgDequantWarps = 8;
constexpr int kPgATile = kPgBM * kPgBK * 2;                         // 16 KB
constexpr int kPgBTile = kPgBN * kPgBK * 2;                         // 32 KB
constexpr int kPgRaw = (kPgBM / kTileRows) * kTileItemBytes;        // 18 KB
constexpr int kPgSmemA = 0;
constexpr int kPgSmemB = kPgSmemA + kPgStages * kPgATile;           // 48 KB
constexpr int kPgSmemRaw = kPgSmemB + kPgStages * kPgBTile;         // 144 KB
constexpr int kPgSmemBars = kPgSmemRaw + 2 * kPgRaw;                // 180 KB
constexpr int kPgSmemBytes = kPgSmemBars + 256 + 1024;              // + barriers + alignment slack

// Epilogues of the prefill GEMM (per output element y[t][m]).
enum PrefillEpi : int {
  PG_STORE = 0,   // out[t][m] = y
  PG_RESID = 1,   // out[t][m] += y (residual_add, src/decoder_ops.rs:420-427)
  PG_SWIGLU = 2,  // rows interleaved gate/up: out[t][m/2] = silu(g) * u
  PG_QKV = 3      // RoPE on Q/K pairs, Q -> q_out[t], K/V -> f16 cache at position pos0 + t
};

struct PrefillGemmArgs {
  const uint8_t* w;        // tile layout, 2304-byte items [n_tiles][nb]
  int32_t n_tiles, nb;     // 16-row tiles, 256-element super-block columns
  int32_t m_rows;          // true output features
  int32_t n_tok;           // tokens in this call
  const float* xscale;     // [n_tok] power-of-two row scales of Xs
  float* out;              // PG_STORE/RESID: [n_tok][ld_out]; PG_SWIGLU: [n_tok][m_rows/2]
  int32_t ld_out;
  // PG_QKV
  float* q_out;            // [n_tok][nq]
  __half* k_cache;         // [ctx][nk], rows from position pos0
  __half* v_cache;
  const float2* rope;      // [ctx][head_dim/2]
  int32_t nq, nk, head_dim, pos0;
};

// ---- tcgen05 / TMA helpers ------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

// K-major operand in the 128-byte-swizzled canonical layout: 8-row atoms of
// 1024 bytes (stride 1024), 16-byte leading offset, descriptor version 1.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);         // start address
  d |= (uint64_t)1u << 16;                         // leading byte offset 16 B
  d |= (uint64_t)(1024u >> 4) << 32;               // stride byte offset 1024 B
  d |= (uint64_t)1u << 46;                         // version (sm_100)
  d |= (uint64_t)2u << 61;                         // 128-byte swizzle
  return d;
}

// kind::f16 instruction descriptor: D f32, A and B f16, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int m, int n) {
  return (1u << 4)                       // D format f32
         | (0u << 7) | (0u << 10)        // A, B f16
         | ((uint32_t)(n >> 3) << 17)    // N / 8
         | ((uint32_t)(m >> 4) << 24);   // M / 16
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

// 32 consecutive f32 columns of this warp's 32 TMEM lanes (one row per lane).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- the kernel -----------------------------------------------------------
template <int EPI>
__global__ void __launch_bounds__(kPgThreads, 1)
    prefill_gemm_kernel(const __grid_constant__ CUtensorMap xs_map, const PrefillGemmArgs a) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* sa = smem + kPgSmemA;
  uint8_t* sb = smem + kPgSmemB;
  uint8_t* sraw = smem + kPgSmemRaw;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPgSmemBars);
  uint64_t* b_full = bars;                    // [3] TMA of Xs landed
  uint64_t* a_full = bars + kPgStages;        // [3] 4 dequant warps wrote A
  uint64_t* s_done = bars + 2 * kPgStages;    // [3] MMAs of the stage finished
  uint64_t* raw_full = bars + 3 * kPgStages;  // [2]
  uint64_t* raw_empty = raw_full + 2;         // [2]
  uint64_t* tile_done = raw_empty + 2;        // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tile_done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tile = blockIdx.x, n_tile = blockIdx.y;
  const int nkb = a.nb * (256 / kPgBK);  // K steps
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPgStages; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&a_full[s], kPgDequantWarps);
      mbar_init(&s_done[s], 1);
    }
    for (int r = 0; r < 2; ++r) {
      mbar_init(&raw_full[r], 1);
      mbar_init(&raw_empty[r], kPgDequantWarps);
    }
    mbar_init(tile_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(kPgBN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      uint64_t policy;
      asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
      const int tiles_here = min(kPgBM / kTileRows, a.n_tiles - m_tile * (kPgBM / kTileRows));
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kPgStages;
        if (kb >= kPgStages) mbar_wait(&s_done[s], ((kb / kPgStages) - 1) & 1);
        if (kb % 4 == 0) {  // raw Q4_K items of super-block column kb / 4
          const int sbk = kb / 4, r = sbk & 1;
          if (sbk >= 2) mbar_wait(&raw_empty[r], ((sbk / 2) - 1) & 1);
          mbar_arrive_expect_tx(&raw_full[r], (uint32_t)(tiles_here * kTileItemBytes));
          for (int i = 0; i < tiles_here; ++i)
            bulk_g2s(sraw + r * kPgRaw + i * kTileItemBytes,
                     a.w + ((size_t)(m_tile * (kPgBM / kTileRows) + i) * a.nb + sbk) * kTileItemBytes,
                     kTileItemBytes, &raw_full[r], policy);
        }
        mbar_arrive_expect_tx(&b_full[s], (uint32_t)kPgBTile);
        tma_load_2d(sb + s * kPgBTile, &xs_map, kb * kPgBK, n_tile * kPgBN, &b_full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(kPgBM, kPgBN);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kPgStages;
        const uint32_t ph = (kb / kPgStages) & 1;
        mbar_wait(&a_full[s], ph);
        mbar_wait(&b_full[s], ph);
        tc_fence_after();
        const uint32_t a0 = smem_addr(sa + s * kPgATile), b0 = smem_addr(sb + s * kPgBTile);
#pragma unroll
        for (int j = 0; j < kPgBK / 16; ++j)  // K 16 = 32 bytes along the swizzled row
          umma_f16(tmem, umma_desc_sw128(a0 + 32 * j), umma_desc_sw128(b0 + 32 * j), idesc,
                   (kb | j) != 0);
        umma_commit(&s_done[s]);
      }
      umma_commit(tile_done);
    }
  } else {
    // dequant: thread i of warps 2-9 owns weight row i % 128 of the tile, the
    // low-nibble half (k 0..31 of the step, warps 2-5) or the high-nibble half
    // (k 32..63, warps 6-9): two dequantizing warps per scheduler
    const int i = threadIdx.x - 64;
    const int row = i & (kPgBM - 1), half = i >> 7;
    const int q_in_tile = row >> 4, row16 = row & 15;
    LaneConst lc;
    asm("mov.b32 %0, 0x64006400;" : "=r"(lc.m1024));
    asm("mov.b32 %0, 0x54005400;" : "=r"(lc.m64));
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % kPgStages, sbk = kb / 4, r = sbk & 1, chunk = kb % 4;
      if (chunk == 0) mbar_wait(&raw_full[r], (sbk / 2) & 1);
      if (kb >= kPgStages) mbar_wait(&s_done[s], ((kb / kPgStages) - 1) & 1);
      const uint8_t* item = sraw + r * kPgRaw + q_in_tile * kTileItemBytes;
      const uint4 hdr = *reinterpret_cast<const uint4*>(item + 16 * row16);
      const uint8_t* qs = item + 256 + 128 * row16 + 32 * chunk;
      const uint4 q0 = *reinterpret_cast<const uint4*>(qs);
      const uint4 q1 = *reinterpret_cast<const uint4*>(qs + 16);
      {
        const uint32_t k = 2u * (uint32_t)(chunk & 1);
        lc.sel = k | (5u << 4) | ((k + 1u) << 8) | (7u << 12);
      }
      const RowScales3 sc = row_scales3(hdr, chunk, lc);
      // this half's scale constants: sub-block 2c (low nibbles) or 2c + 1
      const uint32_t sc2 = half ? sc.schi2 : sc.sclo2, c2 = half ? sc.chi2 : sc.clo2;
      const float nm = half ? sc.nm2 : sc.nm1;
      uint32_t h[16];  // 32 f16: k 32 * half + 0..31
#pragma unroll
      for (int wd = 0; wd < 8; ++wd) {
        const uint32_t w = word_of(wd < 4 ? q0 : q1, wd & 3);
        const uint32_t u = w >> 8;
        // (k0, k2) from bytes 0/2 and (k1, k3) from bytes 1/3 of the word
        const uint32_t p02 = half ? hfma2_u(and_or<0x00f000f0u>(w, lc.m64), sc2, c2)
                                  : hfma2_u(and_or<0x000f000fu>(w, lc.m1024), sc2, c2);
        const uint32_t p13 = half ? hfma2_u(and_or<0x00f000f0u>(u, lc.m64), sc2, c2)
                                  : hfma2_u(and_or<0x000f000fu>(u, lc.m1024), sc2, c2);
        const float2 a02 = mixed_fma_pair(p02, sc.dword, nm);
        const float2 a13 = mixed_fma_pair(p13, sc.dword, nm);
        const uint32_t v02 = pack_half2(a02.x, a02.y), v13 = pack_half2(a13.x, a13.y);
        h[2 * wd] = prmt<0x5410>(v02, v13);      // (k0, k1)
        h[2 * wd + 1] = prmt<0x7632>(v02, v13);  // (k2, k3)
      }
      {
        uint8_t* arow = sa + s * kPgATile + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
          *reinterpret_cast<uint4*>(arow + (((4 * half + cc) ^ (row & 7)) << 4)) =
              make_uint4(h[4 * cc], h[4 * cc + 1], h[4 * cc + 2], h[4 * cc + 3]);
      }
      // generic-proxy writes become visible to the tensor core's async proxy
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&a_full[s]);
        if (chunk == 3) mbar_arrive(&raw_empty[r]);
      }
    }
    // epilogue: this warp's TMEM lane quadrant = rows 32 * (warp % 4) ..,
    // columns split between the two warps of a quadrant
    mbar_wait(tile_done, 0);
    tc_fence_after();
    const int quad = warp & 3;
    const int m = m_tile * kPgBM + quad * 32 + lane;
    const int cbeg = half * (kPgBN / 2);
    for (int c0 = cbeg; c0 < cbeg + kPgBN / 2; c0 += 32) {
      float v[32];
      tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)c0, v);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int t = (n_tile * kPgBN + c0) / 2 + j;
        const bool live = t < a.n_tok;
        const float y = live ? (v[2 * j] + v[2 * j + 1]) * a.xscale[t] : 0.0f;
        if (EPI == PG_STORE) {
          if (live && m < a.m_rows) a.out[(size_t)t * a.ld_out + m] = y;
        } else if (EPI == PG_RESID) {
          if (live && m < a.m_rows) a.out[(size_t)t * a.ld_out + m] += y;
        } else if (EPI == PG_SWIGLU) {
          // rows 2f (gate) and 2f+1 (up) sit in adjacent lanes
          const float u = __shfl_xor_sync(0xffffffffu, y, 1);
          if (live && (lane & 1) == 0 && m + 1 < a.m_rows) {
            const float sg = __fdiv_rn(y, __fadd_rn(1.0f, expf(-y)));
            a.out[(size_t)t * a.ld_out + (m >> 1)] = __fmul_rn(sg, u);
          }
        } else {  // PG_QKV
          const float y1 = __shfl_xor_sync(0xffffffffu, y, 1);
          if (live && m < a.m_rows) {
            const int pos = a.pos0 + t;
            if (m < a.nq + a.nk) {
              // rope_norm pair (m even: first, odd: second) with host cos/sin
              const int kk = (m % a.head_dim) >> 1;
              const float2 cs = a.rope[(size_t)pos * (a.head_dim >> 1) + kk];
              const bool first = (m & 1) == 0;
              const float x0 = first ? y : y1, x1 = first ? y1 : y;
              const float o = first ? __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y))
                                    : __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
              if (m < a.nq) a.q_out[(size_t)t * a.nq + m] = o;
              else a.k_cache[(size_t)pos * a.nk + (m - a.nq)] = __float2half_rn(o);
            } else {
              a.v_cache[(size_t)pos * a.nk + (m - a.nq - a.nk)] = __float2half_rn(y);
            }
          }
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPgBN));
  }
}

// ---- per-token kernels of the prompt pass -----------------------------------

// embed_rows (src/cpu_oracle.rs:538-545) for a block of tokens: rows of the
// f16 table (the oracle's f16-rounded token_embd) to f32. An id outside the
// vocab sets the step status and yields a zero row.
__global__ void prefill_embed_kernel(const int64_t* tokens, const __half* embd, int d, int vocab,
                                     float* h, int32_t* status) {
  const int t = blockIdx.x;
  const int64_t tok = tokens[t];
  const bool ok = tok >= 0 && tok < vocab;
  for (int i = threadIdx.x; i < d; i += blockDim.x)
    h[(size_t)t * d + i] = ok ? __half2float(embd[(size_t)tok * d + i]) : 0.0f;
  if (!ok && threadIdx.x == 0) *status = 1;
}

// One token row per CTA (256 threads): y = rms_norm(x, w) (src/decoder_ops.rs:
// 126-144: f64 sum, IEEE sqrt and divide, two rounded products) or y = x, and
// its exact two-term f16 split into rows 2t (hi) and 2t+1 (lo) of xs, scaled
// by 2^-s with max|y| * 2^-s in [2^13, 2^14); xscale[t] = 2^s.
template <bool NORM>
__global__ void __launch_bounds__(kGemvThreads) prefill_split_kernel(const float* x, int K,
                                                                     const float* w, float eps,
                                                                     __half* xs, float* xscale) {
  __shared__ double redd[kGemvWarps];
  __shared__ float redf[kGemvWarps];
  const int t = blockIdx.x;
  const float* xr = x + (size_t)t * K;
  double ss = 0.0;
  float mx = 0.0f;
  for (int i = threadIdx.x; i < K; i += kGemvThreads) {
    const float v = xr[i];
    if (NORM) {
      ss += (double)v * (double)v;
      mx = fmaxf(mx, fabsf(v * w[i]));
    } else {
      mx = fmaxf(mx, fabsf(v));
    }
  }
  block_sum_max<false>(ss, mx, redd, redf);
  float scale = 1.0f, bound = mx;
  if (NORM) {
    const float mean = (float)(ss / (double)K);
    scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    bound = mx * scale * 1.001f;
  }
  const int s = split_shift(bound);
  const float in_s = ldexpf(1.0f, -s);
  __half* hi = xs + (size_t)(2 * t) * K;
  __half* lo = hi + K;
  for (int i = threadIdx.x; i < K; i += kGemvThreads) {
    const float y = NORM ? __fmul_rn(__fmul_rn(xr[i], scale), w[i]) : xr[i];
    const float v = y * in_s;
    const __half hv = __float2half_rn(v);
    hi[i] = hv;
    lo[i] = __float2half_rn(v - __half2float(hv));
  }
  if (threadIdx.x == 0) xscale[t] = ldexpf(1.0f, s);
}

// Sum over the warp of 32 per-lane values; lane l returns the total of value
// l (levels pair lanes differing in bit 4, 3, 2, 1, 0).
__device__ __forceinline__ float butterfly32(float (&p)[32], int lane) {
#pragma unroll
  for (int level = 0; level < 5; ++level) {
    const int half = 16 >> level;
    const bool upper = (lane & half) != 0;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float keep = upper ? p[i + half] : p[i];
      const float send = upper ? p[i] : p[i + half];
      p[i] = keep + __shfl_xor_sync(0xffffffffu, send, half);
    }
  }
  return p[0];
}

// Causal GQA attention of a prompt block (attention_gqa, src/cpu_oracle.rs:
// 711-792): query t of the block sits at position pos0 + t and attends to the
// cached positions 0..pos0 + t (kv head h / ratio). CTA = (head, 16 queries),
// 4 warps of 4 queries; lanes own head_dim / 32 dims. Keys go 8 at a time:
// per-lane partial dots of 4 queries x 8 keys, a 32-value butterfly leaves
// lane l with the score of (query l >> 3, key l & 7); then an online softmax
// per query (every lane keeps all 4 queries' max and sum) and the p * V
// update with p broadcast by shuffles. scale = 1 / sqrt(head_dim).
template <int HD>
__global__ void __launch_bounds__(128) prefill_attention_kernel(const float* q, const __half* kc,
                                                                const __half* vc, float* ctx,
                                                                int n, int pos0, int n_heads,
                                                                int n_kv_heads, float scale) {
  constexpr int DPL = HD / 32;
  const int h = blockIdx.x, q0 = blockIdx.y * 16;
  const int kh = h / (n_heads / n_kv_heads);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t kvs = (size_t)n_kv_heads * HD, qstride = (size_t)n_heads * HD;
  const size_t col = (size_t)kh * HD + lane * DPL;
  float qv[4][DPL], m[4], l[4], acc[4][DPL];
  int qpos[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = q0 + warp * 4 + i;
    qpos[i] = t < n ? pos0 + t : -1;  // -1: no query (every key masked)
#pragma unroll
    for (int d = 0; d < DPL; ++d) {
      qv[i][d] = t < n ? q[(size_t)t * qstride + (size_t)h * HD + lane * DPL + d] : 0.0f;
      acc[i][d] = 0.0f;
    }
    m[i] = -INFINITY;
    l[i] = 0.0f;
  }
  const int last = max(max(qpos[0], qpos[1]), max(qpos[2], qpos[3]));
  const int qi = lane >> 3, kk = lane & 7;
  for (int j0 = 0; j0 <= last; j0 += 8) {
    float kf[8][DPL];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const bool in = j0 + k <= last;
#pragma unroll
      for (int d = 0; d < DPL; d += 2) {
        float2 f = make_float2(0.0f, 0.0f);
        if (in) f = __half22float2(*reinterpret_cast<const __half2*>(kc + (size_t)(j0 + k) * kvs + col + d));
        kf[k][d] = f.x;
        kf[k][d + 1] = f.y;
      }
    }
    float p[32];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float s = 0.0f;
#pragma unroll
        for (int d = 0; d < DPL; ++d) s = fmaf(qv[i][d], kf[k][d], s);
        p[i * 8 + k] = s;
      }
    const float dot = butterfly32(p, lane);
    int my_pos = qpos[0];
#pragma unroll
    for (int i = 1; i < 4; ++i) my_pos = qi == i ? qpos[i] : my_pos;
    const bool valid = j0 + kk <= my_pos;
    const float sc = valid ? dot * scale : -INFINITY;
    float gm = sc;
    gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, 1));
    gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, 2));
    gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, 4));
    float mn[4], c[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      mn[i] = fmaxf(m[i], __shfl_sync(0xffffffffu, gm, 8 * i));
      c[i] = mn[i] == -INFINITY ? 1.0f : expf(m[i] - mn[i]);
    }
    float my_mn = mn[0];
#pragma unroll
    for (int i = 1; i < 4; ++i) my_mn = qi == i ? mn[i] : my_mn;
    const float e = valid ? expf(sc - my_mn) : 0.0f;
    float es = e;
    es += __shfl_xor_sync(0xffffffffu, es, 1);
    es += __shfl_xor_sync(0xffffffffu, es, 2);
    es += __shfl_xor_sync(0xffffffffu, es, 4);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      l[i] = fmaf(l[i], c[i], __shfl_sync(0xffffffffu, es, 8 * i));
      m[i] = mn[i];
#pragma unroll
      for (int d = 0; d < DPL; ++d) acc[i][d] *= c[i];
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float vf[DPL];
      const bool in = j0 + k <= last;
#pragma unroll
      for (int d = 0; d < DPL; d += 2) {
        float2 f = make_float2(0.0f, 0.0f);
        if (in) f = __half22float2(*reinterpret_cast<const __half2*>(vc + (size_t)(j0 + k) * kvs + col + d));
        vf[d] = f.x;
        vf[d + 1] = f.y;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float pik = __shfl_sync(0xffffffffu, e, 8 * i + k);
#pragma unroll
        for (int d = 0; d < DPL; ++d) acc[i][d] = fmaf(pik, vf[d], acc[i][d]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = q0 + warp * 4 + i;
    if (t >= n) continue;
#pragma unroll
    for (int d = 0; d < DPL; ++d)
      ctx[(size_t)t * qstride + (size_t)h * HD + lane * DPL + d] = acc[i][d] / l[i];
  }
}

}  // namespace faber
