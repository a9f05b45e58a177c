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
//     multicast) into a 4-stage ring;
//   * warp 1: allocates 256 TMEM columns, and lane 0 issues
//     tcgen05.mma.cta_group::1.kind::f16 (M 128, N 256, K 16) from the two
//     shared-memory descriptors, committing each stage back to its mbarrier;
//   * warps 2-9 (two per TMEM lane quadrant): fetch their rows' Q4_K bytes
//     from global memory into registers one super-block column ahead,
//     dequantize 128 rows x 64 weights per stage (a thread makes one row's
//     low- or high-nibble half) with the GEMV's exact f16 formation, write
//     them in the 128-byte-swizzled K-major layout the A descriptor reads
//     (a 6-stage ring; a slot is awaited only just before its store), and
//     finally read the accumulators (tcgen05.ld) for the epilogue.
// Every wait is bounded (g_pipe_error = 1 on expiry, then the CTA proceeds;
// barriers stay balanced).
#pragma once

#include <cudaTypedefs.h>

#include "attention.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "ops.cuh"

namespace faber {

constexpr int kPgBM = 128;
constexpr int kPgBN = 256;       // activation columns per tile in the prompt pass (128 tokens)
constexpr int kPgBK = 64;
constexpr int kPgAStages = 6;    // dequantized weight tiles in flight
constexpr int kPgBStages = 4;    // activation tiles in flight
constexpr int kPgThreads = 320;  // warp 0 loads, warp 1 MMA, warps 2-9 dequant + epilogue
constexpr int kPgDequantWarps = 8;
constexpr int kPgATile = kPgBM * kPgBK * 2;                         // 16 KB

// Shared-memory layout for an activation tile of BN columns (hi/lo rows).
template <int BN>
struct PgLayout {
  static constexpr int kBTile = BN * kPgBK * 2;                     // 32 KB at 256 columns
  static constexpr int kSmemA = 0;
  static constexpr int kSmemB = kSmemA + kPgAStages * kPgATile;     // 96 KB
  static constexpr int kSmemBars = kSmemB + kPgBStages * kBTile;
  static constexpr int kSmemXs = kSmemBars + 256;                    // BN/2 token row scales
  static constexpr int kBytes = kSmemXs + (BN / 2) * 4 + 1024;       // + alignment slack
  static_assert(kBytes <= 227 * 1024, "prefill GEMM shared memory above the per-CTA limit");
  static_assert((2 * kPgAStages + 2 * kPgBStages + 1) * 8 + 4 <= 256, "barrier area");
  static_assert(kSmemB % 1024 == 0 && kBTile % 1024 == 0,
                "128-byte-swizzled tiles start on 1024-byte boundaries");
  static_assert(BN == 32 || BN == 64 || BN == 128 || BN == 256, "TMEM columns: a power of two");
};

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

// 16 consecutive f32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 8 consecutive f32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

template <int CW>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float (&v)[CW]) {
  if constexpr (CW == 32) tmem_ld32(taddr, v);
  else if constexpr (CW == 16) tmem_ld16(taddr, v);
  else tmem_ld8(taddr, v);
}

// ---- the kernel -----------------------------------------------------------
template <int EPI, int BN>
__global__ void __launch_bounds__(kPgThreads, 1)
    prefill_gemm_kernel(const __grid_constant__ CUtensorMap xs_map, const PrefillGemmArgs a) {
  using Lay = PgLayout<BN>;
  constexpr int kPgSmemA = Lay::kSmemA, kPgSmemB = Lay::kSmemB, kPgSmemBars = Lay::kSmemBars;
  constexpr int kPgSmemXs = Lay::kSmemXs, kPgBTile = Lay::kBTile;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* sa = smem + kPgSmemA;
  uint8_t* sb = smem + kPgSmemB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPgSmemBars);
  uint64_t* b_full = bars;                     // [kPgBStages] TMA of Xs landed
  uint64_t* b_empty = b_full + kPgBStages;     // [kPgBStages] MMAs reading it finished
  uint64_t* a_full = b_empty + kPgBStages;     // [kPgAStages] the dequant warps wrote A
  uint64_t* a_empty = a_full + kPgAStages;     // [kPgAStages] MMAs reading it finished
  uint64_t* tile_done = a_empty + kPgAStages;  // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tile_done + 1);
  float* xs_s = reinterpret_cast<float*>(smem + kPgSmemXs);  // row scales of this tile's tokens

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the column tiles of one weight tile are neighbours in launch order, so
  // its Q4_K bytes come from DRAM once and from L2 for the others
  const int n_tile = blockIdx.x, m_tile = blockIdx.y;
  const int nkb = a.nb * (256 / kPgBK);  // K steps
  if (threadIdx.x < BN / 2) {
    const int t = n_tile * (BN / 2) + threadIdx.x;
    xs_s[threadIdx.x] = t < a.n_tok ? a.xscale[t] : 0.0f;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPgBStages; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int s = 0; s < kPgAStages; ++s) {
      mbar_init(&a_full[s], kPgDequantWarps);
      mbar_init(&a_empty[s], 1);
    }
    mbar_init(tile_done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kPgBStages;
        if (kb >= kPgBStages) mbar_wait(&b_empty[s], ((kb / kPgBStages) - 1) & 1);
        mbar_arrive_expect_tx(&b_full[s], (uint32_t)kPgBTile);
        tma_load_2d(sb + s * kPgBTile, &xs_map, kb * kPgBK, n_tile * BN, &b_full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(kPgBM, BN);
      for (int kb = 0; kb < nkb; ++kb) {
        const int sa_i = kb % kPgAStages, sb_i = kb % kPgBStages;
        mbar_wait(&a_full[sa_i], (kb / kPgAStages) & 1);
        mbar_wait(&b_full[sb_i], (kb / kPgBStages) & 1);
        tc_fence_after();
        const uint32_t a0 = smem_addr(sa + sa_i * kPgATile), b0 = smem_addr(sb + sb_i * kPgBTile);
#pragma unroll
        for (int j = 0; j < kPgBK / 16; ++j)  // K 16 = 32 bytes along the swizzled row
          umma_f16(tmem, umma_desc_sw128(a0 + 32 * j), umma_desc_sw128(b0 + 32 * j), idesc,
                   (kb | j) != 0);
        umma_commit(&a_empty[sa_i]);
        umma_commit(&b_empty[sb_i]);
      }
      umma_commit(tile_done);
    }
  } else {
    // dequant: thread i of warps 2-9 owns weight row i % 128 of the tile, the
    // low-nibble half (k 0..31 of the step, warps 2-5) or the high-nibble half
    // (k 32..63, warps 6-9): two dequantizing warps per scheduler. Each
    // thread reads its row's 16-byte header and 128 quant bytes of a
    // super-block column straight from global memory (L2: the column tiles
    // of this weight tile read the same bytes), one column ahead.
    const int i = threadIdx.x - 64;
    const int row = i & (kPgBM - 1), half = i >> 7;
    const int q_in_tile = row >> 4, row16 = row & 15;
    const int tile = m_tile * (kPgBM / kTileRows) + q_in_tile;
    const bool row_live = tile < a.n_tiles;  // rows past the weight read as zero blocks
    const uint8_t* wrow = a.w + (size_t)(row_live ? tile : 0) * a.nb * kTileItemBytes;
    LaneConst lc;
    asm("mov.b32 %0, 0x64006400;" : "=r"(lc.m1024));
    asm("mov.b32 %0, 0x54005400;" : "=r"(lc.m64));
    uint4 nh, nq[8];
    auto fetch = [&](int sbk) {
      const uint8_t* item = wrow + (size_t)sbk * kTileItemBytes;
      const uint4* qp = reinterpret_cast<const uint4*>(item + kTileRows * 16 + 128 * row16);
      const uint4 z = make_uint4(0u, 0u, 0u, 0u);
      nh = row_live ? __ldg(reinterpret_cast<const uint4*>(item + 16 * row16)) : z;
#pragma unroll
      for (int j = 0; j < 8; ++j) nq[j] = row_live ? __ldg(qp + j) : z;
    };
    fetch(0);
    for (int sbk = 0; sbk < a.nb; ++sbk) {
      const uint4 hdr = nh;
      uint4 q[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) q[j] = nq[j];
      if (sbk + 1 < a.nb) fetch(sbk + 1);
#pragma unroll
      for (int chunk = 0; chunk < 4; ++chunk) {
        const int kb = sbk * 4 + chunk, s = kb % kPgAStages;
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
          const uint32_t w = word_of(q[2 * chunk + (wd >> 2)], wd & 3);
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
        // the slot is free once the MMAs of step kb - kPgAStages finished
        if (kb >= kPgAStages) mbar_wait(&a_empty[s], ((kb / kPgAStages) - 1) & 1);
        uint8_t* arow = sa + s * kPgATile + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
          *reinterpret_cast<uint4*>(arow + (((4 * half + cc) ^ (row & 7)) << 4)) =
              make_uint4(h[4 * cc], h[4 * cc + 1], h[4 * cc + 2], h[4 * cc + 3]);
        // generic-proxy writes become visible to the tensor core's async proxy
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[s]);
      }
    }
    // epilogue: this warp's TMEM lane quadrant = rows 32 * (warp % 4) ..,
    // columns split between the two warps of a quadrant
    mbar_wait(tile_done, 0);
    tc_fence_after();
    const int quad = warp & 3;
    const int m = m_tile * kPgBM + quad * 32 + lane;
    constexpr int kCols = BN / 2;                  // columns of this warp
    const int cbeg = half * kCols;
    const bool row_ok = m < a.m_rows;
    constexpr int CW = kCols < 32 ? kCols : 32;    // columns per TMEM read
    constexpr int TPC = CW / 2;                    // tokens per TMEM read
    for (int c0 = cbeg; c0 < cbeg + kCols; c0 += CW) {
      float v[CW];
      tmem_ld_cols<CW>(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)c0, v);
      const int tb = (n_tile * BN + c0) / 2;  // first token of these column pairs
      float y[TPC];
#pragma unroll
      for (int j = 0; j < TPC; ++j) y[j] = (v[2 * j] + v[2 * j + 1]) * xs_s[c0 / 2 + j];
      // every load of a chunk is issued before its stores
      if (EPI == PG_STORE) {
#pragma unroll
        for (int j = 0; j < TPC; ++j)
          if (tb + j < a.n_tok && row_ok) a.out[(size_t)(tb + j) * a.ld_out + m] = y[j];
      } else if (EPI == PG_RESID) {
        float old[TPC];
#pragma unroll
        for (int j = 0; j < TPC; ++j)
          old[j] = (tb + j < a.n_tok && row_ok) ? a.out[(size_t)(tb + j) * a.ld_out + m] : 0.0f;
#pragma unroll
        for (int j = 0; j < TPC; ++j)
          if (tb + j < a.n_tok && row_ok) a.out[(size_t)(tb + j) * a.ld_out + m] = old[j] + y[j];
      } else if (EPI == PG_SWIGLU) {
        // rows 2f (gate) and 2f+1 (up) sit in adjacent lanes; of each token
        // pair the even lane finishes the first token and the odd lane the
        // second, each taking the partner row's value by one shuffle
        const bool odd = (lane & 1) != 0;
#pragma unroll
        for (int jj = 0; jj < TPC / 2; ++jj) {
          const float mine = odd ? y[2 * jj + 1] : y[2 * jj];
          const float other = __shfl_xor_sync(0xffffffffu, odd ? y[2 * jj] : y[2 * jj + 1], 1);
          const float g = odd ? other : mine, u = odd ? mine : other;
          const int t = tb + 2 * jj + (odd ? 1 : 0);
          if (t < a.n_tok && (m | 1) < a.m_rows) {
            const float sg = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
            a.out[(size_t)t * a.ld_out + (m >> 1)] = __fmul_rn(sg, u);
          }
        }
      } else if (EPI == PG_QKV) {
        const bool rope = m < a.nq + a.nk;  // Q and K rows (warp-uniform: head-aligned)
        const int kk = (m % a.head_dim) >> 1;
        int pos[TPC];
#pragma unroll
        for (int j = 0; j < TPC; ++j) pos[j] = a.pos0 + tb + j;
        float2 cs[TPC];
#pragma unroll
        for (int j = 0; j < TPC; ++j)
          cs[j] = (rope && tb + j < a.n_tok) ? a.rope[(size_t)pos[j] * (a.head_dim >> 1) + kk]
                                             : make_float2(0.0f, 0.0f);
#pragma unroll
        for (int j = 0; j < TPC; ++j) {
          const float y1 = __shfl_xor_sync(0xffffffffu, y[j], 1);
          const int t = tb + j;
          if (t < a.n_tok && row_ok) {
            __half* kc = a.k_cache;
            __half* vc = a.v_cache;
            if (rope) {
              // rope_norm pair (m even: first, odd: second) with host cos/sin
              const bool first = (m & 1) == 0;
              const float x0 = first ? y[j] : y1, x1 = first ? y1 : y[j];
              const float o = first ? __fsub_rn(__fmul_rn(x0, cs[j].x), __fmul_rn(x1, cs[j].y))
                                    : __fadd_rn(__fmul_rn(x0, cs[j].y), __fmul_rn(x1, cs[j].x));
              if (m < a.nq) a.q_out[(size_t)t * a.nq + m] = o;
              else kc[(size_t)pos[j] * a.nk + (m - a.nq)] = __float2half_rn(o);
            } else {
              vc[(size_t)pos[j] * a.nk + (m - a.nq - a.nk)] = __float2half_rn(y[j]);
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
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
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

// ---- causal attention of a prompt block on the tensor cores -----------------
//
// attention_gqa (src/cpu_oracle.rs:711-792) for a block of n queries at
// positions pos0 .. pos0 + n - 1 over the f16 K/V cache (positions 0 ..
// pos0 + n - 1, this block's rows already written by the QKV GEMM). Query
// row t of head h attends to the keys 0 .. pos0 + t of kv head h / ratio.
//
// CTA = (head, 64 queries), 4 warps of 16 queries; keys in tiles of 64,
// double-buffered in shared memory by cp.async (rows past the block's last
// key are zero-filled). Both products run on mma.sync m16n8k16 (f16 in, f32
// accumulate) with f32-faithful operands:
//   * each query row is scaled by a power of two 2^-s and split exactly,
//     q * 2^-s = qh + ql (two f16), so S = (qh + ql) K^T carries ~22 bits;
//     the K rows are f16 in the cache, so every product is exact;
//   * the probabilities p = exp(s - m) in [0, 1] are split p = ph + pl the
//     same way for O += (ph + pl) V.
// The softmax is the online (running max and sum) form; the result is O / l.
// Shared-memory rows are HD halfs with 16-byte chunks XOR-swizzled by the
// row's low three bits, so every ldmatrix phase touches 32 distinct banks.
constexpr int kFaQ = 64;
constexpr int kFaK = 64;
constexpr int kFaThreads = 128;

template <int HD>
__host__ __device__ constexpr int fa_tile_bytes() { return kFaK * HD * 2; }
// Qhi, Qlo (64 rows each), then two stages of (K, V)
template <int HD>
__host__ __device__ constexpr int fa_smem_bytes() { return 2 * kFaQ * HD * 2 + 4 * fa_tile_bytes<HD>(); }

template <int HD>
__device__ __forceinline__ uint32_t fa_off(int row, int chunk) {
  return (uint32_t)(row * HD * 2 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// D += A(16x16 f16, row) * B(16x8 f16, col), f32 accumulate (registers
// only, so the compiler may interleave independent accumulators)
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
// exact two-term split of (x, y): hi = f16(x, y), lo = f16 of the remainders
__device__ __forceinline__ void split2(float x, float y, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x, y);
  hi = h2_bits(h);
  lo = h2_bits(__floats2half2_rn(x - __low2float(h), y - __high2float(h)));
}

template <int HD>
__global__ void __launch_bounds__(kFaThreads) prefill_flash_kernel(const float* q, const __half* kc,
                                                                   const __half* vc, float* ctx,
                                                                   int n, int pos0, int n_heads,
                                                                   int n_kv_heads, float scale) {
  constexpr int CH = HD / 8;  // 16-byte chunks per row
  extern __shared__ __align__(128) unsigned char fa_smem[];
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(fa_smem);
  const uint32_t qh_base = sbase, ql_base = sbase + kFaQ * HD * 2;
  const uint32_t kv_base = sbase + 2 * kFaQ * HD * 2;  // stage s: K at +2s tiles, V at +2s+1
  const int h = blockIdx.x;
  const int qb = gridDim.y - 1 - blockIdx.y;  // the longest (causal) blocks start first
  const int q0 = qb * kFaQ;
  const int kh = h / (n_heads / n_kv_heads);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const size_t kvs = (size_t)n_kv_heads * HD, qstride = (size_t)n_heads * HD;
  const int kv_end = pos0 + min(n, q0 + kFaQ);  // keys [0, kv_end) are read
  const int nkb = (kv_end + kFaK - 1) / kFaK;
  const __half* kh_k = kc + (size_t)kh * HD;
  const __half* kh_v = vc + (size_t)kh * HD;

  auto load_tile = [&](int kb, int stage) {
    const uint32_t kdst = kv_base + (uint32_t)(2 * stage) * fa_tile_bytes<HD>();
    const uint32_t vdst = kdst + fa_tile_bytes<HD>();
#pragma unroll
    for (int i = 0; i < kFaK * CH / kFaThreads; ++i) {
      const int c = tid + i * kFaThreads;
      const int row = c / CH, ch = c % CH;
      const int key = kb * kFaK + row;
      const bool valid = key < kv_end;
      const size_t off = (size_t)(valid ? key : 0) * kvs + (size_t)ch * 8;
      cp_async16(kdst + fa_off<HD>(row, ch), kh_k + off, valid);
      cp_async16(vdst + fa_off<HD>(row, ch), kh_v + off, valid);
    }
    cp_async_commit();
  };
  load_tile(0, 0);

  // Q rows of this warp: power-of-two scale per row, exact hi/lo split
  int s_row0 = 0, s_row1 = 0;
  {
    constexpr int PL = HD / 32;  // values per lane
    for (int r = 0; r < 16; ++r) {
      const int row = warp * 16 + r, t = q0 + row;
      float v[PL];
      const float* src = q + (size_t)t * qstride + (size_t)h * HD + lane * PL;
      if constexpr (PL == 4) {
        const float4 f = t < n ? *reinterpret_cast<const float4*>(src) : make_float4(0.f, 0.f, 0.f, 0.f);
        v[0] = f.x;
        v[1] = f.y;
        v[2] = f.z;
        v[3] = f.w;
      } else {
        const float2 f = t < n ? *reinterpret_cast<const float2*>(src) : make_float2(0.f, 0.f);
        v[0] = f.x;
        v[1] = f.y;
      }
      float mx = 0.0f;
#pragma unroll
      for (int i = 0; i < PL; ++i) mx = fmaxf(mx, fabsf(v[i]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const int s = split_shift(mx);
      const float in_s = ldexpf(1.0f, -s);
      if (r == (lane >> 2)) s_row0 = s;
      if (r == (lane >> 2) + 8) s_row1 = s;
      uint32_t hb[PL / 2], lb[PL / 2];
#pragma unroll
      for (int i = 0; i < PL / 2; ++i) split2(v[2 * i] * in_s, v[2 * i + 1] * in_s, hb[i], lb[i]);
      // element d = lane * PL sits in chunk d / 8 at byte (d % 8) * 2
      const uint32_t o = fa_off<HD>(row, (lane * PL) / 8) + (uint32_t)((lane * PL) % 8) * 2;
      if constexpr (PL == 4) {
        asm volatile("st.shared.v2.b32 [%0], {%1,%2};\n" ::"r"(qh_base + o), "r"(hb[0]), "r"(hb[1]));
        asm volatile("st.shared.v2.b32 [%0], {%1,%2};\n" ::"r"(ql_base + o), "r"(lb[0]), "r"(lb[1]));
      } else {
        asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(qh_base + o), "r"(hb[0]));
        asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(ql_base + o), "r"(lb[0]));
      }
    }
  }
  const float f0 = ldexpf(scale, s_row0), f1 = ldexpf(scale, s_row1);
  // query positions of this thread's two accumulator rows, and the last key each may see
  const int t0 = q0 + warp * 16 + (lane >> 2);
  const int lim0 = min(pos0 + t0, kv_end - 1), lim1 = min(pos0 + t0 + 8, kv_end - 1);
  const int warp_min_lim = min(pos0 + q0 + warp * 16, kv_end - 1);

  float o_acc[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o_acc[i][0] = o_acc[i][1] = o_acc[i][2] = o_acc[i][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  const int mi = lane >> 3, r8 = lane & 7;

  for (int kb = 0; kb < nkb; ++kb) {
    const int stage = kb & 1;
    if (kb + 1 < nkb) {
      load_tile(kb + 1, stage ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t kbase = kv_base + (uint32_t)(2 * stage) * fa_tile_bytes<HD>();
    const uint32_t vbase = kbase + fa_tile_bytes<HD>();
    // S = Q K^T: 8 tiles of 16 queries x 8 keys
    float sacc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) sacc[i][0] = sacc[i][1] = sacc[i][2] = sacc[i][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t ah[4], al[4];
      const uint32_t qo = fa_off<HD>(warp * 16 + (mi & 1) * 8 + r8, 2 * kk + (mi >> 1));
      ldsm_x4(qh_base + qo, ah);
      ldsm_x4(ql_base + qo, al);
      uint32_t b[4][4];
#pragma unroll
      for (int np = 0; np < 4; ++np)
        ldsm_x4(kbase + fa_off<HD>(np * 16 + (mi >> 1) * 8 + r8, 2 * kk + (mi & 1)), b[np]);
      // the hi products of all 8 tiles, then the lo ones: no back-to-back
      // MMAs on one accumulator
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        mma16816(sacc[2 * np], ah, b[np][0], b[np][1]);
        mma16816(sacc[2 * np + 1], ah, b[np][2], b[np][3]);
      }
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        mma16816(sacc[2 * np], al, b[np][0], b[np][1]);
        mma16816(sacc[2 * np + 1], al, b[np][2], b[np][3]);
      }
    }
    // scale, mask, online softmax (rows r = lane/4 and r + 8; 4 lanes per row)
    const bool need_mask = kb * kFaK + kFaK - 1 > warp_min_lim;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = kb * kFaK + nt * 8 + 2 * (lane & 3) + e;
        float a = sacc[nt][e] * f0, b = sacc[nt][2 + e] * f1;
        if (need_mask) {
          a = key <= lim0 ? a : -INFINITY;
          b = key <= lim1 ? b : -INFINITY;
        }
        sacc[nt][e] = a;
        sacc[nt][2 + e] = b;
        mx0 = fmaxf(mx0, a);
        mx1 = fmaxf(mx1, b);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float base0 = mn0 == -INFINITY ? 0.0f : mn0, base1 = mn1 == -INFINITY ? 0.0f : mn1;
    const float c0 = expf(m0 - base0), c1 = expf(m1 - base1);
    m0 = mn0;
    m1 = mn1;
    float ps0 = 0.0f, ps1 = 0.0f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        sacc[nt][e] = expf(sacc[nt][e] - base0);
        sacc[nt][2 + e] = expf(sacc[nt][2 + e] - base1);
        ps0 += sacc[nt][e];
        ps1 += sacc[nt][2 + e];
      }
    }
    l0 = fmaf(l0, c0, ps0);
    l1 = fmaf(l1, c1, ps1);
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      o_acc[i][0] *= c0;
      o_acc[i][1] *= c0;
      o_acc[i][2] *= c1;
      o_acc[i][3] *= c1;
    }
    // O += P V: P from the S tiles (2j, 2j+1) as the A operand of key step j
#pragma unroll
    for (int j = 0; j < kFaK / 16; ++j) {
      uint32_t ph[4], pl[4];
      split2(sacc[2 * j][0], sacc[2 * j][1], ph[0], pl[0]);
      split2(sacc[2 * j][2], sacc[2 * j][3], ph[1], pl[1]);
      split2(sacc[2 * j + 1][0], sacc[2 * j + 1][1], ph[2], pl[2]);
      split2(sacc[2 * j + 1][2], sacc[2 * j + 1][3], ph[3], pl[3]);
#pragma unroll
      for (int dp = 0; dp < HD / 16; ++dp) {
        uint32_t b[4];
        ldsm_x4_t(vbase + fa_off<HD>(16 * j + (mi & 1) * 8 + r8, 2 * dp + (mi >> 1)), b);
        mma16816(o_acc[2 * dp], ph, b[0], b[1]);
        mma16816(o_acc[2 * dp + 1], ph, b[2], b[3]);
        mma16816(o_acc[2 * dp], pl, b[0], b[1]);
        mma16816(o_acc[2 * dp + 1], pl, b[2], b[3]);
      }
    }
    __syncthreads();  // the next iteration's load (or the merge rows) overwrites this stage
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
  float* out0 = ctx + (size_t)t0 * qstride + (size_t)h * HD + 2 * (lane & 3);
  float* out1 = out0 + 8 * qstride;
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) {
    if (t0 < n) *reinterpret_cast<float2*>(out0 + 8 * i) = make_float2(o_acc[i][0] * inv0, o_acc[i][1] * inv0);
    if (t0 + 8 < n) *reinterpret_cast<float2*>(out1 + 8 * i) = make_float2(o_acc[i][2] * inv1, o_acc[i][3] * inv1);
  }
}


// ---- grouped-query decode attention on the tensor cores ---------------------
//
// attention_gqa (src/cpu_oracle.rs:711-792) for one query row per sequence
// when several query heads share a kv head (ratio 3..8): the ratio's query
// heads form the 16-row M tile of m16n8k16 MMAs (rows past the ratio are
// zero), the cached keys the N dimension, so each K/V byte feeds every head
// of the group at once. CTA = (kv head, split, sequence), 4 warps; the
// split's keys go in tiles of 64, double-buffered by cp.async into
// XOR-swizzled shared memory, and each warp takes 16 keys of a tile:
//   * S = Q K^T with Q split exactly into hi/lo f16 (a power-of-two scale per
//     head), K f16 from the cache; score = (q . k) * scale;
//   * an online softmax per head row (running max and sum), P split into
//     hi/lo f16 for O += P V;
//   * the 4 warps' states combine in shared memory into the split's
//     (max, sum, context) partial, the same format and the same last-CTA
//     merge in split order as attention_decode_kernel.
constexpr int kGqaKeys = 64;

constexpr int kGqaCtasPerSm = 3;

// Q hi/lo rows, then two stages of K and V; after the key loop the stages
// hold the per-warp context rows (ratio <= 8) and (max, sum) pairs.
template <int HD>
__host__ __device__ constexpr int gqa_smem_bytes() {
  static_assert(4 * 8 * HD * 4 + 4 * 8 * 2 * 4 <= 2 * 2 * kGqaKeys * HD * 2, "merge rows fit the stages");
  return 2 * 16 * HD * 2 + 2 * 2 * kGqaKeys * HD * 2;
}

template <int HD>
__global__ void __launch_bounds__(128, kGqaCtasPerSm) attention_tc_kernel(const AttnArgs a0) {
  const AttnArgs a = slot_args(a0);
  constexpr int CH = HD / 8;
  extern __shared__ __align__(128) unsigned char gq_smem[];
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(gq_smem);
  const uint32_t qh_base = sbase, ql_base = sbase + 16 * HD * 2;
  const uint32_t kv_base = sbase + 2 * 16 * HD * 2;
  float* red = reinterpret_cast<float*>(gq_smem + 2 * 16 * HD * 2);  // aliases the K/V stages
  float* wst = red + 4 * 8 * HD;
  __shared__ int qshift[16];
  __shared__ int is_last;

  const int kh = blockIdx.x, split = blockIdx.y;
  const int ratio = a.n_heads / a.n_kv_heads;  // 3..8
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_wait();  // the step's own K/V row and q come from the preceding kernel
  pdl_launch_dependents();
  const int cur = a.st->cur_pos, n_kv = cur + 1;
  const int n_tiles = (n_kv + kGqaKeys - 1) / kGqaKeys;
  const int per = (n_tiles + gridDim.y - 1) / gridDim.y;
  const int active = (n_tiles + per - 1) / per;
  const int t0 = split * per, t1 = min(n_tiles, t0 + per);
  if (t0 >= t1) return;
  const size_t kvs = (size_t)a.n_kv_heads * HD;
  const __half* kh_k = a.k + (size_t)kh * HD;
  const __half* kh_v = a.v + (size_t)kh * HD;

  auto load_tile = [&](int t, int stage) {
    const uint32_t kdst = kv_base + (uint32_t)(2 * stage) * (kGqaKeys * HD * 2);
    const uint32_t vdst = kdst + kGqaKeys * HD * 2;
#pragma unroll
    for (int i = 0; i < kGqaKeys * CH / 128; ++i) {
      const int c = tid + i * 128;
      const int row = c / CH, ch = c % CH;
      const int key = t * kGqaKeys + row;
      const bool valid = key < n_kv;
      const size_t off = (size_t)(valid ? key : 0) * kvs + (size_t)ch * 8;
      cp_async16(kdst + fa_off<HD>(row, ch), kh_k + off, valid);
      cp_async16(vdst + fa_off<HD>(row, ch), kh_v + off, valid);
    }
    cp_async_commit();
  };
  load_tile(t0, 0);

  // Q rows: head kh * ratio + r for r < ratio, zero past it; per-row
  // power-of-two scale and exact hi/lo split (4 rows per warp)
  {
    constexpr int PL = HD / 32;
    for (int rr = 0; rr < 4; ++rr) {
      const int r = warp * 4 + rr;
      float v[PL];
#pragma unroll
      for (int i = 0; i < PL; ++i) v[i] = 0.0f;
      if (r < ratio) {  // only this kv head's query rows are read
        const float* src = a.q + (size_t)(kh * ratio + r) * HD + lane * PL;
#pragma unroll
        for (int i = 0; i < PL; ++i) v[i] = src[i];
      }
      float mx = 0.0f;
#pragma unroll
      for (int i = 0; i < PL; ++i) mx = fmaxf(mx, fabsf(v[i]));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const int sh = split_shift(mx);
      const float in_s = ldexpf(1.0f, -sh);
      if (lane == 0) qshift[r] = sh;
      uint32_t hb[PL / 2], lb[PL / 2];
#pragma unroll
      for (int i = 0; i < PL / 2; ++i) split2(v[2 * i] * in_s, v[2 * i + 1] * in_s, hb[i], lb[i]);
      const uint32_t o = fa_off<HD>(r, (lane * PL) / 8) + (uint32_t)((lane * PL) % 8) * 2;
      if constexpr (PL == 4) {
        asm volatile("st.shared.v2.b32 [%0], {%1,%2};\n" ::"r"(qh_base + o), "r"(hb[0]), "r"(hb[1]));
        asm volatile("st.shared.v2.b32 [%0], {%1,%2};\n" ::"r"(ql_base + o), "r"(lb[0]), "r"(lb[1]));
      } else {
        asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(qh_base + o), "r"(hb[0]));
        asm volatile("st.shared.b32 [%0], %1;\n" ::"r"(ql_base + o), "r"(lb[0]));
      }
    }
  }
  __syncthreads();
  const float f0 = ldexpf(a.scale, qshift[lane >> 2]), f1 = ldexpf(a.scale, qshift[(lane >> 2) + 8]);
  float o_acc[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o_acc[i][0] = o_acc[i][1] = o_acc[i][2] = o_acc[i][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  const int mi = lane >> 3, r8 = lane & 7;

  for (int t = t0; t < t1; ++t) {
    const int stage = (t - t0) & 1;
    if (t + 1 < t1) {
      load_tile(t + 1, stage ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t kbase = kv_base + (uint32_t)(2 * stage) * (kGqaKeys * HD * 2);
    const uint32_t vbase = kbase + kGqaKeys * HD * 2;
    // S = Q K^T over this warp's 16 keys: 2 tiles of 16 heads x 8 keys
    float sacc[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i) sacc[i][0] = sacc[i][1] = sacc[i][2] = sacc[i][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t ah[4], al[4], b[4];
      const uint32_t qo = fa_off<HD>((mi & 1) * 8 + r8, 2 * kk + (mi >> 1));
      ldsm_x4(qh_base + qo, ah);
      ldsm_x4(ql_base + qo, al);
      ldsm_x4(kbase + fa_off<HD>(warp * 16 + (mi >> 1) * 8 + r8, 2 * kk + (mi & 1)), b);
      mma16816(sacc[0], ah, b[0], b[1]);
      mma16816(sacc[1], ah, b[2], b[3]);
      mma16816(sacc[0], al, b[0], b[1]);
      mma16816(sacc[1], al, b[2], b[3]);
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = t * kGqaKeys + warp * 16 + nt * 8 + 2 * (lane & 3) + e;
        const float x0 = key < n_kv ? sacc[nt][e] * f0 : -INFINITY;
        const float x1 = key < n_kv ? sacc[nt][2 + e] * f1 : -INFINITY;
        sacc[nt][e] = x0;
        sacc[nt][2 + e] = x1;
        mx0 = fmaxf(mx0, x0);
        mx1 = fmaxf(mx1, x1);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float base0 = mn0 == -INFINITY ? 0.0f : mn0, base1 = mn1 == -INFINITY ? 0.0f : mn1;
    const float c0 = expf(m0 - base0), c1 = expf(m1 - base1);
    m0 = mn0;
    m1 = mn1;
    float ps0 = 0.0f, ps1 = 0.0f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        sacc[nt][e] = expf(sacc[nt][e] - base0);
        sacc[nt][2 + e] = expf(sacc[nt][2 + e] - base1);
        ps0 += sacc[nt][e];
        ps1 += sacc[nt][2 + e];
      }
    }
    l0 = fmaf(l0, c0, ps0);
    l1 = fmaf(l1, c1, ps1);
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      o_acc[i][0] *= c0;
      o_acc[i][1] *= c0;
      o_acc[i][2] *= c1;
      o_acc[i][3] *= c1;
    }
    // O += P V over the warp's 16 keys (one k-step)
    uint32_t ph[4], pl[4];
    split2(sacc[0][0], sacc[0][1], ph[0], pl[0]);
    split2(sacc[0][2], sacc[0][3], ph[1], pl[1]);
    split2(sacc[1][0], sacc[1][1], ph[2], pl[2]);
    split2(sacc[1][2], sacc[1][3], ph[3], pl[3]);
#pragma unroll
    for (int dp = 0; dp < HD / 16; ++dp) {
      uint32_t b[4];
      ldsm_x4_t(vbase + fa_off<HD>(warp * 16 + (mi & 1) * 8 + r8, 2 * dp + (mi >> 1)), b);
      mma16816(o_acc[2 * dp], ph, b[0], b[1]);
      mma16816(o_acc[2 * dp + 1], ph, b[2], b[3]);
      mma16816(o_acc[2 * dp], pl, b[0], b[1]);
      mma16816(o_acc[2 * dp + 1], pl, b[2], b[3]);
    }
    __syncthreads();  // the next iteration's load (or the merge rows) overwrites this stage
  }
  // this warp's state for head rows r < ratio (rows lane/4; rows + 8 are padding)
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  const int r = lane >> 2;
  if (r < ratio) {
    if ((lane & 3) == 0) {
      wst[(warp * 8 + r) * 2] = m0;
      wst[(warp * 8 + r) * 2 + 1] = l0;
    }
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      red[(warp * 8 + r) * HD + 8 * i + 2 * (lane & 3)] = o_acc[i][0];
      red[(warp * 8 + r) * HD + 8 * i + 2 * (lane & 3) + 1] = o_acc[i][1];
    }
  }
  __syncthreads();
  const int stride = HD + 2;
  for (int idx = tid; idx < ratio * HD; idx += 128) {
    const int rr = idx / HD, d = idx % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, wst[(w * 8 + rr) * 2]);
    float L = 0.0f, sum = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = wst[(w * 8 + rr) * 2];
      const float f = mw == -INFINITY ? 0.0f : expf(mw - M);
      L = fmaf(wst[(w * 8 + rr) * 2 + 1], f, L);
      sum = fmaf(red[(w * 8 + rr) * HD + d], f, sum);
    }
    float* pp = a.part + ((size_t)(kh * ratio + rr) * a.max_splits + split) * stride;
    pp[2 + d] = sum;
    if (d == 0) {
      pp[0] = M;
      pp[1] = L;
    }
  }
  // the last CTA of this kv head merges all splits in split order
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int ticket = atomicAdd(&a.counters[kh], 1);
    is_last = (ticket == active - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int idx = tid; idx < ratio * HD; idx += 128) {
    const int rr = idx / HD, d = idx % HD;
    const float* base = a.part + (size_t)(kh * ratio + rr) * a.max_splits * stride;
    float M = -INFINITY, L = 0.0f, acc_d = 0.0f;
    for (int s0 = 0; s0 < active; s0 += kAttnMergeBatch) {
      float ms[kAttnMergeBatch], ls[kAttnMergeBatch], vs[kAttnMergeBatch];
#pragma unroll
      for (int u = 0; u < kAttnMergeBatch; ++u) {
        const bool ok = s0 + u < active;
        const float* pq = base + (size_t)(s0 + u) * stride;
        ms[u] = ok ? __ldcg(pq) : -INFINITY;
        ls[u] = ok ? __ldcg(pq + 1) : 0.0f;
        vs[u] = ok ? __ldcg(pq + 2 + d) : 0.0f;
      }
      float mb = M;
#pragma unroll
      for (int u = 0; u < kAttnMergeBatch; ++u) mb = fmaxf(mb, ms[u]);
      const float c = expf(M - mb);
      L *= c;
      acc_d *= c;
#pragma unroll
      for (int u = 0; u < kAttnMergeBatch; ++u) {
        const float f = expf(ms[u] - mb);
        L = fmaf(ls[u], f, L);
        acc_d = fmaf(vs[u], f, acc_d);
      }
      M = mb;
    }
    a.ctx[(size_t)(kh * ratio + rr) * HD + d] = acc_d / L;
  }
  if (tid == 0) a.counters[kh] = 0;
}

}  // namespace faber
