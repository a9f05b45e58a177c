// bgemv.cuh — batched-decode Q4_K GEMV: up to 16 sequences share every exact
// weight formation (sm_100a).
//
// y[s][j] = sum_i w[j][i] * x[s][i] for the sequences s of a batch, with the
// weights formed exactly as in the single-sequence GEMV (gemv.cuh: f16-rounded
// dequant_q4_k values, src/dequant.rs:194-217, src/cpu_oracle.rs:356-360).
// The weight formation, not HBM, bounds the single-sequence kernel, so the
// batch reuses each formed 16x16 weight fragment for NB m16n8k16 MMAs: the B
// operand's 8 columns hold the exact hi/lo f16 split of 4 sequences each
// (columns 2s, 2s+1), so 16 sequences cost 4 MMAs per fragment instead of 16
// formations.
//
// Data path: one CTA per SM, one producer warp streaming 2304-byte tile
// items with bulk copies (no multicast) into a 3-stage ring, 8 consumer
// warps and an epilogue warp. The x rows of every sequence do not all fit in shared memory, so K
// is cut into slabs of whole super-blocks (as many as the x rows of all
// sequences fit); the CTAs are split into one group per slab, each group
// stages its slab once and walks the row tiles. Within a tile the 8 warps
// split the slab's super-blocks and hand their partial tiles to the epilogue
// warp, which sums them in a fixed order. With more than one slab, each (tile, slab) partial
// goes to global scratch and bg_combine_kernel sums the slabs in slab order,
// so results do not depend on timing. Epilogues: the
// batched decode's QKV (RoPE + each sequence's K/V rows at its own position),
// residual add, SwiGLU, logits + per-sequence argmax, and a plain store.
#pragma once

#include "gemv.cuh"
#include "ops.cuh"

namespace faber {

enum BgemvEpilogue : int { BG_STORE = 0, BG_RESID = 1, BG_SWIGLU = 2, BG_QKV = 3, BG_LOGITS = 4 };

constexpr int kBgMaxSeq = 16;
constexpr int kBgStages = 4;
constexpr int kBgParts = 2;  // partial-tile buffers between the warps and the epilogue warp
constexpr size_t kBgSmemMax = 227 * 1024;

struct BgemvArgs {
  const uint8_t* w;        // tiled Q4_K weight (identity layout)
  int32_t n_tiles, nb, n_rows;
  const __half* xs;        // [2B][K] rows: hi and lo of sequence s at rows 2s, 2s+1
  const float* xscale;     // [B] power-of-two scale of each sequence's split
  int32_t B, K;
  int32_t slab_sb, n_slabs;  // super-blocks per K slab, slabs
  float* part;             // n_slabs > 1: [n_slabs][n_tiles][16 * B] scaled partial sums
  float* out;              // STORE/RESID/LOGITS: [B][ld_out]; SWIGLU: [B][ld_out] (half rows)
  int32_t ld_out;
  float* q_out;            // QKV: [B][nq]
  const float2* rope;      // QKV: [ctx][head_dim/2] (cos, sin)
  int32_t nq, nk, head_dim;
  const SlotRef* slots;    // QKV/LOGITS: [B] step state and this layer's K/V rows
  int32_t n_eog;
  int64_t eog[kMaxEog];
};

// Shared-memory plan of one launch: ring, x slab rows, partial tiles, barriers.
// Per-sequence values a launch reads in every epilogue, staged once.
struct BgMeta {
  StepState* st;
  __half* k;
  __half* v;
  int32_t pos;
  float xscale;
};

struct BgLayout {
  size_t ring, xs, part, meta, bars, total;
  int row_halves;  // x row stride (halves): rows start 16 bytes apart mod 128
};

// Shared-memory position (halves) of element j (a multiple of 8) of a staged
// x row: its 16-byte chunk k moves to k ^ (2 * ((k >> 3) & 3)), so the four
// lane groups t of one B-fragment load (chunks 8t apart) use four different
// 16-byte bank slots, and the next row (16 bytes on) the other four.
__host__ __device__ __forceinline__ int bg_swz(int j) {
  const int k = j >> 3;
  return (k ^ (((k >> 3) & 3) << 1)) << 3;
}

__host__ __device__ inline BgLayout bg_layout(int slab_sb, int B) {
  BgLayout L;
  const int n = slab_sb * 256;
  const int rh = n + 8;  // 2n is a multiple of 512: rows 16 bytes apart mod 128
  L.row_halves = rh;
  L.ring = 0;
  L.xs = (size_t)kBgStages * kStageBytes;
  L.part = L.xs + (size_t)2 * B * rh * 2;
  L.part = (L.part + 15) & ~(size_t)15;
  L.meta = L.part + (size_t)kBgParts * kConsumerWarps * kTileRows * kBgMaxSeq * 4;
  L.bars = L.meta + (size_t)kBgMaxSeq * sizeof(BgMeta);
  L.total = L.bars + (size_t)(2 * kBgStages + 2 * kBgParts) * 8;
  return L;
}

// Largest slab (whole super-blocks, a multiple of 8 unless it covers K) whose
// x rows fit the shared memory next to the ring.
__host__ inline int bg_slab_sb(int nb, int B) {
  if (bg_layout(nb, B).total <= kBgSmemMax) return nb;
  int s = 8;
  while (s + 8 < nb && bg_layout(s + 8, B).total <= kBgSmemMax) s += 8;
  return s;
}

// One item for NB column blocks: the weight fragment of each quant word is
// formed once and multiplied into every block's accumulators.
// xlo / xhi: this lane's swizzled x offsets of the item's low and high runs;
// tb = t & 1 swaps the two 16-element halves (pp) of odd lane groups.
template <int NB>
__device__ __forceinline__ void bq4_item(const uint8_t* hdr, const uint8_t* qnt,
                                         const __half* const (&xrow)[NB], int xlo, int xhi, int tb,
                                         float (&acc)[NB][2][4], const ItemConst& ic) {
  using G = ItemGeom<WL_TILED>;
  const uint4 hA = *reinterpret_cast<const uint4*>(hdr);
  const uint4 hB = *reinterpret_cast<const uint4*>(hdr + 8 * G::kHead);
  const RowScales sA = row_scales(hA, ic);
  const RowScales sB = row_scales(hB, ic);
#pragma unroll
  for (int pp = 0; pp < 2; ++pp) {
    const uint4 qa = *reinterpret_cast<const uint4*>(qnt + 16 * pp);
    const uint4 qb = *reinterpret_cast<const uint4*>(qnt + 16 * pp + 8 * G::kQuantRow);
#pragma unroll
    for (int ih = 0; ih < 2; ++ih) {
      uint4 xl[NB], xh[NB];
#pragma unroll
      for (int c = 0; c < NB; ++c) {
        xl[c] = *reinterpret_cast<const uint4*>(xrow[c] + xlo + 16 * (pp ^ tb) + 8 * ih);
        xh[c] = *reinterpret_cast<const uint4*>(xrow[c] + xhi + 16 * (pp ^ tb) + 8 * ih);
      }
#pragma unroll
      for (int i2 = 0; i2 < 2; ++i2) {
        const int i = 2 * ih + i2;
        uint32_t aL0, aL2, aH0, aH2, bL0, bL2, bH0, bH2;
        dequant_word(word_of(qa, i), sA, ic, aL0, aL2, aH0, aH2);
        dequant_word(word_of(qb, i), sB, ic, bL0, bL2, bH0, bH2);
#pragma unroll
        for (int c = 0; c < NB; ++c) {
          const uint32_t l0 = i2 ? xl[c].z : xl[c].x, l1 = i2 ? xl[c].w : xl[c].y;
          const uint32_t h0 = i2 ? xh[c].z : xh[c].x, h1 = i2 ? xh[c].w : xh[c].y;
          // low- and high-nibble products in separate chains (half the
          // dependent MMAs per accumulator)
          float* cl = acc[c][0];
          float* ch = acc[c][1];
          mma_16816(cl[0], cl[1], cl[2], cl[3], aL0, bL0, aL2, bL2, l0, l1);
          mma_16816(ch[0], ch[1], ch[2], ch[3], aH0, bH0, aH2, bH2, h0, h1);
        }
      }
    }
  }
}

// The finished tile (sums y[16][16] in shared memory, scaled back) to the
// epilogue, one warp. Lane -> task (row pair p = task % 8, sequence task / 8),
// up to 4 tasks per lane; every global load of the tile is issued before any
// value is used (one round trip per tile, not one per task).
template <int EPI>
__device__ __forceinline__ void bg_tile_epilogue(const BgemvArgs& a, const BgMeta* meta, int tile,
                                                 const float* y, int lane) {
  constexpr int kRounds = 8 * kBgMaxSeq / 32;
  const int rounds = (8 * a.B + 31) / 32;
  float y0[kRounds], y1[kRounds], o0[kRounds], o1[kRounds];
  float2 cs[kRounds];
#pragma unroll
  for (int k = 0; k < kRounds; ++k) {
    const int task = 32 * k + lane, p = task & 7, sq = task >> 3;
    const int r0 = tile * kTileRows + 2 * p;
    const bool live = k < rounds && sq < a.B && r0 + 1 < a.n_rows;
    y0[k] = live ? y[(2 * p) * kBgMaxSeq + sq] : 0.f;
    y1[k] = live ? y[(2 * p + 1) * kBgMaxSeq + sq] : 0.f;
    o0[k] = o1[k] = 0.f;
    cs[k] = make_float2(0.f, 0.f);
    if (EPI == BG_RESID && live) {
      const float* o = a.out + (size_t)sq * a.ld_out + r0;
      o0[k] = o[0];
      o1[k] = o[1];
    }
    if (EPI == BG_QKV && live && r0 < a.nq + a.nk)
      cs[k] = a.rope[(size_t)meta[sq].pos * (a.head_dim >> 1) + ((r0 % a.head_dim) >> 1)];
  }
#pragma unroll
  for (int k = 0; k < kRounds; ++k) {
    if (k >= rounds) break;  // warp-uniform
    const int task = 32 * k + lane, p = task & 7, sq = task >> 3;
    const int r0 = tile * kTileRows + 2 * p;
    const bool live = sq < a.B && r0 + 1 < a.n_rows;
    if (live) {
      if (EPI == BG_STORE || EPI == BG_LOGITS) {
        float* o = a.out + (size_t)sq * a.ld_out + r0;
        o[0] = y0[k];
        o[1] = y1[k];
      } else if (EPI == BG_RESID) {
        // residual_add (src/decoder_ops.rs:420-427)
        float* o = a.out + (size_t)sq * a.ld_out + r0;
        o[0] = o0[k] + y0[k];
        o[1] = o1[k] + y1[k];
      } else if (EPI == BG_SWIGLU) {
        // rows interleaved gate/up (src/decoder_ops.rs:196-198, 351-362)
        const float sg = __fdiv_rn(y0[k], __fadd_rn(1.0f, expf(-y0[k])));
        a.out[(size_t)sq * a.ld_out + (r0 >> 1)] = __fmul_rn(sg, y1[k]);
      } else if (EPI == BG_QKV) {
        const BgMeta& m = meta[sq];
        if (r0 < a.nq + a.nk) {
          // rope_norm pair (src/decoder_ops.rs:166-188), host cos/sin
          const float r_0 = __fsub_rn(__fmul_rn(y0[k], cs[k].x), __fmul_rn(y1[k], cs[k].y));
          const float r_1 = __fadd_rn(__fmul_rn(y0[k], cs[k].y), __fmul_rn(y1[k], cs[k].x));
          if (r0 < a.nq) {
            a.q_out[(size_t)sq * a.nq + r0] = r_0;
            a.q_out[(size_t)sq * a.nq + r0 + 1] = r_1;
          } else {
            // K stored f16-rounded (kv_f16_round, src/cpu_oracle.rs:878-883)
            *reinterpret_cast<__half2*>(m.k + (size_t)m.pos * a.nk + (r0 - a.nq)) = __floats2half2_rn(r_0, r_1);
          }
        } else {
          *reinterpret_cast<__half2*>(m.v + (size_t)m.pos * a.nk + (r0 - a.nq - a.nk)) =
              __floats2half2_rn(y0[k], y1[k]);
        }
      }
    }
    if (EPI == BG_LOGITS) {
      // top1_non_eog (src/cpu_oracle.rs:979-995) over this tile's rows of
      // sequence sq: strict '>' from -inf (NaN and -inf never win), lowest id
      // wins ties; one atomic per (tile, sequence)
      unsigned long long best = 0ull;
      bool finite = true;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = r0 + h;
        const float v = h ? y1[k] : y0[k];
        if (!live) continue;
        if (!isfinite(v)) finite = false;
        bool eog = false;
        for (int e = 0; e < a.n_eog; ++e) eog |= (a.eog[e] == (int64_t)r);
        if (!eog && v > -INFINITY) {
          const unsigned long long key = ((unsigned long long)ordered_bits(v) << 32) | (0xffffffffu - (uint32_t)r);
          best = key > best ? key : best;
        }
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
      }
      // a non-finite value anywhere in the 8 lanes of this sequence
      const unsigned fmask = __ballot_sync(0xffffffffu, !finite);
      const bool group_bad = ((fmask >> (lane & ~7)) & 0xffu) != 0u;
      if (p == 0 && sq < a.B) {
        StepState* st = meta[sq].st;
        if (best) atomicMax(&st->argmax_key, best);
        if (group_bad) atomicAnd(&st->finite, 0);
      }
    }
  }
}

template <int EPI, int NB>
__global__ void __launch_bounds__(kPipeThreads, 1) bgemv_kernel(const BgemvArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const BgLayout L = bg_layout(a.slab_sb, a.B);
  uint8_t* ring = smem + L.ring;
  __half* xsl = reinterpret_cast<__half*>(smem + L.xs);
  float* pbase = reinterpret_cast<float*>(smem + L.part);
  BgMeta* meta = reinterpret_cast<BgMeta*>(smem + L.meta);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + kBgStages;
  uint64_t* pfull = empty + kBgStages;
  uint64_t* pfree = pfull + kBgParts;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // CTA group of this slab and this CTA's index inside it
  const int G = gridDim.x;
  const int slab = (int)(((long long)blockIdx.x * a.n_slabs) / G);
  const int g_lo = (int)(((long long)slab * G + a.n_slabs - 1) / a.n_slabs);
  const int g_hi = (int)(((long long)(slab + 1) * G + a.n_slabs - 1) / a.n_slabs);
  const int gi = blockIdx.x - g_lo, gs = g_hi - g_lo;
  const int sb0 = slab * a.slab_sb;
  const int S = min(a.slab_sb, a.nb - sb0);  // super-blocks of this slab
  const int R = (S + kConsumerWarps - 1) / kConsumerWarps;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kBgStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    for (int p = 0; p < kBgParts; ++p) {
      mbar_init(&pfull[p], kConsumerWarps);
      mbar_init(&pfree[p], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == kProducerWarp) {
    if (lane == 0) {
      uint64_t policy;
      asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
      int q = 0, s = 0;
      uint32_t ph = 0;
      for (int tile = gi; tile < a.n_tiles; tile += gs) {
        for (int r = 0; r < R; ++r, ++q) {
          if (q >= kBgStages) mbar_wait(&empty[s], ph);
          const int b0 = r * kConsumerWarps;
          const int cnt = min(kConsumerWarps, S - b0);
          mbar_arrive_expect_tx(&full[s], (uint32_t)(cnt * kTileItemBytes));
          bulk_g2s(ring + (size_t)s * kStageBytes, a.w + ((size_t)tile * a.nb + sb0 + b0) * kTileItemBytes,
                   (uint32_t)(cnt * kTileItemBytes), &full[s], policy);
          if (++s == kBgStages) {
            s = 0;
            if (q >= kBgStages) ph ^= 1u;
          }
        }
      }
    }
    return;
  }

  if (warp == kEpilogueWarp) {
    // per-sequence scale, slot pointers and position, read once per launch
    if (lane < a.B) {
      BgMeta m = {};
      m.xscale = a.xscale[lane];
      if (a.slots) {
        const SlotRef sl = a.slots[lane];
        m.st = sl.st;
        m.k = sl.k;
        m.v = sl.v;
        m.pos = sl.st->cur_pos;
      }
      meta[lane] = m;
    }
    __syncwarp();
    // tile by tile in order: the 8 partial tiles summed in warp order
    // (deterministic), scaled back per sequence, then the epilogue or, with
    // several slabs, the slab partial for bg_combine_kernel
    int it = 0;
    for (int tile = gi; tile < a.n_tiles; tile += gs, ++it) {
      const int pi = it % kBgParts;
      mbar_wait(&pfull[pi], (uint32_t)((it / kBgParts) & 1));
      float* pb = pbase + (size_t)pi * kConsumerWarps * kTileRows * kBgMaxSeq;
      // lane: (row, 4 sequences) quads, 16-byte loads of the 8 warps' values
      const int quads = kTileRows * ((a.B + 3) / 4);
      for (int qd = lane; qd < quads; qd += 32) {
        const int row = qd / ((a.B + 3) / 4), s0 = 4 * (qd - row * ((a.B + 3) / 4));
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float4 u = *reinterpret_cast<const float4*>(pb + ((size_t)w * kTileRows + row) * kBgMaxSeq + s0);
          v.x += u.x;
          v.y += u.y;
          v.z += u.z;
          v.w += u.w;
        }
        v.x *= meta[s0].xscale;
        v.y *= meta[min(s0 + 1, a.B - 1)].xscale;
        v.z *= meta[min(s0 + 2, a.B - 1)].xscale;
        v.w *= meta[min(s0 + 3, a.B - 1)].xscale;
        *reinterpret_cast<float4*>(pb + row * kBgMaxSeq + s0) = v;
      }
      __syncwarp();
      if (a.n_slabs > 1) {
        // plain stores: bg_combine_kernel sums the slabs in slab order
        const int E = kTileRows * a.B, e0 = 8 * lane;
        float mine[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int e = e0 + j, row = e / a.B, sq = e - row * a.B;
          mine[j] = e < E ? pb[row * kBgMaxSeq + sq] : 0.f;
        }
        if (e0 < E) {
          float4* d = reinterpret_cast<float4*>(a.part + ((size_t)slab * a.n_tiles + tile) * E + e0);
          __stcg(d, make_float4(mine[0], mine[1], mine[2], mine[3]));
          __stcg(d + 1, make_float4(mine[4], mine[5], mine[6], mine[7]));
        }
      } else {
        bg_tile_epilogue<EPI>(a, meta, tile, pb, lane);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfree[pi]);
    }
    return;
  }

  // stage this slab's x rows (2B rows, natural order in global) into shared
  // memory in the formation order: each group of four as (0, 2, 1, 3);
  // kXB loads per thread in flight before any is used
  {
    constexpr int kXB = 8;
    constexpr int NT = kConsumerWarps * 32;
    const int n = S * 256, n8 = n / 8, total = 2 * a.B * n8;
    for (int base = 0; base < total; base += NT * kXB) {
      uint4 v[kXB];
#pragma unroll
      for (int k = 0; k < kXB; ++k) {
        const int idx = base + k * NT + threadIdx.x;
        if (idx < total) {
          const int c = idx / n8, j = (idx - c * n8) * 8;
          v[k] = __ldcg(reinterpret_cast<const uint4*>(a.xs + (size_t)c * a.K + (size_t)sb0 * 256 + j));
        }
      }
#pragma unroll
      for (int k = 0; k < kXB; ++k) {
        const int idx = base + k * NT + threadIdx.x;
        if (idx < total) {
          const int c = idx / n8, j = (idx - c * n8) * 8;
          uint4 pv;
          pv.x = __byte_perm(v[k].x, v[k].y, 0x5410);  // e0, e2
          pv.y = __byte_perm(v[k].x, v[k].y, 0x7632);  // e1, e3
          pv.z = __byte_perm(v[k].z, v[k].w, 0x5410);
          pv.w = __byte_perm(v[k].z, v[k].w, 0x7632);
          *reinterpret_cast<uint4*>(xsl + (size_t)c * L.row_halves + bg_swz(j)) = pv;
        }
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
  }
  const int g = lane >> 2, t = lane & 3;
  const ItemConst ic = item_const(t);
  const __half* xrow[NB];
#pragma unroll
  for (int c = 0; c < NB; ++c) {
    const int row = 8 * c + g;  // B operand column = x row (2s: hi, 2s+1: lo)
    xrow[c] = xsl + (size_t)(row < 2 * a.B ? row : 0) * L.row_halves;
  }
  using Gm = ItemGeom<WL_TILED>;
  const int off_h = warp * kTileItemBytes + Gm::kHead * g;
  const int off_q = warp * kTileItemBytes + Gm::kQuant0 + Gm::kQuantRow * g + 32 * t;
  constexpr int kRoundHalves = kConsumerWarps * 256;  // 8 super-blocks: the swizzle repeats every 32 chunks
  const int tb = t & 1;
  int s = 0, it = 0;
  uint32_t ph = 0;
  for (int tile = gi; tile < a.n_tiles; tile += gs, ++it) {
    float acc[NB][2][4];
#pragma unroll
    for (int c = 0; c < NB; ++c)
#pragma unroll
      for (int h = 0; h < 2; ++h) acc[c][h][0] = acc[c][h][1] = acc[c][h][2] = acc[c][h][3] = 0.f;
    // element 64t (+32) of this warp's first item, swizzled: chunk 8t (+4)
    // of the super-block, whose bits 1-2 flip by 2t
    int xlo = warp * 256 + 64 * t + 32 * (t >> 1), xhi = warp * 256 + 64 * t + 32 * ((t >> 1) ^ 1);
    for (int r = 0, b = warp; r < R; ++r, b += kConsumerWarps) {
      mbar_wait(&full[s], ph);
      if (b < S) {
        const uint8_t* slot = ring + (size_t)s * kStageBytes;
        bq4_item<NB>(slot + off_h, slot + off_q, xrow, xlo, xhi, tb, acc, ic);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (++s == kBgStages) {
        s = 0;
        ph ^= 1u;
      }
      xlo += kRoundHalves;
      xhi += kRoundHalves;
    }
    // this warp's partial tile (rows g, g+8 of sequence 4c + t per column
    // block) to the epilogue warp
    const int pi = it % kBgParts;
    float* pb = pbase + (size_t)pi * kConsumerWarps * kTileRows * kBgMaxSeq;
    if (it >= kBgParts) mbar_wait(&pfree[pi], (uint32_t)(((it / kBgParts) & 1) ^ 1));
#pragma unroll
    for (int c = 0; c < NB; ++c) {
      const int sq = 4 * c + t;
      if (sq < a.B) {
        float* w0 = pb + ((size_t)warp * kTileRows) * kBgMaxSeq;
        w0[g * kBgMaxSeq + sq] = (acc[c][0][0] + acc[c][0][1]) + (acc[c][1][0] + acc[c][1][1]);
        w0[(g + 8) * kBgMaxSeq + sq] = (acc[c][0][2] + acc[c][0][3]) + (acc[c][1][2] + acc[c][1][3]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&pfull[pi]);
  }
}

// Slab sums of a multi-slab batched GEMV, in slab order (deterministic), then
// the epilogue: one warp per 16-row tile, loads of every slab issued in
// batches of 4 before any is added.
constexpr int kBgCombineWarps = 8;

template <int EPI>
__global__ void __launch_bounds__(kBgCombineWarps * 32) bg_combine_kernel(const BgemvArgs a) {
  __shared__ float ys[kBgCombineWarps][kTileRows * kBgMaxSeq];
  __shared__ BgMeta meta[kBgMaxSeq];
  if (threadIdx.x < a.B) {
    BgMeta m = {};
    if (a.slots) {
      const SlotRef sl = a.slots[threadIdx.x];
      m.st = sl.st;
      m.k = sl.k;
      m.v = sl.v;
      m.pos = sl.st->cur_pos;
    }
    meta[threadIdx.x] = m;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x * kBgCombineWarps + warp;
  if (tile >= a.n_tiles) return;
  const int E = kTileRows * a.B, e0 = 8 * lane;
  float sum[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) sum[j] = 0.f;
  for (int z0 = 0; z0 < a.n_slabs; z0 += 4) {
    float4 f[4][2];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      f[u][0] = f[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (z0 + u < a.n_slabs && e0 < E) {
        const float4* src = reinterpret_cast<const float4*>(a.part + ((size_t)(z0 + u) * a.n_tiles + tile) * E + e0);
        f[u][0] = __ldcg(src);
        f[u][1] = __ldcg(src + 1);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (z0 + u >= a.n_slabs) break;
      sum[0] += f[u][0].x;
      sum[1] += f[u][0].y;
      sum[2] += f[u][0].z;
      sum[3] += f[u][0].w;
      sum[4] += f[u][1].x;
      sum[5] += f[u][1].y;
      sum[6] += f[u][1].z;
      sum[7] += f[u][1].w;
    }
  }
  float* y = ys[warp];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int e = e0 + j, row = e / a.B, sq = e - row * a.B;
    if (e < E) y[row * kBgMaxSeq + sq] = sum[j];
  }
  __syncwarp();
  bg_tile_epilogue<EPI>(a, meta, tile, y, lane);
}

}  // namespace faber
