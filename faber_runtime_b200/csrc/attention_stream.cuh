// attention_stream.cuh — decode attention with K/V tiles streamed into shared
// memory by TMA, scores and context on the tensor cores (attention_gqa,
// src/cpu_oracle.rs:711-792, for one query row). Exact for up to eight query
// heads per kv head; the decode step routes one or two here (the Llama-2-7B
// shape has one), see kAsStreamMaxRatio.
//
//   * grid (kv heads, splits, sequences), three CTAs per SM, the split count
//     chosen from the launch's shape (attention_stream_splits); CTA (kh,
//     split) covers an equal share of the context's 16-key groups, in order.
//     A single sequence's tensor maps are kernel parameters, a batch's are
//     read from a device array (one K and one V map per sequence);
//   * a producer warp moves each group's K and V (16 keys x head_dim f16,
//     64-dim halves with the 128-byte swizzle) into an 8-stage ring with 2D
//     tensor copies, up to 64 KB per CTA in flight. Groups whose keys all
//     precede the step's own position were written by earlier steps: they
//     are requested before the programmatic-dependency wait, so they stream
//     during the tail of the QKV kernel; the group holding row cur after it;
//   * consumer warp w takes groups w, w + 4, ... Each query head is split
//     exactly into f16 hi and lo rows (per-head power-of-two scale) of the
//     MMA A operand, 16 rows for up to 8 heads, so the grouping costs no
//     extra MMAs: S = Q K^T on m16n8k16 (8 k-steps per 16 keys at head_dim
//     128), score = (S_hi + S_lo) * scale; an online softmax per warp; the
//     probabilities, split into hi/lo rows the same way, multiply V (the
//     score accumulator's layout is the A fragment's), so both products keep
//     about f32 accuracy;
//   * the warps and then the splits merge in a fixed order (attn_merge), so
//     results do not depend on CTA timing.
#pragma once

#include <cudaTypedefs.h>

#include <mutex>
#include <string>

#include "attention.cuh"
#include "gemv.cuh"
#include "prefill.cuh"

namespace faber {

constexpr int kAsKeys = 16;                          // keys per stage: one k-step of P V
constexpr int kAsStages = 8;
constexpr int kAsConsumers = kAttnWarps;             // 4 consumer warps
constexpr int kAsThreads = (kAsConsumers + 1) * 32;  // + the producer warp
constexpr int kAsCtasPerSm = 3;
constexpr int kAsMaxRatio = 8;  // 16 MMA rows: each query head's hi and lo
// Groupings the decode step routes here. Up to 8 heads are exact here too,
// but at 8 (the 70B shape) the last CTA's merge of ratio x head_dim outputs
// over up to 55 splits costs more than this kernel saves.
constexpr int kAsStreamMaxRatio = 2;

template <int HD>
struct AsLayout {
  static constexpr int kHalves = HD / 64;            // 64-dim halves: 128-byte rows
  static constexpr int kHalf = kAsKeys * 128;        // one half of a 16-row tile
  static constexpr int kTile = kHalves * kHalf;      // one K (or V, or Q) tile
  static constexpr int kStage = 2 * kTile;
  static constexpr int kQOff = kAsStages * kStage;   // Q hi/lo rows, same layout
  static constexpr int kBarOff = kQOff + kTile;
  static constexpr int kBytes = kBarOff + 2 * kAsStages * 8 + 1024;  // + alignment slack
};

// Byte offset of (row, 16-byte chunk) in a 16-row tile stored as 64-dim
// halves of 128-byte rows with the 128-byte swizzle (chunk ^ row % 8).
__device__ __forceinline__ uint32_t as_off(int row, int chunk) {
  return (uint32_t)((chunk >> 3) * (kAsKeys * 128) + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

__device__ __forceinline__ void tma_load_tile(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void consumer_bar_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kAsConsumers * 32) : "memory");
}

// Online-softmax update of one accumulator row half over a stage's 16 keys.
// s00, s01 / s10, s11: this lane's accumulator values of keys 2 t4, 2 t4 + 1
// / 8 + 2 t4, 9 + 2 t4 in its row; the row's hi and lo partner (4 lanes away)
// adds in, f scales the sum to a score, keys from n_kv on are masked. Returns
// the rescale of the running state; p receives the probabilities.
__device__ __forceinline__ float as_softmax(float s00, float s01, float s10, float s11, float f, int key0,
                                            int t4, int n_kv, float& m, float& l, float (&p)[4]) {
  float x[4] = {s00, s01, s10, s11};
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float v = x[i] + __shfl_xor_sync(0xffffffffu, x[i], 4);
    const int key = key0 + (i >> 1) * 8 + 2 * t4 + (i & 1);
    v = key < n_kv ? v * f : -INFINITY;
    x[i] = v;
    mx = fmaxf(mx, v);
  }
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  const float mn = fmaxf(m, mx);
  const float base = mn == -INFINITY ? 0.0f : mn;
  const float c = expf(m - base);
  m = mn;
  float ps = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    p[i] = expf(x[i] - base);
    ps += p[i];
  }
  l = fmaf(l, c, ps);
  return c;
}

template <int HD>
__global__ void __launch_bounds__(kAsThreads, kAsCtasPerSm)
    attention_stream_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                            const AttnArgs a0) {
  const AttnArgs a = slot_args(a0);
  using Lay = AsLayout<HD>;
  constexpr int R = kAsMaxRatio;
  constexpr int KS = HD / 16;  // k-steps of Q K^T, and 16-dim column pairs of P V
  extern __shared__ uint8_t as_raw[];
  // tensor copies with the 128-byte swizzle land on 1024-byte boundaries
  uint8_t* sm = as_raw + ((1024u - (smem_addr(as_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_addr(sm);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + Lay::kBarOff);
  uint64_t* empty = full + kAsStages;
  __shared__ int qshift[R];
  __shared__ float wstat[kAsConsumers][R][2];
  __shared__ int is_last;

  const int kh = blockIdx.x, split = blockIdx.y;
  // cur_pos was written by this step's embed kernel, which completed before
  // the QKV kernel (whose consumers wait on it) let this grid launch.
  const int cur = a.st->cur_pos;
  const int n_kv = cur + 1;
  const int n_grp = (n_kv + kAsKeys - 1) / kAsKeys;
  const int per = (n_grp + gridDim.y - 1) / gridDim.y;  // groups per split
  const int active = (n_grp + per - 1) / per;           // splits with work
  const int g0 = split * per, g1 = min(n_grp, g0 + per);
  if (g0 >= g1) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kAsStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == kAsConsumers) {
    // producer: each group's K and V halves
    if (lane == 0) {
      const CUtensorMap* km = a0.kvmaps ? a0.kvmaps + 2 * blockIdx.z : &kmap;
      const CUtensorMap* vm = a0.kvmaps ? a0.kvmaps + 2 * blockIdx.z + 1 : &vmap;
      uint64_t policy;
      asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
      bool waited = false;
      for (int g = g0, q = 0; g < g1; ++g, ++q) {
        const int s = q % kAsStages;
        if (q >= kAsStages) mbar_wait(&empty[s], (uint32_t)(((q / kAsStages) - 1) & 1));
        if (!waited && (g + 1) * kAsKeys > cur) {
          // row cur is the QKV kernel's: request its group after that kernel
          pdl_wait();
          asm volatile("fence.proxy.async.global;" ::: "memory");
          waited = true;
        }
        const uint32_t dst = sbase + (uint32_t)(s * Lay::kStage);
        mbar_arrive_expect_tx(&full[s], (uint32_t)Lay::kStage);
#pragma unroll
        for (int h = 0; h < Lay::kHalves; ++h) {
          tma_load_tile(dst + h * Lay::kHalf, km, kh * HD + 64 * h, g * kAsKeys, &full[s], policy);
          tma_load_tile(dst + Lay::kTile + h * Lay::kHalf, vm, kh * HD + 64 * h, g * kAsKeys, &full[s], policy);
        }
      }
    }
    return;
  }

  // consumers
  const int ratio = a.n_heads / a.n_kv_heads;  // <= R
  const int tid = threadIdx.x;
  // Q rows: 2h = hi, 2h + 1 = lo of q_h * 2^-shift_h; rows past 2 * ratio zero
  for (int i = tid; i < Lay::kTile / 16; i += kAsConsumers * 32)
    reinterpret_cast<uint4*>(sm + Lay::kQOff)[i] = make_uint4(0u, 0u, 0u, 0u);
  pdl_wait();
  pdl_launch_dependents();
  consumer_bar_sync();
  for (int hq = warp; hq < ratio; hq += kAsConsumers) {
    constexpr int PL = HD / 32;  // dims per lane
    const float* src = a.q + (size_t)(kh * ratio + hq) * HD + lane * PL;
    float v[PL];
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      v[i] = src[i];
      mx = fmaxf(mx, fabsf(v[i]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const int sh = split_shift(mx);
    const float in_s = ldexpf(1.0f, -sh);
    if (lane == 0) qshift[hq] = sh;
    uint32_t hb[PL / 2], lb[PL / 2];
#pragma unroll
    for (int i = 0; i < PL / 2; ++i) split2(v[2 * i] * in_s, v[2 * i + 1] * in_s, hb[i], lb[i]);
    const int chunk = (lane * PL) / 8, within = ((lane * PL) % 8) * 2;
    uint8_t* qh = sm + Lay::kQOff + as_off(2 * hq, chunk) + within;
    uint8_t* ql = sm + Lay::kQOff + as_off(2 * hq + 1, chunk) + within;
    if constexpr (PL == 4) {
      *reinterpret_cast<uint2*>(qh) = make_uint2(hb[0], hb[1]);
      *reinterpret_cast<uint2*>(ql) = make_uint2(lb[0], lb[1]);
    } else {
      *reinterpret_cast<uint32_t*>(qh) = hb[0];
      *reinterpret_cast<uint32_t*>(ql) = lb[0];
    }
  }
  consumer_bar_sync();
  // Accumulator rows of this lane: g8 (head g8 / 2) and g8 + 8 (head 4 + g8 / 2),
  // hi rows even, lo rows odd; rows past the heads' pairs are zero.
  const int g8 = lane >> 2, t4 = lane & 3;
  const bool hi8 = ratio > 4;  // heads in rows 8-15 (warp-uniform)
  const bool ok_a = g8 < 2 * ratio, ok_b = g8 + 8 < 2 * ratio;
  const float f_a = ok_a ? ldexpf(a.scale, qshift[g8 >> 1]) : 0.0f;
  const float f_b = ok_b ? ldexpf(a.scale, qshift[4 + (g8 >> 1)]) : 0.0f;
  // A fragments of the Q rows for every k-step
  uint32_t qa[KS][4];
#pragma unroll
  for (int kk = 0; kk < KS; ++kk)
    ldsm_x4(sbase + Lay::kQOff + as_off((lane & 7) + ((lane >> 3) & 1) * 8, 2 * kk + (lane >> 4)), qa[kk]);
  float o[2 * KS][4];
#pragma unroll
  for (int i = 0; i < 2 * KS; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m_a = -INFINITY, l_a = 0.0f, m_b = -INFINITY, l_b = 0.0f;
  const int krow = (lane >> 4) * 8 + (lane & 7), kchunk = (lane >> 3) & 1;   // K: non-transposed x4
  const int vrow = ((lane >> 3) & 1) * 8 + (lane & 7), vchunk = lane >> 4;  // V: transposed x4
  for (int g = g0 + warp, q = warp; g < g1; g += kAsConsumers, q += kAsConsumers) {
    const int s = q % kAsStages;
    mbar_wait(&full[s], (uint32_t)((q / kAsStages) & 1));
    const uint32_t kst = sbase + (uint32_t)(s * Lay::kStage), vst = kst + Lay::kTile;
    const int key0 = g * kAsKeys;
    if (key0 + kAsKeys > n_kv) {
      // rows past the step's own position hold old or zero bytes: clear V's
      // (a zero probability times a non-finite value would not vanish)
      const int nv = n_kv - key0;
      for (int i = lane; i < (kAsKeys - nv) * Lay::kHalves * 8; i += 32) {
        const int r = nv + i / (Lay::kHalves * 8), h = (i / 8) % Lay::kHalves, c = i % 8;
        *reinterpret_cast<uint4*>(sm + s * Lay::kStage + Lay::kTile + h * Lay::kHalf + r * 128 + c * 16) =
            make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
    }
    // S = Q K^T: rows (head hi/lo) x 16 keys
    float sc[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i) sc[i][0] = sc[i][1] = sc[i][2] = sc[i][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      uint32_t b[4];
      ldsm_x4(kst + as_off(krow, 2 * kk + kchunk), b);
      mma16816(sc[0], qa[kk], b[0], b[1]);
      mma16816(sc[1], qa[kk], b[2], b[3]);
    }
    float p_a[4], p_b[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const float c_a = as_softmax(sc[0][0], sc[0][1], sc[1][0], sc[1][1], f_a, key0, t4, n_kv, m_a, l_a, p_a);
    float c_b = 1.0f;
    if (hi8) c_b = as_softmax(sc[0][2], sc[0][3], sc[1][2], sc[1][3], f_b, key0, t4, n_kv, m_b, l_b, p_b);
    if (__any_sync(0xffffffffu, (ok_a && c_a != 1.0f) || (ok_b && c_b != 1.0f))) {
#pragma unroll
      for (int i = 0; i < 2 * KS; ++i) {
        o[i][0] *= c_a;
        o[i][1] *= c_a;
        o[i][2] *= c_b;
        o[i][3] *= c_b;
      }
    }
    // P as the A operand: each row holds the hi (even) or lo (odd) part
    uint32_t pa[4];
    {
      uint32_t h01, l01, h23, l23;
      split2(p_a[0], p_a[1], h01, l01);
      split2(p_a[2], p_a[3], h23, l23);
      pa[0] = ok_a ? ((g8 & 1) ? l01 : h01) : 0u;
      pa[2] = ok_a ? ((g8 & 1) ? l23 : h23) : 0u;
      split2(p_b[0], p_b[1], h01, l01);
      split2(p_b[2], p_b[3], h23, l23);
      pa[1] = ok_b ? ((g8 & 1) ? l01 : h01) : 0u;
      pa[3] = ok_b ? ((g8 & 1) ? l23 : h23) : 0u;
    }
    // O += P V over the 16 keys
#pragma unroll
    for (int dp = 0; dp < KS; ++dp) {
      uint32_t b[4];
      ldsm_x4_t(vst + as_off(vrow, 2 * dp + vchunk), b);
      mma16816(o[2 * dp], pa, b[0], b[1]);
      mma16816(o[2 * dp + 1], pa, b[2], b[3]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  // this warp's state: sum over the column lanes, then hi + lo rows
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
#pragma unroll
  for (int i = 0; i < 2 * KS; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[i][e] += __shfl_xor_sync(0xffffffffu, o[i][e], 4);
  // every warp is done with the ring: the warps' contexts go there
  consumer_bar_sync();
  auto& red = *reinterpret_cast<float(*)[kAsConsumers][R][HD]>(sm);
  if ((g8 & 1) == 0) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int h = (g8 >> 1) + 4 * half;
      if (h >= ratio) continue;
      if (t4 == 0) {
        wstat[warp][h][0] = half ? m_b : m_a;
        wstat[warp][h][1] = half ? l_b : l_a;
      }
#pragma unroll
      for (int i = 0; i < 2 * KS; ++i) {
        red[warp][h][8 * i + 2 * t4] = o[i][2 * half];
        red[warp][h][8 * i + 2 * t4 + 1] = o[i][2 * half + 1];
      }
    }
  }
  attn_merge<HD, R>(a, kh, split, active, ratio, wstat, red, &is_last, [] { consumer_bar_sync(); });
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
using TmapEncode = PFN_cuTensorMapEncodeTiled_v12000;

inline TmapEncode tmap_encoder() {
  static TmapEncode fn = nullptr;
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    FABER_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    require(p != nullptr && q == cudaDriverEntryPointSuccess, FABER_STATUS_UNSUPPORTED,
            "cuTensorMapEncodeTiled is not available");
    fn = reinterpret_cast<TmapEncode>(p);
  }
  return fn;
}

// Tensor map over one layer's K (or V) cache [rows][kv_heads * hd] f16, in
// 16-key x 64-dim boxes with the 128-byte swizzle; rows past the cache read
// as zero.
inline CUtensorMap kv_tensor_map(const __half* cache, uint64_t rows, uint64_t span) {
  CUtensorMap map;
  const cuuint64_t dims[2] = {span, rows};
  const cuuint64_t strides[1] = {span * 2};
  const cuuint32_t box[2] = {64u, (cuuint32_t)kAsKeys};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = tmap_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(cache), dims,
                                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  require(r == CUDA_SUCCESS, FABER_STATUS_CUDA_ERROR,
          "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return map;
}

// Splits of the streamed kernel for `pairs` (kv head, sequence) pairs of
// `ratio` query heads over a context of up to `ctx` keys, at most `cap`: the
// count with the shortest modelled time, waves x (a CTA's share of the
// pair's K/V bytes at an equal share of the HBM rate + 3 us of start-up and
// partial write) + the last CTA's merge (one 0.7 us round trip per 16 splits
// for every 128 outputs a thread produces). Measured on the 7B shape: 13
// splits at batch 1 (9: 0.6% slower, 18: 7.6%), 4 at batch 16 (5: 1%, 6: 3.6%).
inline int attention_stream_splits(int sms, int pairs, int ctx, int hd, int ratio, int cap) {
  const double slots = (double)kAsCtasPerSm * sms;
  const double pair_us = (double)ctx * hd * 4 / (6.5e6 / slots);  // one pair at 1/slots of 6.5 TB/s
  const double outputs = std::ceil((double)ratio * hd / (kAsConsumers * 32));
  int best = 1;
  double best_t = 1e30;
  for (int s = 1; s <= std::max(1, cap); ++s) {
    const double waves = std::ceil((double)pairs * s / slots);
    const double t = waves * (pair_us / s + 3.0) + std::ceil(s / 16.0) * outputs * 0.7;
    if (t < best_t * 0.99) {
      best_t = t;
      best = s;
    }
  }
  return best;
}

template <int HD>
void launch_attention_stream(const AttnArgs& a, dim3 grid, cudaStream_t stream, bool pdl) {
  using Lay = AsLayout<HD>;
  auto kern = attention_stream_kernel<HD>;
  static thread_local std::map<int, bool> attr_done;
  int dev = 0;
  FABER_CUDA(cudaGetDevice(&dev));
  if (!attr_done[dev]) {
    FABER_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kBytes));
    // three CTAs of about 75 KB per SM
    FABER_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                    (int)cudaSharedmemCarveoutMaxShared));
    attr_done[dev] = true;
  }
  // a single sequence's maps travel as parameters; a batch's are in a.kvmaps
  CUtensorMap km = {}, vm = {};
  if (!a.kvmaps) {
    const uint64_t span = (uint64_t)grid.x * HD;
    km = kv_tensor_map(a.k, (uint64_t)a.cache_rows, span);
    vm = kv_tensor_map(a.v, (uint64_t)a.cache_rows, span);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kAsThreads);
  cfg.dynamicSmemBytes = Lay::kBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  FABER_CUDA(cudaLaunchKernelEx(&cfg, kern, km, vm, a));
}

}  // namespace faber
