// attention_stream.cuh — decode attention for one or two query heads per kv
// head (the Llama-2-7B step), K/V tiles streamed into shared memory by TMA
// (attention_gqa, src/cpu_oracle.rs:711-792, for one query row).
//
// The register-streamed kernel (attention.cuh) keeps one or two 8-row groups
// per warp in flight, too few bytes per SM to reach HBM rate on a launch of a
// few microseconds. Here a producer warp moves whole 32-position tiles of K
// and V (32 x head_dim f16 each, one 2D tensor copy apiece) into a 4-stage
// shared ring, so every CTA has up to 64 KB requested at once, and three CTAs
// share an SM:
//   * grid (kv heads, splits), splits chosen so the grid is about one wave of
//     three CTAs per SM; CTA (kh, split) covers an equal share of the
//     context's 32-position groups, in order;
//   * tiles whose rows all precede the step's own position were written by
//     earlier steps: the producer requests them before the programmatic-
//     dependency wait, so they stream during the tail of the QKV kernel; the
//     tile holding row cur is requested after the wait;
//   * each consumer warp copies its 8 rows of a stage into registers,
//     releases the slot and scores them exactly as the register-streamed
//     kernel does (per-lane partial dots, butterfly reduction, online softmax
//     per warp), then the warps and splits merge in the same fixed order
//     (attn_finish), so results do not depend on CTA timing.
#pragma once

#include <cudaTypedefs.h>

#include <mutex>
#include <string>

#include "attention.cuh"
#include "gemv.cuh"

namespace faber {

constexpr int kAsRows = 32;                          // positions per stage (8 per consumer warp)
constexpr int kAsStages = 4;
constexpr int kAsConsumers = kAttnWarps;             // 4 consumer warps
constexpr int kAsThreads = (kAsConsumers + 1) * 32;  // + the producer warp
constexpr int kAsCtasPerSm = 3;
static_assert(kAsRows == kAttnRows * kAsConsumers, "one 8-row slice per consumer warp");

template <int HD>
struct AsLayout {
  static constexpr int kTile = kAsRows * HD * 2;  // bytes of one K (or V) tile
  static constexpr int kStage = 2 * kTile;
  static constexpr int kBarOff = kAsStages * kStage;
  static constexpr int kBytes = kBarOff + 2 * kAsStages * 8;
};

__device__ __forceinline__ void tma_load_tile(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void consumer_bar_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kAsConsumers * 32) : "memory");
}

template <int HD, int R>
__global__ void __launch_bounds__(kAsThreads) attention_stream_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                      const __grid_constant__ CUtensorMap vmap,
                                                                      const AttnArgs a) {
  using Lay = AsLayout<HD>;
  constexpr int DPL = HD / 32;
  static_assert(DPL == 2 || DPL == 4, "head_dim 64 or 128");
  extern __shared__ __align__(1024) uint8_t as_smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(as_smem + Lay::kBarOff);
  uint64_t* empty = full + kAsStages;
  __shared__ float pbuf[kAsConsumers][R][kAttnRows];
  __shared__ float wstat[kAsConsumers][R][2];
  __shared__ float red[kAsConsumers][R][HD];
  __shared__ int is_last;

  const int kh = blockIdx.x, split = blockIdx.y;
  // cur_pos was written by this step's embed kernel, which completed before
  // the QKV kernel (whose consumers wait on it) let this grid launch.
  const int cur = a.st->cur_pos;
  const int n_kv = cur + 1;
  const int n_grp = (n_kv + kAsRows - 1) / kAsRows;
  const int per = (n_grp + gridDim.y - 1) / gridDim.y;  // groups per split
  const int active = (n_grp + per - 1) / per;           // splits with work
  const int g0 = split * per, g1 = min(n_grp, g0 + per);
  if (g0 >= g1) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kAsStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kAsConsumers);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == kAsConsumers) {
    // producer: one K and one V tile per stage
    if (lane == 0) {
      uint64_t policy;
      asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
      bool waited = false;
      for (int g = g0, q = 0; g < g1; ++g, ++q) {
        const int s = q % kAsStages;
        if (q >= kAsStages) mbar_wait(&empty[s], (uint32_t)(((q / kAsStages) - 1) & 1));
        if (!waited && (g + 1) * kAsRows > cur) {
          // row cur is the QKV kernel's: request its tile after that kernel
          pdl_wait();
          asm volatile("fence.proxy.async.global;" ::: "memory");
          waited = true;
        }
        uint8_t* dst = as_smem + s * Lay::kStage;
        mbar_arrive_expect_tx(&full[s], (uint32_t)Lay::kStage);
        tma_load_tile(dst, &kmap, kh * HD, g * kAsRows, &full[s], policy);
        tma_load_tile(dst + Lay::kTile, &vmap, kh * HD, g * kAsRows, &full[s], policy);
      }
    }
    return;
  }

  // consumers
  pdl_wait();
  pdl_launch_dependents();
  const int ratio = a.n_heads / a.n_kv_heads;  // <= R
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
  const int slice = warp * kAttnRows * HD * 2 + lane * DPL * 2;  // this lane's bytes of row 0 of the slice
  for (int g = g0, q = 0; g < g1; ++g, ++q) {
    const int s = q % kAsStages;
    mbar_wait(&full[s], (uint32_t)((q / kAsStages) & 1));
    const uint8_t* kt = as_smem + s * Lay::kStage + slice;
    KvGroup<DPL> kv;
#pragma unroll
    for (int i = 0; i < kAttnRows; ++i) {
      kv.k[i].load_smem(kt + i * HD * 2);
      kv.v[i].load_smem(kt + Lay::kTile + i * HD * 2);
    }
    // the rows are in registers: release the slot
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    const int j0 = g * kAsRows + warp * kAttnRows;
    // rows past the step's own position hold old or zero bytes: never used
#pragma unroll
    for (int i = 0; i < kAttnRows; ++i)
      if (j0 + i >= n_kv) {
        kv.k[i].zero();
        kv.v[i].zero();
      }
    kv_consume<DPL, R>(kv, j0, n_kv, ratio, a.scale, qv, m, l, acc, pw, lane);
  }
  attn_finish<HD, R>(a, kh, split, active, ratio, warp, lane, m, l, acc, wstat, red, &is_last,
                     [] { consumer_bar_sync(); });
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
// 32-position x hd boxes; rows past the cache read as zero.
inline CUtensorMap kv_tensor_map(const __half* cache, uint64_t rows, uint64_t span, int hd) {
  CUtensorMap map;
  const cuuint64_t dims[2] = {span, rows};
  const cuuint64_t strides[1] = {span * 2};
  const cuuint32_t box[2] = {(cuuint32_t)hd, (cuuint32_t)kAsRows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = tmap_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(cache), dims,
                                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  require(r == CUDA_SUCCESS, FABER_STATUS_CUDA_ERROR,
          "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return map;
}

// Splits of the streamed kernel: about kAsCtasPerSm CTAs per SM over the kv
// heads, within the partial buffer's capacity.
inline int attention_stream_splits(int sms, int kv_heads, int cap) {
  return std::max(1, std::min(cap, (kAsCtasPerSm * sms + kv_heads - 1) / kv_heads));
}

template <int HD, int R>
void launch_attention_stream(const AttnArgs& a, int kv_heads, int splits, cudaStream_t stream, bool pdl) {
  using Lay = AsLayout<HD>;
  auto kern = attention_stream_kernel<HD, R>;
  static thread_local std::map<int, bool> attr_done;
  int dev = 0;
  FABER_CUDA(cudaGetDevice(&dev));
  if (!attr_done[dev]) {
    FABER_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kBytes));
    attr_done[dev] = true;
  }
  const uint64_t span = (uint64_t)kv_heads * HD;
  const CUtensorMap km = kv_tensor_map(a.k, (uint64_t)a.cache_rows, span, HD);
  const CUtensorMap vm = kv_tensor_map(a.v, (uint64_t)a.cache_rows, span, HD);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kv_heads, splits);
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
