// common.cuh — shared device helpers and host error plumbing.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

#include "faber_gpu.h"

namespace faber {

// A failure carried to the C ABI boundary as a status code plus message.
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

inline void require(bool cond, int code, const std::string& msg) {
  if (!cond) throw Error(code, msg);
}

#define FABER_CUDA(expr)                                                                  \
  do {                                                                                    \
    cudaError_t e_ = (expr);                                                              \
    if (e_ != cudaSuccess)                                                                \
      throw ::faber::Error(FABER_STATUS_CUDA_ERROR,                                       \
                           std::string(#expr) + " failed: " + cudaGetErrorString(e_));    \
  } while (0)

// Q4_K super-block: f16 d @0, f16 dmin @2, scales[12] @4, qs[128] @16.
constexpr int kQ4kBlockBytes = 144;
constexpr int kQ4kBlockElems = 256;
// Tile layout: 16 rows x one super-block column = 16 headers (256 B) then
// 16 rows of qs (16 x 128 B), 2304 B, 256-byte aligned.
constexpr int kTileRows = 16;
constexpr int kTileItemBytes = kTileRows * kQ4kBlockBytes;  // 2304

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------

// Streaming 16-byte read-only load that does not allocate in L1 (weights are
// read exactly once per launch).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }
__device__ __forceinline__ uint32_t f2u(float f) { return __float_as_uint(f); }

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);  // .x (low 16 bits) = lo
  return *reinterpret_cast<uint32_t*>(&h);
}

// f32 -> f16 (RN-even) -> f32: the reference's kv_f16_round.
__device__ __forceinline__ float f16_round(float x) { return __half2float(__float2half_rn(x)); }

// D(16x8,f32) += A(16x16,f16,row) * B(16x8,f16,col) — warp-wide.
__device__ __forceinline__ void mma_16816(float& c0, float& c1, float& c2, float& c3, uint32_t a0,
                                          uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c0), "+f"(c1), "+f"(c2), "+f"(c3)
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Monotonic unsigned image of an f32 (total order for non-NaN values).
__device__ __forceinline__ uint32_t ordered_bits(float v) {
  uint32_t u = f2u(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Programmatic dependent launch: wait for the previous kernel in the stream
// (no-op when launched without the attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace faber
