// synth.cpp — seeded synthetic inputs for the Q4_K decoder workloads.
//
// Counter-based: every output element is a pure function of
// (seed, stream, index), so the bytes are identical for any thread count and
// any chunking. splitmix64's finalizer mixes the counter.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "faber_gpu.h"

namespace {

inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

inline uint64_t stream_key(uint64_t seed, uint64_t stream) {
  return mix64(seed * 0x9e3779b97f4a7c15ull + mix64(stream + 0x632be59bd9b4e019ull));
}

inline uint64_t draw(uint64_t key, uint64_t ctr) { return mix64(key + ctr * 0x9e3779b97f4a7c15ull); }

inline double u01(uint64_t r) { return (double)(r >> 11) * (1.0 / 9007199254740992.0); }

// IEEE binary32 -> binary16, round to nearest even (finite inputs).
uint16_t to_half(float x) {
  uint32_t b;
  std::memcpy(&b, &x, 4);
  const uint32_t sign = (b >> 16) & 0x8000u;
  const uint32_t a = b & 0x7fffffffu;
  if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
  if (a >= 0x38800000u) {
    const uint32_t e = (a >> 23) - 112u;
    const uint32_t mant = a & 0x7fffffu;
    uint32_t h = (e << 10) | (mant >> 13);
    const uint32_t rest = mant & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
  }
  // subnormal: value = a * 2^24 rounded to an integer (ties to even)
  float f;
  std::memcpy(&f, &a, 4);
  const double scaled = (double)f * 16777216.0;
  double fl = std::floor(scaled);
  const double fr = scaled - fl;
  if (fr > 0.5 || (fr == 0.5 && std::fmod(fl, 2.0) != 0.0)) fl += 1.0;
  return (uint16_t)(sign | (uint32_t)fl);
}

template <class F>
void parallel_for(uint64_t n, uint64_t grain, F&& fn) {
  unsigned nt = std::thread::hardware_concurrency();
  if (nt == 0) nt = 1;
  if (n < grain * 2 || nt == 1) {
    fn(0, n);
    return;
  }
  nt = (unsigned)std::min<uint64_t>(nt, (n + grain - 1) / grain);
  std::vector<std::thread> th;
  const uint64_t per = (n + nt - 1) / nt;
  for (unsigned k = 0; k < nt; ++k) {
    const uint64_t a = k * per, b = std::min(n, a + per);
    if (a < b) th.emplace_back([&fn, a, b] { fn(a, b); });
  }
  for (auto& t : th) t.join();
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) FaberRtStatusV1 faber_synth_q4k(uint64_t seed, uint64_t stream, uint64_t n_blocks, uint8_t* out) {
  if (n_blocks > 0 && out == nullptr) return FaberRtStatusV1{FABER_STATUS_INVALID_ARGUMENT};
  const uint64_t key = stream_key(seed, stream);
  parallel_for(n_blocks, 1u << 14, [&](uint64_t b0, uint64_t b1) {
    for (uint64_t b = b0; b < b1; ++b) {
      uint8_t* blk = out + b * 144;
      const uint64_t c = b * 20;
      const float d = (float)(1e-3 + u01(draw(key, c + 0)) * (2e-2 - 1e-3));
      const float dmin = (float)(1e-3 + u01(draw(key, c + 1)) * (2e-2 - 1e-3));
      const uint16_t hd = to_half(d), hm = to_half(dmin);
      blk[0] = (uint8_t)(hd & 0xff);
      blk[1] = (uint8_t)(hd >> 8);
      blk[2] = (uint8_t)(hm & 0xff);
      blk[3] = (uint8_t)(hm >> 8);
      // 140 uniform bytes: scales[12] then qs[128]
      for (int w = 0; w < 18; ++w) {
        uint64_t r = draw(key, c + 2 + (uint64_t)w);
        for (int k = 0; k < 8; ++k) {
          const int pos = 4 + w * 8 + k;
          if (pos < 144) blk[pos] = (uint8_t)(r >> (8 * k));
        }
      }
    }
  });
  return FaberRtStatusV1{FABER_STATUS_OK};
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_synth_normal_f32(uint64_t seed, uint64_t stream, uint64_t n, float mean,
                                       float std_, float* out) {
  if (n > 0 && out == nullptr) return FaberRtStatusV1{FABER_STATUS_INVALID_ARGUMENT};
  const uint64_t key = stream_key(seed, stream);
  parallel_for(n, 1u << 16, [&](uint64_t i0, uint64_t i1) {
    for (uint64_t i = i0; i < i1; ++i) {
      const double a = (double)((draw(key, 2 * i) >> 11) + 1) * (1.0 / 9007199254740992.0);
      const double b = u01(draw(key, 2 * i + 1));
      const double z = std::sqrt(-2.0 * std::log(a)) * std::cos(6.283185307179586 * b);
      out[i] = (float)((double)mean + (double)std_ * z);
    }
  });
  return FaberRtStatusV1{FABER_STATUS_OK};
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_synth_tokens(uint64_t seed, uint64_t stream, uint64_t n, uint32_t vocab,
                                   int64_t* out) {
  if ((n > 0 && out == nullptr) || vocab == 0) return FaberRtStatusV1{FABER_STATUS_INVALID_ARGUMENT};
  const uint64_t key = stream_key(seed, stream);
  for (uint64_t i = 0; i < n; ++i)
    out[i] = (int64_t)(((draw(key, i) >> 32) * (uint64_t)vocab) >> 32);
  return FaberRtStatusV1{FABER_STATUS_OK};
}

}  // extern "C"
