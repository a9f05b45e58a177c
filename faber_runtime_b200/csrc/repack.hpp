// repack.hpp — host-side Q4_K repack into the GEMV tile layout.
//
// The reference keeps GGUF blocks native and only declares a repack
// identity (src/repack_plan.rs, src/quantized_tensor_layout.rs:269-278,
// 483-487). Here the repack is executed, value-preserving:
//   * rows are grouped into 16-row tiles; per tile and 256-element
//     super-block column one 2304-byte item holds the 16 block headers
//     (d, dmin, scales: 16 B each) followed by the 16 rows' quants (128 B
//     each), so a warp reads a tile column with fully coalesced 16-byte
//     loads;
//   * a row whose first element is not 256-aligned in the flat tensor (rows
//     of cols % 256 != 0 straddle super-blocks, e.g. a 1408-wide ffn_down)
//     keeps its source blocks and gets an element offset o (a multiple of
//     32); sub-blocks outside the row get scale and min 0, so their weights
//     dequantize to exactly 0. Rows are grouped by o so one tile shares one
//     offset; a row map restores the output order.
// Every weight in the row dequantizes from the same (d, dmin, sc, m, q) as in
// the source block, so results are bit-identical.
#pragma once

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <functional>
#include <thread>
#include <vector>

#include "common.cuh"

namespace faber {

// One output row: the flat element range [start, start + cols) of a native
// block-packed Q4_K tensor with n_blocks blocks at base.
struct RowSeg {
  const uint8_t* base;
  uint64_t n_blocks;
  uint64_t start;
};

struct TiledQ4k {
  std::vector<uint8_t> data;     // n_tiles * nb * 2304
  std::vector<int32_t> xoff;     // per tile
  std::vector<int32_t> rowmap;   // n_tiles * 16
  int n_tiles = 0, nb = 0, rows = 0, cols = 0;
  bool identity = true;          // all offsets 0 and rows in order
};

inline void unpack_scales(const uint8_t* s, uint8_t sc[8], uint8_t m[8]) {
  for (int j = 0; j < 8; ++j) {
    if (j < 4) {
      sc[j] = s[j] & 63;
      m[j] = s[j + 4] & 63;
    } else {
      sc[j] = (uint8_t)((s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4));
      m[j] = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
  }
}

inline void pack_scales(const uint8_t sc[8], const uint8_t m[8], uint8_t* s) {
  for (int j = 0; j < 4; ++j) {
    s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    s[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
    s[j + 8] = (uint8_t)((sc[j + 4] & 0x0f) | ((m[j + 4] & 0x0f) << 4));
  }
}

inline TiledQ4k repack_q4k(int rows, int cols, const std::function<RowSeg(int)>& seg) {
  require(rows > 0 && cols > 0, FABER_STATUS_INVALID_ARGUMENT, "empty Q4_K tensor");
  require(cols % 32 == 0, FABER_STATUS_UNSUPPORTED,
          "Q4_K rows must be a multiple of 32 elements (one sub-block)");
  TiledQ4k T;
  T.rows = rows;
  T.cols = cols;
  std::vector<RowSeg> segs((size_t)rows);
  std::vector<int> off((size_t)rows);
  int max_o = 0;
  for (int j = 0; j < rows; ++j) {
    segs[(size_t)j] = seg(j);
    off[(size_t)j] = (int)(segs[(size_t)j].start % kQ4kBlockElems);
    require(off[(size_t)j] % 32 == 0, FABER_STATUS_UNSUPPORTED, "row start is not sub-block aligned");
    require((segs[(size_t)j].start + (uint64_t)cols + kQ4kBlockElems - 1) / kQ4kBlockElems <=
                segs[(size_t)j].n_blocks,
            FABER_STATUS_INVALID_ARGUMENT, "row extends past the tensor's blocks");
    max_o = std::max(max_o, off[(size_t)j]);
  }
  T.nb = (cols + max_o + kQ4kBlockElems - 1) / kQ4kBlockElems;
  // group rows by offset class (stable), 16 per tile
  std::vector<int> order((size_t)rows);
  for (int j = 0; j < rows; ++j) order[(size_t)j] = j;
  std::stable_sort(order.begin(), order.end(),
                   [&](int a, int b) { return off[(size_t)a] < off[(size_t)b]; });
  std::vector<int> tile_of_slot;  // flattened tile rows
  for (size_t i = 0; i < order.size();) {
    const int o = off[(size_t)order[i]];
    size_t k = i;
    while (k < order.size() && off[(size_t)order[k]] == o) ++k;
    const int count = (int)(k - i);
    const int tiles = (count + kTileRows - 1) / kTileRows;
    for (int tt = 0; tt < tiles; ++tt) {
      T.xoff.push_back(o);
      for (int r = 0; r < kTileRows; ++r) {
        const size_t idx = i + (size_t)tt * kTileRows + r;
        T.rowmap.push_back(idx < k ? order[idx] : -1);
      }
    }
    i = k;
  }
  T.n_tiles = (int)T.xoff.size();
  for (int tl = 0; tl < T.n_tiles && T.identity; ++tl) {
    if (T.xoff[(size_t)tl] != 0) T.identity = false;
    for (int r = 0; r < kTileRows; ++r) {
      const int row = T.rowmap[(size_t)tl * kTileRows + r];
      const int want = tl * kTileRows + r;
      if (!(row == want || (row < 0 && want >= rows))) T.identity = false;
    }
  }
  T.data.assign((size_t)T.n_tiles * T.nb * kTileItemBytes, 0);

  auto fill_tiles = [&](int t0, int t1) {
    for (int tl = t0; tl < t1; ++tl) {
      for (int r = 0; r < kTileRows; ++r) {
        const int row = T.rowmap[(size_t)tl * kTileRows + r];
        if (row < 0) continue;
        const RowSeg& s = segs[(size_t)row];
        const uint64_t first = s.start / kQ4kBlockElems;
        const uint64_t lo = s.start, hi = s.start + (uint64_t)cols;
        for (int b = 0; b < T.nb; ++b) {
          const uint64_t sb = first + (uint64_t)b;
          if (sb * kQ4kBlockElems >= hi || sb >= s.n_blocks) break;
          uint8_t blk[kQ4kBlockBytes];
          std::memcpy(blk, s.base + sb * kQ4kBlockBytes, kQ4kBlockBytes);
          const uint64_t b0 = sb * kQ4kBlockElems;
          if (b0 < lo || b0 + kQ4kBlockElems > hi) {
            uint8_t sc[8], m[8];
            unpack_scales(blk + 4, sc, m);
            for (int jj = 0; jj < 8; ++jj) {
              const uint64_t e0 = b0 + 32u * jj;
              if (e0 >= lo && e0 + 32 <= hi) continue;
              sc[jj] = 0;
              m[jj] = 0;
              const int c = jj >> 1;
              for (int l = 0; l < 32; ++l) blk[16 + 32 * c + l] &= (jj & 1) ? 0x0f : 0xf0;
            }
            pack_scales(sc, m, blk + 4);
          }
          uint8_t* item = T.data.data() + ((size_t)tl * T.nb + b) * kTileItemBytes;
          std::memcpy(item + 16 * r, blk, 16);
          std::memcpy(item + 256 + 128 * r, blk + 16, 128);
        }
      }
    }
  };
  const size_t bytes = T.data.size();
  unsigned nthr = bytes > (64u << 20) ? std::max(1u, std::min(16u, std::thread::hardware_concurrency())) : 1u;
  if (nthr <= 1) {
    fill_tiles(0, T.n_tiles);
  } else {
    std::vector<std::thread> th;
    const int per = (T.n_tiles + (int)nthr - 1) / (int)nthr;
    for (unsigned k = 0; k < nthr; ++k) {
      const int t0 = (int)k * per, t1 = std::min(T.n_tiles, t0 + per);
      if (t0 < t1) th.emplace_back(fill_tiles, t0, t1);
    }
    for (auto& x : th) x.join();
  }
  return T;
}

// Repack identity: FNV-1a over the layout parameters and a sample of the
// source bytes (the Declared(RepackHash) of the reference's repack plan).
inline uint64_t repack_hash(const TiledQ4k& T) {
  uint64_t h = 1469598103934665603ull;
  auto mix = [&](const void* p, size_t n) {
    const uint8_t* b = static_cast<const uint8_t*>(p);
    for (size_t i = 0; i < n; ++i) {
      h ^= b[i];
      h *= 1099511628211ull;
    }
  };
  const char tag[] = "faber-q4k-tile16-v1";
  mix(tag, sizeof(tag));
  mix(&T.rows, sizeof(int));
  mix(&T.cols, sizeof(int));
  mix(&T.nb, sizeof(int));
  mix(&T.n_tiles, sizeof(int));
  mix(T.xoff.data(), T.xoff.size() * sizeof(int32_t));
  mix(T.rowmap.data(), T.rowmap.size() * sizeof(int32_t));
  const size_t n = T.data.size();
  const size_t step = std::max<size_t>(1, n / 4096);
  for (size_t i = 0; i < n; i += step) mix(&T.data[i], 1);
  return h;
}

}  // namespace faber
