// faber_gpu.cu — the C ABI of the B200 Q4_K decoder path (library entry).
//
// Single translation unit: the kernels (gemv.cuh, ops.cuh), the host-side
// repack (repack.hpp), the model/session engine (engine.cuh) and the
// extern "C" entry points declared in include/faber_gpu.h.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <map>
#include <memory>
#include <mutex>
#include <vector>

#include "abi.hpp"
#include "gemv.cuh"
#include "gemv_rows.cuh"
#include "gguf.hpp"
#include "ops.cuh"
#include "repack.hpp"
#include "tokenizer.hpp"
#include "transaction.hpp"

namespace faber {

// ---------------------------------------------------------------------------
// Device facts
// ---------------------------------------------------------------------------
struct DeviceInfo {
  int sms = 0;
  int major = 0, minor = 0;
};

inline DeviceInfo device_info() {
  static std::mutex mu;
  static std::map<int, DeviceInfo> cache;
  int dev = 0;
  FABER_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  cudaDeviceProp p;
  FABER_CUDA(cudaGetDeviceProperties(&p, dev));
  DeviceInfo d{p.multiProcessorCount, p.major, p.minor};
  cache[dev] = d;
  return d;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ---------------------------------------------------------------------------
// GEMV launch
// ---------------------------------------------------------------------------
template <int WL, int PRO, int EPI>
void launch_gemv_pipe(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  auto kern = gemv_pipe_kernel<WL, PRO, EPI>;
  static thread_local std::map<int, bool> attr_done;
  int dev = 0;
  FABER_CUDA(cudaGetDevice(&dev));
  if (!attr_done[dev]) {
    FABER_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448));
    attr_done[dev] = true;
  }
  const PipeLayout L = pipe_layout(a.nb);
  require(L.total <= 232448, FABER_STATUS_UNSUPPORTED, "GEMV input too long for shared-memory staging");
  // two CTAs per SM: 16 consumer warps hide the dequant dependency chains
  const int per_sm = 2 * L.total <= 227 * 1024 ? 2 : 1;
  const int grid = std::max(1, std::min(a.n_tiles, per_sm * device_info().sms));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kPipeThreads);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  FABER_CUDA(cudaLaunchKernelEx(&cfg, kern, a));
}

template <int WL, int PRO, int EPI>
void launch_gemv(const GemvArgs& a, cudaStream_t stream, bool pdl) {
  if constexpr (WL != WL_F16) {
    launch_gemv_pipe<WL, PRO, EPI>(a, stream, pdl);
    return;
  } else {
  auto kern = gemv_kernel<WL, PRO, EPI>;
  // per device: attribute set once; occupancy cached per shared-memory size
  static thread_local std::map<int, std::map<size_t, int>> occ_cache;
  int dev = 0;
  FABER_CUDA(cudaGetDevice(&dev));
  auto& per_dev = occ_cache[dev];
  if (per_dev.empty())
    FABER_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448));
  const size_t smem = gemv_smem_bytes(a.nb);
  require(smem <= 232448, FABER_STATUS_UNSUPPORTED, "GEMV input too long for shared-memory staging");
  int occ = 0;
  auto it = per_dev.find(smem);
  if (it == per_dev.end()) {
    FABER_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kGemvThreads, smem));
    per_dev[smem] = occ;
  } else {
    occ = it->second;
  }
  occ = std::max(1, occ);
  const int grid = std::max(1, std::min(a.n_tiles, occ * device_info().sms));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  FABER_CUDA(cudaLaunchKernelEx(&cfg, kern, a));
  }
}

template <class K, class... Args>
void launch_pdl(K kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  FABER_CUDA(cudaLaunchKernelEx(&cfg, kern, args...));
}

// ---------------------------------------------------------------------------
// Partition byte accounting: the classes of PartitionBudgetLedger
// (src/partition.rs:111-137). Every device buffer is charged to one class of
// the device it lives on when allocated and credited back when freed. The
// allocator policy charges a buffer below 1 MiB in 512-byte units and a
// larger one in 2 MiB units (the driver's suballocation and large-page
// granularity); the rounding is the allocator-overhead class. With a policy
// limit set, an allocation whose charge would take the device's total above
// it fails before cudaMalloc runs. The tables are constant-initialized and
// trivially destructible, so buffers freed during static destruction still
// find them.
// ---------------------------------------------------------------------------
enum LedgerClass : int {
  kLedgerWeights = 0,
  kLedgerKv = 1,
  kLedgerActivation = 2,
  kLedgerModule = 3,
  kLedgerOverhead = 4,
  kLedgerStaging = 5,
  kLedgerConcurrent = 6,
  kLedgerClasses = 7
};
constexpr int kLedgerMaxDevices = 64;

struct DeviceLedger {
  uint64_t live[kLedgerClasses];
  uint64_t limit;  // 0: no policy limit
  bool touched;    // the device has held a buffer of this library
};

static std::mutex g_ledger_mu;
static DeviceLedger g_ledger[kLedgerMaxDevices];

// Class 4: the allocation-free attention scratch of the module image
// (defined with that entry point), counted from a device's first buffer on.
uint64_t static_attn_module_bytes();

// The policy charge of an n-byte buffer (0 when it cannot be represented).
inline uint64_t ledger_charge(uint64_t n) {
  if (n == 0) return 0;
  const uint64_t unit = n < (uint64_t(1) << 20) ? 512 : (uint64_t(2) << 20);
  if (n > UINT64_MAX - unit) return 0;
  return (n + unit - 1) / unit * unit;
}

inline uint64_t ledger_total(const DeviceLedger& L) {
  uint64_t t = 0;
  for (int c = 0; c < kLedgerClasses; ++c) t += L.live[c];
  return t;
}

// Charges n bytes of class cls to device dev, or throws ALLOCATION when the
// device's policy limit would be passed. Ordinals above the table are not
// accounted (no limit applies there).
inline void ledger_take(int dev, int cls, uint64_t n) {
  if (dev < 0 || dev >= kLedgerMaxDevices || n == 0) return;
  const uint64_t c = ledger_charge(n);
  std::lock_guard<std::mutex> g(g_ledger_mu);
  DeviceLedger& L = g_ledger[dev];
  const uint64_t module = L.touched ? 0 : static_attn_module_bytes();
  const uint64_t held = ledger_total(L) + module;
  if (c == 0 || (L.limit && (c > L.limit || held > L.limit - c)))
    throw Error(FABER_STATUS_ALLOCATION,
                "partition budget: " + std::to_string(n) + " bytes (charged " + std::to_string(c) +
                    ") on device " + std::to_string(dev) + " holding " + std::to_string(held) +
                    " of a " + std::to_string(L.limit) + "-byte limit");
  L.live[kLedgerModule] += module;
  L.live[cls] += n;
  L.live[kLedgerOverhead] += c - n;
  L.touched = true;
}

inline void ledger_give(int dev, int cls, uint64_t n) {
  if (dev < 0 || dev >= kLedgerMaxDevices || n == 0) return;
  const uint64_t c = ledger_charge(n);
  std::lock_guard<std::mutex> g(g_ledger_mu);
  DeviceLedger& L = g_ledger[dev];
  L.live[cls] -= n;
  L.live[kLedgerOverhead] -= c - n;
}

// ---------------------------------------------------------------------------
// Device buffers
// ---------------------------------------------------------------------------
struct DevBuf {
  void* p = nullptr;
  size_t n = 0;
  int dev = -1;
  int cls = kLedgerActivation;
  DevBuf() = default;
  explicit DevBuf(size_t bytes, int ledger_class = kLedgerActivation) { alloc(bytes, ledger_class); }
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  DevBuf(DevBuf&& o) noexcept : p(o.p), n(o.n), dev(o.dev), cls(o.cls) { o.p = nullptr; o.n = 0; }
  DevBuf& operator=(DevBuf&& o) noexcept {
    if (this != &o) {
      release();
      p = o.p;
      n = o.n;
      dev = o.dev;
      cls = o.cls;
      o.p = nullptr;
      o.n = 0;
    }
    return *this;
  }
  ~DevBuf() { release(); }
  void alloc(size_t bytes, int ledger_class = kLedgerActivation) {
    release();
    FABER_CUDA(cudaGetDevice(&dev));
    cls = ledger_class;
    if (bytes) {
      ledger_take(dev, cls, bytes);  // a passed limit allocates nothing
      cudaError_t e = cudaMalloc(&p, bytes);
      if (e != cudaSuccess) {
        cudaGetLastError();
        p = nullptr;
        ledger_give(dev, cls, bytes);
        throw Error(FABER_STATUS_ALLOCATION, "cudaMalloc(" + std::to_string(bytes) + ") failed: " +
                                                 cudaGetErrorString(e));
      }
    }
    n = bytes;
  }
  void release() {
    if (p) {
      int cur = -1;
      cudaGetDevice(&cur);
      if (dev >= 0 && cur != dev) cudaSetDevice(dev);
      cudaFree(p);
      if (dev >= 0 && cur != dev && cur >= 0) cudaSetDevice(cur);
      ledger_give(dev, cls, n);
    }
    p = nullptr;
    n = 0;
  }
  template <class T> T* as() const { return static_cast<T*>(p); }
};

inline void upload(DevBuf& b, const void* host, size_t bytes, int ledger_class = kLedgerActivation) {
  b.alloc(bytes, ledger_class);
  if (bytes) FABER_CUDA(cudaMemcpy(b.p, host, bytes, cudaMemcpyHostToDevice));
}

// A Q4_K weight in tile layout on the device.
struct DeviceTiled {
  DevBuf w, xoff, rowmap;
  int n_tiles = 0, nb = 0, rows = 0, cols = 0;
  bool identity = true;
  uint64_t hash = 0;
  void from(const TiledQ4k& T) {
    upload(w, T.data.data(), T.data.size(), kLedgerWeights);
    n_tiles = T.n_tiles;
    nb = T.nb;
    rows = T.rows;
    cols = T.cols;
    identity = T.identity;
    hash = repack_hash(T);
    if (!identity) {
      upload(xoff, T.xoff.data(), T.xoff.size() * sizeof(int32_t), kLedgerWeights);
      upload(rowmap, T.rowmap.data(), T.rowmap.size() * sizeof(int32_t), kLedgerWeights);
    } else {
      xoff.release();
      rowmap.release();
    }
  }
  GemvArgs args() const {
    GemvArgs a = {};
    a.w = w.as<uint8_t>();
    a.n_tiles = n_tiles;
    a.nb = nb;
    a.n_rows = rows;
    a.n_cols = cols;
    a.tile_xoff = identity ? nullptr : xoff.as<int32_t>();
    a.row_map = identity ? nullptr : rowmap.as<int32_t>();
    return a;
  }
};

// A linear stored as rows of native GGML blocks (any admitted type per row),
// in the fused order of the epilogues, padded to whole 16-row tiles.
struct DeviceRows {
  DevBuf bytes, row_off, row_type;
  int n_tiles = 0, rows = 0, cols = 0;
  bool valid() const { return rows > 0; }
  RowsArgs args() const {
    RowsArgs r;
    r.bytes = bytes.as<uint8_t>();
    r.row_off = row_off.as<uint64_t>();
    r.row_type = row_type.as<uint32_t>();
    r.n_tiles = n_tiles;
    r.cols = cols;
    return r;
  }
  GemvArgs gemv_args() const {
    GemvArgs a = {};
    a.n_tiles = n_tiles;
    a.n_rows = rows;
    a.n_cols = cols;
    return a;
  }
};

template <int PRO, int EPI>
void launch_gemv_rows(const GemvArgs& a, const DeviceRows& W, cudaStream_t stream, bool pdl) {
  auto kern = gemv_rows_kernel<PRO, EPI>;
  static thread_local std::map<int, bool> attr_done;
  int dev = 0;
  FABER_CUDA(cudaGetDevice(&dev));
  if (!attr_done[dev]) {
    FABER_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    attr_done[dev] = true;
  }
  const size_t smem = (size_t)W.cols * 4;
  require(smem <= 200 * 1024, FABER_STATUS_UNSUPPORTED, "input too long for the row GEMV's staging");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)std::max(1, std::min(W.n_tiles, 4 * device_info().sms)));
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  FABER_CUDA(cudaLaunchKernelEx(&cfg, kern, a, W.args()));
}


}  // namespace faber

struct FaberGpuQ4kTensor {
  faber::DeviceTiled t;
  // scratch of faber_gpu_v2_q4k_gemv_batch, allocated on its first call:
  // the x split (16 sequences x hi/lo rows), scales, slab partials
  faber::DevBuf bxs, bscale, bpart;
};

#include "engine.cuh"

using namespace faber;

// ---------------------------------------------------------------------------
// extern "C" entry points
// ---------------------------------------------------------------------------
extern "C" {

__attribute__((visibility("default"))) uint32_t faber_gpu_v2_abi_version(void) { return 2; }

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_last_error(char* buf,
                                                                              uint64_t cap) {
  if (!buf || cap == 0) return status(FABER_STATUS_INVALID_ARGUMENT);
  const size_t n = std::min<size_t>(cap - 1, g_last_error.size());
  std::memcpy(buf, g_last_error.data(), n);
  buf[n] = 0;
  return status(FABER_STATUS_OK);
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_init(int32_t device) {
  return guarded("faber_gpu_v2_init", [&] {
    int count = 0;
    FABER_CUDA(cudaGetDeviceCount(&count));
    FABER_ARG(device >= 0 && device < count, "device ordinal out of range");
    FABER_CUDA(cudaSetDevice(device));
    const DeviceInfo d = device_info();
    require(d.major == 10, FABER_STATUS_UNSUPPORTED,
            "this library is built for sm_100a (B200); device is sm_" +
                std::to_string(d.major * 10 + d.minor));
    FABER_CUDA(cudaFree(nullptr));
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_fault_inject(
    const char* entry, int32_t code, uint32_t count) {
  if (!entry) return status(FABER_STATUS_INVALID_ARGUMENT);
  std::lock_guard<std::mutex> lk(g_faults.mu);
  if (count == 0) g_faults.table.erase(entry);
  else g_faults.table[entry] = {code, count};
  return status(FABER_STATUS_OK);
}

// --- placement ABI (hosts/llvm/src/gpu_placement.rs:53-137) --------------
namespace {
std::mutex g_place_mu;
std::map<uint64_t, DevBuf>& placed() {
  static std::map<uint64_t, DevBuf> m;
  return m;
}
}  // namespace

__attribute__((visibility("default"))) FaberRtStatusV1 __faber_gpu_v1_copy_in(
    uint64_t logical_id, const uint8_t* data_ptr, uint64_t data_len, uint32_t dtype) {
  (void)dtype;
  return guarded("__faber_gpu_v1_copy_in", [&] {
    FABER_ARG(!(data_len > 0 && data_ptr == nullptr), "null data pointer with nonzero length");
    std::lock_guard<std::mutex> lk(g_place_mu);
    DevBuf b;
    upload(b, data_ptr, data_len, kLedgerConcurrent);  // host-keyed runtime state
    placed()[logical_id] = std::move(b);
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 __faber_gpu_v1_readback(
    uint64_t logical_id, uint8_t* dest_ptr, uint64_t dest_capacity, uint64_t* actual_len) {
  return guarded("__faber_gpu_v1_readback", [&] {
    FABER_ARG(dest_ptr != nullptr && actual_len != nullptr, "null destination");
    std::lock_guard<std::mutex> lk(g_place_mu);
    auto it = placed().find(logical_id);
    FABER_ARG(it != placed().end(), "unknown logical buffer id");
    require(it->second.n <= dest_capacity, FABER_STATUS_IO_ERROR, "destination capacity too small");
    if (it->second.n) FABER_CUDA(cudaMemcpy(dest_ptr, it->second.p, it->second.n, cudaMemcpyDeviceToHost));
    *actual_len = it->second.n;
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 __faber_gpu_v1_sync(uint64_t logical_id) {
  (void)logical_id;
  return guarded("__faber_gpu_v1_sync", [&] { FABER_CUDA(cudaDeviceSynchronize()); });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_buffer_device_ptr(
    uint64_t logical_id, void** dev_ptr, uint64_t* len) {
  return guarded("faber_gpu_v2_buffer_device_ptr", [&] {
    FABER_ARG(dev_ptr && len, "null output");
    std::lock_guard<std::mutex> lk(g_place_mu);
    auto it = placed().find(logical_id);
    FABER_ARG(it != placed().end(), "unknown logical buffer id");
    *dev_ptr = it->second.p;
    *len = it->second.n;
  });
}

// --- stateless kernels ------------------------------------------------------
__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_dequant_q4k(
    const uint8_t* blocks, uint64_t n_blocks, float* out, int32_t f16_round, void* stream) {
  return guarded("faber_gpu_v2_dequant_q4k", [&] {
    FABER_ARG(n_blocks == 0 || (blocks && out), "null pointer");
    if (n_blocks == 0) return;
    const uint64_t threads = n_blocks * 32;
    dequant_q4k_native_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, as_stream(stream)>>>(
        blocks, n_blocks, out, f16_round ? 1 : 0);
    FABER_CUDA(cudaGetLastError());
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_dequant_blocks(
    uint32_t ggml_type, const uint8_t* blocks, uint64_t n_blocks, float* out, int32_t f16_round,
    void* stream) {
  return guarded("faber_gpu_v2_dequant_blocks", [&] {
    int be = 0, bb = 0;
    FABER_ARG(ggml_block_geometry(ggml_type, be, bb), "unknown GGML type " + std::to_string(ggml_type));
    FABER_ARG(n_blocks == 0 || (blocks && out), "null pointer");
    if (n_blocks == 0) return;
    const uint64_t threads = n_blocks * 32;
    dequant_blocks_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, as_stream(stream)>>>(
        ggml_type, blocks, n_blocks, out, f16_round ? 1 : 0);
    FABER_CUDA(cudaGetLastError());
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_f16_round(const float* x,
                                                                             float* y, uint64_t n,
                                                                             void* stream) {
  return guarded("faber_gpu_v2_f16_round", [&] {
    FABER_ARG(n == 0 || (x && y), "null pointer");
    if (n == 0) return;
    const unsigned grid = (unsigned)std::min<uint64_t>((n + 255) / 256, 4 * 148 * 8);
    f16_round_kernel<<<grid, 256, 0, as_stream(stream)>>>(x, y, n);
    FABER_CUDA(cudaGetLastError());
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_gemv_q4k(
    const uint8_t* w_blocks, uint64_t rows, uint64_t cols, const float* x, float* y,
    void* stream) {
  return guarded("faber_gpu_v2_gemv_q4k", [&] {
    FABER_ARG(rows > 0 && cols > 0 && w_blocks && x && y, "null pointer or empty shape");
    require(cols % 256 == 0, FABER_STATUS_UNSUPPORTED,
            "native-layout GEMV needs cols % 256 == 0; upload with faber_gpu_v2_q4k_upload");
    FABER_ARG(rows < (1u << 30) && cols < (1u << 20), "shape too large");
    GemvArgs a = {};
    a.w = w_blocks;
    a.n_rows = (int)rows;
    a.n_cols = (int)cols;
    a.nb = (int)(cols / 256);
    a.n_tiles = (int)((rows + kTileRows - 1) / kTileRows);
    a.x = x;
    a.out = y;
    launch_gemv<WL_NATIVE, PRO_PLAIN, EPI_STORE>(a, as_stream(stream), false);
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_q4k_upload(
    const uint8_t* host_blocks, uint64_t nbytes, uint64_t rows, uint64_t cols,
    FaberGpuQ4kTensor** out) {
  return guarded("faber_gpu_v2_q4k_upload", [&] {
    FABER_ARG(out && host_blocks && rows > 0 && cols > 0, "null pointer or empty shape");
    FABER_ARG(rows < (1u << 30) && cols < (1u << 20), "shape too large");
    FABER_ARG((rows * cols) % 256 == 0, "element count is not a multiple of the Q4_K block");
    const uint64_t nblocks = rows * cols / 256;
    FABER_ARG(nbytes == nblocks * kQ4kBlockBytes,
              "packed tensor is " + std::to_string(nbytes) + " bytes, expected exactly " +
                  std::to_string(nblocks * kQ4kBlockBytes));
    TiledQ4k T = repack_q4k((int)rows, (int)cols, [&](int j) {
      return RowSeg{host_blocks, nblocks, (uint64_t)j * cols};
    });
    auto t = std::make_unique<FaberGpuQ4kTensor>();
    t->t.from(T);
    *out = t.release();
  });
}

// A linear of any admitted block type, as typed rows (validation surface of
// the row GEMV the decoder uses for non-Q4_K linears).
struct FaberGpuTypedTensor {
  faber::DeviceRows r;
};

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_typed_upload(
    uint32_t ggml_type, const uint8_t* host_blocks, uint64_t nbytes, uint64_t rows, uint64_t cols,
    FaberGpuTypedTensor** out) {
  return guarded("faber_gpu_v2_typed_upload", [&] {
    FABER_ARG(out != nullptr && host_blocks != nullptr, "null pointer");
    *out = nullptr;
    int be = 0, bb = 0;
    FABER_ARG(ggml_block_geometry(ggml_type, be, bb), "unknown GGML type " + std::to_string(ggml_type));
    FABER_ARG(rows > 0 && cols > 0 && cols % (uint64_t)be == 0, "rows must be whole blocks");
    FABER_ARG(nbytes == rows * cols / be * bb, "packed tensor is " + std::to_string(nbytes) +
                                                   " bytes, expected exactly " +
                                                   std::to_string(rows * cols / be * bb));
    HostTensor h;
    h.type = ggml_type;
    h.rows = rows;
    h.cols = cols;
    h.bytes.assign(host_blocks, host_blocks + nbytes);
    auto t = std::make_unique<FaberGpuTypedTensor>();
    rows_from(t->r, (int)rows, (int)cols,
              [&](int j) { return std::pair<const HostTensor*, uint64_t>(&h, (uint64_t)j); });
    *out = t.release();
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_typed_gemv(
    const FaberGpuTypedTensor* t, const float* x, float* y, void* stream) {
  return guarded("faber_gpu_v2_typed_gemv", [&] {
    FABER_ARG(t && x && y, "null pointer");
    GemvArgs a = t->r.gemv_args();
    a.x = x;
    a.out = y;
    launch_gemv_rows<PRO_PLAIN, EPI_STORE>(a, t->r, as_stream(stream), false);
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_typed_free(FaberGpuTypedTensor* t) {
  return guarded("faber_gpu_v2_typed_free", [&] { delete t; });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_q4k_free(FaberGpuQ4kTensor* t) {
  return guarded("faber_gpu_v2_q4k_free", [&] { delete t; });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_q4k_gemv(
    const FaberGpuQ4kTensor* t, const float* x, float* y, void* stream) {
  return guarded("faber_gpu_v2_q4k_gemv", [&] {
    FABER_ARG(t && x && y, "null pointer");
    GemvArgs a = t->t.args();
    a.x = x;
    a.out = y;
    // programmatic dependent launch, as in the decode step: the producer
    // streams weights while the previous kernel finishes; every read of x
    // and write of y waits for that kernel's completion
    launch_gemv<WL_TILED, PRO_PLAIN, EPI_STORE>(a, as_stream(stream), true);
  });
}

}  // extern "C"

namespace faber {
// Epoch base and grid-barrier words of the exchange validation call.
__device__ uint32_t g_xcheck_epoch;
__device__ unsigned int g_xcheck_bar[2];
}  // namespace faber

extern "C" {

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_q4k_gemv_exchange(
    const FaberGpuQ4kTensor* t, const float* x, const float* norm_w, float eps, const uint64_t* exchange,
    uint32_t tp, uint32_t epoch, uint32_t wait_limit, float* x_sum_out, float* y, void* stream) {
  return guarded("faber_gpu_v2_q4k_gemv_exchange", [&] {
    FABER_ARG(t && x && norm_w && exchange && x_sum_out && y, "null pointer");
    FABER_ARG(tp >= 1 && tp <= (uint32_t)kMaxTp, "tp must be in [1, 8]");
    FABER_ARG(epoch >= 1, "epoch 0 marks an empty exchange word");
    const cudaStream_t st = as_stream(stream);
    // a stale expiry flag of other work on this device is not this call's
    int flag = 0;
    FABER_CUDA(cudaStreamSynchronize(st));
    FABER_CUDA(cudaMemcpyFromSymbol(&flag, g_pipe_error, sizeof(int)));
    require(flag == 0, FABER_STATUS_TIMEOUT, "an earlier device wait on this device expired");
    uint32_t* epoch_dev = nullptr;
    unsigned int* bar_dev = nullptr;
    FABER_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&epoch_dev), g_xcheck_epoch));
    FABER_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&bar_dev), g_xcheck_bar));
    const uint32_t base = epoch - 1u;  // the kernel's epoch: base * stages + stage + 1
    FABER_CUDA(cudaMemcpyToSymbolAsync(g_xcheck_epoch, &base, sizeof(base), 0, cudaMemcpyHostToDevice, st));
    GemvArgs a = t->t.args();
    a.x = x;
    a.norm_w = norm_w;
    a.eps = eps;
    a.x_sum_out = x_sum_out;
    a.out = y;
    a.tp = (int32_t)tp;
    a.tp_stage = 0;
    a.tp_stages = 1;
    a.epoch_ptr = epoch_dev;
    a.red = reinterpret_cast<const unsigned long long*>(exchange);
    a.grid_bar = bar_dev;
    a.peer_wait_limit = wait_limit;
    launch_gemv<WL_TILED, PRO_NORM_PEERS, EPI_STORE>(a, st, false);
    FABER_CUDA(cudaStreamSynchronize(st));
    FABER_CUDA(cudaMemcpyFromSymbol(&flag, g_pipe_error, sizeof(int)));
    if (flag) {
      const int zero = 0;
      FABER_CUDA(cudaMemcpyToSymbol(g_pipe_error, &zero, sizeof(int)));
      throw Error(FABER_STATUS_TIMEOUT, flag == 3 ? "a grid barrier wait expired"
                                                  : "an exchange word did not carry the epoch in time");
    }
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_q4k_gemv_batch(
    FaberGpuQ4kTensor* t, const float* x, uint32_t batch, float* y, void* stream) {
  return guarded("faber_gpu_v2_q4k_gemv_batch", [&] {
    FABER_ARG(t && x && y, "null pointer");
    FABER_ARG(batch >= 1 && batch <= (uint32_t)kBgMaxSeq, "batch must be in [1, 16]");
    require(t->t.identity, FABER_STATUS_UNSUPPORTED, "batched GEMV needs rows in whole super-blocks");
    const cudaStream_t st = as_stream(stream);
    const int K = t->t.cols;
    if (!t->bxs.p) {
      // sized for the largest batch: 16 sequences use the most slabs
      t->bxs.alloc((size_t)2 * kBgMaxSeq * K * 2);
      t->bscale.alloc((size_t)kBgMaxSeq * 4);
      t->bpart.alloc(std::max<size_t>(bgemv_part_floats(t->t, kBgMaxSeq), 1) * 4);
    }
    __half* xs = t->bxs.as<__half>();
    float* xscale = t->bscale.as<float>();
    prefill_split_kernel<false><<<batch, kGemvThreads, 0, st>>>(x, K, nullptr, 0.0f, xs, xscale);
    FABER_CUDA(cudaGetLastError());
    BgemvArgs a = {};
    a.xs = xs;
    a.xscale = xscale;
    a.out = y;
    a.ld_out = t->t.rows;
    a.part = t->bpart.as<float>();
    launch_bgemv<BG_STORE>(t->t, a, (int)batch, K, st);
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_q4k_dequant_rows(
    const FaberGpuQ4kTensor* t, float* out, int32_t f16_round, void* stream) {
  return guarded("faber_gpu_v2_q4k_dequant_rows", [&] {
    FABER_ARG(t && out, "null pointer");
    const DeviceTiled& d = t->t;
    const uint64_t warps = (uint64_t)d.n_tiles * kTileRows * d.nb;
    dequant_q4k_tiled_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, as_stream(stream)>>>(
        d.w.as<uint8_t>(), d.n_tiles, d.nb, d.rows, d.cols,
        d.identity ? nullptr : d.xoff.as<int32_t>(), d.identity ? nullptr : d.rowmap.as<int32_t>(),
        out, f16_round ? 1 : 0);
    FABER_CUDA(cudaGetLastError());
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_q4k_repack_hash(
    const FaberGpuQ4kTensor* t, uint64_t* hash) {
  return guarded("faber_gpu_v2_q4k_repack_hash", [&] {
    FABER_ARG(t && hash, "null pointer");
    *hash = t->t.hash;
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_kv_layout_bytes(
    const FaberKvLayoutV1* l, uint64_t* total, uint64_t* admitted) {
  return guarded("faber_gpu_v2_kv_layout_bytes", [&] {
    FABER_ARG(l && total && admitted, "null pointer");
    FABER_ARG(l->slots && l->context_length && l->layer_count && l->kv_head_count && l->head_dim,
              "a zero-sized KV layout is not a layout");
    FABER_ARG(l->dtype <= 1, "unknown KV dtype");
    const unsigned __int128 per_layer =
        (unsigned __int128)l->context_length * l->kv_head_count * l->head_dim;
    const unsigned __int128 elems = per_layer * l->layer_count * 2u;
    const unsigned __int128 bytes = elems * (l->dtype == 0 ? 4u : 2u) * l->slots;
    require(bytes <= (unsigned __int128)UINT64_MAX, FABER_STATUS_IO_ERROR, "KV byte count overflows");
    require(bytes + l->reserve_bytes <= (unsigned __int128)UINT64_MAX, FABER_STATUS_IO_ERROR,
            "KV admitted byte count overflows");
    *total = (uint64_t)bytes;
    *admitted = (uint64_t)(bytes + l->reserve_bytes);
  });
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free decode attention
//
// For callers that must not allocate device memory: a host whose device
// memory is fully accounted up front (a fixed per-device byte budget, where
// an unaccounted cudaMalloc is a failure), or one on a latency-critical path
// where cudaMalloc / cudaFree may synchronize the whole device. The scratch
// that the split-K attention needs (the per-split partials, the merge
// counters and the position word) lives in one file-scope __device__ array
// instead of session buffers. That array is part of the module image: every
// GPU that loads this library holds it (about 2 MiB) until the process exits,
// whether or not the entry point is ever called.
// ---------------------------------------------------------------------------
namespace faber {

constexpr int kStaticAttnMaxHeads = 128;     // query heads
constexpr int kStaticAttnMaxKvHeads = 128;   // kv heads
constexpr size_t kStaticAttnStateOff = 0;    // StepState (cur_pos)
constexpr size_t kStaticAttnCountersOff = 256;
constexpr size_t kStaticAttnPartOff = kStaticAttnCountersOff + kStaticAttnMaxKvHeads * 4;
constexpr size_t kStaticAttnPartBytes = size_t(2) << 20;
constexpr size_t kStaticAttnBytes = kStaticAttnPartOff + kStaticAttnPartBytes;
constexpr int kStaticAttnMaxDevices = 64;

static __device__ __align__(256) unsigned char g_static_attn_scratch[kStaticAttnBytes];

uint64_t static_attn_module_bytes() { return (uint64_t)kStaticAttnBytes; }

// Argument check that builds its message only on failure (the shared
// require() takes a std::string, which would allocate on every call).
inline void static_check(bool cond, int code, const char* msg) {
  if (!cond) throw Error(code, msg);
}

// Opens one call: the merge counters start at zero and the attention kernel
// reads the last position from the state word.
__global__ void static_attn_open_kernel(StepState* st, int32_t* counters, int n_kv_heads,
                                        int cur_pos) {
  for (int i = threadIdx.x; i < n_kv_heads; i += blockDim.x) counters[i] = 0;
  if (threadIdx.x == 0) st->cur_pos = cur_pos;
}

// Device address of the scratch array on the current device. In host code the
// array's name is only a host-side stand-in, so the address is looked up once
// per device (with that device current) and cached in a fixed table.
inline unsigned char* static_attn_scratch(int dev) {
  static std::mutex mu;
  static unsigned char* table[kStaticAttnMaxDevices] = {};
  static_check(dev >= 0 && dev < kStaticAttnMaxDevices, FABER_STATUS_UNSUPPORTED,
               "device ordinal above 63 has no scratch slot");
  std::lock_guard<std::mutex> lk(mu);
  if (!table[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_attn_scratch);
    if (e != cudaSuccess) {
      cudaGetLastError();
      throw Error(FABER_STATUS_CUDA_ERROR,
                  std::string("cudaGetSymbolAddress(attention scratch) failed: ") +
                      cudaGetErrorString(e));
    }
    table[dev] = static_cast<unsigned char*>(p);
  }
  return table[dev];
}

inline void attention_decode_static(const float* q, const void* k_cache, const void* v_cache,
                                    float* ctx, uint32_t n_heads, uint32_t n_kv_heads,
                                    uint32_t head_dim, uint64_t n_kv, cudaStream_t stream) {
  constexpr int kBad = FABER_STATUS_INVALID_ARGUMENT;
  static_check(q && k_cache && v_cache && ctx, kBad, "null pointer");
  static_check(head_dim == 64 || head_dim == 128, kBad, "head_dim must be 64 or 128");
  static_check(n_kv_heads >= 1 && n_heads >= n_kv_heads && n_heads % n_kv_heads == 0, kBad,
               "n_heads must be a positive multiple of n_kv_heads");
  static_check(n_heads / n_kv_heads <= (uint32_t)kAttnMaxRatio, kBad,
               "more than 8 query heads per kv head");
  static_check(n_heads <= (uint32_t)kStaticAttnMaxHeads &&
                   n_kv_heads <= (uint32_t)kStaticAttnMaxKvHeads,
               kBad, "the static attention scratch holds at most 128 query heads and 128 kv heads");
  // the kernel counts positions and 32-position groups in int: n_kv + 31
  // must not overflow
  static_check(n_kv >= 1 && n_kv <= (uint64_t)(INT32_MAX - kAttnGroup), kBad,
               "n_kv must be in [1, 2^31 - 33]");
  int dev = 0, sms = 0;
  FABER_CUDA(cudaGetDevice(&dev));
  FABER_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  unsigned char* base = static_attn_scratch(dev);
  // the partial block of one split: every query head's (max, sum, context)
  const size_t per_split = (size_t)n_heads * (head_dim + 2) * sizeof(float);
  const int cap = (int)(kStaticAttnPartBytes / per_split);  // >= 31 within the limits above
  const int splits = std::min(attention_splits(sms, (int)n_kv_heads, (int)n_kv), cap);
  StepState* st = reinterpret_cast<StepState*>(base + kStaticAttnStateOff);
  int32_t* counters = reinterpret_cast<int32_t*>(base + kStaticAttnCountersOff);
  static_attn_open_kernel<<<1, 128, 0, stream>>>(st, counters, (int)n_kv_heads, (int)(n_kv - 1));
  FABER_CUDA(cudaGetLastError());
  AttnArgs a = {};
  a.q = q;
  a.k = static_cast<const __half*>(k_cache);
  a.v = static_cast<const __half*>(v_cache);
  a.ctx = ctx;
  a.part = reinterpret_cast<float*>(base + kStaticAttnPartOff);
  a.counters = counters;
  a.st = st;
  a.n_heads = (int32_t)n_heads;
  a.n_kv_heads = (int32_t)n_kv_heads;
  a.head_dim = (int32_t)head_dim;
  a.max_splits = splits;
  a.scale = 1.0f / sqrtf((float)head_dim);
  const dim3 grid(n_kv_heads, splits);
  if (head_dim == 128)
    launch_attention<128>(a, grid, stream, false);
  else
    launch_attention<64>(a, grid, stream, false);
}

}  // namespace faber

extern "C" {

// Not wrapped in the shared guard, whose fault-injection lookup builds a
// std::string key: the success path allocates neither device nor host memory.
__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_attention_decode_static(
    const float* q, const void* k_cache, const void* v_cache, float* ctx, uint32_t n_heads,
    uint32_t n_kv_heads, uint32_t head_dim, uint64_t n_kv, void* stream) {
  try {
    attention_decode_static(q, k_cache, v_cache, ctx, n_heads, n_kv_heads, head_dim, n_kv,
                            as_stream(stream));
    return status(FABER_STATUS_OK);
  } catch (const Error& e) {
    g_last_error = std::string("faber_gpu_v2_attention_decode_static: ") + e.what();
    return status(e.code);
  } catch (const std::exception& e) {
    g_last_error = std::string("faber_gpu_v2_attention_decode_static: ") + e.what();
    return status(FABER_STATUS_PANIC);
  } catch (...) {
    g_last_error = "faber_gpu_v2_attention_decode_static: unknown exception";
    return status(FABER_STATUS_PANIC);
  }
}


// ---- GGUF v3 reader ---------------------------------------------------------
struct FaberGguf {
  faber::GgufFile f;
};

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_gguf_parse(const uint8_t* bytes,
                                                                              uint64_t len,
                                                                              FaberGguf** out) {
  return guarded("faber_gpu_v2_gguf_parse", [&] {
    FABER_ARG(out != nullptr && (bytes != nullptr || len == 0), "null pointer");
    *out = nullptr;
    auto g = std::make_unique<FaberGguf>();
    g->f = gguf_parse(bytes, len);
    *out = g.release();
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_gguf_info(
    const FaberGguf* g, uint32_t* version, uint64_t* n_kv, uint64_t* n_tensors, uint64_t* data_offset,
    uint64_t* alignment) {
  return guarded("faber_gpu_v2_gguf_info", [&] {
    FABER_ARG(g, "null reader");
    if (version) *version = g->f.version;
    if (n_kv) *n_kv = g->f.kv.size();
    if (n_tensors) *n_tensors = g->f.tensors.size();
    if (data_offset) *data_offset = g->f.data_offset;
    if (alignment) *alignment = g->f.alignment;
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_gguf_tensor(const FaberGguf* g,
                                                                               uint64_t index,
                                                                               FaberGgufTensorV1* out) {
  return guarded("faber_gpu_v2_gguf_tensor", [&] {
    FABER_ARG(g && out, "null pointer");
    FABER_ARG(index < g->f.tensors.size(), "tensor index out of range");
    const GgufTensor& t = g->f.tensors[index];
    FABER_ARG(t.name.size() < sizeof(out->name), "tensor name longer than the descriptor holds");
    std::memset(out, 0, sizeof(*out));
    std::memcpy(out->name, t.name.data(), t.name.size());
    out->ggml_type = t.type;
    out->n_dims = t.n_dims;
    for (uint32_t d = 0; d < 4; ++d) out->dims[d] = t.dims[d];
    out->elements = t.elements;
    out->nbytes = t.nbytes;
    out->offset = t.offset;
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_gguf_kv(
    const FaberGguf* g, uint64_t index, char* key, uint64_t key_cap, uint32_t* type, uint32_t* arr_type,
    uint64_t* arr_count) {
  return guarded("faber_gpu_v2_gguf_kv", [&] {
    FABER_ARG(g && key && key_cap > 0, "null pointer");
    FABER_ARG(index < g->f.kv.size(), "KV index out of range");
    const GgufKv& kv = g->f.kv[index];
    require(kv.key.size() < key_cap, FABER_STATUS_IO_ERROR, "key buffer too small");
    std::memcpy(key, kv.key.data(), kv.key.size());
    key[kv.key.size()] = 0;
    if (type) *type = kv.type;
    if (arr_type) *arr_type = kv.arr_type;
    if (arr_count) *arr_count = kv.arr_count;
  });
}

// Scalar lookups by key: any integer type (and BOOL) as int64, F32/F64 as
// double, STRING into buf. A missing key or another type is INVALID_ARGUMENT.
__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_gguf_get_int(const FaberGguf* g,
                                                                                const char* key,
                                                                                int64_t* v) {
  return guarded("faber_gpu_v2_gguf_get_int", [&] {
    FABER_ARG(g && key && v, "null pointer");
    const GgufKv* kv = g->f.find(key);
    FABER_ARG(kv != nullptr, std::string("no metadata key ") + key);
    FABER_ARG(kv->type != GGUF_STRING && kv->type != GGUF_ARRAY && kv->type != GGUF_F32 &&
                  kv->type != GGUF_F64,
              std::string(key) + " is not an integer");
    FABER_ARG(kv->type != GGUF_U64 || kv->u <= (uint64_t)INT64_MAX, std::string(key) + " exceeds int64");
    *v = kv->i;
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_gguf_get_float(const FaberGguf* g,
                                                                                  const char* key,
                                                                                  double* v) {
  return guarded("faber_gpu_v2_gguf_get_float", [&] {
    FABER_ARG(g && key && v, "null pointer");
    const GgufKv* kv = g->f.find(key);
    FABER_ARG(kv != nullptr, std::string("no metadata key ") + key);
    FABER_ARG(kv->type == GGUF_F32 || kv->type == GGUF_F64, std::string(key) + " is not a float");
    *v = kv->f;
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_gguf_get_string(
    const FaberGguf* g, const char* key, char* buf, uint64_t cap, uint64_t* len) {
  return guarded("faber_gpu_v2_gguf_get_string", [&] {
    FABER_ARG(g && key && len, "null pointer");
    const GgufKv* kv = g->f.find(key);
    FABER_ARG(kv != nullptr, std::string("no metadata key ") + key);
    FABER_ARG(kv->type == GGUF_STRING, std::string(key) + " is not a string");
    *len = kv->s.size();
    require(buf != nullptr && kv->s.size() < cap, FABER_STATUS_IO_ERROR, "string buffer too small");
    std::memcpy(buf, kv->s.data(), kv->s.size());
    buf[kv->s.size()] = 0;
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_gguf_free(FaberGguf* g) {
  return guarded("faber_gpu_v2_gguf_free", [&] { delete g; });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_gguf_kv_payload(const FaberGguf* g,
                                                                                    uint64_t index,
                                                                                    uint64_t* offset) {
  return guarded("faber_gpu_v2_gguf_kv_payload", [&] {
    FABER_ARG(g && offset, "null pointer");
    FABER_ARG(index < g->f.kv.size(), "KV index out of range");
    FABER_ARG(g->f.kv[index].type == GGUF_ARRAY, g->f.kv[index].key + " is not an array");
    *offset = g->f.kv[index].payload;
  });
}

// --- tokenizer (src/tokenizer/mod.rs) ----------------------------------------
struct FaberTokenizer {
  faber::tok::Tokenizer t;
};

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_tokenizer_create(
    const FaberTokenizerFactsV1* f, FaberTokenizer** out) {
  return guarded("faber_gpu_v2_tokenizer_create", [&] {
    FABER_ARG(f && out && f->model && f->pre, "null pointer");
    *out = nullptr;
    FABER_ARG((f->tokens && f->token_lens) || !f->n_tokens, "null token arrays");
    FABER_ARG(f->token_types || !f->n_token_types, "null token types");
    FABER_ARG((f->merges && f->merge_lens) || !f->n_merges, "null merge arrays");
    faber::tok::Facts facts;
    facts.model = f->model;
    facts.pre = f->pre;
    facts.tokens.reserve(f->n_tokens);
    for (uint64_t i = 0; i < f->n_tokens; ++i) {
      FABER_ARG(f->tokens[i] || !f->token_lens[i], "null token text");
      facts.tokens.emplace_back(f->tokens[i] ? f->tokens[i] : "", f->token_lens[i]);
    }
    facts.token_types.assign(f->token_types, f->token_types + f->n_token_types);
    facts.merges.reserve(f->n_merges);
    for (uint64_t i = 0; i < f->n_merges; ++i) {
      FABER_ARG(f->merges[i] || !f->merge_lens[i], "null merge text");
      facts.merges.emplace_back(f->merges[i] ? f->merges[i] : "", f->merge_lens[i]);
    }
    facts.scores_present = f->scores_present != 0;
    facts.bos = f->bos_token_id;
    facts.eos = f->eos_token_id;
    facts.pad = f->pad_token_id;
    facts.unk = f->unk_token_id;
    facts.add_bos = f->add_bos_token != 0;
    facts.add_space_prefix = f->add_space_prefix != 0;
    facts.expected_vocab = f->expected_vocab;
    facts.expected_merges = f->expected_merges;
    *out = new FaberTokenizer{faber::tok::Tokenizer(facts)};
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_tokenizer_encode(
    const FaberTokenizer* t, const uint8_t* text, uint64_t len, int32_t parse_special, uint32_t* ids,
    uint64_t cap, uint64_t* n_ids) {
  return guarded("faber_gpu_v2_tokenizer_encode", [&] {
    FABER_ARG(t && n_ids && (text || !len), "null pointer");
    FABER_ARG(len <= faber::tok::kMaxInputBytes,
              "InputTooLarge: encode input " + std::to_string(len) + " bytes exceeds 1 MiB");
    const std::vector<uint32_t> v =
        t->t.encode(std::string(reinterpret_cast<const char*>(text), (size_t)len), parse_special != 0);
    *n_ids = v.size();
    require(ids != nullptr && cap >= v.size(), FABER_STATUS_IO_ERROR,
            "encoding needs " + std::to_string(v.size()) + " ids");
    std::copy(v.begin(), v.end(), ids);
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_tokenizer_decode(
    const FaberTokenizer* t, const uint32_t* ids, uint64_t n, uint8_t* out, uint64_t cap, uint64_t* n_out) {
  return guarded("faber_gpu_v2_tokenizer_decode", [&] {
    FABER_ARG(t && n_out && (ids || !n), "null pointer");
    const std::string s = t->t.decode(std::vector<uint32_t>(ids, ids + n));
    *n_out = s.size();
    require(out != nullptr && cap >= s.size(), FABER_STATUS_IO_ERROR,
            "decoding needs " + std::to_string(s.size()) + " bytes");
    std::memcpy(out, s.data(), s.size());
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_tokenizer_info(
    const FaberTokenizer* t, uint64_t* vocab, uint32_t special_ids[4], uint32_t* eog, uint64_t eog_cap,
    uint64_t* n_eog) {
  return guarded("faber_gpu_v2_tokenizer_info", [&] {
    FABER_ARG(t && vocab && special_ids && n_eog, "null pointer");
    *vocab = t->t.vocab_size();
    special_ids[0] = t->t.bos();
    special_ids[1] = t->t.eos();
    special_ids[2] = t->t.pad();
    special_ids[3] = t->t.unk();
    const auto& e = t->t.eog();
    *n_eog = e.size();
    require(eog != nullptr && eog_cap >= e.size(), FABER_STATUS_IO_ERROR,
            "end-of-generation set has " + std::to_string(e.size()) + " ids");
    std::copy(e.begin(), e.end(), eog);
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_tokenizer_free(FaberTokenizer* t) {
  return guarded("faber_gpu_v2_tokenizer_free", [&] { delete t; });
}

// --- execution transaction (src/execution_transaction/transaction.rs) ------
struct FaberTxn {
  faber::txn::Transaction t;
  faber::txn::Outcome last;
};

struct FaberTxnBackend {
  faber::txn::FaultBackend b;
};

namespace {

faber::txn::Op txn_op(const FaberTxnOpV1& o) {
  FABER_ARG(o.kind <= FABER_TXN_BARRIER, "unknown operation kind " + std::to_string(o.kind));
  FABER_ARG(o.partition < 64 && o.destination < 64, "partition ordinal above 63");
  faber::txn::Op op;
  op.kind = (faber::txn::OpKind)o.kind;
  op.partition = o.partition;
  op.destination = o.kind == FABER_TXN_TRANSFER ? o.destination : 0;
  op.participants = (o.kind == FABER_TXN_BROADCAST || o.kind == FABER_TXN_BARRIER) ? o.participants : 0;
  op.ref = o.ref;
  op.bytes = o.kind == FABER_TXN_BARRIER ? 0 : o.bytes;
  if (o.kind == FABER_TXN_BROADCAST)
    FABER_ARG(o.participants >> o.partition & 1, "a broadcast's source must participate");
  if (o.kind == FABER_TXN_BARRIER) FABER_ARG(o.participants != 0, "a barrier needs participants");
  return op;
}

// Records a lifecycle outcome on the transaction and turns a failure into
// its status code.
void txn_finish(FaberTxn* t, const faber::txn::Outcome& o) {
  using namespace faber::txn;
  t->last = o;
  if (o.ok()) return;
  int code = FABER_STATUS_INVALID_ARGUMENT;
  if (o.kind == kTxnReservationExceedsBudget) code = FABER_STATUS_BUDGET_EXCEEDED;
  if (o.kind == kTxnBoundaryNotReached) code = FABER_STATUS_FALLIBLE;
  if (o.kind == kTxnBackend || o.kind == kTxnPublishFailed) {
    switch (o.backend.cls) {
      case ErrClass::Allocation: code = FABER_STATUS_ALLOCATION; break;
      case ErrClass::Operation: code = FABER_STATUS_KERNEL_ERROR; break;
      case ErrClass::DeviceLoss: code = FABER_STATUS_DEVICE_LOSS; break;
      case ErrClass::Cancelled: code = FABER_STATUS_CANCELLED; break;
      case ErrClass::Timeout: code = FABER_STATUS_TIMEOUT; break;
    }
  }
  throw Error(code, o.message);
}

}  // namespace

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_txn_create(
    const FaberTxnPartitionV1* partitions, uint32_t n_partitions, const FaberTxnOpV1* ops, uint32_t n_ops,
    const uint64_t* boundary_barriers, uint32_t n_barriers, const uint64_t* boundary_launches,
    uint32_t n_launches, FaberTxn** out) {
  return guarded("faber_gpu_v2_txn_create", [&] {
    FABER_ARG(out != nullptr, "null output");
    *out = nullptr;
    FABER_ARG((partitions || !n_partitions) && (ops || !n_ops) && (boundary_barriers || !n_barriers) &&
                  (boundary_launches || !n_launches),
              "null array with a nonzero count");
    std::map<uint32_t, faber::txn::BoundPartition> plan;
    for (uint32_t i = 0; i < n_partitions; ++i) {
      FABER_ARG(partitions[i].partition < 64, "partition ordinal above 63");
      FABER_ARG(!plan.count(partitions[i].partition), "partition bound twice");
      plan[partitions[i].partition] = {partitions[i].admitted != 0, partitions[i].ledger};
    }
    std::vector<faber::txn::Op> v;
    for (uint32_t i = 0; i < n_ops; ++i) v.push_back(txn_op(ops[i]));
    auto t = std::make_unique<FaberTxn>();
    const faber::txn::Outcome o = faber::txn::Transaction::create(
        std::move(plan), std::move(v), std::vector<uint64_t>(boundary_barriers, boundary_barriers + n_barriers),
        std::vector<uint64_t>(boundary_launches, boundary_launches + n_launches), t->t);
    if (!o.ok()) throw Error(FABER_STATUS_INVALID_ARGUMENT, o.message);
    *out = t.release();
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_txn_prepare(FaberTxn* t, FaberTxnBackend* b) {
  return guarded("faber_gpu_v2_txn_prepare", [&] {
    FABER_ARG(t && b, "null pointer");
    txn_finish(t, t->t.prepare(b->b));
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_txn_execute(FaberTxn* t, FaberTxnBackend* b) {
  return guarded("faber_gpu_v2_txn_execute", [&] {
    FABER_ARG(t && b, "null pointer");
    txn_finish(t, t->t.execute(b->b));
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_txn_execute_operation(
    FaberTxn* t, FaberTxnBackend* b, const FaberTxnOpV1* op) {
  return guarded("faber_gpu_v2_txn_execute_operation", [&] {
    FABER_ARG(t && b && op, "null pointer");
    txn_finish(t, t->t.execute_operation(b->b, txn_op(*op)));
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_txn_commit(FaberTxn* t, FaberTxnBackend* b,
                                                                               uint64_t publication_ordinal) {
  return guarded("faber_gpu_v2_txn_commit", [&] {
    FABER_ARG(t && b, "null pointer");
    txn_finish(t, t->t.commit(b->b, publication_ordinal));
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_txn_abort(FaberTxn* t, FaberTxnBackend* b,
                                                                              const char* reason) {
  return guarded("faber_gpu_v2_txn_abort", [&] {
    FABER_ARG(t && b, "null pointer");
    txn_finish(t, t->t.abort(b->b, reason ? reason : ""));
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_txn_receipt(const FaberTxn* t,
                                                                                FaberTxnReceiptV1* out) {
  return guarded("faber_gpu_v2_txn_receipt", [&] {
    FABER_ARG(t && out, "null pointer");
    t->t.receipt(*out);
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_txn_last_error(const FaberTxn* t,
                                                                                   FaberTxnErrorV1* out) {
  return guarded("faber_gpu_v2_txn_last_error", [&] {
    FABER_ARG(t && out, "null pointer");
    const bool be = t->last.kind == faber::txn::kTxnBackend || t->last.kind == faber::txn::kTxnPublishFailed;
    out->kind = t->last.kind;
    out->partition = t->last.partition;
    out->backend_class = be ? (int32_t)t->last.backend.cls : 0;
    out->budget_class = t->last.budget_class;
    out->missing = t->last.missing;
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_txn_reservation(const FaberTxn* t,
                                                                                    uint32_t partition,
                                                                                    uint64_t out[4]) {
  return guarded("faber_gpu_v2_txn_reservation", [&] {
    FABER_ARG(t && out, "null pointer");
    const auto& r = t->t.reservation();
    auto it = r.find(partition);
    FABER_ARG(it != r.end(), "no reservation for partition " + std::to_string(partition));
    out[0] = it->second.staging;
    out[1] = it->second.output;
    out[2] = it->second.events;
    out[3] = it->second.scratch;
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_txn_free(FaberTxn* t) {
  return guarded("faber_gpu_v2_txn_free", [&] { delete t; });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_txn_backend_fake(FaberTxnBackend** out) {
  return guarded("faber_gpu_v2_txn_backend_fake", [&] {
    FABER_ARG(out != nullptr, "null output");
    *out = new FaberTxnBackend();
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_txn_backend_inject(
    FaberTxnBackend* b, uint32_t op_kind, uint64_t ref, uint32_t partition, int32_t fault_class) {
  return guarded("faber_gpu_v2_txn_backend_inject", [&] {
    FABER_ARG(b != nullptr, "null backend");
    FABER_ARG(op_kind <= FABER_TXN_BARRIER && partition < 64, "bad operation kind or partition");
    FABER_ARG(fault_class >= 1 && fault_class <= 5, "fault class must be 1-5");
    b->b.faults.push_back({{op_kind, ref}, partition, (faber::txn::FaultClass)fault_class});
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_txn_backend_fail_publish(
    FaberTxnBackend* b, int32_t backend_class) {
  return guarded("faber_gpu_v2_txn_backend_fail_publish", [&] {
    FABER_ARG(b != nullptr, "null backend");
    FABER_ARG(backend_class >= 1 && backend_class <= 5, "backend error class must be 1-5");
    b->b.fail_publish = (faber::txn::ErrClass)backend_class;
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_txn_backend_set_auto_complete(
    FaberTxnBackend* b, int32_t on) {
  return guarded("faber_gpu_v2_txn_backend_set_auto_complete", [&] {
    FABER_ARG(b != nullptr, "null backend");
    b->b.inner.auto_complete = on != 0;
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_txn_backend_complete_event(
    FaberTxnBackend* b, uint32_t op_kind, uint32_t partition, uint64_t ref) {
  return guarded("faber_gpu_v2_txn_backend_complete_event", [&] {
    FABER_ARG(b != nullptr, "null backend");
    FABER_ARG(op_kind <= FABER_TXN_BARRIER && partition < 64, "bad operation kind or partition");
    b->b.inner.complete_event({op_kind, partition, ref});
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_txn_backend_info(const FaberTxnBackend* b,
                                                                                     FaberTxnBackendInfoV1* out) {
  return guarded("faber_gpu_v2_txn_backend_info", [&] {
    FABER_ARG(b && out, "null pointer");
    const auto& in = b->b.inner;
    *out = FaberTxnBackendInfoV1{};
    for (const auto& kv : in.reservations) out->reserved_partitions |= 1ull << kv.first;
    for (uint32_t p : in.released) out->released_partitions |= 1ull << p;
    for (uint32_t p : in.retired) out->retired_partitions |= 1ull << p;
    out->staged_bytes = in.staged_total;
    out->published_bytes = in.published_total;
    out->committed_bytes = b->b.committed_total;
    out->executed_operations = in.executed.size();
    uint64_t pending = 0;
    for (const auto& e : in.dispatched)
      if (!in.completed.count(e)) ++pending;
    out->pending_events = pending;
    out->delivered_faults = b->b.delivered.size();
    for (const auto& d : b->b.delivered) out->reclaimed_copy_bytes += d.reclaimed_copy_bytes;
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_txn_backend_free(FaberTxnBackend* b) {
  return guarded("faber_gpu_v2_txn_backend_free", [&] { delete b; });
}

// --- partition budget (src/partition.rs:111-155, 293-315) ------------------
__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_partition_admit(
    const FaberPartitionLedgerV1* declared, uint64_t safe_limit_bytes, uint64_t* total_out) {
  return guarded("faber_gpu_v2_partition_admit", [&] {
    FABER_ARG(declared != nullptr && total_out != nullptr, "null ledger or output");
    const uint64_t cls[kLedgerClasses] = {
        declared->weight_bytes,           declared->kv_cache_bytes,
        declared->activation_scratch_bytes, declared->module_storage_bytes,
        declared->allocator_overhead_bytes, declared->transfer_staging_bytes,
        declared->concurrent_state_bytes};
    // PartitionBudgetLedger::total_bytes: checked sum, overflow fails closed
    uint64_t total = 0;
    bool overflow = false;
    for (uint64_t v : cls) {
      if (v > UINT64_MAX - total) {
        overflow = true;
        break;
      }
      total += v;
    }
    *total_out = overflow ? UINT64_MAX : total;
    require(!overflow, FABER_STATUS_BUDGET_EXCEEDED, "declared ledger overflows u64");
    require(total <= safe_limit_bytes, FABER_STATUS_BUDGET_EXCEEDED,
            "declared " + std::to_string(total) + " bytes exceed the " +
                std::to_string(safe_limit_bytes) + "-byte safe limit");
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_partition_usage(
    int32_t device, FaberPartitionLedgerV1* out) {
  return guarded("faber_gpu_v2_partition_usage", [&] {
    FABER_ARG(out != nullptr, "null output");
    FABER_ARG(device >= 0 && device < kLedgerMaxDevices, "device ordinal outside 0-63");
    std::lock_guard<std::mutex> g(g_ledger_mu);
    const DeviceLedger& L = g_ledger[device];
    out->weight_bytes = L.live[kLedgerWeights];
    out->kv_cache_bytes = L.live[kLedgerKv];
    out->activation_scratch_bytes = L.live[kLedgerActivation];
    out->module_storage_bytes = L.live[kLedgerModule];
    out->allocator_overhead_bytes = L.live[kLedgerOverhead];
    out->transfer_staging_bytes = L.live[kLedgerStaging];
    out->concurrent_state_bytes = L.live[kLedgerConcurrent];
  });
}

__attribute__((visibility("default"))) FaberRtStatusV1 faber_gpu_v2_partition_set_limit(
    int32_t device, uint64_t safe_limit_bytes) {
  return guarded("faber_gpu_v2_partition_set_limit", [&] {
    FABER_ARG(device >= 0 && device < kLedgerMaxDevices, "device ordinal outside 0-63");
    std::lock_guard<std::mutex> g(g_ledger_mu);
    DeviceLedger& L = g_ledger[device];
    const uint64_t held = ledger_total(L);
    require(safe_limit_bytes == 0 || held <= safe_limit_bytes, FABER_STATUS_BUDGET_EXCEEDED,
            "device " + std::to_string(device) + " already holds " + std::to_string(held) + " bytes");
    L.limit = safe_limit_bytes;
  });
}

}  // extern "C"
