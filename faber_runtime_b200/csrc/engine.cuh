// engine.cuh — model + session: the device analogue of CpuOracle / ForwardRun
// / run_greedy (src/cpu_oracle.rs:409-445, 808-926; src/greedy_run.rs:186-248)
// under the session contract of src/session.rs.
//
// One decode step ("push") is, per layer:
//   QKV GEMV  [rms_norm(attn_norm) prologue | RoPE + f16 KV append epilogue]
//   attention [split-K over positions, last CTA merges]
//   O GEMV    [residual epilogue]            (TP: store + NCCL all-reduce)
//   GATEUP    [rms_norm(ffn_norm) prologue | SwiGLU epilogue]
//   DOWN GEMV [residual epilogue]            (TP: store + NCCL all-reduce)
// and "logits" is the head GEMV [rms_norm(output_norm) | logits + argmax]
// plus a one-thread finalize. Both are captured once per session as CUDA
// graphs (positions and tokens live in device memory), with programmatic
// dependent launch so each kernel's weight loads overlap its predecessor.
#pragma once

#include <nccl.h>

#include <cmath>
#include <map>
#include <string>
#include <vector>

#include "attention.cuh"
#include "bgemv.cuh"
#include "prefill.cuh"
#include "attention_stream.cuh"

namespace faber {

// f32 -> f16 (RN-even) on the host; finite inputs and overflow to inf.
inline uint16_t host_f32_to_f16(float x) {
  uint32_t b;
  std::memcpy(&b, &x, 4);
  const uint32_t sign = (b >> 16) & 0x8000u;
  const uint32_t a = b & 0x7fffffffu;
  if (a > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);  // NaN
  if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
  if (a >= 0x38800000u) {
    const uint32_t e = (a >> 23) - 112u;
    const uint32_t mant = a & 0x7fffffu;
    uint32_t h = (e << 10) | (mant >> 13);
    const uint32_t rest = mant & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
  }
  float f;
  std::memcpy(&f, &a, 4);
  const double scaled = (double)f * 16777216.0;
  double fl = std::floor(scaled);
  const double fr = scaled - fl;
  if (fr > 0.5 || (fr == 0.5 && std::fmod(fl, 2.0) != 0.0)) fl += 1.0;
  return (uint16_t)(sign | (uint32_t)fl);
}

inline float host_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  uint32_t b;
  if (e == 0) {
    if (m == 0) {
      b = sign;
    } else {
      int p = 31 - __builtin_clz(m);  // leading bit position
      b = sign | ((uint32_t)(p + 103) << 23) | ((m << (23 - p)) & 0x7fffffu);
    }
  } else if (e == 31) {
    b = sign | 0x7f800000u | (m << 13);
  } else {
    b = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}

inline float host_f16_round(float x) { return host_f16_to_f32(host_f32_to_f16(x)); }

#define FABER_NCCL(expr)                                                                   \
  do {                                                                                     \
    ncclResult_t r_ = (expr);                                                              \
    if (r_ != ncclSuccess)                                                                 \
      throw ::faber::Error(FABER_STATUS_IO_ERROR,                                          \
                           std::string(#expr) + " failed: " + ncclGetErrorString(r_));     \
  } while (0)

struct HostTensor {
  uint32_t type = 0;
  std::vector<uint8_t> bytes;  // this rank's shard, native layout
  uint64_t rows = 0, cols = 0; // shard shape
  bool set = false;
};

enum LayerSlot { LS_ATTN_NORM, LS_Q, LS_K, LS_V, LS_O, LS_FFN_NORM, LS_GATE, LS_UP, LS_DOWN, LS_N };
static const char* kLayerSlotNames[LS_N] = {"attn_norm", "attn_q", "attn_k", "attn_v",
                                            "attn_output", "ffn_norm", "ffn_gate", "ffn_up",
                                            "ffn_down"};

struct LayerDev {
  DeviceTiled qkv, o, gateup, down;
  // the same linears as typed rows when a part is not Q4_K (valid() then)
  DeviceRows qkv_r, o_r, gateup_r, down_r;
  DevBuf attn_norm, ffn_norm;
};

struct ModelState {
  FaberModelConfigV1 cfg{};
  int tp = 1, rank = 0;
  // local (per-rank) sizes
  int Hl = 0, Hkvl = 0, Fl = 0, Vl = 0, v0 = 0;
  int f_blk0 = 0, f_blk1 = 0;  // this rank's FFN super-block range
  std::vector<std::array<HostTensor, LS_N>> staged;
  HostTensor st_embd, st_out_norm, st_output;
  bool finalized = false;
  std::vector<LayerDev> layers;
  DevBuf embd_f16;   // [V][d] f16 (f16-rounded token_embd)
  DevBuf out_norm;   // [d] f32, not rounded
  DeviceTiled head;  // untied Q4_K head, local vocab rows
  DeviceRows head_r; // ... as typed rows when it is not Q4_K
  bool all_q4k = true;  // every linear in the Q4_K tile layout
  ncclComm_t comm = nullptr;
  int device = 0;
  uint64_t device_bytes = 0;
  ~ModelState() {
    if (comm) ncclCommDestroy(comm);
  }
};

}  // namespace faber

struct FaberGpuModel {
  faber::ModelState s;
};

namespace faber {

struct SessionState {
  FaberGpuModel* m = nullptr;
  FaberKvLayoutV1 kv{};
  int max_ctx = 0;
  int max_splits = 0;
  int device = 0;
  cudaStream_t stream = nullptr;
  DevBuf kcache, vcache;  // [L][ctx][Hkvl*hd] f16
  DevBuf rope;            // [ctx][hd/2] float2
  DevBuf h, h2, q, ctx, hh, logits, logits_full, opart, dpart;
  DevBuf attn_part, attn_counters;
  // Tensor-parallel exchange: [2][tp][d] epoch-tagged partials (O, down), 8
  // bytes each, then the consumers' grid-barrier words. Every rank maps every
  // other rank's buffer (CUDA IPC) and stores its partials there.
  DevBuf tp_buf;
  // prompt pass scratch (allocated on first use, for up to kPrefillChunk tokens)
  DevBuf pf_h, pf_xs, pf_scale, pf_q, pf_ctx, pf_act;
  int pf_cap = 0;
  std::vector<unsigned char*> tp_base;  // rank r's buffer in this process
  DevBuf state;           // StepState
  DevBuf gen;             // int64 [max_ctx]
  DevBuf prompt;          // int64 staging for pushes
  int64_t* pinned = nullptr;  // pinned host staging
  size_t pinned_n = 0;
  uint64_t n = 0;         // host mirror of the sequence length
  bool h_valid = false;   // h holds the residual stream of position n - 1
  uint32_t peer_wait_limit = 0;  // polls before a tensor-parallel wait gives up (0: kernel default)
  bool prefix_pending = false;
  uint64_t prefix_n = 0;
  std::vector<uint8_t> prefix_layers;
  // graphs
  cudaGraphExec_t g_push = nullptr, g_logits = nullptr, g_step = nullptr;
  std::vector<int64_t> graph_eog;
  bool graphs_valid = false;
  // tracing (eager path)
  bool trace = false;
  DevBuf tr;  // [L][8][maxw] f32
  int tr_w = 0;
  // timing
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  float last_greedy_ms = 0.f;
  // commit contract (src/session.rs:422-456)
  uint32_t c_position = 0;
  uint64_t c_kv_generations = 0;
  std::vector<int64_t> c_history;

  ~SessionState() {
    int cur = -1;
    cudaGetDevice(&cur);
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    destroy_graphs();
    close_tp_exchange();
    if (pinned) cudaFreeHost(pinned);
    if (ev0) cudaEventDestroy(ev0);
    if (ev1) cudaEventDestroy(ev1);
    if (stream) cudaStreamDestroy(stream);
    if (cur >= 0) cudaSetDevice(cur);
  }
  // Peers may still be storing into this rank's buffer until every rank has
  // stopped stepping: a group barrier comes before the mappings go.
  void close_tp_exchange() {
    if (tp_base.empty()) return;
    ncclComm_t comm = m ? m->s.comm : nullptr;
    if (comm && stream) {
      ncclAllReduce(tp_buf.p, tp_buf.p, 1, ncclUint8, ncclMax, comm, stream);  // barrier
      cudaStreamSynchronize(stream);
    }
    for (size_t r = 0; r < tp_base.size(); ++r)
      if (tp_base[r] && tp_base[r] != tp_buf.p) cudaIpcCloseMemHandle(tp_base[r]);
    tp_base.clear();
  }
  void destroy_graphs() {
    if (g_push) cudaGraphExecDestroy(g_push);
    if (g_logits) cudaGraphExecDestroy(g_logits);
    if (g_step) cudaGraphExecDestroy(g_step);
    g_push = g_logits = g_step = nullptr;
    graphs_valid = false;
  }
};

}  // namespace faber

struct FaberGpuSession {
  faber::SessionState s;
};


namespace faber {

// Decode attention with the smallest compiled group size (query heads per kv
// head) that holds this model's ratio.
template <int HD>
void launch_attention(const AttnArgs& a, dim3 grid, cudaStream_t stream, bool pdl) {
  const int ratio = a.n_heads / a.n_kv_heads;
  const dim3 block(kAttnThreads);
  if (ratio <= 1)
    launch_pdl(attention_decode_kernel<HD, 1>, grid, block, 0, stream, pdl, a);
  else if (ratio <= 2)
    launch_pdl(attention_decode_kernel<HD, 2>, grid, block, 0, stream, pdl, a);
  else if (ratio <= 4)
    launch_pdl(attention_decode_kernel<HD, 4>, grid, block, 0, stream, pdl, a);
  else
    launch_pdl(attention_decode_kernel<HD, 8>, grid, block, 0, stream, pdl, a);
}

// Decode attention of a step: one or two query heads per kv head on the
// TMA-streamed tensor-core kernel (a batch through its sequences' tensor
// maps), with the split count from its wave model within the partial
// buffer's capacity grid.y; grouped heads (ratio 3..8) on the tensor-core GQA
// kernel, one wave of CTAs (kv heads x sequences x splits).
template <int HD>
void launch_decode_attention(const AttnArgs& a, dim3 grid, cudaStream_t stream, bool pdl) {
  const int ratio = a.n_heads / a.n_kv_heads;
  if (ratio <= kAsStreamMaxRatio) {
    require(a.cache_rows > 0 && (!a.slots || a.kvmaps), FABER_STATUS_UNSUPPORTED,
            "decode attention needs the cache extent (and a batch its tensor maps)");
    const int splits = attention_stream_splits(device_info().sms, (int)(grid.x * grid.z), a.cache_rows, HD, ratio,
                                               (int)grid.y);
    launch_attention_stream<HD>(a, dim3(grid.x, splits, grid.z), stream, pdl);
    return;
  }
  if (ratio > 8) {
    launch_attention<HD>(a, grid, stream, pdl);
    return;
  }
  auto kern = attention_tc_kernel<HD>;
  static thread_local std::map<int, bool> attr_done;
  int dev = 0;
  FABER_CUDA(cudaGetDevice(&dev));
  if (!attr_done[dev]) {
    FABER_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, gqa_smem_bytes<HD>()));
    attr_done[dev] = true;
  }
  const int kv = (int)(grid.x * grid.z);
  const int want = std::max(1, kGqaCtasPerSm * device_info().sms / kv);
  const dim3 g(grid.x, std::min((int)grid.y, want), grid.z);
  launch_pdl(kern, g, dim3(128), gqa_smem_bytes<HD>(), stream, pdl, a);
}

// ---------------------------------------------------------------------------
// Model construction
// ---------------------------------------------------------------------------
inline void validate_config(const FaberModelConfigV1& c) {
  FABER_ARG(c.n_layers > 0 && c.d_model > 0 && c.n_heads > 0 && c.n_kv_heads > 0 &&
                c.head_dim > 0 && c.ffn > 0 && c.vocab > 0,
            "zero-sized model dimension");
  FABER_ARG(c.n_heads % c.n_kv_heads == 0, "n_heads must be a multiple of n_kv_heads");
  require(c.head_dim == 64 || c.head_dim == 128, FABER_STATUS_UNSUPPORTED, "head_dim must be 64 or 128");
  require(c.n_heads / c.n_kv_heads <= (uint32_t)kAttnMaxRatio, FABER_STATUS_UNSUPPORTED,
          "GQA ratio above 8");
  require(c.d_model % 256 == 0, FABER_STATUS_UNSUPPORTED, "d_model must be a multiple of 256");
  require(c.ffn % 32 == 0, FABER_STATUS_UNSUPPORTED, "ffn must be a multiple of 32");
  FABER_ARG(c.tp_size >= 1 && c.tp_rank < c.tp_size, "bad tensor-parallel rank");
  require(c.tp_size <= (uint32_t)kMaxTp, FABER_STATUS_UNSUPPORTED,
          "at most " + std::to_string(kMaxTp) + " tensor-parallel ranks");
  if (c.tp_size > 1) {
    require(c.n_heads % c.tp_size == 0 && c.n_kv_heads % c.tp_size == 0, FABER_STATUS_UNSUPPORTED,
            "heads must divide evenly across tensor-parallel ranks");
    require(c.ffn % 256 == 0 && c.ffn / 256 >= c.tp_size, FABER_STATUS_UNSUPPORTED,
            "ffn must be whole super-blocks, at least one per rank");
  }
}

// Tensor-parallel plan of one rank: Q/K/V split by head, gate/up by FFN
// super-block and the head by vocab rows (column-parallel); O and down by the
// matching input columns (row-parallel, summed by an all-reduce). Embedding
// and norms are replicated. Host-only: the same plan serves model upload and
// the CPU tests of the sharding.
struct TpPlan {
  int Hl = 0, Hkvl = 0, Fl = 0, Vl = 0, v0 = 0, f_blk0 = 0, f_blk1 = 0;
};

inline TpPlan tp_plan(const FaberModelConfigV1& c) {
  TpPlan P;
  const int tp = (int)c.tp_size, rank = (int)c.tp_rank;
  P.Hl = (int)(c.n_heads / c.tp_size);
  P.Hkvl = (int)(c.n_kv_heads / c.tp_size);
  if (tp == 1) {
    P.Fl = (int)c.ffn;
    P.f_blk0 = 0;
    P.f_blk1 = (int)((c.ffn + 255) / 256);
  } else {
    const int nF = (int)(c.ffn / 256);
    P.f_blk0 = rank * nF / tp;
    P.f_blk1 = (rank + 1) * nF / tp;
    P.Fl = (P.f_blk1 - P.f_blk0) * 256;
  }
  P.v0 = (int)((uint64_t)rank * c.vocab / tp);
  P.Vl = (int)((uint64_t)(rank + 1) * c.vocab / tp) - P.v0;
  return P;
}

// Device buffer sizes of one session (session_open's allocations), from the
// rank's local dimensions. Host-only: the session and the partition plan use
// the same formulas.
struct SessionSizes {
  int max_splits = 0;
  uint64_t cache = 0;          // each of K and V: [L][ctx][Hkvl*hd] f16
  uint64_t rope = 0;           // [ctx][hd/2] (cos, sin)
  uint64_t vec_d = 0;          // each of h, h2, opart, dpart: [d] f32
  uint64_t vec_q = 0;          // each of q, ctx: [Hl*hd] f32
  uint64_t hh = 0;             // [Fl] f32
  uint64_t logits = 0;         // [Vl] f32
  uint64_t logits_full = 0;    // [V] f32 under tensor parallelism
  uint64_t attn_part = 0;      // [Hl][splits][hd+2] f32
  uint64_t attn_counters = 0;  // [Hkvl] i32
  uint64_t state = 0, gen = 0, prompt = 0;
  uint64_t tp_buf = 0;         // exchange partials and barrier words
};

inline SessionSizes session_sizes(const FaberModelConfigV1& c, int Hl, int Hkvl, int Fl, int Vl,
                                  int max_ctx, int sms) {
  SessionSizes z;
  const uint64_t hd = c.head_dim, d = c.d_model, ctx = (uint64_t)max_ctx, tp = c.tp_size;
  z.max_splits = attention_splits(sms, Hkvl, max_ctx);
  z.cache = (uint64_t)c.n_layers * ctx * ((uint64_t)Hkvl * hd) * 2;
  z.rope = ctx * (hd / 2) * sizeof(float2);
  z.vec_d = d * 4;
  z.vec_q = (uint64_t)Hl * hd * 4;
  z.hh = (uint64_t)Fl * 4;
  z.logits = (uint64_t)Vl * 4;
  z.logits_full = tp > 1 ? (uint64_t)c.vocab * 4 : 0;
  z.attn_part = (uint64_t)Hl * (uint64_t)z.max_splits * (hd + 2) * 4;
  z.attn_counters = (uint64_t)Hkvl * 4;
  z.state = sizeof(StepState);
  z.gen = ctx * 8 + 8;
  z.prompt = ctx * 8;
  // partials [2][tp][d], then 256 bytes: the grid-barrier words, and from
  // byte 64 the argmax exchange [tp][3] (key high, key low, finite flag)
  z.tp_buf = tp > 1 ? 2 * tp * d * sizeof(unsigned long long) + 256 : 0;
  return z;
}

// Prompt-pass scratch of a session for chunks of up to cap tokens.
struct PrefillSizes {
  uint64_t h, xs, scale, q, ctx, act;
};

inline PrefillSizes prefill_sizes(uint64_t d, uint64_t nq, uint64_t F, uint64_t cap) {
  const uint64_t kmax = std::max(d, std::max(nq, F));
  return {cap * d * 4, 2 * cap * kmax * 2, cap * 4, cap * nq * 4, cap * nq * 4, cap * F * 4};
}

// Full shape of a named tensor and this rank's block [r0, r0+nr) x [c0, c0+nc).
struct ShardRange {
  uint64_t rows = 0, cols = 0, r0 = 0, nr = 0, c0 = 0, nc = 0;
  bool q4k = false;  // a Q4_K linear (else an f32 vector or the embedding)
};

inline ShardRange tensor_shard(const FaberModelConfigV1& c, const TpPlan& P,
                               const std::string& name) {
  const uint64_t d = c.d_model, hd = c.head_dim, H = c.n_heads, Hkv = c.n_kv_heads, F = c.ffn;
  const uint64_t rank = c.tp_rank;
  auto full = [](uint64_t r, uint64_t k, bool q) {
    ShardRange s;
    s.rows = r;
    s.cols = k;
    s.nr = r;
    s.nc = k;
    s.q4k = q;
    return s;
  };
  auto block = [](uint64_t r, uint64_t k, uint64_t r0, uint64_t nr, uint64_t c0, uint64_t nc) {
    ShardRange s;
    s.rows = r;
    s.cols = k;
    s.r0 = r0;
    s.nr = nr;
    s.c0 = c0;
    s.nc = nc;
    s.q4k = true;
    return s;
  };
  if (name == "token_embd.weight") return full(c.vocab, d, false);
  if (name == "output_norm.weight") return full(d, 1, false);
  if (name == "output.weight") {
    FABER_ARG(!c.tied_head, "output.weight given for a tied-head model");
    return block(c.vocab, d, (uint64_t)P.v0, (uint64_t)P.Vl, 0, d);
  }
  unsigned layer = 0;
  char slot[64] = {0};
  FABER_ARG(std::sscanf(name.c_str(), "blk.%u.%63[a-z_].weight", &layer, slot) == 2 &&
                layer < c.n_layers,
            "unknown tensor name " + name);
  int ls = -1;
  for (int k = 0; k < LS_N; ++k)
    if (std::string(slot) == kLayerSlotNames[k]) ls = k;
  FABER_ARG(ls >= 0, "unknown tensor name " + name);
  const uint64_t fr0 = (uint64_t)P.f_blk0 * 256, fnr = (uint64_t)(P.f_blk1 - P.f_blk0) * 256;
  switch (ls) {
    case LS_ATTN_NORM:
    case LS_FFN_NORM: return full(d, 1, false);
    case LS_Q: return block(H * hd, d, rank * P.Hl * hd, P.Hl * hd, 0, d);
    case LS_K:
    case LS_V: return block(Hkv * hd, d, rank * P.Hkvl * hd, P.Hkvl * hd, 0, d);
    case LS_O: return block(d, H * hd, 0, d, rank * P.Hl * hd, P.Hl * hd);
    case LS_GATE:
    case LS_UP: return c.tp_size == 1 ? block(F, d, 0, F, 0, d) : block(F, d, fr0, fnr, 0, d);
    default: return c.tp_size == 1 ? block(d, F, 0, d, 0, F) : block(d, F, 0, d, fr0, fnr);
  }
}

// Native block sub-tensor [r0, r0+nr) x [c0, c0+nc) of a [rows][cols] Q4_K
// tensor (c0, nc multiples of 256, cols % 256 == 0).
inline std::vector<uint8_t> q4k_shard(const uint8_t* src, uint64_t cols, uint64_t r0, uint64_t nr,
                                      uint64_t c0, uint64_t nc) {
  const uint64_t nbr = cols / 256, b0 = c0 / 256, nbl = nc / 256;
  std::vector<uint8_t> out(nr * nbl * kQ4kBlockBytes);
  for (uint64_t r = 0; r < nr; ++r)
    std::memcpy(out.data() + r * nbl * kQ4kBlockBytes,
                src + ((r0 + r) * nbr + b0) * kQ4kBlockBytes, nbl * kQ4kBlockBytes);
  return out;
}

inline void model_set_tensor(ModelState& M, const std::string& name, uint32_t type,
                             const void* data, uint64_t nbytes, uint64_t rows, uint64_t cols) {
  const FaberModelConfigV1& c = M.cfg;
  FABER_ARG(!M.finalized, "model already finalized");
  FABER_ARG(data != nullptr || nbytes == 0, "null tensor data");
  auto expect_shape = [&](uint64_t er, uint64_t ec) {
    FABER_ARG(rows == er && cols == ec, name + ": shape [" + std::to_string(rows) + "x" +
                                            std::to_string(cols) + "], expected [" +
                                            std::to_string(er) + "x" + std::to_string(ec) + "]");
  };
  auto expect_bytes = [&](uint64_t want) {
    FABER_ARG(nbytes == want, name + ": packed tensor is " + std::to_string(nbytes) +
                                  " bytes, expected exactly " + std::to_string(want));
  };
  auto f32_vec = [&](HostTensor& h, uint64_t n) {
    require(type == FABER_GGML_F32, FABER_STATUS_UNSUPPORTED, name + ": expected F32");
    expect_shape(n, 1);
    expect_bytes(n * 4);
    h.type = type;
    h.rows = n;
    h.cols = 1;
    h.bytes.assign(static_cast<const uint8_t*>(data), static_cast<const uint8_t*>(data) + nbytes);
    h.set = true;
  };
  const uint8_t* src = static_cast<const uint8_t*>(data);
  const TpPlan P = tp_plan(c);
  const ShardRange sr = tensor_shard(c, P, name);
  if (name == "token_embd.weight") {
    require(type == FABER_GGML_F32, FABER_STATUS_UNSUPPORTED, name + ": expected F32");
    expect_shape(sr.rows, sr.cols);
    expect_bytes(sr.rows * sr.cols * 4);
    M.st_embd.type = type;
    M.st_embd.rows = sr.rows;
    M.st_embd.cols = sr.cols;
    M.st_embd.bytes.assign(src, src + nbytes);
    M.st_embd.set = true;
    return;
  }
  HostTensor* h = nullptr;
  if (name == "output_norm.weight") {
    h = &M.st_out_norm;
  } else if (name == "output.weight") {
    h = &M.st_output;
  } else {
    unsigned layer = 0;
    char slot[64] = {0};
    std::sscanf(name.c_str(), "blk.%u.%63[a-z_].weight", &layer, slot);  // checked by tensor_shard
    for (int k = 0; k < LS_N; ++k)
      if (std::string(slot) == kLayerSlotNames[k]) h = &M.staged[layer][(size_t)k];
  }
  if (!sr.q4k) return f32_vec(*h, sr.rows);
  if (type != FABER_GGML_Q4_K) {
    // another admitted block type: kept whole, served by the row GEMV
    int be = 0, bb = 0;
    require(type != FABER_GGML_F32 && ggml_block_geometry(type, be, bb), FABER_STATUS_UNSUPPORTED,
            name + ": linears must be Q4_K, Q6_K, Q5_0 or Q8_0");
    require(M.tp == 1, FABER_STATUS_UNSUPPORTED,
            name + ": only Q4_K linears shard across tensor-parallel ranks");
    expect_shape(sr.rows, sr.cols);
    FABER_ARG(sr.cols % (uint64_t)be == 0, name + ": rows are not whole blocks");
    expect_bytes(sr.rows * sr.cols / be * bb);
    h->type = type;
    h->bytes.assign(src, src + nbytes);
    h->rows = sr.rows;
    h->cols = sr.cols;
    h->set = true;
    return;
  }
  // Q4_K linear: this rank's block rows [r0, r0+nr) x cols [c0, c0+nc)
  expect_shape(sr.rows, sr.cols);
  FABER_ARG((sr.rows * sr.cols) % 256 == 0, name + ": element count not a multiple of 256");
  expect_bytes(sr.rows * sr.cols / 256 * kQ4kBlockBytes);
  h->type = type;
  if (M.tp == 1) {
    h->bytes.assign(src, src + nbytes);
    h->rows = sr.rows;
    h->cols = sr.cols;
  } else {
    h->bytes = q4k_shard(src, sr.cols, sr.r0, sr.nr, sr.c0, sr.nc);
    h->rows = sr.nr;
    h->cols = sr.nc;
  }
  h->set = true;
}

inline uint64_t nblk(const HostTensor& h) { return h.rows * h.cols / 256; }

// Typed rows of a fused linear: output row j is row part_row(j) of part(j).
template <class PartOf>
inline void rows_from(DeviceRows& D, int rows, int cols, PartOf part_of) {
  const int n_tiles = (rows + kTileRows - 1) / kTileRows;
  std::vector<uint64_t> off((size_t)n_tiles * kTileRows, 0);
  std::vector<uint32_t> type((size_t)n_tiles * kTileRows, kNoRow);
  uint64_t total = 0;
  for (int j = 0; j < rows; ++j) {
    const auto pr = part_of(j);
    int be = 0, bb = 0;
    ggml_block_geometry(pr.first->type, be, bb);
    off[j] = total;
    type[j] = pr.first->type;
    total += (uint64_t)cols / be * bb;
  }
  std::vector<uint8_t> bytes(total);
  for (int j = 0; j < rows; ++j) {
    const auto pr = part_of(j);
    int be = 0, bb = 0;
    ggml_block_geometry(pr.first->type, be, bb);
    const uint64_t rb = (uint64_t)cols / be * bb;
    std::memcpy(bytes.data() + off[j], pr.first->bytes.data() + pr.second * rb, rb);
  }
  upload(D.bytes, bytes.data(), bytes.size(), kLedgerWeights);
  upload(D.row_off, off.data(), off.size() * 8, kLedgerWeights);
  upload(D.row_type, type.data(), type.size() * 4, kLedgerWeights);
  D.n_tiles = n_tiles;
  D.rows = rows;
  D.cols = cols;
}

inline void model_finalize(ModelState& M) {
  const FaberModelConfigV1& c = M.cfg;
  FABER_ARG(!M.finalized, "model already finalized");
  // coverage: every tensor present (src/cpu_oracle.rs:409-445)
  FABER_ARG(M.st_embd.set, "missing tensor token_embd.weight");
  FABER_ARG(M.st_out_norm.set, "missing tensor output_norm.weight");
  FABER_ARG(c.tied_head || M.st_output.set, "missing tensor output.weight");
  for (uint32_t l = 0; l < c.n_layers; ++l)
    for (int k = 0; k < LS_N; ++k)
      FABER_ARG(M.staged[l][(size_t)k].set,
                "missing tensor blk." + std::to_string(l) + "." + kLayerSlotNames[k] + ".weight");
  FABER_CUDA(cudaSetDevice(M.device));
  const uint64_t d = c.d_model, hd = c.head_dim;
  M.layers.resize(c.n_layers);
  uint64_t bytes = 0;
  for (uint32_t l = 0; l < c.n_layers; ++l) {
    auto& S = M.staged[l];
    LayerDev& L = M.layers[l];
    const uint64_t nq = (uint64_t)M.Hl * hd, nk = (uint64_t)M.Hkvl * hd;
    auto q4k = [&](std::initializer_list<int> slots) {
      for (int k : slots)
        if (S[(size_t)k].type != FABER_GGML_Q4_K) return false;
      return true;
    };
    // fused QKV: rows [q | k | v]
    auto qkv_part = [&](int j) {
      const HostTensor& t = (uint64_t)j < nq ? S[LS_Q] : ((uint64_t)j < nq + nk ? S[LS_K] : S[LS_V]);
      const uint64_t r = (uint64_t)j < nq ? j : ((uint64_t)j < nq + nk ? j - nq : j - nq - nk);
      return std::pair<const HostTensor*, uint64_t>(&t, r);
    };
    if (q4k({LS_Q, LS_K, LS_V}))
      L.qkv.from(repack_q4k((int)(nq + 2 * nk), (int)d, [&](int j) {
        const auto pr = qkv_part(j);
        return RowSeg{pr.first->bytes.data(), nblk(*pr.first), pr.second * d};
      }));
    else
      rows_from(L.qkv_r, (int)(nq + 2 * nk), (int)d, qkv_part);
    auto o_part = [&](int j) { return std::pair<const HostTensor*, uint64_t>(&S[LS_O], (uint64_t)j); };
    if (q4k({LS_O}))
      L.o.from(repack_q4k((int)d, (int)S[LS_O].cols, [&](int j) {
        return RowSeg{S[LS_O].bytes.data(), nblk(S[LS_O]), (uint64_t)j * S[LS_O].cols};
      }));
    else
      rows_from(L.o_r, (int)d, (int)S[LS_O].cols, o_part);
    // gate/up interleaved: row 2f = gate f, 2f+1 = up f (SwiGLU epilogue pairs)
    const uint64_t Fl = S[LS_GATE].rows;
    auto gu_part = [&](int j) {
      return std::pair<const HostTensor*, uint64_t>((j & 1) ? &S[LS_UP] : &S[LS_GATE], (uint64_t)(j >> 1));
    };
    if (q4k({LS_GATE, LS_UP}))
      L.gateup.from(repack_q4k((int)(2 * Fl), (int)d, [&](int j) {
        const auto pr = gu_part(j);
        return RowSeg{pr.first->bytes.data(), nblk(*pr.first), pr.second * d};
      }));
    else
      rows_from(L.gateup_r, (int)(2 * Fl), (int)d, gu_part);
    auto down_part = [&](int j) { return std::pair<const HostTensor*, uint64_t>(&S[LS_DOWN], (uint64_t)j); };
    if (q4k({LS_DOWN}))
      L.down.from(repack_q4k((int)d, (int)S[LS_DOWN].cols, [&](int j) {
        return RowSeg{S[LS_DOWN].bytes.data(), nblk(S[LS_DOWN]), (uint64_t)j * S[LS_DOWN].cols};
      }));
    else
      rows_from(L.down_r, (int)d, (int)S[LS_DOWN].cols, down_part);
    if (L.qkv_r.valid() || L.o_r.valid() || L.gateup_r.valid() || L.down_r.valid()) M.all_q4k = false;
    // per-layer norms are f16-rounded like every per-layer tensor
    // (src/cpu_oracle.rs:323-331)
    for (int k : {LS_ATTN_NORM, LS_FFN_NORM}) {
      std::vector<float> w(d);
      std::memcpy(w.data(), S[(size_t)k].bytes.data(), d * 4);
      for (auto& v : w) v = host_f16_round(v);
      upload(k == LS_ATTN_NORM ? L.attn_norm : L.ffn_norm, w.data(), d * 4, kLedgerWeights);
    }
    bytes += L.qkv.w.n + L.o.w.n + L.gateup.w.n + L.down.w.n + 2 * d * 4;
    bytes += L.qkv_r.bytes.n + L.o_r.bytes.n + L.gateup_r.bytes.n + L.down_r.bytes.n;
    for (auto& t : S) {
      std::vector<uint8_t>().swap(t.bytes);
    }
  }
  // token_embd stored as f16 (its f16 rounding, src/cpu_oracle.rs:420-421)
  {
    const float* e = reinterpret_cast<const float*>(M.st_embd.bytes.data());
    const uint64_t n = (uint64_t)c.vocab * d;
    std::vector<uint16_t> h(n);
    for (uint64_t i = 0; i < n; ++i) h[i] = host_f32_to_f16(e[i]);
    upload(M.embd_f16, h.data(), n * 2, kLedgerWeights);
    bytes += n * 2;
    std::vector<uint8_t>().swap(M.st_embd.bytes);
  }
  upload(M.out_norm, M.st_out_norm.bytes.data(), d * 4, kLedgerWeights);  // not rounded (src/cpu_oracle.rs:434)
  if (!c.tied_head && M.st_output.type != FABER_GGML_Q4_K) {
    rows_from(M.head_r, (int)M.st_output.rows, (int)d, [&](int j) {
      return std::pair<const HostTensor*, uint64_t>(&M.st_output, (uint64_t)j);
    });
    M.all_q4k = false;
    bytes += M.head_r.bytes.n;
    std::vector<uint8_t>().swap(M.st_output.bytes);
  } else if (!c.tied_head) {
    M.head.from(repack_q4k((int)M.st_output.rows, (int)d, [&](int j) {
      return RowSeg{M.st_output.bytes.data(), nblk(M.st_output), (uint64_t)j * d};
    }));
    bytes += M.head.w.n;
    std::vector<uint8_t>().swap(M.st_output.bytes);
  }
  M.device_bytes = bytes;
  M.finalized = true;
}

// ---------------------------------------------------------------------------
// Session
// ---------------------------------------------------------------------------
// Allocate this rank's exchange buffer, zero it, and map every rank's buffer
// here: the IPC handles travel in one NCCL all-gather, which also orders
// every rank's zeroing before any peer can store into its buffer.
inline void open_tp_exchange(SessionState& S) {
  ModelState& M = S.m->s;
  const size_t tp = (size_t)M.tp;
  // partials, then the grid-barrier words of the consuming kernels
  S.tp_buf.alloc(session_sizes(M.cfg, M.Hl, M.Hkvl, M.Fl, M.Vl, S.max_ctx, device_info().sms).tp_buf,
                kLedgerStaging);
  FABER_CUDA(cudaMemset(S.tp_buf.p, 0, S.tp_buf.n));  // epoch 0 never matches
  cudaIpcMemHandle_t mine;
  FABER_CUDA(cudaIpcGetMemHandle(&mine, S.tp_buf.p));
  DevBuf hb(sizeof(cudaIpcMemHandle_t) * tp, kLedgerStaging);
  unsigned char* slot = hb.as<unsigned char>() + sizeof(mine) * (size_t)M.rank;
  FABER_CUDA(cudaMemcpy(slot, &mine, sizeof(mine), cudaMemcpyHostToDevice));
  FABER_NCCL(ncclAllGather(slot, hb.p, sizeof(mine), ncclUint8, M.comm, S.stream));
  FABER_CUDA(cudaStreamSynchronize(S.stream));
  std::vector<cudaIpcMemHandle_t> all(tp);
  FABER_CUDA(cudaMemcpy(all.data(), hb.p, sizeof(mine) * tp, cudaMemcpyDeviceToHost));
  S.tp_base.assign(tp, nullptr);
  for (size_t r = 0; r < tp; ++r) {
    if ((int)r == M.rank) {
      S.tp_base[r] = S.tp_buf.as<unsigned char>();
      continue;
    }
    void* p = nullptr;
    FABER_CUDA(cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess));
    S.tp_base[r] = static_cast<unsigned char*>(p);
  }
}

// Exchanges per step: O and down of every layer, then the argmax.
inline int tp_stages(const ModelState& M) { return (int)(2 * M.cfg.n_layers) + 1; }

// The argmax exchange words of a rank's buffer: [tp][3] u64 from byte 64 of
// the 256-byte tail after the partials.
inline unsigned long long* tp_argmax_words(const SessionState& S, unsigned char* base) {
  const ModelState& M = S.m->s;
  return reinterpret_cast<unsigned long long*>(base + 2 * (size_t)M.tp * M.cfg.d_model * 8 + 64);
}

// Producer side of exchange `which` (0: O, 1: down) of `layer`.
inline void tp_publish_args(SessionState& S, GemvArgs& a, int which, uint32_t layer) {
  ModelState& M = S.m->s;
  const size_t tp = (size_t)M.tp, d = M.cfg.d_model;
  a.tp = M.tp;
  a.tp_stage = (int)(2 * layer) + which;
  a.tp_stages = tp_stages(M);
  a.epoch_ptr = &S.state.as<StepState>()->tp_epoch;
  for (size_t r = 0; r < tp; ++r)
    a.peer_dst[r] = reinterpret_cast<unsigned long long*>(S.tp_base[r]) +
                    ((size_t)which * tp + (size_t)M.rank) * d;
}

// Consumer side: the next GEMV sums exchange `which` of `layer` into its input.
inline void tp_consume_args(SessionState& S, GemvArgs& a, int which, uint32_t layer) {
  ModelState& M = S.m->s;
  const size_t tp = (size_t)M.tp, d = M.cfg.d_model;
  a.tp = M.tp;
  a.tp_stage = (int)(2 * layer) + which;
  a.tp_stages = tp_stages(M);
  a.epoch_ptr = &S.state.as<StepState>()->tp_epoch;
  a.red = S.tp_buf.as<unsigned long long>() + (size_t)which * tp * d;
  a.grid_bar = reinterpret_cast<unsigned int*>(S.tp_buf.as<unsigned long long>() + 2 * tp * d);
  a.peer_wait_limit = S.peer_wait_limit;
}

inline void session_open(SessionState& S, FaberGpuModel* m, const FaberKvLayoutV1& kv) {
  ModelState& M = m->s;
  const FaberModelConfigV1& c = M.cfg;
  FABER_ARG(M.finalized, "model not finalized");
  FABER_ARG(kv.slots == 1, "one sequence slot per session");
  FABER_ARG(kv.context_length > 0 && kv.layer_count == c.n_layers &&
                kv.kv_head_count == c.n_kv_heads && kv.head_dim == c.head_dim,
            "KV layout does not match the model");
  require(kv.dtype == 1, FABER_STATUS_UNSUPPORTED,
          "the device KV cache stores f16 (dtype 1); every cached K/V is an f16-rounded value");
  S.m = m;
  S.kv = kv;
  S.device = M.device;
  FABER_CUDA(cudaSetDevice(M.device));
  S.max_ctx = (int)kv.context_length;
  const SessionSizes Z = session_sizes(c, M.Hl, M.Hkvl, M.Fl, M.Vl, S.max_ctx, device_info().sms);
  S.max_splits = Z.max_splits;
  const uint64_t hd = c.head_dim;
  S.kcache.alloc(Z.cache, kLedgerKv);
  S.vcache.alloc(Z.cache, kLedgerKv);
  FABER_CUDA(cudaMemset(S.kcache.p, 0, Z.cache));
  FABER_CUDA(cudaMemset(S.vcache.p, 0, Z.cache));
  // RoPE table on the host with the same libm calls as rope_norm
  // (src/decoder_ops.rs:178-186): theta = pos * base^(-(2k)/dim).
  {
    std::vector<float2> t((size_t)S.max_ctx * (hd / 2));
    for (int p = 0; p < S.max_ctx; ++p)
      for (uint64_t k = 0; k < hd / 2; ++k) {
        const float theta = (float)p * powf(c.rope_theta, -(2.0f * (float)k) / (float)hd);
        t[(size_t)p * (hd / 2) + k] = make_float2(cosf(theta), sinf(theta));
      }
    FABER_ARG(t.size() * sizeof(float2) == Z.rope, "RoPE table size");
    upload(S.rope, t.data(), Z.rope, kLedgerConcurrent);
  }
  S.h.alloc(Z.vec_d);
  S.h2.alloc(Z.vec_d);
  S.opart.alloc(Z.vec_d);
  S.dpart.alloc(Z.vec_d);
  S.q.alloc(Z.vec_q);
  S.ctx.alloc(Z.vec_q);
  S.hh.alloc(Z.hh);
  S.logits.alloc(Z.logits);
  if (M.tp > 1) S.logits_full.alloc(Z.logits_full);
  S.attn_part.alloc(Z.attn_part);
  S.attn_counters.alloc(Z.attn_counters);
  FABER_CUDA(cudaMemset(S.attn_counters.p, 0, S.attn_counters.n));
  S.state.alloc(Z.state, kLedgerConcurrent);
  StepState st = {};
  st.finite = 1;
  FABER_CUDA(cudaMemcpy(S.state.p, &st, sizeof(st), cudaMemcpyHostToDevice));
  S.gen.alloc(Z.gen, kLedgerConcurrent);
  S.prompt.alloc(Z.prompt, kLedgerConcurrent);
  FABER_CUDA(cudaStreamCreateWithFlags(&S.stream, cudaStreamNonBlocking));
  FABER_CUDA(cudaEventCreate(&S.ev0));
  FABER_CUDA(cudaEventCreate(&S.ev1));
  FABER_CUDA(cudaMallocHost(&S.pinned, 4096 * sizeof(int64_t)));
  S.pinned_n = 4096;
  S.prefix_layers.assign(c.n_layers, 0);
  if (M.tp > 1) open_tp_exchange(S);
}

inline StepState* st_ptr(SessionState& S) { return S.state.as<StepState>(); }

// The argmax of a tensor-parallel step: every rank holds the best key of its
// vocab shard (ordered value, then inverted id, so the lowest id wins ties,
// src/cpu_oracle.rs:979-995) and its finite flag. Each rank stores them with
// the step's epoch into its slot of every rank's exchange words (8-byte
// single-copy-atomic stores), then takes the maximum key and the minimum
// flag over all ranks' words once they carry the epoch, in rank order, and
// finishes the step like finalize_kernel. Waits are bounded (TIMEOUT).
struct ArgmaxPeers {
  unsigned long long* dst[kMaxTp];  // this rank's slot in rank r's words
  const unsigned long long* src;    // this rank's words [tp][3]
  const uint32_t* epoch_ptr;
  int32_t tp, stage, stages;
  uint32_t limit;                   // polls (0: the default)
};

__global__ void finalize_tp_kernel(StepState* st, int64_t* gen, int32_t gen_cap, const ArgmaxPeers x) {
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t e = *x.epoch_ptr * (uint32_t)x.stages + (uint32_t)x.stage + 1u;
  const unsigned long long mine = st->argmax_key;
  const uint32_t fin = st->finite ? 1u : 0u;
  const int lane = threadIdx.x;
  if (lane < x.tp) {
    unsigned long long* d = x.dst[lane];
    st_peer(d + 0, __uint_as_float((uint32_t)(mine >> 32)), e);
    st_peer(d + 1, __uint_as_float((uint32_t)mine), e);
    st_peer(d + 2, __uint_as_float(fin), e);
  }
  __syncwarp();
  if (lane != 0) return;
  const uint32_t limit = x.limit ? x.limit : kPeerSpinLimit;
  unsigned long long best = 0ull;
  uint32_t all_fin = 1u;
  for (int p = 0; p < x.tp; ++p) {
    const unsigned long long* w = x.src + 3 * p;
    const uint32_t hi = __float_as_uint(peer_value(w + 0, e, limit));
    const uint32_t lo = __float_as_uint(peer_value(w + 1, e, limit));
    const uint32_t f = __float_as_uint(peer_value(w + 2, e, limit));
    const unsigned long long k = ((unsigned long long)hi << 32) | lo;
    best = k > best ? k : best;
    all_fin &= f;
  }
  st->finite = (int32_t)all_fin;
  const int64_t tok = best ? (int64_t)(0xffffffffu - (uint32_t)(best & 0xffffffffull)) : 0;
  st->input_token = tok;
  const int32_t c = st->gen_count;
  if (gen && c >= 0 && c < gen_cap) {
    gen[c] = tok;
    st->gen_count = c + 1;
  }
  st->argmax_key = 0ull;
}

// Enqueue one push step (embedding + all layers) on S.stream.
inline void enqueue_push(SessionState& S, bool pdl) {
  ModelState& M = S.m->s;
  const FaberModelConfigV1& c = M.cfg;
  const int d = (int)c.d_model, hd = (int)c.head_dim;
  const int nq = M.Hl * hd, nk = M.Hkvl * hd;
  const size_t layer_cache = (size_t)S.max_ctx * nk;
  StepState* st = st_ptr(S);
  launch_pdl(embed_kernel, dim3(1), dim3(256), 0, S.stream, pdl, st,
             (const __half*)M.embd_f16.as<__half>(), d, (int)c.vocab, S.h.as<float>());
  for (uint32_t l = 0; l < c.n_layers; ++l) {
    LayerDev& L = M.layers[l];
    float* tr = S.trace ? S.tr.as<float>() + (size_t)l * 8 * S.tr_w : nullptr;
    // QKV
    {
      GemvArgs a = L.qkv_r.valid() ? L.qkv_r.gemv_args() : L.qkv.args();
      a.norm_w = L.attn_norm.as<float>();
      a.eps = c.rms_eps;
      a.q_out = S.q.as<float>();
      a.k_cache = S.kcache.as<__half>() + l * layer_cache;
      a.v_cache = S.vcache.as<__half>() + l * layer_cache;
      a.rope = S.rope.as<float2>();
      a.pos_ptr = &st->cur_pos;
      a.nq = nq;
      a.nk = nk;
      a.head_dim = hd;
      if (tr) {
        a.x_norm_out = tr + 0 * S.tr_w;
        a.k_trace = tr + 2 * S.tr_w;
        a.v_trace = tr + 3 * S.tr_w;
      }
      if (M.tp > 1 && l > 0) {
        // h = h2 + (previous layer's down partials of every rank)
        a.x = S.h2.as<float>();
        a.x_sum_out = S.h.as<float>();
        tp_consume_args(S, a, 1, l - 1);
        launch_gemv<WL_TILED, PRO_NORM_PEERS, EPI_QKV>(a, S.stream, pdl);
      } else {
        a.x = S.h.as<float>();
        if (L.qkv_r.valid()) launch_gemv_rows<PRO_NORM, EPI_QKV>(a, L.qkv_r, S.stream, pdl);
        else launch_gemv<WL_TILED, PRO_NORM, EPI_QKV>(a, S.stream, pdl);
      }
      if (tr) FABER_CUDA(cudaMemcpyAsync(tr + 1 * S.tr_w, S.q.p, nq * 4, cudaMemcpyDeviceToDevice, S.stream));
    }
    // attention
    {
      AttnArgs a = {};
      a.q = S.q.as<float>();
      a.k = S.kcache.as<__half>() + l * layer_cache;
      a.v = S.vcache.as<__half>() + l * layer_cache;
      a.ctx = S.ctx.as<float>();
      a.part = S.attn_part.as<float>();
      a.counters = S.attn_counters.as<int32_t>();
      a.st = st;
      a.n_heads = M.Hl;
      a.n_kv_heads = M.Hkvl;
      a.head_dim = hd;
      a.max_splits = S.max_splits;
      a.scale = 1.0f / sqrtf((float)hd);
      a.cache_rows = S.max_ctx;
      const dim3 grid(M.Hkvl, S.max_splits);
      if (hd == 128)
        launch_decode_attention<128>(a, grid, S.stream, pdl);
      else
        launch_decode_attention<64>(a, grid, S.stream, pdl);
      if (tr) FABER_CUDA(cudaMemcpyAsync(tr + 4 * S.tr_w, S.ctx.p, nq * 4, cudaMemcpyDeviceToDevice, S.stream));
    }
    // O projection (+ residual)
    {
      GemvArgs a = L.o_r.valid() ? L.o_r.gemv_args() : L.o.args();
      a.x = S.ctx.as<float>();
      if (M.tp > 1) {
        tp_publish_args(S, a, 0, l);
        launch_gemv<WL_TILED, PRO_PLAIN, EPI_PEERS>(a, S.stream, pdl);
      } else {
        a.out = S.h2.as<float>();
        a.res = S.h.as<float>();
        if (L.o_r.valid()) launch_gemv_rows<PRO_PLAIN, EPI_RESID>(a, L.o_r, S.stream, pdl);
        else launch_gemv<WL_TILED, PRO_PLAIN, EPI_RESID>(a, S.stream, pdl);
      }
    }
    // gate/up + SwiGLU
    {
      GemvArgs a = L.gateup_r.valid() ? L.gateup_r.gemv_args() : L.gateup.args();
      a.norm_w = L.ffn_norm.as<float>();
      a.eps = c.rms_eps;
      a.out = S.hh.as<float>();
      if (M.tp > 1) {
        // h2 = h + (this layer's O partials of every rank)
        a.x = S.h.as<float>();
        a.x_sum_out = S.h2.as<float>();
        tp_consume_args(S, a, 0, l);
        launch_gemv<WL_TILED, PRO_NORM_PEERS, EPI_SWIGLU>(a, S.stream, pdl);
      } else {
        a.x = S.h2.as<float>();
        if (L.gateup_r.valid()) launch_gemv_rows<PRO_NORM, EPI_SWIGLU>(a, L.gateup_r, S.stream, pdl);
        else launch_gemv<WL_TILED, PRO_NORM, EPI_SWIGLU>(a, S.stream, pdl);
      }
      if (tr) {
        FABER_CUDA(cudaMemcpyAsync(tr + 5 * S.tr_w, S.h2.p, (size_t)d * 4, cudaMemcpyDeviceToDevice, S.stream));
        FABER_CUDA(cudaMemcpyAsync(tr + 6 * S.tr_w, S.hh.p, (size_t)M.Fl * 4, cudaMemcpyDeviceToDevice, S.stream));
      }
    }
    // down (+ residual)
    {
      GemvArgs a = L.down_r.valid() ? L.down_r.gemv_args() : L.down.args();
      a.x = S.hh.as<float>();
      if (M.tp > 1) {
        tp_publish_args(S, a, 1, l);
        launch_gemv<WL_TILED, PRO_PLAIN, EPI_PEERS>(a, S.stream, pdl);
      } else {
        a.out = S.h.as<float>();
        a.res = S.h2.as<float>();
        if (L.down_r.valid()) launch_gemv_rows<PRO_PLAIN, EPI_RESID>(a, L.down_r, S.stream, pdl);
        else launch_gemv<WL_TILED, PRO_PLAIN, EPI_RESID>(a, S.stream, pdl);
        if (tr) FABER_CUDA(cudaMemcpyAsync(tr + 7 * S.tr_w, S.h.p, (size_t)d * 4, cudaMemcpyDeviceToDevice, S.stream));
      }
    }
  }
}

// Enqueue the logits step: head GEMV (+argmax) and finalize.
inline void enqueue_logits(SessionState& S, bool pdl, const std::vector<int64_t>& eog) {
  ModelState& M = S.m->s;
  const FaberModelConfigV1& c = M.cfg;
  StepState* st = st_ptr(S);
  GemvArgs a = {};
  if (c.tied_head) {
    a.w = M.embd_f16.as<uint8_t>() + (size_t)M.v0 * c.d_model * 2;
    a.n_rows = M.Vl;
    a.n_cols = (int)c.d_model;
    a.nb = (int)c.d_model / 256;
    a.n_tiles = (M.Vl + kTileRows - 1) / kTileRows;
  } else {
    a = M.head_r.valid() ? M.head_r.gemv_args() : M.head.args();
  }
  a.norm_w = M.out_norm.as<float>();
  a.eps = c.rms_eps;
  a.out = S.logits.as<float>();
  a.argmax_key = &st->argmax_key;
  a.finite_flag = &st->finite;
  a.row_offset = M.v0;
  a.n_eog = (int)eog.size();
  for (size_t i = 0; i < eog.size(); ++i) a.eog[i] = eog[i];
  const bool res = M.tp > 1;
  if (res) {
    // h = h2 + (the last layer's down partials of every rank)
    a.x = S.h2.as<float>();
    a.x_sum_out = S.h.as<float>();
    tp_consume_args(S, a, 1, c.n_layers - 1);
  } else {
    a.x = S.h.as<float>();
  }
  if (c.tied_head) {
    if (res) launch_gemv<WL_F16, PRO_NORM_PEERS, EPI_LOGITS>(a, S.stream, pdl);
    else launch_gemv<WL_F16, PRO_NORM, EPI_LOGITS>(a, S.stream, pdl);
  } else if (M.head_r.valid()) {
    launch_gemv_rows<PRO_NORM, EPI_LOGITS>(a, M.head_r, S.stream, pdl);
  } else {
    if (res) launch_gemv<WL_TILED, PRO_NORM_PEERS, EPI_LOGITS>(a, S.stream, pdl);
    else launch_gemv<WL_TILED, PRO_NORM, EPI_LOGITS>(a, S.stream, pdl);
  }
  if (M.tp > 1) {
    // the group's argmax and finite flag through peer memory: no collective
    // on the token path, bounded waits like the other exchanges
    ArgmaxPeers x = {};
    for (int r = 0; r < M.tp; ++r) x.dst[r] = tp_argmax_words(S, S.tp_base[r]) + 3 * M.rank;
    x.src = tp_argmax_words(S, S.tp_buf.as<unsigned char>());
    x.epoch_ptr = &st->tp_epoch;
    x.tp = M.tp;
    x.stage = 2 * (int)c.n_layers;
    x.stages = tp_stages(M);
    x.limit = S.peer_wait_limit;
    launch_pdl(finalize_tp_kernel, dim3(1), dim3(32), 0, S.stream, pdl, st, S.gen.as<int64_t>(),
               (int32_t)S.max_ctx, x);
  } else {
    launch_pdl(finalize_kernel, dim3(1), dim3(1), 0, S.stream, pdl, st, S.gen.as<int64_t>(),
               (int32_t)S.max_ctx);
  }
}

// A device-side bounded wait that expired (pipeline stage or tensor-parallel
// peer) is reported once the step has run; the flag is cleared.
// Turns a recorded wait expiry (g_pipe_error, read by the caller) into its
// status, clearing the record.
inline void raise_device_wait(int err) {
  if (!err) return;
  const int zero = 0;
  FABER_CUDA(cudaMemcpyToSymbol(g_pipe_error, &zero, sizeof(int)));
  throw Error(FABER_STATUS_TIMEOUT,
              err == 2   ? "a tensor-parallel peer did not publish its partials in time"
              : err == 3 ? "a grid barrier wait expired"
                         : "a device pipeline wait expired");
}

inline void check_device_waits() {
  int err = 0;
  FABER_CUDA(cudaMemcpyFromSymbol(&err, g_pipe_error, sizeof(int)));
  raise_device_wait(err);
}

// After a step whose device work failed (a bounded wait expired, or a
// kernel-side token check), the device step state goes back to the length
// the host held before the call, so the next push writes the same position
// again. The failed step overwrote the residual stream, so the session needs
// a push before its next logits. The exchange epoch is kept: every launched
// step consumed one, and an epoch is never used twice.
inline void rollback_step(SessionState& S, uint64_t n0) {
  FABER_CUDA(cudaStreamSynchronize(S.stream));
  StepState st;
  FABER_CUDA(cudaMemcpy(&st, S.state.p, sizeof(st), cudaMemcpyDeviceToHost));
  st.n = (int32_t)n0;
  st.cur_pos = n0 > 0 ? (int32_t)(n0 - 1) : 0;
  st.status = 0;
  st.argmax_key = 0ull;
  FABER_CUDA(cudaMemcpy(S.state.p, &st, sizeof(st), cudaMemcpyHostToDevice));
  S.n = n0;
  S.h_valid = false;
}

// Runs a step's device work; a TIMEOUT or KERNEL_ERROR rolls the step back.
template <class F>
inline void with_rollback(SessionState& S, F&& body) {
  const uint64_t n0 = S.n;
  try {
    body();
  } catch (const Error& e) {
    if (e.code == FABER_STATUS_TIMEOUT || e.code == FABER_STATUS_KERNEL_ERROR) rollback_step(S, n0);
    throw;
  }
}

inline void require_residual(const SessionState& S) {
  require(S.h_valid, FABER_STATUS_INVALID_ARGUMENT,
          "the session has no residual for its last position (after an installed prefix, a failed "
          "step or a truncation): push a token first");
}

inline cudaGraphExec_t capture(SessionState& S, const std::function<void()>& body) {
  cudaGraph_t g = nullptr;
  FABER_CUDA(cudaStreamBeginCapture(S.stream, cudaStreamCaptureModeThreadLocal));
  try {
    body();
  } catch (...) {
    cudaStreamEndCapture(S.stream, &g);
    if (g) cudaGraphDestroy(g);
    throw;
  }
  FABER_CUDA(cudaStreamEndCapture(S.stream, &g));
  cudaGraphExec_t e = nullptr;
  cudaError_t err = cudaGraphInstantiate(&e, g, 0);
  cudaGraphDestroy(g);
  FABER_CUDA(err);
  return e;
}

inline void ensure_graphs(SessionState& S, const std::vector<int64_t>& eog) {
  if (S.graphs_valid && eog == S.graph_eog) return;
  S.destroy_graphs();
  const bool pdl = true;
  S.g_push = capture(S, [&] { enqueue_push(S, pdl); });
  S.g_logits = capture(S, [&] { enqueue_logits(S, pdl, eog); });
  S.g_step = capture(S, [&] {
    enqueue_push(S, pdl);
    enqueue_logits(S, pdl, eog);
  });
  S.graph_eog = eog;
  S.graphs_valid = true;
}

inline void check_prefix_complete(SessionState& S) {
  if (!S.prefix_pending) return;
  for (uint8_t v : S.prefix_layers)
    FABER_ARG(v, "K/V prefix installed for some layers only");
  S.prefix_pending = false;
}

// ---------------------------------------------------------------------------
// Prompt pass on the tensor cores: all tokens of a chunk through each layer
// at once (the tcgen05 GEMMs of prefill.cuh), the same values as pushing
// them one by one (src/cpu_oracle.rs:513-534 / 859-912).
// ---------------------------------------------------------------------------
constexpr int kPrefillChunk = 2048;
constexpr uint64_t kPrefillMinTokens = 32;

inline bool prefill_supported(const ModelState& M) {
  const FaberModelConfigV1& c = M.cfg;
  const uint32_t nq = (uint32_t)M.Hl * c.head_dim;
  return M.tp == 1 && M.all_q4k && c.d_model % 256 == 0 && nq % 256 == 0 && M.Fl % 256 == 0;
}

// Tensor map over the split activations [rows][K] f16: 64 x 256 boxes with the
// 128-byte swizzle the UMMA B descriptor reads (rows past the end read 0).
inline CUtensorMap xs_tensor_map(const __half* xs, uint64_t rows, uint64_t K, int box_rows = kPgBN) {
  CUtensorMap map;
  const cuuint64_t dims[2] = {K, rows};
  const cuuint64_t strides[1] = {K * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kPgBK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = tmap_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(xs),
                                    dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  require(r == CUDA_SUCCESS, FABER_STATUS_CUDA_ERROR,
          "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return map;
}

template <int EPI, int BN = kPgBN>
void launch_prefill_gemm(const DeviceTiled& W, const CUtensorMap& map, PrefillGemmArgs a, int n_tok,
                         cudaStream_t stream) {
  auto kern = prefill_gemm_kernel<EPI, BN>;
  constexpr int kPgSmemBytes = PgLayout<BN>::kBytes;
  static thread_local std::map<int, bool> attr_done;
  int dev = 0;
  FABER_CUDA(cudaGetDevice(&dev));
  if (!attr_done[dev]) {
    FABER_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kPgSmemBytes));
    attr_done[dev] = true;
  }
  require(W.identity, FABER_STATUS_UNSUPPORTED, "prefill GEMM needs whole super-block rows");
  a.w = W.w.as<uint8_t>();
  a.n_tiles = W.n_tiles;
  a.nb = W.nb;
  a.m_rows = W.rows;
  a.n_tok = n_tok;
  const dim3 grid((2 * n_tok + BN - 1) / BN, (W.rows + kPgBM - 1) / kPgBM);
  kern<<<grid, kPgThreads, kPgSmemBytes, stream>>>(map, a);
  FABER_CUDA(cudaGetLastError());
}

// Causal attention of a prompt block (queries in pf_q, keys and values of
// positions 0 .. pos0 + n - 1 in this layer's cache) into pf_ctx.
template <int HD>
void launch_prefill_flash(SessionState& S, size_t cache_off, int n, int pos0, float scale) {
  ModelState& M = S.m->s;
  auto kern = prefill_flash_kernel<HD>;
  static thread_local std::map<int, bool> attr_done;
  int dev = 0;
  FABER_CUDA(cudaGetDevice(&dev));
  if (!attr_done[dev]) {
    FABER_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, fa_smem_bytes<HD>()));
    attr_done[dev] = true;
  }
  const dim3 grid(M.Hl, (n + kFaQ - 1) / kFaQ);
  kern<<<grid, kFaThreads, fa_smem_bytes<HD>(), S.stream>>>(
      S.pf_q.as<float>(), S.kcache.as<__half>() + cache_off, S.vcache.as<__half>() + cache_off,
      S.pf_ctx.as<float>(), n, pos0, M.Hl, M.Hkvl, scale);
  FABER_CUDA(cudaGetLastError());
}

inline void ensure_prefill_scratch(SessionState& S, int cap) {
  if (S.pf_cap >= cap) return;
  ModelState& M = S.m->s;
  const FaberModelConfigV1& c = M.cfg;
  const PrefillSizes z = prefill_sizes(c.d_model, (uint64_t)M.Hl * c.head_dim, (uint64_t)M.Fl, (uint64_t)cap);
  S.pf_h.alloc(z.h);
  S.pf_xs.alloc(z.xs);
  S.pf_scale.alloc(z.scale);
  S.pf_q.alloc(z.q);
  S.pf_ctx.alloc(z.ctx);
  S.pf_act.alloc(z.act);
  S.pf_cap = cap;
}

// Tokens [0, count) at positions S.n.. : every layer over the chunk, K/V into
// the cache; afterwards the last token's residual is the session's h.
inline void run_prefill(SessionState& S, const int64_t* dev_tokens, int count) {
  ModelState& M = S.m->s;
  const FaberModelConfigV1& c = M.cfg;
  const int d = (int)c.d_model, hd = (int)c.head_dim, nq = M.Hl * hd, nk = M.Hkvl * hd;
  const int F = M.Fl;
  const size_t layer_cache = (size_t)S.max_ctx * nk;
  ensure_prefill_scratch(S, std::min(count, kPrefillChunk));
  StepState* st = st_ptr(S);
  for (int c0 = 0; c0 < count; c0 += kPrefillChunk) {
    const int n = std::min(kPrefillChunk, count - c0);
    const int pos0 = (int)S.n + c0;
    float* H = S.pf_h.as<float>();
    __half* xs = S.pf_xs.as<__half>();
    float* xscale = S.pf_scale.as<float>();
    const CUtensorMap map_d = xs_tensor_map(xs, 2 * (uint64_t)n, d);
    const CUtensorMap map_q = xs_tensor_map(xs, 2 * (uint64_t)n, nq);
    const CUtensorMap map_f = xs_tensor_map(xs, 2 * (uint64_t)n, F);
    prefill_embed_kernel<<<n, 256, 0, S.stream>>>(dev_tokens + c0, M.embd_f16.as<__half>(), d,
                                                  (int)c.vocab, H, &st->status);
    FABER_CUDA(cudaGetLastError());
    for (uint32_t l = 0; l < c.n_layers; ++l) {
      LayerDev& L = M.layers[l];
      // attention block
      prefill_split_kernel<true><<<n, kGemvThreads, 0, S.stream>>>(H, d, L.attn_norm.as<float>(),
                                                                   c.rms_eps, xs, xscale);
      {
        PrefillGemmArgs a = {};
        a.xscale = xscale;
        a.q_out = S.pf_q.as<float>();
        a.k_cache = S.kcache.as<__half>() + l * layer_cache;
        a.v_cache = S.vcache.as<__half>() + l * layer_cache;
        a.rope = S.rope.as<float2>();
        a.nq = nq;
        a.nk = nk;
        a.head_dim = hd;
        a.pos0 = pos0;
        launch_prefill_gemm<PG_QKV>(L.qkv, map_d, a, n, S.stream);
      }
      {
        const float scale = 1.0f / sqrtf((float)hd);
        if (hd == 128)
          launch_prefill_flash<128>(S, l * layer_cache, n, pos0, scale);
        else
          launch_prefill_flash<64>(S, l * layer_cache, n, pos0, scale);
      }
      prefill_split_kernel<false><<<n, kGemvThreads, 0, S.stream>>>(S.pf_ctx.as<float>(), nq, nullptr,
                                                                    0.0f, xs, xscale);
      {
        PrefillGemmArgs a = {};
        a.xscale = xscale;
        a.out = H;
        a.ld_out = d;
        launch_prefill_gemm<PG_RESID>(L.o, map_q, a, n, S.stream);
      }
      // feed-forward block
      prefill_split_kernel<true><<<n, kGemvThreads, 0, S.stream>>>(H, d, L.ffn_norm.as<float>(),
                                                                   c.rms_eps, xs, xscale);
      {
        PrefillGemmArgs a = {};
        a.xscale = xscale;
        a.out = S.pf_act.as<float>();
        a.ld_out = F;
        launch_prefill_gemm<PG_SWIGLU>(L.gateup, map_d, a, n, S.stream);
      }
      prefill_split_kernel<false><<<n, kGemvThreads, 0, S.stream>>>(S.pf_act.as<float>(), F, nullptr,
                                                                    0.0f, xs, xscale);
      {
        PrefillGemmArgs a = {};
        a.xscale = xscale;
        a.out = H;
        a.ld_out = d;
        launch_prefill_gemm<PG_RESID>(L.down, map_f, a, n, S.stream);
      }
      FABER_CUDA(cudaGetLastError());
    }
    if (c0 + n == count) {
      // the decode state continues from the last prompt token
      FABER_CUDA(cudaMemcpyAsync(S.h.p, H + (size_t)(n - 1) * d, (size_t)d * 4,
                                 cudaMemcpyDeviceToDevice, S.stream));
    }
  }
  FABER_CUDA(cudaStreamSynchronize(S.stream));
  check_device_waits();
  StepState hs;
  FABER_CUDA(cudaMemcpy(&hs, S.state.p, sizeof(hs), cudaMemcpyDeviceToHost));
  require(hs.status == 0, FABER_STATUS_KERNEL_ERROR, "device-side token check failed");
  hs.cur_pos = (int32_t)(S.n + (uint64_t)count - 1);
  hs.n = (int32_t)(S.n + (uint64_t)count);
  FABER_CUDA(cudaMemcpy(S.state.p, &hs, sizeof(hs), cudaMemcpyHostToDevice));
  S.n += (uint64_t)count;
}

inline void run_push(SessionState& S, const int64_t* tokens, uint64_t count) {
  ModelState& M = S.m->s;
  FABER_CUDA(cudaSetDevice(S.device));
  check_prefix_complete(S);
  for (uint64_t i = 0; i < count; ++i)
    FABER_ARG(tokens[i] >= 0 && tokens[i] < (int64_t)M.cfg.vocab,
              "token " + std::to_string(tokens[i]) + " is outside the vocab [0, " +
                  std::to_string(M.cfg.vocab) + ")");
  require(S.n + count <= (uint64_t)S.max_ctx, FABER_STATUS_IO_ERROR, "KV context is full");
  if (count == 0) return;
  with_rollback(S, [&] {
  FABER_CUDA(cudaMemcpyAsync(S.prompt.p, tokens, count * 8, cudaMemcpyHostToDevice, S.stream));
  if (!S.trace && count >= kPrefillMinTokens && prefill_supported(M)) {
    run_prefill(S, S.prompt.as<int64_t>(), (int)count);
    S.h_valid = true;
    return;
  }
  if (S.trace) {
    for (uint64_t i = 0; i < count; ++i) {
      FABER_CUDA(cudaMemcpyAsync(&st_ptr(S)->input_token, S.prompt.as<int64_t>() + i, 8,
                                 cudaMemcpyDeviceToDevice, S.stream));
      enqueue_push(S, false);
    }
  } else {
    ensure_graphs(S, S.graphs_valid ? S.graph_eog : std::vector<int64_t>{});
    for (uint64_t i = 0; i < count; ++i) {
      FABER_CUDA(cudaMemcpyAsync(&st_ptr(S)->input_token, S.prompt.as<int64_t>() + i, 8,
                                 cudaMemcpyDeviceToDevice, S.stream));
      FABER_CUDA(cudaGraphLaunch(S.g_push, S.stream));
    }
  }
  FABER_CUDA(cudaStreamSynchronize(S.stream));
  check_device_waits();
  StepState st;
  FABER_CUDA(cudaMemcpy(&st, S.state.p, sizeof(st), cudaMemcpyDeviceToHost));
  require(st.status == 0, FABER_STATUS_KERNEL_ERROR, "device-side token check failed");
  S.n += count;
  S.h_valid = true;
  });
}

inline void gather_logits(SessionState& S, float* host, uint64_t cap) {
  ModelState& M = S.m->s;
  require(cap >= M.cfg.vocab, FABER_STATUS_IO_ERROR, "logits buffer smaller than the vocab");
  if (M.tp > 1) {
    require(M.cfg.vocab % M.tp == 0, FABER_STATUS_UNSUPPORTED, "vocab must split evenly to gather logits");
    FABER_NCCL(ncclAllGather(S.logits.p, S.logits_full.p, M.Vl, ncclFloat32, M.comm, S.stream));
    FABER_CUDA(cudaMemcpyAsync(host, S.logits_full.p, (size_t)M.cfg.vocab * 4, cudaMemcpyDeviceToHost, S.stream));
  } else {
    FABER_CUDA(cudaMemcpyAsync(host, S.logits.p, (size_t)M.cfg.vocab * 4, cudaMemcpyDeviceToHost, S.stream));
  }
  FABER_CUDA(cudaStreamSynchronize(S.stream));
  check_device_waits();
}

inline void run_position_logits(SessionState& S, float* host, uint64_t cap) {
  FABER_CUDA(cudaSetDevice(S.device));
  FABER_ARG(S.n > 0, "the session holds no tokens");
  FABER_ARG(host != nullptr, "null logits buffer");
  require_residual(S);
  if (S.trace) {
    enqueue_logits(S, false, {});
  } else {
    ensure_graphs(S, S.graphs_valid ? S.graph_eog : std::vector<int64_t>{});
    // the EOG set only affects the argmax, not the logits
    FABER_CUDA(cudaGraphLaunch(S.g_logits, S.stream));
  }
  gather_logits(S, host, cap);
}

inline void run_greedy(SessionState& S, uint32_t n_gen, const int64_t* eog, uint32_t n_eog,
                       int64_t* out, int32_t* all_finite) {
  ModelState& M = S.m->s;
  FABER_CUDA(cudaSetDevice(S.device));
  FABER_ARG(S.n > 0, "greedy decode needs a prompt");
  FABER_ARG(n_eog <= (uint32_t)kMaxEog, "at most 8 EOG ids");
  FABER_ARG(out != nullptr || n_gen == 0, "null output");
  if (n_gen == 0) return;
  require(S.n + n_gen - 1 <= (uint64_t)S.max_ctx, FABER_STATUS_IO_ERROR, "KV context is full");
  check_prefix_complete(S);
  require_residual(S);
  std::vector<int64_t> e(eog, eog + n_eog);
  with_rollback(S, [&] {
  // reset the per-run counters
  StepState st;
  FABER_CUDA(cudaMemcpyAsync(&st, S.state.p, sizeof(st), cudaMemcpyDeviceToHost, S.stream));
  FABER_CUDA(cudaStreamSynchronize(S.stream));
  st.gen_count = 0;
  st.finite = 1;
  st.argmax_key = 0;
  FABER_CUDA(cudaMemcpyAsync(S.state.p, &st, sizeof(st), cudaMemcpyHostToDevice, S.stream));
  if (S.trace) {
    enqueue_logits(S, false, e);
    for (uint32_t i = 1; i < n_gen; ++i) {
      enqueue_push(S, false);
      enqueue_logits(S, false, e);
    }
  } else {
    ensure_graphs(S, e);
    FABER_CUDA(cudaEventRecord(S.ev0, S.stream));
    FABER_CUDA(cudaGraphLaunch(S.g_logits, S.stream));
    for (uint32_t i = 1; i < n_gen; ++i) FABER_CUDA(cudaGraphLaunch(S.g_step, S.stream));
    FABER_CUDA(cudaEventRecord(S.ev1, S.stream));
  }
  FABER_CUDA(cudaMemcpyAsync(out, S.gen.p, (size_t)n_gen * 8, cudaMemcpyDeviceToHost, S.stream));
  FABER_CUDA(cudaMemcpyAsync(&st, S.state.p, sizeof(st), cudaMemcpyDeviceToHost, S.stream));
  FABER_CUDA(cudaStreamSynchronize(S.stream));
  check_device_waits();
  if (!S.trace) FABER_CUDA(cudaEventElapsedTime(&S.last_greedy_ms, S.ev0, S.ev1));
  if (all_finite) *all_finite = st.finite;
  S.n += n_gen - 1;
  S.h_valid = true;
  });
  (void)M;
}

// One step of a host-driven greedy loop: push `token`, then the new
// position's logits and their argmax over the non-EOG ids, returning only
// that id. The token travels in 8 bytes from pinned memory and the answer in
// 8 bytes back; the logits stay on the device. The same graph as a
// run_greedy step, so the ids equal run_greedy's.
inline int64_t run_step_greedy(SessionState& S, int64_t token, const int64_t* eog, uint32_t n_eog) {
  ModelState& M = S.m->s;
  FABER_CUDA(cudaSetDevice(S.device));
  FABER_ARG(n_eog <= (uint32_t)kMaxEog, "at most 8 EOG ids");
  FABER_ARG(eog != nullptr || n_eog == 0, "null EOG ids");
  FABER_ARG(token >= 0 && token < (int64_t)M.cfg.vocab,
            "token " + std::to_string(token) + " is outside the vocab [0, " + std::to_string(M.cfg.vocab) + ")");
  require(S.n + 1 <= (uint64_t)S.max_ctx, FABER_STATUS_IO_ERROR, "KV context is full");
  check_prefix_complete(S);
  std::vector<int64_t> e(eog, eog + n_eog);
  StepState* st = st_ptr(S);
  int64_t* pin = static_cast<int64_t*>(S.pinned);
  with_rollback(S, [&] {
  pin[0] = token;
  FABER_CUDA(cudaMemcpyAsync(&st->input_token, pin, 8, cudaMemcpyHostToDevice, S.stream));
  if (S.trace) {
    enqueue_push(S, false);
    enqueue_logits(S, false, e);
  } else {
    ensure_graphs(S, e);
    FABER_CUDA(cudaGraphLaunch(S.g_step, S.stream));
  }
  FABER_CUDA(cudaMemcpyAsync(pin + 1, &st->input_token, 8, cudaMemcpyDeviceToHost, S.stream));
  // the wait-expiry record comes back with the token: one round trip
  pin[2] = 0;
  FABER_CUDA(cudaMemcpyFromSymbolAsync(pin + 2, g_pipe_error, sizeof(int), 0, cudaMemcpyDeviceToHost, S.stream));
  FABER_CUDA(cudaStreamSynchronize(S.stream));
  raise_device_wait(static_cast<int>(pin[2]));
  S.n += 1;
  S.h_valid = true;
  });
  return pin[1];
}

// ---------------------------------------------------------------------------
// Batched greedy decode: up to kBatchMax sessions of one model advance one
// token per step together. Every linear layer is one tcgen05 Q4_K GEMM whose
// activation tile holds the sequences as (hi, lo) f16 column pairs, so each
// weight byte is read once per step for the whole batch; attention runs per
// sequence in one launch (grid.z = sequence) over each session's own cache.
// The sessions keep their state: afterwards each holds its sequence's
// residual, length and cache, and its own calls continue from there.
// ---------------------------------------------------------------------------
constexpr int kBatchMax = kBgMaxSeq;

struct BatchState {
  std::vector<SessionState*> seq;
  int B = 0, device = 0, max_ctx = 0, splits = 0, gen_cap = 0;
  cudaStream_t stream = nullptr;
  DevBuf slots;  // SlotRef [L][B]
  DevBuf h, xs, xscale, q, ctx, act, logits, attn_part, attn_counters, gen;
  DevBuf kpart;  // the batched GEMV's slab partials
  DevBuf kvmaps;  // CUtensorMap [L][B][K, V]: the streamed attention's maps (ratio <= 2)
  cudaGraphExec_t g_step = nullptr, g_logits = nullptr;
  std::vector<int64_t> graph_eog;
  bool graphs_valid = false;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  float last_ms = 0.f;
  ~BatchState() {
    int cur = -1;
    cudaGetDevice(&cur);
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    if (g_step) cudaGraphExecDestroy(g_step);
    if (g_logits) cudaGraphExecDestroy(g_logits);
    if (ev0) cudaEventDestroy(ev0);
    if (ev1) cudaEventDestroy(ev1);
    if (stream) cudaStreamDestroy(stream);
    if (cur >= 0) cudaSetDevice(cur);
  }
};

inline bool batch_supported(const ModelState& M) {
  return prefill_supported(M) && !M.cfg.tied_head && M.head.identity;
}

// K slabs of a batched GEMV over W for B sequences.
inline int bgemv_slabs(const DeviceTiled& W, int B) {
  const int sb = bg_slab_sb(W.nb, B);
  return (W.nb + sb - 1) / sb;
}

// Partial-sum scratch (floats) and tile tickets a batched GEMV over W needs.
inline size_t bgemv_part_floats(const DeviceTiled& W, int B) {
  const int ns = bgemv_slabs(W, B);
  return ns > 1 ? (size_t)ns * W.n_tiles * kTileRows * B : 0;
}

// One instantiation per (epilogue, column blocks): each sets its own
// shared-memory opt-in once per device.
template <int EPI, int NB>
void launch_bgemv_nb(const BgemvArgs& a, int grid, size_t smem, cudaStream_t stream) {
  auto kern = bgemv_kernel<EPI, NB>;
  static thread_local std::map<int, bool> attr_done;
  int dev = 0;
  FABER_CUDA(cudaGetDevice(&dev));
  if (!attr_done[dev]) {
    FABER_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBgSmemMax));
    attr_done[dev] = true;
  }
  kern<<<grid, kPipeThreads, smem, stream>>>(a);
  FABER_CUDA(cudaGetLastError());
}

template <int EPI>
void launch_bgemv(const DeviceTiled& W, BgemvArgs a, int B, int K, cudaStream_t stream) {
  require(W.identity, FABER_STATUS_UNSUPPORTED, "batched GEMV needs rows in whole super-blocks");
  require(B >= 1 && B <= kBgMaxSeq, FABER_STATUS_INVALID_ARGUMENT, "batched GEMV takes 1 to 16 sequences");
  a.w = W.w.as<uint8_t>();
  a.n_tiles = W.n_tiles;
  a.nb = W.nb;
  a.n_rows = W.rows;
  a.B = B;
  a.K = K;
  a.slab_sb = bg_slab_sb(W.nb, B);
  a.n_slabs = (W.nb + a.slab_sb - 1) / a.slab_sb;
  const BgLayout L = bg_layout(a.slab_sb, B);
  require(L.total <= kBgSmemMax, FABER_STATUS_UNSUPPORTED, "batched GEMV slab exceeds shared memory");
  const int grid = std::max(a.n_slabs, device_info().sms);
  if (B <= 4) launch_bgemv_nb<EPI, 1>(a, grid, L.total, stream);
  else if (B <= 8) launch_bgemv_nb<EPI, 2>(a, grid, L.total, stream);
  else launch_bgemv_nb<EPI, 4>(a, grid, L.total, stream);
  if (a.n_slabs > 1) {
    bg_combine_kernel<EPI><<<(a.n_tiles + kBgCombineWarps - 1) / kBgCombineWarps, kBgCombineWarps * 32, 0, stream>>>(a);
    FABER_CUDA(cudaGetLastError());
  }
}

inline void batch_build(BatchState& Bt, SessionState* const* seqs, int n) {
  FABER_ARG(n >= 1 && n <= kBatchMax, "a batch holds 1 to " + std::to_string(kBatchMax) + " sessions");
  SessionState& S0 = *seqs[0];
  ModelState& M = S0.m->s;
  require(batch_supported(M), FABER_STATUS_UNSUPPORTED,
          "batched decode needs one GPU, an untied Q4_K head and dimensions in whole super-blocks");
  for (int i = 0; i < n; ++i) {
    FABER_ARG(seqs[i] != nullptr, "null session");
    FABER_ARG(seqs[i]->m == S0.m, "every session of a batch must use the same model");
    FABER_ARG(seqs[i]->max_ctx == S0.max_ctx, "every session of a batch must have the same context length");
    FABER_ARG(!seqs[i]->trace, "traced sessions cannot join a batch");
    for (int j = 0; j < i; ++j) FABER_ARG(seqs[j] != seqs[i], "a session appears twice in the batch");
  }
  const FaberModelConfigV1& c = M.cfg;
  Bt.seq.assign(seqs, seqs + n);
  Bt.B = n;
  Bt.device = S0.device;
  Bt.max_ctx = S0.max_ctx;
  FABER_CUDA(cudaSetDevice(Bt.device));
  FABER_CUDA(cudaStreamCreateWithFlags(&Bt.stream, cudaStreamNonBlocking));
  FABER_CUDA(cudaEventCreate(&Bt.ev0));
  FABER_CUDA(cudaEventCreate(&Bt.ev1));
  const int d = (int)c.d_model, hd = (int)c.head_dim, nq = M.Hl * hd, nk = M.Hkvl * hd;
  const size_t layer_cache = (size_t)Bt.max_ctx * nk;
  std::vector<SlotRef> refs((size_t)c.n_layers * n);
  for (uint32_t l = 0; l < c.n_layers; ++l)
    for (int i = 0; i < n; ++i) {
      SessionState& S = *seqs[i];
      refs[(size_t)l * n + i] = SlotRef{st_ptr(S), S.kcache.as<__half>() + l * layer_cache,
                                        S.vcache.as<__half>() + l * layer_cache};
    }
  Bt.slots.alloc(refs.size() * sizeof(SlotRef), kLedgerConcurrent);
  FABER_CUDA(cudaMemcpy(Bt.slots.p, refs.data(), Bt.slots.n, cudaMemcpyHostToDevice));
  const size_t kmax = std::max((size_t)d, std::max((size_t)nq, (size_t)M.Fl));
  Bt.h.alloc((size_t)n * d * 4);
  // the hi/lo split of every sequence's input row (2n rows of the widest K)
  Bt.xs.alloc((size_t)2 * n * kmax * 2);
  FABER_CUDA(cudaMemset(Bt.xs.p, 0, Bt.xs.n));
  Bt.xscale.alloc((size_t)kBatchMax * 4);
  FABER_CUDA(cudaMemset(Bt.xscale.p, 0, Bt.xscale.n));
  Bt.q.alloc((size_t)n * nq * 4);
  Bt.ctx.alloc((size_t)n * nq * 4);
  Bt.act.alloc((size_t)n * M.Fl * 4);
  Bt.logits.alloc((size_t)n * c.vocab * 4);
  Bt.splits = attention_splits(device_info().sms, M.Hkvl * n, Bt.max_ctx);
  if (M.Hl / M.Hkvl <= kAsStreamMaxRatio) {
    // the streamed attention: its split count, and every (layer, sequence)'s
    // K and V tensor maps
    Bt.splits = std::max(Bt.splits, attention_stream_splits(device_info().sms, M.Hkvl * n, Bt.max_ctx, hd,
                                                            M.Hl / M.Hkvl,
                                                            std::max(1, (Bt.max_ctx + kAsKeys - 1) / kAsKeys)));
    std::vector<CUtensorMap> maps((size_t)c.n_layers * n * 2);
    for (uint32_t l = 0; l < c.n_layers; ++l)
      for (int i = 0; i < n; ++i) {
        maps[((size_t)l * n + i) * 2] = kv_tensor_map(refs[(size_t)l * n + i].k, (uint64_t)Bt.max_ctx, nk);
        maps[((size_t)l * n + i) * 2 + 1] = kv_tensor_map(refs[(size_t)l * n + i].v, (uint64_t)Bt.max_ctx, nk);
      }
    Bt.kvmaps.alloc(maps.size() * sizeof(CUtensorMap), kLedgerConcurrent);
    FABER_CUDA(cudaMemcpy(Bt.kvmaps.p, maps.data(), Bt.kvmaps.n, cudaMemcpyHostToDevice));
  }
  Bt.attn_part.alloc((size_t)n * M.Hl * Bt.splits * (hd + 2) * 4);
  Bt.attn_counters.alloc((size_t)n * M.Hkvl * 4);
  FABER_CUDA(cudaMemset(Bt.attn_counters.p, 0, Bt.attn_counters.n));
  Bt.gen_cap = Bt.max_ctx;
  Bt.gen.alloc((size_t)n * Bt.gen_cap * 8, kLedgerConcurrent);
  // the batched GEMV's slab partials (the largest over the step's linears)
  size_t part = 0;
  auto need = [&](const DeviceTiled& W) { part = std::max(part, bgemv_part_floats(W, n)); };
  for (const LayerDev& L : M.layers) {
    need(L.qkv);
    need(L.o);
    need(L.gateup);
    need(L.down);
  }
  need(M.head);
  Bt.kpart.alloc(std::max<size_t>(part, 1) * 4);
}

// The head over the batch's residual rows: logits, argmax keys, next tokens.
inline void enqueue_batch_logits(BatchState& Bt, const std::vector<int64_t>& eog) {
  ModelState& M = Bt.seq[0]->m->s;
  const FaberModelConfigV1& c = M.cfg;
  const int d = (int)c.d_model, n = Bt.B;
  const SlotRef* sl0 = Bt.slots.as<SlotRef>();
  __half* xs = Bt.xs.as<__half>();
  prefill_split_kernel<true><<<n, kGemvThreads, 0, Bt.stream>>>(Bt.h.as<float>(), d, M.out_norm.as<float>(),
                                                                 c.rms_eps, xs, Bt.xscale.as<float>());
  BgemvArgs a = {};
  a.xs = xs;
  a.xscale = Bt.xscale.as<float>();
  a.out = Bt.logits.as<float>();
  a.ld_out = (int)c.vocab;
  a.slots = sl0;
  a.n_eog = (int)eog.size();
  for (size_t i = 0; i < eog.size(); ++i) a.eog[i] = eog[i];
  a.part = Bt.kpart.as<float>();
  launch_bgemv<BG_LOGITS>(M.head, a, n, d, Bt.stream);
  slots_finalize_kernel<<<n, 32, 0, Bt.stream>>>(sl0, Bt.gen.as<int64_t>(), Bt.gen_cap);
  FABER_CUDA(cudaGetLastError());
}

// One batched step: every sequence pushes its input token through all layers.
inline void enqueue_batch_push(BatchState& Bt) {
  ModelState& M = Bt.seq[0]->m->s;
  SessionState& S0 = *Bt.seq[0];
  const FaberModelConfigV1& c = M.cfg;
  const int n = Bt.B, d = (int)c.d_model, hd = (int)c.head_dim, nq = M.Hl * hd, nk = M.Hkvl * hd;
  const int F = M.Fl;
  const SlotRef* sl = Bt.slots.as<SlotRef>();
  float* H = Bt.h.as<float>();
  __half* xs = Bt.xs.as<__half>();
  float* xscale = Bt.xscale.as<float>();
  slots_embed_kernel<<<n, 256, 0, Bt.stream>>>(sl, M.embd_f16.as<__half>(), d, (int)c.vocab, H);
  FABER_CUDA(cudaGetLastError());
  for (uint32_t l = 0; l < c.n_layers; ++l) {
    LayerDev& L = M.layers[l];
    const SlotRef* sll = sl + (size_t)l * n;
    prefill_split_kernel<true><<<n, kGemvThreads, 0, Bt.stream>>>(H, d, L.attn_norm.as<float>(), c.rms_eps,
                                                                   xs, xscale);
    {
      BgemvArgs a = {};
      a.xs = xs;
      a.xscale = xscale;
      a.q_out = Bt.q.as<float>();
      a.rope = S0.rope.as<float2>();
      a.nq = nq;
      a.nk = nk;
      a.head_dim = hd;
      a.slots = sll;
      a.part = Bt.kpart.as<float>();
      launch_bgemv<BG_QKV>(L.qkv, a, n, d, Bt.stream);
    }
    {
      AttnArgs a = {};
      a.q = Bt.q.as<float>();
      a.ctx = Bt.ctx.as<float>();
      a.part = Bt.attn_part.as<float>();
      a.counters = Bt.attn_counters.as<int32_t>();
      a.n_heads = M.Hl;
      a.n_kv_heads = M.Hkvl;
      a.head_dim = hd;
      a.max_splits = Bt.splits;
      a.scale = 1.0f / sqrtf((float)hd);
      a.slots = sll;
      a.slot_q_stride = nq;
      a.slot_part_stride = M.Hl * Bt.splits * (hd + 2);
      a.slot_counter_stride = M.Hkvl;
      a.cache_rows = Bt.max_ctx;
      if (Bt.kvmaps.p) a.kvmaps = Bt.kvmaps.as<CUtensorMap>() + (size_t)l * n * 2;
      const dim3 grid(M.Hkvl, Bt.splits, n);
      if (hd == 128)
        launch_decode_attention<128>(a, grid, Bt.stream, false);
      else
        launch_decode_attention<64>(a, grid, Bt.stream, false);
    }
    prefill_split_kernel<false><<<n, kGemvThreads, 0, Bt.stream>>>(Bt.ctx.as<float>(), nq, nullptr, 0.0f,
                                                                    xs, xscale);
    {
      BgemvArgs a = {};
      a.xs = xs;
      a.xscale = xscale;
      a.out = H;
      a.ld_out = d;
      a.part = Bt.kpart.as<float>();
      launch_bgemv<BG_RESID>(L.o, a, n, nq, Bt.stream);
    }
    prefill_split_kernel<true><<<n, kGemvThreads, 0, Bt.stream>>>(H, d, L.ffn_norm.as<float>(), c.rms_eps,
                                                                   xs, xscale);
    {
      BgemvArgs a = {};
      a.xs = xs;
      a.xscale = xscale;
      a.out = Bt.act.as<float>();
      a.ld_out = F;
      a.part = Bt.kpart.as<float>();
      launch_bgemv<BG_SWIGLU>(L.gateup, a, n, d, Bt.stream);
    }
    prefill_split_kernel<false><<<n, kGemvThreads, 0, Bt.stream>>>(Bt.act.as<float>(), F, nullptr, 0.0f,
                                                                    xs, xscale);
    {
      BgemvArgs a = {};
      a.xs = xs;
      a.xscale = xscale;
      a.out = H;
      a.ld_out = d;
      a.part = Bt.kpart.as<float>();
      launch_bgemv<BG_RESID>(L.down, a, n, F, Bt.stream);
    }
    FABER_CUDA(cudaGetLastError());
  }
}

inline void batch_graphs(BatchState& Bt, const std::vector<int64_t>& eog) {
  if (Bt.graphs_valid && Bt.graph_eog == eog) return;
  if (Bt.g_step) cudaGraphExecDestroy(Bt.g_step);
  if (Bt.g_logits) cudaGraphExecDestroy(Bt.g_logits);
  Bt.g_step = Bt.g_logits = nullptr;
  cudaGraph_t g;
  FABER_CUDA(cudaStreamBeginCapture(Bt.stream, cudaStreamCaptureModeThreadLocal));
  enqueue_batch_logits(Bt, eog);
  FABER_CUDA(cudaStreamEndCapture(Bt.stream, &g));
  FABER_CUDA(cudaGraphInstantiate(&Bt.g_logits, g, 0));
  FABER_CUDA(cudaGraphDestroy(g));
  FABER_CUDA(cudaStreamBeginCapture(Bt.stream, cudaStreamCaptureModeThreadLocal));
  enqueue_batch_push(Bt);
  enqueue_batch_logits(Bt, eog);
  FABER_CUDA(cudaStreamEndCapture(Bt.stream, &g));
  FABER_CUDA(cudaGraphInstantiate(&Bt.g_step, g, 0));
  FABER_CUDA(cudaGraphDestroy(g));
  Bt.graph_eog = eog;
  Bt.graphs_valid = true;
}

// run_greedy (src/greedy_run.rs:186-248) for every sequence of the batch at
// once: n_gen tokens each, out[i * n_gen + j] = token j of sequence i.
inline void run_batch_greedy(BatchState& Bt, uint32_t n_gen, const int64_t* eog, uint32_t n_eog,
                             int64_t* out, int32_t* all_finite) {
  FABER_CUDA(cudaSetDevice(Bt.device));
  FABER_ARG(n_eog <= (uint32_t)kMaxEog, "at most 8 EOG ids");
  FABER_ARG(out != nullptr || n_gen == 0, "null output");
  if (n_gen == 0) return;
  FABER_ARG(n_gen <= (uint32_t)Bt.gen_cap, "n_gen above the context length");
  ModelState& M = Bt.seq[0]->m->s;
  const size_t d = M.cfg.d_model;
  for (int i = 0; i < Bt.B; ++i) {
    SessionState& S = *Bt.seq[i];
    FABER_ARG(S.n > 0, "greedy decode needs a prompt in every session");
    require(S.n + n_gen - 1 <= (uint64_t)S.max_ctx, FABER_STATUS_IO_ERROR, "KV context is full");
    check_prefix_complete(S);
    require_residual(S);
    // the session's own work has finished before the batch stream reads it
    FABER_CUDA(cudaStreamSynchronize(S.stream));
    StepState st;
    FABER_CUDA(cudaMemcpy(&st, S.state.p, sizeof(st), cudaMemcpyDeviceToHost));
    st.gen_count = 0;
    st.finite = 1;
    st.argmax_key = 0;
    FABER_CUDA(cudaMemcpy(S.state.p, &st, sizeof(st), cudaMemcpyHostToDevice));
    FABER_CUDA(cudaMemcpyAsync(Bt.h.as<float>() + (size_t)i * d, S.h.p, d * 4, cudaMemcpyDeviceToDevice,
                               Bt.stream));
  }
  std::vector<int64_t> e(eog, eog + n_eog);
  batch_graphs(Bt, e);
  FABER_CUDA(cudaEventRecord(Bt.ev0, Bt.stream));
  FABER_CUDA(cudaGraphLaunch(Bt.g_logits, Bt.stream));
  for (uint32_t j = 1; j < n_gen; ++j) FABER_CUDA(cudaGraphLaunch(Bt.g_step, Bt.stream));
  FABER_CUDA(cudaEventRecord(Bt.ev1, Bt.stream));
  std::vector<int64_t> gen((size_t)Bt.B * Bt.gen_cap);
  FABER_CUDA(cudaMemcpyAsync(gen.data(), Bt.gen.p, Bt.gen.n, cudaMemcpyDeviceToHost, Bt.stream));
  for (int i = 0; i < Bt.B; ++i)  // each session continues from its sequence's residual
    FABER_CUDA(cudaMemcpyAsync(Bt.seq[i]->h.p, Bt.h.as<float>() + (size_t)i * d, d * 4,
                               cudaMemcpyDeviceToDevice, Bt.stream));
  FABER_CUDA(cudaStreamSynchronize(Bt.stream));
  check_device_waits();
  FABER_CUDA(cudaEventElapsedTime(&Bt.last_ms, Bt.ev0, Bt.ev1));
  for (int i = 0; i < Bt.B; ++i) {
    SessionState& S = *Bt.seq[i];
    StepState st;
    FABER_CUDA(cudaMemcpy(&st, S.state.p, sizeof(st), cudaMemcpyDeviceToHost));
    require(st.status == 0, FABER_STATUS_KERNEL_ERROR, "device-side token check failed");
    if (all_finite) all_finite[i] = st.finite;
    for (uint32_t j = 0; j < n_gen; ++j) out[(size_t)i * n_gen + j] = gen[(size_t)i * Bt.gen_cap + j];
    S.n += n_gen - 1;
    S.h_valid = true;
  }
}

inline void set_prefix(SessionState& S, uint32_t layer, const float* k, const float* v, uint64_t n) {
  ModelState& M = S.m->s;
  const FaberModelConfigV1& c = M.cfg;
  FABER_CUDA(cudaSetDevice(S.device));
  FABER_ARG(layer < c.n_layers && k && v, "bad layer or null K/V");
  FABER_ARG(n > 0 && n < (uint64_t)S.max_ctx, "prefix length must leave room in the context");
  FABER_ARG(S.n == 0 || S.prefix_pending, "prefix must be installed into an empty session");
  if (S.prefix_pending) FABER_ARG(n == S.prefix_n, "every layer must get the same prefix length");
  const uint64_t hd = c.head_dim, kvs_full = (uint64_t)c.n_kv_heads * hd;
  const uint64_t kvs = (uint64_t)M.Hkvl * hd, off = (uint64_t)M.rank * kvs;
  std::vector<uint16_t> hk(n * kvs), hv(n * kvs);
  for (uint64_t p = 0; p < n; ++p)
    for (uint64_t i = 0; i < kvs; ++i) {
      hk[p * kvs + i] = host_f32_to_f16(k[p * kvs_full + off + i]);
      hv[p * kvs + i] = host_f32_to_f16(v[p * kvs_full + off + i]);
    }
  const size_t layer_cache = (size_t)S.max_ctx * kvs;
  FABER_CUDA(cudaMemcpy(S.kcache.as<__half>() + layer * layer_cache, hk.data(), hk.size() * 2, cudaMemcpyHostToDevice));
  FABER_CUDA(cudaMemcpy(S.vcache.as<__half>() + layer * layer_cache, hv.data(), hv.size() * 2, cudaMemcpyHostToDevice));
  S.prefix_layers[layer] = 1;
  S.prefix_pending = true;
  S.prefix_n = n;
  S.n = n;
  S.h_valid = false;
  StepState st;
  FABER_CUDA(cudaMemcpy(&st, S.state.p, sizeof(st), cudaMemcpyDeviceToHost));
  st.n = (int32_t)n;
  FABER_CUDA(cudaMemcpy(S.state.p, &st, sizeof(st), cudaMemcpyHostToDevice));
}

// One decode step of a tensor-parallel group as a transaction plan
// (src/execution_transaction/transaction.rs over the group's ranks): a
// launch per rank, whose published output is the position's K/V rows of
// its kv heads (f16) and the token, then a barrier over all ranks: the
// step's exchanges. The O and down partials cross through each rank's
// exchange buffer and are consumed inside the step, so they publish
// nothing; that buffer is admitted with the session (class 6). A rank whose
// exchange fails is a fault of the barrier on that rank. The commit
// boundary is the barrier and every launch. References: position << 16 |
// tag << 8 | rank (tag 1 launch, 3 barrier).
inline void tp_step_plan(const FaberModelConfigV1& c, uint32_t position, std::vector<FaberTxnOpV1>& ops,
                         uint64_t& barrier_ref, std::vector<uint64_t>& launch_refs) {
  validate_config(c);
  FABER_ARG(c.tp_size >= 2, "a single rank runs no group transaction");
  const uint64_t tp = c.tp_size, hd = c.head_dim;
  const uint64_t kv_rows = (uint64_t)c.n_layers * (c.n_kv_heads / tp) * hd * 2 * 2;
  const uint64_t base = (uint64_t)position << 16;
  ops.clear();
  launch_refs.clear();
  for (uint32_t r = 0; r < tp; ++r) {
    FaberTxnOpV1 op{};
    op.kind = FABER_TXN_LAUNCH;
    op.partition = r;
    op.ref = base | 1u << 8 | r;
    op.bytes = kv_rows + 8;
    ops.push_back(op);
    launch_refs.push_back(op.ref);
  }
  FaberTxnOpV1 op{};
  op.kind = FABER_TXN_BARRIER;
  op.participants = tp >= 64 ? ~0ull : (1ull << tp) - 1;
  op.ref = base | 3u << 8;
  ops.push_back(op);
  barrier_ref = op.ref;
}

// The device buffers of a tiled Q4_K linear whose row j starts at element
// start(j) of its source: repack_q4k groups rows by their offset inside a
// super-block, 16 rows per tile, and keeps a tile offset and row map unless
// every row starts on a block boundary.
inline void plan_tiled(std::vector<std::pair<uint64_t, int>>& bufs, uint64_t rows, uint64_t cols,
                       const std::function<uint64_t(uint64_t)>& start) {
  std::map<uint64_t, uint64_t> per_offset;
  uint64_t max_o = 0;
  for (uint64_t j = 0; j < rows; ++j) {
    const uint64_t o = start(j) % kQ4kBlockElems;
    ++per_offset[o];
    max_o = std::max(max_o, o);
  }
  uint64_t tiles = 0;
  for (const auto& kv : per_offset) tiles += (kv.second + kTileRows - 1) / kTileRows;
  const uint64_t nb = (cols + max_o + kQ4kBlockElems - 1) / kQ4kBlockElems;
  bufs.push_back({tiles * nb * kTileItemBytes, kLedgerWeights});
  if (!(per_offset.size() == 1 && per_offset.begin()->first == 0)) {
    bufs.push_back({tiles * 4, kLedgerWeights});
    bufs.push_back({tiles * kTileRows * 4, kLedgerWeights});
  }
}

// The ledger one rank's model and `sessions` sessions of context_length
// positions draw on a device with `sms` SMs, before anything is allocated:
// every buffer the model upload, session_open and (where the prompt pass
// runs) its scratch allocate, each charged by the allocator policy. Assumes
// Q4_K linears (the tiled GEMV layout); other block types are charged as
// they upload.
inline FaberPartitionLedgerV1 partition_plan(const FaberModelConfigV1& c, uint32_t context_length,
                                             uint32_t sessions, int sms) {
  validate_config(c);
  FABER_ARG(context_length > 0 && sms > 0, "zero context length or SM count");
  const TpPlan P = tp_plan(c);
  const uint64_t d = c.d_model, hd = c.head_dim, nq = (uint64_t)P.Hl * hd, nk = (uint64_t)P.Hkvl * hd;
  const uint64_t fl = (uint64_t)P.Fl;
  std::vector<std::pair<uint64_t, int>> bufs;
  // row starts as model_finalize builds them (shards are compact copies)
  const uint64_t o_cols = c.tp_size == 1 ? (uint64_t)c.n_heads * hd : nq;
  const uint64_t down_cols = c.tp_size == 1 ? (uint64_t)c.ffn : fl;
  for (uint32_t l = 0; l < c.n_layers; ++l) {
    plan_tiled(bufs, nq + 2 * nk, d, [&](uint64_t j) {
      return (j < nq ? j : (j < nq + nk ? j - nq : j - nq - nk)) * d;
    });
    plan_tiled(bufs, d, o_cols, [&](uint64_t j) { return j * o_cols; });
    plan_tiled(bufs, 2 * fl, d, [&](uint64_t j) { return (j >> 1) * d; });
    plan_tiled(bufs, d, down_cols, [&](uint64_t j) { return j * down_cols; });
    bufs.push_back({d * 4, kLedgerWeights});  // attn_norm
    bufs.push_back({d * 4, kLedgerWeights});  // ffn_norm
  }
  bufs.push_back({(uint64_t)c.vocab * d * 2, kLedgerWeights});  // token_embd as f16
  bufs.push_back({d * 4, kLedgerWeights});                      // output_norm
  if (!c.tied_head) plan_tiled(bufs, (uint64_t)P.Vl, d, [&](uint64_t j) { return j * d; });
  const SessionSizes z = session_sizes(c, P.Hl, P.Hkvl, P.Fl, P.Vl, (int)context_length, sms);
  const bool prompt_pass = c.tp_size == 1 && d % 256 == 0 && nq % 256 == 0 && fl % 256 == 0;
  const PrefillSizes pz =
      prefill_sizes(d, nq, fl, std::min<uint64_t>(context_length, (uint64_t)kPrefillChunk));
  for (uint32_t i = 0; i < sessions; ++i) {
    bufs.push_back({z.cache, kLedgerKv});
    bufs.push_back({z.cache, kLedgerKv});
    bufs.push_back({z.rope, kLedgerConcurrent});
    for (int k = 0; k < 4; ++k) bufs.push_back({z.vec_d, kLedgerActivation});
    for (int k = 0; k < 2; ++k) bufs.push_back({z.vec_q, kLedgerActivation});
    for (uint64_t b : {z.hh, z.logits, z.logits_full, z.attn_part, z.attn_counters})
      bufs.push_back({b, kLedgerActivation});
    for (uint64_t b : {z.state, z.gen, z.prompt}) bufs.push_back({b, kLedgerConcurrent});
    bufs.push_back({z.tp_buf, kLedgerStaging});
    if (prompt_pass)
      for (uint64_t b : {pz.h, pz.xs, pz.scale, pz.q, pz.ctx, pz.act}) bufs.push_back({b, kLedgerActivation});
  }
  uint64_t live[kLedgerClasses] = {};
  for (const auto& b : bufs) {
    if (b.first == 0) continue;
    const uint64_t charged = ledger_charge(b.first);
    FABER_ARG(charged != 0, "buffer size overflows the allocator policy");
    live[b.second] += b.first;
    live[kLedgerOverhead] += charged - b.first;
  }
  FaberPartitionLedgerV1 L;
  L.weight_bytes = live[kLedgerWeights];
  L.kv_cache_bytes = live[kLedgerKv];
  L.activation_scratch_bytes = live[kLedgerActivation];
  L.module_storage_bytes = static_attn_module_bytes();
  L.allocator_overhead_bytes = live[kLedgerOverhead];
  L.transfer_staging_bytes = live[kLedgerStaging];
  L.concurrent_state_bytes = live[kLedgerConcurrent];
  return L;
}

}  // namespace faber

// ---------------------------------------------------------------------------
// extern "C": model + session
// ---------------------------------------------------------------------------
extern "C" {

#define FABER_EXPORT __attribute__((visibility("default")))

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_model_create(const FaberModelConfigV1* cfg,
                                                       FaberGpuModel** out) {
  using namespace faber;
  return guarded("faber_gpu_v2_model_create", [&] {
    FABER_ARG(cfg && out, "null pointer");
    validate_config(*cfg);
    auto m = std::make_unique<FaberGpuModel>();
    ModelState& M = m->s;
    M.cfg = *cfg;
    M.tp = (int)cfg->tp_size;
    M.rank = (int)cfg->tp_rank;
    FABER_CUDA(cudaGetDevice(&M.device));
    const TpPlan P = tp_plan(*cfg);
    M.Hl = P.Hl;
    M.Hkvl = P.Hkvl;
    M.Fl = P.Fl;
    M.f_blk0 = P.f_blk0;
    M.f_blk1 = P.f_blk1;
    M.v0 = P.v0;
    M.Vl = P.Vl;
    M.staged.resize(cfg->n_layers);
    if (M.tp > 1) {
      ncclUniqueId id;
      static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
      std::memcpy(&id, cfg->nccl_unique_id, 128);
      FABER_NCCL(ncclCommInitRank(&M.comm, M.tp, id, M.rank));
    }
    *out = m.release();
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_partition_plan(const FaberModelConfigV1* cfg,
                                                         uint32_t context_length, uint32_t sessions,
                                                         int32_t sms, FaberPartitionLedgerV1* out) {
  using namespace faber;
  return guarded("faber_gpu_v2_partition_plan", [&] {
    FABER_ARG(cfg && out, "null pointer");
    *out = partition_plan(*cfg, context_length, sessions, sms);
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_tp_step_plan(const FaberModelConfigV1* cfg, uint32_t position,
                                                       FaberTxnOpV1* ops, uint32_t cap, uint32_t* n_ops,
                                                       uint64_t* boundary_barrier, uint64_t* boundary_launches) {
  using namespace faber;
  return guarded("faber_gpu_v2_tp_step_plan", [&] {
    FABER_ARG(cfg && n_ops && boundary_barrier, "null pointer");
    std::vector<FaberTxnOpV1> v;
    std::vector<uint64_t> launches;
    uint64_t barrier = 0;
    tp_step_plan(*cfg, position, v, barrier, launches);
    *n_ops = (uint32_t)v.size();
    require(ops != nullptr && boundary_launches != nullptr && cap >= v.size(), FABER_STATUS_IO_ERROR,
            "plan needs " + std::to_string(v.size()) + " operations");
    std::copy(v.begin(), v.end(), ops);
    std::copy(launches.begin(), launches.end(), boundary_launches);
    *boundary_barrier = barrier;
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_tp_shard(const FaberModelConfigV1* cfg, const char* name,
                                                   uint64_t out[6]) {
  using namespace faber;
  return guarded("faber_gpu_v2_tp_shard", [&] {
    FABER_ARG(cfg && name && out, "null pointer");
    validate_config(*cfg);
    const ShardRange sr = tensor_shard(*cfg, tp_plan(*cfg), name);
    out[0] = sr.rows;
    out[1] = sr.cols;
    out[2] = sr.r0;
    out[3] = sr.nr;
    out[4] = sr.c0;
    out[5] = sr.nc;
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_model_set_tensor(FaberGpuModel* m, const char* name,
                                                           uint32_t type, const void* data,
                                                           uint64_t nbytes, uint64_t rows,
                                                           uint64_t cols) {
  using namespace faber;
  return guarded("faber_gpu_v2_model_set_tensor", [&] {
    FABER_ARG(m && name, "null pointer");
    model_set_tensor(m->s, name, type, data, nbytes, rows, cols);
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_model_finalize(FaberGpuModel* m) {
  using namespace faber;
  return guarded("faber_gpu_v2_model_finalize", [&] {
    FABER_ARG(m, "null model");
    model_finalize(m->s);
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_model_free(FaberGpuModel* m) {
  using namespace faber;
  return guarded("faber_gpu_v2_model_free", [&] {
    if (m) {
      cudaSetDevice(m->s.device);
      delete m;
    }
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_model_device_bytes(const FaberGpuModel* m,
                                                             uint64_t* bytes) {
  using namespace faber;
  return guarded("faber_gpu_v2_model_device_bytes", [&] {
    FABER_ARG(m && bytes, "null pointer");
    *bytes = m->s.device_bytes;
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_session_open(FaberGpuModel* m, const FaberKvLayoutV1* kv,
                                                       FaberGpuSession** out) {
  using namespace faber;
  return guarded("faber_gpu_v2_session_open", [&] {
    FABER_ARG(m && kv && out, "null pointer");
    auto s = std::make_unique<FaberGpuSession>();
    session_open(s->s, m, *kv);
    *out = s.release();
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_session_close(FaberGpuSession* s) {
  using namespace faber;
  return guarded("faber_gpu_v2_session_close", [&] { delete s; });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_session_reset(FaberGpuSession* s) {
  using namespace faber;
  return guarded("faber_gpu_v2_session_reset", [&] {
    FABER_ARG(s, "null session");
    SessionState& S = s->s;
    FABER_CUDA(cudaSetDevice(S.device));
    FABER_CUDA(cudaStreamSynchronize(S.stream));
    StepState st = {};
    FABER_CUDA(cudaMemcpy(&st, S.state.p, sizeof(st), cudaMemcpyDeviceToHost));
    const uint32_t epoch = st.tp_epoch;  // exchange epochs never repeat
    st = StepState{};
    st.finite = 1;
    st.tp_epoch = epoch;
    FABER_CUDA(cudaMemcpy(S.state.p, &st, sizeof(st), cudaMemcpyHostToDevice));
    S.n = 0;
    S.h_valid = false;
    S.prefix_pending = false;
    std::fill(S.prefix_layers.begin(), S.prefix_layers.end(), 0);
    S.c_position = 0;
    S.c_kv_generations = 0;
    S.c_history.clear();
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_session_truncate(FaberGpuSession* s, uint64_t n) {
  using namespace faber;
  return guarded("faber_gpu_v2_session_truncate", [&] {
    FABER_ARG(s, "null session");
    SessionState& S = s->s;
    FABER_ARG(n <= S.n, "truncate cannot lengthen the sequence (" + std::to_string(n) + " > " +
                            std::to_string(S.n) + ")");
    FABER_ARG(!S.prefix_pending || n >= S.prefix_n, "truncate cannot cut into an installed prefix");
    if (n == S.n) return;
    FABER_CUDA(cudaSetDevice(S.device));
    rollback_step(S, n);
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_session_set_wait_limit(FaberGpuSession* s, uint32_t polls) {
  using namespace faber;
  return guarded("faber_gpu_v2_session_set_wait_limit", [&] {
    FABER_ARG(s, "null session");
    SessionState& S = s->s;
    if (S.peer_wait_limit == polls) return;
    FABER_CUDA(cudaSetDevice(S.device));
    FABER_CUDA(cudaStreamSynchronize(S.stream));
    S.peer_wait_limit = polls;
    S.destroy_graphs();  // the limit is a kernel argument: capture again
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_session_exchange_epoch(FaberGpuSession* s, uint32_t raise_to,
                                                                uint32_t* epoch) {
  using namespace faber;
  return guarded("faber_gpu_v2_session_exchange_epoch", [&] {
    FABER_ARG(s, "null session");
    SessionState& S = s->s;
    FABER_CUDA(cudaSetDevice(S.device));
    FABER_CUDA(cudaStreamSynchronize(S.stream));
    StepState st;
    FABER_CUDA(cudaMemcpy(&st, S.state.p, sizeof(st), cudaMemcpyDeviceToHost));
    if (raise_to > st.tp_epoch) {  // never lowered: an epoch is used once
      st.tp_epoch = raise_to;
      FABER_CUDA(cudaMemcpy(S.state.p, &st, sizeof(st), cudaMemcpyHostToDevice));
    }
    if (epoch) *epoch = st.tp_epoch;
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_session_len(const FaberGpuSession* s, uint64_t* n) {
  using namespace faber;
  return guarded("faber_gpu_v2_session_len", [&] {
    FABER_ARG(s && n, "null pointer");
    *n = s->s.n;
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_session_push_token(FaberGpuSession* s, int64_t token) {
  using namespace faber;
  return guarded("faber_gpu_v2_session_push_token", [&] {
    FABER_ARG(s, "null session");
    run_push(s->s, &token, 1);
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_session_step_greedy(FaberGpuSession* s, int64_t token,
                                                             const int64_t* eog, uint32_t n_eog,
                                                             int64_t* next_token) {
  using namespace faber;
  return guarded("faber_gpu_v2_session_step_greedy", [&] {
    FABER_ARG(s && next_token, "null pointer");
    *next_token = run_step_greedy(s->s, token, eog, n_eog);
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_session_push_tokens(FaberGpuSession* s,
                                                              const int64_t* tokens, uint64_t n) {
  using namespace faber;
  return guarded("faber_gpu_v2_session_push_tokens", [&] {
    FABER_ARG(s && (tokens || n == 0), "null pointer");
    run_push(s->s, tokens, n);
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_session_position_logits(FaberGpuSession* s, float* logits,
                                                                  uint64_t cap) {
  using namespace faber;
  return guarded("faber_gpu_v2_session_position_logits", [&] {
    FABER_ARG(s, "null session");
    run_position_logits(s->s, logits, cap);
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_session_greedy(FaberGpuSession* s, uint32_t n_gen,
                                                         const int64_t* eog, uint32_t n_eog,
                                                         int64_t* out_tokens, int32_t* all_finite) {
  using namespace faber;
  return guarded("faber_gpu_v2_session_greedy", [&] {
    FABER_ARG(s && (eog || n_eog == 0), "null pointer");
    run_greedy(s->s, n_gen, eog, n_eog, out_tokens, all_finite);
  });
}

struct FaberGpuBatch {
  faber::BatchState b;
};

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_batch_open(FaberGpuSession* const* sessions, uint32_t n,
                                                    FaberGpuBatch** out) {
  using namespace faber;
  return guarded("faber_gpu_v2_batch_open", [&] {
    FABER_ARG(sessions && out, "null pointer");
    *out = nullptr;
    FABER_ARG(n >= 1 && n <= (uint32_t)kBatchMax,
              "a batch holds 1 to " + std::to_string(kBatchMax) + " sessions");
    std::vector<SessionState*> seqs(n);
    for (uint32_t i = 0; i < n; ++i) {
      FABER_ARG(sessions[i] != nullptr, "null session");
      seqs[i] = &sessions[i]->s;
    }
    auto b = std::make_unique<FaberGpuBatch>();
    batch_build(b->b, seqs.data(), (int)n);
    *out = b.release();
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_batch_greedy(FaberGpuBatch* b, uint32_t n_gen, const int64_t* eog,
                                                      uint32_t n_eog, int64_t* out_tokens,
                                                      int32_t* all_finite) {
  using namespace faber;
  return guarded("faber_gpu_v2_batch_greedy", [&] {
    FABER_ARG(b, "null batch");
    FABER_ARG(eog != nullptr || n_eog == 0, "null EOG list");
    run_batch_greedy(b->b, n_gen, eog, n_eog, out_tokens, all_finite);
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_batch_last_ms(const FaberGpuBatch* b, float* ms) {
  using namespace faber;
  return guarded("faber_gpu_v2_batch_last_ms", [&] {
    FABER_ARG(b && ms, "null pointer");
    *ms = b->b.last_ms;
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_batch_close(FaberGpuBatch* b) {
  using namespace faber;
  return guarded("faber_gpu_v2_batch_close", [&] { delete b; });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_session_set_prefix(FaberGpuSession* s, uint32_t layer,
                                                             const float* k, const float* v,
                                                             uint64_t n) {
  using namespace faber;
  return guarded("faber_gpu_v2_session_set_prefix", [&] {
    FABER_ARG(s, "null session");
    set_prefix(s->s, layer, k, v, n);
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_session_set_trace(FaberGpuSession* s, int32_t on) {
  using namespace faber;
  return guarded("faber_gpu_v2_session_set_trace", [&] {
    FABER_ARG(s, "null session");
    SessionState& S = s->s;
    ModelState& M = S.m->s;
    FABER_CUDA(cudaSetDevice(S.device));
    S.trace = on != 0;
    if (S.trace && !S.tr.p) {
      S.tr_w = (int)std::max<uint64_t>({M.cfg.d_model, (uint64_t)M.Fl,
                                        (uint64_t)M.Hl * M.cfg.head_dim});
      S.tr.alloc((size_t)M.cfg.n_layers * 8 * S.tr_w * 4);
      FABER_CUDA(cudaMemset(S.tr.p, 0, S.tr.n));
    }
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_session_trace(FaberGpuSession* s, uint32_t layer,
                                                        uint32_t which, float* out, uint64_t cap,
                                                        uint64_t* n) {
  using namespace faber;
  return guarded("faber_gpu_v2_session_trace", [&] {
    FABER_ARG(s && out && n, "null pointer");
    SessionState& S = s->s;
    ModelState& M = S.m->s;
    FABER_ARG(S.trace && S.tr.p, "tracing is off");
    FABER_ARG(layer < M.cfg.n_layers && which < 8, "bad trace index");
    const uint64_t hd = M.cfg.head_dim;
    const uint64_t sizes[8] = {M.cfg.d_model, (uint64_t)M.Hl * hd, (uint64_t)M.Hkvl * hd,
                               (uint64_t)M.Hkvl * hd, (uint64_t)M.Hl * hd, M.cfg.d_model,
                               (uint64_t)M.Fl, M.cfg.d_model};
    const uint64_t cnt = sizes[which];
    require(cap >= cnt, FABER_STATUS_IO_ERROR, "trace buffer too small");
    FABER_CUDA(cudaSetDevice(S.device));
    FABER_CUDA(cudaStreamSynchronize(S.stream));
    FABER_CUDA(cudaMemcpy(out, S.tr.as<float>() + ((size_t)layer * 8 + which) * S.tr_w, cnt * 4,
                          cudaMemcpyDeviceToHost));
    *n = cnt;
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_session_last_greedy_ms(const FaberGpuSession* s,
                                                                 float* ms) {
  using namespace faber;
  return guarded("faber_gpu_v2_session_last_greedy_ms", [&] {
    FABER_ARG(s && ms, "null pointer");
    *ms = s->s.last_greedy_ms;
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_session_commit(FaberGpuSession* s, int64_t token,
                                                         uint32_t position, uint64_t kv_generation,
                                                         uint64_t publication_boundary,
                                                         int32_t* outcome) {
  using namespace faber;
  return guarded("faber_gpu_v2_session_commit", [&] {
    FABER_ARG(s && outcome, "null pointer");
    SessionState& S = s->s;
    // SequenceState::commit (src/session.rs:422-456), in its order.
    FABER_ARG(publication_boundary != 0, "no publication boundary: nothing publishes");
    if (!S.c_history.empty() && position + 1 == S.c_position &&
        kv_generation == S.c_kv_generations && S.c_history.back() == token) {
      *outcome = 1;  // idempotent replay
      return;
    }
    FABER_ARG(position == S.c_position, "out-of-order position: expected " +
                                            std::to_string(S.c_position) + ", attempted " +
                                            std::to_string(position));
    FABER_ARG(kv_generation == S.c_kv_generations + 1,
              "KV generation gap: expected " + std::to_string(S.c_kv_generations + 1) +
                  ", attempted " + std::to_string(kv_generation));
    S.c_history.push_back(token);
    S.c_position += 1;
    S.c_kv_generations += 1;
    *outcome = 0;
  });
}

FABER_EXPORT FaberRtStatusV1 faber_gpu_v2_nccl_unique_id(uint8_t out[128]) {
  using namespace faber;
  return guarded("faber_gpu_v2_nccl_unique_id", [&] {
    FABER_ARG(out, "null pointer");
    ncclUniqueId id;
    FABER_NCCL(ncclGetUniqueId(&id));
    std::memcpy(out, &id, 128);
  });
}

}  // extern "C"
