/* faber_gpu.h — C ABI of the B200 (sm_100a) Q4_K decoder path.
 *
 * Every entry point returns FaberRtStatusV1 by value, never throws or
 * unwinds across the boundary, and takes plain pointers and sizes (no torch
 * or C++ types). Status conventions follow faber-runtime's host ABI
 * (src/host_abi.rs:313-323, 378-389): OK 0, INVALID_ARGUMENT 1, IO_ERROR 2,
 * PANIC 3 (an internal C++ exception, the analogue of catch_unwind ->
 * STATUS_PANIC in hosts/llvm/src/gpu_placement.rs:29-31), UNSUPPORTED 4,
 * FALLIBLE 5. Codes >= 16 are the device-runtime failures named by the
 * reference's backend error taxonomy
 * (src/execution_transaction/backend.rs:17-54). The message of the last
 * failure on the calling thread is available from faber_gpu_v2_last_error.
 *
 * Threading: one process may drive several devices; calls on one model or
 * session must be serialized by the caller (the reference's per-session
 * rule, src/session.rs:625). The placement ABI (v1 symbols) is guarded by
 * one process-wide mutex like hosts/llvm/src/gpu_placement.rs:27.
 */
#ifndef FABER_GPU_H
#define FABER_GPU_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct FaberRtStatusV1 {
  int32_t code;
} FaberRtStatusV1;

enum {
  FABER_STATUS_OK = 0,
  FABER_STATUS_INVALID_ARGUMENT = 1,
  FABER_STATUS_IO_ERROR = 2,
  FABER_STATUS_PANIC = 3,
  FABER_STATUS_UNSUPPORTED = 4,
  FABER_STATUS_FALLIBLE = 5,
  FABER_STATUS_TIMEOUT = 16,
  FABER_STATUS_DEVICE_LOSS = 17,
  FABER_STATUS_CANCELLED = 18,
  FABER_STATUS_ALLOCATION = 19,
  FABER_STATUS_CUDA_ERROR = 20,
  FABER_STATUS_KERNEL_ERROR = 21,
  /* admission refused: the declared ledger exceeds the partition's safe
   * limit (AdmissionError::BudgetExceeded, src/partition.rs:236-247) */
  FABER_STATUS_BUDGET_EXCEEDED = 22
};

/* GGUF dtype ids of the admitted tensor types (src/gguf.rs:135-144). */
enum {
  FABER_GGML_F32 = 0,
  FABER_GGML_Q5_0 = 6,
  FABER_GGML_Q8_0 = 8,
  FABER_GGML_Q4_K = 12,
  FABER_GGML_Q6_K = 14
};

typedef struct FaberGpuModel FaberGpuModel;
typedef struct FaberGpuSession FaberGpuSession;
typedef struct FaberGpuBatch FaberGpuBatch;
typedef struct FaberGguf FaberGguf;

/* One tensor of a parsed GGUF file. dims are in GGML order (dims[0] is the
 * contiguous one: a row's length); unused dims are 1. The data is
 * bytes[offset, offset + nbytes) of the parsed buffer. */
typedef struct FaberGgufTensorV1 {
  char name[256];
  uint32_t ggml_type;
  uint32_t n_dims;
  uint64_t dims[4];
  uint64_t elements;
  uint64_t nbytes;
  uint64_t offset;
} FaberGgufTensorV1;

/* ------------------------------------------------------------------------
 * Library / diagnostics
 * ------------------------------------------------------------------------ */

/* ABI version of this header (2). */
uint32_t faber_gpu_v2_abi_version(void);

/* Copy the last failure message of the calling thread (NUL-terminated,
 * truncated to cap). */
FaberRtStatusV1 faber_gpu_v2_last_error(char* buf, uint64_t cap);

/* Select the CUDA device for subsequent calls on this thread and check that
 * it is an sm_100 part. */
FaberRtStatusV1 faber_gpu_v2_init(int32_t device_ordinal);

/* Host-side fault table (test support): the next `count` calls to the entry
 * point named `entry` fail with `status` before any device work is issued,
 * mirroring the fault classes of src/fake_device.rs:44-75. count 0 clears. */
FaberRtStatusV1 faber_gpu_v2_fault_inject(const char* entry, int32_t status, uint32_t count);

/* ------------------------------------------------------------------------
 * Placement ABI — replaces hosts/llvm/src/gpu_placement.rs:53-137
 * (__faber_gpu_v1_copy_in / readback / sync), now backed by device memory on
 * the current device. Same argument meaning and error behaviour: a null
 * pointer with a nonzero length is INVALID_ARGUMENT, an unknown id is
 * INVALID_ARGUMENT, a too-small destination is IO_ERROR, copy_in replaces an
 * existing buffer.
 * ------------------------------------------------------------------------ */
FaberRtStatusV1 __faber_gpu_v1_copy_in(uint64_t logical_id, const uint8_t* data_ptr,
                                       uint64_t data_len, uint32_t dtype);
FaberRtStatusV1 __faber_gpu_v1_readback(uint64_t logical_id, uint8_t* dest_ptr,
                                        uint64_t dest_capacity, uint64_t* actual_len);
FaberRtStatusV1 __faber_gpu_v1_sync(uint64_t logical_id);
/* Device address and length of a placed buffer (for the kernels below). */
FaberRtStatusV1 faber_gpu_v2_buffer_device_ptr(uint64_t logical_id, void** dev_ptr,
                                               uint64_t* len);

/* ------------------------------------------------------------------------
 * Stateless kernels on device pointers. `stream` is a cudaStream_t (NULL:
 * the legacy default stream). All are asynchronous.
 * ------------------------------------------------------------------------ */

/* dequant_row for Q4_K — src/dequant.rs:194-217 via :323-340: n_blocks
 * native 144-byte super-blocks -> 256*n_blocks f32. f16_round != 0 applies
 * the oracle's weight rounding f32->f16(RN)->f32 (src/cpu_oracle.rs:356-360).
 * Bit-exact with the reference. */
FaberRtStatusV1 faber_gpu_v2_dequant_q4k(const uint8_t* blocks, uint64_t n_blocks, float* out,
                                         int32_t f16_round, void* stream);
/* Every admitted block type (dequant_q8_0 / dequant_q5_0 / dequant_q4_k /
 * dequant_q6_k, src/dequant.rs:151-255, and F32/F16), bit-exact: n_blocks
 * blocks of ggml_type on the device -> f32 (f16-rounded if f16_round). */
FaberRtStatusV1 faber_gpu_v2_dequant_blocks(uint32_t ggml_type, const uint8_t* blocks,
                                            uint64_t n_blocks, float* out, int32_t f16_round,
                                            void* stream);
/* A linear of any admitted block type (Q4_K, Q6_K, Q5_0, Q8_0, F32, F16),
 * uploaded as typed rows, and y = dense(W, x) through the row GEMV that
 * serves the decoder's non-Q4_K linears (dense, src/decoder_ops.rs:378-406,
 * with f16-rounded weights, src/cpu_oracle.rs:356-360). */
typedef struct FaberGpuTypedTensor FaberGpuTypedTensor;
FaberRtStatusV1 faber_gpu_v2_typed_upload(uint32_t ggml_type, const uint8_t* host_blocks,
                                          uint64_t nbytes, uint64_t rows, uint64_t cols,
                                          FaberGpuTypedTensor** out);
FaberRtStatusV1 faber_gpu_v2_typed_gemv(const FaberGpuTypedTensor* t, const float* x, float* y,
                                        void* stream);
FaberRtStatusV1 faber_gpu_v2_typed_free(FaberGpuTypedTensor* t);

/* f32 -> f16 (round-to-nearest-even) -> f32, element-wise: kv_f16_round
 * (src/cpu_oracle.rs:225-294). */
FaberRtStatusV1 faber_gpu_v2_f16_round(const float* x, float* y, uint64_t n, void* stream);

/* dense over a Q4_K weight — src/decoder_ops.rs:378-406 applied to the
 * f16-rounded dequantized weight (src/cpu_oracle.rs:302-360):
 * y[j] = sum_i w[j][i] * x[i], w given as rows*cols/256 native super-blocks
 * in GGUF order (row j = elements [j*cols, (j+1)*cols) of the flat tensor;
 * cols must be a multiple of 32). The weight is repacked into the kernel's
 * tile layout on every call (a scratch allocation); the model API uploads
 * once instead. */
FaberRtStatusV1 faber_gpu_v2_gemv_q4k(const uint8_t* w_blocks, uint64_t rows, uint64_t cols,
                                      const float* x, float* y, void* stream);

/* A Q4_K weight resident on the device in the repacked tile layout
 * (the reference's Declared repack identity, src/quantized_tensor_layout.rs:
 * 269-278,483-487). Created from native GGUF bytes on the host. */
typedef struct FaberGpuQ4kTensor FaberGpuQ4kTensor;
FaberRtStatusV1 faber_gpu_v2_q4k_upload(const uint8_t* host_blocks, uint64_t nbytes,
                                        uint64_t rows, uint64_t cols, FaberGpuQ4kTensor** out);
FaberRtStatusV1 faber_gpu_v2_q4k_free(FaberGpuQ4kTensor* t);
/* y = dense(w, x) with the resident weight (x, y device pointers). */
FaberRtStatusV1 faber_gpu_v2_q4k_gemv(const FaberGpuQ4kTensor* t, const float* x, float* y,
                                      void* stream);
/* Validation surface of the tensor-parallel exchange (the row-parallel
 * all-reduce of src/partition.rs's plan, fused into the next GEMV): with
 * the resident weight, x_sum = x + sum over r < tp of exchange[r] (rank
 * order) and y = dense(w, rms_norm(x_sum) * norm_w), where exchange is a
 * device array [tp][cols] of 8-byte words (epoch << 32 | f32 bits) and a
 * word counts only once it carries `epoch`. A word that never does makes the
 * kernel's bounded wait give up after wait_limit polls (0: the default): the
 * call then returns TIMEOUT and the device stays usable. Synchronizes
 * `stream`; calls must not overlap (they share two device words). */
FaberRtStatusV1 faber_gpu_v2_q4k_gemv_exchange(const FaberGpuQ4kTensor* t, const float* x,
                                               const float* norm_w, float eps, const uint64_t* exchange,
                                               uint32_t tp, uint32_t epoch, uint32_t wait_limit,
                                               float* x_sum_out, float* y, void* stream);
/* Batched dense over the resident weight, the per-sequence linear of a
 * batched decode step (src/decoder_ops.rs:378-406 for each of `batch`
 * inputs): y[b] = dense(w, x[b]) for b < batch <= 16, x [batch][cols] and
 * y [batch][rows] f32 device arrays. Every exact weight fragment is formed
 * once for all sequences. Rows must be in whole super-blocks. The tensor
 * keeps its scratch after the first call; calls on one tensor must not
 * overlap. */
FaberRtStatusV1 faber_gpu_v2_q4k_gemv_batch(FaberGpuQ4kTensor* t, const float* x, uint32_t batch,
                                            float* y, void* stream);
/* Dequantize the resident (repacked) weight back to [rows][cols] f32 —
 * proves the repack is value-identical to dequant_tensor. */
FaberRtStatusV1 faber_gpu_v2_q4k_dequant_rows(const FaberGpuQ4kTensor* t, float* out,
                                              int32_t f16_round, void* stream);
/* Repack identity (a 64-bit hash of the layout parameters and source bytes). */
FaberRtStatusV1 faber_gpu_v2_q4k_repack_hash(const FaberGpuQ4kTensor* t, uint64_t* hash);

/* ------------------------------------------------------------------------
 * Model + session — the device analogue of CpuOracle / ForwardRun /
 * run_greedy (src/cpu_oracle.rs:409-445, 808-926; src/greedy_run.rs:186-248)
 * under the session contract of src/session.rs and the KV layout of
 * src/kv_cache.rs.
 * ------------------------------------------------------------------------ */

typedef struct FaberModelConfigV1 {
  uint32_t n_layers;
  uint32_t d_model;
  uint32_t n_heads;
  uint32_t n_kv_heads;
  uint32_t head_dim;
  uint32_t ffn;
  uint32_t vocab;
  uint32_t tied_head; /* 1: logits use token_embd (no output.weight) */
  float rms_eps;
  float rope_theta;
  /* tensor parallelism: this process is rank tp_rank of tp_size. tp_size 1
   * is single-GPU. For tp_size > 1, nccl_unique_id holds the 128-byte
   * ncclUniqueId shared by the group. */
  uint32_t tp_size;
  uint32_t tp_rank;
  uint8_t nccl_unique_id[128];
} FaberModelConfigV1;

/* KvCacheLayout — src/kv_cache.rs:504-626. dtype 0 = f32 (the reference's
 * only admitted dtype), 1 = f16 (value-identical: every cached K/V is an
 * f16-rounded value, src/cpu_oracle.rs:598-601). */
typedef struct FaberKvLayoutV1 {
  uint32_t slots;
  uint32_t context_length;
  uint32_t layer_count;
  uint32_t kv_head_count;
  uint32_t head_dim;
  uint32_t dtype;
  uint64_t reserve_bytes;
} FaberKvLayoutV1;

/* Storage and admitted bytes of a layout (KvCacheLayout::total_bytes /
 * admitted_bytes, src/kv_cache.rs:605-626). A zero dimension is
 * INVALID_ARGUMENT (KvCacheLayout::new returns None), overflow is IO_ERROR. */
FaberRtStatusV1 faber_gpu_v2_kv_layout_bytes(const FaberKvLayoutV1* layout, uint64_t* total,
                                             uint64_t* admitted);

/* One partition's device bytes by class: PartitionBudgetLedger
 * (src/partition.rs:111-155), classes 1-7 in field order; class 8 of the
 * reference's admission equation is the safe limit passed beside it. */
typedef struct FaberPartitionLedgerV1 {
  uint64_t weight_bytes;             /* 1: weights, including repack */
  uint64_t kv_cache_bytes;           /* 2: KV cache */
  uint64_t activation_scratch_bytes; /* 3: activations and operation scratch */
  uint64_t module_storage_bytes;     /* 4: module-resident device storage */
  uint64_t allocator_overhead_bytes; /* 5: allocator granularity */
  uint64_t transfer_staging_bytes;   /* 6: exchange and staging buffers */
  uint64_t concurrent_state_bytes;   /* 7: per-request state (tokens, positions) */
} FaberPartitionLedgerV1;

/* Admission of a declared ledger against a policy limit
 * (VirtualDevicePartition::admit, src/partition.rs:293-315): OK when the
 * checked sum of the seven classes is at most safe_limit_bytes, else
 * BUDGET_EXCEEDED, also when the sum overflows (then *total_out is
 * UINT64_MAX). Arithmetic only: nothing is allocated, no device is needed. */
FaberRtStatusV1 faber_gpu_v2_partition_admit(const FaberPartitionLedgerV1* declared,
                                             uint64_t safe_limit_bytes, uint64_t* total_out);

/* The bytes this library holds on a device, by class. Every device buffer is
 * charged to one class when it is allocated and credited back when freed.
 * Class 5 is this library's allocator policy: a buffer below 1 MiB is
 * charged in 512-byte units and a larger one in 2 MiB units, and the
 * rounding is class 5. Class 4 is the allocation-free attention scratch of
 * the module image, counted once the device holds any buffer. Arithmetic on
 * host counters only (no device call). Device ordinals 0-63. */
FaberRtStatusV1 faber_gpu_v2_partition_usage(int32_t device, FaberPartitionLedgerV1* out);

/* Sets a device's policy limit in bytes (0 removes it). While a limit is
 * set, an allocation whose charge would take the device's total (classes
 * 1-7) above it fails with ALLOCATION before cudaMalloc runs: growth after
 * admission is an allocation outcome, never a ledger rewrite
 * (src/partition.rs:111-114). A limit below what the device already holds
 * is BUDGET_EXCEEDED and leaves the previous limit in place. */
FaberRtStatusV1 faber_gpu_v2_partition_set_limit(int32_t device, uint64_t safe_limit_bytes);

/* The ledger of one tensor-parallel rank (cfg->tp_size, cfg->tp_rank) before
 * anything is allocated, for the admission check: the model's Q4_K linears
 * in their tiled layout, the f16 embedding and the norms, then `sessions`
 * sessions of context_length positions (KV cache, step buffers, and the
 * prompt pass's scratch where that pass runs), with the attention split
 * count of a device with `sms` SMs. Every buffer is charged by the allocator
 * policy of faber_gpu_v2_partition_usage, so a model and its sessions built
 * from Q4_K tensors hold exactly this ledger. Host-only. */
FaberRtStatusV1 faber_gpu_v2_partition_plan(const FaberModelConfigV1* cfg, uint32_t context_length,
                                            uint32_t sessions, int32_t sms,
                                            FaberPartitionLedgerV1* out);

/* --- execution transaction (src/execution_transaction/transaction.rs) ------
 * prepare / execute / commit / abort of an operation plan over the ranks of
 * a group (partitions 0-63). Lifecycle calls return OK, INVALID_ARGUMENT for
 * a contract violation (wrong state, unknown partition, duplicate or
 * undeclared operation, missing admitted budget, an operation outside the
 * accepted snapshot, abort after commit), BUDGET_EXCEEDED when a
 * reservation exceeds an admitted class, FALLIBLE when commit finds the
 * boundary not yet reached (nothing published; commit may be called
 * again), and for a backend failure the code of its class: ALLOCATION,
 * KERNEL_ERROR (an operation or transfer error), DEVICE_LOSS, CANCELLED or
 * TIMEOUT. faber_gpu_v2_txn_last_error gives the error's kind. */
typedef struct FaberTxn FaberTxn;
typedef struct FaberTxnBackend FaberTxnBackend;

enum { FABER_TXN_LAUNCH = 0, FABER_TXN_TRANSFER = 1, FABER_TXN_BROADCAST = 2, FABER_TXN_BARRIER = 3 };

/* One operation (TransactionOperation, mirror.rs:635-656); identity is
 * (kind, ref). launch: partition, bytes = output bytes; transfer: partition
 * = source, destination, bytes; broadcast: partition = source, participants
 * mask, bytes; barrier: participants mask. */
typedef struct FaberTxnOpV1 {
  uint32_t kind;
  uint32_t partition;
  uint32_t destination;
  uint32_t reserved;
  uint64_t participants;
  uint64_t ref;
  uint64_t bytes;
} FaberTxnOpV1;

/* A partition of the bound plan and its admitted ledger (admitted = 0: none,
 * which prepare refuses for a partition an operation uses). */
typedef struct FaberTxnPartitionV1 {
  uint32_t partition;
  uint32_t admitted;
  FaberPartitionLedgerV1 ledger;
} FaberTxnPartitionV1;

/* TransactionReceipt figures (receipt.rs). decision 0 none, 1 committed,
 * 2 aborted; state 0 New, 1 Prepared, 2 Executing, 3 Committed, 4 Failed,
 * 5 Aborted; failure_kind 0 none, 1 backend, 2 publish failed, 3 cancelled;
 * failure_class 1 allocation, 2 operation, 3 device loss, 4 cancelled,
 * 5 timeout. Partition sets are masks. */
typedef struct FaberTxnReceiptV1 {
  int32_t decision;
  int32_t state;
  int32_t failure_kind;
  int32_t failure_class;
  uint32_t failure_partition;
  uint32_t published;
  uint64_t publication_ordinal;
  uint64_t declared_write_bytes;
  uint64_t executed_operations;
  uint64_t executed_bytes;
  uint64_t completed_events;
  uint64_t staged_bytes;
  uint64_t published_bytes;
  uint64_t released_partitions;
  uint64_t retired_partitions;
  uint32_t partial_publication;
  uint32_t reserved;
  uint64_t prepare_ns;
  uint64_t execute_ns;
  uint64_t finalize_ns;
} FaberTxnReceiptV1;

/* The last lifecycle error (errors.rs): kind 0 none, 1 DegeneratePlan,
 * 2 EmptySnapshot, 3 InvalidState, 4 UnknownPartition, 5 DuplicateOperation,
 * 6 UndeclaredBoundaryBarrier, 7 UndeclaredBoundaryLaunch,
 * 8 MissingAdmittedBudget, 9 ReservationExceedsBudget (budget_class 6 or 3),
 * 10 Backend, 11 OperationOutsideSnapshot, 12 BoundaryNotReached (missing =
 * boundary refs pending), 13 PublishFailed, 14 AlreadyCommitted. */
typedef struct FaberTxnErrorV1 {
  int32_t kind;
  uint32_t partition;
  int32_t backend_class;
  int32_t budget_class;
  uint64_t missing;
} FaberTxnErrorV1;

/* ExecutionTransaction::new: INVALID_ARGUMENT for fewer than two partitions
 * (DegeneratePlan) or no operations (EmptySnapshot). */
FaberRtStatusV1 faber_gpu_v2_txn_create(const FaberTxnPartitionV1* partitions, uint32_t n_partitions,
                                        const FaberTxnOpV1* ops, uint32_t n_ops,
                                        const uint64_t* boundary_barriers, uint32_t n_barriers,
                                        const uint64_t* boundary_launches, uint32_t n_launches,
                                        FaberTxn** out);
FaberRtStatusV1 faber_gpu_v2_txn_prepare(FaberTxn* t, FaberTxnBackend* b);
FaberRtStatusV1 faber_gpu_v2_txn_execute(FaberTxn* t, FaberTxnBackend* b);
FaberRtStatusV1 faber_gpu_v2_txn_execute_operation(FaberTxn* t, FaberTxnBackend* b, const FaberTxnOpV1* op);
FaberRtStatusV1 faber_gpu_v2_txn_commit(FaberTxn* t, FaberTxnBackend* b, uint64_t publication_ordinal);
FaberRtStatusV1 faber_gpu_v2_txn_abort(FaberTxn* t, FaberTxnBackend* b, const char* reason);
FaberRtStatusV1 faber_gpu_v2_txn_receipt(const FaberTxn* t, FaberTxnReceiptV1* out);
FaberRtStatusV1 faber_gpu_v2_txn_last_error(const FaberTxn* t, FaberTxnErrorV1* out);
/* Reservation held for a partition after prepare: staging (class 6),
 * output, event and scratch bytes (class 3). */
FaberRtStatusV1 faber_gpu_v2_txn_reservation(const FaberTxn* t, uint32_t partition, uint64_t out[4]);
FaberRtStatusV1 faber_gpu_v2_txn_free(FaberTxn* t);

/* The fault-injecting host backend (src/fake_device.rs:184-318): the
 * happy-path fake plus one-shot faults per (operation, partition). Fault
 * classes: 1 cancel, 2 timeout, 3 transfer error, 4 kernel error, 5 device
 * loss. Injection is on the host; no device is touched. */
typedef struct FaberTxnBackendInfoV1 {
  uint64_t reserved_partitions; /* mask of partitions holding a reservation */
  uint64_t released_partitions;
  uint64_t retired_partitions;
  uint64_t staged_bytes;
  uint64_t published_bytes;
  uint64_t committed_bytes; /* the last successful publication */
  uint64_t executed_operations;
  uint64_t pending_events; /* dispatched, not yet completed */
  uint64_t delivered_faults;
  uint64_t reclaimed_copy_bytes;
} FaberTxnBackendInfoV1;

FaberRtStatusV1 faber_gpu_v2_txn_backend_fake(FaberTxnBackend** out);
FaberRtStatusV1 faber_gpu_v2_txn_backend_inject(FaberTxnBackend* b, uint32_t op_kind, uint64_t ref,
                                                uint32_t partition, int32_t fault_class);
FaberRtStatusV1 faber_gpu_v2_txn_backend_fail_publish(FaberTxnBackend* b, int32_t backend_class);
FaberRtStatusV1 faber_gpu_v2_txn_backend_set_auto_complete(FaberTxnBackend* b, int32_t on);
FaberRtStatusV1 faber_gpu_v2_txn_backend_complete_event(FaberTxnBackend* b, uint32_t op_kind,
                                                        uint32_t partition, uint64_t ref);
FaberRtStatusV1 faber_gpu_v2_txn_backend_info(const FaberTxnBackend* b, FaberTxnBackendInfoV1* out);
FaberRtStatusV1 faber_gpu_v2_txn_backend_free(FaberTxnBackend* b);

/* One decode step of the tensor-parallel group cfg->tp_size (>= 2) as a
 * transaction plan over its ranks: per rank a launch (its step; published
 * output the position's K/V rows of its kv heads and the token), then a
 * barrier over all ranks (the step's exchanges, whose partials are consumed
 * inside the step through the session's exchange buffer). The commit
 * boundary is the barrier and the tp_size launches.
 * *n_ops is always set; with cap below it the call is IO_ERROR and writes
 * nothing else. boundary_launches holds tp_size references. Host-only. */
FaberRtStatusV1 faber_gpu_v2_tp_step_plan(const FaberModelConfigV1* cfg, uint32_t position,
                                          FaberTxnOpV1* ops, uint32_t cap, uint32_t* n_ops,
                                          uint64_t* boundary_barrier, uint64_t* boundary_launches);

FaberRtStatusV1 faber_gpu_v2_model_create(const FaberModelConfigV1* cfg, FaberGpuModel** out);
/* Upload one tensor by its GGUF name (token_embd.weight, output_norm.weight,
 * output.weight, blk.N.{attn_norm,attn_q,attn_k,attn_v,attn_output,ffn_norm,
 * ffn_gate,ffn_up,ffn_down}.weight). rows = out_features, cols =
 * in_features (1 for vectors). The byte count must be exactly the packed
 * size (src/dequant.rs:323-333, RowBytesMismatch -> INVALID_ARGUMENT). With
 * tp_size > 1 every rank passes the full tensor and keeps its shard. */
FaberRtStatusV1 faber_gpu_v2_model_set_tensor(FaberGpuModel* m, const char* name,
                                              uint32_t ggml_type, const void* host_data,
                                              uint64_t nbytes, uint64_t rows, uint64_t cols);
/* This rank's block of a named tensor under tensor parallelism (host only,
 * no device call): out = {rows, cols, r0, nr, c0, nc}, the full shape and the
 * rows [r0, r0+nr) x cols [c0, c0+nc) that rank cfg->tp_rank keeps. Q/K/V
 * split by head, gate/up by FFN super-block and output by vocab row
 * (column-parallel); attn_output and ffn_down by the matching input columns
 * (row-parallel, summed across ranks). Vectors and the embedding are whole.
 * The reference partitions devices (src/partition.rs:115-417) but has no
 * tensor-parallel plan; this is the plan model_set_tensor applies. */
FaberRtStatusV1 faber_gpu_v2_tp_shard(const FaberModelConfigV1* cfg, const char* name,
                                      uint64_t out[6]);
/* Check coverage (every tensor present, src/cpu_oracle.rs:409-445) and
 * build the per-model device state. */
FaberRtStatusV1 faber_gpu_v2_model_finalize(FaberGpuModel* m);
FaberRtStatusV1 faber_gpu_v2_model_free(FaberGpuModel* m);
/* Bytes of weights resident on this device. */
FaberRtStatusV1 faber_gpu_v2_model_device_bytes(const FaberGpuModel* m, uint64_t* bytes);

FaberRtStatusV1 faber_gpu_v2_session_open(FaberGpuModel* m, const FaberKvLayoutV1* kv,
                                          FaberGpuSession** out);
FaberRtStatusV1 faber_gpu_v2_session_close(FaberGpuSession* s);
/* Forget every position (a new sequence epoch; weights stay resident). */
FaberRtStatusV1 faber_gpu_v2_session_reset(FaberGpuSession* s);
FaberRtStatusV1 faber_gpu_v2_session_len(const FaberGpuSession* s, uint64_t* n);
/* Shorten the sequence to n positions (n <= the current length, not into an
 * installed prefix): the one-position rollback of a step whose group
 * aborted (src/execution_transaction/transaction.rs:427-488 pairs an abort
 * with no token commit, src/session.rs:422-456). The K/V rows past n stay
 * in memory and are overwritten by the next pushes; the session needs a
 * push before its next logits. A step whose device work fails with TIMEOUT
 * or KERNEL_ERROR is rolled back the same way by the call itself. */
FaberRtStatusV1 faber_gpu_v2_session_truncate(FaberGpuSession* s, uint64_t n);
/* Polls before a tensor-parallel peer wait or grid-barrier wait of this
 * session's kernels gives up and the step returns TIMEOUT (0: the default,
 * 2^20 polls, well under a second). Mirrors the bounded waits behind
 * BackendError::Timeout (src/execution_transaction/backend.rs:17-54). */
FaberRtStatusV1 faber_gpu_v2_session_set_wait_limit(FaberGpuSession* s, uint32_t polls);
/* The session's tensor-parallel exchange epoch (one per launched step): the
 * current value in *epoch, after raising it to raise_to when that is
 * larger (never lowered, so no epoch is used twice). After a group abort
 * the ranks raise every session to the largest epoch of the group, so that
 * their next exchanges match again. */
FaberRtStatusV1 faber_gpu_v2_session_exchange_epoch(FaberGpuSession* s, uint32_t raise_to,
                                                    uint32_t* epoch);
/* ForwardRun::push_token (src/cpu_oracle.rs:859-912): append one token.
 * A token outside [0, vocab) or a full context is INVALID_ARGUMENT / IO_ERROR
 * and leaves the session unchanged. */
FaberRtStatusV1 faber_gpu_v2_session_push_token(FaberGpuSession* s, int64_t token);
/* Append n tokens (the prompt) — same as n push_token calls. */
FaberRtStatusV1 faber_gpu_v2_session_push_tokens(FaberGpuSession* s, const int64_t* tokens,
                                                 uint64_t n);
/* One step of a host-driven greedy loop (run_greedy's step,
 * src/greedy_run.rs:186-248, with the host choosing each input): push
 * `token`, then write the argmax of the new position's logits over the ids
 * not in eog[0..n_eog) (top1_non_eog, src/cpu_oracle.rs:980-1016) to
 * *next_token. Only those 8 bytes leave the device; the ids equal
 * session_greedy's. Errors as push_token. */
FaberRtStatusV1 faber_gpu_v2_session_step_greedy(FaberGpuSession* s, int64_t token, const int64_t* eog,
                                                 uint32_t n_eog, int64_t* next_token);
/* ForwardRun::position_logits (src/cpu_oracle.rs:920-926): full-vocab raw
 * logits at the sequence end into a host buffer of cap floats. */
FaberRtStatusV1 faber_gpu_v2_session_position_logits(FaberGpuSession* s, float* logits,
                                                     uint64_t cap);
/* run_greedy's loop (src/greedy_run.rs:186-248): n_gen steps of
 * logits -> argmax over non-EOG ids (lowest id wins ties,
 * src/cpu_oracle.rs:979-995) -> feed back. Tokens go to out_tokens (host);
 * *all_finite receives the finite gate over every step's logits. The token
 * stays on the device between steps. */
FaberRtStatusV1 faber_gpu_v2_session_greedy(FaberGpuSession* s, uint32_t n_gen,
                                            const int64_t* eog, uint32_t n_eog,
                                            int64_t* out_tokens, int32_t* all_finite);
/* GGUF v3 reader — the structural admission of src/gguf.rs:581-812 without
 * its pin on one file (no SHA-256, size or count expectations):
 *   - magic and version 3;
 *   - counts bounded by the bytes left;
 *   - length-capped UTF-8 keys, strings and names; unique keys and names;
 *   - BOOL 0/1; no nested arrays;
 *   - 1..4 dims, overflow-checked sizes;
 *   - admitted dtypes F32, F16, Q5_0, Q8_0, Q4_K, Q6_K, in whole blocks;
 *   - aligned, sequential, non-overlapping ranges inside the buffer.
 * The first violation returns INVALID_ARGUMENT, and last_error names the
 * reference's AdmissionError kind. The reader keeps offsets only; the
 * caller keeps the bytes alive while it reads tensors. */
FaberRtStatusV1 faber_gpu_v2_gguf_parse(const uint8_t* bytes, uint64_t len, FaberGguf** out);
FaberRtStatusV1 faber_gpu_v2_gguf_info(const FaberGguf* g, uint32_t* version, uint64_t* n_kv,
                                       uint64_t* n_tensors, uint64_t* data_offset,
                                       uint64_t* alignment);
FaberRtStatusV1 faber_gpu_v2_gguf_tensor(const FaberGguf* g, uint64_t index,
                                         FaberGgufTensorV1* out);
/* KV index -> key (NUL-terminated into key_cap bytes; IO_ERROR if short),
 * value type, and for arrays the element type and count. */
FaberRtStatusV1 faber_gpu_v2_gguf_kv(const FaberGguf* g, uint64_t index, char* key,
                                     uint64_t key_cap, uint32_t* type, uint32_t* arr_type,
                                     uint64_t* arr_count);
/* Scalar metadata by key: any integer type or BOOL, F32/F64, STRING. A
 * missing key or another type is INVALID_ARGUMENT. */
FaberRtStatusV1 faber_gpu_v2_gguf_get_int(const FaberGguf* g, const char* key, int64_t* v);
FaberRtStatusV1 faber_gpu_v2_gguf_get_float(const FaberGguf* g, const char* key, double* v);
FaberRtStatusV1 faber_gpu_v2_gguf_get_string(const FaberGguf* g, const char* key, char* buf,
                                             uint64_t cap, uint64_t* len);
FaberRtStatusV1 faber_gpu_v2_gguf_free(FaberGguf* g);
/* The buffer offset of an array KV's first element (strings: a u64 length,
 * then the bytes, back to back), for reading arrays such as the tokenizer's
 * from the parsed bytes. INVALID_ARGUMENT for a non-array KV. */
FaberRtStatusV1 faber_gpu_v2_gguf_kv_payload(const FaberGguf* g, uint64_t index, uint64_t* offset);

/* --- tokenizer (src/tokenizer/mod.rs) ---------------------------------------
 * GPT-2 byte-level BPE with the `smollm` pre-tokenizer: text in, token ids
 * out, for prompts given as text. Host-only. The facts are the GGUF's
 * tokenizer.ggml.* metadata (Gpt2BpeTokenizer::new, mod.rs:329-530).
 * Construction refuses, as INVALID_ARGUMENT whose message begins with the
 * reference's TokenizerError kind: a model other than "gpt2"
 * (UnsupportedModel), a pre-tokenizer other than "smollm"
 * (UnsupportedPreTokenizer), vocabulary or merge counts other than the
 * expected (VocabSizeMismatch, MergesCountMismatch), a token_type count
 * other than the vocabulary's (TokenTypeCountMismatch), scores
 * (ScoresPresent), add_bos_token or add_space_prefix set, a malformed merge
 * (MalformedMergeString), an empty, overlong or space-holding token text
 * (ByteBoundaryViolation), a special id out of range (TokenIdOutOfRange). */
typedef struct FaberTokenizer FaberTokenizer;

typedef struct FaberTokenizerFactsV1 {
  const char* model;               /* tokenizer.ggml.model */
  const char* pre;                 /* tokenizer.ggml.pre */
  const char* const* tokens;       /* tokenizer.ggml.tokens (token_lens bytes each) */
  const uint64_t* token_lens;
  uint64_t n_tokens;
  const int32_t* token_types;      /* tokenizer.ggml.token_type */
  uint64_t n_token_types;
  const char* const* merges;       /* tokenizer.ggml.merges (merge_lens bytes each) */
  const uint64_t* merge_lens;
  uint64_t n_merges;
  int32_t scores_present;          /* tokenizer.ggml.scores exists */
  uint32_t bos_token_id, eos_token_id, pad_token_id, unk_token_id;
  int32_t add_bos_token, add_space_prefix;
  uint64_t expected_vocab;         /* the pinned row: 49152 */
  uint64_t expected_merges;        /* the pinned row: 48900 */
} FaberTokenizerFactsV1;

FaberRtStatusV1 faber_gpu_v2_tokenizer_create(const FaberTokenizerFactsV1* facts, FaberTokenizer** out);
/* encode (mod.rs:690-770): UTF-8 text -> ids. parse_special turns control,
 * unknown and user-defined token texts into their ids (user-defined ones
 * always). *n_ids is always set; with cap below it the call is IO_ERROR and
 * writes no ids (2 x len + 1024 is always enough). INVALID_ARGUMENT for
 * invalid UTF-8 (InvalidUtf8) or more than 1 MiB (InputTooLarge). */
FaberRtStatusV1 faber_gpu_v2_tokenizer_encode(const FaberTokenizer* t, const uint8_t* text, uint64_t len,
                                              int32_t parse_special, uint32_t* ids, uint64_t cap,
                                              uint64_t* n_ids);
/* ids -> bytes: each token's text through the inverse byte map (special
 * texts as they are). *n_out is always set; IO_ERROR when cap is short. */
FaberRtStatusV1 faber_gpu_v2_tokenizer_decode(const FaberTokenizer* t, const uint32_t* ids, uint64_t n,
                                              uint8_t* out, uint64_t cap, uint64_t* n_out);
/* Vocabulary size, {bos, eos, pad, unk} ids and the end-of-generation ids
 * (tokens with an end-of-turn text, then eos; *n_eog always set, IO_ERROR
 * when eog_cap is short). */
FaberRtStatusV1 faber_gpu_v2_tokenizer_info(const FaberTokenizer* t, uint64_t* vocab, uint32_t special_ids[4],
                                            uint32_t* eog, uint64_t eog_cap, uint64_t* n_eog);
FaberRtStatusV1 faber_gpu_v2_tokenizer_free(FaberTokenizer* t);

/* Batched greedy decode — run_greedy (src/greedy_run.rs:186-248) for up to
 * 16 sequences in lockstep, the batch-16 decode of the reference's
 * multi-sequence KvCacheLayout (src/kv_cache.rs:504-626, `slots`). The batch
 * is a view over n open sessions of one model (same context length, one
 * GPU, untied Q4_K head, dimensions in whole super-blocks): each session
 * holds one sequence with its prompt already pushed. Every linear layer
 * reads its weights once per step for all sequences. The sessions stay
 * usable: after batch_greedy each holds its sequence's state, exactly as if
 * session_greedy had run on it. Unsupported models give UNSUPPORTED. */
FaberRtStatusV1 faber_gpu_v2_batch_open(FaberGpuSession* const* sessions, uint32_t n,
                                        FaberGpuBatch** out);
/* n_gen greedy tokens per sequence: out_tokens[i * n_gen + j] is token j of
 * sequence i; all_finite[i] (optional, n entries) its finite gate. The EOG
 * ids are excluded from every argmax, as in session_greedy. */
FaberRtStatusV1 faber_gpu_v2_batch_greedy(FaberGpuBatch* b, uint32_t n_gen, const int64_t* eog,
                                          uint32_t n_eog, int64_t* out_tokens,
                                          int32_t* all_finite);
/* Device time of the last batch_greedy (CUDA events around its steps). */
FaberRtStatusV1 faber_gpu_v2_batch_last_ms(const FaberGpuBatch* b, float* ms);
FaberRtStatusV1 faber_gpu_v2_batch_close(FaberGpuBatch* b);
/* Install a K/V prefix of n positions for one layer (host f32 [n][kv_heads*
 * head_dim]; stored f16-rounded like every cached value). All layers must be
 * given the same n before the next push. */
FaberRtStatusV1 faber_gpu_v2_session_set_prefix(FaberGpuSession* s, uint32_t layer,
                                                const float* k, const float* v, uint64_t n);
/* Layer intermediates of the last push (test support): which = 0 attn_in,
 * 1 q_rot, 2 k_rot, 3 v, 4 ctx, 5 h2, 6 hh, 7 h_out; only when the session
 * was opened with tracing (faber_gpu_v2_session_set_trace). */
FaberRtStatusV1 faber_gpu_v2_session_set_trace(FaberGpuSession* s, int32_t on);
FaberRtStatusV1 faber_gpu_v2_session_trace(FaberGpuSession* s, uint32_t layer, uint32_t which,
                                           float* out, uint64_t cap, uint64_t* n);
/* Device timing of the last greedy call: milliseconds between the first and
 * last decode step on the device (CUDA events). */
FaberRtStatusV1 faber_gpu_v2_session_last_greedy_ms(const FaberGpuSession* s, float* ms);

/* Token commit — SequenceState::commit (src/session.rs:422-456): advances
 * token/position/kv-generation together; an exact replay of the last commit
 * is a no-op success (*outcome = 1), out-of-order position or a KV
 * generation gap is INVALID_ARGUMENT and changes nothing; an empty
 * publication boundary is INVALID_ARGUMENT. *outcome = 0 when applied. */
FaberRtStatusV1 faber_gpu_v2_session_commit(FaberGpuSession* s, int64_t token,
                                            uint32_t position, uint64_t kv_generation,
                                            uint64_t publication_boundary, int32_t* outcome);

/* ------------------------------------------------------------------------
 * Seeded synthetic inputs (counter-based splitmix64; identical bytes for
 * any thread count). stream separates independent tensors.
 * ------------------------------------------------------------------------ */
/* Q4_K super-blocks: d, dmin = f16(U[1e-3, 2e-2]); scales[12], qs[128]
 * uniform bytes (every 6-bit scale/min and 4-bit quant uniform). */
FaberRtStatusV1 faber_synth_q4k(uint64_t seed, uint64_t stream, uint64_t n_blocks,
                                uint8_t* out);
/* f32 N(mean, std) (Box-Muller in double). */
FaberRtStatusV1 faber_synth_normal_f32(uint64_t seed, uint64_t stream, uint64_t n, float mean,
                                       float std, float* out);
/* token ids uniform in [0, vocab). */
FaberRtStatusV1 faber_synth_tokens(uint64_t seed, uint64_t stream, uint64_t n, uint32_t vocab,
                                   int64_t* out);
/* The 128-byte ncclUniqueId for a TP group (rank 0 creates, then shares). */
FaberRtStatusV1 faber_gpu_v2_nccl_unique_id(uint8_t out[128]);

/* ------------------------------------------------------------------------
 * Allocation-free decode attention. This entry point has no counterpart in
 * the reference.
 *
 * It is the split-K decode attention of a session, for one query row, for
 * callers that must not allocate device memory. That means a host whose
 * device memory is fully accounted up front (a fixed per-device byte budget
 * in which an unaccounted cudaMalloc is a failure), or code on a
 * latency-critical path where cudaMalloc / cudaFree may synchronize the
 * whole device.
 *
 * Inputs and outputs belong to the caller, all in device memory:
 *   q      f32 [n_heads][head_dim]  post-RoPE queries;
 *   k, v   f16 [n_kv][n_kv_heads * head_dim]  the cached keys and values;
 *   ctx    f32 [n_heads][head_dim]  the attention output.
 * Query head h uses kv head h / (n_heads / n_kv_heads). The result agrees
 * with the session path within floating-point summation order.
 *
 * Scratch: one static device array of about 2 MiB (split partials, merge
 * counters, a position word). It is part of the library image, so every GPU
 * that loads the library holds it until the process exits. Each call clears
 * the counters first; the other contents are written before they are read.
 *
 * Limits: head_dim 64 or 128; n_heads and n_kv_heads at most 128; at most
 * 8 query heads per kv head; 1 <= n_kv <= 2^31 - 33. Sizes beyond these return
 * INVALID_ARGUMENT with a message, before any work is queued.
 *
 * Set-up: the first call on a device looks up the array's device address
 * with that device current. Make that first call before any stream capture
 * on the device.
 *
 * Concurrency: all calls on a device share the array, so calls that overlap
 * on the GPU (different streams, or different host threads without ordering)
 * race and give wrong results. Serialize them, for example on one stream.
 * The call only enqueues work on `stream`; the output is ready when that
 * stream has reached the call. */
FaberRtStatusV1 faber_gpu_v2_attention_decode_static(const float* q, const void* k_cache,
                                                     const void* v_cache, float* ctx,
                                                     uint32_t n_heads, uint32_t n_kv_heads,
                                                     uint32_t head_dim, uint64_t n_kv,
                                                     void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FABER_GPU_H */
