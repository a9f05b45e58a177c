"""ctypes binding of libfaber_gpu.so (the C ABI in include/faber_gpu.h).

The library is built in-tree (``__graft_entry__.build()`` or
``python faber_runtime_b200/build.py``). There is no fallback: importing a
GPU entry point without the library raises.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libfaber_gpu.so"

OK, INVALID_ARGUMENT, IO_ERROR, PANIC, UNSUPPORTED, FALLIBLE = 0, 1, 2, 3, 4, 5
TIMEOUT, DEVICE_LOSS, CANCELLED, ALLOCATION, CUDA_ERROR, KERNEL_ERROR = 16, 17, 18, 19, 20, 21
BUDGET_EXCEEDED = 22
STATUS_NAMES = {0: "OK", 1: "INVALID_ARGUMENT", 2: "IO_ERROR", 3: "PANIC", 4: "UNSUPPORTED",
                5: "FALLIBLE", 16: "TIMEOUT", 17: "DEVICE_LOSS", 18: "CANCELLED",
                19: "ALLOCATION", 20: "CUDA_ERROR", 21: "KERNEL_ERROR", 22: "BUDGET_EXCEEDED"}

GGML_F32, GGML_Q5_0, GGML_Q8_0, GGML_Q4_K, GGML_Q6_K = 0, 6, 8, 12, 14


class Status(ctypes.Structure):
    _fields_ = [("code", ctypes.c_int32)]


class ModelConfigC(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_uint32), ("d_model", ctypes.c_uint32),
                ("n_heads", ctypes.c_uint32), ("n_kv_heads", ctypes.c_uint32),
                ("head_dim", ctypes.c_uint32), ("ffn", ctypes.c_uint32),
                ("vocab", ctypes.c_uint32), ("tied_head", ctypes.c_uint32),
                ("rms_eps", ctypes.c_float), ("rope_theta", ctypes.c_float),
                ("tp_size", ctypes.c_uint32), ("tp_rank", ctypes.c_uint32),
                ("nccl_unique_id", ctypes.c_uint8 * 128)]


class KvLayoutC(ctypes.Structure):
    _fields_ = [("slots", ctypes.c_uint32), ("context_length", ctypes.c_uint32),
                ("layer_count", ctypes.c_uint32), ("kv_head_count", ctypes.c_uint32),
                ("head_dim", ctypes.c_uint32), ("dtype", ctypes.c_uint32),
                ("reserve_bytes", ctypes.c_uint64)]


class PartitionLedgerC(ctypes.Structure):
    _fields_ = [("weight_bytes", ctypes.c_uint64), ("kv_cache_bytes", ctypes.c_uint64),
                ("activation_scratch_bytes", ctypes.c_uint64), ("module_storage_bytes", ctypes.c_uint64),
                ("allocator_overhead_bytes", ctypes.c_uint64), ("transfer_staging_bytes", ctypes.c_uint64),
                ("concurrent_state_bytes", ctypes.c_uint64)]


class TxnOpC(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_uint32), ("partition", ctypes.c_uint32), ("destination", ctypes.c_uint32),
                ("reserved", ctypes.c_uint32), ("participants", ctypes.c_uint64), ("ref", ctypes.c_uint64),
                ("bytes", ctypes.c_uint64)]


class TxnPartitionC(ctypes.Structure):
    _fields_ = [("partition", ctypes.c_uint32), ("admitted", ctypes.c_uint32), ("ledger", PartitionLedgerC)]


class TxnReceiptC(ctypes.Structure):
    _fields_ = [("decision", ctypes.c_int32), ("state", ctypes.c_int32), ("failure_kind", ctypes.c_int32),
                ("failure_class", ctypes.c_int32), ("failure_partition", ctypes.c_uint32),
                ("published", ctypes.c_uint32), ("publication_ordinal", ctypes.c_uint64),
                ("declared_write_bytes", ctypes.c_uint64), ("executed_operations", ctypes.c_uint64),
                ("executed_bytes", ctypes.c_uint64), ("completed_events", ctypes.c_uint64),
                ("staged_bytes", ctypes.c_uint64), ("published_bytes", ctypes.c_uint64),
                ("released_partitions", ctypes.c_uint64), ("retired_partitions", ctypes.c_uint64),
                ("partial_publication", ctypes.c_uint32), ("reserved", ctypes.c_uint32),
                ("prepare_ns", ctypes.c_uint64), ("execute_ns", ctypes.c_uint64), ("finalize_ns", ctypes.c_uint64)]


class TxnErrorC(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("partition", ctypes.c_uint32), ("backend_class", ctypes.c_int32),
                ("budget_class", ctypes.c_int32), ("missing", ctypes.c_uint64)]


class TxnBackendInfoC(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in (
        "reserved_partitions", "released_partitions", "retired_partitions", "staged_bytes", "published_bytes",
        "committed_bytes", "executed_operations", "pending_events", "delivered_faults", "reclaimed_copy_bytes")]


class TokenizerFactsC(ctypes.Structure):
    _fields_ = [("model", ctypes.c_char_p), ("pre", ctypes.c_char_p), ("tokens", ctypes.c_void_p),
                ("token_lens", ctypes.c_void_p), ("n_tokens", ctypes.c_uint64), ("token_types", ctypes.c_void_p),
                ("n_token_types", ctypes.c_uint64), ("merges", ctypes.c_void_p), ("merge_lens", ctypes.c_void_p),
                ("n_merges", ctypes.c_uint64), ("scores_present", ctypes.c_int32),
                ("bos_token_id", ctypes.c_uint32), ("eos_token_id", ctypes.c_uint32),
                ("pad_token_id", ctypes.c_uint32), ("unk_token_id", ctypes.c_uint32),
                ("add_bos_token", ctypes.c_int32), ("add_space_prefix", ctypes.c_int32),
                ("expected_vocab", ctypes.c_uint64), ("expected_merges", ctypes.c_uint64)]


class FaberError(RuntimeError):
    """A failed C-ABI call: ``code`` is the FaberRtStatusV1 code."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {message}")
        self.code = code
        self.message = message
        self.message = message


P = ctypes.c_void_p
U64, U32, I32, I64 = ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int32, ctypes.c_int64
PP = ctypes.POINTER(ctypes.c_void_p)

SIGNATURES = {
    "faber_gpu_v2_abi_version": (U32, []),
    "faber_gpu_v2_last_error": (Status, [ctypes.c_char_p, U64]),
    "faber_gpu_v2_init": (Status, [I32]),
    "faber_gpu_v2_fault_inject": (Status, [ctypes.c_char_p, I32, U32]),
    "__faber_gpu_v1_copy_in": (Status, [U64, P, U64, U32]),
    "__faber_gpu_v1_readback": (Status, [U64, P, U64, ctypes.POINTER(U64)]),
    "__faber_gpu_v1_sync": (Status, [U64]),
    "faber_gpu_v2_buffer_device_ptr": (Status, [U64, PP, ctypes.POINTER(U64)]),
    "faber_gpu_v2_dequant_q4k": (Status, [P, U64, P, I32, P]),
    "faber_gpu_v2_dequant_blocks": (Status, [U32, P, U64, P, I32, P]),
    "faber_gpu_v2_typed_upload": (Status, [U32, P, U64, U64, U64, PP]),
    "faber_gpu_v2_typed_gemv": (Status, [P, P, P, P]),
    "faber_gpu_v2_typed_free": (Status, [P]),
    "faber_gpu_v2_f16_round": (Status, [P, P, U64, P]),
    "faber_gpu_v2_gemv_q4k": (Status, [P, U64, U64, P, P, P]),
    "faber_gpu_v2_q4k_upload": (Status, [P, U64, U64, U64, PP]),
    "faber_gpu_v2_q4k_free": (Status, [P]),
    "faber_gpu_v2_q4k_gemv": (Status, [P, P, P, P]),
    "faber_gpu_v2_q4k_gemv_exchange": (Status, [P, P, P, ctypes.c_float, P, U32, U32, U32, P, P, P]),
    "faber_gpu_v2_q4k_gemv_batch": (Status, [P, P, U32, P, P]),
    "faber_gpu_v2_q4k_dequant_rows": (Status, [P, P, I32, P]),
    "faber_gpu_v2_q4k_repack_hash": (Status, [P, ctypes.POINTER(U64)]),
    "faber_gpu_v2_kv_layout_bytes": (Status, [ctypes.POINTER(KvLayoutC), ctypes.POINTER(U64),
                                              ctypes.POINTER(U64)]),
    "faber_gpu_v2_partition_admit": (Status, [ctypes.POINTER(PartitionLedgerC), U64, ctypes.POINTER(U64)]),
    "faber_gpu_v2_partition_usage": (Status, [I32, ctypes.POINTER(PartitionLedgerC)]),
    "faber_gpu_v2_partition_set_limit": (Status, [I32, U64]),
    "faber_gpu_v2_partition_plan": (Status, [ctypes.POINTER(ModelConfigC), U32, U32, I32,
                                             ctypes.POINTER(PartitionLedgerC)]),
    "faber_gpu_v2_txn_create": (Status, [P, U32, P, U32, P, U32, P, U32, PP]),
    "faber_gpu_v2_txn_prepare": (Status, [P, P]),
    "faber_gpu_v2_txn_execute": (Status, [P, P]),
    "faber_gpu_v2_txn_execute_operation": (Status, [P, P, P]),
    "faber_gpu_v2_txn_commit": (Status, [P, P, U64]),
    "faber_gpu_v2_txn_abort": (Status, [P, P, ctypes.c_char_p]),
    "faber_gpu_v2_txn_receipt": (Status, [P, P]),
    "faber_gpu_v2_txn_last_error": (Status, [P, P]),
    "faber_gpu_v2_txn_reservation": (Status, [P, U32, P]),
    "faber_gpu_v2_txn_free": (Status, [P]),
    "faber_gpu_v2_txn_backend_fake": (Status, [PP]),
    "faber_gpu_v2_txn_backend_inject": (Status, [P, U32, U64, U32, I32]),
    "faber_gpu_v2_txn_backend_fail_publish": (Status, [P, I32]),
    "faber_gpu_v2_txn_backend_set_auto_complete": (Status, [P, I32]),
    "faber_gpu_v2_txn_backend_complete_event": (Status, [P, U32, U32, U64]),
    "faber_gpu_v2_txn_backend_info": (Status, [P, P]),
    "faber_gpu_v2_txn_backend_free": (Status, [P]),
    "faber_gpu_v2_tp_step_plan": (Status, [ctypes.POINTER(ModelConfigC), U32, P, U32, ctypes.POINTER(U32),
                                           ctypes.POINTER(U64), P]),
    "faber_gpu_v2_gguf_kv_payload": (Status, [P, U64, ctypes.POINTER(U64)]),
    "faber_gpu_v2_tokenizer_create": (Status, [ctypes.POINTER(TokenizerFactsC), PP]),
    "faber_gpu_v2_tokenizer_encode": (Status, [P, P, U64, I32, P, U64, ctypes.POINTER(U64)]),
    "faber_gpu_v2_tokenizer_decode": (Status, [P, P, U64, P, U64, ctypes.POINTER(U64)]),
    "faber_gpu_v2_tokenizer_info": (Status, [P, ctypes.POINTER(U64), P, P, U64, ctypes.POINTER(U64)]),
    "faber_gpu_v2_tokenizer_free": (Status, [P]),
    "faber_gpu_v2_model_create": (Status, [ctypes.POINTER(ModelConfigC), PP]),
    "faber_gpu_v2_model_set_tensor": (Status, [P, ctypes.c_char_p, U32, P, U64, U64, U64]),
    "faber_gpu_v2_tp_shard": (Status, [ctypes.POINTER(ModelConfigC), ctypes.c_char_p, P]),
    "faber_gpu_v2_model_finalize": (Status, [P]),
    "faber_gpu_v2_model_free": (Status, [P]),
    "faber_gpu_v2_model_device_bytes": (Status, [P, ctypes.POINTER(U64)]),
    "faber_gpu_v2_session_open": (Status, [P, ctypes.POINTER(KvLayoutC), PP]),
    "faber_gpu_v2_session_close": (Status, [P]),
    "faber_gpu_v2_session_reset": (Status, [P]),
    "faber_gpu_v2_session_len": (Status, [P, ctypes.POINTER(U64)]),
    "faber_gpu_v2_session_truncate": (Status, [P, U64]),
    "faber_gpu_v2_session_set_wait_limit": (Status, [P, U32]),
    "faber_gpu_v2_session_exchange_epoch": (Status, [P, U32, ctypes.POINTER(U32)]),
    "faber_gpu_v2_session_push_token": (Status, [P, I64]),
    "faber_gpu_v2_session_push_tokens": (Status, [P, P, U64]),
    "faber_gpu_v2_session_step_greedy": (Status, [P, I64, P, U32, ctypes.POINTER(I64)]),
    "faber_gpu_v2_session_position_logits": (Status, [P, P, U64]),
    "faber_gpu_v2_session_greedy": (Status, [P, U32, P, U32, P, ctypes.POINTER(I32)]),
    "faber_gpu_v2_session_set_prefix": (Status, [P, U32, P, P, U64]),
    "faber_gpu_v2_session_set_trace": (Status, [P, I32]),
    "faber_gpu_v2_session_trace": (Status, [P, U32, U32, P, U64, ctypes.POINTER(U64)]),
    "faber_gpu_v2_session_last_greedy_ms": (Status, [P, ctypes.POINTER(ctypes.c_float)]),
    "faber_gpu_v2_session_commit": (Status, [P, I64, U32, U64, U64, ctypes.POINTER(I32)]),
    "faber_gpu_v2_nccl_unique_id": (Status, [P]),
    "faber_gpu_v2_gguf_parse": (Status, [P, U64, PP]),
    "faber_gpu_v2_gguf_info": (Status, [P, ctypes.POINTER(U32), ctypes.POINTER(U64), ctypes.POINTER(U64),
                                        ctypes.POINTER(U64), ctypes.POINTER(U64)]),
    "faber_gpu_v2_gguf_tensor": (Status, [P, U64, P]),
    "faber_gpu_v2_gguf_kv": (Status, [P, U64, ctypes.c_char_p, U64, ctypes.POINTER(U32), ctypes.POINTER(U32),
                                      ctypes.POINTER(U64)]),
    "faber_gpu_v2_gguf_get_int": (Status, [P, ctypes.c_char_p, ctypes.POINTER(I64)]),
    "faber_gpu_v2_gguf_get_float": (Status, [P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)]),
    "faber_gpu_v2_gguf_get_string": (Status, [P, ctypes.c_char_p, ctypes.c_char_p, U64, ctypes.POINTER(U64)]),
    "faber_gpu_v2_gguf_free": (Status, [P]),
    "faber_gpu_v2_batch_open": (Status, [P, U32, PP]),
    "faber_gpu_v2_batch_greedy": (Status, [P, U32, P, U32, P, P]),
    "faber_gpu_v2_batch_last_ms": (Status, [P, ctypes.POINTER(ctypes.c_float)]),
    "faber_gpu_v2_batch_close": (Status, [P]),
    "faber_gpu_v2_attention_decode_static": (Status, [P, P, P, P, U32, U32, U32, U64, P]),
    "faber_synth_q4k": (Status, [U64, U64, U64, P]),
    "faber_synth_normal_f32": (Status, [U64, U64, U64, ctypes.c_float, ctypes.c_float, P]),
    "faber_synth_tokens": (Status, [U64, U64, U64, U32, P]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load the library (raises when it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(
                f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                "(the Q4_K path has no CPU fallback)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(2048)
    lib().faber_gpu_v2_last_error(buf, 2048)
    return buf.value.decode(errors="replace")


def check(st: Status) -> None:
    if st.code != OK:
        raise FaberError(st.code, last_error())


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
