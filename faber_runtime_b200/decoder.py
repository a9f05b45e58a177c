"""Device decoder: the GPU counterpart of CpuOracle / ForwardRun / run_greedy.

Mirrors the reference's interface for the path (src/cpu_oracle.rs:409-445,
513-534, 808-926; src/greedy_run.rs:186-248): a model is built once from its
tensors (``DeviceModel`` ~ ``CpuOracle::build``), a ``ForwardRun`` pushes
tokens and returns the logits at the sequence end, and ``run_greedy`` feeds
its own predictions back. Errors follow the reference's fail-closed rules:
an empty prompt or an out-of-range token id raises ``OracleError`` before any
device work, and a failed C-ABI call raises ``FaberError`` with its status.
"""

from __future__ import annotations

import ctypes
import json
from dataclasses import dataclass, field
from typing import Iterable

import numpy as np

from . import _lib
from .config import KV_F16, KvCacheLayout, ModelConfig


class OracleError(ValueError):
    """Typed rejection mirroring OracleError (src/cpu_oracle.rs:162-175)."""

    def __init__(self, kind: str, detail: str):
        super().__init__(f"{kind}: {detail}")
        self.kind = kind


class DeviceModel:
    """Weights resident on one GPU (or this rank's shard of a TP group)."""

    def __init__(self, cfg: ModelConfig, tensors: Iterable, device: int = 0,
                 tp_size: int = 1, tp_rank: int = 0, nccl_uid: bytes = b""):
        self.cfg = cfg
        self.device = device
        self.tp_size, self.tp_rank = tp_size, tp_rank
        _lib.call("faber_gpu_v2_init", device)
        c = cfg.c_struct(tp_size, tp_rank, nccl_uid)
        h = ctypes.c_void_p()
        _lib.call("faber_gpu_v2_model_create", ctypes.byref(c), ctypes.byref(h))
        self._h = h
        try:
            for name, gtype, arr, rows, cols in tensors:
                self.set_tensor(name, gtype, arr, rows, cols)
            _lib.call("faber_gpu_v2_model_finalize", self._h)
        except BaseException:
            self.close()  # a failed upload frees what it had placed on the device
            raise

    def set_tensor(self, name: str, gtype: int, arr: np.ndarray, rows: int, cols: int) -> None:
        a = np.ascontiguousarray(arr)
        full = name if name.endswith(".weight") else name + ".weight"
        _lib.call("faber_gpu_v2_model_set_tensor", self._h, full.encode(), gtype,
                  a.ctypes.data, a.nbytes, rows, cols)

    def device_bytes(self) -> int:
        n = _lib.U64()
        _lib.call("faber_gpu_v2_model_device_bytes", self._h, ctypes.byref(n))
        return n.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.call("faber_gpu_v2_init", self.device)
            _lib.call("faber_gpu_v2_model_free", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward_one(self, tokens, context_length: int | None = None) -> np.ndarray:
        """Raw logits for the position after ``tokens`` (CpuOracle::forward_one)."""
        toks = list(tokens)
        run = ForwardRun(self, toks, context_length=context_length or max(len(toks), 1))
        try:
            return run.position_logits()
        finally:
            run.close()


class ForwardRun:
    """Incremental decode over a device KV cache (ForwardRun,
    src/cpu_oracle.rs:808-926) plus the session contract's token commit
    (SequenceState::commit, src/session.rs:422-456)."""

    def __init__(self, model: DeviceModel, tokens=(), context_length: int = 4096,
                 kv_dtype: int = KV_F16, trace: bool = False):
        toks = list(tokens)
        self.model = model
        self.cfg = model.cfg
        self.layout = KvCacheLayout.for_model(model.cfg, context_length, kv_dtype)
        _lib.call("faber_gpu_v2_init", model.device)
        c = self.layout.c_struct()
        h = ctypes.c_void_p()
        _lib.call("faber_gpu_v2_session_open", model._h, ctypes.byref(c), ctypes.byref(h))
        self._h = h
        if trace:
            _lib.call("faber_gpu_v2_session_set_trace", self._h, 1)
        if toks:
            self.push_tokens(toks)

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.call("faber_gpu_v2_session_close", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self) -> int:
        n = _lib.U64()
        _lib.call("faber_gpu_v2_session_len", self._h, ctypes.byref(n))
        return n.value

    def _check_tokens(self, toks: np.ndarray) -> None:
        bad = toks[(toks < 0) | (toks >= self.cfg.vocab)]
        if bad.size:
            raise OracleError("TokenOutOfRange",
                              f"token {int(bad[0])} is outside the admitted vocab [0, {self.cfg.vocab})")

    def push_token(self, token: int) -> None:
        self._check_tokens(np.array([token], np.int64))
        _lib.call("faber_gpu_v2_session_push_token", self._h, int(token))

    def step_greedy(self, token: int, eog=()) -> int:
        """Push ``token`` and return the greedy id of the new position (the
        argmax over ids not in ``eog``): one step of a host-driven greedy
        loop, with 8 bytes each way between host and device."""
        self._check_tokens(np.array([token], np.int64))
        e = np.ascontiguousarray(list(eog), dtype=np.int64)
        nxt = _lib.I64()
        _lib.call("faber_gpu_v2_session_step_greedy", self._h, int(token), e.ctypes.data if e.size else None,
                  e.size, ctypes.byref(nxt))
        return nxt.value

    def push_tokens(self, tokens) -> None:
        t = np.ascontiguousarray(tokens, dtype=np.int64)
        if t.size == 0:
            raise OracleError("EmptyTokens", "oracle needs at least one token")
        self._check_tokens(t)
        _lib.call("faber_gpu_v2_session_push_tokens", self._h, t.ctypes.data, t.size)

    def set_prefix(self, layer: int, k: np.ndarray, v: np.ndarray, n: int) -> None:
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        _lib.call("faber_gpu_v2_session_set_prefix", self._h, layer, k.ctypes.data,
                  v.ctypes.data, n)

    def position_logits(self) -> np.ndarray:
        if len(self) == 0:
            raise OracleError("EmptyTokens", "oracle needs at least one token")
        out = np.empty(self.cfg.vocab, np.float32)
        _lib.call("faber_gpu_v2_session_position_logits", self._h, out.ctypes.data, out.size)
        return out

    def greedy(self, n_gen: int, eog=()) -> tuple[np.ndarray, bool]:
        out = np.empty(max(n_gen, 1), np.int64)
        e = np.ascontiguousarray(list(eog) or [0], np.int64)
        fin = ctypes.c_int32(1)
        _lib.call("faber_gpu_v2_session_greedy", self._h, n_gen, e.ctypes.data, len(eog),
                  out.ctypes.data, ctypes.byref(fin))
        return out[:n_gen].copy(), bool(fin.value)

    def last_greedy_ms(self) -> float:
        ms = ctypes.c_float()
        _lib.call("faber_gpu_v2_session_last_greedy_ms", self._h, ctypes.byref(ms))
        return ms.value

    def trace(self, layer: int, which: str) -> np.ndarray:
        idx = {"attn_in": 0, "q_rot": 1, "k_rot": 2, "v": 3, "ctx": 4, "h2": 5, "hh": 6,
               "h_out": 7}[which]
        cap = max(self.cfg.d_model, self.cfg.ffn, self.cfg.n_heads * self.cfg.head_dim)
        out = np.empty(cap, np.float32)
        n = _lib.U64()
        _lib.call("faber_gpu_v2_session_trace", self._h, layer, idx, out.ctypes.data, cap,
                  ctypes.byref(n))
        return out[:n.value].copy()

    def reset(self) -> None:
        _lib.call("faber_gpu_v2_session_reset", self._h)

    def truncate(self, n: int) -> None:
        """Shorten the sequence to ``n`` positions (the rollback of a step whose
        group aborted); the next call must be a push."""
        _lib.call("faber_gpu_v2_session_truncate", self._h, int(n))

    def set_wait_limit(self, polls: int) -> None:
        """Polls before a tensor-parallel peer or grid-barrier wait gives up
        and the step fails with TIMEOUT (0: the kernels' default)."""
        _lib.call("faber_gpu_v2_session_set_wait_limit", self._h, int(polls))

    def exchange_epoch(self, raise_to: int = 0) -> int:
        """The tensor-parallel exchange epoch, after raising it to
        ``raise_to`` if that is larger (it is never lowered)."""
        e = _lib.U32()
        _lib.call("faber_gpu_v2_session_exchange_epoch", self._h, int(raise_to), ctypes.byref(e))
        return e.value

    def commit(self, token: int, position: int, kv_generation: int,
               publication_boundary: int = 1) -> str:
        """SequenceState::commit: returns "applied" or "idempotent_replay"."""
        out = ctypes.c_int32()
        _lib.call("faber_gpu_v2_session_commit", self._h, int(token), int(position),
                  int(kv_generation), int(publication_boundary), ctypes.byref(out))
        return "idempotent_replay" if out.value == 1 else "applied"


class BatchRun:
    """Batched greedy decode over open ForwardRuns of one model: every step
    reads each weight once for all sequences (up to 16), and each run keeps
    its own sequence state afterwards (its next call continues from there)."""

    def __init__(self, runs):
        self.runs = list(runs)
        arr = (ctypes.c_void_p * len(self.runs))(*[r._h.value for r in self.runs])
        h = ctypes.c_void_p()
        _lib.call("faber_gpu_v2_batch_open", ctypes.addressof(arr), len(self.runs), ctypes.byref(h))
        self._h = h

    def greedy(self, n_gen: int, eog=()) -> tuple[np.ndarray, np.ndarray]:
        """Tokens [n_runs][n_gen] and the per-run finite gate."""
        n = len(self.runs)
        out = np.empty((n, max(n_gen, 1)), np.int64)
        fin = np.ones(n, np.int32)
        e = np.ascontiguousarray(list(eog) or [0], np.int64)
        _lib.call("faber_gpu_v2_batch_greedy", self._h, n_gen, e.ctypes.data, len(eog),
                  out.ctypes.data, fin.ctypes.data)
        return out[:, :n_gen].copy(), fin.astype(bool)

    def last_ms(self) -> float:
        ms = ctypes.c_float()
        _lib.call("faber_gpu_v2_batch_last_ms", self._h, ctypes.byref(ms))
        return ms.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.call("faber_gpu_v2_batch_close", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class GreedyDivergence:
    position: int
    comparator_trace_token: int
    oracle_token: int
    failing_thresholds: list = field(default_factory=lambda: ["top-1"])
    max_band_deviation: float | None = None


@dataclass
class GreedyRunRecord:
    """GreedyRunRecord (src/greedy_run.rs:110-140)."""

    generated_tokens: list
    all_finite: bool
    first_divergence: GreedyDivergence | None

    def divergence_field(self) -> str:
        d = self.first_divergence
        if d is None:
            return "none"
        return (f"position {d.position} (comparator {d.comparator_trace_token} vs oracle "
                f"{d.oracle_token}; {','.join(d.failing_thresholds)})")


RECORD_SCHEMA = "gi2-4-greedy-record-v1"


def _tokens_sha256(tokens) -> str:
    """SHA-256 of the ids as little-endian u64s (src/greedy_run.rs:342-350)."""
    import hashlib
    return hashlib.sha256(np.asarray(tokens, dtype=np.int64).astype("<u8").tobytes()).hexdigest()


def record_to_json(record: GreedyRunRecord, prompt_tokens, trace: dict | None = None) -> str:
    """The committed-record wire format (record_to_json,
    src/greedy_run.rs:271-340): one compact JSON object with sorted keys and
    a trailing newline. ``trace`` is the comparator trace's provenance
    object, when the run followed one."""
    d = record.first_divergence
    root = {
        "schema": RECORD_SCHEMA,
        "prompt_tokens": [int(t) for t in prompt_tokens],
        "generated_token_count": len(record.generated_tokens),
        "all_finite": bool(record.all_finite),
        "all_agree": d is None,
        "generated_tokens": [int(t) for t in record.generated_tokens],
        "generated_tokens_sha256": _tokens_sha256(record.generated_tokens),
        "first_divergence": None if d is None else {
            "position": d.position, "comparator_trace_token": d.comparator_trace_token,
            "oracle_token": d.oracle_token, "failing_thresholds": list(d.failing_thresholds),
            "max_band_deviation": d.max_band_deviation},
    }
    if trace is not None:
        root["trace"] = trace
    return json.dumps(root, sort_keys=True, separators=(",", ":")) + "\n"


def record_from_json(text: str):
    """(GreedyRunRecord, prompt tokens, trace provenance or None) from the
    committed-record wire format; refuses another schema, a count or hash
    that contradicts the tokens, and all_agree contradicting the divergence."""
    root = json.loads(text)
    if root.get("schema") != RECORD_SCHEMA:
        raise OracleError("RecordSchema", f"schema {root.get('schema')!r} is not {RECORD_SCHEMA!r}")
    toks = [int(t) for t in root["generated_tokens"]]
    if root["generated_token_count"] != len(toks):
        raise OracleError("RecordCount", "generated_token_count does not match the tokens")
    if root["generated_tokens_sha256"] != _tokens_sha256(toks):
        raise OracleError("RecordHash", "generated_tokens_sha256 does not match the tokens")
    dv = root["first_divergence"]
    if root["all_agree"] != (dv is None):
        raise OracleError("RecordAgreement", "all_agree contradicts first_divergence")
    div = None if dv is None else GreedyDivergence(
        int(dv["position"]), int(dv["comparator_trace_token"]), int(dv["oracle_token"]),
        list(dv["failing_thresholds"]), dv.get("max_band_deviation"))
    return GreedyRunRecord(toks, bool(root["all_finite"]), div), root["prompt_tokens"], root.get("trace")


def run_greedy(model: DeviceModel, prompt, trace_tokens, eog=(), context_length: int | None = None,
               ) -> GreedyRunRecord:
    """run_greedy (src/greedy_run.rs:186-248) on the device: prompt, then
    len(trace_tokens) free-running greedy steps compared token by token."""
    trace = list(trace_tokens)
    if not trace:
        raise OracleError("EmptyTokens", "trace must be non-empty")
    p = list(prompt)
    if not p:
        raise OracleError("EmptyTokens", "oracle needs at least one token")
    run = ForwardRun(model, p, context_length=context_length or (len(p) + len(trace)))
    try:
        toks, finite = run.greedy(len(trace), eog)
    finally:
        run.close()
    first = None
    for i, (a, b) in enumerate(zip(toks.tolist(), trace)):
        if a != b:
            first = GreedyDivergence(i, int(b), int(a),
                                     ["top-1"] + ([] if finite else ["finite"]))
            break
    return GreedyRunRecord(toks.tolist(), finite, first)
