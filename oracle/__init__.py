"""CPU oracle for the Q4_K decoder path — TEST INFRASTRUCTURE ONLY.

A ctypes wrapper over ``oracle/faber_oracle.cpp``, the C++ restatement of
faber-runtime's CPU oracle (src/dequant.rs, src/decoder_ops.rs,
src/cpu_oracle.rs, src/greedy_run.rs). Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline / reference arm
may import this module, and only as the checker: the product package
``faber_runtime_b200`` never imports it.

Parity pinning: the restatement is checked against the reference's in-tree
known-answer tests (half_to_f32, f32_to_f16_rn, the decoder-op KATs) and the
six per-op goldens of ``testdata/gi2-2-op-goldens`` (committed here as
``tests/golden/op_goldens.npz``). The Q4_K block goldens the reference names
(gi2-dequant-goldens.json) are not vendored in the reference tree, so Q4_K
dequant is pinned by hand-derived known answers from src/dequant.rs:178-217.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "_build" / "libfaber_oracle.so"

# GGUF dtype ids of the admitted block types (src/gguf.rs:135-144).
F32, Q5_0, Q8_0, Q4_K, Q6_K = 0, 6, 8, 12, 14
BLOCK_GEOMETRY = {F32: (1, 4), Q5_0: (32, 22), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}

# Model tensor slots (per layer) and global slots.
SLOT = {"attn_norm": 0, "attn_q": 1, "attn_k": 2, "attn_v": 3, "attn_output": 4,
        "ffn_norm": 5, "ffn_gate": 6, "ffn_up": 7, "ffn_down": 8}
GSLOT = {"token_embd": 0, "output_norm": 1, "output": 2}
TRACE = {"attn_in": 0, "q_rot": 1, "k_rot": 2, "v": 3, "ctx": 4, "h2": 5, "hh": 6, "h_out": 7}

_lib = None


def build(force: bool = False) -> Path:
    """Compile the oracle into oracle/_build (g++, -ffp-contract=off, OpenMP)."""
    from . import make as _b
    return _b.build(force=force)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        _declare(_lib)
        _lib.orc_set_threads(int(os.environ.get("FABER_ORACLE_THREADS", os.cpu_count() or 1)))
    return _lib


def _declare(L: ctypes.CDLL) -> None:
    P, I64, I32, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float
    sig = {
        "orc_half_to_f32": (F, [ctypes.c_uint16]),
        "orc_f32_to_f16_rn": (ctypes.c_uint16, [F]),
        "orc_f16_round": (F, [F]),
        "orc_f16_round_array": (None, [P, P, I64]),
        "orc_half_to_f32_array": (None, [P, P, I64]),
        "orc_f32_to_f16_array": (None, [P, P, I64]),
        "orc_block_geometry": (ctypes.c_int, [I32, P, P]),
        "orc_dequant_block": (ctypes.c_int, [I32, P, P]),
        "orc_dequant_row": (ctypes.c_int, [I32, P, I64, P]),
        "orc_dequant_range": (ctypes.c_int, [I32, P, I64, I64, P]),
        "orc_rms_norm": (None, [P, P, I64, F, P]),
        "orc_rope_norm": (None, [P, ctypes.c_uint32, F, I64, P]),
        "orc_rope_all_heads": (None, [P, I64, I64, ctypes.c_uint32, F, P]),
        "orc_rope_cos_sin": (None, [ctypes.c_uint32, I64, F, I64, P, P]),
        "orc_silu": (F, [F]),
        "orc_softmax_row": (None, [P, I64, P]),
        "orc_attention_gqa": (ctypes.c_int, [P, P, P, I64, I64, I64, I64, I64, F, P]),
        "orc_attention_causal": (ctypes.c_int, [P, P, P, I64, I64, I64, I64, I64, F, P]),
        "orc_swiglu": (None, [P, P, I64, P]),
        "orc_dense": (None, [P, P, I64, I64, P]),
        "orc_dense_q": (ctypes.c_int, [I32, P, I64, I64, P, P, ctypes.c_int]),
        "orc_residual_add": (None, [P, P, I64, P]),
        "orc_log_softmax": (ctypes.c_int, [P, I64, P]),
        "orc_top1_non_eog": (I64, [P, I64, P, I64]),
        "orc_set_threads": (None, [ctypes.c_int]),
        "orc_get_threads": (ctypes.c_int, []),
        "orc_model_new": (P, [P, P]),
        "orc_model_free": (None, [P]),
        "orc_model_set": (ctypes.c_int, [P, I32, I32, I32, P, I64, I64]),
        "orc_run_new": (P, [P, I64, ctypes.c_int]),
        "orc_run_free": (None, [P]),
        "orc_run_len": (I64, [P]),
        "orc_run_set_prefix": (ctypes.c_int, [P, I32, P, P, I64]),
        "orc_run_push": (ctypes.c_int, [P, I64]),
        "orc_run_trace": (I64, [P, I32, I32, P]),
        "orc_run_hidden": (ctypes.c_int, [P, P]),
        "orc_run_logits": (ctypes.c_int, [P, P]),
        "orc_run_greedy": (ctypes.c_int, [P, P, I64, I64, P, I64, P, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


# --- scalar / element ops ---------------------------------------------------

def half_to_f32(bits: int) -> float:
    return lib().orc_half_to_f32(bits)


def half_to_f32_bits(bits: int) -> int:
    return int(np.float32(lib().orc_half_to_f32(bits)).view(np.uint32))


def f32_to_f16_rn(x) -> int:
    return int(lib().orc_f32_to_f16_rn(ctypes.c_float(np.float32(x))))


def half_to_f32_array(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    y = np.empty(h.size, np.float32)
    lib().orc_half_to_f32_array(_p(h), _p(y), h.size)
    return y


def f32_to_f16_array(x: np.ndarray) -> np.ndarray:
    x = _f32(x)
    h = np.empty(x.size, np.uint16)
    lib().orc_f32_to_f16_array(_p(x), _p(h), x.size)
    return h


def f16_round(x: np.ndarray) -> np.ndarray:
    x = _f32(x)
    y = np.empty_like(x)
    lib().orc_f16_round_array(_p(x), _p(y), x.size)
    return y


def dequant_block(gtype: int, block: bytes | np.ndarray) -> np.ndarray:
    b = np.frombuffer(bytes(block), dtype=np.uint8)
    elems, nbytes = BLOCK_GEOMETRY[gtype]
    if b.size != nbytes:
        raise ValueError(f"block buffer is {b.size} bytes, expected {nbytes}")
    out = np.empty(elems, np.float32)
    lib().orc_dequant_block(gtype, _p(b), _p(out))
    return out


def dequant_row(gtype: int, packed: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(packed, dtype=np.uint8).reshape(-1)
    elems, nbytes = BLOCK_GEOMETRY[gtype]
    if b.size % nbytes:
        raise ValueError(f"packed row is {b.size} bytes, not a multiple of {nbytes}")
    nb = b.size // nbytes
    out = np.empty(nb * elems, np.float32)
    lib().orc_dequant_row(gtype, _p(b), nb, _p(out))
    return out


def dequant_range(gtype: int, packed: np.ndarray, start: int, count: int) -> np.ndarray:
    b = np.ascontiguousarray(packed, dtype=np.uint8).reshape(-1)
    out = np.empty(count, np.float32)
    lib().orc_dequant_range(gtype, _p(b), start, count, _p(out))
    return out


def rms_norm(x, w, eps: float) -> np.ndarray:
    x, w = _f32(x), _f32(w)
    if x.size != w.size:
        raise ValueError("rms_norm: x and weight must have equal length")
    y = np.empty_like(x)
    lib().orc_rms_norm(_p(x), _p(w), x.size, eps, _p(y))
    return y


def rope_norm(x, pos: int, base: float, dim: int) -> np.ndarray:
    x = _f32(x)
    if x.size != dim or dim % 2:
        raise ValueError("rope_norm: x must have exactly dim (even) elements")
    y = np.empty_like(x)
    lib().orc_rope_norm(_p(x), pos, base, dim, _p(y))
    return y


def rope_all_heads(x, n_heads: int, head_dim: int, pos: int, base: float) -> np.ndarray:
    x = _f32(x)
    y = np.empty_like(x)
    lib().orc_rope_all_heads(_p(x), n_heads, head_dim, pos, base, _p(y))
    return y


def rope_cos_sin(pos: int, k: int, base: float, dim: int) -> tuple[float, float]:
    c, s = ctypes.c_float(), ctypes.c_float()
    lib().orc_rope_cos_sin(pos, k, base, dim, ctypes.byref(c), ctypes.byref(s))
    return c.value, s.value


def silu(x: float) -> float:
    return lib().orc_silu(x)


def softmax_row(s) -> np.ndarray:
    s = _f32(s)
    p = np.empty_like(s)
    lib().orc_softmax_row(_p(s), s.size, _p(p))
    return p


def attention_gqa(q, k, v, n_q, n_kv, n_heads, n_kv_heads, head_dim, scale) -> np.ndarray:
    q, k, v = _f32(q), _f32(k), _f32(v)
    _check_attention("attention_gqa", q, k, v, n_q, n_kv, n_heads, n_kv_heads, head_dim)
    ctx = np.empty(n_q * n_heads * head_dim, np.float32)
    lib().orc_attention_gqa(_p(q), _p(k), _p(v), n_q, n_kv, n_heads, n_kv_heads, head_dim,
                            scale, _p(ctx))
    return ctx


def attention_causal(q, k, v, n_q, n_kv, n_heads, n_kv_heads, head_dim, scale) -> np.ndarray:
    q, k, v = _f32(q), _f32(k), _f32(v)
    _check_attention("attention_causal", q, k, v, n_q, n_kv, n_heads, n_kv_heads, head_dim)
    ctx = np.empty(n_q * n_heads * head_dim, np.float32)
    lib().orc_attention_causal(_p(q), _p(k), _p(v), n_q, n_kv, n_heads, n_kv_heads, head_dim,
                               scale, _p(ctx))
    return ctx


def _check_attention(op, q, k, v, n_q, n_kv, n_heads, n_kv_heads, head_dim):
    # Shape guards of src/cpu_oracle.rs:735-766 / src/decoder_ops.rs:271-304.
    if n_q > n_kv:
        raise ValueError(f"{op}: n_q ({n_q}) must be <= n_kv ({n_kv})")
    if n_heads % n_kv_heads:
        raise ValueError(f"{op}: n_heads ({n_heads}) must be a multiple of n_kv_heads ({n_kv_heads})")
    if q.size != n_q * n_heads * head_dim:
        raise ValueError(f"{op}: q has wrong length")
    if k.size != n_kv * n_kv_heads * head_dim or v.size != n_kv * n_kv_heads * head_dim:
        raise ValueError(f"{op}: k/v have wrong length")


def swiglu(g, u) -> np.ndarray:
    g, u = _f32(g), _f32(u)
    if g.size != u.size:
        raise ValueError("swiglu: gate and up must have equal length")
    y = np.empty_like(g)
    lib().orc_swiglu(_p(g), _p(u), g.size, _p(y))
    return y


def dense(w, x, in_features: int, out_features: int) -> np.ndarray:
    w, x = _f32(w), _f32(x)
    if x.size != in_features or w.size != in_features * out_features:
        raise ValueError("dense: shape mismatch")
    y = np.empty(out_features, np.float32)
    lib().orc_dense(_p(w), _p(x), in_features, out_features, _p(y))
    return y


def dense_q(gtype: int, packed: np.ndarray, x, in_features: int, out_features: int,
            f16_round: bool = True) -> np.ndarray:
    """dense over a block-packed weight, dequantized row by row (+ f16 rounding)."""
    b = np.ascontiguousarray(packed, dtype=np.uint8).reshape(-1)
    x = _f32(x)
    y = np.empty(out_features, np.float32)
    lib().orc_dense_q(gtype, _p(b), in_features, out_features, _p(x), _p(y), int(f16_round))
    return y


def residual_add(a, b) -> np.ndarray:
    a, b = _f32(a), _f32(b)
    y = np.empty_like(a)
    lib().orc_residual_add(_p(a), _p(b), a.size, _p(y))
    return y


def log_softmax(x) -> np.ndarray:
    x = _f32(x)
    y = np.empty_like(x)
    if lib().orc_log_softmax(_p(x), x.size, _p(y)) != 0:
        raise ValueError("finite gate: log_softmax input empty or non-finite")
    return y


def top1_non_eog(logits, eog=()) -> int:
    lg = _f32(logits)
    e = np.ascontiguousarray(list(eog) or [0], dtype=np.int64)
    return int(lib().orc_top1_non_eog(_p(lg), lg.size, _p(e), len(eog)))


# --- model ------------------------------------------------------------------

class OracleModel:
    """Shape-parametric CpuOracle (src/cpu_oracle.rs:409-445) over host tensors.

    ``tensors`` maps names to (gtype, array, rows, cols); names are
    ``token_embd``, ``output_norm``, ``output`` and ``blk.{i}.{slot}``. The
    arrays are kept referenced for the model's lifetime.
    """

    def __init__(self, cfg, tensors: dict):
        L = lib()
        self.cfg = cfg
        ci = np.array([cfg.n_layers, cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim,
                       cfg.ffn, cfg.vocab, int(cfg.tied_head)], np.int32)
        cf = np.array([cfg.rms_eps, cfg.rope_theta], np.float32)
        self._h = L.orc_model_new(_p(ci), _p(cf))
        self._keep = []
        for name, (gtype, arr, rows, cols) in tensors.items():
            arr = np.ascontiguousarray(arr)
            self._keep.append(arr)
            if name.startswith("blk."):
                _, i, slot = name.split(".", 2)
                rc = L.orc_model_set(self._h, int(i), SLOT[slot], gtype, _p(arr), rows, cols)
            else:
                rc = L.orc_model_set(self._h, -1, GSLOT[name], gtype, _p(arr), rows, cols)
            if rc != 0:
                raise ValueError(f"oracle rejected tensor {name}")

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            lib().orc_model_free(h)
            self._h = None

    def greedy(self, prompt, n_gen: int, eog=(), want_logits: bool = False):
        """run_greedy (src/greedy_run.rs:186-248): tokens (+ per-step logits)."""
        L = lib()
        pr = np.ascontiguousarray(prompt, dtype=np.int64)
        if pr.size == 0:
            raise ValueError("oracle needs at least one token")
        out = np.empty(n_gen, np.int64)
        e = np.ascontiguousarray(list(eog) or [0], dtype=np.int64)
        lg = np.empty((n_gen, self.cfg.vocab), np.float32) if want_logits else None
        fin = ctypes.c_int32(1)
        rc = L.orc_run_greedy(self._h, _p(pr), pr.size, n_gen, _p(e), len(eog), _p(out),
                              _p(lg) if lg is not None else None, ctypes.byref(fin))
        if rc != 0:
            raise ValueError(f"oracle greedy run failed ({rc})")
        return out, lg, bool(fin.value)


class OracleRun:
    """ForwardRun (src/cpu_oracle.rs:808-926) over an OracleModel."""

    def __init__(self, model: OracleModel, max_ctx: int, trace: bool = False):
        self.model = model
        self._h = lib().orc_run_new(model._h, max_ctx, int(trace))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            lib().orc_run_free(h)
            self._h = None

    def __len__(self):
        return int(lib().orc_run_len(self._h))

    def set_prefix(self, layer: int, k, v, n: int):
        k, v = _f32(k), _f32(v)
        if lib().orc_run_set_prefix(self._h, layer, _p(k), _p(v), n) != 0:
            raise ValueError("bad prefix")

    def push_token(self, token: int):
        rc = lib().orc_run_push(self._h, int(token))
        if rc == -1:
            raise ValueError(f"token {token} is outside the vocab")
        if rc != 0:
            raise ValueError(f"push_token failed ({rc})")

    def position_logits(self) -> np.ndarray:
        out = np.empty(self.model.cfg.vocab, np.float32)
        if lib().orc_run_logits(self._h, _p(out)) != 0:
            raise ValueError("oracle needs at least one token")
        return out

    def hidden(self) -> np.ndarray:
        out = np.empty(self.model.cfg.d_model, np.float32)
        lib().orc_run_hidden(self._h, _p(out))
        return out

    def trace(self, layer: int, which: str) -> np.ndarray:
        c = self.model.cfg
        n = max(c.d_model, c.ffn, c.n_heads * c.head_dim)
        out = np.empty(n, np.float32)
        got = lib().orc_run_trace(self._h, layer, TRACE[which], _p(out))
        if got < 0:
            raise ValueError("trace not recorded")
        return out[:got].copy()
