"""Seeded synthetic inputs (counter-based, identical bytes for any chunking).

Q4_K super-blocks: d, dmin = f16(U[1e-3, 2e-2]); the 12 scale bytes and 128
quant bytes uniform (every 6-bit scale/min and every 4-bit quant uniform).
Activations x ~ N(0, 1); token embedding and output norm ~ N(0, 0.02);
per-layer norm weights 1.0 (``norms="ones"``) or N(1, 0.1) (``"random"``).
"""

from __future__ import annotations

import ctypes
from typing import Iterator

import numpy as np

from . import _lib
from .config import ModelConfig


def stream_id(name: str) -> int:
    """Stable 64-bit stream id of a tensor name (FNV-1a)."""
    h = 1469598103934665603
    for b in name.encode():
        h ^= b
        h = (h * 1099511628211) % (1 << 64)
    return h


def q4k_blocks(seed: int, stream: int, n_blocks: int) -> np.ndarray:
    out = np.empty(n_blocks * 144, np.uint8)
    _lib.call("faber_synth_q4k", seed, stream, n_blocks, out.ctypes.data)
    return out


def normal(seed: int, stream: int, n: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    _lib.call("faber_synth_normal_f32", seed, stream, n, ctypes.c_float(mean),
              ctypes.c_float(std), out.ctypes.data)
    return out


def tokens(seed: int, stream: int, n: int, vocab: int) -> np.ndarray:
    out = np.empty(n, np.int64)
    _lib.call("faber_synth_tokens", seed, stream, n, vocab, out.ctypes.data)
    return out


def q4k_tensor(seed: int, name: str, rows: int, cols: int) -> np.ndarray:
    assert (rows * cols) % 256 == 0
    return q4k_blocks(seed, stream_id(name), rows * cols // 256)


def model_tensors(cfg: ModelConfig, seed: int, norms: str = "ones",
                  layers: range | None = None) -> Iterator[tuple[str, int, np.ndarray, int, int]]:
    """Yield (name, ggml_type, array, rows, cols) one tensor at a time."""
    d, hd, F, V = cfg.d_model, cfg.head_dim, cfg.ffn, cfg.vocab
    yield ("token_embd", _lib.GGML_F32, normal(seed, stream_id("token_embd.weight"), V * d, 0.0, 0.02),
           V, d)
    yield ("output_norm", _lib.GGML_F32, normal(seed, stream_id("output_norm.weight"), d, 0.0, 0.02),
           d, 1)
    if not cfg.tied_head:
        yield ("output", _lib.GGML_Q4_K, q4k_tensor(seed, "output.weight", V, d), V, d)
    shapes = {"attn_q": (cfg.n_heads * hd, d), "attn_k": (cfg.n_kv_heads * hd, d),
              "attn_v": (cfg.n_kv_heads * hd, d), "attn_output": (d, cfg.n_heads * hd),
              "ffn_gate": (F, d), "ffn_up": (F, d), "ffn_down": (d, F)}
    for i in (layers if layers is not None else range(cfg.n_layers)):
        for nm in ("attn_norm", "ffn_norm"):
            if norms == "ones":
                w = np.ones(d, np.float32)
            else:
                w = normal(seed, stream_id(f"blk.{i}.{nm}.weight"), d, 1.0, 0.1)
            yield (f"blk.{i}.{nm}", _lib.GGML_F32, w, d, 1)
        for nm, (r, c) in shapes.items():
            yield (f"blk.{i}.{nm}", _lib.GGML_Q4_K, q4k_tensor(seed, f"blk.{i}.{nm}.weight", r, c), r, c)
