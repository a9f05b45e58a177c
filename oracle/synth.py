"""Seeded synthetic model tensors through the oracle library — TEST
INFRASTRUCTURE ONLY.

The same counter-based generator as ``faber_runtime_b200.synth`` (the C++
source ``faber_runtime_b200/csrc/synth.cpp`` is linked into the oracle
library too), so a CPU-only caller such as the benchmark's reference leg
draws bit-identical weights, prompts and K/V prefixes without loading the
GPU library. ``tests/test_oracle_synth.py`` checks that both generators
agree byte for byte.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, replace
from typing import Iterator

import numpy as np

from . import F32, Q4_K, lib

_declared = False


def _lib():
    global _declared
    L = lib()
    if not _declared:
        U64, P = ctypes.c_uint64, ctypes.c_void_p
        L.faber_synth_q4k.argtypes = [U64, U64, U64, P]
        L.faber_synth_normal_f32.argtypes = [U64, U64, U64, ctypes.c_float, ctypes.c_float, P]
        L.faber_synth_tokens.argtypes = [U64, U64, U64, ctypes.c_uint32, P]
        for f in (L.faber_synth_q4k, L.faber_synth_normal_f32, L.faber_synth_tokens):
            f.restype = ctypes.c_int32
        _declared = True
    return L


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise ValueError(f"{what} failed with status {rc}")


@dataclass(frozen=True)
class Shape:
    """The decoder shape fields the oracle model reads."""

    n_layers: int
    d_model: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    tied_head: bool
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    name: str = "custom"

    def with_layers(self, n: int) -> "Shape":
        return replace(self, n_layers=n, name=f"{self.name}-L{n}")


LLAMA2_7B = Shape(n_layers=32, d_model=4096, n_heads=32, n_kv_heads=32, head_dim=128, ffn=11008,
                  vocab=32000, tied_head=False, rope_theta=10000.0, name="llama2-7b-shape")


def stream_id(name: str) -> int:
    """Stable 64-bit stream id of a tensor name (FNV-1a)."""
    h = 1469598103934665603
    for b in name.encode():
        h ^= b
        h = (h * 1099511628211) % (1 << 64)
    return h


def q4k_blocks(seed: int, stream: int, n_blocks: int) -> np.ndarray:
    out = np.empty(n_blocks * 144, np.uint8)
    _check(_lib().faber_synth_q4k(seed, stream, n_blocks, out.ctypes.data), "faber_synth_q4k")
    return out


def normal(seed: int, stream: int, n: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    _check(_lib().faber_synth_normal_f32(seed, stream, n, mean, std, out.ctypes.data), "faber_synth_normal_f32")
    return out


def tokens(seed: int, stream: int, n: int, vocab: int) -> np.ndarray:
    out = np.empty(n, np.int64)
    _check(_lib().faber_synth_tokens(seed, stream, n, vocab, out.ctypes.data), "faber_synth_tokens")
    return out


def model_tensors(cfg, seed: int, norms: str = "ones") -> Iterator[tuple[str, int, np.ndarray, int, int]]:
    """(name, ggml_type, array, rows, cols), the tensors and order of
    ``faber_runtime_b200.synth.model_tensors``."""
    d, hd, F, V = cfg.d_model, cfg.head_dim, cfg.ffn, cfg.vocab
    yield ("token_embd", F32, normal(seed, stream_id("token_embd.weight"), V * d, 0.0, 0.02), V, d)
    yield ("output_norm", F32, normal(seed, stream_id("output_norm.weight"), d, 0.0, 0.02), d, 1)
    if not cfg.tied_head:
        yield ("output", Q4_K, q4k_blocks(seed, stream_id("output.weight"), V * d // 256), V, d)
    shapes = {"attn_q": (cfg.n_heads * hd, d), "attn_k": (cfg.n_kv_heads * hd, d),
              "attn_v": (cfg.n_kv_heads * hd, d), "attn_output": (d, cfg.n_heads * hd),
              "ffn_gate": (F, d), "ffn_up": (F, d), "ffn_down": (d, F)}
    for i in range(cfg.n_layers):
        for nm in ("attn_norm", "ffn_norm"):
            if norms == "ones":
                w = np.ones(d, np.float32)
            else:
                w = normal(seed, stream_id(f"blk.{i}.{nm}.weight"), d, 1.0, 0.1)
            yield (f"blk.{i}.{nm}", F32, w, d, 1)
        for nm, (r, c) in shapes.items():
            yield (f"blk.{i}.{nm}", Q4_K, q4k_blocks(seed, stream_id(f"blk.{i}.{nm}.weight"), r * c // 256), r, c)
