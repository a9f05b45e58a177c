"""Model shapes and the KV layout (src/kv_cache.rs) of the Q4_K decoder path.

The reference hard-codes one model's facts as constants
(src/decoder_ops.rs:60-79, src/cpu_oracle.rs:128-154); here they are one
``ModelConfig``. The presets are the decoder workloads this path is measured
on: a 4-layer 512-wide model (tiny), Llama-2-7B's shape and Llama-3-70B's
shape (GQA 64/8).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, replace

from . import _lib


@dataclass(frozen=True)
class ModelConfig:
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

    def with_layers(self, n: int) -> "ModelConfig":
        return replace(self, n_layers=n, name=f"{self.name}-L{n}")

    def c_struct(self, tp_size: int = 1, tp_rank: int = 0, uid: bytes = b"") -> _lib.ModelConfigC:
        c = _lib.ModelConfigC()
        c.n_layers, c.d_model, c.n_heads = self.n_layers, self.d_model, self.n_heads
        c.n_kv_heads, c.head_dim, c.ffn, c.vocab = self.n_kv_heads, self.head_dim, self.ffn, self.vocab
        c.tied_head = int(self.tied_head)
        c.rms_eps, c.rope_theta = self.rms_eps, self.rope_theta
        c.tp_size, c.tp_rank = tp_size, tp_rank
        if uid:
            ctypes.memmove(c.nccl_unique_id, uid, 128)
        return c

    # --- byte accounting (algorithmic bytes per decoded token) --------------
    def linear_bytes(self) -> int:
        """Q4_K bytes of all per-layer linears (0.5625 B per weight)."""
        d, hd, F = self.d_model, self.head_dim, self.ffn
        per = (self.n_heads * hd * d + 2 * self.n_kv_heads * hd * d + d * self.n_heads * hd
               + 3 * F * d)
        return self.n_layers * per * 144 // 256

    def head_bytes(self) -> int:
        if self.tied_head:
            return self.vocab * self.d_model * 2  # f16-rounded embedding read as f16
        return self.vocab * self.d_model * 144 // 256

    def kv_bytes_per_position(self, dtype_bytes: int = 2) -> int:
        return 2 * self.n_layers * self.n_kv_heads * self.head_dim * dtype_bytes


TINY = ModelConfig(n_layers=4, d_model=512, n_heads=8, n_kv_heads=8, head_dim=64, ffn=1408,
                   vocab=32000, tied_head=True, rope_theta=10000.0, name="tiny-L4-d512")
LLAMA2_7B = ModelConfig(n_layers=32, d_model=4096, n_heads=32, n_kv_heads=32, head_dim=128,
                        ffn=11008, vocab=32000, tied_head=False, rope_theta=10000.0,
                        name="llama2-7b-shape")
LLAMA3_70B = ModelConfig(n_layers=80, d_model=8192, n_heads=64, n_kv_heads=8, head_dim=128,
                         ffn=28672, vocab=128256, tied_head=False, rope_theta=500000.0,
                         name="llama3-70b-shape")

KV_F32, KV_F16 = 0, 1


@dataclass(frozen=True)
class KvCacheLayout:
    """KvCacheLayout (src/kv_cache.rs:504-626): slots x context x layers x
    kv heads x head_dim, K and V both resident."""

    slots: int
    context_length: int
    layer_count: int
    kv_head_count: int
    head_dim: int
    dtype: int = KV_F16
    reserve_bytes: int = 0

    @staticmethod
    def for_model(cfg: ModelConfig, context_length: int, dtype: int = KV_F16) -> "KvCacheLayout":
        return KvCacheLayout(1, context_length, cfg.n_layers, cfg.n_kv_heads, cfg.head_dim, dtype)

    def c_struct(self) -> _lib.KvLayoutC:
        c = _lib.KvLayoutC()
        c.slots, c.context_length, c.layer_count = self.slots, self.context_length, self.layer_count
        c.kv_head_count, c.head_dim, c.dtype = self.kv_head_count, self.head_dim, self.dtype
        c.reserve_bytes = self.reserve_bytes
        return c

    def dtype_byte_size(self) -> int:
        return 4 if self.dtype == KV_F32 else 2

    def elements_per_slot(self) -> int:
        return self.context_length * self.kv_head_count * self.head_dim * self.layer_count * 2

    def total_bytes(self) -> int | None:
        """Storage bytes; None when a dimension is zero or the count overflows u64."""
        if 0 in (self.slots, self.context_length, self.layer_count, self.kv_head_count,
                 self.head_dim):
            return None
        b = self.elements_per_slot() * self.dtype_byte_size() * self.slots
        return b if b < 2 ** 64 else None

    def admitted_bytes(self) -> int | None:
        t = self.total_bytes()
        if t is None or t + self.reserve_bytes >= 2 ** 64:
            return None
        return t + self.reserve_bytes

    def device_bytes(self) -> tuple[int, int]:
        """(total, admitted) computed by the C ABI (raises on a bad layout)."""
        tot, adm = _lib.U64(), _lib.U64()
        c = self.c_struct()
        _lib.call("faber_gpu_v2_kv_layout_bytes", ctypes.byref(c), ctypes.byref(tot),
                  ctypes.byref(adm))
        return tot.value, adm.value
