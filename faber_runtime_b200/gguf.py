"""GGUF v3 files: the library's fail-closed reader (faber_gpu_v2_gguf_*) and
a loader that builds a DeviceModel from a llama-architecture file.

The reference admits one pinned file (src/gguf.rs:581-812); the reader here
keeps its structural checks without the pin. The loader maps the llama.*
metadata to a ModelConfig and uploads every tensor as its raw GGUF blocks
(the same bytes src/gguf.rs hands to CpuOracle::build). Linears may be
Q4_K (the tiled tensor-core GEMV) or Q6_K, Q5_0 and Q8_0 (the typed-row
GEMV; a Q4_K_M file mixes them); others are refused with UNSUPPORTED. The
embedding may be F32, F16 (widened exactly) or any of those block types
(dequantized exactly on the GPU; the model then rounds it to f16 like the
reference's token_embd).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import _lib
from .config import ModelConfig

GGML_F32, GGML_F16, GGML_Q5_0, GGML_Q8_0, GGML_Q4_K, GGML_Q6_K = 0, 1, 6, 8, 12, 14
GGML_NAMES = {0: "F32", 1: "F16", 6: "Q5_0", 8: "Q8_0", 12: "Q4_K", 14: "Q6_K"}


class GgufTensorC(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 256), ("ggml_type", ctypes.c_uint32),
                ("n_dims", ctypes.c_uint32), ("dims", ctypes.c_uint64 * 4),
                ("elements", ctypes.c_uint64), ("nbytes", ctypes.c_uint64),
                ("offset", ctypes.c_uint64)]


@dataclass(frozen=True)
class TensorInfo:
    name: str
    ggml_type: int
    dims: tuple          # GGML order: dims[0] is a row's length
    elements: int
    nbytes: int
    offset: int          # into the file

    @property
    def rows(self) -> int:
        return int(np.prod(self.dims[1:])) if len(self.dims) > 1 else self.dims[0]

    @property
    def cols(self) -> int:
        return self.dims[0] if len(self.dims) > 1 else 1


class GgufFile:
    """A parsed GGUF file (a path, memory-mapped, or bytes)."""

    def __init__(self, source):
        if isinstance(source, (bytes, bytearray, memoryview)):
            self.buf = np.frombuffer(source, dtype=np.uint8)
        elif isinstance(source, np.ndarray):
            self.buf = np.ascontiguousarray(source, dtype=np.uint8)
        else:
            p = Path(source)
            self.buf = (np.memmap(p, dtype=np.uint8, mode="r") if p.stat().st_size
                        else np.zeros(0, np.uint8))
        h = ctypes.c_void_p()
        ptr = self.buf.ctypes.data if self.buf.size else None
        _lib.call("faber_gpu_v2_gguf_parse", ptr, self.buf.size, ctypes.byref(h))
        self._h = h
        ver, nkv, nt, doff, al = _lib.U32(), _lib.U64(), _lib.U64(), _lib.U64(), _lib.U64()
        _lib.call("faber_gpu_v2_gguf_info", self._h, ctypes.byref(ver), ctypes.byref(nkv),
                  ctypes.byref(nt), ctypes.byref(doff), ctypes.byref(al))
        self.version, self.data_offset, self.alignment = ver.value, doff.value, al.value
        self.tensors: dict[str, TensorInfo] = {}
        for i in range(nt.value):
            t = GgufTensorC()
            _lib.call("faber_gpu_v2_gguf_tensor", self._h, i, ctypes.addressof(t))
            name = t.name.decode()
            self.tensors[name] = TensorInfo(name, t.ggml_type, tuple(t.dims[:t.n_dims]),
                                            t.elements, t.nbytes, t.offset)
        self.keys = []
        for i in range(nkv.value):
            key = ctypes.create_string_buffer(1025)
            ty, at, ac = _lib.U32(), _lib.U32(), _lib.U64()
            _lib.call("faber_gpu_v2_gguf_kv", self._h, i, key, 1025, ctypes.byref(ty),
                      ctypes.byref(at), ctypes.byref(ac))
            self.keys.append((key.value.decode(), ty.value, at.value, ac.value))

    def has(self, key: str) -> bool:
        return any(k == key for k, *_ in self.keys)

    def get_int(self, key: str, default=None) -> int:
        if default is not None and not self.has(key):
            return default
        v = _lib.I64()
        _lib.call("faber_gpu_v2_gguf_get_int", self._h, key.encode(), ctypes.byref(v))
        return v.value

    def get_float(self, key: str, default=None) -> float:
        if default is not None and not self.has(key):
            return default
        v = ctypes.c_double()
        _lib.call("faber_gpu_v2_gguf_get_float", self._h, key.encode(), ctypes.byref(v))
        return v.value

    def get_string(self, key: str) -> str:
        n = _lib.U64()
        try:
            _lib.call("faber_gpu_v2_gguf_get_string", self._h, key.encode(), None, 0, ctypes.byref(n))
        except _lib.FaberError as e:
            if e.code != 2:  # IO_ERROR: the length is known now
                raise
        buf = ctypes.create_string_buffer(n.value + 1)
        _lib.call("faber_gpu_v2_gguf_get_string", self._h, key.encode(), buf, n.value + 1, ctypes.byref(n))
        return buf.raw[:n.value].decode()

    def tensor_bytes(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        return self.buf[t.offset:t.offset + t.nbytes]

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.call("faber_gpu_v2_gguf_free", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def llama_config(g: GgufFile, name: str = "gguf") -> ModelConfig:
    """ModelConfig from the llama.* metadata (src/gguf.rs:80-120 admits the
    same keys for its row)."""
    arch = g.get_string("general.architecture")
    if arch != "llama":
        raise _lib.FaberError(4, f"GGUF ArchitectureMismatch: {arch!r} (the decoder runs llama)")
    d = g.get_int(f"{arch}.embedding_length")
    heads = g.get_int(f"{arch}.attention.head_count")
    emb = g.tensors.get("token_embd.weight")
    if emb is None or len(emb.dims) != 2:
        raise _lib.FaberError(1, "GGUF file has no 2-D token_embd.weight")
    return ModelConfig(
        n_layers=g.get_int(f"{arch}.block_count"), d_model=d, n_heads=heads,
        n_kv_heads=g.get_int(f"{arch}.attention.head_count_kv", heads),
        head_dim=g.get_int(f"{arch}.attention.key_length", d // heads),
        ffn=g.get_int(f"{arch}.feed_forward_length"), vocab=emb.dims[1],
        tied_head="output.weight" not in g.tensors,
        rms_eps=g.get_float(f"{arch}.attention.layer_norm_rms_epsilon", 1e-5),
        rope_theta=g.get_float(f"{arch}.rope.freq_base", 10000.0), name=name)


def _embedding_f32(g: GgufFile, t: TensorInfo, device: int) -> np.ndarray:
    raw = g.tensor_bytes(t.name)
    if t.ggml_type == GGML_F32:
        return raw.view(np.float32)
    if t.ggml_type == GGML_F16:
        return raw.view(np.float16).astype(np.float32)
    if t.ggml_type in (GGML_Q4_K, GGML_Q6_K, GGML_Q5_0, GGML_Q8_0):
        import torch
        from . import dequant
        be = 256 if t.ggml_type in (GGML_Q4_K, GGML_Q6_K) else 32
        blocks = torch.from_numpy(np.ascontiguousarray(raw)).to(f"cuda:{device}")
        out = torch.empty(t.elements, dtype=torch.float32, device=f"cuda:{device}")
        dequant.dequant_blocks(t.ggml_type, blocks.data_ptr(), t.elements // be, out.data_ptr(),
                               f16_round=False, stream=torch.cuda.current_stream(device).cuda_stream)
        torch.cuda.synchronize(device)
        return out.cpu().numpy()
    raise _lib.FaberError(4, f"{t.name}: a {GGML_NAMES[t.ggml_type]} embedding is not supported")


def model_tensors(g: GgufFile, cfg: ModelConfig, device: int = 0):
    """(name, ggml_type, array, rows, cols) for DeviceModel, in file order."""
    for t in g.tensors.values():
        if t.name == "token_embd.weight":
            yield t.name, GGML_F32, _embedding_f32(g, t, device), t.rows, t.cols
        elif t.name.endswith("norm.weight"):
            if t.ggml_type != GGML_F32:
                raise _lib.FaberError(4, f"{t.name}: norms must be F32")
            yield t.name, GGML_F32, g.tensor_bytes(t.name).view(np.float32), t.rows, 1
        else:
            if t.ggml_type not in (GGML_Q4_K, GGML_Q6_K, GGML_Q5_0, GGML_Q8_0):
                raise _lib.FaberError(4, f"{t.name}: {GGML_NAMES[t.ggml_type]} linears are not supported "
                                         "(the decoder takes Q4_K, Q6_K, Q5_0 and Q8_0)")
            yield t.name, t.ggml_type, g.tensor_bytes(t.name), t.rows, t.cols


def load_llama(path, device: int = 0, tp_size: int = 1, tp_rank: int = 0, nccl_uid: bytes = b""):
    """Parse a llama GGUF file and upload it: returns (DeviceModel, GgufFile)."""
    from .decoder import DeviceModel
    g = GgufFile(path)
    cfg = llama_config(g, name=Path(str(path)).stem if not isinstance(path, (bytes, bytearray)) else "gguf")
    model = DeviceModel(cfg, model_tensors(g, cfg, device), device=device, tp_size=tp_size,
                        tp_rank=tp_rank, nccl_uid=nccl_uid)
    return model, g
