"""Device Q4_K kernels on caller-owned device memory.

``dequant_q4k`` is dequant_row for Q4_K (src/dequant.rs:194-217,323-340),
bit-exact with the reference; ``gemv_q4k`` / ``Q4kTensor.gemv`` compute the
reference's dense (src/decoder_ops.rs:378-406) over the f16-rounded
dequantized weight (src/cpu_oracle.rs:356-360). Device buffers are passed as
integer addresses (e.g. ``torch.Tensor.data_ptr()``); ``stream`` is a
cudaStream_t address or 0.
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import _lib

Q4K_BLOCK_BYTES = 144
Q4K_BLOCK_ELEMS = 256


def dequant_q4k(blocks_ptr: int, n_blocks: int, out_ptr: int, f16_round: bool = False,
                stream: int = 0) -> None:
    _lib.call("faber_gpu_v2_dequant_q4k", blocks_ptr, n_blocks, out_ptr, int(f16_round), stream)


def dequant_blocks(ggml_type: int, blocks_ptr: int, n_blocks: int, out_ptr: int,
                   f16_round: bool = False, stream: int = 0) -> None:
    """Any admitted block type (Q4_K, Q6_K, Q5_0, Q8_0, F32, F16) to f32."""
    _lib.call("faber_gpu_v2_dequant_blocks", ggml_type, blocks_ptr, n_blocks, out_ptr, int(f16_round),
              stream)


def f16_round(x_ptr: int, y_ptr: int, n: int, stream: int = 0) -> None:
    _lib.call("faber_gpu_v2_f16_round", x_ptr, y_ptr, n, stream)


def gemv_q4k(w_ptr: int, rows: int, cols: int, x_ptr: int, y_ptr: int, stream: int = 0) -> None:
    """GEMV over native GGUF-ordered Q4_K blocks already on the device."""
    _lib.call("faber_gpu_v2_gemv_q4k", w_ptr, rows, cols, x_ptr, y_ptr, stream)


class Q4kTensor:
    """A Q4_K weight uploaded once and repacked into the kernel's tile layout."""

    def __init__(self, host_blocks: np.ndarray, rows: int, cols: int):
        b = np.ascontiguousarray(host_blocks, dtype=np.uint8)
        h = ctypes.c_void_p()
        _lib.call("faber_gpu_v2_q4k_upload", b.ctypes.data, b.nbytes, rows, cols, ctypes.byref(h))
        self._h = h
        self.rows, self.cols = rows, cols

    def gemv(self, x_ptr: int, y_ptr: int, stream: int = 0) -> None:
        _lib.call("faber_gpu_v2_q4k_gemv", self._h, x_ptr, y_ptr, stream)

    def gemv_batch(self, x_ptr: int, batch: int, y_ptr: int, stream: int = 0) -> None:
        """y[b] = dense(w, x[b]) for b < batch (1..16): x [batch][cols] and y
        [batch][rows] f32 device arrays; each exact weight fragment serves
        every sequence."""
        _lib.call("faber_gpu_v2_q4k_gemv_batch", self._h, x_ptr, int(batch), y_ptr, stream)

    def dequant_rows(self, out_ptr: int, f16_round: bool = True, stream: int = 0) -> None:
        _lib.call("faber_gpu_v2_q4k_dequant_rows", self._h, out_ptr, int(f16_round), stream)

    def gemv_exchange(self, x_ptr: int, norm_w_ptr: int, eps: float, exchange_ptr: int, tp: int,
                      epoch: int, wait_limit: int, x_sum_ptr: int, y_ptr: int, stream: int = 0) -> None:
        """The exchange-consuming GEMV of a tensor-parallel step on local
        buffers: x_sum = x + the tp partial rows of ``exchange`` whose words
        carry ``epoch``; y = dense(w, rms_norm(x_sum) * norm_w). Raises
        FaberError(TIMEOUT) when a word never carries the epoch."""
        _lib.call("faber_gpu_v2_q4k_gemv_exchange", self._h, x_ptr, norm_w_ptr, float(eps), exchange_ptr,
                  int(tp), int(epoch), int(wait_limit), x_sum_ptr, y_ptr, stream)

    def repack_hash(self) -> int:
        v = _lib.U64()
        _lib.call("faber_gpu_v2_q4k_repack_hash", self._h, ctypes.byref(v))
        return v.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.call("faber_gpu_v2_q4k_free", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# --- placement ABI (hosts/llvm/src/gpu_placement.rs) --------------------------

def copy_in(logical_id: int, data: bytes | np.ndarray, dtype: int = 0) -> None:
    a = np.frombuffer(bytes(data), np.uint8) if isinstance(data, (bytes, bytearray)) else \
        np.ascontiguousarray(data).view(np.uint8).reshape(-1)
    _lib.call("__faber_gpu_v1_copy_in", logical_id, a.ctypes.data if a.size else None, a.size, dtype)


def readback(logical_id: int, capacity: int) -> bytes:
    buf = (ctypes.c_uint8 * max(capacity, 1))()
    n = _lib.U64()
    _lib.call("__faber_gpu_v1_readback", logical_id, ctypes.addressof(buf), capacity, ctypes.byref(n))
    return bytes(buf[:n.value])


def sync(logical_id: int = 0) -> None:
    _lib.call("__faber_gpu_v1_sync", logical_id)


def device_ptr(logical_id: int) -> tuple[int, int]:
    p, n = ctypes.c_void_p(), _lib.U64()
    _lib.call("faber_gpu_v2_buffer_device_ptr", logical_id, ctypes.byref(p), ctypes.byref(n))
    return p.value or 0, n.value


class TypedTensor:
    """A linear of any admitted block type as typed rows (the row GEMV of
    the decoder's non-Q4_K linears)."""

    def __init__(self, ggml_type: int, host_blocks: np.ndarray, rows: int, cols: int):
        b = np.ascontiguousarray(host_blocks, dtype=np.uint8)
        h = ctypes.c_void_p()
        _lib.call("faber_gpu_v2_typed_upload", ggml_type, b.ctypes.data, b.nbytes, rows, cols,
                  ctypes.byref(h))
        self._h = h
        self.rows, self.cols = rows, cols

    def gemv(self, x_ptr: int, y_ptr: int, stream: int = 0) -> None:
        _lib.call("faber_gpu_v2_typed_gemv", self._h, x_ptr, y_ptr, stream)

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.call("faber_gpu_v2_typed_free", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
