"""faber_runtime_b200 — B200 (sm_100a) implementation of faber-runtime's
quantized decoder hot path: GGUF Q4_K dequant -> RMSNorm/RoPE -> GQA
attention -> SwiGLU -> greedy decode, as hand-written CUDA behind the C ABI
in include/faber_gpu.h.

The Python modules mirror the reference's interface for the path (CpuOracle /
ForwardRun / run_greedy / KvCacheLayout / compare_gpu_logits); every compute
call goes through libfaber_gpu.so. There is no CPU fallback.
"""

from . import _lib
from ._lib import FaberError
from .config import LLAMA2_7B, LLAMA3_70B, TINY, KV_F16, KV_F32, KvCacheLayout, ModelConfig
from .decoder import BatchRun, DeviceModel, ForwardRun, GreedyRunRecord, OracleError, run_greedy
from .prefill import compare_gpu_logits, top1_non_eog

__all__ = ["FaberError", "ModelConfig", "KvCacheLayout", "TINY", "LLAMA2_7B", "LLAMA3_70B",
           "KV_F16", "KV_F32", "DeviceModel", "ForwardRun", "BatchRun", "GreedyRunRecord", "OracleError",
           "run_greedy", "compare_gpu_logits", "top1_non_eog", "lib"]


def lib():
    """The loaded C-ABI library (raises when it has not been built)."""
    return _lib.lib()
