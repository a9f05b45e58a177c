"""Partition byte budgets: the PartitionBudgetLedger of src/partition.rs and
its admission rule, over the library's per-device accounting.

* ``PartitionLedger`` holds the seven byte classes of the reference's ledger
  (src/partition.rs:111-137); ``total_bytes`` is its checked sum
  (src/partition.rs:139-155): ``None`` when it overflows u64.
* ``admit`` is VirtualDevicePartition::admit (src/partition.rs:293-315): the
  declared ledger against a policy limit, BUDGET_EXCEEDED (also on
  overflow) before anything is allocated.
* ``plan`` is what one tensor-parallel rank's model and sessions will hold,
  computed on the host from the configuration with the engine's own buffer
  formulas, so it can be admitted before the upload starts.
* ``usage`` is what the library holds on a device right now, by class, and
  ``set_limit`` makes every later allocation on that device fail with
  ALLOCATION once its charge would pass the limit: growth after admission is
  an allocation outcome, not a ledger rewrite (src/partition.rs:111-114).
"""

from __future__ import annotations

import ctypes
from dataclasses import astuple, dataclass, fields

from . import _lib
from .config import ModelConfig

U64_MAX = (1 << 64) - 1


@dataclass(frozen=True)
class PartitionLedger:
    weight_bytes: int = 0
    kv_cache_bytes: int = 0
    activation_scratch_bytes: int = 0
    module_storage_bytes: int = 0
    allocator_overhead_bytes: int = 0
    transfer_staging_bytes: int = 0
    concurrent_state_bytes: int = 0

    def total_bytes(self) -> int | None:
        """Checked u64 sum of the seven classes (None on overflow)."""
        total = 0
        for v in astuple(self):
            total += v
            if total > U64_MAX:
                return None
        return total

    def c_struct(self) -> _lib.PartitionLedgerC:
        c = _lib.PartitionLedgerC()
        for f in fields(self):
            setattr(c, f.name, getattr(self, f.name))
        return c

    @classmethod
    def from_c(cls, c: _lib.PartitionLedgerC) -> "PartitionLedger":
        return cls(**{f.name: int(getattr(c, f.name)) for f in fields(cls)})


def admit(declared: PartitionLedger, safe_limit_bytes: int) -> int:
    """The declared total when it fits the limit; raises FaberError
    (BUDGET_EXCEEDED) otherwise, also when the classes overflow u64."""
    total = _lib.U64()
    _lib.call("faber_gpu_v2_partition_admit", ctypes.byref(declared.c_struct()), int(safe_limit_bytes),
              ctypes.byref(total))
    return total.value


def plan(cfg: ModelConfig, context_length: int, sessions: int = 1, sms: int = 148,
         tp_size: int = 1, tp_rank: int = 0) -> PartitionLedger:
    """The ledger of rank ``tp_rank`` of ``tp_size`` for an all-Q4_K model
    and ``sessions`` sessions of ``context_length`` positions on a device
    with ``sms`` SMs (148 on a B200)."""
    out = _lib.PartitionLedgerC()
    _lib.call("faber_gpu_v2_partition_plan", ctypes.byref(cfg.c_struct(tp_size, tp_rank)),
              int(context_length), int(sessions), int(sms), ctypes.byref(out))
    return PartitionLedger.from_c(out)


def usage(device: int = 0) -> PartitionLedger:
    """The bytes this library holds on ``device`` now, by class."""
    out = _lib.PartitionLedgerC()
    _lib.call("faber_gpu_v2_partition_usage", int(device), ctypes.byref(out))
    return PartitionLedger.from_c(out)


def set_limit(device: int, safe_limit_bytes: int) -> None:
    """Policy limit of ``device`` (0 removes it)."""
    _lib.call("faber_gpu_v2_partition_set_limit", int(device), int(safe_limit_bytes))
