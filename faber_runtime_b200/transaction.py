"""Execution transactions over the ranks of a group, mirroring
src/execution_transaction (ExecutionTransaction, the fault-injecting
backend of src/fake_device.rs) on the library's C ABI.

A transaction runs an accepted plan of operations over partitions (the
ranks of a tensor-parallel group, 0-63):

* ``prepare`` checks, in the reference's order, that every partition an
  operation uses is in the plan, that operation identities are unique, that
  the commit boundary names declared barriers and launches, and that every
  used partition has an admitted ledger. It then derives the reservation
  (staging in class 6; outputs, event objects and scratch in class 3),
  checks it against the admitted ledgers and holds it on the backend.
* ``execute`` runs the operations in plan order. A backend failure leaves
  the transaction Failed, and it cannot run again.
* ``commit`` publishes the whole staged write-set at once, after every
  boundary barrier and launch has completed on all its partitions. A
  missing boundary is transient (BoundaryNotReached): nothing is published,
  and commit can be called again.
* ``abort`` retires the partitions holding staged writes and releases the
  rest, and never publishes in part. It is idempotent.

Operation references are integers (the reference's LaunchRef /
TransferRef / CollectiveRef / BarrierRef strings).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Iterable

from . import _lib
from .partition import PartitionLedger

LAUNCH, TRANSFER, BROADCAST, BARRIER = 0, 1, 2, 3

ERROR_KINDS = ["", "DegeneratePlan", "EmptySnapshot", "InvalidState", "UnknownPartition", "DuplicateOperation",
               "UndeclaredBoundaryBarrier", "UndeclaredBoundaryLaunch", "MissingAdmittedBudget",
               "ReservationExceedsBudget", "Backend", "OperationOutsideSnapshot", "BoundaryNotReached",
               "PublishFailed", "AlreadyCommitted"]
STATES = ["New", "Prepared", "Executing", "Committed", "Failed", "Aborted"]
BACKEND_CLASSES = {1: "Allocation", 2: "Operation", 3: "DeviceLoss", 4: "Cancelled", 5: "Timeout"}
FAILURE_KINDS = ["", "Backend", "PublishFailed", "Cancelled"]

# fault classes of src/fake_device.rs
CANCEL, TIMEOUT, TRANSFER_ERROR, KERNEL_ERROR, DEVICE_LOSS = 1, 2, 3, 4, 5


def _mask(parts: Iterable[int]) -> int:
    m = 0
    for p in parts:
        m |= 1 << int(p)
    return m


@dataclass(frozen=True)
class Op:
    kind: int
    ref: int
    partition: int = 0
    destination: int = 0
    participants: int = 0   # mask
    bytes: int = 0

    def c_struct(self) -> _lib.TxnOpC:
        return _lib.TxnOpC(self.kind, self.partition, self.destination, 0, self.participants, self.ref,
                           self.bytes)


def launch(partition: int, ref: int, output_bytes: int) -> Op:
    return Op(LAUNCH, ref, partition=partition, bytes=output_bytes)


def transfer(ref: int, source: int, destination: int, byte_count: int) -> Op:
    return Op(TRANSFER, ref, partition=source, destination=destination, bytes=byte_count)


def broadcast(ref: int, source: int, participants: Iterable[int], byte_count: int) -> Op:
    return Op(BROADCAST, ref, partition=source, participants=_mask(participants), bytes=byte_count)


def barrier(ref: int, participants: Iterable[int]) -> Op:
    return Op(BARRIER, ref, participants=_mask(participants))


class TransactionError(_lib.FaberError):
    """A refused lifecycle call: ``kind`` is the reference's error variant
    (errors.rs), ``backend_class`` the backend error class for Backend and
    PublishFailed."""

    def __init__(self, code: int, message: str, kind: str, partition: int = 0, backend_class: str = "",
                 budget_class: int = 0, missing: int = 0):
        super().__init__(code, message)
        self.kind, self.partition, self.backend_class = kind, partition, backend_class
        self.budget_class, self.missing = budget_class, missing


@dataclass(frozen=True)
class Receipt:
    decision: str            # "", "Committed", "Aborted"
    state: str
    failure_kind: str
    failure_class: str
    failure_partition: int
    published: bool
    publication_ordinal: int
    declared_write_bytes: int
    executed_operations: int
    executed_bytes: int
    completed_events: int
    staged_bytes: int
    published_bytes: int
    released_partitions: frozenset
    retired_partitions: frozenset
    partial_publication: bool


def _parts(mask: int) -> frozenset:
    return frozenset(p for p in range(64) if mask >> p & 1)


class FaultBackend:
    """The happy-path fake with one-shot faults per (operation, partition)
    (FaultInjectingBackend). All state is host-side."""

    def __init__(self):
        h = ctypes.c_void_p()
        _lib.call("faber_gpu_v2_txn_backend_fake", ctypes.byref(h))
        self._h = h

    def inject(self, op: Op, partition: int, fault_class: int) -> None:
        _lib.call("faber_gpu_v2_txn_backend_inject", self._h, op.kind, op.ref, partition, fault_class)

    def fail_publish(self, backend_class: int = 2) -> None:
        _lib.call("faber_gpu_v2_txn_backend_fail_publish", self._h, backend_class)

    def set_auto_complete(self, on: bool) -> None:
        _lib.call("faber_gpu_v2_txn_backend_set_auto_complete", self._h, int(on))

    def complete_event(self, op: Op, partition: int) -> None:
        _lib.call("faber_gpu_v2_txn_backend_complete_event", self._h, op.kind, partition, op.ref)

    def info(self) -> dict:
        c = _lib.TxnBackendInfoC()
        _lib.call("faber_gpu_v2_txn_backend_info", self._h, ctypes.byref(c))
        d = {n: int(getattr(c, n)) for n, _ in c._fields_}
        for k in ("reserved_partitions", "released_partitions", "retired_partitions"):
            d[k] = _parts(d[k])
        return d

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.call("faber_gpu_v2_txn_backend_free", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Transaction:
    """ExecutionTransaction over ``partitions`` ({partition: admitted ledger
    or None}) and the accepted ``operations`` with the commit boundary."""

    def __init__(self, partitions: dict, operations: list, boundary_barriers: Iterable[int] = (),
                 boundary_launches: Iterable[int] = ()):
        parts = (_lib.TxnPartitionC * max(1, len(partitions)))()
        for i, (p, led) in enumerate(sorted(partitions.items())):
            parts[i].partition = p
            parts[i].admitted = int(led is not None)
            if led is not None:
                parts[i].ledger = led.c_struct()
        ops = (_lib.TxnOpC * max(1, len(operations)))(*[o.c_struct() for o in operations])
        bb = list(boundary_barriers)
        bl = list(boundary_launches)
        barr = (ctypes.c_uint64 * max(1, len(bb)))(*bb)
        larr = (ctypes.c_uint64 * max(1, len(bl)))(*bl)
        h = ctypes.c_void_p()
        try:
            _lib.call("faber_gpu_v2_txn_create", parts, len(partitions), ops, len(operations), barr, len(bb),
                      larr, len(bl), ctypes.byref(h))
        except _lib.FaberError as e:
            kind = next((k for k in ERROR_KINDS[1:3] if k in e.message), "")
            raise TransactionError(e.code, e.message, kind) from None
        self._h = h

    def _run(self, name: str, *args) -> None:
        try:
            _lib.call(name, self._h, *args)
        except _lib.FaberError as e:
            c = _lib.TxnErrorC()
            _lib.call("faber_gpu_v2_txn_last_error", self._h, ctypes.byref(c))
            raise TransactionError(e.code, e.message, ERROR_KINDS[c.kind], c.partition,
                                   BACKEND_CLASSES.get(c.backend_class, ""), c.budget_class, c.missing) from None

    def prepare(self, backend: FaultBackend) -> None:
        self._run("faber_gpu_v2_txn_prepare", backend._h)

    def execute(self, backend: FaultBackend) -> None:
        self._run("faber_gpu_v2_txn_execute", backend._h)

    def execute_operation(self, backend: FaultBackend, op: Op) -> None:
        c = op.c_struct()
        self._run("faber_gpu_v2_txn_execute_operation", backend._h, ctypes.byref(c))

    def commit(self, backend: FaultBackend, ordinal: int) -> Receipt:
        self._run("faber_gpu_v2_txn_commit", backend._h, ordinal)
        return self.receipt()

    def abort(self, backend: FaultBackend, reason: str = "") -> Receipt:
        self._run("faber_gpu_v2_txn_abort", backend._h, reason.encode())
        return self.receipt()

    @property
    def state(self) -> str:
        return self.receipt().state

    def reservation(self, partition: int) -> dict:
        out = (ctypes.c_uint64 * 4)()
        self._run("faber_gpu_v2_txn_reservation", partition, out)
        staging, output, events, scratch = (int(v) for v in out)
        return {"staging": staging, "output": output, "events": events, "scratch": scratch,
                "class_six": staging, "class_three": output + events + scratch}

    def receipt(self) -> Receipt:
        c = _lib.TxnReceiptC()
        _lib.call("faber_gpu_v2_txn_receipt", self._h, ctypes.byref(c))
        return Receipt(decision=["", "Committed", "Aborted"][c.decision], state=STATES[c.state],
                       failure_kind=FAILURE_KINDS[c.failure_kind],
                       failure_class=BACKEND_CLASSES.get(c.failure_class, ""),
                       failure_partition=c.failure_partition, published=bool(c.published),
                       publication_ordinal=c.publication_ordinal, declared_write_bytes=c.declared_write_bytes,
                       executed_operations=c.executed_operations, executed_bytes=c.executed_bytes,
                       completed_events=c.completed_events, staged_bytes=c.staged_bytes,
                       published_bytes=c.published_bytes, released_partitions=_parts(c.released_partitions),
                       retired_partitions=_parts(c.retired_partitions),
                       partial_publication=bool(c.partial_publication))

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.call("faber_gpu_v2_txn_free", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def tp_step_plan(cfg, tp_size: int, position: int):
    """One decode step of a ``tp_size``-rank group as (operations, boundary
    barriers, boundary launches): per rank its step launch, publishing its
    K/V rows and the token, then the group's exchange barrier."""
    c = cfg.c_struct(tp_size, 0)
    n = _lib.U32()
    barrier_ref = _lib.U64()
    ops = (_lib.TxnOpC * (tp_size + 1))()
    launches = (ctypes.c_uint64 * tp_size)()
    _lib.call("faber_gpu_v2_tp_step_plan", ctypes.byref(c), position, ops, len(ops), ctypes.byref(n),
              ctypes.byref(barrier_ref), launches)
    out = [Op(o.kind, o.ref, o.partition, o.destination, o.participants, o.bytes) for o in ops[:n.value]]
    return out, [barrier_ref.value], list(launches)


def admitted(transfer_staging_bytes: int, activation_scratch_bytes: int, **classes) -> PartitionLedger:
    """A ledger with the two classes a transaction reserves against."""
    return PartitionLedger(transfer_staging_bytes=transfer_staging_bytes,
                           activation_scratch_bytes=activation_scratch_bytes, **classes)


def realign_after_abort(session, length: int, group=None) -> None:
    """Put a tensor-parallel session back where the group agreed after an
    aborted step: the sequence is truncated to ``length`` (on a rank whose
    step ran; a rank whose step failed was rolled back by the call itself),
    and every rank raises its exchange epoch to the largest in the group, so
    that the next step's exchanges match on every rank again and no epoch
    is used twice. Every rank of the group must call it."""
    import torch
    import torch.distributed as dist
    if len(session) > length:
        session.truncate(length)
    e = torch.tensor([session.exchange_epoch()], dtype=torch.int64)
    dist.all_reduce(e, op=dist.ReduceOp.MAX, group=group)
    session.exchange_epoch(int(e.item()))


def run_group_step(t: Transaction, backend: FaultBackend, ordinal: int, group=None, step=None,
                   publish=None, session=None) -> Receipt:
    """Execute this rank's transaction, then agree with every rank of the
    process group on the outcome before anything is published: commit only
    when every rank executed its step, abort everywhere otherwise.

    ``step`` is this rank's device work for the position (for example
    ``lambda: run.step_greedy(token)``). Any exception from it counts as
    this rank failing: a FaberError (a TIMEOUT of a bounded exchange wait,
    DEVICE_LOSS, ...), and also any other error, such as the OracleError a
    rejected token id raises. The rank still joins the group's vote, so the
    other ranks abort at once instead of waiting for the group's timeout.
    After the abort, an error that is not a FaberError or TransactionError
    is raised again, so that a programming error is not mistaken for a
    device fault.

    ``publish(result)`` runs only after the group committed (for example
    the session's token commit). A rank that fails, or a collective that
    fails (a rank that died or never joined, ending in the group's
    timeout), makes every rank abort; nothing is published on any rank.
    The device state is not rolled back: on a rank whose step ran, the
    session has already written that position's K/V rows and advanced its
    length, so after an abort the caller resets the session and replays its
    committed tokens before the next step. Given the rank's ``session`` (a
    ForwardRun of the group's model), an abort instead truncates it back to
    the length it had before the step and realigns the group's exchange
    epochs (``realign_after_abort``), so the step can simply be retried."""
    import torch
    import torch.distributed as dist
    reason, result, foreign = "", None, None
    length = len(session) if session is not None else 0
    try:
        t.execute(backend)
        if step is not None:
            result = step()
        ok = 1
    except TransactionError as e:
        ok, reason = 0, f"{e.kind} on partition {e.partition}"
    except _lib.FaberError as e:
        ok, reason = 0, f"step failed: {_lib.STATUS_NAMES.get(e.code, e.code)}"
    except Exception as e:  # noqa: BLE001 - the vote must happen whatever failed
        ok, reason, foreign = 0, f"step raised {type(e).__name__}: {e}", e
    flag = torch.tensor([ok], dtype=torch.int32)
    try:
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    except Exception as e:  # the group itself failed
        flag[0] = 0
        reason = reason or f"group decision failed: {type(e).__name__}"
    if int(flag.item()) == 1:
        receipt = t.commit(backend, ordinal)
        if publish is not None:
            publish(result)
        return receipt
    receipt = t.abort(backend, reason or "another rank failed")
    if session is not None:
        try:
            realign_after_abort(session, length, group)
        except Exception:  # noqa: BLE001 - a group that failed cannot realign
            if len(session) > length:
                session.truncate(length)
    if foreign is not None:
        raise foreign
    return receipt
