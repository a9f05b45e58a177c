"""Execution transactions and host-side fault injection (no GPU), on the
two-partition fixture of the reference's own transaction and fault tests
(src/execution_transaction_test.rs, src/fault_test.rs): a launch on
partition 0, a host-staged transfer 0 -> 1, a broadcast from 0 to both, a
barrier over both and a launch on partition 1, committed at the barrier and
the last launch. The admitted ledgers are the fixture's: 10 240 B of
staging on each partition, 8 448 B and 30 976 B of class-3 bytes, which the
fixture's reservation fills exactly.
"""

import pytest

from faber_runtime_b200 import _lib
from faber_runtime_b200 import transaction as tx

LAUNCH_A, T1, C1, BARRIER_MAIN, LAUNCH_B, T_EXTRA = 1, 2, 3, 4, 5, 6
LAUNCH_A_OUTPUT, TRANSFER_BYTES, BROADCAST_BYTES, LAUNCH_B_OUTPUT = 4096, 8192, 2048, 16_384
EVENT, SCRATCH = 64, 4096


def ledgers(p1_class3=30_976):
    return {0: tx.admitted(10_240, 8_448), 1: tx.admitted(10_240, p1_class3)}


def fixture_ops():
    return [tx.launch(0, LAUNCH_A, LAUNCH_A_OUTPUT),
            tx.transfer(T1, 0, 1, TRANSFER_BYTES),
            tx.broadcast(C1, 0, [0, 1], BROADCAST_BYTES),
            tx.barrier(BARRIER_MAIN, [0, 1]),
            tx.launch(1, LAUNCH_B, LAUNCH_B_OUTPUT)]


def fixture(ops=None, parts=None, barriers=(BARRIER_MAIN,), launches=(LAUNCH_B,)):
    return tx.Transaction(ledgers() if parts is None else parts, fixture_ops() if ops is None else ops,
                          barriers, launches)


DECLARED = LAUNCH_A_OUTPUT + TRANSFER_BYTES + BROADCAST_BYTES + LAUNCH_B_OUTPUT


def refused(call, kind, code=_lib.INVALID_ARGUMENT):
    with pytest.raises(tx.TransactionError) as e:
        call()
    assert e.value.kind == kind and e.value.code == code, (e.value.kind, e.value.code)
    return e.value


# --- construction and prepare ------------------------------------------------------

def test_construct_rejects_degenerate_plan_and_empty_snapshot():
    refused(lambda: tx.Transaction({0: tx.admitted(1 << 20, 1 << 20)}, fixture_ops()[:1]), "DegeneratePlan")
    refused(lambda: tx.Transaction(ledgers(), []), "EmptySnapshot")


def test_prepare_reserves_within_admitted_budget():
    t, b = fixture(), tx.FaultBackend()
    t.prepare(b)
    assert t.state == "Prepared"
    p0, p1 = t.reservation(0), t.reservation(1)
    assert p0["class_six"] == TRANSFER_BYTES + BROADCAST_BYTES
    assert p0["output"] == LAUNCH_A_OUTPUT
    assert p0["class_three"] == LAUNCH_A_OUTPUT + 4 * EVENT + SCRATCH
    assert p1["class_six"] == TRANSFER_BYTES + BROADCAST_BYTES
    assert p1["output"] == LAUNCH_B_OUTPUT + TRANSFER_BYTES + BROADCAST_BYTES
    assert p1["class_three"] == LAUNCH_B_OUTPUT + TRANSFER_BYTES + BROADCAST_BYTES + 4 * EVENT + SCRATCH
    assert b.info()["reserved_partitions"] == {0, 1}
    assert t.receipt().declared_write_bytes == DECLARED


def test_reservation_over_an_admitted_class_fails_at_prepare():
    ops = fixture_ops()
    ops[1] = tx.transfer(T1, 0, 1, 1 << 20)
    b = tx.FaultBackend()
    e = refused(lambda: fixture(ops).prepare(b), "ReservationExceedsBudget", _lib.BUDGET_EXCEEDED)
    assert e.budget_class == 6 and e.partition == 0
    ops = fixture_ops()
    ops[4] = tx.launch(1, LAUNCH_B, 1 << 20)
    e = refused(lambda: fixture(ops).prepare(b), "ReservationExceedsBudget", _lib.BUDGET_EXCEEDED)
    assert e.budget_class == 3 and e.partition == 1
    # a tampered but consistent plan: one more transfer over-commits staging
    e = refused(lambda: fixture(fixture_ops() + [tx.transfer(T_EXTRA, 0, 1, 65_536)]).prepare(b),
                "ReservationExceedsBudget", _lib.BUDGET_EXCEEDED)
    assert e.budget_class == 6 and e.partition == 0
    assert b.info()["reserved_partitions"] == set()  # a refused prepare reserves nothing


def test_prepare_checks_in_order():
    b = tx.FaultBackend()
    ops = fixture_ops()
    ops[4] = tx.launch(63, LAUNCH_B, 0)
    assert refused(lambda: fixture(ops).prepare(b), "UnknownPartition").partition == 63
    refused(lambda: fixture(fixture_ops() + [tx.launch(1, LAUNCH_A, 0)]).prepare(b), "DuplicateOperation")
    refused(lambda: fixture(barriers=(99,)).prepare(b), "UndeclaredBoundaryBarrier")
    refused(lambda: fixture(launches=(99,)).prepare(b), "UndeclaredBoundaryLaunch")
    parts = ledgers()
    parts[1] = None
    assert refused(lambda: fixture(parts=parts).prepare(b), "MissingAdmittedBudget").partition == 1
    # topology comes first: an unknown partition is reported even with a bad boundary
    refused(lambda: fixture(ops, barriers=(99,)).prepare(b), "UnknownPartition")
    t = fixture()
    t.prepare(b)
    refused(lambda: t.prepare(b), "InvalidState")


# --- execute and commit -------------------------------------------------------------

def test_execute_runs_in_plan_order_and_commit_publishes_atomically():
    t, b = fixture(), tx.FaultBackend()
    refused(lambda: t.commit(b, 1), "InvalidState")  # before execute
    t.prepare(b)
    t.execute(b)
    assert t.state == "Executing"
    info = b.info()
    assert info["executed_operations"] == 5 and info["staged_bytes"] == DECLARED
    assert info["published_bytes"] == 0
    r = t.commit(b, 7)
    assert r.decision == "Committed" and r.state == "Committed" and r.published
    assert r.publication_ordinal == 7
    assert r.published_bytes == DECLARED and r.staged_bytes == DECLARED
    assert r.executed_operations == 5 and r.executed_bytes == TRANSFER_BYTES + BROADCAST_BYTES
    assert r.completed_events == 1 + 2 + 2 + 2 + 1
    assert r.released_partitions == {0, 1} and not r.retired_partitions and not r.partial_publication
    assert b.info()["reserved_partitions"] == set()
    assert b.info()["committed_bytes"] == DECLARED
    refused(lambda: t.commit(b, 8), "InvalidState")  # commit twice
    refused(lambda: t.abort(b, "late"), "AlreadyCommitted")


def test_commit_waits_for_the_declared_boundary():
    t, b = fixture(), tx.FaultBackend()
    b.set_auto_complete(False)
    t.prepare(b)
    t.execute(b)
    e = refused(lambda: t.commit(b, 1), "BoundaryNotReached", _lib.FALLIBLE)
    assert e.missing == 2 and t.state == "Executing" and b.info()["published_bytes"] == 0
    barrier = tx.barrier(BARRIER_MAIN, [0, 1])
    b.complete_event(barrier, 0)
    assert refused(lambda: t.commit(b, 1), "BoundaryNotReached", _lib.FALLIBLE).missing == 2
    b.complete_event(barrier, 1)  # every participant of the barrier
    assert refused(lambda: t.commit(b, 1), "BoundaryNotReached", _lib.FALLIBLE).missing == 1
    b.complete_event(tx.launch(1, LAUNCH_B, LAUNCH_B_OUTPUT), 1)
    r = t.commit(b, 2)
    assert r.decision == "Committed" and r.published_bytes == DECLARED


def test_operation_outside_the_snapshot_never_runs():
    t, b = fixture(), tx.FaultBackend()
    t.prepare(b)
    refused(lambda: t.execute_operation(b, fixture_ops()[0]), "InvalidState")  # not executing yet
    t.execute(b)
    refused(lambda: t.execute_operation(b, tx.launch(0, 77, 1)), "OperationOutsideSnapshot")
    # same identity, other declared facts
    refused(lambda: t.execute_operation(b, tx.launch(0, LAUNCH_A, LAUNCH_A_OUTPUT + 1)),
            "OperationOutsideSnapshot")
    assert b.info()["executed_operations"] == 5


# --- abort -------------------------------------------------------------------------

def test_abort_releases_and_is_idempotent():
    t, b = fixture(), tx.FaultBackend()
    r = t.abort(b, "before prepare")
    assert r.decision == "Aborted" and r.failure_kind == "Cancelled"
    assert not r.released_partitions and not r.retired_partitions
    assert t.abort(b, "again") == r
    t = fixture()
    t.prepare(b)
    r = t.abort(b, "after prepare")
    assert r.released_partitions == {0, 1} and not r.retired_partitions
    assert b.info()["reserved_partitions"] == set()


def test_cancel_before_commit_retires_all_staged_state():
    t, b = fixture(), tx.FaultBackend()
    t.prepare(b)
    t.execute(b)
    r = t.abort(b, "cancelled by the coordinator")
    assert r.failure_kind == "Cancelled" and r.retired_partitions == {0, 1}
    info = b.info()
    assert info["staged_bytes"] == 0 and info["published_bytes"] == 0 and info["reserved_partitions"] == set()
    assert not r.published


# --- fault injection ---------------------------------------------------------------

FAULT_CODES = {tx.CANCEL: (_lib.CANCELLED, "Cancelled"), tx.TIMEOUT: (_lib.TIMEOUT, "Timeout"),
               tx.TRANSFER_ERROR: (_lib.KERNEL_ERROR, "Operation"),
               tx.KERNEL_ERROR: (_lib.KERNEL_ERROR, "Operation"),
               tx.DEVICE_LOSS: (_lib.DEVICE_LOSS, "DeviceLoss")}


@pytest.mark.parametrize("fault_class", sorted(FAULT_CODES))
def test_every_fault_class_fails_closed_without_partial_commit(fault_class):
    t, b = fixture(), tx.FaultBackend()
    ops = fixture_ops()
    # cancel on the last launch (partition 1), the others on the transfer
    target = ops[4] if fault_class == tx.CANCEL else ops[1]
    b.inject(target, 1, fault_class)
    t.prepare(b)
    code, cls = FAULT_CODES[fault_class]
    e = refused(lambda: t.execute(b), "Backend", code)
    assert e.backend_class == cls and e.partition == 1
    assert t.state == "Failed"
    refused(lambda: t.commit(b, 1), "InvalidState")
    assert b.info()["published_bytes"] == 0
    r = t.abort(b, "injected fault")
    assert r.state == "Aborted" and r.decision == "Aborted"
    assert r.failure_kind == "Backend" and r.failure_class == cls and r.failure_partition == 1
    info = b.info()
    assert info["reserved_partitions"] == set() and info["staged_bytes"] == 0
    assert info["published_bytes"] == 0 and not r.published and not r.partial_publication
    # partitions holding staged writes are retired, the others released
    assert r.retired_partitions | r.released_partitions == {0, 1}
    assert not (r.retired_partitions & r.released_partitions)
    assert 0 in r.retired_partitions  # launch A staged on partition 0 before the fault
    refused(lambda: t.execute(b), "InvalidState")  # no retry


def test_faults_are_per_partition_and_one_shot():
    ops = fixture_ops()
    b = tx.FaultBackend()
    b.inject(ops[0], 1, tx.KERNEL_ERROR)  # launch A involves only partition 0: never fires
    t = fixture()
    t.prepare(b)
    t.execute(b)
    assert b.info()["delivered_faults"] == 0
    t.commit(b, 1)
    b.inject(ops[1], 0, tx.TIMEOUT)  # the transfer involves partition 0 as its source
    t = fixture()
    t.prepare(b)
    refused(lambda: t.execute(b), "Backend", _lib.TIMEOUT)
    info = b.info()
    assert info["delivered_faults"] == 1 and info["reclaimed_copy_bytes"] == TRANSFER_BYTES
    t.abort(b, "timeout")
    t = fixture()  # delivered faults do not fire again
    t.prepare(b)
    t.execute(b)
    assert t.commit(b, 2).decision == "Committed"


def test_last_committed_state_remains_authoritative_after_failure():
    b = tx.FaultBackend()
    t = fixture()
    t.prepare(b)
    t.execute(b)
    t.commit(b, 1)
    assert b.info()["committed_bytes"] == DECLARED
    ops = fixture_ops()
    ops[4] = tx.launch(1, LAUNCH_B, 8192)  # a smaller second write-set
    b.inject(ops[3], 1, tx.DEVICE_LOSS)
    t2 = fixture(ops)
    t2.prepare(b)
    refused(lambda: t2.execute(b), "Backend", _lib.DEVICE_LOSS)
    t2.abort(b, "device loss")
    assert b.info()["committed_bytes"] == DECLARED  # the failed transaction changed nothing


def test_publish_failure_publishes_nothing():
    t, b = fixture(), tx.FaultBackend()
    b.fail_publish(2)
    t.prepare(b)
    t.execute(b)
    e = refused(lambda: t.commit(b, 1), "PublishFailed", _lib.KERNEL_ERROR)
    assert e.backend_class == "Operation"
    assert t.state == "Failed" and b.info()["published_bytes"] == 0
    r = t.abort(b, "publication failed")
    assert r.failure_kind == "PublishFailed" and not r.published
    assert b.info()["reserved_partitions"] == set() and b.info()["staged_bytes"] == 0


def test_degraded_mesh_fails_closed_at_the_boundary():
    """One partition's backend fails mid-execution: commit is refused, nothing
    publishes, abort tears down, and the receipt names the failed partition."""
    t, b = fixture(), tx.FaultBackend()
    b.inject(fixture_ops()[3], 1, tx.DEVICE_LOSS)  # the barrier, on partition 1
    t.prepare(b)
    refused(lambda: t.execute(b), "Backend", _lib.DEVICE_LOSS)
    assert b.info()["executed_operations"] == 3  # launch A, transfer, broadcast
    refused(lambda: t.commit(b, 1), "InvalidState")
    r = t.abort(b, "degraded")
    assert r.failure_class == "DeviceLoss" and r.failure_partition == 1
    assert r.retired_partitions == {0, 1} and r.published_bytes == 0


# --- the tensor-parallel decode step as a transaction ---------------------------------

def _group_ledgers(cfg, tp, ctx):
    from faber_runtime_b200 import partition as pt
    return {r: pt.plan(cfg, ctx, tp_size=tp, tp_rank=r) for r in range(tp)}


@pytest.mark.parametrize("which,tp", [("7b", 2), ("7b", 8), ("70b", 4), ("70b", 8)])
def test_tp_step_commits_within_each_rank_admitted_ledger(which, tp):
    from faber_runtime_b200 import LLAMA2_7B, LLAMA3_70B
    cfg = LLAMA2_7B if which == "7b" else LLAMA3_70B
    ops, barriers, launches = tx.tp_step_plan(cfg, tp, 4096)
    assert len(ops) == tp + 1 and len(launches) == tp and len(barriers) == 1
    kv_rows = cfg.n_layers * (cfg.n_kv_heads // tp) * cfg.head_dim * 2 * 2
    assert [o.bytes for o in ops[:tp]] == [kv_rows + 8] * tp
    assert ops[tp].kind == tx.BARRIER and ops[tp].participants == (1 << tp) - 1
    t, b = tx.Transaction(_group_ledgers(cfg, tp, 4096 + 128), ops, barriers, launches), tx.FaultBackend()
    t.prepare(b)
    for r in range(tp):
        res = t.reservation(r)
        assert res["class_six"] == 0  # the exchange buffer is the session's, admitted with it
        assert res["class_three"] == kv_rows + 8 + 2 * EVENT + SCRATCH
    t.execute(b)
    r = t.commit(b, 4096)
    assert r.published_bytes == tp * (kv_rows + 8) and r.executed_operations == tp + 1
    assert r.released_partitions == set(range(tp))


def test_tp_step_fails_closed_when_a_rank_is_lost():
    from faber_runtime_b200 import LLAMA3_70B
    tp = 8
    ops, barriers, launches = tx.tp_step_plan(LLAMA3_70B, tp, 100)
    ledgers8 = _group_ledgers(LLAMA3_70B, tp, 4096)
    # rank 5's step reports a lost device: no rank publishes the position
    t, b = tx.Transaction(ledgers8, ops, barriers, launches), tx.FaultBackend()
    b.inject(ops[5], 5, tx.DEVICE_LOSS)
    t.prepare(b)
    e = refused(lambda: t.execute(b), "Backend", _lib.DEVICE_LOSS)
    assert e.partition == 5
    r = t.abort(b, "rank 5 lost")
    assert r.retired_partitions == set(range(5))  # ranks 0-4 had staged their rows
    assert r.released_partitions == {5, 6, 7} and r.published_bytes == 0
    # rank 6's exchange times out (a peer's partials never arrived)
    t, b = tx.Transaction(ledgers8, ops, barriers, launches), tx.FaultBackend()
    b.inject(ops[tp], 6, tx.TIMEOUT)
    t.prepare(b)
    e = refused(lambda: t.execute(b), "Backend", _lib.TIMEOUT)
    assert e.partition == 6
    r = t.abort(b, "exchange timed out")
    assert r.retired_partitions == set(range(tp)) and r.published_bytes == 0
    assert b.info()["committed_bytes"] == 0


def test_tp_step_plan_needs_a_group():
    from faber_runtime_b200 import LLAMA2_7B, FaberError
    with pytest.raises(FaberError):
        tx.tp_step_plan(LLAMA2_7B, 1, 0)
    with pytest.raises(FaberError):
        tx.tp_step_plan(LLAMA2_7B, 3, 0)  # 32 heads do not divide over 3 ranks
