"""The group decision of a tensor-parallel step on 2 gloo ranks (CPU): each
rank runs the step's transaction, and the ranks agree before anything is
published. Failures are made on the host: a fault injected into one
rank's backend, and a rank that dies before the decision. No GPU is used.
"""

import multiprocessing as mp
import os
import socket
from datetime import timedelta

WORLD = 2


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from faber_runtime_b200 import LLAMA2_7B, partition
    from faber_runtime_b200 import transaction as tx
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=20))
    try:
        cfg = LLAMA2_7B.with_layers(2)
        ops, barriers, launches = tx.tp_step_plan(cfg, WORLD, 300)
        ledgers = {r: partition.plan(cfg, 512, tp_size=WORLD, tp_rank=r) for r in range(WORLD)}
        t, b = tx.Transaction(ledgers, ops, barriers, launches), tx.FaultBackend()
        t.prepare(b)
        if mode == "fault" and rank == 1:
            b.inject(ops[1], 1, tx.KERNEL_ERROR)  # this rank's own step fails
        if mode == "dies" and rank == 1:
            os._exit(3)  # gone before the decision, nothing in flight
        published = []

        class FakeSession:  # the length / truncate / epoch surface of a ForwardRun
            def __init__(self):
                self.n, self.epoch, self.calls = 40, 100 + rank, []

            def __len__(self):
                return self.n

            def truncate(self, n):
                self.calls.append(("truncate", n))
                self.n = n

            def exchange_epoch(self, raise_to=0):
                self.epoch = max(self.epoch, raise_to)
                return self.epoch

        sess = FakeSession() if mode == "session" else None

        def step():
            if sess is not None:  # rank 0's step ran (length advanced); rank 1's failed
                if rank == 1:
                    from faber_runtime_b200 import _lib
                    raise _lib.FaberError(_lib.TIMEOUT, "exchange wait expired")
                sess.n += 1
                sess.epoch += 1
                return 1000 + rank
            # this rank's device work; rank 1's exchange wait expires in "timeout"
            if mode == "timeout" and rank == 1:
                from faber_runtime_b200 import _lib
                raise _lib.FaberError(_lib.TIMEOUT, "a tensor-parallel peer did not publish its partials in time")
            if mode == "value_error" and rank == 1:
                raise ValueError("TokenOutOfRange: token 99999 is outside the admitted vocab")
            return 1000 + rank

        try:
            r = tx.run_group_step(t, b, ordinal=300, step=step, publish=published.append, session=sess)
        except ValueError as e:  # raised again after this rank aborted
            info = b.info()
            q.put((rank, "raised", str(e), info["committed_bytes"], t.receipt().decision, published))
            return
        if sess is not None:
            published = [len(sess), sess.epoch, sess.calls]
        q.put((rank, r.decision, r.published_bytes, b.info()["committed_bytes"], r.failure_kind, published))
    except Exception as e:  # reported, not hidden
        q.put((rank, "error", repr(e), 0, "", []))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank, args=(r, port, mode, q)) for r in range(WORLD)]
    for p in ps:
        p.start()
    expect = 1 if mode == "dies" else WORLD
    out = sorted(q.get(timeout=120) for _ in range(expect))
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_every_rank_commits_when_every_step_ran():
    out = _run("ok")
    assert [o[1] for o in out] == ["Committed"] * WORLD
    assert out[0][2] == out[1][2] > 0 and all(o[3] == o[2] for o in out)


def test_one_rank_failing_aborts_every_rank():
    out = _run("fault")
    assert [o[1] for o in out] == ["Aborted"] * WORLD, out
    assert all(o[2] == 0 and o[3] == 0 for o in out)  # nothing published anywhere
    assert out[1][4] == "Backend" and out[0][4] == "Cancelled"


def test_a_step_timeout_on_one_rank_aborts_every_rank():
    out = _run("timeout")
    assert [o[1] for o in out] == ["Aborted"] * WORLD, out
    assert all(o[2] == 0 and o[5] == [] for o in out)  # nothing published, no token committed
    assert out[1][4] == "Cancelled"  # the step failed outside the backend: aborted with its reason


def test_a_step_raising_a_foreign_error_still_votes_and_aborts_every_rank():
    """A step that raises something other than a FaberError (here the
    ValueError of a rejected token id) must not skip the group's vote: the
    other rank aborts at once (not after the group's timeout), the failing
    rank aborts too and then raises the error again."""
    import time
    t0 = time.monotonic()
    out = _run("value_error")
    assert time.monotonic() - t0 < 60  # well inside the 20 s group timeout plus start-up
    assert out[0][1] == "Aborted" and out[0][2] == 0 and out[0][5] == []
    assert out[1][1] == "raised" and "TokenOutOfRange" in out[1][2]
    assert out[1][3] == 0 and out[1][4] == "Aborted" and out[1][5] == []


def test_publish_runs_only_after_the_group_commits():
    out = _run("ok")
    assert [o[5] for o in out] == [[1000], [1001]]


def test_a_rank_that_dies_aborts_the_survivor():
    out = _run("dies")
    assert len(out) == 1 and out[0][0] == 0
    assert out[0][1] == "Aborted" and out[0][2] == 0, out


def test_an_abort_truncates_the_session_and_realigns_the_exchange_epochs():
    """With the rank's session given, an aborted step leaves every rank at
    the length it had before the step and at the group's largest exchange
    epoch, so the step can be retried."""
    out = _run("session")
    assert [o[1] for o in out] == ["Aborted"] * WORLD, out
    (n0, e0, c0), (n1, e1, c1) = out[0][5], out[1][5]
    assert n0 == n1 == 40
    assert e0 == e1 == 101  # rank 0 advanced 100 -> 101; rank 1 raised from 101
    assert c0 == [("truncate", 40)] and c1 == []
