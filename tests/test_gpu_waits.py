"""Bounded device waits that run out, and the session rollback after a failed
step (BackendError::Timeout, src/execution_transaction/backend.rs:17-54;
no token commit after an abort, src/session.rs:422-456).

No GPU is faulted, trapped or hung here. A wait runs out because a word it
polls never carries the expected epoch: the kernel gives up after a short
poll limit, records the expiry, and returns; the host reports TIMEOUT.

* The exchange-consuming GEMV of a tensor-parallel step (the product
  kernel, on local buffers): with every word present it matches the oracle;
  with one stale word it returns TIMEOUT quickly, and the device keeps
  working (the same call, then a session's decode, match the oracle).
* Truncation: a session shortened by one position and pushed the same
  token again continues exactly like an uninterrupted one.
* Two GPUs (skipped with fewer): rank 1 skips a step while rank 0 runs it
  with a short wait limit; rank 0's push fails with TIMEOUT and is rolled
  back, the ranks raise their exchange epochs to the group's largest, and
  the retried step and the following greedy tokens equal the oracle's. The
  waiting rank spins only on its own exchange buffer (peer stores, no
  multicast), and rank 1 has nothing in flight while it waits.
"""

import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RMS_TOL = 1e-3


def within(gpu, ref, tol=RMS_TOL):
    gpu = np.asarray(gpu, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(ref ** 2))
    err = np.max(np.abs(gpu - ref))
    assert np.all(np.isfinite(gpu))
    assert err <= tol * rms, f"max|err| {err:.3e} > {tol} x RMS {rms:.3e}"


def _words(parts: np.ndarray, epoch: int) -> np.ndarray:
    bits = parts.astype(np.float32).view(np.uint32).astype(np.uint64)
    return (np.uint64(epoch) << np.uint64(32)) | bits


def _exchange_case(cuda, rows=2048, cols=4096, tp=3, seed=9):
    import torch
    import oracle as o
    from faber_runtime_b200 import dequant, synth
    blocks = synth.q4k_blocks(seed, 1, rows * cols // 256)
    w = dequant.Q4kTensor(blocks, rows, cols)
    x = synth.normal(seed, 2, cols)
    parts = synth.normal(seed, 3, tp * cols).reshape(tp, cols)
    norm_w = synth.normal(seed, 4, cols, 1.0, 0.1)
    eps = 1e-5
    # the kernel's sum: x + ((p0 + p1) + p2), in f32
    s = parts[0].copy()
    for r in range(1, tp):
        s = (s + parts[r]).astype(np.float32)
    x_sum = (x + s).astype(np.float32)
    want = o.dense_q(o.Q4_K, blocks, o.rms_norm(x_sum, norm_w, eps), cols, rows)
    dev = {k: torch.from_numpy(np.ascontiguousarray(v)).to(cuda) for k, v in
           (("x", x), ("norm_w", norm_w))}
    dev["x_sum"] = torch.empty(cols, dtype=torch.float32, device=cuda)
    dev["y"] = torch.empty(rows, dtype=torch.float32, device=cuda)

    def call(words: np.ndarray, epoch: int, limit: int):
        ex = torch.from_numpy(words.view(np.int64)).to(cuda)
        dev["x_sum"].fill_(float("nan"))
        dev["y"].fill_(float("nan"))
        w.gemv_exchange(dev["x"].data_ptr(), dev["norm_w"].data_ptr(), eps, ex.data_ptr(), tp, epoch, limit,
                        dev["x_sum"].data_ptr(), dev["y"].data_ptr(),
                        torch.cuda.current_stream().cuda_stream)
        return dev["x_sum"].cpu().numpy(), dev["y"].cpu().numpy()

    return w, parts, x_sum, want, call


@pytest.mark.parametrize("tp", [2, 3, 8])  # every CTA sums all (<= 4) / slices + grid barrier (8)
def test_exchange_gemv_matches_the_oracle_when_every_word_arrived(cuda, tp):
    w, parts, x_sum, want, call = _exchange_case(cuda, tp=tp)
    got_sum, y = call(_words(parts, 7), 7, 0)
    assert np.array_equal(got_sum.view(np.uint32), x_sum.view(np.uint32))
    within(y, want)
    w.close()


def test_a_word_that_never_arrives_times_out_and_the_device_keeps_working(cuda):
    from faber_runtime_b200 import FaberError, _lib
    w, parts, x_sum, want, call = _exchange_case(cuda)
    words = _words(parts, 7)
    words[2, 1234] = _words(parts[2:3, 1234:1235], 6)[0, 0]  # one stale word of rank 2
    t0 = time.monotonic()
    with pytest.raises(FaberError) as e:
        call(words, 7, 4096)
    assert e.value.code == _lib.TIMEOUT, str(e.value)
    assert time.monotonic() - t0 < 10.0
    # the same call with every word present still matches
    got_sum, y = call(_words(parts, 8), 8, 4096)
    assert np.array_equal(got_sum.view(np.uint32), x_sum.view(np.uint32))
    within(y, want)
    w.close()
    # and a session on this device decodes like the oracle
    import oracle as o
    from faber_runtime_b200 import TINY, DeviceModel, synth
    from faber_runtime_b200.decoder import run_greedy
    tensors = list(synth.model_tensors(TINY, 5))
    om = o.OracleModel(TINY, {n: (t, a, r, c) for n, t, a, r, c in tensors})
    dm = DeviceModel(TINY, tensors)
    prompt = synth.tokens(5, 1, 10, TINY.vocab)
    ref, _, _ = om.greedy(prompt, 8)
    rec = run_greedy(dm, prompt, ref.tolist())
    assert rec.divergence_field() == "none"
    dm.close()


def test_truncate_then_push_continues_like_an_uninterrupted_session(cuda):
    from faber_runtime_b200 import TINY, DeviceModel, FaberError, ForwardRun, synth
    dm = DeviceModel(TINY, synth.model_tensors(TINY, 6))
    prompt = synth.tokens(6, 1, 12, TINY.vocab)
    ref = ForwardRun(dm, prompt, context_length=64)
    want, _ = ref.greedy(10)
    ref_logits = ref.position_logits()
    run = ForwardRun(dm, prompt, context_length=64)
    first, _ = run.greedy(4)  # positions 12..14 pushed, logits of 15 taken
    n = len(run)
    assert n == 12 + 3
    e0 = run.exchange_epoch()
    run.truncate(n - 1)
    assert len(run) == n - 1
    with pytest.raises(FaberError) as e:
        run.position_logits()  # the residual of the last position is gone
    assert e.value.code == 1
    with pytest.raises(FaberError):
        run.truncate(n)  # never lengthens
    run.push_token(int(first[2]))  # the token of the truncated position again
    rest, _ = run.greedy(7)
    assert first.tolist()[:4] + rest.tolist()[1:] == want.tolist()
    assert np.array_equal(run.position_logits(), ref_logits)
    # the exchange epoch counts launched steps and is never lowered
    e1 = run.exchange_epoch()
    assert e1 > e0
    assert run.exchange_epoch(e1 + 10) == e1 + 10
    assert run.exchange_epoch(3) == e1 + 10
    run.close()
    ref.close()
    dm.close()


WORLD = 2


def _tp_cfg():
    from faber_runtime_b200 import ModelConfig
    return ModelConfig(n_layers=2, d_model=1024, n_heads=16, n_kv_heads=4, head_dim=64, ffn=2816,
                       vocab=4096, tied_head=False, rope_theta=500000.0, name="tp-wait")


def _tp_worker(rank, uid, port, result_q):
    import os
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist
    from faber_runtime_b200 import DeviceModel, FaberError, ForwardRun, _lib, synth
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60))
    try:
        cfg = _tp_cfg()
        _lib.call("faber_gpu_v2_init", rank)
        model = DeviceModel(cfg, synth.model_tensors(cfg, 43, norms="random"), device=rank, tp_size=WORLD,
                            tp_rank=rank, nccl_uid=uid)
        prompt = synth.tokens(43, 3, 20, cfg.vocab)
        run = ForwardRun(model, prompt, context_length=64)
        first, _ = run.greedy(3)
        n0 = len(run)
        out = {"rank": rank, "first": first.tolist()}
        dist.barrier()
        if rank == 0:  # rank 1 skips this step: rank 0's exchange wait runs out
            run.set_wait_limit(4096)
            t0 = time.monotonic()
            try:
                run.push_token(int(first[-1]))
                out["timeout"] = "no error"
            except FaberError as e:
                out["timeout"] = e.code
            out["timeout_s"] = time.monotonic() - t0
            out["len_after_timeout"] = len(run)
            run.set_wait_limit(0)
        dist.barrier()  # nothing of either rank is in flight past this point
        e = torch.tensor([run.exchange_epoch()], dtype=torch.int64)
        dist.all_reduce(e, op=dist.ReduceOp.MAX)
        run.exchange_epoch(int(e.item()))
        run.push_token(int(first[-1]))  # the retried step, on both ranks
        assert len(run) == n0 + 1
        rest, fin = run.greedy(6)
        out["rest"] = rest.tolist()
        out["finite"] = bool(fin)
        run.close()
        model.close()
        result_q.put(out)
    except Exception as e:
        result_q.put({"rank": rank, "error": repr(e)})
        raise
    finally:
        dist.destroy_process_group()


def test_tp2_step_timeout_rolls_back_and_the_retry_matches_the_oracle(cuda):
    import ctypes
    import socket
    import torch
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    import oracle as o
    from faber_runtime_b200 import _lib, synth
    uid = (ctypes.c_uint8 * 128)()
    _lib.call("faber_gpu_v2_nccl_unique_id", ctypes.addressof(uid))
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    q = mp.get_context("spawn").SimpleQueue()
    mp.start_processes(_tp_worker, args=(bytes(uid), port, q), nprocs=WORLD, join=True, start_method="spawn")
    res = sorted((q.get() for _ in range(WORLD)), key=lambda r: r["rank"])
    for r in res:
        assert "error" not in r, r
    assert res[0]["timeout"] == _lib.TIMEOUT, res[0]
    assert res[0]["timeout_s"] < 10.0
    assert res[0]["len_after_timeout"] == 20 + 2  # the failed position is not kept
    cfg = _tp_cfg()
    om = o.OracleModel(cfg, {n: (t, a, r, c) for n, t, a, r, c in synth.model_tensors(cfg, 43, norms="random")})
    ref, _, _ = om.greedy(synth.tokens(43, 3, 20, cfg.vocab), 9)
    for r in res:
        assert r["finite"]
        assert r["first"] + r["rest"] == ref.tolist(), r
