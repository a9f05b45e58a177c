"""Tensor-parallel decode on 2 GPUs (NCCL all-reduce after O and down).

One process per GPU builds its shard of a small GQA model from the same
seeded tensors, and both run the same session calls. The greedy tokens must
equal the CPU oracle's, and the gathered logits must be within 1e-3 x RMS.
Skipped when fewer than 2 GPUs are visible.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WORLD = 2
N_GEN = 12


def _cfg():
    from faber_runtime_b200 import ModelConfig
    return ModelConfig(n_layers=2, d_model=1024, n_heads=16, n_kv_heads=4, head_dim=64, ffn=2816,
                       vocab=4096, tied_head=False, rope_theta=500000.0, name="tp-gpu")


def _worker(rank, uid, result_q):
    from faber_runtime_b200 import DeviceModel, ForwardRun, _lib, synth
    try:
        cfg = _cfg()
        _lib.call("faber_gpu_v2_init", rank)
        tensors = list(synth.model_tensors(cfg, 41, norms="random"))
        model = DeviceModel(cfg, tensors, device=rank, tp_size=WORLD, tp_rank=rank, nccl_uid=uid)
        prompt = synth.tokens(41, 3, 70, cfg.vocab)
        run = ForwardRun(model, prompt, context_length=128)
        toks, finite = run.greedy(N_GEN)
        logits = run.position_logits()
        run.close()  # graphs holding NCCL calls go before the communicator
        model.close()
        result_q.put((rank, toks.tolist(), bool(finite), logits))
    except Exception as e:
        result_q.put((rank, repr(e), False, None))
        raise


def test_tp2_greedy_matches_oracle(cuda):
    import torch
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    import ctypes

    import torch.multiprocessing as mp

    import oracle as o
    from faber_runtime_b200 import _lib, synth
    uid = (ctypes.c_uint8 * 128)()
    _lib.call("faber_gpu_v2_nccl_unique_id", ctypes.addressof(uid))
    q = mp.get_context("spawn").SimpleQueue()
    mp.start_processes(_worker, args=(bytes(uid), q), nprocs=WORLD, join=True,
                       start_method="spawn")
    res = sorted((q.get() for _ in range(WORLD)), key=lambda r: r[0])
    for rank, toks, finite, _ in res:
        assert isinstance(toks, list), f"rank {rank}: {toks}"
        assert finite
    cfg = _cfg()
    om = o.OracleModel(cfg, {n: (t, a, r, c) for n, t, a, r, c in synth.model_tensors(cfg, 41, norms="random")})
    prompt = synth.tokens(41, 3, 70, cfg.vocab)
    ref_toks, ref_logits, _ = om.greedy(prompt, N_GEN, want_logits=True)
    for rank, toks, _, logits in res:
        assert toks == ref_toks.tolist(), (rank, toks, ref_toks.tolist())
        # greedy(n) feeds back n - 1 tokens: the session ends at the logits
        # that chose the last token
        ref = np.asarray(ref_logits[N_GEN - 1], np.float64)
        err = np.max(np.abs(np.asarray(logits, np.float64) - ref))
        assert err <= 1e-3 * np.sqrt(np.mean(ref ** 2)), (rank, err)
