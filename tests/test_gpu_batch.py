"""Batched greedy decode (faber_gpu_v2_batch_*) against the CPU oracle.

Several sessions of one model, each with its own prompt (short ones pushed
token by token, long ones through the tensor-core prompt pass), decode in
lockstep: every linear layer is one batched Q4_K GEMV over all sequences
(each exact weight fragment feeds 1, 2 or 4 MMA column blocks for up to 4, 8
or 16 sequences; the 2816-wide down projection at 16 sequences is cut into
two K slabs summed through the per-tile ticket).
With one query head per kv head the step's attention is the TMA-streamed
tensor-core kernel over each sequence's own tensor maps.
Each sequence's tokens must equal the oracle's run_greedy for its prompt
alone, and afterwards each session must hold its own state: its
position_logits equal the oracle's logits that chose its last token
(within 1e-3 x RMS), and it keeps decoding on its own.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N_GEN = 8


def within(gpu, ref, tol=1e-3):
    gpu = np.asarray(gpu, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(ref ** 2))
    err = np.max(np.abs(gpu - ref))
    assert np.all(np.isfinite(gpu))
    assert err <= tol * rms, f"max|err| {err:.3e} > {tol} x RMS {rms:.3e}"


def _cfg(kv_heads=4, head_dim=64, heads=16):
    from faber_runtime_b200 import ModelConfig
    return ModelConfig(n_layers=2, d_model=1024, n_heads=heads, n_kv_heads=kv_heads, head_dim=head_dim,
                       ffn=2816, vocab=4096, tied_head=False, rope_theta=500000.0, name="batch-test")


@pytest.fixture(scope="module")
def pair(cuda):
    import oracle as o
    from faber_runtime_b200 import DeviceModel, synth
    cfg = _cfg()
    tensors = list(synth.model_tensors(cfg, 61, norms="random"))
    om = o.OracleModel(cfg, {n: (t, a, r, c) for n, t, a, r, c in tensors})
    return cfg, om, DeviceModel(cfg, tensors)


@pytest.mark.parametrize("lengths", [
    [40, 7, 100, 33, 64],                # mixed: token-by-token and prompt-pass prompts
    [20, 45, 70],                        # one MMA column block
    [9 * i + 5 for i in range(8)],       # two full column blocks
    [33 + i for i in range(16)],         # a full batch of 16
])
def test_batch_greedy_matches_oracle(pair, lengths):
    from faber_runtime_b200 import BatchRun, ForwardRun, synth
    cfg, om, dm = pair
    prompts = [synth.tokens(61, 100 + i, n, cfg.vocab) for i, n in enumerate(lengths)]
    runs = [ForwardRun(dm, p, context_length=max(lengths) + N_GEN + 8) for p in prompts]
    batch = BatchRun(runs)
    toks, fin = batch.greedy(N_GEN)
    assert fin.all()
    for i, p in enumerate(prompts):
        ref_tokens, ref_logits, _ = om.greedy(p, N_GEN, want_logits=True)
        assert toks[i].tolist() == ref_tokens.tolist(), (i, toks[i].tolist(), ref_tokens.tolist())
        assert len(runs[i]) == len(p) + N_GEN - 1
        within(runs[i].position_logits(), ref_logits[N_GEN - 1])
    # a session continues on its own after the batch
    more, ok = runs[0].greedy(3)
    ref_more, _, _ = om.greedy(prompts[0], N_GEN + 2)
    assert ok and more.tolist() == ref_more[N_GEN - 1:].tolist()
    batch.close()
    for r in runs:
        r.close()


@pytest.fixture(scope="module")
def mha_pair(cuda):
    import oracle as o
    from faber_runtime_b200 import DeviceModel, synth
    cfg = _cfg(kv_heads=8, head_dim=128, heads=8)
    tensors = list(synth.model_tensors(cfg, 67, norms="random"))
    om = o.OracleModel(cfg, {n: (t, a, r, c) for n, t, a, r, c in tensors})
    return cfg, om, DeviceModel(cfg, tensors)


@pytest.mark.parametrize("lengths", [
    [40, 7, 100, 33, 64],
    [33 + 3 * i for i in range(16)],
])
def test_batch_mha_greedy_matches_oracle(mha_pair, lengths):
    """One query head per kv head: the batched step's attention runs on the
    TMA-streamed tensor-core kernel with every sequence's own K/V tensor
    maps (grid.z = sequence)."""
    from faber_runtime_b200 import BatchRun, ForwardRun, synth
    cfg, om, dm = mha_pair
    prompts = [synth.tokens(67, 200 + i, n, cfg.vocab) for i, n in enumerate(lengths)]
    runs = [ForwardRun(dm, p, context_length=max(lengths) + N_GEN + 8) for p in prompts]
    batch = BatchRun(runs)
    toks, fin = batch.greedy(N_GEN)
    assert fin.all()
    for i, p in enumerate(prompts):
        ref_tokens, ref_logits, _ = om.greedy(p, N_GEN, want_logits=True)
        assert toks[i].tolist() == ref_tokens.tolist(), (i, toks[i].tolist(), ref_tokens.tolist())
        within(runs[i].position_logits(), ref_logits[N_GEN - 1])
    batch.close()
    for r in runs:
        r.close()


def test_batch_rejects_mixed_sessions(pair):
    from faber_runtime_b200 import BatchRun, FaberError, ForwardRun, synth
    cfg, om, dm = pair
    a = ForwardRun(dm, synth.tokens(61, 1, 5, cfg.vocab), context_length=64)
    b = ForwardRun(dm, synth.tokens(61, 2, 5, cfg.vocab), context_length=128)
    with pytest.raises(FaberError) as e:
        BatchRun([a, b])
    assert e.value.code == 1 and "context length" in str(e.value)
    with pytest.raises(FaberError):
        BatchRun([a, a])
    with pytest.raises(FaberError):
        BatchRun([a] * 17)
    a.close()
    b.close()
