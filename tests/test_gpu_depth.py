"""Greedy decode at the benchmarked depth and context, against the CPU oracle.

* The Llama-2-7B shape at all 32 layers, with the weights of the decode
  benchmark (the same seed), over a 2048-position K/V prefix installed in
  every layer: 8 greedy tokens token-identical to the oracle's run_greedy
  loop (src/greedy_run.rs:186-248 over ForwardRun::push_token,
  src/cpu_oracle.rs:859-912), and the logits of every step within
  1e-3 x RMS on a teacher-forced second session.
* The Llama-3-70B shape (GQA 64/8, FFN 28672, vocab 128256) at full width
  and 8 layers, over a 4096-position prefix, batch 1: the same two checks.

The oracle cannot run a 2048-token prompt pass through 32 layers of the 7B
shape in test time (hours on a CPU), so both sides get the same seeded K/V
prefix through set_prefix, as the benchmark's CPU sample does; the decode
steps after it run the full model on both sides. The GPU tokens come from
the graph-replayed greedy loop that the benchmark times.
"""

import numpy as np
import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

RMS_TOL = 1e-3
BENCH_SEED = 20261201  # the decode benchmark's weights


def within(gpu, ref, tol=RMS_TOL):
    gpu = np.asarray(gpu, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(ref ** 2))
    err = np.max(np.abs(gpu - ref))
    assert np.all(np.isfinite(gpu))
    assert err <= tol * rms, f"max|err| {err:.3e} > {tol} x RMS {rms:.3e}"
    return err / rms


def _depth_case(cfg, seed, n_prefix, kv_std, norms, n_gen, first_token):
    import oracle as o
    from faber_runtime_b200 import DeviceModel, ForwardRun, synth
    tensors = {n: (t, a, r, c) for n, t, a, r, c in synth.model_tensors(cfg, seed, norms=norms)}
    om = o.OracleModel(cfg, tensors)
    dm = DeviceModel(cfg, ((n, t, a, r, c) for n, (t, a, r, c) in tensors.items()))
    ctx = n_prefix + n_gen + 8
    orun = o.OracleRun(om, ctx)
    greedy_run = ForwardRun(dm, context_length=ctx)
    forced_run = ForwardRun(dm, context_length=ctx)
    span = cfg.n_kv_heads * cfg.head_dim
    for layer in range(cfg.n_layers):
        k = synth.normal(seed, 5000 + layer, n_prefix * span, 0.0, kv_std)
        v = synth.normal(seed, 6000 + layer, n_prefix * span, 0.0, kv_std)
        orun.set_prefix(layer, k, v, n_prefix)
        greedy_run.set_prefix(layer, k, v, n_prefix)
        forced_run.set_prefix(layer, k, v, n_prefix)
    del tensors
    # oracle: run_greedy's loop over push_token / position_logits / top1_non_eog
    orun.push_token(first_token)
    ref_tokens, ref_logits = [], []
    for i in range(n_gen):
        lg = orun.position_logits()
        ref_logits.append(lg)
        ref_tokens.append(o.top1_non_eog(lg))
        if i + 1 < n_gen:
            orun.push_token(ref_tokens[-1])
    # device: the benchmark's graph-replayed greedy loop
    greedy_run.push_token(first_token)
    toks, finite = greedy_run.greedy(n_gen)
    assert finite
    assert toks.tolist() == ref_tokens, (toks.tolist(), ref_tokens)
    assert len(greedy_run) == n_prefix + n_gen
    # device, teacher-forced: the logits of every step
    forced_run.push_token(first_token)
    worst = 0.0
    for i in range(n_gen):
        lg = forced_run.position_logits()
        worst = max(worst, within(lg, ref_logits[i]))
        assert o.top1_non_eog(lg) == ref_tokens[i]
        forced_run.push_token(ref_tokens[i])
    greedy_run.close()
    forced_run.close()
    dm.close()
    return worst


def test_7b_full_depth_over_2048_prefix(cuda):
    from faber_runtime_b200 import LLAMA2_7B
    assert LLAMA2_7B.n_layers == 32
    worst = _depth_case(LLAMA2_7B, BENCH_SEED, n_prefix=2048, kv_std=50.0, norms="ones", n_gen=8,
                        first_token=1)
    assert worst < RMS_TOL


def test_70b_width_eight_layers_over_4096_prefix(cuda):
    from faber_runtime_b200 import LLAMA3_70B
    cfg = LLAMA3_70B.with_layers(8)
    worst = _depth_case(cfg, 70, n_prefix=4096, kv_std=4.0, norms="random", n_gen=8,
                        first_token=128000 % 32000)
    assert worst < RMS_TOL
