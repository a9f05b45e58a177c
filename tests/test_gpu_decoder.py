"""GPU decoder parity against the CPU oracle (through the C ABI).

* tiny (4 layers, d 512, 8 heads x 64, FFN 1408, vocab 32000, tied head): a
  32-token prompt then 64 greedy tokens, token-identical to run_greedy, and
  teacher-forced logits at every step within 1e-3 x RMS;
* layer-level intermediates of the first pushes (trace mode);
* the 7B shape (d 4096, 32 heads x 128, FFN 11008, vocab 32000) cut to two
  layers, over an installed 256-position K/V prefix (the oracle cannot
  prefill thousands of 7B positions in test time);
* the 70B shape's GQA (64/8 heads) cut to one layer and 1/8 width is covered
  by the gqa config below;
* fail-closed behaviour (empty prompt, out-of-range token, full context) and
  the token-commit contract of src/session.rs:422-456.
"""

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
    return err / rms


def build_pair(cfg, seed, norms="ones"):
    import oracle as o
    from faber_runtime_b200 import DeviceModel, synth
    tensors = list(synth.model_tensors(cfg, seed, norms=norms))
    om = o.OracleModel(cfg, {n: (t, a, r, c) for n, t, a, r, c in tensors})
    dm = DeviceModel(cfg, tensors)
    return om, dm, tensors


@pytest.fixture(scope="module")
def tiny(cuda):
    from faber_runtime_b200 import TINY
    return build_pair(TINY, 2024)


def test_tiny_greedy_token_identical_and_logits_close(tiny):
    import oracle as o
    from faber_runtime_b200 import TINY, ForwardRun, run_greedy, synth
    om, dm, _ = tiny
    prompt = synth.tokens(2024, 99, 32, TINY.vocab)
    ref_tokens, ref_logits, ref_finite = om.greedy(prompt, 64, eog=(), want_logits=True)
    rec = run_greedy(dm, prompt, ref_tokens.tolist())
    assert rec.all_finite and ref_finite
    assert rec.generated_tokens == ref_tokens.tolist(), rec.divergence_field()
    assert rec.divergence_field() == "none"
    # teacher-forced logits at every step
    run = ForwardRun(dm, prompt, context_length=128)
    worst = 0.0
    for i in range(64):
        worst = max(worst, within(run.position_logits(), ref_logits[i]))
        run.push_token(int(ref_tokens[i]))
    assert worst < 1e-4
    assert len(run) == 32 + 64


def test_step_greedy_follows_session_greedy(tiny):
    """A host-driven loop of step_greedy (push the id, read back the next)
    yields the same ids as session greedy, with and without EOG ids."""
    from faber_runtime_b200 import ForwardRun, synth
    _, dm, _ = tiny
    prompt = synth.tokens(2024, 9, 20, 32000)
    for eog in ((), (5, 17)):
        ref = ForwardRun(dm, prompt, context_length=64)
        want, _ = ref.greedy(12, eog=eog)
        ref.close()
        run = ForwardRun(dm, prompt, context_length=64)
        first, _ = run.greedy(1, eog=eog)
        got = [int(first[0])]
        for _ in range(11):
            got.append(run.step_greedy(got[-1], eog=eog))
        assert got == want.tolist()
        assert len(run) == 20 + 11
        run.close()


def test_tiny_forward_one_matches(tiny):
    import oracle as o
    from faber_runtime_b200 import synth
    om, dm, _ = tiny
    toks = synth.tokens(7, 7, 9, 32000)
    r = o.OracleRun(om, 16)
    for t in toks:
        r.push_token(int(t))
    within(dm.forward_one(toks), r.position_logits())


def test_tiny_layer_trace(tiny):
    import oracle as o
    from faber_runtime_b200 import ForwardRun, synth
    om, dm, _ = tiny
    toks = synth.tokens(3, 3, 5, 32000)
    orun = o.OracleRun(om, 16, trace=True)
    drun = ForwardRun(dm, context_length=16, trace=True)
    for i, t in enumerate(toks):
        orun.push_token(int(t))
        drun.push_token(int(t))
        if i == 0:
            # layer 0 normalizes the exact (f16-rounded) embedding: rms_norm is
            # reproduced to the bit (f64 sum, IEEE sqrt/div, two rounded muls)
            a, b = drun.trace(0, "attn_in"), orun.trace(0, "attn_in")
            ulp = np.abs(a.view(np.int32).astype(np.int64) - b.view(np.int32).astype(np.int64))
            assert ulp.max() <= 1
        # The first token attends to one key, so every op is a GEMV or an
        # element-wise step: 1e-3 x RMS holds everywhere. Later tokens mix
        # near-tied softmax scores, where ~1e-7 relative score differences
        # (summation order) move the context by up to ~1e-3 relative; the
        # intermediates are then held to 1e-2 and the logits to 1e-3.
        tol = 1e-3 if i == 0 else 1e-2
        for layer in range(om.cfg.n_layers):
            for which in ("attn_in", "q_rot", "k_rot", "v", "ctx", "h2", "hh", "h_out"):
                a, b = drun.trace(layer, which), orun.trace(layer, which)
                if which in ("k_rot", "v") or (which == "ctx" and i == 0):
                    # cached in f16 (and the first context is one cached V
                    # row): an input difference far below tolerance can still
                    # move the rounding by one f16 ulp
                    ulp16 = np.spacing(np.abs(b).astype(np.float16)).astype(np.float64)
                    rms = np.sqrt(np.mean(np.asarray(b, np.float64) ** 2))
                    err = np.abs(np.asarray(a, np.float64) - b)
                    assert np.all(err <= tol * rms + ulp16), (layer, which, err.max())
                else:
                    try:
                        within(a, b, tol)
                    except AssertionError as e:
                        raise AssertionError(f"token {i} layer {layer} {which}: {e}") from None
    within(drun.position_logits(), orun.position_logits())


GQA_CASES = [
    # (query heads, kv heads, head_dim, prompt length)
    (16, 4, 128, 12),   # ratio 4, one attention split
    (16, 2, 64, 150),   # ratio 8 (the 70B grouping), three splits, ragged last chunk
    (12, 4, 64, 70),    # ratio 3 (no exact kernel group size), two splits
    (8, 8, 128, 129),   # ratio 1, the step's own row opens a new split
]


@pytest.mark.parametrize("heads,kv_heads,head_dim,n_prompt", GQA_CASES)
def test_random_norm_weights_gqa_model(cuda, heads, kv_heads, head_dim, n_prompt):
    """GQA groupings with random per-layer norm weights (so the f16 rounding
    of norms is exercised), over prompts that span several 64-position
    attention splits."""
    import oracle as o
    from faber_runtime_b200 import ForwardRun, ModelConfig, synth
    cfg = ModelConfig(n_layers=2, d_model=1024, n_heads=heads, n_kv_heads=kv_heads,
                      head_dim=head_dim, ffn=2816, vocab=4096, tied_head=False,
                      rope_theta=500000.0, name="gqa-test")
    om, dm, _ = build_pair(cfg, 77, norms="random")
    prompt = synth.tokens(77, 1, n_prompt, cfg.vocab)
    ref_tokens, ref_logits, _ = om.greedy(prompt, 12, want_logits=True)
    run = ForwardRun(dm, prompt, context_length=n_prompt + 16)
    toks, fin = run.greedy(12)
    assert fin and toks.tolist() == ref_tokens.tolist()
    run2 = ForwardRun(dm, prompt, context_length=n_prompt + 16)
    for i in range(12):
        within(run2.position_logits(), ref_logits[i])
        run2.push_token(int(ref_tokens[i]))


def test_7b_shape_two_layers_over_prefix(cuda):
    import oracle as o
    from faber_runtime_b200 import LLAMA2_7B, ForwardRun, synth
    cfg = LLAMA2_7B.with_layers(2)
    om, dm, _ = build_pair(cfg, 7)
    n_prefix = 256
    span = cfg.n_kv_heads * cfg.head_dim
    orun = o.OracleRun(om, n_prefix + 8)
    drun = ForwardRun(dm, context_length=n_prefix + 8)
    for layer in range(cfg.n_layers):
        k = synth.normal(7, 1000 + layer, n_prefix * span, 0.0, 50.0)
        v = synth.normal(7, 2000 + layer, n_prefix * span, 0.0, 50.0)
        orun.set_prefix(layer, k, v, n_prefix)
        drun.set_prefix(layer, k, v, n_prefix)
    toks = synth.tokens(7, 5, 4, cfg.vocab)
    for t in toks:
        orun.push_token(int(t))
        drun.push_token(int(t))
        within(drun.position_logits(), orun.position_logits())
    assert len(drun) == n_prefix + 4


@pytest.mark.parametrize("heads,kv_heads,head_dim,n_prefix", [
    (8, 8, 128, 9001),   # ratio 1: six 32-position tiles per split CTA, the 4-stage ring wraps
    (16, 8, 64, 8190),   # ratio 2: five tiles per split CTA, ragged last tile
])
def test_streamed_attention_over_long_prefix(cuda, heads, kv_heads, head_dim, n_prefix):
    """One and two query heads per kv head over a long installed K/V prefix:
    the TMA-streamed decode attention (each split CTA several 32-position
    tiles through its ring, the tile holding the step's own row requested
    after the dependency wait) gives the oracle's logits."""
    import oracle as o
    from faber_runtime_b200 import ForwardRun, ModelConfig, synth
    cfg = ModelConfig(n_layers=2, d_model=1024, n_heads=heads, n_kv_heads=kv_heads, head_dim=head_dim,
                      ffn=2816, vocab=4096, tied_head=False, rope_theta=500000.0, name="stream-attn")
    om, dm, _ = build_pair(cfg, 31, norms="random")
    span = kv_heads * head_dim
    orun = o.OracleRun(om, n_prefix + 8)
    drun = ForwardRun(dm, context_length=n_prefix + 8)
    for layer in range(cfg.n_layers):
        k = synth.normal(31, 3000 + layer, n_prefix * span, 0.0, 2.0)
        v = synth.normal(31, 4000 + layer, n_prefix * span, 0.0, 2.0)
        orun.set_prefix(layer, k, v, n_prefix)
        drun.set_prefix(layer, k, v, n_prefix)
    for t in synth.tokens(31, 6, 4, cfg.vocab):
        orun.push_token(int(t))
        drun.push_token(int(t))
        within(drun.position_logits(), orun.position_logits())
    assert len(drun) == n_prefix + 4


def test_70b_shape_one_layer_over_prefix(cuda):
    """The 70B shape at full width (d 8192, 64/8 heads of 128, FFN 28672 =
    112 super-blocks, vocab 128256) cut to one layer, over an installed
    96-position K/V prefix: logits of three pushes within tolerance and the
    same greedy argmax."""
    import oracle as o
    from faber_runtime_b200 import LLAMA3_70B, ForwardRun, synth
    cfg = LLAMA3_70B.with_layers(1)
    om, dm, _ = build_pair(cfg, 70, norms="random")
    n_prefix = 96
    span = cfg.n_kv_heads * cfg.head_dim
    orun = o.OracleRun(om, n_prefix + 8)
    drun = ForwardRun(dm, context_length=n_prefix + 8)
    k = synth.normal(70, 1000, n_prefix * span, 0.0, 4.0)
    v = synth.normal(70, 2000, n_prefix * span, 0.0, 4.0)
    orun.set_prefix(0, k, v, n_prefix)
    drun.set_prefix(0, k, v, n_prefix)
    for t in synth.tokens(70, 5, 3, 32000):
        orun.push_token(int(t))
        drun.push_token(int(t))
        ref = orun.position_logits()
        got = drun.position_logits()
        within(got, ref)
        assert o.top1_non_eog(got) == o.top1_non_eog(ref)
    drun.close()
    dm.close()


PREFILL_CASES = [
    # (model, prompt length): the prompt goes through the tensor-core prompt
    # pass (tcgen05 GEMMs, tensor-core flash attention) in chunks of 2048
    ("7b-width-2-layers", 300),
    ("gqa-small", 2100),  # two chunks: the second attends to the first's cache
]


@pytest.mark.parametrize("which,n_prompt", PREFILL_CASES)
def test_prompt_pass_matches_oracle(cuda, which, n_prompt):
    import oracle as o
    from faber_runtime_b200 import LLAMA2_7B, ForwardRun, ModelConfig, synth
    if which == "gqa-small":
        cfg = ModelConfig(n_layers=2, d_model=1024, n_heads=16, n_kv_heads=4, head_dim=64,
                          ffn=2816, vocab=4096, tied_head=False, rope_theta=500000.0,
                          name="prefill-gqa")
    else:
        cfg = LLAMA2_7B.with_layers(2)
    om, dm, _ = build_pair(cfg, 91, norms="random")
    prompt = synth.tokens(91, 4, n_prompt, cfg.vocab)
    ref_tokens, ref_logits, _ = om.greedy(prompt, 4, want_logits=True)
    run = ForwardRun(dm, prompt, context_length=n_prompt + 8)
    assert len(run) == n_prompt
    within(run.position_logits(), ref_logits[0])
    toks, fin = run.greedy(4)
    assert fin and toks.tolist() == ref_tokens.tolist()


def test_prompt_pass_2048_tokens_7b_width_matches_incremental_decode(cuda):
    """The benchmark's prompt pass (2048 ids, 7B width, one chunk of tcgen05
    GEMMs and tensor-core flash attention) against the same prompt pushed
    one token at a time through the decode path, which the oracle tests pin
    (an oracle prompt pass over 2048 7B-width positions takes CPU-hours):
    the last position's logits within 1e-3 x RMS, the same argmax, and the
    same greedy continuation over the two caches."""
    from faber_runtime_b200 import LLAMA2_7B, DeviceModel, ForwardRun, synth
    cfg = LLAMA2_7B.with_layers(2)
    dm = DeviceModel(cfg, synth.model_tensors(cfg, 93, norms="random"))
    prompt = synth.tokens(93, 4, 2048, cfg.vocab)
    fast = ForwardRun(dm, context_length=2048 + 8)
    fast.push_tokens(prompt)  # one prompt-pass chunk
    slow = ForwardRun(dm, context_length=2048 + 8)
    for t in prompt:
        slow.push_token(int(t))  # the decode step, token by token
    assert len(fast) == len(slow) == 2048
    a, b = fast.position_logits(), slow.position_logits()
    within(a, b)
    assert int(np.argmax(a)) == int(np.argmax(b))
    ta, fa = fast.greedy(4)
    tb, fb = slow.greedy(4)
    assert fa and fb and ta.tolist() == tb.tolist()
    fast.close()
    slow.close()
    dm.close()


def test_reset_session_reruns_prompt_pass_identically(cuda):
    """A session reset and the same prompt pushed again through the prompt
    pass gives bit-identical
    logits and tokens: the pass reuses the session's scratch, and every
    reduction (split-K GEMMs, attention splits) runs in a fixed order."""
    from faber_runtime_b200 import ForwardRun, ModelConfig, synth
    cfg = ModelConfig(n_layers=2, d_model=1024, n_heads=16, n_kv_heads=4, head_dim=64,
                      ffn=2816, vocab=4096, tied_head=False, rope_theta=500000.0, name="reset-gqa")
    _, dm, _ = build_pair(cfg, 17, norms="random")
    prompt = synth.tokens(17, 4, 300, cfg.vocab)
    run = ForwardRun(dm, context_length=320)
    run.push_tokens(prompt)
    first = run.position_logits().copy()
    toks1, fin1 = run.greedy(4)
    run.reset()
    assert len(run) == 0
    run.push_tokens(prompt)
    assert np.array_equal(run.position_logits(), first)
    toks2, fin2 = run.greedy(4)
    assert fin1 and fin2 and toks1.tolist() == toks2.tolist()
    run.close()
    dm.close()


def test_fail_closed_and_commit_contract(tiny):
    from faber_runtime_b200 import FaberError, ForwardRun, OracleError
    _, dm, _ = tiny
    run = ForwardRun(dm, context_length=4)
    with pytest.raises(OracleError):
        run.position_logits()
    with pytest.raises(OracleError):
        run.push_tokens([])
    with pytest.raises(OracleError):
        run.push_token(32000)
    with pytest.raises(OracleError):
        run.push_token(-1)
    assert len(run) == 0
    run.push_tokens([1, 2, 3, 4])
    with pytest.raises(FaberError) as e:
        run.push_token(5)
    assert e.value.code == 2 and len(run) == 4
    # SequenceState::commit
    assert run.commit(10, 0, 1) == "applied"
    assert run.commit(10, 0, 1) == "idempotent_replay"
    with pytest.raises(FaberError):
        run.commit(11, 3, 2)  # out of order
    with pytest.raises(FaberError):
        run.commit(11, 1, 5)  # KV generation gap
    with pytest.raises(FaberError):
        run.commit(11, 1, 2, publication_boundary=0)
    assert run.commit(11, 1, 2) == "applied"
    run.reset()
    assert len(run) == 0
    run.push_token(3)
    assert len(run) == 1
