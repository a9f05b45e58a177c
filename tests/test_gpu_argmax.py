"""The device argmax against top1_non_eog's rule (src/cpu_oracle.rs:979-995):
strict '>' from -inf, so among bitwise-equal logits the lowest id wins, and
ids in the EOG set never win.

Ties are made by duplicating weight rows: the head row of the natural
winner is copied into a lower and a higher id (Q4_K bytes for an untied
head, the embedding row for a tied head), so those ids get bitwise-equal
logits on both sides. The checks cover the batch-1 head GEMV epilogue
(session greedy and step_greedy), the batched-decode GEMM epilogue, and
the f16 tied-head kernel, with EOG sets that hide the tied ids one by one.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _cfg(tied):
    from faber_runtime_b200 import ModelConfig
    return ModelConfig(n_layers=1, d_model=512, n_heads=4, n_kv_heads=4, head_dim=128, ffn=1024,
                       vocab=4096, tied_head=tied, rope_theta=10000.0,
                       name="argmax-tied" if tied else "argmax")


def _tensors(cfg, seed):
    from faber_runtime_b200 import synth
    return [(n, t, np.array(a, copy=True), r, c) for n, t, a, r, c in synth.model_tensors(cfg, seed)]


def _with_ties(tensors, cfg, winner, ids):
    """Copy the head row of `winner` into every id of `ids`."""
    out = []
    for n, t, a, r, c in tensors:
        if (n == "output" and not cfg.tied_head) or (n == "token_embd" and cfg.tied_head):
            a = a.copy()
            row = a.size // r
            for i in ids:
                a[i * row:(i + 1) * row] = a[winner * row:(winner + 1) * row]
        out.append((n, t, a, r, c))
    return out


def _oracle(cfg, tensors):
    import oracle as o
    return o.OracleModel(cfg, {n: (t, a, r, c) for n, t, a, r, c in tensors})


def _expected(logits, eog):
    import oracle as o
    return o.top1_non_eog(logits, eog)


@pytest.mark.parametrize("tied", [False, True])
def test_ties_go_to_the_lowest_id_and_eog_ids_are_skipped(cuda, tied):
    import oracle as o
    from faber_runtime_b200 import DeviceModel, ForwardRun, synth
    cfg = _cfg(tied)
    base = _tensors(cfg, 31)
    prompt = synth.tokens(31, 2, 12, cfg.vocab)
    # the natural winner after the prompt, on the oracle
    orun = o.OracleRun(_oracle(cfg, base), 32)
    for t in prompt:
        orun.push_token(int(t))
    winner = o.top1_non_eog(orun.position_logits())
    # a lower id in another 16-row tile, a higher id in the winner's own tile
    # (or the next one), and the last id; none of them in the prompt
    used = set(int(t) for t in prompt) | {winner}
    low = next(i for i in range(3, cfg.vocab) if i not in used and i // 16 != winner // 16)
    high = next((i for i in range(winner + 1, cfg.vocab) if i not in used), None)
    last = cfg.vocab - 1 if cfg.vocab - 1 not in used | {high} else None
    ties = sorted({i for i in (low, high, last) if i is not None})
    tensors = _with_ties(base, cfg, winner, ties)
    om = _oracle(cfg, tensors)
    dm = DeviceModel(cfg, tensors)
    orun = o.OracleRun(om, 32)
    for t in prompt:
        orun.push_token(int(t))
    ref = orun.position_logits()
    run = ForwardRun(dm, prompt, context_length=32)
    lg = run.position_logits()
    tied_ids = sorted(set(ties) | {winner})
    # the duplicated rows give bitwise-equal logits on both sides
    assert len({ref[i].tobytes() for i in tied_ids}) == 1
    assert len({lg[i].tobytes() for i in tied_ids}) == 1, [lg[i] for i in tied_ids]
    assert o.top1_non_eog(ref) == tied_ids[0] == min(low, winner)
    eog_sets = [(), (tied_ids[0],), tuple(tied_ids[:2]), tuple(tied_ids[:-1]), tuple(tied_ids),
                tuple(tied_ids) + (5, 6)]
    for eog in eog_sets:
        want = _expected(lg, eog)
        assert want == _expected(ref, eog), eog  # the oracle agrees on its own logits
        if len(eog) < len(tied_ids):
            assert want == tied_ids[len(eog)], (eog, want)
        else:
            assert want not in tied_ids
        r1 = ForwardRun(dm, prompt, context_length=32)
        toks, fin = r1.greedy(1, eog=eog)
        assert fin and int(toks[0]) == want, (eog, int(toks[0]), want)
        r1.close()
        # step_greedy: the argmax of the next position after pushing the
        # prompt's last token again through a host-driven step
        r2 = ForwardRun(dm, prompt[:-1], context_length=32)
        assert r2.step_greedy(int(prompt[-1]), eog=eog) == want
        r2.close()
    run.close()
    dm.close()


def test_batched_argmax_epilogue_keeps_the_tie_rule(cuda):
    """The batched-decode head GEMM's argmax epilogue: every sequence of a
    batch whose logits tie picks the lowest id, and EOG ids are skipped."""
    import oracle as o
    from faber_runtime_b200 import BatchRun, DeviceModel, ForwardRun, synth
    cfg = _cfg(False)
    base = _tensors(cfg, 41)
    prompt = synth.tokens(41, 3, 40, cfg.vocab)
    orun = o.OracleRun(_oracle(cfg, base), 64)
    for t in prompt:
        orun.push_token(int(t))
    winner = o.top1_non_eog(orun.position_logits())
    used = set(int(t) for t in prompt) | {winner}
    low = next(i for i in range(1, cfg.vocab) if i not in used and i // 128 != winner // 128)
    high = next((i for i in range(winner + 1, cfg.vocab) if i not in used), None)
    if high is None:  # the winner is the last id: tie with a second lower id
        high = next(i for i in range(low + 1, cfg.vocab) if i not in used)
    tensors = _with_ties(base, cfg, winner, [low, high])
    om = _oracle(cfg, tensors)
    orun = o.OracleRun(om, 64)
    for t in prompt:
        orun.push_token(int(t))
    ref = orun.position_logits()
    tied_ids = sorted({low, winner, high})
    dm = DeviceModel(cfg, tensors)
    for eog in [(), (tied_ids[0],), tuple(tied_ids[:2])]:
        want = _expected(ref, eog)
        assert want == tied_ids[len(eog)]
        runs = [ForwardRun(dm, prompt, context_length=64) for _ in range(3)]
        batch = BatchRun(runs)
        toks, fin = batch.greedy(1, eog=eog)
        assert fin.all() and toks[:, 0].tolist() == [want] * 3, (eog, toks[:, 0].tolist(), want)
        batch.close()
        for r in runs:
            r.close()
    dm.close()
