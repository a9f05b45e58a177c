"""The oracle's copy of the seeded generator draws the same bytes as the
product package's, so the benchmark's reference leg (which loads only the
oracle library) runs on the benchmarked weights."""

import numpy as np


def test_oracle_generator_matches_the_package_generator():
    from oracle import synth as osyn
    from faber_runtime_b200 import LLAMA2_7B, ModelConfig, synth
    cfg = ModelConfig(n_layers=2, d_model=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn=1024,
                      vocab=1000, tied_head=False, name="synth-check")
    for norms in ("ones", "random"):
        a = list(synth.model_tensors(cfg, 11, norms=norms))
        b = list(osyn.model_tensors(cfg, 11, norms=norms))
        assert [x[0] for x in a] == [x[0] for x in b]
        for (na, ta, aa, ra, ca), (nb, tb, ab, rb, cb) in zip(a, b):
            assert (na, ta, ra, ca) == (nb, tb, rb, cb)
            assert aa.dtype == ab.dtype and np.array_equal(aa.view(np.uint8), ab.view(np.uint8)), na
    assert np.array_equal(synth.tokens(5, 6, 100, 32000), osyn.tokens(5, 6, 100, 32000))
    assert np.array_equal(synth.normal(5, 7, 1000, 0.0, 50.0), osyn.normal(5, 7, 1000, 0.0, 50.0))
    for f in ("n_layers", "d_model", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab", "tied_head",
              "rms_eps", "rope_theta", "name"):
        assert getattr(LLAMA2_7B, f) == getattr(osyn.LLAMA2_7B, f), f
