"""Allocation-free decode attention: faber_gpu_v2_attention_decode_static.

Some callers of this library cannot allocate device memory: a host that
accounts every byte of device memory up front (where an unaccounted
cudaMalloc is a failure), or code on a latency-critical path where
cudaMalloc / cudaFree may synchronize the device. This entry point serves
them: its scratch is a static device array inside the library, and the
caller passes only inputs and outputs.

Two comparators check its output. One is the existing session entry
points, whose attention uses session-allocated scratch: a traced push over
an installed K/V prefix gives that path's query, its new K/V row and its
attention output, and the static entry point gets the same query and cache
rows. The other is the CPU oracle's attention_gqa (src/cpu_oracle.rs:711-792)
on the same f16-rounded rows. Two calls in a row must both agree, because
the static scratch keeps the previous call's contents, and the calls must
leave the device's free memory unchanged. The file is named to be collected
last.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

RMS_TOL = 1e-3  # the tolerance of the other parity tests


def within(gpu, ref, tol=RMS_TOL):
    gpu = np.asarray(gpu, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(ref ** 2))
    err = np.max(np.abs(gpu - ref))
    assert np.all(np.isfinite(gpu)), "non-finite output"
    assert err <= tol * rms, f"max|err| {err:.3e} > {tol} x RMS {rms:.3e}"


def static_attention(q, k, v, out, heads, kv_heads, head_dim, n_kv):
    from faber_runtime_b200 import _lib
    _lib.call("faber_gpu_v2_attention_decode_static", q.data_ptr(), k.data_ptr(), v.data_ptr(),
              out.data_ptr(), heads, kv_heads, head_dim, n_kv,
              torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("heads,kv_heads,head_dim,n_prefix", [
    (16, 4, 128, 150),  # GQA ratio 4, several splits, ragged last group
    (8, 8, 64, 70),     # no grouping, head_dim 64
])
def test_static_attention_matches_session_attention(cuda, heads, kv_heads, head_dim, n_prefix):
    from faber_runtime_b200 import DeviceModel, ForwardRun, ModelConfig, synth
    cfg = ModelConfig(n_layers=1, d_model=1024, n_heads=heads, n_kv_heads=kv_heads,
                      head_dim=head_dim, ffn=1024, vocab=512, tied_head=False,
                      rope_theta=10000.0, name="static-attention")
    model = DeviceModel(cfg, synth.model_tensors(cfg, 5))
    run = ForwardRun(model, context_length=n_prefix + 4, trace=True)
    span = kv_heads * head_dim
    k = synth.normal(5, 100, n_prefix * span, 0.0, 1.0)
    v = synth.normal(5, 101, n_prefix * span, 0.0, 1.0)
    run.set_prefix(0, k, v, n_prefix)
    run.push_token(3)
    q = run.trace(0, "q_rot")
    ref = run.trace(0, "ctx")
    # the session caches K and V as f16 (round to nearest even, like numpy)
    kc = np.concatenate([k.reshape(n_prefix, span), run.trace(0, "k_rot").reshape(1, span)])
    vc = np.concatenate([v.reshape(n_prefix, span), run.trace(0, "v").reshape(1, span)])
    dq = torch.from_numpy(q).to(cuda)
    dk = torch.from_numpy(kc.astype(np.float16)).to(cuda)
    dv = torch.from_numpy(vc.astype(np.float16)).to(cuda)
    # the oracle's attention over the same f16-rounded cache rows
    import oracle as o
    want = o.attention_gqa(q, kc.astype(np.float16).astype(np.float32),
                           vc.astype(np.float16).astype(np.float32), 1, n_prefix + 1, heads,
                           kv_heads, head_dim, 1.0 / np.sqrt(np.float32(head_dim)))
    # every buffer exists before the first call, so nothing below allocates
    # on the caller's side either
    outs_dev = [torch.full((heads * head_dim,), float("nan"), dtype=torch.float32, device=cuda)
                for _ in range(2)]
    torch.cuda.synchronize()
    outs = []
    for i, out in enumerate(outs_dev):
        static_attention(dq, dk, dv, out, heads, kv_heads, head_dim, n_prefix + 1)
        torch.cuda.synchronize()
        if i == 0:  # after the first call: lazy module loading has happened
            free0 = torch.cuda.mem_get_info()[0]
        outs.append(out.cpu().numpy())
        within(outs[-1], ref)
        within(outs[-1], want)
    for _ in range(3):
        static_attention(dq, dk, dv, outs_dev[0], heads, kv_heads, head_dim, n_prefix + 1)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0, "a call changed the device's free memory"
    assert np.array_equal(outs[0], outs[1]), "two calls in a row differ"
    run.close()
    model.close()


def test_static_attention_rejects_sizes_beyond_its_scratch(cuda):
    from faber_runtime_b200 import FaberError, _lib
    buf = torch.zeros(1 << 16, dtype=torch.float32, device=cuda)
    p = buf.data_ptr()
    cases = [
        (256, 32, 128, 10, "at most 128 query heads"),   # more heads than the scratch holds
        (16, 4, 96, 10, "head_dim must be 64 or 128"),
        (32, 2, 128, 10, "more than 8 query heads"),
        (16, 4, 128, 0, "n_kv must be"),
        (16, 4, 128, (1 << 31) - 32, "n_kv must be"),  # would overflow the 32-bit group count
    ]
    for heads, kv_heads, hd, n_kv, text in cases:
        with pytest.raises(FaberError) as e:
            _lib.call("faber_gpu_v2_attention_decode_static", p, p, p, p, heads, kv_heads, hd, n_kv,
                      torch.cuda.current_stream().cuda_stream)
        assert e.value.code == 1 and text in str(e.value), str(e.value)
