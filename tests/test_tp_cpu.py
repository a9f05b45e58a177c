"""Tensor-parallel sharding on CPU: two gloo ranks, one decode step.

Each rank takes its block of every tensor from the library's plan
(faber_gpu_v2_tp_shard, the same function the GPU upload applies), computes
its part of one decoder layer and the head with the oracle's CPU ops on that
block only, and gloo collectives recombine the parts:

* column-parallel outputs (Q/K/V by head, gate/up by FFN super-block,
  logits by vocab row) are gathered and must equal the unsharded oracle's
  trace bit for bit (every output row is computed from the same weights);
* row-parallel partial sums (O and down) are all-reduced and must match
  within 1e-5 x RMS (only the order of one f32 sum differs);
* the greedy argmax of the gathered logits is the oracle's token.

No GPU is used: this covers the host-side plan and the collective algebra
of the multi-GPU decode step.
"""

import socket

import numpy as np
import pytest

WORLD = 2


def _cfg():
    from faber_runtime_b200 import ModelConfig
    return ModelConfig(n_layers=1, d_model=512, n_heads=8, n_kv_heads=4, head_dim=64, ffn=1536,
                       vocab=4096, tied_head=False, rope_theta=10000.0, name="tp-cpu")


def _shard(cfg, rank, name):
    import ctypes
    from faber_runtime_b200 import _lib
    c = cfg.c_struct(tp_size=WORLD, tp_rank=rank)
    out = (ctypes.c_uint64 * 6)()
    _lib.call("faber_gpu_v2_tp_shard", ctypes.byref(c), name.encode(), ctypes.addressof(out))
    return tuple(int(v) for v in out)


def _block(arr, rows, cols, r0, nr, c0, nc):
    """Native Q4_K blocks of rows [r0, r0+nr) x cols [c0, c0+nc)."""
    b = arr.reshape(rows, cols // 256, 144)
    return np.ascontiguousarray(b[r0:r0 + nr, c0 // 256:(c0 + nc) // 256]).reshape(-1)


def _within(a, b, tol):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    rms = np.sqrt(np.mean(b ** 2))
    assert np.max(np.abs(a - b)) <= tol * rms, (np.max(np.abs(a - b)), rms)


def _worker(rank, port, result_q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import oracle as o
    from faber_runtime_b200 import synth
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=WORLD, timeout=timedelta(seconds=60))
    try:
        cfg = _cfg()
        tensors = {n: (t, a, r, c) for n, t, a, r, c in synth.model_tensors(cfg, 31, norms="random")}

        def T(gguf_name):  # generator names carry no ".weight" suffix
            return tensors[gguf_name[:-len(".weight")]]
        d, hd, eps = cfg.d_model, cfg.head_dim, cfg.rms_eps
        n_prefix, token = 40, 17
        span = cfg.n_kv_heads * hd
        kp = synth.normal(31, 700, n_prefix * span, 0.0, 1.0)
        vp = synth.normal(31, 701, n_prefix * span, 0.0, 1.0)
        # unsharded reference: the oracle's traced decode step
        om = o.OracleModel(cfg, tensors)
        run = o.OracleRun(om, n_prefix + 4, trace=True)
        run.set_prefix(0, kp, vp, n_prefix)
        run.push_token(token)
        ref = {w: run.trace(0, w) for w in ("attn_in", "q_rot", "k_rot", "v", "ctx", "h2", "hh",
                                             "h_out")}
        ref_logits = run.position_logits()

        def wq(name, x):  # this rank's Q4_K block times x, f16-rounded weights
            rows, cols, r0, nr, c0, nc = _shard(cfg, rank, name)
            _, arr, _, _ = T(name)
            blk = _block(arr, rows, cols, r0, nr, c0, nc)
            return o.dense_q(o.Q4_K, blk, np.asarray(x, np.float32)[c0:c0 + nc], nc, nr, f16_round=True), (r0, nr)

        def gather(local):
            parts = [torch.zeros(0)] * WORLD
            lens = [torch.zeros(1, dtype=torch.int64) for _ in range(WORLD)]
            dist.all_gather(lens, torch.tensor([local.size], dtype=torch.int64))
            buf = [torch.zeros(int(n.item()), dtype=torch.float32) for n in lens]
            dist.all_gather(buf, torch.from_numpy(np.ascontiguousarray(local, np.float32)))
            return np.concatenate([b.numpy() for b in buf])

        def allreduce(local):
            t = torch.from_numpy(np.ascontiguousarray(local, np.float32)).clone()
            dist.all_reduce(t)
            return t.numpy()

        emb = T("token_embd.weight")[1].reshape(cfg.vocab, d)
        h = o.f16_round(emb[token])
        attn_in = o.rms_norm(h, o.f16_round(T("blk.0.attn_norm.weight")[1]), eps)
        assert np.array_equal(attn_in, ref["attn_in"])  # replicated, identical
        q, (q0, nq) = wq("blk.0.attn_q.weight", attn_in)
        k, (k0, nk) = wq("blk.0.attn_k.weight", attn_in)
        v, _ = wq("blk.0.attn_v.weight", attn_in)
        hl, hkvl = nq // hd, nk // hd
        q = o.rope_all_heads(q, hl, hd, n_prefix, cfg.rope_theta)
        k = o.rope_all_heads(k, hkvl, hd, n_prefix, cfg.rope_theta)
        assert np.array_equal(gather(q), ref["q_rot"])
        assert np.array_equal(gather(k), ref["k_rot"])
        assert np.array_equal(gather(v), ref["v"])
        # this rank's kv heads of the cache (f16-rounded like the reference)
        kc = np.concatenate([kp.reshape(n_prefix, span)[:, k0:k0 + nk], o.f16_round(k)[None]])
        vc = np.concatenate([vp.reshape(n_prefix, span)[:, k0:k0 + nk], o.f16_round(v)[None]])
        ctx = o.attention_gqa(q, o.f16_round(kc).reshape(-1), o.f16_round(vc).reshape(-1), 1,
                              n_prefix + 1, hl, hkvl, hd, 1.0 / np.sqrt(np.float32(hd)))
        assert np.array_equal(gather(ctx), ref["ctx"])
        o_part, _ = wq("blk.0.attn_output.weight", _place(ctx, q0, cfg.n_heads * hd))
        h2 = o.residual_add(h, allreduce(o_part))
        _within(h2, ref["h2"], 1e-5)
        hh = o.rms_norm(ref["h2"], o.f16_round(T("blk.0.ffn_norm.weight")[1]), eps)
        gate, (f0, nf) = wq("blk.0.ffn_gate.weight", hh)
        up, _ = wq("blk.0.ffn_up.weight", hh)
        act = o.swiglu(gate, up)
        down_part, _ = wq("blk.0.ffn_down.weight", _place(act, f0, cfg.ffn))
        h_out = o.residual_add(ref["h2"], allreduce(down_part))
        _within(h_out, ref["h_out"], 1e-5)
        xo = o.rms_norm(ref["h_out"], T("output_norm.weight")[1], eps)
        lg, _ = wq("output.weight", xo)
        logits = gather(lg)
        assert np.array_equal(logits, ref_logits)
        assert o.top1_non_eog(logits) == o.top1_non_eog(ref_logits)
        result_q.put((rank, "ok"))
    except Exception as e:  # report to the parent, then fail the rank
        result_q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def _place(local, start, total):
    """A full-length input vector holding `local` at [start, start+len)."""
    x = np.zeros(total, np.float32)
    x[start:start + local.size] = local
    return x


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_plan_covers_every_tensor_once(faber):
    """Column blocks tile the rows and row blocks tile the columns, in rank
    order, for every tensor of a GQA layer; vectors stay whole."""
    cfg = _cfg()
    names = ["token_embd.weight", "output_norm.weight", "output.weight",
             *[f"blk.0.{s}.weight" for s in ("attn_norm", "attn_q", "attn_k", "attn_v",
                                            "attn_output", "ffn_norm", "ffn_gate", "ffn_up",
                                            "ffn_down")]]
    for name in names:
        parts = [_shard(cfg, r, name) for r in range(WORLD)]
        rows, cols = parts[0][:2]
        if name.endswith(("norm.weight",)) or name == "token_embd.weight":
            assert all(p == (rows, cols, 0, rows, 0, cols) for p in parts), name
            continue
        if name.endswith(("attn_output.weight", "ffn_down.weight")):
            assert [p[4] for p in parts] == [0, parts[0][5]] and sum(p[5] for p in parts) == cols
            assert all(p[2:4] == (0, rows) and p[4] % 256 == 0 for p in parts), name
        else:
            assert [p[2] for p in parts] == [0, parts[0][3]] and sum(p[3] for p in parts) == rows
            assert all(p[4:6] == (0, cols) for p in parts), name


def test_two_gloo_ranks_reproduce_the_unsharded_step(faber, oracle):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    mp.start_processes(_worker, args=(_free_port(), q), nprocs=WORLD, join=True,
                       start_method="spawn")
    got = sorted(q.get() for _ in range(WORLD))
    assert got == [(0, "ok"), (1, "ok")], got


@pytest.mark.parametrize("world", [4, 8])
@pytest.mark.parametrize("which", ["7b", "70b"])
def test_plan_tiles_full_shapes_at_4_and_8_ranks(faber, which, world):
    """The 7B (43 FFN super-blocks: uneven split) and 70B (8 kv heads: one
    per rank at 8) plans: every rank's blocks are whole super-blocks, tile
    the rows (column-parallel) or the columns (row-parallel) in rank order,
    and the FFN split of gate/up matches the input split of down."""
    import ctypes

    from faber_runtime_b200 import LLAMA2_7B, LLAMA3_70B, _lib
    cfg = LLAMA2_7B if which == "7b" else LLAMA3_70B

    def shard(rank, name):
        c = cfg.c_struct(tp_size=world, tp_rank=rank)
        out = (ctypes.c_uint64 * 6)()
        _lib.call("faber_gpu_v2_tp_shard", ctypes.byref(c), name.encode(), ctypes.addressof(out))
        return tuple(int(v) for v in out)

    col = ["attn_q", "attn_k", "attn_v", "ffn_gate", "ffn_up"]
    for slot in col + ["attn_output", "ffn_down"]:
        parts = [shard(r, f"blk.3.{slot}.weight") for r in range(world)]
        rows, cols = parts[0][:2]
        if slot in col:
            starts = [p[2] for p in parts]
            assert starts == sorted(starts) and starts[0] == 0
            assert all(p[2] + p[3] == q[2] for p, q in zip(parts, parts[1:])), slot
            assert sum(p[3] for p in parts) == rows and all(p[3] > 0 for p in parts)
            if slot.startswith("attn"):
                assert all(p[3] % cfg.head_dim == 0 for p in parts)
            else:
                assert all(p[2] % 256 == 0 and p[3] % 256 == 0 for p in parts)
        else:
            assert all(p[4] + p[5] == q[4] for p, q in zip(parts, parts[1:])), slot
            assert sum(p[5] for p in parts) == cols and all(p[4] % 256 == 0 for p in parts)
    for r in range(world):  # down's input block is this rank's FFN block
        g, dn = shard(r, "blk.0.ffn_gate.weight"), shard(r, "blk.0.ffn_down.weight")
        assert (g[2], g[3]) == (dn[4], dn[5])
        o, q = shard(r, "blk.0.attn_output.weight"), shard(r, "blk.0.attn_q.weight")
        assert (q[2], q[3]) == (o[4], o[5])
    heads = [shard(r, "output.weight") for r in range(world)]
    assert sum(h[3] for h in heads) == cfg.vocab
