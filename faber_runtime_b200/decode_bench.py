"""Decode-step micro-benchmark: greedy tokens over an installed K/V prefix.

    python -m faber_runtime_b200.decode_bench --layers 32 --ctx 2048 --steps 8
    python -m faber_runtime_b200.decode_bench --model 70b --ctx 4096 --steps 32
    python -m faber_runtime_b200.decode_bench --model 70b --ctx 4096 --steps 16 --batch 16

Builds the Llama-2-7B-shape model (or, with ``--model 70b``, the 70B shape:
80 layers, d 8192, 64/8 heads, FFN 28672, vocab 128256; 39 GB of Q4_K), cut
to ``--layers`` when given, installs
a ``--ctx``-position K/V prefix in every layer directly (the same seeded
random rows in each layer, instead of decoding ``--ctx`` tokens), pushes one
token, then runs ``--warmup`` and ``--steps`` greedy tokens as CUDA-graph
replays. Each token launches 5 kernels per layer plus embed, head GEMV and
finalize (5 * layers + 3), which is what an ncu launch list of one token
holds. With ``--batch B`` that many sessions (each with the prefix, then a
different first token) decode together through the batched path; tok/s is
then the aggregate over all sequences and ``kv_bytes`` counts every
sequence's cache.
"""

from __future__ import annotations

import argparse
import json


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", choices=("7b", "70b"), default="7b")
    ap.add_argument("--layers", type=int, default=0, help="0: every layer of the shape")
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--batch", type=int, default=1, help="sequences decoded together (1-16)")
    args = ap.parse_args()

    import torch

    from . import LLAMA2_7B, LLAMA3_70B, BatchRun, DeviceModel, ForwardRun, synth
    cfg = LLAMA2_7B if args.model == "7b" else LLAMA3_70B
    if args.layers:
        cfg = cfg.with_layers(args.layers)
    seed = 20261201
    model = DeviceModel(cfg, synth.model_tensors(cfg, seed))
    span = cfg.n_kv_heads * cfg.head_dim
    k = synth.normal(seed, 5000, args.ctx * span, 0.0, 1.0)
    v = synth.normal(seed, 6000, args.ctx * span, 0.0, 1.0)
    runs = []
    for i in range(args.batch):
        run = ForwardRun(model, context_length=args.ctx + args.warmup + args.steps + 4)
        for layer in range(cfg.n_layers):
            run.set_prefix(layer, k, v, args.ctx)
        run.push_token(1 + i)
        runs.append(run)
    if args.batch == 1:
        run = runs[0]
        run.greedy(args.warmup)
        torch.cuda.synchronize()
        toks, finite = run.greedy(args.steps)
        ms = run.last_greedy_ms()
    else:
        batch = BatchRun(runs)
        batch.greedy(args.warmup)
        torch.cuda.synchronize()
        toks, fin = batch.greedy(args.steps)
        ms = batch.last_ms()
        finite = bool(fin.all())
        batch.close()
    kv_bytes = args.batch * cfg.n_layers * 2 * span * 2 * (args.ctx + args.warmup + args.steps // 2)
    w_bytes = cfg.linear_bytes() + cfg.head_bytes()
    print(json.dumps({"model": cfg.name, "layers": cfg.n_layers, "ctx": args.ctx, "batch": args.batch,
                      "steps": args.steps, "ms_per_step": ms / args.steps,
                      "tok_s": args.batch * args.steps / (ms * 1e-3),
                      "weight_bytes": w_bytes, "kv_bytes": kv_bytes,
                      "gbs": (w_bytes + kv_bytes) / (ms / args.steps * 1e-3) / 1e9,
                      "finite": finite}))
    for r in runs:
        r.close()
    model.close()


if __name__ == "__main__":
    main()
