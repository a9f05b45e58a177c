"""Prompt-pass benchmark: one prompt through every layer on the tensor cores.

    python -m faber_runtime_b200.prefill_bench --layers 32 --tokens 2048 --reps 3

Builds the Llama-2-7B-shape model (optionally cut to ``--layers``) and times
``push_tokens`` of ``--tokens`` random ids on a reset session (device
synchronized on both sides, after one untimed warm-up pass). Reports
tokens/s and the linear layers' throughput: useful FLOP = 2 x params x
tokens; the tensor cores execute twice that, since each activation row runs
as an exact (hi, lo) f16 pair.
"""

from __future__ import annotations

import argparse
import json
import time


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--tokens", type=int, default=2048)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()

    import torch

    from . import LLAMA2_7B, DeviceModel, ForwardRun, synth
    cfg = LLAMA2_7B.with_layers(args.layers)
    model = DeviceModel(cfg, synth.model_tensors(cfg, 20261201))
    run = ForwardRun(model, context_length=args.tokens + 8)
    prompt = synth.tokens(20261201, 1, args.tokens, cfg.vocab)
    run.push_tokens(prompt)  # warm-up: scratch allocation, kernel attributes
    times = []
    for _ in range(args.reps):
        run.reset()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        run.push_tokens(prompt)
        torch.cuda.synchronize()
        times.append(time.perf_counter() - t0)
    best = min(times)
    d, hd, F = cfg.d_model, cfg.head_dim, cfg.ffn
    params = cfg.n_layers * ((cfg.n_heads + 2 * cfg.n_kv_heads) * hd * d + d * cfg.n_heads * hd + 3 * F * d)
    flop = 2.0 * params * args.tokens
    print(json.dumps({"layers": cfg.n_layers, "tokens": args.tokens, "ms": best * 1e3,
                      "tok_s": args.tokens / best, "linear_tflops_useful": flop / best / 1e12,
                      "tensor_tflops_hilo": 2 * flop / best / 1e12,
                      "reps_ms": [t * 1e3 for t in times]}))
    run.close()
    model.close()


if __name__ == "__main__":
    main()
