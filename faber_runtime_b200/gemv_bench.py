"""Q4_K GEMV micro-benchmark: y = dense(W, x) with the resident tiled weight.

    python -m faber_runtime_b200.gemv_bench --rows 4096 --cols 4096 --copies 16 --iters 20

With ``--batch B`` it times the batched GEMV (B inputs per weight pass)
instead. Rotates over ``copies`` distinct weights (so the total exceeds L2 when
copies * rows * cols * 0.5625 B > 126 MB) and reports device time per
launch with CUDA events, and the achieved HBM bandwidth on the algorithmic
bytes (weights + x + y). Also the small-case driver for ncu captures.
"""

from __future__ import annotations

import argparse
import json

import numpy as np


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=4096)
    ap.add_argument("--cols", type=int, default=4096)
    ap.add_argument("--copies", type=int, default=16)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--native", action="store_true", help="native GGUF layout instead of tiles")
    ap.add_argument("--batch", type=int, default=0,
                    help="1-16: the batched GEMV (one weight pass for that many inputs)")
    args = ap.parse_args()

    import torch

    from . import _lib, dequant, synth
    _lib.call("faber_gpu_v2_init", 0)
    r, c = args.rows, args.cols
    blocks = [synth.q4k_blocks(1, 100 + k, r * c // 256) for k in range(args.copies)]
    nb_ = max(1, args.batch)
    x = torch.from_numpy(np.concatenate([synth.normal(1, 7 + i, c) for i in range(nb_)])).cuda()
    y = torch.empty(nb_ * r, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    if args.batch:
        ts = [dequant.Q4kTensor(b, r, c) for b in blocks]
        launch = [lambda t=t: t.gemv_batch(x.data_ptr(), args.batch, y.data_ptr(), s) for t in ts]
    elif args.native:
        ws = [torch.from_numpy(b).cuda() for b in blocks]
        launch = [lambda w=w: dequant.gemv_q4k(w.data_ptr(), r, c, x.data_ptr(), y.data_ptr(), s) for w in ws]
    else:
        ts = [dequant.Q4kTensor(b, r, c) for b in blocks]
        launch = [lambda t=t: t.gemv(x.data_ptr(), y.data_ptr(), s) for t in ts]
    for f in launch:
        f()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.iters):
        for f in launch:
            f()
    e1.record()
    torch.cuda.synchronize()
    n = args.iters * len(launch)
    us = e0.elapsed_time(e1) * 1e3 / n
    nbytes = r * c * 144 // 256 + 4 * nb_ * (r + c)
    print(json.dumps({"rows": r, "cols": c, "batch": nb_, "layout": "native" if args.native else "tiled",
                      "us_per_launch": us, "gbs": nbytes / (us * 1e-6) / 1e9,
                      "bytes_per_launch": nbytes, "launches": n}))


if __name__ == "__main__":
    main()
