#!/usr/bin/env python
"""Decode benchmark of the B200 Q4_K decoder path.

Workload (default): Llama-2-7B-shape decoder (32 layers, d 4096, 32 heads x
128, SwiGLU 11008, vocab 32000, RMSNorm eps 1e-5, RoPE theta 1e4), every
linear Q4_K with seeded random fields, f32 N(0, 0.02) token embedding and
output norm, batch 1. The KV cache is filled by the prompt pass over 2048
random token ids (tcgen05 GEMMs and tensor-core flash attention on one GPU; token
by token under tensor parallelism), then W warm-up and K timed greedy tokens
run as CUDA-graph replays.

prefill    the same prompt pass timed once more on a reset session
           (wall clock around the synchronizing call, max over ranks).

value      tokens/s over the K timed tokens (CUDA events on the decode
           stream, max over ranks), weights and KV resident in HBM
           (3.7 GB of weights per token: far larger than L2).
e2e        tokens/s through the public API with host buffers: per token
           one step_greedy call (the id host->device from pinned memory,
           the step and its greedy argmax, the next id device->host).
roofline   the Q4_K dequant-GEMV (the dominant kernel) over this rank's
           7B layer shapes + head, replayed in a CUDA graph over three
           weight copies per shape (411 MB > L2), CUDA events.
prefill_batch8   eight more 2048-id prompts through the prompt pass, one
           after another (one GPU; wall clock, tokens/s).
decode_batch16   sixteen sessions with their own prompts decoding K greedy
           tokens together through the batched path (one GPU; CUDA events;
           aggregate tokens/s). --no-batch skips both legs.
cpu_baseline  the C++ oracle restatement of the reference's CPU path on
           this host's cores: a 2-layer sample of the same model at
           context 2048, extrapolated to 32 layers; beside it the same on
           one thread (the reference's execution model) and the 4096 x 4096
           Q4_K GEMV per call on all cores and on one.

--impl reference times the reference's CPU path as its own line: whole
greedy tokens through all 32 layers of the same model (the reference is Rust
with no toolchain here; its restatement is the oracle port, which loads no
GPU code).
Multi-GPU (torchrun): tensor parallel over N ranks, the O and down partial
sums exchanged over NVLink peer memory inside the GEMVs; same tokens on
every rank.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

METRIC = "decode tok/s (7B-shape Q4_K, bs1) and Q4_K GEMV HBM GB/s vs peak"
SEED = 20261201
PREFILL = 2048


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi clock/throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.25)
        return self

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.15)
            self.proc.terminate()
            self.proc.wait()

    def summary(self):
        self.f.flush()
        rows = [r.split(",") for r in Path(self.f.name).read_text().splitlines() if r.strip()]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for k, nm in enumerate(names):
                if len(r) > 5 + k and r[5 + k].strip() == "Active":
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def build_model(cfg, device, tp, rank, uid):
    from faber_runtime_b200 import DeviceModel, synth
    return DeviceModel(cfg, synth.model_tensors(cfg, SEED), device=device, tp_size=tp,
                       tp_rank=rank, nccl_uid=uid)


def gemv_roofline(cfg, tp, stream_ptr, reps=6):
    """Dominant kernel: the tiled Q4_K GEMV over this rank's decode shapes."""
    import torch
    from faber_runtime_b200 import dequant, synth
    d, hd, F = cfg.d_model, cfg.head_dim, cfg.ffn
    Fl = (F // 256) // tp * 256 if tp > 1 else F
    shapes = [("qkv", (cfg.n_heads + 2 * cfg.n_kv_heads) * hd // tp, d), ("o", d, cfg.n_heads * hd // tp),
              ("gateup", 2 * Fl, d), ("down", d, Fl), ("head", cfg.vocab // tp, d)]
    copies = 3
    tens, bytes_per_round = [], 0
    for name, r, c in shapes:
        for k in range(copies):
            blocks = synth.q4k_blocks(SEED + k, synth.stream_id(name) + k, r * c // 256)
            tens.append((dequant.Q4kTensor(blocks, r, c), r, c))
            bytes_per_round += r * c * 144 // 256 + 4 * c + 4 * r
    xmax = max(c for _, _, c in tens)
    x = torch.randn(xmax, device="cuda")
    y = torch.empty(max(r for _, r, _ in tens), device="cuda")
    s = torch.cuda.current_stream()
    for t, r, c in tens:  # warm (and set kernel attributes) outside capture
        t.gemv(x.data_ptr(), y.data_ptr(), s.cuda_stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        cs = torch.cuda.current_stream().cuda_stream
        for _ in range(reps):
            for t, r, c in tens:
                t.gemv(x.data_ptr(), y.data_ptr(), cs)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(3):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    launches = 3 * reps * len(tens)
    total_bytes = 3 * reps * bytes_per_round
    # C0 shape alone (4096 x 4096, 9 469 952 B per matvec), 16 copies (151 MB)
    c0 = [dequant.Q4kTensor(synth.q4k_blocks(SEED, 900 + k, 65536), 4096, 4096) for k in range(16)]
    for t in c0:
        t.gemv(x.data_ptr(), y.data_ptr(), s.cuda_stream)
    torch.cuda.synchronize()
    g0 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g0):
        cs = torch.cuda.current_stream().cuda_stream
        for _ in range(8):
            for t in c0:
                t.gemv(x.data_ptr(), y.data_ptr(), cs)
    g0.replay()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(3):
        g0.replay()
    e1.record()
    torch.cuda.synchronize()
    ms0 = e0.elapsed_time(e1)
    n0 = 3 * 8 * 16
    return {"launches": launches, "avg_us": ms * 1e3 / launches, "bytes_per_launch": total_bytes / launches,
            "achieved_gbs": total_bytes / (ms * 1e-3) / 1e9,
            "c0_us": ms0 * 1e3 / n0, "c0_gbs": 9469952 * n0 / (ms0 * 1e-3) / 1e9}


GEMV_TRAFFIC_RATIO = (50775552 + 3840) / 50829312


def prefill_line(cfg, tokens, seconds, ws):
    """The prompt pass (C3 shape): tokens/s and tensor-core throughput. Useful
    FLOP = 2 x linear params x tokens; the tensor cores run twice that (exact
    hi/lo f16 activation pairs). With tensor parallelism the prompt is pushed
    token by token (the tensor-core pass is single-GPU)."""
    d, hd, F = cfg.d_model, cfg.head_dim, cfg.ffn
    params = cfg.n_layers * ((cfg.n_heads + 2 * cfg.n_kv_heads) * hd * d + d * cfg.n_heads * hd + 3 * F * d)
    flop = 2.0 * params * tokens
    return {"tokens": tokens, "ms": seconds * 1e3, "tok_s": tokens / seconds,
            "path": "tensor-core prompt pass" if ws == 1 else "token by token",
            "linear_tflops_useful": flop / seconds / 1e12,
            "tensor_tflops_hilo": 2 * flop / seconds / 1e12}


def cpu_sample(cfg, threads=None):
    """The oracle on this host's cores: 2 layers of cfg at context 2048,
    one token (push + logits), extrapolated to cfg.n_layers."""
    import oracle
    from faber_runtime_b200 import synth
    threads = threads or os.cpu_count() or 1
    oracle.set_threads(threads)
    sub = cfg.with_layers(2)
    tensors = {n: (t, a, r, c) for n, t, a, r, c in synth.model_tensors(sub, SEED)}
    om = oracle.OracleModel(sub, tensors)
    span = cfg.n_kv_heads * cfg.head_dim
    run = oracle.OracleRun(om, PREFILL + 64)
    for layer in range(2):
        k = synth.normal(SEED, 5000 + layer, PREFILL * span, 0.0, 50.0)
        v = synth.normal(SEED, 6000 + layer, PREFILL * span, 0.0, 50.0)
        run.set_prefix(layer, k, v, PREFILL)
    tok = 1
    times = []
    t_end = time.perf_counter() + 20.0
    while True:
        t0 = time.perf_counter()
        run.push_token(tok)
        t1 = time.perf_counter()
        logits = run.position_logits()
        t2 = time.perf_counter()
        tok = oracle.top1_non_eog(logits)
        times.append((t1 - t0, t2 - t1))
        if len(times) >= 2 and time.perf_counter() > t_end or len(times) >= 8:
            break
    push = float(np.median([a for a, _ in times]))
    head = float(np.median([b for _, b in times]))
    per_token = push * cfg.n_layers / 2 + head
    # one thread, the reference's own execution model: one more token
    oracle.set_threads(1)
    t0 = time.perf_counter()
    run.push_token(tok)
    t1 = time.perf_counter()
    run.position_logits()
    t2 = time.perf_counter()
    per_token_1 = (t1 - t0) * cfg.n_layers / 2 + (t2 - t1)
    # the 4096 x 4096 Q4_K GEMV (dequant fused, no materialization) per call
    w = synth.q4k_blocks(SEED, 77, 4096 * 4096 // 256)
    x = synth.normal(SEED, 78, 4096)
    gemv_ms = {}
    for n in (threads, 1):
        oracle.set_threads(n)
        reps, g0 = 0, time.perf_counter()
        while reps < 3 or (time.perf_counter() - g0 < 0.5 and reps < 50):
            oracle.dense_q(oracle.Q4_K, w, x, 4096, 4096)
            reps += 1
        gemv_ms[n] = (time.perf_counter() - g0) / reps * 1e3
    oracle.set_threads(threads)
    return {"value": 1.0 / per_token, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"C++ oracle, {cfg.name} cut to 2 of {cfg.n_layers} layers at context {PREFILL}, "
                      f"{len(times)} tokens (push {push:.3f} s + logits {head:.3f} s), per-token time "
                      f"extrapolated as push*{cfg.n_layers // 2} + logits",
            "per_token_s": per_token,
            "single_thread": {"value": 1.0 / per_token_1, "unit": "tok/s", "cores": 1,
                              "sample": "one token of the same sample on one thread, extrapolated alike"},
            "gemv_4096x4096_ms": {"cores": threads, "value": gemv_ms[threads], "single_thread": gemv_ms[1]}}


def run_reference(args):
    """The reference's CPU decode path (its oracle, restated in C++ because the
    Rust reference has no toolchain here) timed on this host's cores: every
    step is one whole greedy token through all 32 layers of the 7B shape at
    context 2048 plus the head (push_token, position_logits, top1_non_eog),
    measured, not extrapolated. Only the oracle library is loaded: the
    weights come from its own copy of the seeded generator, so nothing of the
    GPU package is imported. The K/V of the 2048 context positions are
    installed directly (a CPU prompt pass over 2048 ids would take hours);
    the work of a decode token does not depend on their values."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    import oracle
    from oracle import synth as osyn
    cfg = osyn.LLAMA2_7B
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    om = oracle.OracleModel(cfg, {n: (t, a, r, c) for n, t, a, r, c in osyn.model_tensors(cfg, SEED)})
    span = cfg.n_kv_heads * cfg.head_dim
    run = oracle.OracleRun(om, PREFILL + args.warmup + args.steps + 8)
    for layer in range(cfg.n_layers):
        run.set_prefix(layer, osyn.normal(SEED, 5000 + layer, PREFILL * span, 0.0, 50.0),
                       osyn.normal(SEED, 6000 + layer, PREFILL * span, 0.0, 50.0), PREFILL)
    tok = 1

    def step():
        nonlocal tok
        run.push_token(tok)
        tok = oracle.top1_non_eog(run.position_logits())

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    total = time.perf_counter() - t0
    value = args.steps / total
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded Q4_K fields, random token ids)",
            "config": {"workload": f"{cfg.name} greedy decode, batch 1, context {PREFILL}",
                       "global_batch": 1, "seq_len": PREFILL, "parallelism": "cpu",
                       "l2": "n/a (CPU)", "kv_prefix": f"{PREFILL} positions installed directly"},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": f"C++ restatement of the reference's CPU oracle (the Rust reference "
                                       f"has no toolchain here): {args.steps} whole greedy token(s), all "
                                       f"{cfg.n_layers} layers + head at context {PREFILL}, timed"},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_faber(args):
    import torch
    ws, rank, local = dist_env()
    n = args.gpus
    torch.cuda.set_device(local)
    from faber_runtime_b200 import LLAMA2_7B, ForwardRun, _lib, synth
    cfg = LLAMA2_7B
    uid = b""
    pg = None
    if ws > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("gloo", timeout=timedelta(seconds=600))
        pg = dist
        buf = torch.zeros(128, dtype=torch.uint8)
        if rank == 0:
            u = (ctypes_uid())
            buf = torch.frombuffer(bytearray(u), dtype=torch.uint8)
        dist.broadcast(buf, 0)
        uid = bytes(buf.tolist())
    model = build_model(cfg, local, ws, rank, uid)
    ctx = PREFILL + args.warmup + args.steps + args.e2e_steps + 16
    run = ForwardRun(model, context_length=ctx)
    prompt = synth.tokens(SEED, 1, PREFILL, cfg.vocab)
    run.push_tokens(prompt)  # first prompt pass: scratch allocation, kernel set-up
    # timed prompt pass (tcgen05 GEMMs + flash attention) on a reset session
    run.reset()
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    t_pf = time.perf_counter()
    run.push_tokens(prompt)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t_pf
    if pg:
        t = torch.tensor([prefill_s], dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        prefill_s = float(t.item())
    run.greedy(args.warmup)
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    with Clocks(local) as clk:
        toks, finite = run.greedy(args.steps)
        torch.cuda.synchronize()
    ms = run.last_greedy_ms()
    if pg:
        t = torch.tensor([ms], dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
    value = args.steps / (ms * 1e-3)
    # end to end through the public API with host buffers
    t0 = time.perf_counter()
    tok = int(toks[-1])
    for _ in range(args.e2e_steps):
        tok = run.step_greedy(tok)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    if pg:
        t = torch.tensor([wall], dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        wall = float(t.item())
    e2e = args.e2e_steps / wall
    roof = gemv_roofline(cfg, ws, torch.cuda.current_stream().cuda_stream)
    peak, peak_kind = peaks()
    step_bytes = (cfg.linear_bytes() + cfg.head_bytes()) / ws + \
        cfg.kv_bytes_per_position() * (PREFILL + args.warmup + args.steps / 2) / ws
    # per layer QKV, attention, O, gate/up, down; per token embed, head, finalize
    launches_per_token = 5 * cfg.n_layers + 3
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": n, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if ws > 1 else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded Q4_K fields, random token ids)",
            "config": {"workload": f"{cfg.name} greedy decode, batch 1, KV filled by the prompt pass over "
                                   f"{PREFILL} random ids, {args.steps} timed tokens",
                       "global_batch": 1, "seq_len": PREFILL, "parallelism": f"tp{ws}" if ws > 1 else "single",
                       "l2": "inputs larger than L2 (3.7 GB weights per token)", "kv_dtype": "f16 (value-identical)"},
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8},
            "gpu_launches": launches_per_token * args.steps,
            "roofline": {"bound": "hbm", "achieved": roof["achieved_gbs"], "peak": peak, "unit": "GB/s",
                         "frac": roof["achieved_gbs"] / peak, "peak_kind": peak_kind,
                         # DRAM bytes per launch: the ncu capture of gemv_pipe_kernel on
                         # 22016 x 4096 read 50 779 392 B for 50 829 312 algorithmic
                         # bytes (ratio 0.99902), scaled to this launch mix
                         "traffic": roof["bytes_per_launch"] * GEMV_TRAFFIC_RATIO,
                         "traffic_source": "ncu dram__bytes_read+write of gemv_pipe_kernel 22016x4096, "
                                           "scaled by algorithmic bytes per launch",
                         "kernel": "gemv_pipe_kernel (Q4_K dequant-GEMV) over 7B decode shapes",
                         "avg_launch_us": roof["avg_us"], "bytes_per_launch": roof["bytes_per_launch"]},
            "gemv_4096x4096": {"us": roof["c0_us"], "gbs": roof["c0_gbs"], "frac": roof["c0_gbs"] / peak},
            "decode_step_gbs": step_bytes / (ms / args.steps * 1e-3) / 1e9,
            "prefill": prefill_line(cfg, PREFILL, prefill_s, ws),
            "greedy_all_finite": bool(finite),
            "clocks": clk.summary()}
    if ws == 1 and not args.no_batch:
        line["prefill_batch8"], line["decode_batch16"] = batch_legs(cfg, model, args)
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_sample(cfg)
    if rank == 0:
        print(json.dumps(line), flush=True)
    run.close()
    model.close()
    if pg:
        pg.barrier()
        pg.destroy_process_group()


def batch_legs(cfg, model, args):
    """Batch-8 prompt pass and batch-16 decode (one GPU): 16 sessions, each
    with its own 2048-id prompt; 8 prompts are timed on reset sessions
    (sequences after one another through the tensor-core prompt pass), then all 16
    decode together through the batched path (every weight read once per
    step for the 16 sequences), CUDA events around the greedy steps."""
    import torch
    from faber_runtime_b200 import BatchRun, ForwardRun, synth
    ctx = PREFILL + args.warmup + args.steps + 8
    runs = [ForwardRun(model, context_length=ctx) for _ in range(16)]
    prompts = [synth.tokens(SEED, 100 + i, PREFILL, cfg.vocab) for i in range(16)]
    # first pushes allocate each session's prompt-pass scratch; the eight
    # timed prompts run again on reset sessions
    for r, p in zip(runs, prompts):
        r.push_tokens(p)
    for r in runs[:8]:
        r.reset()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for r, p in zip(runs[:8], prompts[:8]):
        r.push_tokens(p)
    torch.cuda.synchronize()
    pf_s = time.perf_counter() - t0
    batch = BatchRun(runs)
    batch.greedy(args.warmup)
    torch.cuda.synchronize()
    _, fin = batch.greedy(args.steps)
    ms = batch.last_ms()
    batch.close()
    for r in runs:
        r.close()
    flop = 2.0 * (cfg.linear_bytes() * 256 / 144) * 8 * PREFILL
    return ({"sequences": 8, "tokens": 8 * PREFILL, "ms": pf_s * 1e3, "tok_s": 8 * PREFILL / pf_s,
             "linear_tflops_useful": flop / pf_s / 1e12, "path": "tensor-core prompt pass per sequence"},
            {"sequences": 16, "steps": args.steps, "ms_per_step": ms / args.steps,
             "tok_s": 16 * args.steps / (ms * 1e-3), "all_finite": bool(fin.all()),
             "path": "batched Q4_K GEMV (one weight formation for all 16 sequences), per-sequence attention",
             "context": f"{PREFILL} + up to {args.warmup + args.steps}"})


def ctypes_uid() -> bytes:
    import ctypes
    from faber_runtime_b200 import _lib
    b = (ctypes.c_uint8 * 128)()
    _lib.call("faber_gpu_v2_nccl_unique_id", ctypes.addressof(b))
    return bytes(b)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--e2e-steps", type=int, default=64)
    ap.add_argument("--impl", default="faber", choices=["faber", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batch", action="store_true", help="skip the batch-8 prompt and batch-16 decode legs")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_faber(args)


if __name__ == "__main__":
    main()
