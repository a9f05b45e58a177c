"""Partition byte budgets on the host (no GPU): PartitionBudgetLedger's
checked sum and VirtualDevicePartition::admit (src/partition.rs:111-155,
293-315), the per-device usage table and its policy limit, and the
pre-allocation plan of one tensor-parallel rank against an independent
restatement of the engine's buffer formulas and the byte counts of the 7B
and 70B shapes.
"""

import ctypes
import math
from collections import Counter

import pytest

from faber_runtime_b200 import LLAMA2_7B, LLAMA3_70B, TINY, FaberError, ModelConfig
from faber_runtime_b200 import _lib
from faber_runtime_b200 import partition as pt

U64_MAX = (1 << 64) - 1
MODULE_BYTES = 256 + 128 * 4 + (2 << 20)  # the allocation-free attention scratch


# --- admission ----------------------------------------------------------------

def test_total_bytes_is_a_checked_sum():
    led = pt.PartitionLedger(1, 2, 3, 4, 5, 6, 7)
    assert led.total_bytes() == 28
    assert pt.PartitionLedger(weight_bytes=U64_MAX).total_bytes() == U64_MAX
    assert pt.PartitionLedger(weight_bytes=U64_MAX, kv_cache_bytes=1).total_bytes() is None


def test_admit_at_and_above_the_limit():
    led = pt.PartitionLedger(weight_bytes=1000, kv_cache_bytes=200, activation_scratch_bytes=30,
                             module_storage_bytes=4, allocator_overhead_bytes=5,
                             transfer_staging_bytes=6, concurrent_state_bytes=7)
    assert pt.admit(led, 1252) == 1252  # exactly at the limit admits
    with pytest.raises(FaberError) as e:
        pt.admit(led, 1251)
    assert e.value.code == _lib.BUDGET_EXCEEDED
    # every class counts toward the total
    for i in range(7):
        one = [0] * 7
        one[i] = 11
        with pytest.raises(FaberError):
            pt.admit(pt.PartitionLedger(*one), 10)
        assert pt.admit(pt.PartitionLedger(*one), 11) == 11


def test_admit_fails_closed_on_overflow():
    led = pt.PartitionLedger(weight_bytes=1 << 63, kv_cache_bytes=1 << 63)
    total = _lib.U64()
    st = _lib.lib().faber_gpu_v2_partition_admit(ctypes.byref(led.c_struct()), U64_MAX, ctypes.byref(total))
    assert st.code == _lib.BUDGET_EXCEEDED and total.value == U64_MAX
    assert pt.admit(pt.PartitionLedger(), 0) == 0  # an empty ledger fits a zero limit


# --- per-device accounting (host counters only) -----------------------------------

def test_usage_starts_empty_and_limits_are_per_device():
    for dev in (0, 7, 63):
        assert pt.usage(dev) == pt.PartitionLedger()
    with pytest.raises(FaberError) as e:
        pt.usage(64)
    assert e.value.code == _lib.INVALID_ARGUMENT
    with pytest.raises(FaberError):
        pt.usage(-1)
    pt.set_limit(5, 1 << 30)  # nothing held there: any limit is accepted
    pt.set_limit(5, 0)
    with pytest.raises(FaberError):
        pt.set_limit(64, 1)


# --- the pre-allocation plan --------------------------------------------------------

def charge(n: int) -> int:
    """The allocator policy: 512-byte units below 1 MiB, 2 MiB units above."""
    if n == 0:
        return 0
    unit = 512 if n < (1 << 20) else (2 << 20)
    return -(-n // unit) * unit


def tiled(rows, cols, start):
    """Buffers of repack_q4k's tile layout for rows starting at start(j)."""
    offs = Counter(start(j) % 256 for j in range(rows))
    tiles = sum(-(-c // 16) for c in offs.values())
    nb = -(-(cols + max(offs)) // 256)
    bufs = [tiles * nb * 2304]
    if set(offs) != {0}:
        bufs += [tiles * 4, tiles * 16 * 4]
    return bufs


STEP_STATE_BYTES = 40  # int64 token, six 32-bit fields, u64 argmax key


def expected_plan(cfg: ModelConfig, ctx: int, sessions: int, sms: int, tp: int, rank: int):
    """Restatement of the buffers a rank's model upload and sessions
    allocate, class by class (the engine's tp_plan and session buffers)."""
    d, hd, F, V = cfg.d_model, cfg.head_dim, cfg.ffn, cfg.vocab
    Hl, Hkvl = cfg.n_heads // tp, cfg.n_kv_heads // tp
    if tp == 1:
        Fl = F
    else:
        nF = F // 256
        Fl = ((rank + 1) * nF // tp - rank * nF // tp) * 256
    Vl = (rank + 1) * V // tp - rank * V // tp
    nq, nk = Hl * hd, Hkvl * hd
    w = []
    o_cols = cfg.n_heads * hd if tp == 1 else nq
    down_cols = F if tp == 1 else Fl
    for _ in range(cfg.n_layers):
        w += tiled(nq + 2 * nk, d, lambda j: (j if j < nq else (j - nq if j < nq + nk else j - nq - nk)) * d)
        w += tiled(d, o_cols, lambda j: j * o_cols)
        w += tiled(2 * Fl, d, lambda j: (j >> 1) * d)
        w += tiled(d, down_cols, lambda j: j * down_cols)
        w += [d * 4, d * 4]
    w += [V * d * 2, d * 4]
    if not cfg.tied_head:
        w += tiled(Vl, d, lambda j: j * d)
    splits = max(1, min(-(-6 * sms // Hkvl), -(-ctx // 32)))
    kv, act, state, staging = [], [], [], []
    for _ in range(sessions):
        kv += [cfg.n_layers * ctx * nk * 2] * 2
        state += [ctx * (hd // 2) * 8, STEP_STATE_BYTES, ctx * 8 + 8, ctx * 8]
        act += [d * 4] * 4 + [nq * 4] * 2 + [Fl * 4, Vl * 4, V * 4 if tp > 1 else 0,
                                             Hl * splits * (hd + 2) * 4, Hkvl * 4]
        staging += [2 * tp * d * 8 + 256 if tp > 1 else 0]
        if tp == 1 and d % 256 == 0 and nq % 256 == 0 and Fl % 256 == 0:
            cap = min(ctx, 2048)
            kmax = max(d, nq, Fl)
            act += [cap * d * 4, 2 * cap * kmax * 2, cap * 4, cap * nq * 4, cap * nq * 4, cap * Fl * 4]
    overhead = sum(charge(b) - b for b in w + kv + act + state + staging)
    return pt.PartitionLedger(sum(w), sum(kv), sum(act), MODULE_BYTES, overhead, sum(staging), sum(state))


@pytest.mark.parametrize("cfg,ctx,sessions,tp", [
    (TINY, 96, 1, 1),                    # tied head, FFN not in whole super-blocks (two row offsets)
    (TINY, 4096, 3, 1),
    (LLAMA2_7B, 2048, 1, 1),             # with the prompt pass's scratch
    (LLAMA2_7B.with_layers(2), 300, 2, 2),
    (LLAMA2_7B, 2048, 1, 8),             # uneven FFN shares (43 super-blocks over 8 ranks)
    (LLAMA3_70B, 4096, 1, 8),
    (LLAMA3_70B.with_layers(3), 4096, 16, 4),
])
def test_plan_matches_the_restated_buffers(cfg, ctx, sessions, tp):
    for rank in sorted({0, tp - 1}):
        got = pt.plan(cfg, ctx, sessions=sessions, sms=148, tp_size=tp, tp_rank=rank)
        assert got == expected_plan(cfg, ctx, sessions, 148, tp, rank)


def test_plan_byte_counts_of_the_decoder_shapes():
    # 7B shape, one GPU: every linear tiles exactly (3 642 753 024 B of Q4_K
    # linears plus the 73 728 000 B head), the f16 embedding and 65 f32 norms
    p = pt.plan(LLAMA2_7B, 2048)
    assert p.weight_bytes == 3_642_753_024 + 73_728_000 + 32000 * 4096 * 2 + 65 * 4096 * 4
    assert p.kv_cache_bytes == 524_288 * 2048  # f16 K and V per position
    assert p.transfer_staging_bytes == 0
    # 70B shape over 8 ranks: the linears and the head split across ranks,
    # embedding and norms replicated, one kv head of K/V per rank
    ranks = [pt.plan(LLAMA3_70B, 4096, tp_size=8, tp_rank=r) for r in range(8)]
    replicated = 128256 * 8192 * 2 + (2 * 80 + 1) * 8192 * 4
    assert sum(r.weight_bytes - replicated for r in ranks) == 38_503_710_720 + 591_003_648
    assert all(r.kv_cache_bytes == 2 * 80 * 4096 * 128 * 2 for r in ranks)
    assert all(r.transfer_staging_bytes == 2 * 8 * 8192 * 8 + 256 for r in ranks)
    # and the whole rank fits one B200 with room to spare
    assert all(pt.admit(r, 180 * 10**9) < 8 * 10**9 for r in ranks)


def test_plan_admission_refuses_an_oversized_context():
    p = pt.plan(LLAMA3_70B, 131072, sessions=16)
    with pytest.raises(FaberError) as e:
        pt.admit(p, 180 * 10**9)
    assert e.value.code == _lib.BUDGET_EXCEEDED


def test_plan_rejects_invalid_configs():
    bad = ModelConfig(n_layers=1, d_model=500, n_heads=4, n_kv_heads=4, head_dim=128, ffn=1024,
                      vocab=100, tied_head=True)
    with pytest.raises(FaberError) as e:
        pt.plan(bad, 64)
    assert e.value.code == _lib.UNSUPPORTED
    with pytest.raises(FaberError):
        pt.plan(TINY, 0)
    with pytest.raises(FaberError):
        pt.plan(LLAMA2_7B, 64, tp_size=3)  # heads do not divide
