"""GPU parity of the Q4_K kernels against the CPU oracle (through the C ABI).

Bar: dequantized weights bit-exact (NaN payloads excepted, NaN positions
equal); GEMV outputs within max|gpu - oracle| <= 1e-3 x RMS(oracle).
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

RMS_TOL = 1e-3  # max-abs error <= 1e-3 x RMS of the oracle output


def within(gpu, ref, tol=RMS_TOL):
    gpu = np.asarray(gpu, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(ref ** 2))
    err = np.max(np.abs(gpu - ref)) if ref.size else 0.0
    assert np.all(np.isfinite(gpu)), "non-finite GPU output"
    assert err <= tol * rms, f"max|err| {err:.3e} > {tol} x RMS {rms:.3e}"
    return err / rms if rms else 0.0


def same_bits(gpu, ref):
    g, r = np.asarray(gpu, np.float32), np.asarray(ref, np.float32)
    gn, rn = np.isnan(g), np.isnan(r)
    assert np.array_equal(gn, rn), "NaN positions differ"
    gb, rb = g.view(np.uint32)[~gn], r.view(np.uint32)[~rn]
    bad = np.nonzero(gb != rb)[0]
    assert bad.size == 0, f"{bad.size} mismatches, first at {bad[:5]}"


def to_dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_dequant_q4k_bit_exact_4096x4096(cuda, oracle):
    from faber_runtime_b200 import dequant, synth
    blocks = synth.q4k_blocks(11, 1, 65536)
    d = to_dev(blocks)
    out = torch.empty(65536 * 256, dtype=torch.float32, device=cuda)
    ref = oracle.dequant_row(oracle.Q4_K, blocks)
    dequant.dequant_q4k(d.data_ptr(), 65536, out.data_ptr(), f16_round=False)
    torch.cuda.synchronize()
    same_bits(out.cpu().numpy(), ref)
    dequant.dequant_q4k(d.data_ptr(), 65536, out.data_ptr(), f16_round=True)
    torch.cuda.synchronize()
    same_bits(out.cpu().numpy(), oracle.f16_round(ref))


def test_dequant_q4k_adversarial_blocks(cuda, oracle):
    from faber_runtime_b200 import dequant
    rng = np.random.default_rng(5)
    specials = [0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x3C00, 0x7BFF, 0xFBFF, 0x7C00,
                0xFC00, 0x7E00, 0x7C01, 0x3555, 0x1000]
    blocks = []
    for d in specials:
        for m in specials:
            b = rng.integers(0, 256, 144, dtype=np.uint8)
            b[0:2] = np.frombuffer(np.uint16(d).tobytes(), np.uint8)
            b[2:4] = np.frombuffer(np.uint16(m).tobytes(), np.uint8)
            blocks.append(b)
    # all-zero and all-ones scale bytes
    for fill in (0x00, 0xFF):
        b = rng.integers(0, 256, 144, dtype=np.uint8)
        b[4:16] = fill
        blocks.append(b)
    blocks = np.concatenate(blocks)
    n = blocks.size // 144
    out = torch.empty(n * 256, dtype=torch.float32, device=cuda)
    dequant.dequant_q4k(to_dev(blocks).data_ptr(), n, out.data_ptr(), f16_round=False)
    torch.cuda.synchronize()
    same_bits(out.cpu().numpy(), oracle.dequant_row(oracle.Q4_K, blocks))


def test_f16_rounding_matches_oracle(cuda, oracle):
    from faber_runtime_b200 import dequant
    rng = np.random.default_rng(9)
    pats = rng.integers(0, 2 ** 32, 1 << 22, dtype=np.uint64).astype(np.uint32)
    edge = []
    for e in range(0x30, 0x4A):  # every f16 exponent band incl. subnormals and overflow
        base = np.uint32(e << 23)
        edge.append(base + np.arange(0, 1 << 13, dtype=np.uint32))
        edge.append(base + np.uint32(0x7FE000) + np.arange(0, 1 << 13, dtype=np.uint32))
    x = np.concatenate([pats, *edge]).view(np.float32)
    x = np.concatenate([x, -x])
    dx = to_dev(x)
    y = torch.empty_like(dx)
    dequant.f16_round(dx.data_ptr(), y.data_ptr(), x.size)
    torch.cuda.synchronize()
    same_bits(y.cpu().numpy(), oracle.f16_round(x))


REPACK_SHAPES = [(4096, 4096), (512, 1408), (1408, 512), (37, 256), (48, 1408), (32, 96)]


@pytest.mark.parametrize("rows,cols", REPACK_SHAPES)
def test_repacked_tensor_dequantizes_bit_exact(cuda, oracle, rows, cols):
    from faber_runtime_b200 import dequant, synth
    blocks = synth.q4k_blocks(3, rows * 7 + cols, rows * cols // 256)
    t = dequant.Q4kTensor(blocks, rows, cols)
    out = torch.full((rows * cols,), float("nan"), dtype=torch.float32, device=cuda)
    t.dequant_rows(out.data_ptr(), f16_round=True)
    torch.cuda.synchronize()
    ref = oracle.f16_round(oracle.dequant_range(oracle.Q4_K, blocks, 0, rows * cols))
    same_bits(out.cpu().numpy(), ref)
    assert t.repack_hash() == dequant.Q4kTensor(blocks, rows, cols).repack_hash()


def test_repack_rejects_bad_byte_length(cuda):
    from faber_runtime_b200 import FaberError, dequant
    with pytest.raises(FaberError) as e:
        dequant.Q4kTensor(np.zeros(143, np.uint8), 1, 256)
    assert e.value.code == 1


# 4096 rows: fewer tiles than CTA slots, every tile split between CTAs;
# 11008 rows: two whole-tile waves and a split tail; 4752 x 256 and
# 4800 x 512: one wave and a tail of fewer items than CTAs
GEMV_SHAPES = [(4096, 4096), (16, 256), (17, 512), (2 * 1408, 512), (512, 1408), (11008, 4096),
               (4096, 11008), (100, 1024), (4752, 256), (4800, 512)]


@pytest.mark.parametrize("rows,cols", GEMV_SHAPES)
def test_gemv_q4k_matches_oracle(cuda, oracle, rows, cols):
    from faber_runtime_b200 import dequant, synth
    blocks = synth.q4k_blocks(21, rows + 1000 * cols, rows * cols // 256)
    x = synth.normal(21, cols, cols)
    ref = oracle.dense_q(oracle.Q4_K, blocks, x, cols, rows, f16_round=True)
    dx = to_dev(x)
    y = torch.empty(rows, dtype=torch.float32, device=cuda)
    t = dequant.Q4kTensor(blocks, rows, cols)
    t.gemv(dx.data_ptr(), y.data_ptr())
    torch.cuda.synchronize()
    rel = within(y.cpu().numpy(), ref)
    assert rel < 1e-4  # the hi/lo split keeps ~f32 accuracy (oracle's own sum error dominates)
    if cols % 256 == 0:
        w = to_dev(blocks)
        y2 = torch.empty(rows, dtype=torch.float32, device=cuda)
        dequant.gemv_q4k(w.data_ptr(), rows, cols, dx.data_ptr(), y2.data_ptr())
        torch.cuda.synchronize()
        within(y2.cpu().numpy(), ref)


@pytest.mark.parametrize("rows,cols,batch", [
    (4096, 4096, 1),
    (4096, 4096, 3),      # one MMA column block, padding columns
    (100, 1024, 8),       # partial last tile, two column blocks
    (4096, 11008, 16),    # four column blocks, six K slabs summed in order
    (2816, 2048, 13),
])
def test_batched_gemv_matches_oracle(cuda, oracle, rows, cols, batch):
    """faber_gpu_v2_q4k_gemv_batch: each sequence's output equals the
    oracle's dense of that sequence's input (the batched decode's linear)."""
    from faber_runtime_b200 import dequant, synth
    blocks = synth.q4k_blocks(23, rows + 7 * cols, rows * cols // 256)
    xs = np.stack([synth.normal(23, 100 + b, cols) * np.float32(1.0 + b) for b in range(batch)])
    t = dequant.Q4kTensor(blocks, rows, cols)
    dx = to_dev(xs)
    y = torch.full((batch, rows), float("nan"), dtype=torch.float32, device=cuda)
    for _ in range(2):  # the second call reuses the tensor's scratch
        t.gemv_batch(dx.data_ptr(), batch, y.data_ptr())
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        for b in range(batch):
            ref = oracle.dense_q(oracle.Q4_K, blocks, xs[b], cols, rows, f16_round=True)
            assert within(got[b], ref) < 1e-4
    t.close()


@pytest.mark.parametrize("scale", [0.0, 1e-30, 1e-6, 1e8, 3e30])
def test_gemv_dynamic_range(cuda, oracle, scale):
    from faber_runtime_b200 import dequant, synth
    rows, cols = 64, 2048
    blocks = synth.q4k_blocks(4, 77, rows * cols // 256)
    x = (synth.normal(4, 78, cols) * np.float32(scale)).astype(np.float32)
    x[5] *= 1000.0  # one dominant element
    ref = oracle.dense_q(oracle.Q4_K, blocks, x, cols, rows, f16_round=True)
    dx = to_dev(x)
    y = torch.empty(rows, dtype=torch.float32, device=cuda)
    dequant.Q4kTensor(blocks, rows, cols).gemv(dx.data_ptr(), y.data_ptr())
    torch.cuda.synchronize()
    if scale == 0.0:
        assert np.all(y.cpu().numpy() == 0.0)
    else:
        within(y.cpu().numpy(), ref)


def _adversarial_q4k(rng, n_rand, rows_cols):
    """Blocks with edge-case d/dmin (subnormal, signed zero, f16 min/one) and
    scale bytes all-zero / all-ones, kept finite after f16 rounding."""
    specials = [0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x3C00, 0xBC00, 0x3555, 0x1000, 0x5000]
    n = rows_cols[0] * rows_cols[1] // 256
    blocks = rng.integers(0, 256, (n, 144), dtype=np.uint8)
    for i in range(n):
        if i < n - n_rand:
            d, m = specials[i % len(specials)], specials[(i // len(specials)) % len(specials)]
            blocks[i, 0:2] = np.frombuffer(np.uint16(d).tobytes(), np.uint8)
            blocks[i, 2:4] = np.frombuffer(np.uint16(m).tobytes(), np.uint8)
            if i % 7 == 3:
                blocks[i, 4:16] = 0xFF if (i // 7) % 2 else 0x00
        else:
            blocks[i, 0:4] = np.frombuffer(np.float16([0.01, 0.003]).tobytes(), np.uint8)
    return blocks.reshape(-1)


@pytest.mark.parametrize("rows,cols", [(32, 512), (48, 1408)])
def test_gemv_weights_bit_exact_one_hot(cuda, oracle, rows, cols):
    """y = W e_j returns column j of the f16-rounded dequantized weight to the
    bit: the weights the GEMV forms in registers (never stored) are exactly
    the oracle's. Every column of a plain (512) and an offset-class (1408)
    shape is probed, with adversarial block headers."""
    from faber_runtime_b200 import dequant
    rng = np.random.default_rng(rows + cols)
    blocks = _adversarial_q4k(rng, 8, (rows, cols))
    w = oracle.f16_round(oracle.dequant_range(oracle.Q4_K, blocks, 0, rows * cols)).reshape(rows, cols)
    assert np.all(np.isfinite(w))
    t = dequant.Q4kTensor(blocks, rows, cols)
    x = torch.zeros(cols, dtype=torch.float32, device=cuda)
    ys = torch.empty((cols, rows), dtype=torch.float32, device=cuda)
    for j in range(cols):
        x.zero_()
        x[j] = 1.0
        t.gemv(x.data_ptr(), ys[j].data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    got = ys.cpu().numpy().T
    bad = np.argwhere(got != w)
    assert bad.size == 0, f"{len(bad)} weights differ, first (row, col) {bad[:4].tolist()}"


def test_placement_abi_round_trip(cuda):
    from faber_runtime_b200 import FaberError, dequant
    data = np.arange(1000, dtype=np.uint8)
    dequant.copy_in(42, data)
    assert dequant.readback(42, 1000) == data.tobytes()
    ptr, n = dequant.device_ptr(42)
    assert ptr != 0 and n == 1000
    with pytest.raises(FaberError) as e:
        dequant.readback(42, 999)
    assert e.value.code == 2
    with pytest.raises(FaberError) as e:
        dequant.readback(4242, 10)
    assert e.value.code == 1
    dequant.copy_in(42, b"")  # replaces with an empty buffer
    assert dequant.readback(42, 10) == b""
    dequant.sync(42)


@pytest.mark.parametrize("gtype", [6, 8, 14])  # Q5_0, Q8_0, Q6_K
def test_dequant_other_block_types_bit_exact(cuda, oracle, gtype):
    """dequant_q5_0 / dequant_q8_0 / dequant_q6_k (src/dequant.rs:151-255)
    on the GPU equal the oracle's to the bit, raw and f16-rounded, over random
    blocks whose f16 scale runs through the special values."""
    from faber_runtime_b200 import dequant
    bb, be, at = {6: (22, 32, 0), 8: (34, 32, 0), 14: (210, 256, 208)}[gtype]
    rng = np.random.default_rng(gtype)
    n = 4096
    blocks = rng.integers(0, 256, (n, bb), dtype=np.uint8)
    specials = [0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x3C00, 0xBC00, 0x3555, 0x1000, 0x5000, 0x7BFF]
    for i in range(n):
        v = specials[i % len(specials)] if i < 8 * len(specials) else int(rng.integers(0x1000, 0x2400))
        blocks[i, at:at + 2] = np.frombuffer(np.uint16(v).tobytes(), np.uint8)
    blocks = blocks.reshape(-1)
    d = to_dev(blocks)
    out = torch.empty(n * be, dtype=torch.float32, device=cuda)
    ref = oracle.dequant_row(gtype, blocks)
    dequant.dequant_blocks(gtype, d.data_ptr(), n, out.data_ptr(), f16_round=False)
    torch.cuda.synchronize()
    same_bits(out.cpu().numpy(), ref)
    dequant.dequant_blocks(gtype, d.data_ptr(), n, out.data_ptr(), f16_round=True)
    torch.cuda.synchronize()
    same_bits(out.cpu().numpy(), oracle.f16_round(ref))


TYPED_SHAPES = [(14, 4096, 4096), (14, 64, 11008), (8, 300, 1536), (6, 100, 512), (12, 33, 1024)]


@pytest.mark.parametrize("gtype,rows,cols", TYPED_SHAPES)
def test_typed_row_gemv_matches_oracle(cuda, oracle, gtype, rows, cols):
    """The row GEMV (Q6_K, Q8_0, Q5_0 and Q4_K rows) against the oracle's
    dense with f16-rounded weights: within 1e-4 x RMS (f32 sums in another
    order), including ragged tiles (rows not a multiple of 16)."""
    from faber_runtime_b200 import dequant, synth
    be, bb, at = {6: (32, 22, 0), 8: (32, 34, 0), 12: (256, 144, 0), 14: (256, 210, 208)}[gtype]
    n = rows * cols // be
    if gtype == 12:
        blocks = synth.q4k_blocks(31, rows + cols, n)
    else:
        rng = np.random.default_rng(rows * 7 + cols)
        b = rng.integers(0, 256, (n, bb), dtype=np.uint8)
        b[:, at:at + 2] = rng.uniform(1e-3, 2e-2, n).astype(np.float16).view(np.uint8).reshape(n, 2)
        blocks = b.reshape(-1)
    x = synth.normal(31, cols, cols)
    ref = oracle.dense_q(gtype, blocks, x, cols, rows, f16_round=True)
    t = dequant.TypedTensor(gtype, blocks, rows, cols)
    y = torch.full((rows,), float("nan"), dtype=torch.float32, device=cuda)
    t.gemv(to_dev(x).data_ptr(), y.data_ptr())
    torch.cuda.synchronize()
    assert within(y.cpu().numpy(), ref) < 1e-4
    t.close()
