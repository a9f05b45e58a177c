"""CPU-side checks of the C ABI library and host logic (no GPU calls)."""

import ctypes
import re

import numpy as np
import pytest

from conftest import GOLDEN, ROOT


def header_symbols():
    text = (ROOT / "include" / "faber_gpu.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b((?:__faber_gpu_v1_|faber_gpu_v2_|faber_synth_)\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol(faber):
    syms = header_symbols()
    assert len(syms) >= 35
    L = faber.lib()
    for s in syms:
        assert hasattr(L, s), s
    from faber_runtime_b200 import _lib
    assert set(syms) <= set(_lib.SIGNATURES), set(syms) - set(_lib.SIGNATURES)
    assert L.faber_gpu_v2_abi_version() == 2


def test_oracle_never_imported_by_product():
    for p in (ROOT / "faber_runtime_b200").rglob("*.py"):
        src = p.read_text()
        assert "import oracle" not in src and "from oracle" not in src, p
    for p in (ROOT / "faber_runtime_b200" / "csrc").iterdir():
        assert "faber_oracle" not in p.read_text(), p


def test_status_codes_and_null_pointer_rules(faber):
    from faber_runtime_b200 import _lib
    L = _lib.lib()
    # copy_in with a null pointer and a nonzero length (gpu_placement.rs:61)
    st = L.__faber_gpu_v1_copy_in(7, None, 16, 0)
    assert st.code == _lib.INVALID_ARGUMENT
    st = L.__faber_gpu_v1_readback(7, None, 0, None)
    assert st.code == _lib.INVALID_ARGUMENT
    assert "null" in _lib.last_error()
    st = L.faber_gpu_v2_dequant_q4k(None, 4, None, 0, None)
    assert st.code == _lib.INVALID_ARGUMENT


def test_fault_injection_fails_before_device_work(faber):
    from faber_runtime_b200 import _lib
    L = _lib.lib()
    L.faber_gpu_v2_fault_inject(b"faber_gpu_v2_dequant_q4k", _lib.TIMEOUT, 2)
    for _ in range(2):
        assert L.faber_gpu_v2_dequant_q4k(None, 0, None, 0, None).code == _lib.TIMEOUT
    assert L.faber_gpu_v2_dequant_q4k(None, 0, None, 0, None).code == _lib.OK
    L.faber_gpu_v2_fault_inject(b"faber_gpu_v2_session_push_token", _lib.DEVICE_LOSS, 1)
    assert L.faber_gpu_v2_session_push_token(None, 0).code == _lib.DEVICE_LOSS
    assert L.faber_gpu_v2_session_push_token(None, 0).code == _lib.INVALID_ARGUMENT


def test_kv_layout_accounting(faber):
    from faber_runtime_b200 import KvCacheLayout
    # the reference's pinned-row figure (src/kv_cache_test.rs:70-81): 1 slot x
    # ctx 8192 x 32 layers x 5 kv heads x 64 x K,V x f32 = 671 088 640 B
    lay = KvCacheLayout(1, 8192, 32, 5, 64, dtype=0)
    assert lay.total_bytes() == 671_088_640
    assert lay.device_bytes() == (671_088_640, 671_088_640)
    lay = KvCacheLayout(1, 8192, 32, 5, 64, dtype=0, reserve_bytes=4096)
    assert lay.device_bytes() == (671_088_640, 671_092_736)
    assert KvCacheLayout(1, 2048, 32, 32, 128, dtype=1).total_bytes() == 2048 * 32 * 32 * 128 * 2 * 2
    bad = KvCacheLayout(1, 0, 32, 5, 64)
    assert bad.total_bytes() is None
    with pytest.raises(faber.FaberError) as e:
        bad.device_bytes()
    assert e.value.code == 1
    huge = KvCacheLayout(2 ** 31, 2 ** 31, 2 ** 31, 1, 1, dtype=0)
    with pytest.raises(faber.FaberError) as e:
        huge.device_bytes()
    assert e.value.code == 2


def test_synth_is_deterministic_and_in_range(faber):
    from faber_runtime_b200 import synth
    import oracle as o
    a = synth.q4k_blocks(7, 3, 1000)
    b = np.concatenate([synth.q4k_blocks(7, 3, 1000)[: 144 * 500], synth.q4k_blocks(7, 3, 1000)[144 * 500:]])
    assert np.array_equal(a, b)
    assert not np.array_equal(a, synth.q4k_blocks(8, 3, 1000))
    blk = a.reshape(-1, 144)
    d = o.half_to_f32_array(blk[:, 0:2].copy().view(np.uint16).reshape(-1))
    dm = o.half_to_f32_array(blk[:, 2:4].copy().view(np.uint16).reshape(-1))
    for v in (d, dm):
        assert v.min() >= 0.00099 and v.max() <= 0.02001
    q = np.concatenate([blk[:, 16:] & 15, blk[:, 16:] >> 4]).reshape(-1)
    assert set(np.unique(q)) == set(range(16))
    x = synth.normal(1, 2, 100000)
    assert abs(x.mean()) < 0.02 and abs(x.std() - 1) < 0.02
    t = synth.tokens(1, 3, 10000, 32000)
    assert t.min() >= 0 and t.max() < 32000


def test_compare_gpu_logits_harness_on_reference_golden(faber):
    from faber_runtime_b200 import compare_gpu_logits
    lg = np.load(GOLDEN / "logits_pos0.npz")["raw_logits"]
    v = compare_gpu_logits(lg, lg)
    assert v.ok and v.divergence_field() == "none" and v.gpu_top1 == 30
    p = lg.copy()
    p[5] += 1e-3
    v = compare_gpu_logits(p, lg)
    assert not v.ok and v.failing_thresholds == ["band"] and v.top1_matches
    p = lg.copy()
    p[2] = 1e6  # an EOG id never wins the top-1 surface
    assert compare_gpu_logits(p, lg, rms_tol=1e9).top1_matches
    p[7] = 1e6
    v = compare_gpu_logits(p, lg)
    assert "top-1" in v.failing_thresholds and v.gpu_top1 == 7
    p = lg.copy()
    p[9] = np.nan
    v = compare_gpu_logits(p, lg)
    assert "finite" in v.failing_thresholds
    assert compare_gpu_logits(lg * (1 + 1e-6), lg, rms_tol=1e-3).ok


def test_model_config_byte_accounting(faber):
    from faber_runtime_b200 import LLAMA2_7B, LLAMA3_70B
    # 7B-shape linears: 6.476e9 weights x 144/256 B
    assert LLAMA2_7B.linear_bytes() == 3_642_753_024
    assert LLAMA2_7B.head_bytes() == 73_728_000
    assert LLAMA3_70B.linear_bytes() == 38_503_710_720
    assert LLAMA3_70B.head_bytes() == 591_003_648


def test_upload_fail_closed_matrix_on_the_host(faber):
    """The dequant fail-closed matrix (src/dequant_test.rs:423-574,775-839)
    at the C ABI: exact byte lengths, whole blocks, known types and non-null
    buffers are checked on the host before any device work, so every
    refusal here is INVALID_ARGUMENT with no GPU present."""
    import ctypes

    import numpy as np
    from faber_runtime_b200 import _lib
    L = _lib.lib()
    out = ctypes.c_void_p()
    ok = np.zeros(144, np.uint8)
    for nbytes, rows, cols in [(143, 1, 256), (145, 1, 256), (0, 1, 256), (288, 1, 256),  # byte lengths
                               (144, 0, 256), (144, 1, 0), (144, 1, 128),                  # shapes
                               (144 * 3, 3, 255)]:                                        # not whole blocks
        buf = np.zeros(max(nbytes, 1), np.uint8)
        st = L.faber_gpu_v2_q4k_upload(buf.ctypes.data, nbytes, rows, cols, ctypes.byref(out))
        assert st.code == _lib.INVALID_ARGUMENT, (nbytes, rows, cols)
    assert L.faber_gpu_v2_q4k_upload(None, 144, 1, 256, ctypes.byref(out)).code == _lib.INVALID_ARGUMENT
    assert L.faber_gpu_v2_q4k_upload(ok.ctypes.data, 144, 1, 256, None).code == _lib.INVALID_ARGUMENT
    # typed rows: per type the exact bytes of whole blocks (Q8_0 34 B / 32, Q5_0 22 B / 32, Q6_K 210 B / 256)
    for gtype, be, bb in [(8, 32, 34), (6, 32, 22), (14, 256, 210)]:
        good = 2 * (64 // be if be == 32 else 1) * bb
        cols = 64 if be == 32 else 256
        for nbytes in (good - 1, good + 1, 0):
            buf = np.zeros(max(nbytes, 1), np.uint8)
            st = L.faber_gpu_v2_typed_upload(gtype, buf.ctypes.data, nbytes, 2, cols, ctypes.byref(out))
            assert st.code == _lib.INVALID_ARGUMENT, (gtype, nbytes)
        st = L.faber_gpu_v2_typed_upload(gtype, ok.ctypes.data, good, 2, cols + 1, ctypes.byref(out))
        assert st.code == _lib.INVALID_ARGUMENT  # ragged rows
    for bad_type in (2, 3, 10, 13, 99):  # Q4_0, Q4_1, Q2_K, Q5_K, unknown: not admitted
        assert L.faber_gpu_v2_typed_upload(bad_type, ok.ctypes.data, 144, 1, 256,
                                           ctypes.byref(out)).code == _lib.INVALID_ARGUMENT
        assert L.faber_gpu_v2_dequant_blocks(bad_type, ok.ctypes.data, 1, None, 1,
                                             None).code == _lib.INVALID_ARGUMENT
    assert L.faber_gpu_v2_dequant_blocks(12, None, 1, None, 1, None).code == _lib.INVALID_ARGUMENT
