"""GGUF v3 reader (faber_gpu_v2_gguf_*) and the llama loader.

A small writer below produces GGUF v3 files the way the format lays them out
(header, KVs, tensor infos, aligned data). The CPU tests check that the
reader returns exactly what was written, and that each structural check of
src/gguf.rs:581-812 fails closed: INVALID_ARGUMENT with the reference's
AdmissionError kind in the message. The GPU test loads a written file as a
model and decodes it token-identically with the CPU oracle built from the
same tensors.
"""

import struct

import numpy as np
import pytest

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f",
          BOOL: "<B", U64: "<Q", I64: "<q", F64: "<d"}
BLOCK = {0: (1, 4), 1: (1, 2), 6: (32, 22), 8: (32, 34), 12: (256, 144), 14: (256, 210)}


def _str(s) -> bytes:
    b = s if isinstance(s, bytes) else s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(ty, v) -> bytes:
    if ty == STRING:
        return _str(v)
    if ty == ARRAY:
        et, items = v
        out = struct.pack("<IQ", et, len(items))
        for it in items:
            out += _value(et, it)
        return out
    if ty not in SCALAR:
        return b""  # an unknown value type: no payload
    return struct.pack(SCALAR[ty], v)


def write_gguf(kvs, tensors, alignment=32, version=3, magic=b"GGUF", offsets=None, dims_override=None):
    """kvs: [(key, type, value)]; tensors: [(name, ggml_type, dims, bytes)]."""
    out = bytearray(magic + struct.pack("<IQQ", version, len(tensors), len(kvs)))
    for key, ty, v in kvs:
        out += _str(key) + struct.pack("<I", ty) + _value(ty, v)
    rel, data = [], bytearray()
    for name, ty, dims, raw in tensors:
        pad = (-len(data)) % alignment
        data += b"\0" * pad
        rel.append(len(data))
        data += raw
    if offsets is not None:
        rel = offsets
    for i, (name, ty, dims, raw) in enumerate(tensors):
        d = dims_override[i] if dims_override and i in dims_override else dims
        out += _str(name) + struct.pack("<I", len(d)) + b"".join(struct.pack("<Q", x) for x in d)
        out += struct.pack("<IQ", ty, rel[i])
    out += b"\0" * ((-len(out)) % alignment)
    return bytes(out + data)


def _cfg():
    from faber_runtime_b200 import ModelConfig
    return ModelConfig(n_layers=1, d_model=512, n_heads=8, n_kv_heads=4, head_dim=64, ffn=1536,
                       vocab=4096, tied_head=False, rope_theta=10000.0, rms_eps=1e-5, name="gguf-test")


def llama_file(seed=3):
    """A llama GGUF of the test config from the seeded synthetic tensors."""
    from faber_runtime_b200 import synth
    cfg = _cfg()
    tensors = []
    for name, ty, arr, rows, cols in synth.model_tensors(cfg, seed, norms="random"):
        dims = [rows] if cols == 1 else [cols, rows]
        tensors.append((name + ".weight", ty, dims, np.ascontiguousarray(arr).tobytes()))
    kvs = [("general.architecture", STRING, "llama"),
           ("general.name", STRING, "gguf-test"),
           ("llama.block_count", U32, cfg.n_layers),
           ("llama.embedding_length", U32, cfg.d_model),
           ("llama.attention.head_count", U32, cfg.n_heads),
           ("llama.attention.head_count_kv", U32, cfg.n_kv_heads),
           ("llama.feed_forward_length", U32, cfg.ffn),
           ("llama.attention.layer_norm_rms_epsilon", F32, cfg.rms_eps),
           ("llama.rope.freq_base", F32, cfg.rope_theta),
           ("tokenizer.ggml.tokens", ARRAY, (STRING, ["<s>", "é", "токен", "▁a"])),
           ("tokenizer.ggml.scores", ARRAY, (F32, [0.0, -1.5, 2.25, 3.0])),
           ("tokenizer.ggml.add_bos_token", BOOL, 1)]
    return cfg, kvs, tensors


def test_reader_returns_what_was_written(faber):
    from faber_runtime_b200 import gguf
    cfg, kvs, tensors = llama_file()
    blob = write_gguf(kvs, tensors)
    g = gguf.GgufFile(blob)
    assert g.version == 3 and g.alignment == 32 and g.data_offset % 32 == 0
    assert [k for k, *_ in g.keys] == [k for k, _, _ in kvs]
    assert g.get_string("general.architecture") == "llama"
    assert g.get_int("llama.block_count") == 1
    assert g.get_int("tokenizer.ggml.add_bos_token") == 1
    assert g.get_float("llama.attention.layer_norm_rms_epsilon") == np.float32(1e-5)
    tok = [x for x in g.keys if x[0] == "tokenizer.ggml.tokens"][0]
    assert tok[1:] == (ARRAY, STRING, 4)
    assert list(g.tensors) == [t[0] for t in tensors]
    for name, ty, dims, raw in tensors:
        t = g.tensors[name]
        assert t.ggml_type == ty and list(t.dims) == dims and t.nbytes == len(raw)
        assert t.offset % 32 == 0
        assert g.tensor_bytes(name).tobytes() == raw
    c = gguf.llama_config(g)
    assert (c.n_layers, c.d_model, c.n_heads, c.n_kv_heads, c.head_dim, c.ffn, c.vocab, c.tied_head) == \
        (cfg.n_layers, cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab, False)
    assert np.float32(c.rms_eps) == np.float32(cfg.rms_eps) and c.rope_theta == cfg.rope_theta
    g.close()


def test_alignment_override_and_file_path(faber, tmp_path):
    from faber_runtime_b200 import gguf
    _, kvs, tensors = llama_file()
    blob = write_gguf(kvs + [("general.alignment", U32, 64)], tensors, alignment=64)
    p = tmp_path / "m.gguf"
    p.write_bytes(blob)
    g = gguf.GgufFile(p)
    assert g.alignment == 64 and all(t.offset % 64 == 0 for t in g.tensors.values())
    g.close()


def _fails(blob, *kinds):
    from faber_runtime_b200 import FaberError, gguf
    with pytest.raises(FaberError) as e:
        gguf.GgufFile(blob)
    assert e.value.code == 1 and any(k in str(e.value) for k in kinds), str(e.value)


def _small():
    t = [("a.weight", 0, [8], np.arange(8, dtype=np.float32).tobytes()),
         ("b.weight", 12, [256, 2], bytes(288))]
    return [("general.architecture", STRING, "llama")], t


def test_fail_closed_container(faber):
    kvs, t = _small()
    good = write_gguf(kvs, t)
    _fails(write_gguf(kvs, t, magic=b"GGUX"), "InvalidMagic")
    _fails(write_gguf(kvs, t, version=2), "UnsupportedVersion")
    _fails(b"", "TruncatedFile")
    for cut in (3, 12, 30, 60, len(good) - 300, len(good) - 1):
        # a cut header may first show as counts that cannot fit
        _fails(good[:cut], "Truncated", "CountMismatch")
    huge_kv = bytearray(good)
    huge_kv[16:24] = struct.pack("<Q", 1 << 40)
    _fails(bytes(huge_kv), "MetadataKvCountMismatch")
    huge_t = bytearray(good)
    huge_t[8:16] = struct.pack("<Q", 1 << 40)
    _fails(bytes(huge_t), "TensorCountMismatch")


def test_fail_closed_metadata(faber):
    kvs, t = _small()
    _fails(write_gguf(kvs + [("general.architecture", STRING, "x")], t), "DuplicateMetadataKey")
    _fails(write_gguf(kvs + [("k" * 1025, U32, 1)], t), "KeyTooLong")
    _fails(write_gguf(kvs + [(b"\xff\xfe", U32, 1)], t), "InvalidUtf8")
    _fails(write_gguf(kvs + [("s", STRING, b"\xc0\x80")], t), "InvalidUtf8")  # overlong NUL
    _fails(write_gguf(kvs + [("b", BOOL, 2)], t), "MalformedBool")
    _fails(write_gguf(kvs + [("b", ARRAY, (BOOL, [0, 1, 3]))], t), "MalformedBool")
    _fails(write_gguf(kvs + [("n", ARRAY, (ARRAY, []))], t), "MetadataValueMismatch")
    _fails(write_gguf(kvs + [("v", 13, 0)], t), "MetadataValueMismatch")
    _fails(write_gguf(kvs + [("general.alignment", U32, 48)], t), "MetadataValueMismatch")


def test_fail_closed_tensors(faber):
    kvs, t = _small()
    _fails(write_gguf(kvs, t + [("a.weight", 0, [4], bytes(16))]), "DuplicateTensorName")
    _fails(write_gguf(kvs, [("x" * 1025, 0, [1], bytes(4))]), "TensorNameTooLong")
    _fails(write_gguf(kvs, [("q", 2, [32], bytes(18))]), "UnknownDtype")  # Q4_0 is not admitted
    _fails(write_gguf(kvs, t, dims_override={0: []}), "TensorDimCountMismatch")
    _fails(write_gguf(kvs, t, dims_override={0: [1, 1, 1, 1, 8]}), "TensorDimCountMismatch")
    _fails(write_gguf(kvs, t, dims_override={0: [8, 0]}), "TensorDimTooLarge")
    _fails(write_gguf(kvs, t, dims_override={0: [1 << 40, 1 << 40]}), "ArithmeticOverflow")
    _fails(write_gguf(kvs, [("b.weight", 12, [100, 2], bytes(144))]), "TensorElementsNotBlockAligned")
    _fails(write_gguf(kvs, [("b.weight", 12, [128, 2], bytes(144))]), "TensorElementsNotBlockAligned")
    _fails(write_gguf(kvs, t, offsets=[0, 16]), "MisalignedTensorOffset")
    _fails(write_gguf(kvs, t, offsets=[0, 0]), "OverlappingTensorRanges")
    _fails(write_gguf(kvs, t, offsets=[0, 64]), "NonSequentialTensorOffsets")
    _fails(write_gguf(kvs, t, dims_override={1: [256, 4]}), "TruncatedTensorData")


def test_loader_refuses_unsupported_files(faber):
    from faber_runtime_b200 import FaberError, gguf
    cfg, kvs, tensors = llama_file()
    bad = [(n, ty, d, r) for n, ty, d, r in tensors]
    kvs2 = [(k, ty, ("mamba" if k == "general.architecture" else v)) for k, ty, v in kvs]
    with pytest.raises(FaberError) as e:
        gguf.llama_config(gguf.GgufFile(write_gguf(kvs2, bad)))
    assert e.value.code == 4 and "ArchitectureMismatch" in str(e.value)
    # an F16 linear parses, but the decoder takes Q4_K, Q6_K, Q5_0 and Q8_0
    i = [n for n, *_ in tensors].index("blk.0.attn_q.weight")
    n, _, d, _ = tensors[i]
    f16 = tensors[:i] + [(n, 1, d, bytes(d[0] * d[1] * 2))] + tensors[i + 1:]
    g = gguf.GgufFile(write_gguf(kvs, f16))
    with pytest.raises(FaberError) as e:
        list(gguf.model_tensors(g, gguf.llama_config(g)))
    assert e.value.code == 4 and "F16" in str(e.value)


@pytest.mark.gpu
def test_loaded_gguf_decodes_like_the_oracle(cuda, tmp_path):
    import oracle as o
    from faber_runtime_b200 import ForwardRun, gguf, synth
    cfg, kvs, tensors = llama_file(seed=5)
    p = tmp_path / "m.gguf"
    p.write_bytes(write_gguf(kvs, tensors))
    model, g = gguf.load_llama(p)
    om = o.OracleModel(cfg, {n: (t, a, r, c) for n, t, a, r, c in synth.model_tensors(cfg, 5, norms="random")})
    prompt = synth.tokens(5, 9, 20, cfg.vocab)
    ref, _, _ = om.greedy(prompt, 8, want_logits=True)
    run = ForwardRun(model, prompt, context_length=64)
    toks, fin = run.greedy(8)
    assert fin and toks.tolist() == ref.tolist()
    run.close()
    model.close()
    g.close()


def typed_blocks(rng, gtype, n_blocks, scale=1.0):
    """Random blocks of Q8_0 / Q5_0 / Q6_K; at scale 1 the weights are near
    the synthetic Q4_K ones in size."""
    from faber_runtime_b200 import gguf
    bb = {gguf.GGML_Q8_0: 34, gguf.GGML_Q5_0: 22, gguf.GGML_Q6_K: 210}[gtype]
    b = rng.integers(0, 256, (n_blocks, bb), dtype=np.uint8)
    lo, hi, at = {gguf.GGML_Q8_0: (2e-3, 1e-2, 0), gguf.GGML_Q5_0: (1e-2, 5e-2, 0),
                  gguf.GGML_Q6_K: (2e-4, 1e-3, 208)}[gtype]
    d = (rng.uniform(lo, hi, n_blocks) * scale).astype(np.float16)
    b[:, at:at + 2] = d.view(np.uint8).reshape(n_blocks, 2)
    return b.reshape(-1)


@pytest.mark.gpu
def test_mixed_type_gguf_decodes_like_the_oracle(cuda, tmp_path):
    """A Q4_K_M-like file: attn_k Q5_0, attn_v Q6_K, ffn_down Q8_0 and the head
    Q6_K in every layer; the rest Q4_K. The typed-row GEMV serves the mixed
    linears; tokens equal the oracle's and logits stay within 1e-3 x RMS.
    The prompt is short: with random weights the residual stream swings by
    orders of magnitude from token to token, and at some later positions it
    nearly cancels, where rounding-level differences exceed the bar (the
    sensitivity the trace test allows for). The row GEMV's own accuracy is
    tested per type in test_gpu_kernels.py."""
    import oracle as o
    from faber_runtime_b200 import ForwardRun, ModelConfig, gguf, synth
    cfg = ModelConfig(n_layers=2, d_model=512, n_heads=8, n_kv_heads=4, head_dim=64, ffn=1536,
                      vocab=4096, tied_head=False, rope_theta=10000.0, name="mixed")
    rng = np.random.default_rng(17)
    swap = {"blk.{}.attn_k": gguf.GGML_Q5_0, "blk.{}.attn_v": gguf.GGML_Q6_K,
            "blk.{}.ffn_down": gguf.GGML_Q8_0}
    tensors, oracle_t = [], {}
    for name, ty, arr, rows, cols in synth.model_tensors(cfg, 17, norms="random"):
        layer_key = name.replace(name.split(".")[1], "{}") if name.startswith("blk.") else name
        nt = swap.get(layer_key, gguf.GGML_Q6_K if name == "output" else None)
        if nt is not None:
            be = 32 if nt in (gguf.GGML_Q8_0, gguf.GGML_Q5_0) else 256
            ty, arr = nt, typed_blocks(rng, nt, rows * cols // be)
        oracle_t[name] = (ty, arr, rows, cols)
        dims = [rows] if cols == 1 else [cols, rows]
        tensors.append((name + ".weight", ty, dims, np.ascontiguousarray(arr).tobytes()))
    _, kvs, _ = llama_file()
    kvs = [(k, t, v) for k, t, v in kvs]
    p = tmp_path / "mixed.gguf"
    p.write_bytes(write_gguf(kvs_for(cfg, kvs), tensors))
    model, g = gguf.load_llama(p)
    om = o.OracleModel(cfg, oracle_t)
    prompt = synth.tokens(17, 2, 3, cfg.vocab)  # pushed token by token (typed rows)
    ref, ref_logits, _ = om.greedy(prompt, 3, want_logits=True)
    run = ForwardRun(model, prompt, context_length=64)
    for i in range(3):
        got = run.position_logits()
        rms = np.sqrt(np.mean(np.asarray(ref_logits[i], np.float64) ** 2))
        assert np.max(np.abs(got - ref_logits[i])) <= 1e-3 * rms
        run.push_token(int(ref[i]))
    run2 = ForwardRun(model, prompt, context_length=64)
    toks, fin = run2.greedy(3)
    assert fin and toks.tolist() == ref.tolist()
    run.close()
    run2.close()
    model.close()
    g.close()


def kvs_for(cfg, kvs):
    """The test file's llama metadata rewritten for cfg."""
    vals = {"llama.block_count": cfg.n_layers, "llama.embedding_length": cfg.d_model,
            "llama.attention.head_count": cfg.n_heads, "llama.attention.head_count_kv": cfg.n_kv_heads,
            "llama.feed_forward_length": cfg.ffn}
    return [(k, t, vals.get(k, v)) for k, t, v in kvs]
