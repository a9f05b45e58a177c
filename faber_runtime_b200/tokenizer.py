"""Text in, token ids out: the GPT-2 byte-level BPE tokenizer with the
`smollm` pre-tokenizer of src/tokenizer (Gpt2BpeTokenizer), through the
library's C ABI.

``TokenizerFacts`` are the GGUF's tokenizer.ggml.* metadata
(src/tokenizer/mod.rs:254-280); ``Tokenizer`` checks them fail-closed the
way Gpt2BpeTokenizer::new does, and raises ``TokenizerError`` whose
``kind`` is the reference's TokenizerError variant. ``from_gguf`` reads the
facts from a parsed GGUF file. The counts expected are the pinned row's
(49 152 tokens, 48 900 merges) unless stated.
"""

from __future__ import annotations

import ctypes
import re
from dataclasses import dataclass, field

import numpy as np

from . import _lib

PINNED_VOCAB, PINNED_MERGES = 49152, 48900
NORMAL, UNKNOWN, CONTROL, USER_DEFINED = 1, 2, 3, 4


class TokenizerError(_lib.FaberError):
    """A refused tokenizer call; ``kind`` is the reference's TokenizerError
    variant (UnsupportedModel, VocabSizeMismatch, InputTooLarge, ...)."""

    def __init__(self, code: int, message: str):
        super().__init__(code, message)
        m = re.search(r"(?:^|: )([A-Z][A-Za-z0-9]+): ", message)
        self.kind = m.group(1) if m else ""


@dataclass
class TokenizerFacts:
    tokens: list
    token_types: list
    merges: list
    model: str = "gpt2"
    pre: str = "smollm"
    scores_present: bool = False
    bos_token_id: int = 1
    eos_token_id: int = 2
    pad_token_id: int = 2
    unk_token_id: int = 0
    add_bos_token: bool = False
    add_space_prefix: bool = False
    expected_vocab: int = PINNED_VOCAB
    expected_merges: int = PINNED_MERGES
    _keep: list = field(default_factory=list, repr=False)


def _str_array(items):
    raw = [s.encode() if isinstance(s, str) else bytes(s) for s in items]
    ptrs = (ctypes.c_char_p * max(1, len(raw)))(*raw)
    lens = (ctypes.c_uint64 * max(1, len(raw)))(*[len(b) for b in raw])
    return raw, ptrs, lens


class Tokenizer:
    def __init__(self, facts: TokenizerFacts):
        c = _lib.TokenizerFactsC()
        c.model, c.pre = facts.model.encode(), facts.pre.encode()
        traw, tptr, tlen = _str_array(facts.tokens)
        mraw, mptr, mlen = _str_array(facts.merges)
        types = np.ascontiguousarray(facts.token_types, dtype=np.int32)
        c.tokens, c.token_lens, c.n_tokens = ctypes.addressof(tptr), ctypes.addressof(tlen), len(traw)
        c.token_types, c.n_token_types = types.ctypes.data if types.size else None, types.size
        c.merges, c.merge_lens, c.n_merges = ctypes.addressof(mptr), ctypes.addressof(mlen), len(mraw)
        c.scores_present = int(facts.scores_present)
        c.bos_token_id, c.eos_token_id = facts.bos_token_id, facts.eos_token_id
        c.pad_token_id, c.unk_token_id = facts.pad_token_id, facts.unk_token_id
        c.add_bos_token, c.add_space_prefix = int(facts.add_bos_token), int(facts.add_space_prefix)
        c.expected_vocab, c.expected_merges = facts.expected_vocab, facts.expected_merges
        h = ctypes.c_void_p()
        try:
            _lib.call("faber_gpu_v2_tokenizer_create", ctypes.byref(c), ctypes.byref(h))
        except _lib.FaberError as e:
            raise TokenizerError(e.code, e.message) from None
        self._h = h
        vocab, n_eog = _lib.U64(), _lib.U64()
        ids = (ctypes.c_uint32 * 4)()
        eog = (ctypes.c_uint32 * 64)()
        _lib.call("faber_gpu_v2_tokenizer_info", self._h, ctypes.byref(vocab), ids, eog, 64, ctypes.byref(n_eog))
        self.vocab_size = vocab.value
        self.bos_token_id, self.eos_token_id, self.pad_token_id, self.unk_token_id = list(ids)
        self.eog_tokens = list(eog[:n_eog.value])

    def encode(self, text: str | bytes, parse_special: bool = True) -> list:
        b = text.encode() if isinstance(text, str) else bytes(text)
        cap = 2 * len(b) + 1024
        out = (ctypes.c_uint32 * cap)()
        n = _lib.U64()
        src = ctypes.create_string_buffer(b, len(b))
        try:
            _lib.call("faber_gpu_v2_tokenizer_encode", self._h, src, len(b), int(parse_special), out, cap,
                      ctypes.byref(n))
        except _lib.FaberError as e:
            raise TokenizerError(e.code, e.message) from None
        return list(out[:n.value])

    def decode(self, ids) -> bytes:
        arr = (ctypes.c_uint32 * max(1, len(ids)))(*ids)
        n = _lib.U64()
        try:
            _lib.call("faber_gpu_v2_tokenizer_decode", self._h, arr, len(ids), None, 0, ctypes.byref(n))
        except _lib.FaberError as e:
            if e.code != _lib.IO_ERROR:
                raise TokenizerError(e.code, e.message) from None
        buf = ctypes.create_string_buffer(max(1, n.value))
        _lib.call("faber_gpu_v2_tokenizer_decode", self._h, arr, len(ids), buf, n.value, ctypes.byref(n))
        return buf.raw[:n.value]

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.call("faber_gpu_v2_tokenizer_free", self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _kv_index(g, key: str) -> int:
    for i, (k, *_rest) in enumerate(g.keys):
        if k == key:
            return i
    raise TokenizerError(_lib.INVALID_ARGUMENT, f"MissingMetadataKey: {key}")


def _read_strings(g, key: str) -> list:
    i = _kv_index(g, key)
    _, ty, at, count = g.keys[i]
    if ty != 9 or at != 8:
        raise TokenizerError(_lib.INVALID_ARGUMENT, f"WrongMetadataValueType: {key}")
    off = _lib.U64()
    _lib.call("faber_gpu_v2_gguf_kv_payload", g._h, i, ctypes.byref(off))
    buf, pos, out = g.buf, off.value, []
    for _ in range(count):
        n = int(buf[pos:pos + 8].view(np.uint64)[0])
        out.append(bytes(buf[pos + 8:pos + 8 + n]).decode())
        pos += 8 + n
    return out


def _read_i32(g, key: str) -> list:
    i = _kv_index(g, key)
    _, ty, at, count = g.keys[i]
    if ty != 9 or at not in (4, 5):  # UINT32 or INT32 elements
        raise TokenizerError(_lib.INVALID_ARGUMENT, f"WrongMetadataValueType: {key}")
    off = _lib.U64()
    _lib.call("faber_gpu_v2_gguf_kv_payload", g._h, i, ctypes.byref(off))
    return g.buf[off.value:off.value + 4 * count].view(np.int32).tolist()


def facts_from_gguf(g, expected_vocab: int = PINNED_VOCAB, expected_merges: int = PINNED_MERGES) -> TokenizerFacts:
    """TokenizerFacts from a GgufFile's tokenizer.ggml.* metadata
    (Gpt2BpeTokenizer::from_admission, src/tokenizer/mod.rs:537-680)."""
    def need_int(key):
        _kv_index(g, key)
        return g.get_int(key)
    return TokenizerFacts(
        tokens=_read_strings(g, "tokenizer.ggml.tokens"), token_types=_read_i32(g, "tokenizer.ggml.token_type"),
        merges=_read_strings(g, "tokenizer.ggml.merges"), model=g.get_string("tokenizer.ggml.model"),
        pre=g.get_string("tokenizer.ggml.pre"), scores_present=g.has("tokenizer.ggml.scores"),
        bos_token_id=need_int("tokenizer.ggml.bos_token_id"), eos_token_id=need_int("tokenizer.ggml.eos_token_id"),
        pad_token_id=need_int("tokenizer.ggml.padding_token_id"),
        unk_token_id=need_int("tokenizer.ggml.unknown_token_id"),
        add_bos_token=bool(need_int("tokenizer.ggml.add_bos_token")),
        add_space_prefix=bool(need_int("tokenizer.ggml.add_space_prefix")),
        expected_vocab=expected_vocab, expected_merges=expected_merges)


def from_gguf(g, **expected) -> Tokenizer:
    return Tokenizer(facts_from_gguf(g, **expected))
