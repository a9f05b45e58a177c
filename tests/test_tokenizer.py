"""The tokenizer (no GPU): Gpt2BpeTokenizer's fail-closed construction on
the reference's synthetic fact set (src/tokenizer_test.rs:30-55 and its
negative cases), and the encode pipeline on small synthetic vocabularies:
the pre-tokenizer against Python's `regex` module running the smollm split
(number codepoints alone, then the GPT-2 pattern), BPE rank order and ties,
special-token partition, byte fallback, the end-of-generation set, and
decode(encode(text)) == text.

The reference's positive probes pin ids of the SmolLM2 vocabulary, which is
not in the reference tree, so they are not reproduced here.
"""

import random

import pytest
import regex

from faber_runtime_b200 import _lib
from faber_runtime_b200 import tokenizer as tk

GPT2_PATTERN = regex.compile(r"""'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+""")


def byte_to_display():
    keep = list(range(0x21, 0x7F)) + list(range(0xA1, 0xAD)) + list(range(0xAE, 0x100))
    out, extra = {}, 0
    for b in range(256):
        if b in keep:
            out[b] = chr(b)
        else:
            out[b] = chr(256 + extra)
            extra += 1
    return out


B2D = byte_to_display()


def display(s: str) -> str:
    return "".join(B2D[b] for b in s.encode())


def smollm_words(text: str) -> list:
    """The smollm pre-tokenizer restated with `regex`: each \\p{N} codepoint
    alone, then the GPT-2 pattern over every piece between them."""
    words, cur = [], ""
    for ch in text:
        if regex.match(r"\p{N}", ch):
            if cur:
                words += GPT2_PATTERN.findall(cur)
            words.append(ch)
            cur = ""
        else:
            cur += ch
    if cur:
        words += GPT2_PATTERN.findall(cur)
    return words


def synthetic_pinned():
    """The reference's minimal valid fact set (exact pinned counts)."""
    return tk.TokenizerFacts(tokens=[f"tok{i}" for i in range(tk.PINNED_VOCAB)],
                             token_types=[tk.NORMAL] * tk.PINNED_VOCAB, merges=["a b"] * tk.PINNED_MERGES)


def refused(facts, kind):
    with pytest.raises(tk.TokenizerError) as e:
        tk.Tokenizer(facts)
    assert e.value.kind == kind and e.value.code == _lib.INVALID_ARGUMENT, e.value
    return e.value


# --- fail-closed construction ----------------------------------------------------------

def test_synthetic_pinned_facts_construct():
    t = tk.Tokenizer(synthetic_pinned())
    assert t.vocab_size == tk.PINNED_VOCAB
    assert (t.bos_token_id, t.eos_token_id, t.pad_token_id, t.unk_token_id) == (1, 2, 2, 0)
    assert t.eog_tokens == [2]  # no end-of-turn texts: eos alone


@pytest.mark.parametrize("mutate,kind", [
    (lambda f: setattr(f, "model", "llama"), "UnsupportedModel"),
    (lambda f: setattr(f, "pre", "gpt2"), "UnsupportedPreTokenizer"),
    (lambda f: (setattr(f, "tokens", ["a"] * 10), setattr(f, "token_types", [1] * 10)), "VocabSizeMismatch"),
    (lambda f: setattr(f, "merges", ["a b"] * 100), "MergesCountMismatch"),
    (lambda f: setattr(f, "token_types", [1] * 5), "TokenTypeCountMismatch"),
    (lambda f: setattr(f, "scores_present", True), "ScoresPresent"),
    (lambda f: f.merges.__setitem__(0, "no-separator"), "MalformedMergeString"),
    (lambda f: f.merges.__setitem__(7, " ab"), "MalformedMergeString"),
    (lambda f: f.merges.__setitem__(9, "ab "), "MalformedMergeString"),
    (lambda f: f.tokens.__setitem__(0, "has space"), "ByteBoundaryViolation"),
    (lambda f: f.tokens.__setitem__(0, ""), "ByteBoundaryViolation"),
    (lambda f: f.tokens.__setitem__(3, "x" * 4097), "ByteBoundaryViolation"),
    (lambda f: setattr(f, "bos_token_id", tk.PINNED_VOCAB), "TokenIdOutOfRange"),
    (lambda f: setattr(f, "unk_token_id", 1 << 31), "TokenIdOutOfRange"),
    (lambda f: setattr(f, "add_bos_token", True), "AddBosTokenNotSupported"),
    (lambda f: setattr(f, "add_space_prefix", True), "AddSpacePrefixNotSupported"),
])
def test_construction_refuses(mutate, kind):
    f = synthetic_pinned()
    mutate(f)
    refused(f, kind)


def test_checks_run_in_the_reference_order():
    f = synthetic_pinned()
    f.model, f.scores_present, f.add_bos_token = "llama", True, True
    refused(f, "UnsupportedModel")
    f = synthetic_pinned()
    f.scores_present, f.add_bos_token = True, True
    refused(f, "ScoresPresent")
    f = synthetic_pinned()
    f.tokens[0], f.merges[0] = "", "bad"
    refused(f, "ByteBoundaryViolation")  # tokens before merges


def test_encode_input_ceiling_and_invalid_utf8():
    t = tk.Tokenizer(synthetic_pinned())
    with pytest.raises(tk.TokenizerError) as e:
        t.encode("a" * ((1 << 20) + 1))
    assert e.value.kind == "InputTooLarge"
    with pytest.raises(tk.TokenizerError) as e:
        t.encode(b"ok\xff")
    assert e.value.kind == "InvalidUtf8"
    assert t.encode("") == []


# --- encode on synthetic vocabularies -----------------------------------------------------

SPECIALS = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]


def build(words=(), extra_merges=(), drop=(), specials=SPECIALS, user_defined=()):
    """A vocabulary: the 256 byte display characters, every substring of
    each display word with a merge for every split of it (so any two
    adjacent symbols inside a word merge, whatever the rank order, and each
    word ends as one token), then the specials (control) and user-defined
    texts."""
    tokens = [B2D[b] for b in range(256) if B2D[b] not in drop]
    merges = list(extra_merges)
    seen, seen_merges = set(tokens), set(merges)
    for w in words:
        d = display(w)
        for i in range(len(d)):
            for j in range(i + 2, len(d) + 1):
                sub = d[i:j]
                if sub not in seen:
                    tokens.append(sub)
                    seen.add(sub)
                for k in range(1, len(sub)):
                    m = f"{sub[:k]} {sub[k:]}"
                    if m not in seen_merges:
                        merges.append(m)
                        seen_merges.add(m)
    types = [tk.NORMAL] * len(tokens)
    for s in specials:
        tokens.append(s)
        types.append(tk.CONTROL)
    for s in user_defined:
        tokens.append(s)
        types.append(tk.USER_DEFINED)
    eos = tokens.index("<|im_end|>") if "<|im_end|>" in tokens else 2
    f = tk.TokenizerFacts(tokens=tokens, token_types=types, merges=merges, bos_token_id=1, eos_token_id=eos,
                          pad_token_id=eos, unk_token_id=0, expected_vocab=len(tokens),
                          expected_merges=len(merges))
    return tk.Tokenizer(f), tokens


TEXTS = [
    "Hello world",
    "The quick brown fox jumps over the lazy dog.",
    "it's they're we've I'm we'll he'd don't IT'S",
    "  leading spaces, trailing   \n\n  and\ttabs\t\tmixed  ",
    "numbers 12345 and 3.14159, 1,000,000; x2y3",
    "punctuation!!! ...?? (brackets) [x] {y} <z> @#$%^&*",
    "naïve café — “quotes” über straße 東京 😀 emoji",
    "line one\nline two\r\nline three\n",
    "mixed     spaces and　ideographic",
]


@pytest.mark.parametrize("text", TEXTS)
def test_pre_tokenizer_matches_the_regex(text):
    """With merges that collapse every expected word into one token, the
    encoding is one token per word exactly when the splits agree."""
    words = smollm_words(text)
    t, tokens = build(words)
    ids = t.encode(text, parse_special=False)
    assert [tokens[i] for i in ids] == [display(w) for w in words]


def test_random_text_round_trips_and_splits_like_the_regex():
    rng = random.Random(7)
    alphabet = "abcXYZ019 '\n\t.,!?é東😀-_ " + "sldvmtr"
    for _ in range(60):
        text = "".join(rng.choice(alphabet) for _ in range(rng.randint(1, 40)))
        words = smollm_words(text)
        t, tokens = build(words)
        ids = t.encode(text, parse_special=False)
        assert [tokens[i] for i in ids] == [display(w) for w in words], repr(text)
        assert t.decode(ids) == text.encode()


def test_bpe_lowest_rank_first_and_leftmost_ties():
    t, tok = build(extra_merges=["a b", "b c"])
    toks = tok + []
    assert [toks[i] for i in t.encode("abc")] == ["a", "b", "c"]  # "ab"/"bc" are not tokens: byte fallback
    # with the merged texts as tokens: rank 0 ("a b") wins over "b c"
    f_tokens = [B2D[b] for b in range(256)] + ["ab", "bc"]
    for merges, want in ((["a b", "b c"], ["ab", "c"]), (["b c", "a b"], ["a", "bc"]),
                         (["a a"], ["aa", "a"])):
        f = tk.TokenizerFacts(tokens=f_tokens + (["aa"] if "a a" in merges else []),
                              token_types=[1] * (len(f_tokens) + ("a a" in merges)), merges=merges,
                              bos_token_id=0, eos_token_id=0, pad_token_id=0, unk_token_id=0,
                              expected_vocab=len(f_tokens) + ("a a" in merges), expected_merges=len(merges))
        tt = tk.Tokenizer(f)
        text = "aaa" if merges == ["a a"] else "abc"
        assert [f.tokens[i] for i in tt.encode(text)] == want, merges


def test_digits_are_split_one_by_one():
    t, tok = build(words=["12", "123"])  # merges exist, but digits never share a word
    assert [tok[i] for i in t.encode("12345")] == list("12345")
    assert [tok[i] for i in t.encode(" 7x")] == ["Ġ", "7", "x"]


def test_special_tokens_partition_only_when_parsed():
    t, tok = build(words=["x", "y"])
    end, start = tok.index("<|im_end|>"), tok.index("<|im_start|>")
    assert t.encode("x<|im_end|>y") == [tok.index("x"), end, tok.index("y")]
    assert t.encode("<|im_start|><|im_end|>") == [start, end]
    plain = t.encode("x<|im_end|>y", parse_special=False)
    assert end not in plain and t.decode(plain) == b"x<|im_end|>y"
    # user-defined texts partition even without parse_special
    t2, tok2 = build(user_defined=["<sep>"])
    assert tok2.index("<sep>") in t2.encode("a<sep>b", parse_special=False)


def test_longest_special_text_wins():
    t, tok = build(specials=["<|im_end|>", "<|im_end|>x"])
    assert t.encode("<|im_end|>x") == [tok.index("<|im_end|>x")]


def test_byte_fallback_and_unmapped_bytes():
    t, tok = build(drop=["z"])
    assert t.encode("z") == []  # no token and no single-byte fallback: dropped
    # a merge whose result is not a token falls back to its ASCII bytes
    f_tokens = [B2D[b] for b in range(256)]
    f = tk.TokenizerFacts(tokens=f_tokens, token_types=[1] * 256, merges=["x y"], bos_token_id=0,
                          eos_token_id=0, pad_token_id=0, unk_token_id=0, expected_vocab=256, expected_merges=1)
    tt = tk.Tokenizer(f)
    assert [f_tokens[i] for i in tt.encode("xy")] == ["x", "y"]


def test_end_of_generation_set():
    t, tok = build()
    assert sorted(t.eog_tokens) == sorted([tok.index("<|endoftext|>"), tok.index("<|im_end|>")])


def test_unicode_heavy_random_text_splits_like_the_regex():
    """Other whitespace (no-break, em, ideographic space, CR, VT), numbers of
    other scripts and letter-like numerals, combining marks, contractions in
    odd places."""
    rng = random.Random(11)
    alphabet = ["a", "Z", "ß", "é", "é", "東", "한", "ع", "٣", "Ⅻ", "²", "5", " ", "  ", " ", " ",
                "　", "\r", "\x0b", "\n", "'s", "'re", "'ll", "'S", "'", "!", "—", "😀", "​", "_", "$"]
    for _ in range(150):
        text = "".join(rng.choice(alphabet) for _ in range(rng.randint(1, 24)))
        words = smollm_words(text)
        t, tokens = build(words)
        ids = t.encode(text, parse_special=False)
        assert [tokens[i] for i in ids] == [display(w) for w in words], repr(text)
        assert t.decode(ids) == text.encode()


# --- facts from a GGUF file ----------------------------------------------------------------

def test_facts_from_gguf_build_the_same_tokenizer():
    from faber_runtime_b200.gguf import GgufFile
    from test_gguf import ARRAY, BOOL, I32, STRING, U32, write_gguf
    words = smollm_words("Hello world, it's 42!")
    t_ref, tokens = build(words)
    ref = t_ref.encode("Hello world, it's 42! <|im_end|>")
    d = {n: getattr(t_ref, n) for n in ("bos_token_id", "eos_token_id", "pad_token_id", "unk_token_id")}
    # the same facts as build() made, written as GGUF metadata
    types = [tk.NORMAL] * (len(tokens) - len(SPECIALS)) + [tk.CONTROL] * len(SPECIALS)
    merges = [m for m in build_merges(words)]
    kvs = [("general.architecture", STRING, "llama"),
           ("tokenizer.ggml.model", STRING, "gpt2"), ("tokenizer.ggml.pre", STRING, "smollm"),
           ("tokenizer.ggml.tokens", ARRAY, (STRING, tokens)), ("tokenizer.ggml.token_type", ARRAY, (I32, types)),
           ("tokenizer.ggml.merges", ARRAY, (STRING, merges)),
           ("tokenizer.ggml.bos_token_id", U32, d["bos_token_id"]),
           ("tokenizer.ggml.eos_token_id", U32, d["eos_token_id"]),
           ("tokenizer.ggml.padding_token_id", U32, d["pad_token_id"]),
           ("tokenizer.ggml.unknown_token_id", U32, d["unk_token_id"]),
           ("tokenizer.ggml.add_bos_token", BOOL, 0), ("tokenizer.ggml.add_space_prefix", BOOL, 0)]
    g = GgufFile(write_gguf(kvs, []))
    t = tk.from_gguf(g, expected_vocab=len(tokens), expected_merges=len(merges))
    assert t.encode("Hello world, it's 42! <|im_end|>") == ref
    assert t.eog_tokens == t_ref.eog_tokens
    # the pinned counts refuse this small vocabulary, and scores are refused
    with pytest.raises(tk.TokenizerError) as e:
        tk.from_gguf(g)
    assert e.value.kind == "VocabSizeMismatch"
    from test_gguf import F32
    g2 = GgufFile(write_gguf(kvs + [("tokenizer.ggml.scores", ARRAY, (F32, [0.0] * len(tokens)))], []))
    with pytest.raises(tk.TokenizerError) as e:
        tk.from_gguf(g2, expected_vocab=len(tokens), expected_merges=len(merges))
    assert e.value.kind == "ScoresPresent"
    g3 = GgufFile(write_gguf([kv for kv in kvs if kv[0] != "tokenizer.ggml.merges"], []))
    with pytest.raises(tk.TokenizerError) as e:
        tk.from_gguf(g3, expected_vocab=len(tokens), expected_merges=len(merges))
    assert e.value.kind == "MissingMetadataKey"


def build_merges(words):
    seen, out = set(), []
    for w in words:
        d = display(w)
        for i in range(len(d)):
            for j in range(i + 2, len(d) + 1):
                sub = d[i:j]
                for k in range(1, len(sub)):
                    m = f"{sub[:k]} {sub[k:]}"
                    if m not in seen:
                        seen.add(m)
                        out.append(m)
    return out
