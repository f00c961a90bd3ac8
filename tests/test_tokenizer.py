"""The tokenizer (holo_tokenize, csrc/tokenizer.cpp): a byte trie built once
from the vocabulary, against the reference's own llm_tokenize
(src/ai/llm.c:178-221, compiled into oracle/_ref) and the oracle's literal
restatement of it (ho_tokenize, oracle/holo_oracle.c), which the first pins.
Bar: identical token ids, case by case -- the longest match at each
position, the lowest index among equal strings, the byte fallback order
("<0xNN>", then the byte-level string, then unk), BOS and the max_tokens cut.
Also the GGUF vocabulary (tokenizer.ggml.*) as the reference's
load_tokenizer reads it (llm.c:61-100).  CPU only.
"""
import json
import pathlib
import sys
import time

import numpy as np
import pytest

import holo_b200 as hb
from holo_b200 import gguf

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))
import tok_cases  # noqa: E402

SEEDS = [(11, True, True), (12, True, False), (13, False, True), (14, False, False), (15, True, True)]


def cases():
    for seed, bt, bl in SEEDS:
        vocab = tok_cases.vocabulary(seed, 500, bt, bl)
        for i, text in enumerate(tok_cases.texts(seed, n=10)):
            yield seed, vocab, text, bool(i & 1)


def test_restatement_matches_reference(oracle, reference):
    n = 0
    for seed, vocab, text, add_bos in cases():
        want = reference.tokenize(vocab, 1, 0, text, add_bos=add_bos)
        got = oracle.tokenize(vocab, 1, 0, text, add_bos=add_bos)
        assert np.array_equal(got, want), (seed, text)
        n += len(want)
    assert n > 1000


def test_trie_matches_reference(reference):
    for seed, vocab, text, add_bos in cases():
        tok = hb.Tokenizer(vocab, bos=1, unk=0)
        want = reference.tokenize(vocab, 1, 0, text, add_bos=add_bos)
        assert np.array_equal(tok.encode(text, add_bos=add_bos), want), (seed, text)
        tok.close()


def test_golden_cases(oracle):
    """Fixture ids from the compiled reference (tests/golden/make_golden.py):
    the trie and the restatement reproduce them without the reference."""
    g = json.loads((HERE / "golden" / "tokenize_cases.json").read_text())
    toks = {}
    for c in g["cases"]:
        s = str(c["seed"])
        vocab = [None if t is None else bytes.fromhex(t) for t in g["vocabs"][s]]
        bos, unk = g["bos_unk"][s]
        if s not in toks:
            toks[s] = hb.Tokenizer(vocab, bos=bos, unk=unk)
        text = bytes.fromhex(c["text"])
        got = toks[s].encode(text, add_bos=c["add_bos"], max_tokens=c["max_tokens"])
        assert got.tolist() == c["ids"]
        assert oracle.tokenize(vocab, bos, unk, text, c["max_tokens"], c["add_bos"]).tolist() == c["ids"]
    assert len(g["cases"]) >= 18


def test_edge_cases(oracle):
    v = [b"<unk>", b"<s>", b"ab", b"abc", b"ab", b"", None, b"b", b"<0x7A>", b"<0x7a>", b"c\xc3", chr(0x0120).encode()]
    tok = hb.Tokenizer(v, bos=1, unk=0)

    def both(text, **kw):
        got = tok.encode(text, **kw)
        want = oracle.tokenize(v, 1, 0, text, kw.get("max_tokens"), kw.get("add_bos", False))
        assert np.array_equal(got, want), (text, kw, got, want)
        return got.tolist()

    assert both(b"abcab") == [3, 2]            # longest first; "ab" at 2, not its repeat at 4
    assert both(b"z") == [8]                   # upper-case byte token, not "<0x7a>"
    assert both(b" ") == [11]                  # byte 0x20 -> its byte-level string U+0120
    assert both(b"q") == [0]                   # no token, no byte token, no byte-level string -> unk
    assert both(b"c\xc3\xa9") == [10, 0]       # a token may end inside a UTF-8 sequence
    assert both(b"", add_bos=True) == [1]
    assert both(b"ab", add_bos=True, max_tokens=0) == []
    assert both(b"ab", add_bos=True, max_tokens=1) == [1]
    assert both(b"abab", max_tokens=1) == [2]
    assert both(b"ab\x00ab") == [2]            # the text ends at its first NUL
    assert tok.lib.holo_tokenize(tok.h, None, None, 4, 0) == -1
    assert tok.lib.holo_tokenize(tok.h, b"ab", None, 4, 0) == -1
    assert tok.lib.holo_tokenize(tok.h, b"ab", None, 0, 1) == 0
    tok.close()
    # an empty vocabulary: every byte is unk
    empty = hb.Tokenizer([], bos=5, unk=3)
    assert empty.encode(b"xy", add_bos=True).tolist() == [5, 3, 3]
    assert oracle.tokenize([], 5, 3, b"xy", add_bos=True).tolist() == [5, 3, 3]


def test_large_vocabulary(oracle, reference):
    """A 32000-entry vocabulary (the 7B model's size) and a 3 KB text: the
    trie against the reference, and both timed."""
    rng = np.random.default_rng(7)
    vocab = tok_cases.vocabulary(21, 6000)
    seen = set(vocab)
    while len(vocab) < 32000:
        t = tok_cases._piece_string(rng, 2, 7)
        if t not in seen:
            seen.add(t)
            vocab.append(t)
    text = b"".join(tok_cases.texts(21, n=20, max_len=300))[:3000]
    t0 = time.perf_counter()
    want = reference.tokenize(vocab, 1, 0, text, add_bos=True)
    t_ref = time.perf_counter() - t0
    t0 = time.perf_counter()
    tok = hb.Tokenizer(vocab, bos=1, unk=0)
    t_build = time.perf_counter() - t0
    t0 = time.perf_counter()
    got = tok.encode(text, add_bos=True)
    t_ours = time.perf_counter() - t0
    tok.close()
    print(f"{len(text)} bytes, {len(want)} ids, vocab {len(vocab)}: reference llm_tokenize {t_ref * 1e3:.1f} ms, "
          f"trie {t_ours * 1e6:.0f} us (+ {t_build * 1e3:.1f} ms once to build)")
    assert np.array_equal(got, want)


def test_gguf_vocabulary(tmp_path, reference):
    """tokenizer.ggml.tokens / *_token_id read as the reference's
    load_tokenizer does (strings cut at a NUL, its default ids), and the
    tokenizer built from the file gives the reference's ids."""
    vocab = [b"" if t is None else t for t in tok_cases.vocabulary(31, 400)]
    vocab[10] = b"ab\x00cd"   # strdup keeps "ab"
    path = tmp_path / "tok.gguf"
    meta = {"general.architecture": "llama", "tokenizer.ggml.model": "llama", "tokenizer.ggml.tokens": vocab,
            "tokenizer.ggml.scores": [float(-i) for i in range(len(vocab))], "tokenizer.ggml.bos_token_id": 1,
            "tokenizer.ggml.unknown_token_id": 0}
    gguf.write(path, meta, {"t": (hb.F32, (8,), np.zeros(8, np.float32))})
    with gguf.GGUFFile(path) as g:
        v = gguf.tokenizer_vocab(g)
        tok = gguf.load_tokenizer(g)
    assert v["tokens"] == reference.gguf_tokens(path)
    assert v["tokens"][10] == b"ab"
    assert (v["bos"], v["eos"], v["pad"], v["unk"]) == (1, 2, 0, 0)   # eos and pad: the reference's defaults
    for key, want in (("bos_token_id", 1), ("unknown_token_id", 0)):
        assert reference.gguf_int(path, f"tokenizer.ggml.{key}") == want
    for text in tok_cases.texts(31, n=5):
        assert np.array_equal(tok.encode(text, add_bos=True),
                              reference.tokenize(v["tokens"], 1, 0, text, add_bos=True))
    tok.close()
    # no vocabulary: an error, as the reference's loader fails
    gguf.write(path, {"general.architecture": "llama"}, {"t": (hb.F32, (8,), np.zeros(8, np.float32))})
    with gguf.GGUFFile(path) as g, pytest.raises(ValueError, match="no vocabulary"):
        gguf.tokenizer_vocab(g)


def test_concurrent_use():
    """One tokenizer, eight threads at once (ctypes drops the GIL during the
    call): the same ids as one thread."""
    from concurrent.futures import ThreadPoolExecutor
    vocab = tok_cases.vocabulary(41, 2000)
    tok = hb.Tokenizer(vocab, bos=1, unk=0)
    texts = [t * 20 for t in tok_cases.texts(41, n=16, max_len=200)]
    want = [tok.encode(t, add_bos=True) for t in texts]
    with ThreadPoolExecutor(8) as ex:
        for _ in range(4):
            got = list(ex.map(lambda t: tok.encode(t, add_bos=True), texts))
            assert all(np.array_equal(g, w) for g, w in zip(got, want))
    tok.close()
