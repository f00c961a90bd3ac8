"""Seeded tokenizer cases -- vocabularies and texts -- shared by
tests/test_tokenizer.py and tests/golden/make_golden.py.

A vocabulary mixes what real GGUF vocabularies hold and what stresses the
greedy longest match (llm_tokenize, src/ai/llm.c:178-221): short pieces over
a small alphabet (many tokens prefix one another), SentencePiece word pieces
(U+2581), multi-byte UTF-8, "<0xNN>" byte tokens for some bytes (and
lower-case look-alikes, which the byte fallback must not take), GPT-2
byte-level code points U+0100..U+0199 for some bytes, special tokens,
repeated strings (the lowest index wins), empty strings and missing (None)
entries.  Texts draw from the same pieces plus raw bytes 1..255, so they
also hold invalid UTF-8 and bytes that no token covers.
"""
import numpy as np

SP = "▁"
PIECES = ["a", "b", "c", "d", "e", " ", SP, "x", "y", "é", "ß", "中", "\n", "th", "he", "the"]


def _piece_string(rng, lo, hi):
    return "".join(PIECES[i] for i in rng.integers(0, len(PIECES), rng.integers(lo, hi + 1))).encode()


def vocabulary(seed: int, size: int = 400, byte_tokens: bool = True, byte_level: bool = True) -> list:
    """A vocabulary of about `size` entries: bytes, or None for a missing entry."""
    rng = np.random.default_rng(seed)
    v = [b"<unk>", b"<s>", b"</s>"]
    while len(v) < size * 6 // 10:
        v.append(_piece_string(rng, 1, 4))
    if byte_tokens:   # upper-case hex for a random half of the bytes, a few lower-case look-alikes
        for b in rng.permutation(256)[:128]:
            v.append(b"<0x%02X>" % b)
        for b in rng.integers(0, 256, 8):
            v.append(b"<0x%02x>" % b)
    if byte_level:    # two-byte code points from U+0100 on, the range of the byte-level map
        for cp in rng.permutation(np.arange(256, 410))[:100]:
            v.append(chr(int(cp)).encode())
    for _ in range(size // 20):   # repeated strings at later indices
        v.append(v[int(rng.integers(3, len(v)))])
    v += [b"", None, b"", None]
    order = rng.permutation(len(v) - 3) + 3   # the three specials stay at ids 0..2
    return v[:3] + [v[i] for i in order]


def texts(seed: int, n: int = 8, max_len: int = 300) -> list:
    """Texts (bytes, no NUL) for a vocabulary from vocabulary()."""
    rng = np.random.default_rng(seed + 1000)
    out = [b""]
    for _ in range(n - 1):
        t = bytearray()
        target = int(rng.integers(1, max_len))
        while len(t) < target:
            if rng.random() < 0.15:
                t += bytes(rng.integers(1, 256, rng.integers(1, 4)).astype(np.uint8))
            else:
                t += _piece_string(rng, 1, 3)
        out.append(bytes(t))
    return out
