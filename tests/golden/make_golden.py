"""Generates the golden fixtures of tests/test_oracle_pin.py.

Run where the reference sources are present (they are compiled from source
into oracle/_ref/libholo_ref.so by oracle/Makefile):

    python tests/golden/make_golden.py [fixture names]   # all when none given

Each fixture holds the inputs (GGUF blocks, activation) and the outputs of the
REFERENCE's own CPU functions on them: matmul_q (src/ai/llm.c:770-926) and
dequantize_row_* (src/ai/quant.c:118-311); tokenize_cases.json holds
vocabularies and texts (tests/golden/tok_cases.py) with the token ids of the
reference's llm_tokenize (llm.c:178-221).  The Q8-activation outputs come
from the build's restatement (the reference has no such code) and pin it
against regressions only.
"""
import pathlib
import sys

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "google-classic_b200"))
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(pathlib.Path(__file__).resolve().parent))

import holo_b200 as hb  # noqa: E402
from holo_b200 import synth  # noqa: E402
import holo_oracle  # noqa: E402
import tok_cases  # noqa: E402

CASES = [
    # name, type, rows, cols, seed
    ("q8_0_48x256", hb.Q8_0, 48, 256, 11),
    ("q4_0_40x512", hb.Q4_0, 40, 512, 12),
    ("q4_k_33x512", hb.Q4_K, 33, 512, 13),
    ("q4_k_16x2304", hb.Q4_K, 16, 2304, 14),
    ("q6_k_24x512", hb.Q6_K, 24, 512, 16),
]


def main(only=()):
    ref = holo_oracle.Reference()
    orc = holo_oracle.Oracle()
    out = pathlib.Path(__file__).resolve().parent
    for name, gt, rows, cols, seed in CASES:
        if only and name not in only:
            continue
        W = synth.quant_matrix(gt, rows, cols, seed)
        x = synth.activation(cols, seed)
        y_ref = ref.matmul_q(gt, W, x, rows, cols)
        deq_ref = ref.dequant(gt, W, rows, cols)
        q, d, s = orc.quantize_act(x)
        y_q8, isums = orc.matvec_q8(gt, W, x, rows, cols, want_isums=True)
        np.savez_compressed(out / f"{name}.npz", gtype=gt, rows=rows, cols=cols, W=W, x=x,
                            y_ref=y_ref, deq_ref=deq_ref, act_q=q, act_d=d, act_s=s,
                            y_q8=y_q8, isums=isums)
        print("wrote", name)
    if not only or "tokenize_cases" in only:
        tokenize_cases(ref, out)
    if only and "q4_k_ref_8x512" not in only:
        return
    # ggml-semantics Q4_K: the same values as a quant.c-semantics block set
    W = synth.quant_matrix(hb.Q4_K, 8, 512, 15)
    deq = ref.dequant(hb.Q4_K, W, 8, 512)
    np.savez_compressed(out / "q4_k_ref_8x512.npz", W=W, deq_ref=deq)
    print("wrote q4_k_ref_8x512")


# (seed, vocabulary size, "<0xNN>" tokens, byte-level tokens, bos, unk)
TOKENIZE_CASES = [(1, 300, True, True, 1, 0), (2, 300, False, True, 1, 0), (3, 300, False, False, 2, 7)]


def tokenize_cases(ref, out):
    import json
    cases = []
    for seed, size, bt, bl, bos, unk in TOKENIZE_CASES:
        vocab = tok_cases.vocabulary(seed, size, bt, bl)
        for i, text in enumerate(tok_cases.texts(seed, n=6, max_len=160)):
            add_bos, cap = bool(i % 2), (None if i != 3 else 17)   # one case cut at 17 ids
            ids = ref.tokenize(vocab, bos, unk, text, max_tokens=cap, add_bos=add_bos)
            cases.append(dict(seed=seed, text=text.hex(), add_bos=add_bos, max_tokens=cap, ids=ids.tolist()))
    vocabs = {str(seed): [None if t is None else t.hex() for t in tok_cases.vocabulary(seed, size, bt, bl)]
              for seed, size, bt, bl, _, _ in TOKENIZE_CASES}
    ids = {str(seed): [bos, unk] for seed, _, _, _, bos, unk in TOKENIZE_CASES}
    (out / "tokenize_cases.json").write_text(json.dumps(dict(vocabs=vocabs, bos_unk=ids, cases=cases)))
    print("wrote tokenize_cases")


if __name__ == "__main__":
    main(tuple(sys.argv[1:]))
