"""Generates the golden fixtures of tests/test_oracle_pin.py.

Run where the reference sources are present (they are compiled from source
into oracle/_ref/libholo_ref.so by oracle/Makefile):

    python tests/golden/make_golden.py [fixture names]   # all when none given

Each fixture holds the inputs (GGUF blocks, activation) and the outputs of the
REFERENCE's own CPU functions on them: matmul_q (src/ai/llm.c:770-926) and
dequantize_row_* (src/ai/quant.c:118-311).  The Q8-activation outputs come
from the build's restatement (the reference has no such code) and pin it
against regressions only.
"""
import pathlib
import sys

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "google-classic_b200"))
sys.path.insert(0, str(ROOT / "oracle"))

import holo_b200 as hb  # noqa: E402
from holo_b200 import synth  # noqa: E402
import holo_oracle  # noqa: E402

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
    if only and "q4_k_ref_8x512" not in only:
        return
    # ggml-semantics Q4_K: the same values as a quant.c-semantics block set
    W = synth.quant_matrix(hb.Q4_K, 8, 512, 15)
    deq = ref.dequant(hb.Q4_K, W, 8, 512)
    np.savez_compressed(out / "q4_k_ref_8x512.npz", W=W, deq_ref=deq)
    print("wrote q4_k_ref_8x512")


if __name__ == "__main__":
    main(tuple(sys.argv[1:]))
