"""The oracle, pinned: against committed fixtures made by the reference's own
C code (tests/golden/make_golden.py) and, where it is built, against that code
directly.  CPU only."""
import numpy as np
import pytest

import holo_b200 as hb
from holo_b200 import synth
from conftest import GOLDEN

FIXTURES = ["q8_0_48x256", "q4_0_40x512", "q4_k_33x512", "q4_k_16x2304", "q6_k_24x512"]


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("name", FIXTURES)
def test_oracle_matches_reference_fixture(oracle, name):
    f = np.load(GOLDEN / f"{name}.npz")
    gt, rows, cols = int(f["gtype"]), int(f["rows"]), int(f["cols"])
    # fp32-activation matvec: bit-exact with src/ai/llm.c matmul_q
    y = oracle.matvec_f32(gt, f["W"], f["x"], rows, cols)
    assert np.array_equal(bits(y), bits(f["y_ref"]))
    # dequantized values: bit-exact with src/ai/quant.c dequantize_row_*
    assert np.array_equal(bits(oracle.dequant(gt, f["W"], rows, cols)), bits(f["deq_ref"]))
    # Q8 restatement: regression pin
    q, d, s = oracle.quantize_act(f["x"])
    assert np.array_equal(q, f["act_q"]) and np.array_equal(bits(d), bits(f["act_d"])) and np.array_equal(s, f["act_s"])
    yq, isums = oracle.matvec_q8(gt, f["W"], f["x"], rows, cols, want_isums=True)
    assert np.array_equal(isums, f["isums"])
    assert np.array_equal(bits(yq), bits(f["y_q8"]))


def test_fixture_inputs_are_reproducible():
    """The generators still produce the fixture inputs (seeded, documented order)."""
    f = np.load(GOLDEN / "q4_k_33x512.npz")
    assert np.array_equal(synth.quant_matrix(hb.Q4_K, 33, 512, 13), f["W"])
    assert np.array_equal(synth.activation(512, 13), f["x"])


@pytest.mark.parametrize("gt,rows,cols", [(hb.Q8_0, 37, 1024), (hb.Q4_0, 5, 11008), (hb.Q4_K, 3, 11008),
                                          (hb.Q4_K, 65, 4096), (hb.Q8_0, 1, 32), (hb.Q4_0, 2, 32),
                                          (hb.Q6_K, 7, 4096), (hb.Q6_K, 1, 256)])
def test_oracle_matches_compiled_reference(oracle, reference, gt, rows, cols):
    seed = rows * 7 + cols
    W = synth.quant_matrix(gt, rows, cols, seed)
    x = synth.activation(cols, seed)
    assert np.array_equal(bits(oracle.matvec_f32(gt, W, x, rows, cols)), bits(reference.matmul_q(gt, W, x, rows, cols)))
    assert np.array_equal(bits(oracle.dequant(gt, W, rows, cols)), bits(reference.dequant(gt, W, rows, cols)))


def test_f16_table_matches_reference(oracle, reference):
    h = np.arange(65536, dtype=np.uint16)
    mine = np.array([oracle.lib.ho_f16_to_f32(int(v)) for v in h[::7]], np.float32)
    theirs = np.array([reference.lib.f16_to_f32(int(v)) for v in h[::7]], np.float32)
    assert np.array_equal(bits(mine), bits(theirs))


def test_f16_rn_matches_numpy(oracle):
    rng = np.random.default_rng(0)
    v = np.concatenate([rng.normal(0, 1e-5, 2000), rng.normal(0, 100, 2000), [65519.0, 65520.0, 1e-8, 0.0, -0.0]]).astype(np.float32)
    mine = np.array([oracle.lib.ho_f32_to_f16_rn(float(a)) for a in v], np.uint16)
    assert np.array_equal(mine, v.astype(np.float16).view(np.uint16))


def ggml_from_ref(blocks):
    """Rewrite quant.c-semantics Q4_K blocks into the llama.cpp (ggml) packing
    with the same values: scales via the inverse of get_scale_min_k4
    (src/ai/cuda_ops.cu:684-692), nibbles 32 bytes per 64 values."""
    b = blocks.reshape(-1, 144)
    sp = b[:, 4:16].astype(np.int32)
    sc = np.empty((b.shape[0], 8), np.int32)
    mn = np.empty((b.shape[0], 8), np.int32)
    sc[:, :4] = sp[:, 0:4] & 63
    mn[:, :4] = sp[:, 4:8] & 63
    sc[:, 4:] = ((sp[:, 8:12] & 0xF) << 2) | (sp[:, 0:4] >> 6)
    mn[:, 4:] = ((sp[:, 8:12] >> 4) << 2) | (sp[:, 4:8] >> 6)
    qs = b[:, 16:].reshape(-1, 8, 16)
    vals = np.concatenate([qs & 0xF, qs >> 4], axis=2).reshape(-1, 256)  # position order
    out = np.empty_like(b)
    out[:, :4] = b[:, :4]
    out[:, 4:8] = (sc[:, :4] & 63) | ((sc[:, 4:] >> 4) << 6)
    out[:, 8:12] = (mn[:, :4] & 63) | ((mn[:, 4:] >> 4) << 6)
    out[:, 12:16] = (sc[:, 4:] & 0xF) | ((mn[:, 4:] & 0xF) << 4)
    g = vals.reshape(-1, 4, 2, 32)
    out[:, 16:] = (g[:, :, 0, :] | (g[:, :, 1, :] << 4)).reshape(-1, 128)
    return out.reshape(-1)


def test_ggml_q4k_semantics_roundtrip(oracle):
    f = np.load(GOLDEN / "q4_k_ref_8x512.npz")
    g = ggml_from_ref(f["W"])
    assert not np.array_equal(g, f["W"])
    deq = oracle.dequant(hb.Q4_K, g, 8, 512, q4k_layout=hb.Q4K_GGML)
    assert np.array_equal(bits(deq), bits(f["deq_ref"]))
    assert np.array_equal(oracle.q4k_to_ref(g, hb.Q4K_GGML), f["W"])


def test_quantize_act_properties(oracle):
    x = synth.activation(4096, 3)
    x[:32] = 0.0                       # an all-zero block
    x[32:64] = np.linspace(-1, 1, 32)  # exact ties at the block max
    q, d, s = oracle.quantize_act(x)
    assert q.dtype == np.int8 and np.abs(q.astype(int)).max() <= 127
    assert d[0] == 0 and not q[:32].any() and s[0] == 0
    assert np.array_equal(s, q.reshape(-1, 32).astype(np.int32).sum(axis=1))
    err = np.abs(q.reshape(-1, 32) * d[:, None] - x.reshape(-1, 32))
    assert (err <= d[:, None] * 0.5 + 1e-7).all()
