"""Parity of the CUDA matvecs (called through the C ABI) with the oracle.

Bars (fixed here):
* dequantized values and per-block integer sums: bit-exact;
* fp32 outputs: max|y - r| / max|r| <= 1e-3, where r is
  - the reference's own matmul_q (src/ai/llm.c:770-926) for HOLO_ACT_F32,
  - the oracle's Q8 restatement for HOLO_ACT_Q8.
"""
import ctypes as C

import numpy as np
import pytest

import holo_b200 as hb
from holo_b200 import synth
from conftest import rel_err
from test_oracle_pin import ggml_from_ref

pytestmark = pytest.mark.gpu
TOL = 1e-3
TYPES = [hb.Q8_0, hb.Q4_0, hb.Q4_K]

SHAPES = [  # rows, cols  (ragged rows, one K-chunk, several, tails)
    (1, 256), (31, 512), (33, 2304), (100, 4096), (257, 1024), (64, 11008 - 11008 % 256),
]


def run_matvec(dev, Wd, gtype, x, rows, cols, act, residual=None):
    lib = dev.lib
    xd = dev.upload(x.astype(np.float32))
    yd = dev.alloc(rows * 4)
    rd = None
    if residual is not None:
        rd = dev.upload(residual.astype(np.float32))
    lib.cuda_matvec(yd, Wd, xd, rows, cols, gtype, act, rd)
    y = dev.download(yd, (rows,), np.float32)
    dev.check("matvec")
    for p in (xd, yd, rd):
        dev.free(p)
    return y


@pytest.mark.parametrize("gtype", TYPES)
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_tiled_matvec_parity(dev, oracle, reference, gtype, rows, cols):
    if gtype == hb.Q8_0 and cols % 32:
        pytest.skip()
    seed = rows + 3 * cols + gtype
    W = synth.quant_matrix(gtype, rows, cols, seed)
    x = synth.activation(cols, seed)
    Wd = dev.upload_quant(W, gtype, rows, cols)
    y32 = run_matvec(dev, Wd, gtype, x, rows, cols, hb.ACT_F32)
    assert rel_err(y32, reference.matmul_q(gtype, W, x, rows, cols)) <= TOL
    y8 = run_matvec(dev, Wd, gtype, x, rows, cols, hb.ACT_Q8)
    assert rel_err(y8, oracle.matvec_q8(gtype, W, x, rows, cols)) <= TOL
    dev.free(Wd)


@pytest.mark.parametrize("rows,cols", SHAPES)
def test_tiled_q6_k_parity(dev, oracle, reference, rows, cols):
    """Q6_K in the unit layout (one 128-value half of a super-block a unit):
    HOLO_ACT_F32 against the reference's matmul_q (mat_vec_q6_k), HOLO_ACT_Q8
    against the oracle's restatement; the reference entry point on the same
    (registered) pointer gives the fp32 result."""
    gtype = hb.Q6_K
    seed = rows + 3 * cols + gtype
    W = synth.quant_matrix(gtype, rows, cols, seed)
    x = synth.activation(cols, seed)
    Wd = dev.upload_quant(W, gtype, rows, cols)
    want = reference.matmul_q(gtype, W, x, rows, cols)
    y32 = run_matvec(dev, Wd, gtype, x, rows, cols, hb.ACT_F32)
    assert rel_err(y32, want) <= TOL
    y8 = run_matvec(dev, Wd, gtype, x, rows, cols, hb.ACT_Q8)
    assert rel_err(y8, oracle.matvec_q8(gtype, W, x, rows, cols)) <= TOL
    xd, yd = dev.upload(x), dev.alloc(rows * 4)
    dev.lib.cuda_matmul_q6_k(yd, Wd, xd, rows, cols)
    assert np.array_equal(dev.download(yd, (rows,), np.float32), y32)
    dev.check("cuda_matmul_q6_k")
    for p in (Wd, xd, yd):
        dev.free(p)


@pytest.mark.parametrize("rows,cols", [(1, 64), (33, 512), (100, 4096), (257, 1024), (64, 11008)])
def test_tiled_f16_parity(dev, reference, rows, cols):
    """F16 weights in the unit layout (64 values a row a unit), fp32
    activations in both modes: against the reference's matmul_q (llm.c:818-828)
    and an fp64 product of the same values."""
    gtype = hb.F16
    Wh = synth.f16_matrix(rows, cols, seed=rows + cols)
    W = Wh.view(np.uint8).reshape(-1)
    x = synth.activation(cols, rows)
    Wd = dev.upload_quant(W, gtype, rows, cols)
    exact = (Wh.astype(np.float64) @ x.astype(np.float64)).astype(np.float32)
    for act in (hb.ACT_F32, hb.ACT_Q8):
        y = run_matvec(dev, Wd, gtype, x, rows, cols, act)
        assert rel_err(y, reference.matmul_q(gtype, W, x, rows, cols)) <= TOL
        assert rel_err(y, exact) <= 1e-5
    dev.free(Wd)


@pytest.mark.parametrize("gtype", [hb.Q8_0, hb.Q4_0])
@pytest.mark.parametrize("rows,cols", [(45, 96), (70, 1440), (33, 4128), (5, 32)])
def test_padded_last_unit_parity(dev, oracle, reference, gtype, rows, cols):
    """Rows whose 32-block count is not a multiple of the unit's (4 blocks for
    Q8_0, 8 for Q4_0): the tiled copy pads the last unit with zero blocks."""
    seed = 7 * rows + cols + gtype
    W = synth.quant_matrix(gtype, rows, cols, seed)
    x = synth.activation(cols, seed)
    Wd = dev.upload_quant(W, gtype, rows, cols)
    y32 = run_matvec(dev, Wd, gtype, x, rows, cols, hb.ACT_F32)
    assert rel_err(y32, reference.matmul_q(gtype, W, x, rows, cols)) <= TOL
    y8 = run_matvec(dev, Wd, gtype, x, rows, cols, hb.ACT_Q8)
    assert rel_err(y8, oracle.matvec_q8(gtype, W, x, rows, cols)) <= TOL
    dev.free(Wd)


@pytest.mark.parametrize("gtype", TYPES)
def test_raw_blocks_path_parity(dev, oracle, reference, gtype):
    """Weights uploaded as the reference's upload_tensor does (cuda_malloc +
    cuda_memcpy_h2d of raw GGUF bytes), through the reference entry points."""
    rows, cols = 200, 2304
    W = synth.quant_matrix(gtype, rows, cols, 5)
    x = synth.activation(cols, 5)
    Wd = dev.upload(W)
    xd, yd = dev.upload(x), dev.alloc(rows * 4)
    fn = {hb.Q8_0: dev.lib.cuda_matmul_q8_0, hb.Q4_0: dev.lib.cuda_matmul_q4_0, hb.Q4_K: dev.lib.cuda_matmul_q4_k}[gtype]
    for act, ref in ((hb.ACT_F32, reference.matmul_q(gtype, W, x, rows, cols)),
                     (hb.ACT_Q8, oracle.matvec_q8(gtype, W, x, rows, cols))):
        dev.lib.cuda_set_act_mode(act)
        fn(yd, Wd, xd, rows, cols)
        y = dev.download(yd, (rows,), np.float32)
        dev.check()
        assert rel_err(y, ref) <= TOL
    dev.lib.cuda_set_act_mode(hb.ACT_Q8)
    for p in (Wd, xd, yd):
        dev.free(p)


@pytest.mark.parametrize("gtype", TYPES)
@pytest.mark.parametrize("tiled", [True, False])
def test_dequantized_values_bit_exact(dev, reference, gtype, tiled):
    rows, cols = 45, (2304 if gtype == hb.Q4_K else 2336)   # 73 blocks: a padded last unit
    W = synth.quant_matrix(gtype, rows, cols, 21)
    Wd = dev.upload_quant(W, gtype, rows, cols) if tiled else dev.upload(W)
    od = dev.alloc(rows * cols * 4)
    dev.lib.cuda_dequantize_rows(od, Wd, gtype, rows, cols)
    got = dev.download(od, (rows, cols), np.float32)
    dev.check()
    assert np.array_equal(got.view(np.uint32), reference.dequant(gtype, W, rows, cols).view(np.uint32))
    dev.free(od)
    dev.free(Wd)


@pytest.mark.parametrize("gtype", TYPES)
@pytest.mark.parametrize("tiled", [True, False])
def test_block_integer_sums_bit_exact(dev, oracle, gtype, tiled):
    rows, cols = 70, (4096 if gtype == hb.Q4_K else 4128)
    W = synth.quant_matrix(gtype, rows, cols, 31)
    x = synth.activation(cols, 31)
    Wd = dev.upload_quant(W, gtype, rows, cols) if tiled else dev.upload(W)
    xd = dev.upload(x)
    od = dev.alloc(rows * (cols // 32) * 4)
    dev.lib.cuda_block_sums_q8(od, Wd, xd, gtype, rows, cols)
    got = dev.download(od, (rows, cols // 32), np.int32)
    dev.check()
    _, isums = oracle.matvec_q8(gtype, W, x, rows, cols, want_isums=True)
    assert np.array_equal(got, isums)
    for p in (Wd, xd, od):
        dev.free(p)


def test_activation_quantizer_bit_exact(dev, oracle):
    x = synth.activation(11008, 4)
    x[:32] = 0.0
    xd = dev.upload(x)
    q, d, s = dev.alloc(x.size), dev.alloc(x.size // 8), dev.alloc(x.size // 8)
    dev.lib.cuda_quantize_act_q8(q, d, s, xd, x.size)
    gq = dev.download(q, (x.size,), np.int8)
    gd = dev.download(d, (x.size // 32,), np.float32)
    gs = dev.download(s, (x.size // 32,), np.int32)
    dev.check()
    oq, od, os_ = oracle.quantize_act(x)
    assert np.array_equal(gq, oq) and np.array_equal(gd.view(np.uint32), od.view(np.uint32)) and np.array_equal(gs, os_)
    for p in (xd, q, d, s):
        dev.free(p)


def test_residual_epilogue(dev, oracle):
    rows, cols = 4096, 4096
    W = synth.quant_matrix(hb.Q4_K, rows, cols, 8)
    x = synth.activation(cols, 8)
    res = synth.activation(rows, 9)
    Wd = dev.upload_quant(W, hb.Q4_K, rows, cols)
    y = run_matvec(dev, Wd, hb.Q4_K, x, rows, cols, hb.ACT_Q8, residual=res)
    assert rel_err(y, oracle.matvec_q8(hb.Q4_K, W, x, rows, cols) + res) <= TOL
    dev.free(Wd)


def test_ggml_q4k_layout_is_normalised(dev, reference):
    """Blocks in the llama.cpp packing (src/ai/cuda_ops.cu:684-732) upload to
    the same device values as the equivalent quant.c-packing blocks."""
    rows, cols = 64, 2048
    W = synth.quant_matrix(hb.Q4_K, rows, cols, 40)
    G = ggml_from_ref(W)
    x = synth.activation(cols, 40)
    dev.lib.cuda_set_q4k_layout(hb.Q4K_GGML)
    try:
        Gd = dev.upload_quant(G, hb.Q4_K, rows, cols)
        Gr = dev.upload(G)
    finally:
        dev.lib.cuda_set_q4k_layout(hb.Q4K_REF)
    od = dev.alloc(rows * cols * 4)
    dev.lib.cuda_dequantize_rows(od, Gd, hb.Q4_K, rows, cols)
    got = dev.download(od, (rows, cols), np.float32)
    dev.check()
    assert np.array_equal(got.view(np.uint32), reference.dequant(hb.Q4_K, W, rows, cols).view(np.uint32))
    y = run_matvec(dev, Gd, hb.Q4_K, x, rows, cols, hb.ACT_F32)
    assert rel_err(y, reference.matmul_q(hb.Q4_K, W, x, rows, cols)) <= TOL
    # raw ggml blocks decoded in place
    dev.lib.cuda_set_q4k_layout(hb.Q4K_GGML)
    try:
        y_raw = run_matvec(dev, Gr, hb.Q4_K, x, rows, cols, hb.ACT_F32)
    finally:
        dev.lib.cuda_set_q4k_layout(hb.Q4K_REF)
    assert rel_err(y_raw, reference.matmul_q(hb.Q4_K, W, x, rows, cols)) <= TOL
    for p in (Gd, Gr, od):
        dev.free(p)


def test_reference_gpu_kernel_pins_ggml_semantics(dev):
    """The reference's own thread-per-row Q4_K kernel (used for out_dim <=
    4096, src/ai/cuda_ops.cu:694-732) on ggml-packed blocks agrees with this
    library's decoding of the same blocks in the ggml layout."""
    import holo_oracle
    so = holo_oracle.HERE / "_ref" / "libholo_ref_cuda.so"
    if not so.exists():
        pytest.skip("reference CUDA library not built")
    ref = C.CDLL(str(so))
    ref.cuda_matmul_q4_k.argtypes = [C.c_void_p] * 3 + [C.c_int, C.c_int]
    rows, cols = 256, 1024
    W = synth.quant_matrix(hb.Q4_K, rows, cols, 41)
    G = ggml_from_ref(W)
    x = synth.activation(cols, 41)
    Gd, xd, yd = dev.upload(G), dev.upload(x), dev.alloc(rows * 4)
    dev.sync()
    ref.cuda_matmul_q4_k(yd, Gd, xd, rows, cols)
    dev.sync()
    y_ref_gpu = dev.download(yd, (rows,), np.float32)
    dev.lib.cuda_set_q4k_layout(hb.Q4K_GGML)
    try:
        y = run_matvec(dev, Gd, hb.Q4_K, x, rows, cols, hb.ACT_F32)
    finally:
        dev.lib.cuda_set_q4k_layout(hb.Q4K_REF)
    assert rel_err(y, y_ref_gpu) <= TOL
    for p in (Gd, xd, yd):
        dev.free(p)


@pytest.mark.parametrize("gtype,rows,cols", [(hb.Q8_0, 4096, 4096), (hb.Q4_0, 11008, 4096), (hb.Q4_0, 4096, 11008),
                                             (hb.Q4_K, 11008, 4096), (hb.Q4_K, 4096, 11008)])
def test_benchmark_shapes_parity(dev, oracle, gtype, rows, cols):
    """Full benchmark-config shapes (seed 0): both activation modes."""
    W = synth.quant_matrix(gtype, rows, cols, 0)
    x = synth.activation(cols, 0)
    Wd = dev.upload_quant(W, gtype, rows, cols)
    for act in (hb.ACT_F32, hb.ACT_Q8):
        y = run_matvec(dev, Wd, gtype, x, rows, cols, act)
        r = oracle.matvec_f32(gtype, W, x, rows, cols, threads=8) if act == hb.ACT_F32 else \
            oracle.matvec_q8(gtype, W, x, rows, cols, threads=8)
        assert rel_err(y, r) <= TOL
    dev.free(Wd)


def test_repeated_calls_are_deterministic(dev):
    """Split-K rows are combined in a fixed order: identical bits every call."""
    rows, cols = 1024, 8192
    W = synth.quant_matrix(hb.Q4_0, rows, cols, 2)
    x = synth.activation(cols, 2)
    Wd = dev.upload_quant(W, hb.Q4_0, rows, cols)
    ys = [run_matvec(dev, Wd, hb.Q4_0, x, rows, cols, hb.ACT_Q8) for _ in range(4)]
    for y in ys[1:]:
        assert np.array_equal(y.view(np.uint32), ys[0].view(np.uint32))
    dev.free(Wd)


def test_dependent_chain_with_pdl_and_graph(dev, oracle):
    """A chain of dependent matvecs (y1 = W1.x; y2 = y1 + W2.y1) gives the same
    bits with programmatic dependent launch on and off, and replayed from a
    CUDA graph."""
    n = 4096
    W1 = synth.quant_matrix(hb.Q4_K, n, n, 50)
    W2 = synth.quant_matrix(hb.Q8_0, n, n, 51)
    x = synth.activation(n, 50)
    W1d, W2d = dev.upload_quant(W1, hb.Q4_K, n, n), dev.upload_quant(W2, hb.Q8_0, n, n)
    xd, y1, y2 = dev.upload(x), dev.alloc(4 * n), dev.alloc(4 * n)

    def chain():
        dev.lib.cuda_matvec(y1, W1d, xd, n, n, hb.Q4_K, hb.ACT_Q8, None)
        dev.lib.cuda_matvec(y2, W2d, y1, n, n, hb.Q8_0, hb.ACT_Q8, y1)

    outs = []
    for pdl in (0, 1):
        dev.lib.cuda_set_pdl(pdl)
        chain()
        outs.append(dev.download(y2, (n,), np.float32))
    dev.lib.cuda_set_pdl(1)
    assert dev.lib.cuda_capture_begin() == 0
    chain()
    g = dev.lib.cuda_capture_end()
    dev.lib.cuda_memset(y2, 0, 4 * n)
    for _ in range(3):
        dev.lib.cuda_graph_launch(g)
    outs.append(dev.download(y2, (n,), np.float32))
    dev.lib.cuda_graph_free(g)
    dev.lib.cuda_set_pdl(0)
    dev.check()
    for o in outs[1:]:
        assert np.array_equal(o.view(np.uint32), outs[0].view(np.uint32))
    r1 = oracle.matvec_q8(hb.Q4_K, W1, x, n, n)
    assert rel_err(outs[0], r1 + oracle.matvec_q8(hb.Q8_0, W2, r1, n, n)) <= 1e-3
    for p in (W1d, W2d, xd, y1, y2):
        dev.free(p)


def test_unsupported_shape_sets_status_not_fault(dev):
    """A K extent beyond the tiled kernel's shared memory is refused on the
    host with HOLO_E_UNSUPPORTED; the context stays usable."""
    rows, cols = 32, 256 * 1024
    W = np.zeros(rows * hb.row_bytes(hb.Q4_K, cols), np.uint8)
    Wd = dev.upload_quant(W, hb.Q4_K, rows, cols)
    xd, yd = dev.upload(np.zeros(cols, np.float32)), dev.alloc(rows * 4)
    dev.lib.cuda_matvec(yd, Wd, xd, rows, cols, hb.Q4_K, hb.ACT_Q8, None)
    assert dev.lib.cuda_last_status() == hb.HOLO_E_UNSUPPORTED
    dev.lib.cuda_clear_status()
    # bad type / shape
    dev.lib.cuda_matvec(yd, Wd, xd, rows, 100, hb.Q4_K, hb.ACT_Q8, None)
    assert dev.lib.cuda_last_status() == hb.HOLO_E_ARG
    dev.lib.cuda_clear_status()
    for p in (Wd, xd, yd):
        dev.free(p)
    dev.check()
