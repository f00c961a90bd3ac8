"""cuda_matvec_noalloc: the tiled matvec with its split-K scratch in static
device memory (no allocation in the call), for callers that cannot allocate
device memory once running (a fixed device budget handed out at start-up, or
a latency loop where cudaMalloc would synchronise the device).

The file name sorts last, so in a full run these tests execute after every
other GPU test in the same process; they also pass run alone.  Each case
compares two consecutive no-alloc calls with the existing entry point
(cuda_matvec) on the same uploaded weight.
"""
import numpy as np
import pytest

import holo_b200 as hb
from holo_b200 import synth
from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-6   # same kernel and grid as cuda_matvec: equal up to rounding


def _matvec(dev, fn_name, Wd, xd, rows, cols, gtype, act):
    yd = dev.alloc(rows * 4)
    if fn_name == "cuda_matvec":
        dev.lib.cuda_matvec(yd, Wd, xd, rows, cols, gtype, act, None)
        rc = 0
    else:
        rc = dev.lib.cuda_matvec_noalloc(yd, Wd, xd, rows, cols, gtype, act)
    y = dev.download(yd, (rows,), np.float32)
    dev.free(yd)
    return rc, y


@pytest.mark.parametrize("gtype,rows,cols", [
    (hb.Q4_K, 11008, 4096),   # row-blocks cut between CTAs (split-K fix-up)
    (hb.Q4_0, 4096, 11008),
    (hb.Q8_0, 333, 4128),     # ragged rows, padded last unit
    (hb.Q6_K, 4099, 2304),    # ragged rows, half-super-block units
    (hb.F16, 1000, 4096),     # ragged rows; F16 always takes fp32 activations
])
@pytest.mark.parametrize("act", [hb.ACT_Q8, hb.ACT_F32])
def test_noalloc_matches_existing_entry_point(dev, gtype, rows, cols, act):
    seed = rows + cols + gtype
    if gtype == hb.F16:
        W = synth.quantize(np.random.default_rng(seed).normal(0, 0.02, (rows, cols)).astype(np.float32), gtype)
    else:
        W = synth.quant_matrix(gtype, rows, cols, seed)
    x = synth.activation(cols, seed)
    Wd = dev.upload_quant(W, gtype, rows, cols)
    xd = dev.upload(x)
    _, y_ref = _matvec(dev, "cuda_matvec", Wd, xd, rows, cols, gtype, act)
    dev.check("cuda_matvec")
    for _ in range(2):
        rc, y = _matvec(dev, "cuda_matvec_noalloc", Wd, xd, rows, cols, gtype, act)
        assert rc == hb.HOLO_OK
        dev.check("cuda_matvec_noalloc")
        assert rel_err(y, y_ref) <= TOL
    dev.free(Wd)
    dev.free(xd)


def test_noalloc_rejects_rows_beyond_static_scratch(dev):
    rows, cols = 262144 + 32, 256          # 8193 row-blocks > 8192
    W = synth.quant_matrix(hb.Q4_K, rows, cols, 3)
    Wd = dev.upload_quant(W, hb.Q4_K, rows, cols)
    xd = dev.upload(synth.activation(cols, 3))
    yd = dev.alloc(rows * 4)
    dev.lib.cuda_clear_status()
    rc = dev.lib.cuda_matvec_noalloc(yd, Wd, xd, rows, cols, hb.Q4_K, hb.ACT_Q8)
    assert rc == hb.HOLO_E_UNSUPPORTED
    assert dev.lib.cuda_last_status() == hb.HOLO_E_UNSUPPORTED
    assert b"262144" in dev.lib.cuda_last_status_string()
    dev.lib.cuda_clear_status()
    for p in (Wd, xd, yd):
        dev.free(p)


def test_noalloc_rejects_unregistered_weight(dev):
    W = synth.quant_matrix(hb.Q4_K, 64, 256, 4)
    Wd = dev.upload(W)                        # raw blocks: not a tiled weight
    xd = dev.upload(synth.activation(256, 4))
    yd = dev.alloc(64 * 4)
    dev.lib.cuda_clear_status()
    rc = dev.lib.cuda_matvec_noalloc(yd, Wd, xd, 64, 256, hb.Q4_K, hb.ACT_Q8)
    assert rc == hb.HOLO_E_ARG
    dev.lib.cuda_clear_status()
    for p in (Wd, xd, yd):
        dev.free(p)


def test_noalloc_timeout_word_is_reported_and_cleared(dev):
    """A launch whose bounded wait gives up leaves HOLO_E_TIMEOUT in the
    path's status word.  The word is written here the way such a launch
    writes it (no wait is made to run out): cuda_last_status must report it,
    and cuda_clear_status must reset it so later calls report success."""
    import ctypes
    rows, cols = 96, 1024
    W = synth.quant_matrix(hb.Q4_K, rows, cols, 9)
    x = synth.activation(cols, 9)
    Wd = dev.upload_quant(W, hb.Q4_K, rows, cols)
    xd = dev.upload(x)
    dev.lib.cuda_clear_status()
    word = dev.lib.cuda_matvec_noalloc_status_word()
    assert word
    code = np.array([hb.HOLO_E_TIMEOUT], dtype=np.int32)
    dev.lib.cuda_memcpy_h2d(word, code.ctypes.data_as(ctypes.c_void_p), 4)
    assert dev.lib.cuda_last_status() == hb.HOLO_E_TIMEOUT
    assert b"noalloc" in dev.lib.cuda_last_status_string()
    dev.lib.cuda_clear_status()
    assert dev.lib.cuda_last_status() == hb.HOLO_OK
    _, y_ref = _matvec(dev, "cuda_matvec", Wd, xd, rows, cols, hb.Q4_K, hb.ACT_Q8)
    rc, y = _matvec(dev, "cuda_matvec_noalloc", Wd, xd, rows, cols, hb.Q4_K, hb.ACT_Q8)
    assert rc == hb.HOLO_OK and dev.lib.cuda_last_status() == hb.HOLO_OK
    assert rel_err(y, y_ref) <= TOL
    dev.free(Wd)
    dev.free(xd)
