"""cuda_matvec_batch: independent matvecs in one persistent launch per weight
type (csrc/matvec_multi.cu), called through the C ABI.

Bars: every output within 1e-6 norm-wise of cuda_matvec on the same problem
(the same per-unit arithmetic; only the split-K cut points differ) and within
1e-3 of the oracle (the reference's matmul_q in HOLO_ACT_F32, the Q8
restatement in HOLO_ACT_Q8); two calls give identical bits; mixed types,
ragged shapes and more problems than one launch takes; unregistered weights
rejected."""
import ctypes as C

import numpy as np
import pytest

import holo_b200 as hb
from holo_b200 import synth
from conftest import rel_err

pytestmark = pytest.mark.gpu


def _mat(gt, rows, cols, seed):
    if gt == hb.F16:
        return synth.quantize(np.random.default_rng(seed).normal(0, 0.02, (rows, cols)).astype(np.float32), gt)
    return synth.quant_matrix(gt, rows, cols, seed)


def _problems(dev, shapes):
    out = []
    for i, (gt, r, c) in enumerate(shapes):
        W = _mat(gt, r, c, 100 + i)
        x = synth.activation(c, 100 + i)
        out.append(dict(gt=gt, r=r, c=c, W=W, x=x, Wd=dev.upload_quant(W, gt, r, c), xd=dev.upload(x),
                        yd=dev.alloc(4 * r), y1=dev.alloc(4 * r)))
    return out


def _batch(dev, probs, act, key="yd"):
    n = len(probs)
    dst = (C.c_void_p * n)(*[p[key] for p in probs])
    M = (C.c_void_p * n)(*[p["Wd"] for p in probs])
    v = (C.c_void_p * n)(*[p["xd"] for p in probs])
    return dev.lib.cuda_matvec_batch(n, dst, M, v, act)


def _free(dev, probs):
    for p in probs:
        for k in ("Wd", "xd", "yd", "y1"):
            dev.free(p[k])


SHAPES = [(hb.Q4_K, 11008, 4096), (hb.Q4_0, 4096, 11008), (hb.Q4_K, 4096, 11008), (hb.Q4_0, 11008, 4096),
          (hb.Q8_0, 333, 4128), (hb.Q6_K, 4099, 2304), (hb.F16, 1000, 4096), (hb.Q4_K, 31, 512), (hb.Q8_0, 4096, 4096),
          (hb.Q4_0, 1, 256)]


@pytest.mark.parametrize("act", [hb.ACT_Q8, hb.ACT_F32], ids=["q8", "f32"])
def test_batch_matches_single_matvecs_and_oracle(dev, oracle, reference, act):
    probs = _problems(dev, SHAPES)
    assert _batch(dev, probs, act) == hb.HOLO_OK
    dev.check("cuda_matvec_batch")
    for p in probs:
        dev.lib.cuda_matvec(p["y1"], p["Wd"], p["xd"], p["r"], p["c"], p["gt"], act, None)
        y = dev.download(p["yd"], (p["r"],), np.float32)
        y1 = dev.download(p["y1"], (p["r"],), np.float32)
        assert rel_err(y, y1) <= 1e-6, (p["gt"], p["r"], p["c"])
        if act == hb.ACT_F32 or p["gt"] == hb.F16:
            want = reference.matmul_q(p["gt"], p["W"], p["x"], p["r"], p["c"], threads=8) if p["gt"] != hb.F16 \
                else oracle.matvec_f32(p["gt"], p["W"], p["x"], p["r"], p["c"])
        else:
            want = oracle.matvec_q8(p["gt"], p["W"], p["x"], p["r"], p["c"])
        assert rel_err(y, want) <= 1e-3, (p["gt"], p["r"], p["c"])
    # deterministic: a second call gives the same bits
    assert _batch(dev, probs, act, key="y1") == hb.HOLO_OK
    for p in probs:
        assert np.array_equal(dev.download(p["yd"], (p["r"],), np.float32), dev.download(p["y1"], (p["r"],), np.float32))
    _free(dev, probs)


def test_more_problems_than_one_launch(dev):
    shapes = [(hb.Q4_K, 64 + 32 * (i % 5), 256 * (1 + i % 3)) for i in range(40)]
    probs = _problems(dev, shapes)
    assert _batch(dev, probs, hb.ACT_Q8) == hb.HOLO_OK
    for p in probs:
        dev.lib.cuda_matvec(p["y1"], p["Wd"], p["xd"], p["r"], p["c"], p["gt"], hb.ACT_Q8, None)
        assert rel_err(dev.download(p["yd"], (p["r"],), np.float32), dev.download(p["y1"], (p["r"],), np.float32)) <= 1e-6
    dev.check("cuda_matvec_batch 40")
    _free(dev, probs)


def test_batch_rejects_raw_weight(dev):
    W = synth.quant_matrix(hb.Q4_K, 64, 256, 1)
    Wd, xd, yd = dev.upload(W), dev.upload(synth.activation(256, 1)), dev.alloc(256)
    dev.lib.cuda_clear_status()
    rc = dev.lib.cuda_matvec_batch(1, (C.c_void_p * 1)(yd), (C.c_void_p * 1)(Wd), (C.c_void_p * 1)(xd), hb.ACT_Q8)
    assert rc == hb.HOLO_E_ARG
    dev.lib.cuda_clear_status()
    for q in (Wd, xd, yd):
        dev.free(q)
