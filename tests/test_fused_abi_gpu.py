"""The reference ABI's fused entry points, called through the C ABI:
cuda_batched_qkv_q8_0 (src/ai/cuda_ops.cu:1282-1294: q, k, v = Wq.x, Wk.x,
Wv.x) and cuda_batched_ffn_gate_up_q8_0 (cuda_ops.cu:1386-1395:
out = silu(W1.x) * (W3.x), silu(g) = g / (1 + exp(-g))).

Bars (those of test_matvec_gpu): max|y - r| / max|r| <= 1e-3, where r is
built from the reference's own matmul_q (src/ai/llm.c:770-926) and silu
(src/ai/tensor.c:218-222) in HOLO_ACT_F32, and from the oracle's Q8
restatement in HOLO_ACT_Q8; weights raw (the reference loader's
upload_tensor) or tiled (cuda_upload_quant).
"""
import numpy as np
import pytest

import holo_b200 as hb
from holo_b200 import synth
from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _upload(dev, W, rows, cols, tiled):
    return dev.upload_quant(W, hb.Q8_0, rows, cols) if tiled else dev.upload(W)


def _want(oracle, reference, act, W, x, rows, cols):
    if act == hb.ACT_F32:
        return reference.matmul_q(hb.Q8_0, W, x, rows, cols)
    return oracle.matvec_q8(hb.Q8_0, W, x, rows, cols)


@pytest.fixture
def act_mode(dev):
    before = dev.lib.cuda_get_act_mode()
    yield
    dev.lib.cuda_set_act_mode(before)


@pytest.mark.parametrize("tiled", [False, True], ids=["raw", "tiled"])
@pytest.mark.parametrize("act", [hb.ACT_F32, hb.ACT_Q8], ids=["f32", "q8"])
@pytest.mark.parametrize("q_dim,kv_dim,in_dim", [(512, 128, 1024), (4096, 1024, 4096), (96, 32, 4128)])
def test_batched_qkv_q8_0(dev, oracle, reference, act_mode, tiled, act, q_dim, kv_dim, in_dim):
    seed = q_dim + kv_dim + in_dim
    Ws = [synth.quant_matrix(hb.Q8_0, r, in_dim, seed + i) for i, r in enumerate((q_dim, kv_dim, kv_dim))]
    x = synth.activation(in_dim, seed)
    Wd = [_upload(dev, W, r, in_dim, tiled) for W, r in zip(Ws, (q_dim, kv_dim, kv_dim))]
    xd = dev.upload(x)
    outs = [dev.alloc(4 * r) for r in (q_dim, kv_dim, kv_dim)]
    dev.lib.cuda_set_act_mode(act)
    dev.lib.cuda_batched_qkv_q8_0(outs[0], outs[1], outs[2], Wd[0], Wd[1], Wd[2], xd, q_dim, kv_dim, in_dim)
    dev.check("cuda_batched_qkv_q8_0")
    for W, r, o in zip(Ws, (q_dim, kv_dim, kv_dim), outs):
        y = dev.download(o, (r,), np.float32)
        assert rel_err(y, _want(oracle, reference, act, W, x, r, in_dim)) <= TOL
    for p in Wd + outs + [xd]:
        dev.free(p)


@pytest.mark.parametrize("tiled", [False, True], ids=["raw", "tiled"])
@pytest.mark.parametrize("act", [hb.ACT_F32, hb.ACT_Q8], ids=["f32", "q8"])
@pytest.mark.parametrize("ffn_dim,in_dim", [(768, 512), (11008, 4096), (200, 4128)])
def test_batched_ffn_gate_up_q8_0(dev, oracle, reference, act_mode, tiled, act, ffn_dim, in_dim):
    seed = 7 * ffn_dim + in_dim
    W1 = synth.quant_matrix(hb.Q8_0, ffn_dim, in_dim, seed)
    W3 = synth.quant_matrix(hb.Q8_0, ffn_dim, in_dim, seed + 1)
    x = synth.activation(in_dim, seed)
    W1d, W3d = _upload(dev, W1, ffn_dim, in_dim, tiled), _upload(dev, W3, ffn_dim, in_dim, tiled)
    xd, od = dev.upload(x), dev.alloc(4 * ffn_dim)
    dev.lib.cuda_set_act_mode(act)
    dev.lib.cuda_batched_ffn_gate_up_q8_0(od, W1d, W3d, xd, ffn_dim, in_dim)
    dev.check("cuda_batched_ffn_gate_up_q8_0")
    y = dev.download(od, (ffn_dim,), np.float32)
    g = _want(oracle, reference, act, W1, x, ffn_dim, in_dim)
    u = _want(oracle, reference, act, W3, x, ffn_dim, in_dim)
    want = (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32) * u   # tensor.c:218-222, then vec_mul
    assert rel_err(y, want) <= TOL
    for p in (W1d, W3d, xd, od):
        dev.free(p)
