"""The non-matvec entry points of the reference ABI against the reference's CPU
arithmetic (src/ai/tensor.c, src/ai/llm.c) restated in numpy (fp64)."""
import numpy as np
import pytest

import holo_b200 as hb
from holo_b200 import synth
from conftest import rel_err

pytestmark = pytest.mark.gpu


def up(dev, a):
    return dev.upload(np.ascontiguousarray(a))


def test_vector_ops(dev):
    n = 10007
    a, b = synth.activation(n, 1), synth.activation(n, 2)
    ad, bd, od = up(dev, a), up(dev, b), dev.alloc(n * 4)
    dev.lib.cuda_vec_add(od, ad, bd, n)
    assert np.array_equal(dev.download(od, (n,), np.float32), a + b)
    dev.lib.cuda_vec_mul(od, ad, bd, n)
    assert np.array_equal(dev.download(od, (n,), np.float32), a * b)
    dev.lib.cuda_vec_scale(od, ad, np.float32(0.37), n)
    assert np.array_equal(dev.download(od, (n,), np.float32), a * np.float32(0.37))
    dot = dev.lib.cuda_vec_dot(ad, bd, n)
    assert abs(dot - float(np.dot(a.astype(np.float64), b))) <= 1e-4 * np.abs(a * b).sum()
    dev.check()
    for p in (ad, bd, od):
        dev.free(p)


def test_activations(dev):
    n = 4096
    a, b = synth.activation(n, 3) * 4, synth.activation(n, 4)
    ad, bd, od = up(dev, a), up(dev, b), dev.alloc(n * 4)
    dev.lib.cuda_silu_mul(od, ad, bd, n)
    a64 = a.astype(np.float64)
    assert rel_err(dev.download(od, (n,), np.float32), a64 / (1 + np.exp(-a64)) * b) <= 1e-6
    xd = up(dev, a)
    dev.lib.cuda_silu(xd, n)
    assert rel_err(dev.download(xd, (n,), np.float32), a64 / (1 + np.exp(-a64))) <= 1e-6
    xd2 = up(dev, a)
    dev.lib.cuda_relu(xd2, n)
    assert np.array_equal(dev.download(xd2, (n,), np.float32), np.maximum(a, 0))
    dev.check()
    for p in (ad, bd, od, xd, xd2):
        dev.free(p)


@pytest.mark.parametrize("n", [4096, 8192, 11008])
def test_rms_norm(dev, n):
    x = synth.activation(n, 5) * 3
    w = 1 + 0.1 * synth.activation(n, 6)
    xd, wd, od = up(dev, x), up(dev, w), dev.alloc(n * 4)
    dev.lib.cuda_rms_norm(od, xd, wd, n, np.float32(1e-5))
    x64 = x.astype(np.float64)
    r = x64 / np.sqrt((x64 ** 2).mean() + 1e-5) * w
    assert rel_err(dev.download(od, (n,), np.float32), r) <= 1e-5
    dev.check()
    for p in (xd, wd, od):
        dev.free(p)


def test_softmax(dev):
    n = 32000
    x = synth.activation(n, 7) * 5
    xd, od = up(dev, x), dev.alloc(n * 4)
    dev.lib.cuda_softmax(od, xd, n)
    e = np.exp(x.astype(np.float64) - x.max())
    assert rel_err(dev.download(od, (n,), np.float32), e / e.sum()) <= 1e-5
    dev.check()
    dev.free(xd)
    dev.free(od)


def rope_ref(v, pos, hd, base):
    v = v.astype(np.float64).reshape(-1, hd).copy()
    half = hd // 2
    i = np.arange(half)
    # float32 angle as in src/ai/llm.c:1139-1141, with a correctly rounded pow,
    # cos and sin (fp64 rounded once to float32)
    ex = (2 * i).astype(np.float32) / np.float32(hd)
    pw = np.power(np.float64(base), ex.astype(np.float64)).astype(np.float32)
    freq = (np.float32(1.0) / pw).astype(np.float32)
    th = (np.float32(pos) * freq).astype(np.float32).astype(np.float64)
    c, s = np.cos(th).astype(np.float32).astype(np.float64), np.sin(th).astype(np.float32).astype(np.float64)
    a, b = v[:, :half].copy(), v[:, half:].copy()
    v[:, :half] = a * c - b * s
    v[:, half:] = a * s + b * c
    return v.reshape(-1)


@pytest.mark.parametrize("pos,base", [(0, 10000.0), (17, 10000.0), (2047, 10000.0), (4000, 500000.0)])
def test_rope(dev, reference, pos, base):
    """Against the reference's own rope_apply (src/ai/tensor.c:347, glibc libm).
    The angle is pos * freq in float32, so a one-ulp difference of powf between
    two libms moves it by up to pos * ulp(freq): the bound grows with pos."""
    hd, nh, nkv = 128, 32, 8
    q, k = synth.activation(nh * hd, 8), synth.activation(nkv * hd, 9)
    qd, kd = up(dev, q), up(dev, k)
    dev.lib.cuda_rope_apply(qd, kd, pos, hd, nh, nkv, np.float32(base))
    tol = 2e-6 + 1.5e-7 * pos
    assert np.abs(dev.download(qd, (nh * hd,), np.float32) - reference.rope(q, pos, hd, nh, base)).max() <= tol
    assert np.abs(dev.download(kd, (nkv * hd,), np.float32) - reference.rope(k, pos, hd, nkv, base)).max() <= tol
    # and against the correctly rounded restatement: the same angle bits
    assert np.abs(dev.download(qd, (nh * hd,), np.float32) - rope_ref(q, pos, hd, base)).max() <= 1e-6
    dev.check()
    dev.free(qd)
    dev.free(kd)


def attention_ref(q, kc, vc, kv_len, hd, nh, nkv):
    """src/ai/llm.c:1173-1203 in fp64."""
    out = np.zeros(nh * hd)
    group = nh // nkv
    for h in range(nh):
        kvh = h // group
        qh = q[h * hd:(h + 1) * hd].astype(np.float64)
        K = kc[:kv_len, kvh * hd:(kvh + 1) * hd].astype(np.float64)
        V = vc[:kv_len, kvh * hd:(kvh + 1) * hd].astype(np.float64)
        s = K @ qh / np.sqrt(hd)
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h * hd:(h + 1) * hd] = p @ V
    return out


@pytest.mark.parametrize("kv_len,nh,nkv", [(1, 32, 32), (129, 32, 32), (2048, 32, 32), (777, 64, 8)])
def test_multi_head_attention(dev, kv_len, nh, nkv):
    hd, max_seq = 128, 2048
    q = synth.activation(nh * hd, 10)
    kc = synth.activation(max_seq * nkv * hd, 11).reshape(max_seq, nkv * hd)
    vc = synth.activation(max_seq * nkv * hd, 12).reshape(max_seq, nkv * hd)
    qd, kd, vd, od = up(dev, q), up(dev, kc), up(dev, vc), dev.alloc(nh * hd * 4)
    dev.lib.cuda_multi_head_attention(od, qd, kd, vd, kv_len, hd, nh, nkv)
    got = dev.download(od, (nh * hd,), np.float32)
    dev.check()
    assert rel_err(got, attention_ref(q, kc, vc, kv_len, hd, nh, nkv)) <= 1e-4
    # single-head entry point on KV head 3
    dev.lib.cuda_attention_single(od, qd, kd, vd, None, kv_len, hd, min(3, nkv - 1), nkv * hd)
    got1 = dev.download(od, (hd,), np.float32)
    kvh = min(3, nkv - 1)
    ref1 = attention_ref(q[:hd], kc[:, kvh * hd:(kvh + 1) * hd], vc[:, kvh * hd:(kvh + 1) * hd], kv_len, hd, 1, 1)
    assert rel_err(got1, ref1) <= 1e-4
    for p in (qd, kd, vd, od):
        dev.free(p)


def test_attention_scores_apply(dev):
    seq, kv, hd = 3, 1500, 64
    Q, K, V = synth.activation(seq * hd, 13), synth.activation(kv * hd, 14), synth.activation(kv * hd, 15)
    Qd, Kd, Vd, Sd, Od = up(dev, Q), up(dev, K), up(dev, V), dev.alloc(seq * kv * 4), dev.alloc(seq * hd * 4)
    dev.lib.cuda_attention_scores(Sd, Qd, Kd, seq, kv, hd, np.float32(0.125))
    S = dev.download(Sd, (seq, kv), np.float32)
    Sr = (Q.reshape(seq, hd).astype(np.float64) @ K.reshape(kv, hd).T) * 0.125
    assert rel_err(S, Sr) <= 1e-5
    dev.lib.cuda_attention_apply(Od, Sd, Vd, seq, kv, hd)
    O = dev.download(Od, (seq, hd), np.float32)
    assert rel_err(O, S.astype(np.float64) @ V.reshape(kv, hd)) <= 1e-5
    dev.check()
    for p in (Qd, Kd, Vd, Sd, Od):
        dev.free(p)


@pytest.mark.parametrize("layout", [hb.Q4K_REF, hb.Q4K_GGML], ids=["quant_c", "ggml"])
def test_q4_k_and_q6_k_embeddings(dev, reference, layout):
    """cuda_get_embedding_q4_k (no Q4_K case in the reference's dispatcher)
    in both Q4_K packings, and cuda_get_embedding_q6_k: bit-exact with the
    reference's dequantize_row_q4_k / _q6_k of the same row."""
    from test_oracle_pin import ggml_from_ref
    vocab, dim = 300, 512
    table = synth.quant_matrix(hb.Q4_K, vocab, dim, 18)
    stored = ggml_from_ref(table) if layout == hb.Q4K_GGML else table
    q6 = synth.quant_matrix(hb.Q6_K, vocab, dim, 19)
    old = dev.lib.cuda_get_q4k_layout()
    dev.lib.cuda_set_q4k_layout(layout)
    try:
        td, t6, od = up(dev, stored), up(dev, q6), dev.alloc(dim * 4)
        for tok in (0, 77, vocab - 1):
            dev.lib.cuda_get_embedding_q4_k(od, td, tok, dim, vocab)
            rb = hb.row_bytes(hb.Q4_K, dim)
            want = reference.dequant(hb.Q4_K, table[tok * rb:(tok + 1) * rb], 1, dim)[0]
            assert np.array_equal(dev.download(od, (dim,), np.float32).view(np.uint32), want.view(np.uint32))
            dev.lib.cuda_get_embedding_q6_k(od, t6, tok, dim, vocab)
            rb = hb.row_bytes(hb.Q6_K, dim)
            want = reference.dequant(hb.Q6_K, q6[tok * rb:(tok + 1) * rb], 1, dim)[0]
            assert np.array_equal(dev.download(od, (dim,), np.float32).view(np.uint32), want.view(np.uint32))
        dev.check()
        for p in (td, t6, od):
            dev.free(p)
    finally:
        dev.lib.cuda_set_q4k_layout(old)


@pytest.mark.parametrize("gtype", [hb.F16, hb.Q8_0, hb.Q4_0])
def test_embeddings(dev, reference, gtype):
    vocab, dim = 300, 4096
    if gtype == hb.F16:
        table = synth.f16_matrix(vocab, dim, 16).view(np.uint8).reshape(-1)
        fn = dev.lib.cuda_get_embedding_f16
    else:
        table = synth.quant_matrix(gtype, vocab, dim, 16)
        fn = dev.lib.cuda_get_embedding_q8_0 if gtype == hb.Q8_0 else dev.lib.cuda_get_embedding_q4_0
    td, od = up(dev, table), dev.alloc(dim * 4)
    for tok in (0, 123, vocab - 1):
        fn(od, td, tok, dim, vocab)
        got = dev.download(od, (dim,), np.float32)
        if gtype == hb.F16:
            want = table.view(np.float16).reshape(vocab, dim)[tok].astype(np.float32)
        else:
            rb = hb.row_bytes(gtype, dim)
            want = reference.dequant(gtype, table[tok * rb:(tok + 1) * rb], 1, dim)[0]
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    dev.check()
    dev.free(td)
    dev.free(od)


def test_argmax_first_maximum(dev):
    n = 128256
    x = synth.activation(n, 17)
    x[5000] = x[90000] = x[127000] = 50.0   # ties: the first index wins (tensor.c:460-470)
    xd = up(dev, x)
    assert dev.lib.cuda_argmax(xd, n) == 5000
    assert dev.lib.cuda_argmax(xd, 3000) == int(np.argmax(x[:3000]))
    dev.check()
    dev.free(xd)


def test_memory_helpers(dev):
    a = np.arange(1000, dtype=np.float32)
    ad, bd = up(dev, a), dev.alloc(4000)
    dev.lib.cuda_memcpy_d2d(bd, ad, 4000)
    assert np.array_equal(dev.download(bd, (1000,), np.float32), a)
    dev.lib.cuda_memset(bd, 0, 4000)
    assert not dev.download(bd, (1000,), np.float32).any()
    dev.lib.cuda_memcpy_d2d_async(bd, ad, 4000)
    dev.lib.cuda_sync_copy()
    assert np.array_equal(dev.download(bd, (1000,), np.float32), a)
    assert dev.lib.cuda_available() and dev.lib.cuda_get_device_count() >= 1
    assert dev.lib.cuda_get_free_memory() > 0 and dev.lib.cuda_sm_count() > 0
    dev.check()
    dev.free(ad)
    dev.free(bd)
