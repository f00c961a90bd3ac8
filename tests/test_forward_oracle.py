"""The end-to-end restatement of llm_forward (oracle/holo_forward.c) pinned to
the reference's own llm_forward, compiled from source (CPU only).

* HOLO_ACT_F32 with an fp32 KV cache is the reference's arithmetic: logits
  must be bit-identical at every position, for each layer type, GQA, and the
  per-tensor types of mixed files (wv / w2 in another type, llm.c:335-342).
* HOLO_ACT_Q8 (the device engine's default) swaps every matmul_q for the
  pinned Q8 matvec restatement: it must stay close to the reference (the
  activation quantization error) and be deterministic.
* The greedy loop helper reproduces the reference's own llm_generate stream
  when fed the reference's logits.
"""
import numpy as np
import pytest

import holo_b200 as hb
from holo_b200 import synth
from holo_oracle import ForwardModel, RefModel, greedy_stream
from conftest import rel_err, typed_weights

BASE = dict(n_layers=2, dim=256, n_heads=4, n_kv_heads=2, head_dim=64, ffn_dim=512, vocab=300, max_seq=48,
            rope_base=10000.0, eps=1e-5, layer_type=hb.Q4_K, emb_type=1, out_type=hb.Q8_0)


def _weights(cfg, seed):
    return typed_weights(cfg, seed)


def _tokens(cfg, n, seed):
    return np.random.default_rng(seed).integers(0, cfg["vocab"], size=n)


@pytest.mark.parametrize("over", [
    dict(layer_type=hb.Q4_K),
    dict(layer_type=hb.Q4_0, out_type=hb.Q4_0),
    dict(layer_type=hb.Q8_0, n_kv_heads=4),
    dict(layer_type=hb.Q6_K, out_type=hb.Q6_K, emb_type=0),
    dict(layer_type=hb.Q4_K, wv_type=hb.Q6_K, w2_type=hb.Q6_K, out_type=hb.Q6_K),   # Q4_K_M-style mix
    dict(layer_type=hb.Q4_0, n_kv_heads=1, head_dim=128, n_heads=2, dim=256),
    # per-layer wv / w2 types and a Q4_K embedding table (Q4_K_M-style file)
    dict(layer_type=hb.Q4_K, wv_types=[hb.Q6_K, hb.Q4_K], w2_types=[hb.Q4_K, hb.Q6_K], out_type=hb.Q6_K,
         emb_type=hb.Q4_K),
])
def test_f32_forward_bit_identical_to_reference(reference, over):
    cfg = dict(BASE, **over)
    w = _weights(cfg, 21)
    ref = RefModel(reference, cfg, w)
    fwd = ForwardModel(cfg, w, hb.ACT_F32, kv_f16=False)
    for i, t in enumerate(_tokens(cfg, 24, 5)):
        r = ref.forward(int(t))
        y = fwd.forward(int(t))
        assert np.array_equal(y.view(np.uint32), r.view(np.uint32)), \
            f"position {i}: max abs diff {np.abs(y - r).max():.3e}"
    ref.close()
    fwd.close()


def test_q8_forward_close_to_reference_and_deterministic(reference):
    cfg = dict(BASE)
    w = _weights(cfg, 22)
    ref = RefModel(reference, cfg, w)
    a = ForwardModel(cfg, w, hb.ACT_Q8, kv_f16=True, threads=4)
    b = ForwardModel(cfg, w, hb.ACT_Q8, kv_f16=True, threads=1)
    worst = 0.0
    for t in _tokens(cfg, 24, 6):
        r = ref.forward(int(t))
        ya, yb = a.forward(int(t)), b.forward(int(t))
        assert np.array_equal(ya, yb)          # row threads change nothing
        worst = max(worst, rel_err(ya, r))
    # Q8 activations move each matvec by ~0.5 % of its output scale
    assert 1e-5 < worst <= 5e-2, worst
    for m in (ref, a, b):
        m.close()


def test_greedy_loop_reproduces_reference_generate(reference):
    """greedy_stream (logits from any forward, the reference's sampler) fed
    the reference's own llm_forward gives RefModel.generate's stream."""
    cfg = dict(BASE)
    w = _weights(cfg, 23)
    ref_gen = RefModel(reference, cfg, w)
    ref_fwd = RefModel(reference, cfg, w)
    ref_smp = RefModel(reference, cfg, w)
    p = _tokens(cfg, 8, 7)
    want = ref_gen.generate(p, 16, 0.0, 0.95, 40, 1.1, 64, seed=1)
    margins = []
    got = greedy_stream(ref_fwd, ref_smp, p, 16, 1.1, 64, margins=margins)
    assert np.array_equal(got, want)
    assert len(margins) == 16 and min(margins) >= 0.0
    for m in (ref_gen, ref_fwd, ref_smp):
        m.close()
