"""Per-tensor weight types in the decode engine (holo_model_set_layer_types),
the layout of llama.cpp's Q4_K_M files: attn_q/attn_k/attn_output/ffn_gate/
ffn_up in Q4_K, attn_v and ffn_down in Q6_K on some layers and Q4_K on others,
a Q6_K output matrix and a Q4_K token-embedding table.  The reference binds
wv / w2 types per layer (src/ai/llm.c:445-507) and dispatches each matmul on
its tensor's type (llm.c:1092, 1239; llm_cuda.c:140-163).

Bars (those of test_decode_gpu):
* HOLO_ACT_F32, fp32 KV cache, against the reference's own llm_forward:
  logits within 1e-2 absolute and 1e-3 norm-wise at every position; greedy
  64-step stream identical to the reference's llm_generate loop;
* HOLO_ACT_Q8, fp16 KV cache: the distance to the reference's fp32 logits
  within 1.25x of the Q8 restatement's own (oracle/holo_forward.c), the
  greedy stream the restatement's up to a near tie (the bars of
  test_decode_7b_gpu, which says why);
* the same model written as a GGUF file and loaded by holo_b200.gguf
  .load_model: the reference's greedy stream;
* per-layer types on a sharded or batched model: HOLO_E_UNSUPPORTED.
"""
import numpy as np
import pytest

import holo_b200 as hb
from holo_b200 import gguf
from holo_b200.model import Model, SamplerDesc
from holo_oracle import ForwardModel, RefModel, greedy_stream
from conftest import rel_err, typed_weights

pytestmark = pytest.mark.gpu

CFG = dict(n_layers=3, dim=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=768, vocab=1000, max_seq=128,
           rope_base=10000.0, eps=1e-5, layer_type=hb.Q4_K, emb_type=hb.Q4_K, out_type=hb.Q6_K,
           wv_types=[hb.Q6_K, hb.Q4_K, hb.Q6_K], w2_types=[hb.Q6_K, hb.Q6_K, hb.Q4_K])
GREEDY = SamplerDesc(0.0, 0.95, 40, 1.1, 64)
ABS_TOL, REL_TOL = 1e-2, 1e-3


@pytest.fixture(scope="module")
def weights():
    return typed_weights(CFG, seed=31)


def _prompt(n, seed):
    return np.random.default_rng(seed).integers(0, CFG["vocab"], size=n).astype(np.int32)


def _model(weights, act, kv_f16):
    m = Model(CFG, act_mode=act, kv_f16=kv_f16)
    m.set_weights(weights)
    return m


def test_f32_logits_and_greedy_stream_match_reference(dev, reference, weights):
    m = _model(weights, hb.ACT_F32, False)
    ref = RefModel(reference, CFG, weights)
    worst_abs = worst_rel = 0.0
    for t in _prompt(24, 1):
        y, r = m.forward(int(t)), ref.forward(int(t))
        worst_abs = max(worst_abs, float(np.abs(y - r).max()))
        worst_rel = max(worst_rel, rel_err(y, r))
    p = _prompt(16, 2)
    got = m.generate(p, 64, GREEDY, seed=3)
    margins = []
    want = ref.generate(p, 64, 0.0, 0.95, 40, 1.1, 64, seed=3, margins=margins)
    print(f"mixed types f32: logits max abs {worst_abs:.3e}, norm-wise {worst_rel:.3e}; greedy equal "
          f"{np.array_equal(got, want)}, smallest margin {min(margins):.3e}")
    ref.close()
    m.close()
    assert worst_abs <= ABS_TOL and worst_rel <= REL_TOL
    assert np.array_equal(got, want)


def test_q8_within_quantizer_noise(dev, reference, weights):
    """HOLO_ACT_Q8 / fp16 KV: the device's distance to the reference's fp32
    logits stays within 1.25x of the Q8 restatement's own (max and median
    over the positions), and its greedy stream follows the restatement's Q8
    stream up to a near tie (tests/test_decode_7b_gpu.py explains why Q8
    logits are compared at the quantizer's noise level)."""
    m = _model(weights, hb.ACT_Q8, True)
    q8 = ForwardModel(CFG, weights, hb.ACT_Q8, kv_f16=True, threads=4)
    f32 = ForwardModel(CFG, weights, hb.ACT_F32, kv_f16=False, threads=4)
    smp = RefModel(reference, CFG, weights)
    p = _prompt(16, 4)
    margins, logits = [], []
    want = greedy_stream(q8, smp, p, 64, 1.1, 64, margins=margins, logits_out=logits)
    got = m.generate(p, 64, GREEDY, seed=5)
    m.reset()
    q8.reset()
    dev_rel, res_rel, noise = [], [], 0.0
    for t in np.concatenate([p, want]):
        y, r, ref32 = m.forward(int(t)), q8.forward(int(t)), f32.forward(int(t))
        dev_rel.append(rel_err(y, ref32))
        res_rel.append(rel_err(r, ref32))
        noise = max(noise, float(np.abs(y - r).max()))
    dev_rel, res_rel = np.array(dev_rel), np.array(res_rel)
    print(f"mixed types q8, distance to fp32: device max {dev_rel.max():.3e} median {np.median(dev_rel):.3e}; "
          f"restatement max {res_rel.max():.3e} median {np.median(res_rel):.3e}; noise {noise:.3e}; greedy equal "
          f"{np.array_equal(got, want)}")
    for h in (q8, f32, smp, m):
        h.close()
    assert dev_rel.max() <= 1.25 * res_rel.max() and np.median(dev_rel) <= 1.25 * np.median(res_rel)
    if not np.array_equal(got, want):
        k = int(np.argmax(got != np.array(want)))
        assert margins[k] <= 2 * noise, (k, margins[k], noise)


def test_gguf_file_with_mixed_types_loads_and_matches_reference(dev, reference, weights, tmp_path):
    path = tmp_path / "q4_k_m_style.gguf"
    gguf.write_model(path, CFG, weights)
    with gguf.GGUFFile(path) as g:
        cfg = gguf.model_config(g)
    assert cfg["wv_types"] == CFG["wv_types"] and cfg["w2_types"] == CFG["w2_types"]
    assert cfg["emb_type"] == hb.Q4_K and cfg["out_type"] == hb.Q6_K
    m = gguf.load_model(path, act_mode=hb.ACT_F32, kv_f16=False)
    ref = RefModel(reference, CFG, weights)
    p = _prompt(16, 6)
    got = m.generate(p, 64, GREEDY, seed=7)
    want = ref.generate(p, 64, 0.0, 0.95, 40, 1.1, 64, seed=7)
    ref.close()
    m.close()
    assert np.array_equal(got, want)


@pytest.mark.parametrize("kw", [dict(batch=4), dict(world=2, rank=0)])
def test_per_layer_types_need_one_gpu_batch_1(dev, kw):
    cfg = dict(CFG, emb_type=1, out_type=hb.Q8_0)
    cfg.pop("wv_types")
    cfg.pop("w2_types")
    m = Model(cfg, act_mode=hb.ACT_Q8, kv_f16=True, **kw)
    dev.lib.cuda_clear_status()
    assert dev.lib.holo_model_set_layer_types(m.h, 0, hb.Q6_K, hb.Q4_K) == hb.HOLO_E_UNSUPPORTED
    assert dev.lib.holo_model_set_layer_types(m.h, 0, hb.Q4_K, hb.Q4_K) == hb.HOLO_OK   # uniform is fine
    dev.lib.cuda_clear_status()
    m.close()


def test_bad_layer_type_rejected(dev):
    cfg = dict(CFG, emb_type=1)
    cfg.pop("wv_types")
    cfg.pop("w2_types")
    m = Model(cfg, act_mode=hb.ACT_Q8, kv_f16=True)
    dev.lib.cuda_clear_status()
    assert dev.lib.holo_model_set_layer_types(m.h, 0, hb.F16, hb.Q4_K) == hb.HOLO_E_ARG
    assert dev.lib.holo_model_set_layer_types(m.h, 7, hb.Q4_K, hb.Q4_K) == hb.HOLO_E_ARG
    dev.lib.cuda_clear_status()
    m.close()
