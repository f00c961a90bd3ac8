"""Prompt passes (holo_model_prefill; csrc/decode.cu enqueue_rows and
pf_attn_kernel, with the tensor-core matmul of csrc/prefill.cu): the positions
of a prompt go through each layer together, every projection one matmul over
the rows, the attention causal over the KV cache.  holo_model_generate runs
the prompt before its last token this way.

The projections multiply fp16 operands (the Q8-quantized activation and the
weight value, each rounded once, fp32 accumulation), as in the batched
decode engine.  Bars, fixed here:
* logits at the end of each prompt segment -- passes that start at position
  0 and later, so the attention reads keys appended by the pass itself and
  keys cached before it -- and at the decode positions that follow (one
  position a step, reading the cache the passes wrote) within 2e-2 of the
  reference engine's llm_forward, norm-wise (max|y - r| / max|r|), with an
  fp32 KV cache; with an fp16 cache (the bench configuration) within 5e-2,
  the batch-1 Q8 engine's bound;
* the same for a prompt longer than one pass (512 positions) and for a GQA
  group of 8 query heads per KV head;
* a batched model passes the prompts of all its sequences together: each
  sequence's logits within 2e-2 of the reference engine on that sequence
  alone, also at the batched decode positions that follow;
* generate with row passes gives the tokens of the same passes followed by
  one step a position (greedy, no penalty), bit for bit.
"""
import numpy as np
import pytest

import holo_b200 as hb
from holo_b200 import synth
from holo_b200.model import Model, SamplerDesc, _ptr
from conftest import rel_err
from holo_oracle import RefModel

pytestmark = pytest.mark.gpu

CFG = dict(n_layers=2, dim=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=768, vocab=1000, max_seq=160,
           rope_base=10000.0, eps=1e-5, layer_type=hb.Q4_K, emb_type=1, out_type=hb.Q8_0)
CFG_G8 = dict(CFG, n_heads=8, n_kv_heads=1, layer_type=hb.Q4_0, out_type=hb.Q4_0)
CFG_LONG = dict(CFG, max_seq=640)


def tokens(cfg, n, seed):
    return np.random.default_rng(seed).integers(0, cfg["vocab"], size=n).astype(np.int32)


def segments_vs_reference(reference, cfg, kv_f16, segs, n_decode, seed):
    w = synth.llama_weights(cfg, seed=seed)
    m = Model(cfg, act_mode=hb.ACT_Q8, kv_f16=kv_f16)
    m.set_weights(w)
    ref = RefModel(reference, cfg, w)
    toks = tokens(cfg, sum(segs) + n_decode, seed + 1)
    worst, pos = 0.0, 0
    for n in segs:
        y = m.prefill(toks[pos:pos + n])
        for t in toks[pos:pos + n]:
            r = ref.forward(int(t))
        worst = max(worst, rel_err(y, r))
        pos += n
    for t in toks[pos:]:
        worst = max(worst, rel_err(m.forward(int(t)), ref.forward(int(t))))
    ref.close()
    m.close()
    return worst


@pytest.mark.parametrize("kv_f16,bound", [(False, 2e-2), (True, 5e-2)], ids=["f32kv", "f16kv"])
def test_prompt_segments_match_reference(dev, reference, kv_f16, bound):
    worst = segments_vs_reference(reference, CFG, kv_f16, [24, 1, 40, 7], 8, seed=31)
    print(f"prompt passes (kv f16 {kv_f16}): max norm-wise rel {worst:.3e}")
    assert worst <= bound


def test_gqa_group_of_8_matches_reference(dev, reference):
    worst = segments_vs_reference(reference, CFG_G8, False, [33, 20], 6, seed=32)
    print(f"GQA 8: max norm-wise rel {worst:.3e}")
    assert worst <= 2e-2


def test_prompt_longer_than_one_pass(dev, reference):
    worst = segments_vs_reference(reference, CFG_LONG, False, [600], 4, seed=33)
    print(f"600-position prompt: max norm-wise rel {worst:.3e}")
    assert worst <= 2e-2


def test_batched_prompts_match_reference(dev, reference):
    cfg = dict(CFG)
    B = 4
    w = synth.llama_weights(cfg, seed=41)
    m = Model(cfg, act_mode=hb.ACT_Q8, kv_f16=False, batch=B)
    m.set_weights(w)
    refs = [RefModel(reference, cfg, w) for _ in range(B)]
    toks = np.random.default_rng(42).integers(0, cfg["vocab"], size=(B, 36 + 5)).astype(np.int32)
    worst, pos = 0.0, 0
    for n in (29, 7):
        y = m.prefill(toks[:, pos:pos + n])
        for b in range(B):
            for t in toks[b, pos:pos + n]:
                r = refs[b].forward(int(t))
            worst = max(worst, rel_err(y[b], r))
        pos += n
    for i in range(pos, toks.shape[1]):
        y = m.forward_batch(toks[:, i])
        for b in range(B):
            worst = max(worst, rel_err(y[b], refs[b].forward(int(toks[b, i]))))
    for r in refs:
        r.close()
    m.close()
    print(f"batched prompt passes: max norm-wise rel {worst:.3e}")
    assert worst <= 2e-2


def test_generate_equals_passes_then_steps(dev):
    w = synth.llama_weights(CFG, seed=34)
    m = Model(CFG, act_mode=hb.ACT_Q8, kv_f16=True)
    m.set_weights(w)
    p = tokens(CFG, 30, 35)
    got = m.generate(p, 12, SamplerDesc(0.0, 0.95, 40, 1.0, 64), seed=1)
    m.reset()
    m.prefill(p[:-1], want_logits=False)
    want, t = [], int(p[-1])
    for _ in range(12):
        t = int(np.argmax(m.forward(t)))
        want.append(t)
    m.close()
    assert np.array_equal(got, np.array(want, np.int32)), (got, want)


def test_prompt_modes_agree(dev):
    """generate with row passes and one position a step: the logits after the
    prompt differ only by the matmul's fp16 operand rounding."""
    w = synth.llama_weights(CFG, seed=36)
    m = Model(CFG, act_mode=hb.ACT_Q8, kv_f16=True)
    m.set_weights(w)
    p = tokens(CFG, 40, 37)
    ys = []
    for rows in (True, False):
        m.set_prompt_mode(rows)
        m.reset()
        if rows:
            m.prefill(p[:-1], want_logits=False)
        else:
            for t in p[:-1]:
                m.forward(int(t), want_logits=False)
        ys.append(m.forward(int(p[-1])))
    m.close()
    err = rel_err(ys[0], ys[1])
    print(f"row passes vs steps: norm-wise rel {err:.3e}")
    assert err <= 2e-2


def test_prefill_rejects(dev):
    w = synth.llama_weights(CFG, seed=38)
    m = Model(CFG, act_mode=hb.ACT_F32, kv_f16=False)   # fp32 activations: no row passes
    m.set_weights(w)
    p = tokens(CFG, 8, 39)
    dev.lib.cuda_clear_status()
    assert dev.lib.holo_model_prefill(m.h, _ptr(p), len(p), None) == hb.HOLO_E_UNSUPPORTED
    dev.lib.cuda_clear_status()
    m.close()
    m = Model(CFG, act_mode=hb.ACT_Q8, kv_f16=True)
    m.set_weights(w)
    long = tokens(CFG, CFG["max_seq"] + 1, 40)
    assert dev.lib.holo_model_prefill(m.h, _ptr(long), len(long), None) == hb.HOLO_E_ARG
    dev.lib.cuda_clear_status()
    m.close()
