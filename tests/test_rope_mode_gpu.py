"""holo_model_desc.rope_mode = HOLO_ROPE_ADJACENT: RoPE on pairs (2i, 2i+1),
the rotation llama.cpp applies to Llama weights converted to GGUF, where the
reference (and the default, HOLO_ROPE_HALF) rotates (i, i + hd/2).

A model whose q/k weight rows are reordered within each head -- row i from
row 2i, row i + hd/2 from row 2i + 1 -- computes, with rotate-half, the same
rotated vectors up to that reordering, so its attention scores and outputs
are those of the adjacent-pair model on the original rows.  Bar, fixed here:
logits of the two within 1e-4 norm-wise (only summation orders differ) on
the persistent step (head_dim 128), the per-op graph path (head_dim 64) and
prompt passes; the modes differ by far more on the same weights."""
import numpy as np
import pytest

import holo_b200 as hb
from holo_b200 import synth
from holo_b200.model import Model
from conftest import rel_err

pytestmark = pytest.mark.gpu

BASE = dict(n_layers=2, dim=512, n_heads=4, n_kv_heads=2, ffn_dim=768, vocab=1000, max_seq=96,
            rope_base=10000.0, eps=1e-5, layer_type=hb.Q4_K, emb_type=1, out_type=hb.Q8_0)


def half_order(w, cfg):
    """Copy of w with the q and k rows of every head reordered for rotate-half."""
    hd = cfg["head_dim"]
    perm = np.empty(hd, np.int64)
    perm[:hd // 2] = np.arange(0, hd, 2)
    perm[hd // 2:] = np.arange(1, hd, 2)
    rb = hb.row_bytes(cfg["layer_type"], cfg["dim"])
    out = {k: v for k, v in w.items() if k != "layers"}
    out["layers"] = []
    for L in w["layers"]:
        L2 = dict(L)
        for key, heads in (("wq", cfg["n_heads"]), ("wk", cfg["n_kv_heads"])):
            rows = L[key].reshape(heads * hd, rb)
            idx = (np.arange(heads)[:, None] * hd + perm[None, :]).reshape(-1)
            L2[key] = np.ascontiguousarray(rows[idx]).reshape(-1)
        out["layers"].append(L2)
    return out


@pytest.mark.parametrize("head_dim,act", [(128, hb.ACT_F32), (128, hb.ACT_Q8), (64, hb.ACT_F32)],
                         ids=["step-f32", "step-q8", "graph-f32"])
def test_adjacent_pairs_equal_reordered_rotate_half(dev, head_dim, act):
    cfg = dict(BASE, head_dim=head_dim, n_heads=512 // head_dim, n_kv_heads=256 // head_dim)
    w = synth.llama_weights(cfg, seed=51)
    adj = Model(dict(cfg, rope_mode=hb.ROPE_ADJACENT), act_mode=act, kv_f16=False)
    adj.set_weights(w)
    half = Model(cfg, act_mode=act, kv_f16=False)
    half.set_weights(half_order(w, cfg))
    plain = Model(cfg, act_mode=act, kv_f16=False)
    plain.set_weights(w)
    toks = np.random.default_rng(7).integers(0, cfg["vocab"], size=20)
    worst, apart = 0.0, 0.0
    if act == hb.ACT_Q8 and head_dim == 128:   # prompt passes first, then steps
        ya, yh, yp = adj.prefill(toks[:12]), half.prefill(toks[:12]), plain.prefill(toks[:12])
        worst, apart = rel_err(ya, yh), rel_err(ya, yp)
        toks = toks[12:]
    for t in toks:
        ya, yh, yp = adj.forward(int(t)), half.forward(int(t)), plain.forward(int(t))
        worst = max(worst, rel_err(ya, yh))
        apart = max(apart, rel_err(ya, yp))
    for m in (adj, half, plain):
        m.close()
    print(f"hd {head_dim}: adjacent vs reordered rotate-half {worst:.2e}, vs plain rotate-half {apart:.2e}")
    assert worst <= 1e-4
    assert apart > 1e-2


def test_rejects_unknown_rope_mode(dev):
    cfg = dict(BASE, head_dim=128, rope_mode=2)
    dev.lib.cuda_clear_status()
    with pytest.raises(RuntimeError):
        Model(cfg)
    dev.lib.cuda_clear_status()
