"""A GGUF file into the decode engine (holo_b200.gguf.load_model): the model
loaded from the file -- written with general.alignment 64, which the
reference's own loader would misplace -- gives bit-identical logits to the
model built from the same host arrays directly, and its logits match the
reference engine's llm_forward on those arrays (fp32 activations, the bars
of test_decode_gpu)."""
import numpy as np
import pytest

import holo_b200 as hb
from holo_b200 import gguf, synth
from holo_b200.model import Model
from conftest import rel_err
from holo_oracle import RefModel

pytestmark = pytest.mark.gpu

CFG = dict(n_layers=2, dim=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=768, vocab=1000, max_seq=160,
           rope_base=10000.0, eps=1e-5, layer_type=hb.Q4_K, emb_type=1, out_type=hb.Q8_0)


def test_gguf_model_matches_direct_and_reference(dev, reference, tmp_path):
    w = synth.llama_weights(CFG, seed=17)
    path = tmp_path / "model.gguf"
    gguf.write_model(path, CFG, w, alignment=64)
    mf = gguf.load_model(path, act_mode=hb.ACT_F32, kv_f16=False)
    md = Model(CFG, act_mode=hb.ACT_F32, kv_f16=False)
    md.set_weights(w)
    ref = RefModel(reference, CFG, w)
    toks = np.random.default_rng(3).integers(0, CFG["vocab"], size=12)
    worst_abs = worst_rel = 0.0
    for t in toks:
        yf, yd, r = mf.forward(int(t)), md.forward(int(t)), ref.forward(int(t))
        assert np.array_equal(yf, yd)
        worst_abs = max(worst_abs, float(np.abs(yf - r).max()))
        worst_rel = max(worst_rel, rel_err(yf, r))
    ref.close()
    mf.close()
    md.close()
    print(f"GGUF-loaded model vs reference: max abs {worst_abs:.3e}, max rel {worst_rel:.3e}")
    assert worst_abs <= 1e-2 and worst_rel <= 1e-3
