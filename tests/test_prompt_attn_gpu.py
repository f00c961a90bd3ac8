"""Causal prompt attention on the tensor cores (csrc/prompt_attn.cu,
pf_attn_tc_kernel: fp16 cache, head_dim 128) against the SIMT kernel it
replaces (pf_attn_kernel, selected with HOLO_PROMPT_ATTN=simt in a child
process) and the reference engine's llm_forward.

The tensor-core kernel rounds the queries and the softmax weights to fp16
(fp32 accumulation); the SIMT kernel keeps them fp32.  Bars: over the logits
of every prompt position checked, the tensor-core engine's distance to the
reference's fp32 logits (norm-wise) is within 1.25x (max) of the SIMT
engine's own distance, plus 1e-3 -- both engines are Q8 engines with an fp16
cache, so the shared part of that distance is the Q8 quantizer's; and the two
engines' logits agree within 5e-2 norm-wise.  Cases: one key tile (127
positions), several tiles (300), a prompt longer than one pass (two passes of
up to 1024 rows, 1100 positions: the second pass reads the first's keys), a
GQA group of 4 query heads per KV head, and a batch of 3 sequences.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

import holo_b200 as hb
from holo_b200 import synth
from holo_b200.model import Model
from conftest import ROOT, rel_err
from holo_oracle import RefModel

pytestmark = pytest.mark.gpu

CFG = dict(n_layers=2, dim=1024, n_heads=8, n_kv_heads=2, head_dim=128, ffn_dim=1024, vocab=1000, max_seq=1200,
           rope_base=10000.0, eps=1e-5, layer_type=hb.Q4_K, emb_type=1, out_type=hb.Q8_0)
CHILD = r"""
import json, sys
import numpy as np
sys.path[:0] = [sys.argv[1] + '/google-classic_b200', sys.argv[1] + '/tests']
import holo_b200 as hb
from holo_b200 import synth
from holo_b200.model import Model
cfg, n, batch, seed = json.loads(sys.argv[2]), int(sys.argv[3]), int(sys.argv[4]), int(sys.argv[5])
hb.Device(0, 1)
w = synth.llama_weights(cfg, seed=seed)
m = Model(cfg, act_mode=hb.ACT_Q8, kv_f16=True, batch=batch)
m.set_weights(w)
toks = np.random.default_rng(seed + 1).integers(0, cfg['vocab'], size=(batch, n)).astype(np.int32)
y = m.prefill(toks if batch > 1 else toks[0])
np.save(sys.argv[6], y)
"""


def _engine_logits(tmp_path, cfg, n, batch, seed, simt):
    out = tmp_path / f"y_{'simt' if simt else 'tc'}_{n}_{batch}.npy"
    env = dict(os.environ, HOLO_PROMPT_ATTN="simt" if simt else "tc")
    p = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), json.dumps(cfg), str(n), str(batch), str(seed),
                        str(out)], env=env, capture_output=True, text=True, timeout=240)
    assert p.returncode == 0, p.stderr[-3000:]
    return np.load(out)


@pytest.mark.parametrize("n,batch,cfg_over", [
    (127, 1, {}), (300, 1, {}), (1100, 1, {}), (200, 1, dict(n_kv_heads=8)), (150, 3, {}),
])
def test_tensor_core_prompt_attention(dev, reference, tmp_path, n, batch, cfg_over):
    cfg = dict(CFG, **cfg_over)
    seed = 7 + n
    tc = _engine_logits(tmp_path, cfg, n, batch, seed, simt=False)
    simt = _engine_logits(tmp_path, cfg, n, batch, seed, simt=True)
    w = synth.llama_weights(cfg, seed=seed)
    toks = np.random.default_rng(seed + 1).integers(0, cfg["vocab"], size=(batch, n)).astype(np.int32)
    tc, simt = tc.reshape(batch, -1), simt.reshape(batch, -1)
    worst = []
    for b in range(batch):
        ref = RefModel(reference, cfg, w)
        for t in toks[b]:
            r = ref.forward(int(t))
        ref.close()
        worst.append((rel_err(tc[b], r), rel_err(simt[b], r), rel_err(tc[b], simt[b])))
    d_tc = max(a for a, _, _ in worst)
    d_simt = max(b for _, b, _ in worst)
    d_pair = max(c for _, _, c in worst)
    print(f"prompt {n} x {batch}: distance to the reference tensor cores {d_tc:.3e}, SIMT {d_simt:.3e}; "
          f"tensor cores vs SIMT {d_pair:.3e}")
    assert d_tc <= 1.25 * d_simt + 1e-3
    assert d_pair <= 5e-2
