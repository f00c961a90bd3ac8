"""The drop-in, run: the reference's own GPU host code (src/ai/llm.c +
llm_cuda.c with HOLO_USE_CUDA, compiled from source by oracle/Makefile
`dropin`) linked against this repository's libholo_cuda.so in place of the
reference's cuda_ops.cu, unchanged.  llm_cuda_init uploads the model with the
reference's upload_tensor (raw GGUF blocks through cuda_malloc +
cuda_memcpy_h2d, llm_cuda.c:189-196) and llm_forward_cuda
(llm_cuda.c:558-946) runs each position through this library's cuda_ops.h
entry points.  Bars (HOLO_ACT_F32, the reference's arithmetic): logits within
1e-2 absolute and 1e-3 norm-wise of the reference's CPU llm_forward at every
position, and the greedy stream of llm_generate's loop identical for 32
steps.

The reference's llm_cuda_cleanup ends with cuda_cleanup(), which releases
this library's state of the device (it is re-created on the next call); the
file name sorts it after the other GPU tests but the no-allocation one.
"""
import numpy as np
import pytest

import holo_b200 as hb
from holo_b200 import synth
from holo_oracle import DROPIN_SO, RefModel, Reference, greedy_stream
from conftest import rel_err

pytestmark = pytest.mark.gpu

CFG = dict(n_layers=2, dim=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=768, vocab=1000, max_seq=64,
           rope_base=10000.0, eps=1e-5, layer_type=hb.Q4_K, emb_type=1, out_type=hb.Q8_0)


class DropinForward:
    """forward/reset over the drop-in library's llm_forward_cuda."""

    def __init__(self, m):
        self.m = m

    def forward(self, t):
        assert self.m.lib.href_cuda_forward(self.m.h, int(t)) == 0
        return np.ctypeslib.as_array(self.m.lib.href_logits(self.m.h), shape=(CFG["vocab"],)).copy()

    def reset(self):
        self.m.lib.href_cuda_reset(self.m.h)


@pytest.mark.parametrize("layer_type", [hb.Q4_K, hb.Q8_0, hb.Q4_0])
def test_reference_gpu_host_path_on_this_library(dev, reference, layer_type):
    if not DROPIN_SO.exists():
        pytest.skip("oracle/_ref/libholo_ref_dropin.so not built")
    cfg = dict(CFG, layer_type=layer_type)
    w = synth.llama_weights(cfg, seed=13)
    before = dev.lib.cuda_get_act_mode()
    dev.lib.cuda_set_act_mode(hb.ACT_F32)
    drop = RefModel(Reference(DROPIN_SO), cfg, w)
    try:
        assert drop.lib.href_cuda_init(drop.h) == 0
        cpu = RefModel(reference, cfg, w)
        fwd = DropinForward(drop)
        fwd.reset()
        worst_abs = worst_rel = 0.0
        for t in np.random.default_rng(3).integers(0, cfg["vocab"], size=24):
            y, r = fwd.forward(t), cpu.forward(int(t))
            worst_abs = max(worst_abs, float(np.abs(y - r).max()))
            worst_rel = max(worst_rel, rel_err(y, r))
        p = np.random.default_rng(4).integers(0, cfg["vocab"], size=12).astype(np.int32)
        got = greedy_stream(fwd, cpu, p, 32, 1.1, 64)
        want = cpu.generate(p, 32, 0.0, 0.95, 40, 1.1, 64, seed=1)
        print(f"drop-in llm_forward_cuda ({hb.TYPE_NAMES[layer_type]} layers) vs CPU llm_forward: max abs "
              f"{worst_abs:.3e}, norm-wise {worst_rel:.3e}; greedy equal {np.array_equal(got, want)}")
        cpu.close()
        assert worst_abs <= 1e-2 and worst_rel <= 1e-3
        assert np.array_equal(got, want)
    finally:
        drop.lib.href_cuda_cleanup()
        drop.close()
        dev.lib.cuda_set_act_mode(before)
        dev.check("drop-in")
