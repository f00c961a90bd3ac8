"""Generates tests/golden/greedy64_7b_q8.json: the one-GPU greedy stream of
bench.py's 7B decode model (Llama-2-7B shape, Q4_K
layers, Q8_0 output matrix, fp16 embeddings and KV cache, HOLO_ACT_Q8; weights
cuda_synth_weights seed 0; the bench's 128-token prompt), 64 steps at
temperature 0 with repetition penalty 1.1 over the last 64 tokens.

bench.py --gpus N regenerates the stream on the row-sharded model and reports
whether it equals this one (greedy64_equal_1gpu).  Run on one B200:

    python tests/golden/make_greedy64_7b.py [out.json]
"""
import json
import pathlib
import sys

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "google-classic_b200"))

import holo_b200 as hb  # noqa: E402
from holo_b200 import model as hm  # noqa: E402
from holo_b200.model import SamplerDesc, synthetic_model  # noqa: E402


def main(out_path):
    hb.Device(0, 1)
    cfg = dict(hm.LLAMA2_7B)
    m = synthetic_model(cfg, seed=0, act_mode=hb.ACT_Q8, kv_f16=True)
    prompt = np.random.default_rng(0).integers(0, cfg["vocab"], size=128).astype(np.int32)
    toks = m.generate(prompt, 64, SamplerDesc(0.0, 0.95, 40, 1.1, 64), seed=0)
    m.close()
    rec = {"what": "one-GPU greedy stream of bench.py's 7B decode model (HOLO_ACT_Q8, fp16 KV cache)",
           "weights": "cuda_synth_weights seed 0", "prompt": "np.random.default_rng(0).integers(0, 32000, 128)",
           "sampler": {"temperature": 0.0, "top_p": 0.95, "top_k": 40, "repeat_penalty": 1.1, "repeat_last_n": 64},
           "tokens": [int(t) for t in toks]}
    pathlib.Path(out_path).write_text(json.dumps(rec, indent=1))
    print(f"wrote {out_path}: {rec['tokens'][:8]}...")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(pathlib.Path(__file__).resolve().parent / "greedy64_7b_q8.json"))
