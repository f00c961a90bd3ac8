"""Generates tests/golden/stream_7b_f32.json: the reference's own greedy token
stream on the full Llama-2-7B-shape model of BASELINE configs[3].

The weights are made on the GPU by cuda_synth_weights (seed 0, N(0, 0.02),
quantized round-to-nearest into GGUF Q4_K layers, a Q8_0 output matrix and
fp16 embeddings), copied back to the host, and handed to the REFERENCE's own
llm_forward / llm_sample (src/ai/llm.c:1015, 1281; compiled from source into
oracle/_ref/libholo_ref.so by oracle/Makefile) through llm_generate's loop
(llm.c:1340-1420) at temperature 0 with repetition penalty 1.1 over the last
64 tokens.  The reference runs Q4_K matvecs on one core, so this takes a few
minutes (about 4 s a position on the GPU box's host).  Run on a machine with
a B200 and the prebuilt oracle/_ref:

    python tests/golden/make_golden_7b_stream.py [out.json]

The fixture records the prompt, the 64 greedy tokens, the reference's
top-1/top-2 logit margin before each pick, the logits of the last prompt
position and of the last step, and CRC-32s of two generated tensors, so a
change of the generator shows up as such (tests/test_decode_7b_gpu.py).
"""
import base64
import json
import pathlib
import sys
import time
import zlib

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "google-classic_b200"))
sys.path.insert(0, str(ROOT / "oracle"))

import holo_b200 as hb  # noqa: E402
from holo_b200.model import LLAMA2_7B, synthetic_model  # noqa: E402
import holo_oracle  # noqa: E402

SEED = 0
N_PROMPT = 16
N_NEW = 64
PENALTY, LAST_N = 1.1, 64
CFG = dict(LLAMA2_7B, max_seq=N_PROMPT + N_NEW + 8)


def prompt_ids():
    return np.random.default_rng(SEED).integers(0, CFG["vocab"], size=N_PROMPT).astype(np.int32)


def f32_b64(a):
    """float32 little-endian bytes, base64 (decode with np.frombuffer)."""
    return base64.b64encode(np.ascontiguousarray(a, "<f4").tobytes()).decode()


def tensor_crcs(host):
    return {"layer0_wq": zlib.crc32(host["layers"][0]["wq"].tobytes()),
            "output": zlib.crc32(host["output"].tobytes())}


def main(out_path):
    hb.Device(0, 1)
    t0 = time.time()
    m, host = synthetic_model(CFG, seed=SEED, act_mode=hb.ACT_F32, kv_f16=False, keep_host=True)
    m.close()
    print(f"weights made and copied back in {time.time() - t0:.1f} s", flush=True)
    ref = holo_oracle.RefModel(holo_oracle.Reference(), CFG, host)
    p = prompt_ids()
    ref.reset()
    for t in p:
        ref.push(int(t))
    t0 = time.time()
    for t in p:
        logits = ref.forward(int(t))
    last_prompt_logits = logits.copy()
    print(f"prompt: {time.time() - t0:.1f} s", flush=True)
    toks, margins = [], []
    for i in range(N_NEW):
        top2 = np.sort(logits)[-2:]
        margins.append(float(top2[1] - top2[0]))
        tok = ref.sample(0.0, 0.95, 40, PENALTY, LAST_N)
        toks.append(int(tok))
        ref.push(tok)
        logits = ref.forward(tok)
        if i % 8 == 7:
            print(f"step {i + 1}: {time.time() - t0:.1f} s", flush=True)
    rec = {
        "what": "reference llm_forward + llm_sample greedy stream, Llama-2-7B shape (BASELINE configs[3]), "
                "fp32 activations and fp32 KV cache",
        "generator": "cuda_synth_weights (holo_b200.model.synthetic_model), seed 0, std 0.02",
        "cfg": CFG, "seed": SEED, "prompt": [int(t) for t in p], "n_new": N_NEW,
        "sampler": {"temperature": 0.0, "top_p": 0.95, "top_k": 40, "repeat_penalty": PENALTY,
                    "repeat_last_n": LAST_N},
        "tokens": toks, "margins": margins, "crc32": tensor_crcs(host),
        "logits_last_prompt": f32_b64(last_prompt_logits), "logits_last_step": f32_b64(logits),
    }
    pathlib.Path(out_path).write_text(json.dumps(rec))
    ref.close()
    print(f"wrote {out_path}: tokens {toks[:8]}..., smallest margin {min(margins):.3e}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(pathlib.Path(__file__).resolve().parent / "stream_7b_f32.json"))
