"""Python owner of the decode engine (include/holo_b200.h, holo_model_*).

Mirrors the reference's llm_forward / llm_sample / llm_generate
(src/ai/llm.c:1015, 1281, 1335) on a model object whose weights live on the
device; the arithmetic is the library's (csrc/decode.cu).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import load, ACT_Q8, HOLO_OK


class ModelDesc(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("dim", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("ffn_dim", C.c_int), ("vocab", C.c_int), ("max_seq", C.c_int),
                ("rope_base", C.c_float), ("eps", C.c_float), ("layer_type", C.c_int), ("emb_type", C.c_int),
                ("out_type", C.c_int), ("kv_f16", C.c_int), ("act_mode", C.c_int)]


class SamplerDesc(C.Structure):
    """llm_sampler_t (src/ai/llm.h:167-174) without the seed."""
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int),
                ("repeat_penalty", C.c_float), ("repeat_last_n", C.c_int)]


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class Model:
    """One decode model on the current device (raises on library errors)."""

    def __init__(self, cfg: dict, act_mode: int = ACT_Q8, kv_f16: bool = True):
        self.lib = load()
        self.cfg = dict(cfg)
        d = ModelDesc(cfg["n_layers"], cfg["dim"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"],
                      cfg["ffn_dim"], cfg["vocab"], cfg["max_seq"], cfg.get("rope_base", 10000.0),
                      cfg.get("eps", 1e-5), cfg["layer_type"], cfg.get("emb_type", 1), cfg["out_type"],
                      int(kv_f16), act_mode)
        self.desc = d
        self.h = self.lib.holo_model_create(C.byref(d))
        self._check("holo_model_create", ok=bool(self.h))

    def _check(self, what: str, ok: bool = True):
        st = self.lib.cuda_last_status()
        if st != HOLO_OK or not ok:
            msg = self.lib.cuda_last_status_string().decode(errors="replace")
            self.lib.cuda_clear_status()
            raise RuntimeError(f"{what}: status {st} ({msg})")

    def set_weights(self, w: dict):
        """w: the host arrays of synth.llama_weights (GGUF blocks, fp32 norms)."""
        for l, L in enumerate(w["layers"]):
            rc = self.lib.holo_model_set_layer(self.h, l, _ptr(L["attn_norm"]), _ptr(L["wq"]), _ptr(L["wk"]),
                                               _ptr(L["wv"]), _ptr(L["wo"]), _ptr(L["ffn_norm"]), _ptr(L["w1"]),
                                               _ptr(L["w2"]), _ptr(L["w3"]))
            self._check(f"holo_model_set_layer {l}", rc == HOLO_OK)
        rc = self.lib.holo_model_set_globals(self.h, _ptr(w["tok_emb"]), _ptr(w["final_norm"]), _ptr(w["output"]))
        self._check("holo_model_set_globals", rc == HOLO_OK)

    def forward(self, token: int, want_logits: bool = True) -> np.ndarray | None:
        out = np.empty(self.cfg["vocab"], np.float32) if want_logits else None
        rc = self.lib.holo_model_forward(self.h, int(token), _ptr(out) if want_logits else None)
        self._check("holo_model_forward", rc == HOLO_OK)
        return out

    def load_logits(self, logits: np.ndarray):
        logits = np.ascontiguousarray(logits, np.float32)
        self._check("holo_model_load_logits", self.lib.holo_model_load_logits(self.h, _ptr(logits)) == HOLO_OK)

    def push_token(self, token: int):
        self._check("holo_model_push_token", self.lib.holo_model_push_token(self.h, int(token)) == HOLO_OK)

    def sample(self, s: SamplerDesc, r: float) -> int:
        tok = self.lib.holo_model_sample(self.h, C.byref(s), float(r))
        self._check("holo_model_sample", tok >= 0)
        return tok

    def generate(self, prompt, n_new: int, s: SamplerDesc, seed: int) -> np.ndarray:
        prompt = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(n_new, np.int32)
        n = self.lib.holo_model_generate(self.h, _ptr(prompt), len(prompt), n_new, C.byref(s), seed, _ptr(out))
        self._check("holo_model_generate", n == n_new)
        return out

    def reset(self):
        self.lib.holo_model_reset(self.h)

    def close(self):
        if self.h:
            self.lib.holo_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
