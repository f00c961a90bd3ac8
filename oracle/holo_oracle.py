"""ctypes binding of the checker libraries (TEST INFRASTRUCTURE ONLY).

* ``Oracle``    -> oracle/_build/liboracle.so: the CPU restatement (holo_oracle.c)
* ``Reference`` -> oracle/_ref/libholo_ref.so: the reference engine's own C code
                   compiled from source (oracle/Makefile)

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs import this module; the product library never does.
"""
from __future__ import annotations

import ctypes as C
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "liboracle.so"
REF_SO = HERE / "_ref" / "libholo_ref.so"

_vp, _i, _f = C.c_void_p, C.c_int, C.c_float
_i64 = C.c_int64


def build():
    """Compile the restatement (and the reference, where its sources exist)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class Oracle:
    def __init__(self):
        if not ORACLE_SO.exists():
            build()
        lib = C.CDLL(str(ORACLE_SO))
        lib.ho_f16_to_f32.restype = _f
        lib.ho_f16_to_f32.argtypes = [C.c_uint16]
        lib.ho_f32_to_f16_rn.restype = C.c_uint16
        lib.ho_f32_to_f16_rn.argtypes = [_f]
        lib.ho_row_bytes.restype = _i64
        lib.ho_row_bytes.argtypes = [_i, _i64]
        lib.ho_dequant_row.argtypes = [_i, _vp, _vp, _i64, _i]
        lib.ho_matvec_f32act.argtypes = [_i, _vp, _vp, _vp, _i, _i, _i, _i]
        lib.ho_quantize_act_q8.argtypes = [_vp, _i64, _vp, _vp, _vp]
        lib.ho_matvec_q8act.argtypes = [_i, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp, _i]
        lib.ho_q4k_to_ref_layout.argtypes = [_vp, _vp, _i]
        lib.ho_tokenize.restype = _i
        lib.ho_tokenize.argtypes = [C.POINTER(C.c_char_p), _i, _i, _i, C.c_char_p, C.POINTER(_i), _i, _i]
        self.lib = lib

    def dequant(self, gtype, blocks, rows, cols, q4k_layout=0):
        blocks = np.ascontiguousarray(blocks)
        out = np.empty((rows, cols), np.float32)
        rb = self.lib.ho_row_bytes(gtype, cols)
        for r in range(rows):
            self.lib.ho_dequant_row(gtype, _ptr(blocks) + r * rb, _ptr(out) + r * cols * 4, cols, q4k_layout)
        return out

    def matvec_f32(self, gtype, blocks, x, rows, cols, q4k_layout=0, threads=1):
        blocks = np.ascontiguousarray(blocks)
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(rows, np.float32)
        self.lib.ho_matvec_f32act(gtype, _ptr(blocks), _ptr(x), _ptr(y), rows, cols, q4k_layout, threads)
        return y

    def quantize_act(self, x):
        x = np.ascontiguousarray(x, np.float32)
        n = x.size
        q = np.empty(n, np.int8)
        d = np.empty(n // 32, np.float32)
        s = np.empty(n // 32, np.int32)
        self.lib.ho_quantize_act_q8(_ptr(x), n, _ptr(q), _ptr(d), _ptr(s))
        return q, d, s

    def matvec_q8(self, gtype, blocks, x, rows, cols, q4k_layout=0, want_isums=False, threads=1):
        blocks = np.ascontiguousarray(blocks)
        q, d, s = self.quantize_act(x)
        y = np.empty(rows, np.float32)
        isums = np.empty((rows, cols // 32), np.int32) if want_isums else None
        self.lib.ho_matvec_q8act(gtype, _ptr(blocks), _ptr(q), _ptr(d), _ptr(s), _ptr(y), rows, cols,
                                 q4k_layout, _ptr(isums) if want_isums else None, threads)
        return (y, isums) if want_isums else y

    def q4k_to_ref(self, blocks, layout):
        blocks = np.ascontiguousarray(blocks).reshape(-1, 144)
        out = np.empty_like(blocks)
        for i in range(blocks.shape[0]):
            self.lib.ho_q4k_to_ref_layout(_ptr(blocks) + i * 144, _ptr(out) + i * 144, layout)
        return out.reshape(-1)

    def tokenize(self, vocab, bos, unk, text, max_tokens=None, add_bos=False):
        """llm_tokenize restated (ho_tokenize): the whole vocabulary scanned at
        every position -- small vocabularies only."""
        return _tok_call(self.lib.ho_tokenize, vocab, bos, unk, text, max_tokens, add_bos)


def _tok_call(fn, vocab, bos, unk, text, max_tokens, add_bos):
    """fn(vocab**, size, bos, unk, text, out*, max_tokens, add_bos) -> ids"""
    enc = [v.encode() if isinstance(v, str) else v for v in vocab]
    arr = (C.c_char_p * max(len(enc), 1))(*enc)
    b = text.encode() if isinstance(text, str) else bytes(text)
    cap = len(b) + 1 if max_tokens is None else int(max_tokens)
    out = (_i * max(cap, 1))()
    n = fn(arr, len(enc), int(bos), int(unk), b, out, cap, int(add_bos))
    return np.array(out[:n], np.int32)


def layer_types(cfg: dict):
    """(wv type, w2 type) of every layer: cfg's per-layer lists wv_types /
    w2_types, else wv_type / w2_type, else layer_type."""
    lt, n = cfg["layer_type"], cfg["n_layers"]
    wv = cfg.get("wv_types") or [cfg.get("wv_type", lt)] * n
    w2 = cfg.get("w2_types") or [cfg.get("w2_type", lt)] * n
    return list(zip(wv, w2))


class ForwardModel:
    """llm_forward restated (holo_forward.c, ho_fwd_*): one position per
    forward() call, in the device engine's activation mode (HOLO_ACT_F32 = 0,
    HOLO_ACT_Q8 = 1, as include/holo_b200.h numbers them) and KV precision.  `w` holds the host arrays of
    holo_b200.synth.llama_weights (or synthetic_model(keep_host=True)); they
    are kept alive here because the restatement reads them in place.
    cfg may carry wv_type / w2_type (per-tensor types, llm.c:335-342)."""

    def __init__(self, cfg: dict, w: dict, act_mode: int, kv_f16: bool, threads: int = 1):
        lib = Oracle().lib
        lib.ho_fwd_create.restype = _vp
        lib.ho_fwd_create.argtypes = [_i] * 8 + [_f, _f, _i, _i, _i]
        lib.ho_fwd_set_types.argtypes = [_vp] + [_i] * 5
        lib.ho_fwd_set_layer.argtypes = [_vp, _i] + [_vp] * 9
        lib.ho_fwd_set_layer_types.argtypes = [_vp, _i, _i, _i]
        lib.ho_fwd_set_globals.argtypes = [_vp, _vp, _vp, _vp]
        lib.ho_fwd_forward.restype = _i
        lib.ho_fwd_forward.argtypes = [_vp, _i]
        lib.ho_fwd_logits.restype = C.POINTER(C.c_float)
        lib.ho_fwd_logits.argtypes = [_vp]
        lib.ho_fwd_reset.argtypes = [_vp]
        lib.ho_fwd_free.argtypes = [_vp]
        self.lib, self.cfg, self.w = lib, dict(cfg), w
        self.h = lib.ho_fwd_create(cfg["n_layers"], cfg["dim"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"],
                                   cfg["ffn_dim"], cfg["vocab"], cfg["max_seq"], cfg.get("rope_base", 10000.0),
                                   cfg.get("eps", 1e-5), int(act_mode), int(bool(kv_f16)), int(threads))
        if not self.h:
            raise MemoryError("ho_fwd_create")
        lt = cfg["layer_type"]
        lib.ho_fwd_set_types(self.h, lt, cfg.get("wv_type", lt), cfg.get("w2_type", lt), cfg.get("emb_type", 1),
                             cfg["out_type"])
        for l, (tv, t2) in enumerate(layer_types(cfg)):
            lib.ho_fwd_set_layer_types(self.h, l, tv, t2)
        for l, L in enumerate(w["layers"]):
            lib.ho_fwd_set_layer(self.h, l, _ptr(L["attn_norm"]), _ptr(L["wq"]), _ptr(L["wk"]), _ptr(L["wv"]),
                                 _ptr(L["wo"]), _ptr(L["ffn_norm"]), _ptr(L["w1"]), _ptr(L["w2"]), _ptr(L["w3"]))
        lib.ho_fwd_set_globals(self.h, _ptr(w["tok_emb"]), _ptr(w["final_norm"]), _ptr(w["output"]))

    def forward(self, token: int) -> np.ndarray:
        if self.lib.ho_fwd_forward(self.h, int(token)) != 0:
            raise ValueError(f"ho_fwd_forward({token}): bad token or full cache")
        return np.ctypeslib.as_array(self.lib.ho_fwd_logits(self.h), shape=(self.cfg["vocab"],)).copy()

    def reset(self):
        self.lib.ho_fwd_reset(self.h)

    def close(self):
        if self.h:
            self.lib.ho_fwd_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def greedy_stream(fwd, ref_model, prompt, n_new: int, penalty: float, last_n: int, margins=None, logits_out=None):
    """llm_generate's loop (src/ai/llm.c:1340-1420) at temperature 0 with the
    logits of `fwd` (ForwardModel, or anything with forward/reset) and the
    reference's own llm_sample (`ref_model`, a RefModel used for its sampler
    and token history only).  margins collects top-1 minus top-2 of the
    penalised logits before each pick; logits_out the logits of every
    position (prompt and generated)."""
    fwd.reset()
    ref_model.reset()
    hist = [int(t) for t in prompt]
    for t in prompt:
        ref_model.push(t)
    for t in prompt:
        logits = fwd.forward(t)
        if logits_out is not None:
            logits_out.append(logits)
    out = []
    for _ in range(n_new):
        ref_model.set_logits(logits)
        if margins is not None:
            margins.append(penalised_margin(logits, hist[-last_n:] if last_n > 0 else [], penalty))
        tok = ref_model.sample(0.0, 0.95, 40, penalty, last_n)
        out.append(tok)
        hist.append(tok)
        ref_model.push(tok)
        logits = fwd.forward(tok)
        if logits_out is not None:
            logits_out.append(logits)
    return np.array(out, np.int32)


def penalised_margin(logits, hist, penalty):
    """top-1 minus top-2 of the logits after the repetition penalty of
    tensor.c:654-667 over the history tokens `hist` (a diagnostic)."""
    lg = np.asarray(logits, np.float32).copy()
    for t in hist:
        lg[t] = lg[t] / np.float32(penalty) if lg[t] > 0 else lg[t] * np.float32(penalty)
    top2 = np.sort(lg)[-2:]
    return float(top2[1] - top2[0])


DROPIN_SO = HERE / "_ref" / "libholo_ref_dropin.so"


class Reference:
    """The reference engine's own CPU functions (src/ai/*.c built from source).
    path = DROPIN_SO: the drop-in build of the same code, whose GPU host path
    (llm_cuda.c) runs on this repository's libholo_cuda.so (href_cuda_*)."""

    def __init__(self, path=None):
        so = pathlib.Path(path) if path else REF_SO
        if not so.exists() and not path:
            build()
        if not so.exists():
            raise RuntimeError(f"{so} is absent and the reference sources are not here")
        lib = C.CDLL(str(so))
        if hasattr(lib, "href_cuda_init"):
            lib.href_cuda_init.restype = _i
            lib.href_cuda_init.argtypes = [_vp]
            lib.href_cuda_forward.restype = _i
            lib.href_cuda_forward.argtypes = [_vp, _i]
            lib.href_cuda_reset.argtypes = [_vp]
            lib.href_cuda_cleanup.argtypes = []
        lib.matmul_q.argtypes = [_vp, _vp, _vp, _i, _i, _i]
        lib.href_matmul_q_threads.argtypes = [_vp, _vp, _vp, _i, _i, _i, _i]
        for name in ("dequantize_row_q8_0", "dequantize_row_q4_0", "dequantize_row_q4_k", "dequantize_row_q6_k"):
            getattr(lib, name).argtypes = [_vp, _vp, _i]
        lib.href_gguf_tensor.restype = C.c_longlong
        lib.href_gguf_tensor.argtypes = [C.c_char_p, C.c_char_p, _vp, C.c_longlong, C.POINTER(C.c_int)]
        lib.href_gguf_int.restype = C.c_longlong
        lib.href_gguf_int.argtypes = [C.c_char_p, C.c_char_p, C.c_longlong]
        lib.href_gguf_float.restype = C.c_double
        lib.href_gguf_float.argtypes = [C.c_char_p, C.c_char_p, C.c_double]
        lib.href_tokenize.restype = _i
        lib.href_tokenize.argtypes = [C.POINTER(C.c_char_p), _i, _i, _i, C.c_char_p, C.POINTER(_i), _i, _i]
        lib.href_gguf_string_at.restype = C.c_longlong
        lib.href_gguf_string_at.argtypes = [C.c_char_p, C.c_char_p, C.c_longlong, C.c_char_p, C.c_longlong]
        lib.href_gguf_array_len.restype = C.c_longlong
        lib.href_gguf_array_len.argtypes = [C.c_char_p, C.c_char_p]
        lib.f16_to_f32.restype = _f
        lib.f16_to_f32.argtypes = [C.c_uint16]
        lib.href_model_create.restype = _vp
        lib.href_model_create.argtypes = [_i, _i, _i, _i, _i, _i, _i, _i, _f, _f]
        lib.href_model_set_types.argtypes = [_vp, _i, _i, _i]
        lib.href_model_set_types_mixed.argtypes = [_vp, _i, _i, _i, _i, _i]
        lib.href_model_set_layer_types.argtypes = [_vp, _i, _i, _i]
        lib.href_model_set_layer.argtypes = [_vp, _i] + [_vp] * 9
        lib.href_model_set_globals.argtypes = [_vp, _vp, _vp, _vp]
        lib.href_forward.restype = _i
        lib.href_forward.argtypes = [_vp, _i]
        lib.href_logits.restype = C.POINTER(C.c_float)
        lib.href_logits.argtypes = [_vp]
        lib.href_reset.argtypes = [_vp]
        lib.href_push_token.argtypes = [_vp, _i]
        lib.href_sample.restype = _i
        lib.href_sample.argtypes = [_vp, _f, _f, _i, _f, _i]
        lib.href_model_free.argtypes = [_vp]
        lib.rope_apply.argtypes = [_vp, _vp, _i, _i, _i, _f]
        self.lib = lib

    def rope(self, v, pos, head_dim, n_heads, base):
        """src/ai/tensor.c:347-373 applied to one tensor of n_heads heads."""
        a = np.ascontiguousarray(v, np.float32).copy()
        b = np.zeros_like(a)
        self.lib.rope_apply(_ptr(a), _ptr(b), pos, head_dim, n_heads, base)
        return a

    def matmul_q(self, gtype, blocks, x, rows, cols, threads=1):
        blocks = np.ascontiguousarray(blocks)
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(rows, np.float32)
        self.lib.href_matmul_q_threads(_ptr(y), _ptr(blocks), _ptr(x), rows, cols, gtype, threads)
        return y

    def gguf_tensor(self, path, name, cap):
        """The bytes the reference's loader reads for tensor `name` of a GGUF
        file (its own parser), and their ggml type."""
        buf = np.zeros(cap, np.uint8)
        t = C.c_int(0)
        n = self.lib.href_gguf_tensor(str(path).encode(), name.encode(), _ptr(buf), cap, C.byref(t))
        if n < 0:
            raise RuntimeError(f"reference gguf parser: {n} for {name}")
        return buf[:n], t.value

    def gguf_int(self, path, key, default=-1):
        return self.lib.href_gguf_int(str(path).encode(), key.encode(), default)

    def gguf_float(self, path, key, default=-1.0):
        return self.lib.href_gguf_float(str(path).encode(), key.encode(), default)

    def tokenize(self, vocab, bos, unk, text, max_tokens=None, add_bos=False):
        """The reference's own llm_tokenize (src/ai/llm.c:178-221)."""
        return _tok_call(self.lib.href_tokenize, vocab, bos, unk, text, max_tokens, add_bos)

    def gguf_tokens(self, path, key="tokenizer.ggml.tokens", cap=1 << 16):
        """A GGUF string array as load_tokenizer copies it (llm.c:78-81)."""
        n = self.lib.href_gguf_array_len(str(path).encode(), key.encode())
        buf = C.create_string_buffer(cap)
        out = []
        for i in range(n):
            r = self.lib.href_gguf_string_at(str(path).encode(), key.encode(), i, buf, cap)
            if r < 0:
                raise RuntimeError(f"href_gguf_string_at({key}, {i}) = {r}")
            out.append(buf.raw[:r])
        return out

    def dequant(self, gtype, blocks, rows, cols):
        name = {8: "dequantize_row_q8_0", 2: "dequantize_row_q4_0", 12: "dequantize_row_q4_k",
                14: "dequantize_row_q6_k"}[gtype]
        blocks = np.ascontiguousarray(blocks)
        out = np.empty((rows, cols), np.float32)
        getattr(self.lib, name)(_ptr(blocks), _ptr(out), rows * cols)
        return out


class RefModel:
    """A model in the reference engine's own structs (oracle/ref_harness.c),
    run by its llm_forward (src/ai/llm.c:1015) and llm_sample (llm.c:1281).
    `w` holds the host arrays of holo_b200.synth.llama_weights; they are kept
    alive here because the reference reads them in place."""

    def __init__(self, ref: Reference, cfg: dict, w: dict):
        self.lib = ref.lib
        self.cfg = cfg
        self.w = w
        self.h = self.lib.href_model_create(cfg["n_layers"], cfg["dim"], cfg["n_heads"], cfg["n_kv_heads"],
                                            cfg["head_dim"], cfg["ffn_dim"], cfg["vocab"], cfg["max_seq"],
                                            cfg.get("rope_base", 10000.0), cfg.get("eps", 1e-5))
        lt = cfg["layer_type"]
        self.lib.href_model_set_types_mixed(self.h, lt, cfg.get("wv_type", lt), cfg.get("w2_type", lt),
                                            cfg.get("emb_type", 1), cfg["out_type"])
        for l, (tv, t2) in enumerate(layer_types(cfg)):
            self.lib.href_model_set_layer_types(self.h, l, tv, t2)
        for l, L in enumerate(w["layers"]):
            self.lib.href_model_set_layer(self.h, l, _ptr(L["attn_norm"]), _ptr(L["wq"]), _ptr(L["wk"]),
                                          _ptr(L["wv"]), _ptr(L["wo"]), _ptr(L["ffn_norm"]), _ptr(L["w1"]),
                                          _ptr(L["w2"]), _ptr(L["w3"]))
        self.lib.href_model_set_globals(self.h, _ptr(w["tok_emb"]), _ptr(w["final_norm"]), _ptr(w["output"]))
        self.libc = C.CDLL(None)
        self.libc.rand.restype = _i

    def forward(self, token: int) -> np.ndarray:
        assert self.lib.href_forward(self.h, int(token)) == 0
        return np.ctypeslib.as_array(self.lib.href_logits(self.h), shape=(self.cfg["vocab"],)).copy()

    def set_logits(self, logits: np.ndarray):
        dst = np.ctypeslib.as_array(self.lib.href_logits(self.h), shape=(self.cfg["vocab"],))
        dst[:] = np.asarray(logits, np.float32)

    def push(self, token: int):
        self.lib.href_push_token(self.h, int(token))

    def sample(self, temperature, top_p, top_k, penalty, last_n) -> int:
        return self.lib.href_sample(self.h, temperature, top_p, top_k, penalty, last_n)

    def srand(self, seed: int):
        self.libc.srand(C.c_uint(seed))

    def rand_r(self) -> float:
        """(float)rand() / RAND_MAX, as llm_sample draws it (llm.c:1320)."""
        return float(np.float32(np.float32(self.libc.rand()) / np.float32(2147483647)))

    def reset(self):
        self.lib.href_reset(self.h)

    def generate(self, prompt, n_new, temperature, top_p, top_k, penalty, last_n, seed, margins=None):
        """llm_generate's loop (llm.c:1340-1420) without tokenizer or EOS.
        margins (a list) collects the top-1 minus top-2 logit before each draw."""
        self.srand(seed)
        self.reset()
        for t in prompt:
            self.push(t)
        for t in prompt:
            logits = self.forward(t)
        out = []
        for _ in range(n_new):
            if margins is not None:
                top2 = np.sort(logits)[-2:]
                margins.append(float(top2[1] - top2[0]))
            tok = self.sample(temperature, top_p, top_k, penalty, last_n)
            out.append(tok)
            self.push(tok)
            logits = self.forward(tok)
        return np.array(out, np.int32)

    def close(self):
        if self.h:
            self.lib.href_model_free(self.h)
            self.h = None
