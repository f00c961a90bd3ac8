"""Python owner of the decode engine (include/holo_b200.h, holo_model_*).

Mirrors the reference's llm_forward / llm_sample / llm_generate
(src/ai/llm.c:1015, 1281, 1335) on a model object whose weights live on the
device; the arithmetic is the library's (csrc/decode.cu).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import load, ACT_Q8, HOLO_OK, COMM_HANDLE_BYTES


def layer_types(cfg: dict):
    """(wv type, w2 type) of every layer: cfg's per-layer lists wv_types /
    w2_types, else wv_type / w2_type, else layer_type (the reference binds
    these two per layer, src/ai/llm.c:445-507)."""
    lt, n = cfg["layer_type"], cfg["n_layers"]
    wv = cfg.get("wv_types") or [cfg.get("wv_type", lt)] * n
    w2 = cfg.get("w2_types") or [cfg.get("w2_type", lt)] * n
    return list(zip(wv, w2))


class ModelDesc(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("dim", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("ffn_dim", C.c_int), ("vocab", C.c_int), ("max_seq", C.c_int),
                ("rope_base", C.c_float), ("eps", C.c_float), ("layer_type", C.c_int), ("emb_type", C.c_int),
                ("out_type", C.c_int), ("kv_f16", C.c_int), ("act_mode", C.c_int), ("world", C.c_int),
                ("rank", C.c_int), ("batch", C.c_int), ("rope_mode", C.c_int)]


class SamplerDesc(C.Structure):
    """llm_sampler_t (src/ai/llm.h:167-174) without the seed."""
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int),
                ("repeat_penalty", C.c_float), ("repeat_last_n", C.c_int)]


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class Model:
    """One decode model on the current device (raises on library errors).

    world > 1: this process's row shard of a model sharded over `world` GPUs
    (one process per GPU); set the weights (the full matrices: each rank keeps
    its rows), then connect_peers, then make every step call on every rank."""

    def __init__(self, cfg: dict, act_mode: int = ACT_Q8, kv_f16: bool = True, world: int = 1, rank: int = 0,
                 batch: int = 1):
        self.lib = load()
        self.cfg = dict(cfg)
        self.world, self.rank, self.batch = world, rank, batch
        d = ModelDesc(cfg["n_layers"], cfg["dim"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"],
                      cfg["ffn_dim"], cfg["vocab"], cfg["max_seq"], cfg.get("rope_base", 10000.0),
                      cfg.get("eps", 1e-5), cfg["layer_type"], cfg.get("emb_type", 1), cfg["out_type"],
                      int(kv_f16), act_mode, world, rank, batch, cfg.get("rope_mode", 0))
        self.desc = d
        self.h = self.lib.holo_model_create(C.byref(d))
        self._check("holo_model_create", ok=bool(self.h))

    def _check(self, what: str, ok: bool = True):
        st = self.lib.cuda_last_status()
        if st != HOLO_OK or not ok:
            msg = self.lib.cuda_last_status_string().decode(errors="replace")
            self.lib.cuda_clear_status()
            raise RuntimeError(f"{what}: status {st} ({msg})")

    def set_layer_types(self, layer: int, wv_type: int, w2_type: int):
        """GGUF types of one layer's wv and w2 (holo_model_set_layer_types),
        before that layer's weights are set."""
        rc = self.lib.holo_model_set_layer_types(self.h, int(layer), int(wv_type), int(w2_type))
        self._check(f"holo_model_set_layer_types {layer}", rc == HOLO_OK)

    def set_weights(self, w: dict):
        """w: the host arrays of synth.llama_weights (GGUF blocks, fp32 norms).
        Per-layer wv / w2 types come from the config (layer_types)."""
        lt = self.cfg["layer_type"]
        for l, (tv, t2) in enumerate(layer_types(self.cfg)):
            if tv != lt or t2 != lt:
                self.set_layer_types(l, tv, t2)
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

    def prefill(self, tokens, want_logits: bool = True) -> np.ndarray | None:
        """Prompt pass over tokens ([batch][n] for a batched model) at the next
        positions (row passes on the tensor cores); each sequence's last
        position's logits."""
        tokens = np.ascontiguousarray(tokens, np.int32)
        shape = (self.batch, self.cfg["vocab"]) if self.batch > 1 else (self.cfg["vocab"],)
        out = np.empty(shape, np.float32) if want_logits else None
        rc = self.lib.holo_model_prefill(self.h, _ptr(tokens), tokens.shape[-1], _ptr(out) if want_logits else None)
        self._check("holo_model_prefill", rc == HOLO_OK)
        return out

    def set_prompt_mode(self, rows: bool):
        """generate's prompt: row passes (True, the default) or one position a step."""
        self._check("holo_model_set_prompt_mode", self.lib.holo_model_set_prompt_mode(self.h, int(bool(rows))) == HOLO_OK)

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

    def forward_batch(self, tokens, want_logits: bool = True) -> np.ndarray | None:
        """One position of every sequence of a batched model: logits [batch][vocab]."""
        tokens = np.ascontiguousarray(tokens, np.int32)
        out = np.empty((self.batch, self.cfg["vocab"]), np.float32) if want_logits else None
        rc = self.lib.holo_model_forward_batch(self.h, _ptr(tokens), _ptr(out) if want_logits else None)
        self._check("holo_model_forward_batch", rc == HOLO_OK)
        return out

    def generate_batch(self, prompts, n_new: int, s: SamplerDesc, seeds) -> np.ndarray:
        """llm_generate for every sequence: prompts [batch][n_prompt], seeds [batch]."""
        prompts = np.ascontiguousarray(prompts, np.int32)
        seeds = np.ascontiguousarray(seeds, np.int32)
        out = np.zeros((self.batch, n_new), np.int32)
        n = self.lib.holo_model_generate_batch(self.h, _ptr(prompts), prompts.shape[1], n_new, C.byref(s),
                                               _ptr(seeds), _ptr(out))
        self._check("holo_model_generate_batch", n == n_new)
        return out

    def last_timing(self) -> tuple[float, float]:
        """(prefill_ms, decode_ms) of the last generate, device time."""
        a, b = C.c_float(), C.c_float()
        self.lib.holo_model_last_timing(self.h, C.byref(a), C.byref(b))
        return a.value, b.value

    def comm_handle(self) -> bytes:
        """This rank's handle for the other ranks (HOLO_COMM_HANDLE_BYTES)."""
        buf = C.create_string_buffer(COMM_HANDLE_BYTES)
        self._check("holo_model_comm_handle", self.lib.holo_model_comm_handle(self.h, buf) == HOLO_OK)
        return buf.raw

    def open_peers(self, handles: list[bytes]):
        """Every rank's handle, in rank order."""
        if len(handles) != self.world or any(len(h) != COMM_HANDLE_BYTES for h in handles):
            raise ValueError("open_peers: one handle of COMM_HANDLE_BYTES per rank")
        blob = C.create_string_buffer(b"".join(handles), COMM_HANDLE_BYTES * self.world)
        self._check("holo_model_open_peers", self.lib.holo_model_open_peers(self.h, blob) == HOLO_OK)

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


def connect_peers(model, group=None):
    """All-gather of the ranks' comm handles over torch.distributed (any
    backend), then open them: the set-up collective of a sharded model."""
    import torch.distributed as dist
    handles = [None] * model.world
    dist.all_gather_object(handles, model.comm_handle(), group=group)
    model.open_peers(handles)


def shard_ranges(cfg: dict, world: int, rank: int) -> dict:
    """The rows a rank of a sharded model holds (holo_model_shard, host
    only): query heads, KV heads, rows of Wo/W2, SwiGLU outputs (whole 16-row
    bands), output-matrix rows, each (first, count)."""
    lib = load()
    d = ModelDesc(cfg["n_layers"], cfg["dim"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"],
                  cfg["ffn_dim"], cfg["vocab"], cfg["max_seq"], cfg.get("rope_base", 10000.0),
                  cfg.get("eps", 1e-5), cfg["layer_type"], cfg.get("emb_type", 1), cfg["out_type"], 1, ACT_Q8,
                  world, rank, 1, cfg.get("rope_mode", 0))
    r = (C.c_int * 10)()
    if lib.holo_model_shard(C.byref(d), r) != HOLO_OK:
        lib.cuda_clear_status()
        raise ValueError(f"shard_ranges: cannot shard over {world} (rank {rank})")
    names = ("heads", "kv_heads", "dim", "ffn", "vocab")
    return {n: (r[2 * i], r[2 * i + 1]) for i, n in enumerate(names)}


LLAMA2_7B = dict(n_layers=32, dim=4096, n_heads=32, n_kv_heads=32, head_dim=128, ffn_dim=11008, vocab=32000,
                 max_seq=2048, rope_base=10000.0, eps=1e-5, layer_type=12, emb_type=1, out_type=8)
LLAMA3_70B = dict(n_layers=80, dim=8192, n_heads=64, n_kv_heads=8, head_dim=128, ffn_dim=28672, vocab=128256,
                  max_seq=4096, rope_base=500000.0, eps=1e-5, layer_type=2, emb_type=1, out_type=2)


def _tensor_seed(seed: int, layer: int, idx: int) -> int:
    return (seed * 1000003 + layer * 64 + idx) & 0xFFFFFFFFFFFFFFFF


def synthetic_model(cfg: dict, seed: int, act_mode: int = ACT_Q8, kv_f16: bool = True, std: float = 0.02,
                    keep_host: bool = False, world: int = 1, rank: int = 0, batch: int = 1):
    """A random-init model built on the device: every weight N(0, std),
    quantized round-to-nearest by cuda_synth_weights into GGUF blocks, then
    repacked by holo_model_set_layer/_globals.  keep_host also returns the raw
    blocks (the dict layout of synth.llama_weights) for the reference engine."""
    lib = load()
    m = Model(cfg, act_mode=act_mode, kv_f16=kv_f16, world=world, rank=rank, batch=batch)
    dim, hd, ffn, V = cfg["dim"], cfg["head_dim"], cfg["ffn_dim"], cfg["vocab"]
    q_dim, kv_dim = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd
    lt, ot, et = cfg["layer_type"], cfg["out_type"], cfg.get("emb_type", 1)
    from . import row_bytes
    shapes = {"wq": (q_dim, dim), "wk": (kv_dim, dim), "wv": (kv_dim, dim), "wo": (dim, q_dim),
              "w1": (ffn, dim), "w2": (dim, ffn), "w3": (ffn, dim)}
    ones = np.ones(dim, np.float32)
    host = {"layers": []} if keep_host else None

    def gen(t, rows, cols, s):
        nbytes = rows * (row_bytes(t, cols) if t not in (0, 1) else cols * (4 if t == 0 else 2))
        p = lib.cuda_malloc(nbytes)
        if not p:
            raise MemoryError("synthetic_model: cuda_malloc")
        rc = lib.cuda_synth_weights(p, t, rows, cols, s, std)
        m._check("cuda_synth_weights", rc == HOLO_OK)
        return p, nbytes

    def to_host(p, nbytes, dtype=np.uint8):
        a = np.empty(nbytes // np.dtype(dtype).itemsize, dtype)
        lib.cuda_memcpy_d2h(a.ctypes.data, p, a.nbytes)
        return a

    for l in range(cfg["n_layers"]):
        ptrs = {}
        for i, (name, (r, c)) in enumerate(shapes.items()):
            ptrs[name] = gen(lt, r, c, _tensor_seed(seed, l, i))
        rc = lib.holo_model_set_layer(m.h, l, ones.ctypes.data, ptrs["wq"][0], ptrs["wk"][0], ptrs["wv"][0],
                                      ptrs["wo"][0], ones.ctypes.data, ptrs["w1"][0], ptrs["w2"][0], ptrs["w3"][0])
        m._check(f"holo_model_set_layer {l}", rc == HOLO_OK)
        if keep_host:
            L = {k: to_host(*v) for k, v in ptrs.items()}
            L["attn_norm"], L["ffn_norm"] = ones.copy(), ones.copy()
            host["layers"].append(L)
        for p, _ in ptrs.values():
            lib.cuda_free(p)
    emb = gen(et, V, dim, _tensor_seed(seed, 1 << 20, 0))
    out = gen(ot, V, dim, _tensor_seed(seed, 1 << 20, 1))
    rc = lib.holo_model_set_globals(m.h, emb[0], ones.ctypes.data, out[0])
    m._check("holo_model_set_globals", rc == HOLO_OK)
    if keep_host:
        host["tok_emb"] = to_host(*emb, dtype=np.float16 if et == 1 else np.float32).reshape(V, dim)
        host["final_norm"] = ones.copy()
        host["output"] = to_host(*out)
    lib.cuda_free(emb[0])
    lib.cuda_free(out[0])
    return (m, host) if keep_host else m
