"""GGUF files for the decode engine: read a Llama-architecture model file into
the host arrays that Model.set_weights takes, and write such files.

The format is the one the reference's loader reads (src/ai/gguf.c:280-395:
header, key/value metadata, tensor infos, then the tensor data) with one
difference: the data section starts at the next multiple of the file's
general.alignment (32 when the key is absent), where gguf.c:354-356 always
rounds to 32 -- so files written with a larger alignment load correctly
here.  Tensors are read in place from a memory map; nothing is converted,
the GGUF blocks go to cuda_upload_quant as they are.

Tensor names and the metadata keys of the configuration follow the
reference's load_weights (src/ai/llm.c:344-528) and gguf_open
(gguf.c:357-393): token_embd / output_norm / output, blk.N.{attn_norm,
attn_q, attn_k, attn_v, attn_output, ffn_norm, ffn_gate (W1), ffn_down (W2),
ffn_up (W3)}.weight; {arch}.block_count, .embedding_length,
.attention.head_count(_kv), .attention.key_length, .feed_forward_length,
.rope.freq_base, .attention.layer_norm_rms_epsilon, .context_length.
"""
from __future__ import annotations

import mmap
import struct

import numpy as np

from . import BLOCK_BYTES, BLOCK_ELEMS, F16, F32

MAGIC = 0x46554747          # "GGUF", little-endian
DEFAULT_ALIGNMENT = 32

# metadata value types (src/ai/gguf.h:23-37)
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)
_SCALAR = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f",
           T_BOOL: "<?", T_U64: "<Q", T_I64: "<q", T_F64: "<d"}

LAYER_TENSORS = {"attn_norm": "attn_norm", "wq": "attn_q", "wk": "attn_k", "wv": "attn_v", "wo": "attn_output",
                 "ffn_norm": "ffn_norm", "w1": "ffn_gate", "w2": "ffn_down", "w3": "ffn_up"}


def tensor_nbytes(gtype: int, dims) -> int:
    n = 1
    for d in dims:
        n *= int(d)
    return n // BLOCK_ELEMS[gtype] * BLOCK_BYTES[gtype]


class GGUFFile:
    """A GGUF file, memory-mapped: .meta (key -> value), .tensors (name ->
    (dims, type, offset into the data section)), .alignment, .data_offset."""

    def __init__(self, path):
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self._pos = 0
        magic, version = self._unpack("<II")
        if magic != MAGIC:
            raise ValueError(f"{path}: not a GGUF file")
        if version not in (2, 3):
            raise ValueError(f"{path}: GGUF version {version} (2 and 3 are read)")
        n_tensors, n_kv = self._unpack("<QQ")
        self.version = version
        self.meta = {}
        self._value_at = {}   # key -> (type, file offset of the value)
        for _ in range(n_kv):
            key = self._string()
            (vtype,) = self._unpack("<I")
            self._value_at[key] = (vtype, self._pos)
            self.meta[key] = self._value(vtype)
        self.tensors = {}
        for _ in range(n_tensors):
            name = self._string()
            (nd,) = self._unpack("<I")
            dims = self._unpack(f"<{nd}Q")
            gtype, offset = self._unpack("<IQ")
            self.tensors[name] = (tuple(int(d) for d in dims), int(gtype), int(offset))
        self.alignment = int(self.meta.get("general.alignment", DEFAULT_ALIGNMENT))
        if self.alignment <= 0 or self.alignment & (self.alignment - 1):
            raise ValueError(f"{path}: general.alignment {self.alignment} is not a power of two")
        self.data_offset = (self._pos + self.alignment - 1) // self.alignment * self.alignment

    # ---- parsing ----
    def _unpack(self, fmt):
        size = struct.calcsize(fmt)
        if self._pos + size > len(self._mm):
            raise ValueError("GGUF file truncated")
        v = struct.unpack_from(fmt, self._mm, self._pos)
        self._pos += size
        return v

    def _string(self, raw=False):
        (n,) = self._unpack("<Q")
        if self._pos + n > len(self._mm):
            raise ValueError("GGUF file truncated")
        b = bytes(self._mm[self._pos:self._pos + n])
        self._pos += n
        return b if raw else b.decode("utf-8", errors="replace")

    def string_array(self, key) -> list[bytes] | None:
        """A metadata array of strings as raw bytes (.meta holds them
        decoded), or None when the key is absent or not such an array."""
        if key not in self._value_at:
            return None
        vtype, pos = self._value_at[key]
        if vtype != T_ARR:
            return None
        saved, self._pos = self._pos, pos
        try:
            etype, n = self._unpack("<IQ")
            return [self._string(raw=True) for _ in range(n)] if etype == T_STR else None
        finally:
            self._pos = saved

    def _value(self, vtype):
        if vtype == T_STR:
            return self._string()
        if vtype == T_ARR:
            etype, n = self._unpack("<IQ")
            return [self._value(etype) for _ in range(n)]
        if vtype not in _SCALAR:
            raise ValueError(f"GGUF metadata type {vtype}")
        return self._unpack(_SCALAR[vtype])[0]

    # ---- access ----
    def tensor(self, name) -> np.ndarray:
        """The tensor's bytes (uint8, read-only view of the map); F32 tensors
        as float32 and F16 as float16 arrays [rows][cols]."""
        dims, gtype, off = self.tensors[name]
        nbytes = tensor_nbytes(gtype, dims)
        start = self.data_offset + off
        if start + nbytes > len(self._mm):
            raise ValueError(f"tensor {name} runs past the end of the file")
        raw = np.frombuffer(self._mm, np.uint8, count=nbytes, offset=start)
        if gtype == F32:
            return raw.view(np.float32).reshape(tuple(reversed(dims)))
        if gtype == F16:
            return raw.view(np.float16).reshape(tuple(reversed(dims)))
        return raw

    def close(self):
        """Closes the file; the map itself stays until the last array that
        views it (from tensor()) is gone."""
        try:
            self._mm.close()
        except BufferError:
            pass
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def model_config(g: GGUFFile, max_seq: int | None = None) -> dict:
    """Model configuration (holo_b200.model.ModelDesc keys) from the metadata
    and tensor types.  attn_q / attn_k / attn_output / ffn_gate / ffn_up share
    one type (layer_type, the reference's g_weight_type); attn_v and ffn_down
    may differ per layer (wv_types / w2_types, as Q4_K_M files keep some of
    them in Q6_K; the reference binds them per layer, llm.c:445-507)."""
    arch = g.meta.get("general.architecture", "llama")

    def key(k, default):
        return g.meta.get(f"{arch}.{k}", default)

    dim = int(key("embedding_length", 4096))
    nh = int(key("attention.head_count", 32))
    emb_dims, emb_type, _ = g.tensors["token_embd.weight"]
    n_layers = int(key("block_count", 32))
    layer_types = {g.tensors[f"blk.{l}.{n}.weight"][1] for l in range(n_layers)
                   for n in ("attn_q", "attn_k", "attn_output", "ffn_gate", "ffn_up")}
    if len(layer_types) != 1:
        raise ValueError(f"attn_q/attn_k/attn_output/ffn_gate/ffn_up of several types {sorted(layer_types)}: "
                         "the engine (as the reference) takes one type for these")
    wv_types = [g.tensors[f"blk.{l}.attn_v.weight"][1] for l in range(n_layers)]
    w2_types = [g.tensors[f"blk.{l}.ffn_down.weight"][1] for l in range(n_layers)]
    out_name = "output.weight" if "output.weight" in g.tensors else "token_embd.weight"
    ctx = int(key("context_length", 4096))
    lt = layer_types.pop()
    cfg = dict(n_layers=n_layers, dim=dim, n_heads=nh,
               n_kv_heads=int(key("attention.head_count_kv", nh)),
               head_dim=int(key("attention.key_length", dim // nh)), ffn_dim=int(key("feed_forward_length", 11008)),
               vocab=int(emb_dims[1]), max_seq=min(ctx, max_seq) if max_seq else ctx,
               rope_base=float(key("rope.freq_base", 10000.0)),
               eps=float(key("attention.layer_norm_rms_epsilon", 1e-5)), layer_type=lt,
               emb_type=emb_type, out_type=g.tensors[out_name][1])
    if any(t != lt for t in wv_types + w2_types):   # per-layer types only where the file mixes them
        cfg.update(wv_types=wv_types, w2_types=w2_types)
    return cfg


def model_weights(g: GGUFFile, cfg: dict) -> dict:
    """The host arrays of Model.set_weights, views of the file where possible
    (an absent output matrix is the token embedding: tied weights)."""
    layers = []
    for l in range(cfg["n_layers"]):
        layers.append({k: np.ascontiguousarray(g.tensor(f"blk.{l}.{n}.weight")).reshape(-1)
                       if k not in ("attn_norm", "ffn_norm") else np.ascontiguousarray(g.tensor(f"blk.{l}.{n}.weight"),
                                                                                       np.float32)
                       for k, n in LAYER_TENSORS.items()})
    out = "output.weight" if "output.weight" in g.tensors else "token_embd.weight"
    output = np.ascontiguousarray(g.tensor(out))
    return {"layers": layers, "tok_emb": np.ascontiguousarray(g.tensor("token_embd.weight")),
            "final_norm": np.ascontiguousarray(g.tensor("output_norm.weight"), np.float32),
            "output": output.reshape(-1) if output.dtype == np.uint8 else output}


def tokenizer_vocab(g: GGUFFile) -> dict:
    """The tokenizer fields the reference's load_tokenizer reads
    (src/ai/llm.c:61-100): the token strings of tokenizer.ggml.tokens as
    bytes, each cut at its first NUL as strdup does, and the special ids with
    the reference's defaults (bos 1, eos 2, padding 0, unknown 0)."""
    toks = g.string_array("tokenizer.ggml.tokens")
    if not toks:
        raise ValueError("no vocabulary (tokenizer.ggml.tokens) in the file")
    ids = {k: int(g.meta.get(f"tokenizer.ggml.{key}", d)) for k, key, d in
           (("bos", "bos_token_id", 1), ("eos", "eos_token_id", 2), ("pad", "padding_token_id", 0),
            ("unk", "unknown_token_id", 0))}
    return dict(tokens=[t.split(b"\0", 1)[0] for t in toks], **ids)


def load_tokenizer(g: GGUFFile):
    """A holo_b200.Tokenizer over the file's vocabulary (llm_tokenize's)."""
    from . import Tokenizer
    v = tokenizer_vocab(g)
    return Tokenizer(v["tokens"], bos=v["bos"], unk=v["unk"])


def load_model(path, max_seq: int | None = None, rope_mode: int = 0, **model_kw):
    """A decode Model with the weights of a GGUF file (uploaded and repacked
    once); model_kw go to Model (act_mode, kv_f16, world, rank, batch).
    rope_mode 0 rotates pairs (i, i + hd/2) as the reference does; files
    converted by llama.cpp's tools expect 1, pairs (2i, 2i+1)
    (holo_model_desc.rope_mode)."""
    from .model import Model
    with GGUFFile(path) as g:
        cfg = model_config(g, max_seq)
        cfg["rope_mode"] = rope_mode
        m = Model(cfg, **model_kw)
        m.set_weights(model_weights(g, cfg))
    return m


# ---------------------------------------------------------------------------
# writing
# ---------------------------------------------------------------------------
def _pack_value(v):
    if isinstance(v, bool):
        return struct.pack("<I?", T_BOOL, v)
    if isinstance(v, int):
        return struct.pack("<Iq", T_I64, v) if v < 0 else struct.pack("<IQ", T_U64, v) if v >= 2 ** 32 \
            else struct.pack("<II", T_U32, v)
    if isinstance(v, float):
        return struct.pack("<If", T_F32, v)
    if isinstance(v, (str, bytes)):
        b = v.encode() if isinstance(v, str) else v
        return struct.pack("<IQ", T_STR, len(b)) + b
    if isinstance(v, (list, tuple)):
        # arrays: of strings, of float32 or of int32 (the tokenizer.ggml.* kinds)
        if all(isinstance(e, (str, bytes)) for e in v):
            return struct.pack("<IIQ", T_ARR, T_STR, len(v)) + b"".join(_pack_value(e)[4:] for e in v)
        if all(isinstance(e, float) for e in v):
            return struct.pack("<IIQ", T_ARR, T_F32, len(v)) + np.asarray(v, "<f4").tobytes()
        if all(isinstance(e, int) and not isinstance(e, bool) for e in v):
            return struct.pack("<IIQ", T_ARR, T_I32, len(v)) + np.asarray(v, "<i4").tobytes()
    raise TypeError(f"metadata value {v!r}")


def write(path, meta: dict, tensors: dict, alignment: int = DEFAULT_ALIGNMENT):
    """Write a GGUF v3 file: meta (str -> int/float/str/bool), tensors (name ->
    (gguf type, dims (cols first), bytes-like data)).  general.alignment is
    stored when it differs from 32; every tensor starts on a multiple of it."""
    meta = dict(meta)
    if alignment != DEFAULT_ALIGNMENT:
        meta["general.alignment"] = int(alignment)
    head = struct.pack("<IIQQ", MAGIC, 3, len(tensors), len(meta))
    for k, v in meta.items():
        kb = k.encode()
        head += struct.pack("<Q", len(kb)) + kb + _pack_value(v)
    offset, blobs = 0, []
    for name, (gtype, dims, data) in tensors.items():
        data = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        if data.nbytes != tensor_nbytes(gtype, dims):
            raise ValueError(f"{name}: {data.nbytes} bytes for dims {dims} of type {gtype}")
        nb = name.encode()
        head += struct.pack("<Q", len(nb)) + nb + struct.pack(f"<I{len(dims)}QIQ", len(dims), *dims, gtype, offset)
        blobs.append((offset, data))
        offset = (offset + data.nbytes + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * (-len(head) % alignment))
        base = f.tell()
        for off, data in blobs:
            f.write(b"\0" * (base + off - f.tell()))
            f.write(data.tobytes())


def write_model(path, cfg: dict, w: dict, alignment: int = DEFAULT_ALIGNMENT, arch: str = "llama"):
    """A model of shape cfg with the host arrays w (synth.llama_weights) as a
    GGUF file of the reference's tensor names and metadata keys."""
    dim, hd, nh, nkv, ffn, V = (cfg[k] for k in ("dim", "head_dim", "n_heads", "n_kv_heads", "ffn_dim", "vocab"))
    lt, ot = cfg["layer_type"], cfg["out_type"]
    meta = {"general.architecture": arch, f"{arch}.block_count": cfg["n_layers"],
            f"{arch}.embedding_length": dim, f"{arch}.attention.head_count": nh,
            f"{arch}.attention.head_count_kv": nkv, f"{arch}.attention.key_length": hd,
            f"{arch}.feed_forward_length": ffn, f"{arch}.context_length": cfg["max_seq"],
            f"{arch}.rope.freq_base": float(cfg["rope_base"]),
            f"{arch}.attention.layer_norm_rms_epsilon": float(cfg["eps"]), f"{arch}.vocab_size": V}
    emb_t = F16 if w["tok_emb"].dtype == np.float16 else F32 if w["tok_emb"].dtype == np.float32 \
        else cfg["emb_type"]   # GGUF blocks (uint8)
    t = {"token_embd.weight": (emb_t, (dim, V), w["tok_emb"]),
         "output_norm.weight": (F32, (dim,), w["final_norm"]),
         "output.weight": (ot, (dim, V), w["output"])}
    shapes = {"wq": (dim, nh * hd), "wk": (dim, nkv * hd), "wv": (dim, nkv * hd), "wo": (nh * hd, dim),
              "w1": (dim, ffn), "w2": (ffn, dim), "w3": (dim, ffn)}
    from .model import layer_types
    for l, (L, (tv, t2)) in enumerate(zip(w["layers"], layer_types(cfg))):
        for k, n in LAYER_TENSORS.items():
            if k in ("attn_norm", "ffn_norm"):
                t[f"blk.{l}.{n}.weight"] = (F32, (dim,), L[k])
            else:
                t[f"blk.{l}.{n}.weight"] = ({"wv": tv, "w2": t2}.get(k, lt), shapes[k], L[k])
    write(path, meta, t, alignment)
