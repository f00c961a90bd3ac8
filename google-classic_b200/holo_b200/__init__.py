"""Python host mirror of the B200 decode-path library.

Loads ``lib/libholo_cuda.so`` (built by ``google-classic_b200/Makefile``) with
ctypes and declares the C signatures of ``include/cuda_ops.h`` (the reference
engine's op ABI, kept name for name) and ``include/holo_b200.h`` (additive
entry points).  Nothing here computes: every numeric call goes through the
shared library, and a missing library raises instead of falling back.
"""
from __future__ import annotations

import ctypes as C
import os
import pathlib

import numpy as np

PKG_DIR = pathlib.Path(__file__).resolve().parent.parent
REPO_ROOT = PKG_DIR.parent
LIB_PATH = PKG_DIR / "lib" / "libholo_cuda.so"
INCLUDE_DIR = REPO_ROOT / "include"

# ggml type ids (src/ai/quant.h:20-33 of the reference)
F32, F16, Q4_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 8, 12, 14
TYPE_NAMES = {F32: "f32", F16: "f16", Q4_0: "q4_0", Q8_0: "q8_0", Q4_K: "q4_k", Q6_K: "q6_k"}
BLOCK_ELEMS = {Q8_0: 32, Q4_0: 32, Q4_K: 256, Q6_K: 256, F16: 1, F32: 1}
BLOCK_BYTES = {Q8_0: 34, Q4_0: 18, Q4_K: 144, Q6_K: 210, F16: 2, F32: 4}

ACT_F32, ACT_Q8 = 0, 1
Q4K_REF, Q4K_GGML = 0, 1
ROPE_HALF, ROPE_ADJACENT = 0, 1          # holo_model_desc.rope_mode

HOLO_OK = HOLO_STATUS_OK = 0   # HOLO_STATUS_OK in include/holo_b200.h
HOLO_E_ARG, HOLO_E_NOMEM, HOLO_E_UNSUPPORTED, HOLO_E_TIMEOUT, HOLO_E_COMM = 1001, 1002, 1003, 1004, 1005
COMM_HANDLE_BYTES = 128   # HOLO_COMM_HANDLE_BYTES


def row_bytes(gtype: int, cols: int) -> int:
    return cols // BLOCK_ELEMS[gtype] * BLOCK_BYTES[gtype]


_vp, _fp, _i, _f, _sz = C.c_void_p, C.POINTER(C.c_float), C.c_int, C.c_float, C.c_size_t

# name -> (restype, argtypes); the C declarations are in include/*.h
SIGNATURES = {
    # cuda_ops.h
    "cuda_init": (_i, []), "cuda_cleanup": (None, []), "cuda_available": (C.c_bool, []),
    "cuda_print_info": (None, []), "cuda_get_device_count": (_i, []), "cuda_get_free_memory": (_sz, []),
    "cuda_get_device_name": (C.c_char_p, []),
    "cuda_malloc": (_vp, [_sz]), "cuda_free": (None, [_vp]),
    "cuda_memcpy_h2d": (None, [_vp, _vp, _sz]), "cuda_memcpy_d2h": (None, [_vp, _vp, _sz]),
    "cuda_memcpy_d2d": (None, [_vp, _vp, _sz]), "cuda_memcpy_d2d_async": (None, [_vp, _vp, _sz]),
    "cuda_memcpy_d2h_async": (None, [_vp, _vp, _sz]), "cuda_memset": (None, [_vp, _i, _sz]),
    "cuda_sync": (None, []), "cuda_sync_copy": (None, []),
    "cuda_vec_add": (None, [_vp, _vp, _vp, _i]), "cuda_vec_mul": (None, [_vp, _vp, _vp, _i]),
    "cuda_vec_scale": (None, [_vp, _vp, _f, _i]), "cuda_vec_dot": (_f, [_vp, _vp, _i]),
    "cuda_matmul_f32": (None, [_vp, _vp, _vp, _i, _i]), "cuda_matmul_f16": (None, [_vp, _vp, _vp, _i, _i]),
    "cuda_matmul_q8_0": (None, [_vp, _vp, _vp, _i, _i]), "cuda_matmul_q4_0": (None, [_vp, _vp, _vp, _i, _i]),
    "cuda_matmul_q4_k": (None, [_vp, _vp, _vp, _i, _i]), "cuda_matmul_q6_k": (None, [_vp, _vp, _vp, _i, _i]),
    "cuda_batched_qkv_q8_0": (None, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i]),
    "cuda_batched_ffn_gate_up_q8_0": (None, [_vp, _vp, _vp, _vp, _i, _i]),
    "cuda_silu": (None, [_vp, _i]), "cuda_silu_mul": (None, [_vp, _vp, _vp, _i]),
    "cuda_gelu": (None, [_vp, _i]), "cuda_relu": (None, [_vp, _i]),
    "cuda_rms_norm": (None, [_vp, _vp, _vp, _i, _f]), "cuda_layer_norm": (None, [_vp, _vp, _vp, _vp, _i, _f]),
    "cuda_softmax": (None, [_vp, _vp, _i]), "cuda_softmax_inplace": (None, [_vp, _i]),
    "cuda_attention_scores": (None, [_vp, _vp, _vp, _i, _i, _i, _f]),
    "cuda_attention_apply": (None, [_vp, _vp, _vp, _i, _i, _i]),
    "cuda_attention_single": (None, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i]),
    "cuda_multi_head_attention": (None, [_vp, _vp, _vp, _vp, _i, _i, _i, _i]),
    "cuda_rope_apply": (None, [_vp, _vp, _i, _i, _i, _i, _f]),
    "cuda_get_embedding_f32": (None, [_vp, _vp, _i, _i, _i]), "cuda_get_embedding_f16": (None, [_vp, _vp, _i, _i, _i]),
    "cuda_get_embedding_q8_0": (None, [_vp, _vp, _i, _i, _i]), "cuda_get_embedding_q4_0": (None, [_vp, _vp, _i, _i, _i]),
    "cuda_get_embedding_q6_k": (None, [_vp, _vp, _i, _i, _i]),
    "cuda_get_embedding_q4_k": (None, [_vp, _vp, _i, _i, _i]),
    "cuda_argmax": (_i, [_vp, _i]),
    # holo_b200.h
    "cuda_last_status": (_i, []), "cuda_last_status_string": (C.c_char_p, []), "cuda_clear_status": (None, []),
    "cuda_set_act_mode": (None, [_i]), "cuda_get_act_mode": (_i, []),
    "cuda_set_q4k_layout": (None, [_i]), "cuda_get_q4k_layout": (_i, []),
    "cuda_upload_quant": (_vp, [_vp, _i, _i, _i]), "cuda_repack_quant": (_vp, [_vp, _i, _i, _i]),
    "cuda_quant_tiled_bytes": (_sz, [_i, _i, _i]),
    "cuda_matvec": (None, [_vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "cuda_matvec_batch": (_i, [_i, _vp, _vp, _vp, _i]),
    "cuda_matvec_noalloc": (_i, [_vp, _vp, _vp, _i, _i, _i, _i]),
    "cuda_matvec_noalloc_status_word": (_vp, []),
    "cuda_dequantize_rows": (None, [_vp, _vp, _i, _i, _i]),
    "cuda_quantize_act_q8": (None, [_vp, _vp, _vp, _vp, _i]),
    "cuda_block_sums_q8": (None, [_vp, _vp, _vp, _i, _i, _i]),
    "cuda_get_stream": (_vp, []), "cuda_set_stream": (None, [_vp]),
    "cuda_memcpy_h2d_stream": (None, [_vp, _vp, _sz]), "cuda_memcpy_d2h_stream": (None, [_vp, _vp, _sz]),
    "cuda_init_rank": (_i, [_i, _i]), "cuda_sm_count": (_i, []),
    "cuda_set_pdl": (None, [_i]), "cuda_get_pdl": (_i, []),
    "cuda_capture_begin": (_i, []), "cuda_capture_end": (_vp, []),
    "cuda_graph_launch": (None, [_vp]), "cuda_graph_free": (None, [_vp]),
    "holo_model_create": (_vp, [_vp]),
    "holo_model_set_layer": (_i, [_vp, _i] + [_vp] * 9),
    "holo_model_set_layer_types": (_i, [_vp, _i, _i, _i]),
    "holo_model_debug_vector": (_i, [_vp, _i, _vp]),
    "holo_model_set_globals": (_i, [_vp, _vp, _vp, _vp]),
    "holo_model_forward": (_i, [_vp, _i, _vp]),
    "holo_model_prefill": (_i, [_vp, _vp, _i, _vp]),
    "holo_model_set_prompt_mode": (_i, [_vp, _i]),
    "holo_model_load_logits": (_i, [_vp, _vp]),
    "holo_model_push_token": (_i, [_vp, _i]),
    "holo_model_sample": (_i, [_vp, _vp, _f]),
    "holo_model_generate": (_i, [_vp, _vp, _i, _i, _vp, _i, _vp]),
    "holo_model_launch_steps": (_i, [_vp, _i]),
    "cuda_synth_weights": (_i, [_vp, _i, _i, _i, C.c_ulonglong, _f]),
    "holo_model_last_timing": (_i, [_vp, _vp, _vp]),
    "holo_model_pos": (_i, [_vp]), "holo_model_reset": (None, [_vp]), "holo_model_free": (None, [_vp]),
    "cuda_matmul_quant_batched": (_i, [_vp, _vp, _vp, _i, _i, _i]),
    "holo_model_forward_batch": (_i, [_vp, _vp, _vp]),
    "holo_model_generate_batch": (_i, [_vp, _vp, _i, _i, _vp, _vp, _vp]),
    "holo_model_comm_handle": (_i, [_vp, _vp]), "holo_model_shard": (_i, [_vp, _vp]), "holo_model_open_peers": (_i, [_vp, _vp]),
    "holo_tokenizer_create": (_vp, [C.POINTER(C.c_char_p), _i, _i, _i]),
    "holo_tokenize": (_i, [_vp, C.c_char_p, C.POINTER(C.c_int), _i, _i]),
    "holo_tokenizer_free": (None, [_vp]),
}

_LIB = None


def load(path: str | os.PathLike | None = None):
    """Load the shared library and declare its signatures (no device needed)."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = pathlib.Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"{p} is missing: build it with `make -C {PKG_DIR}` (or __graft_entry__.build())")
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _LIB = lib
    return lib


def header_symbols() -> list[str]:
    """Every function name declared in include/*.h (the exported C ABI)."""
    import re
    names = []
    for h in sorted(INCLUDE_DIR.glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w \*]*?\b(\w+)\s*\([^;{]*\)\s*;", text, flags=re.M):
            names.append(m.group(1))
    return names


class Tokenizer:
    """The reference's greedy longest-match tokenizer (llm_tokenize,
    src/ai/llm.c:178-221) through holo_tokenize: host code, no device needed.

    vocab: token strings (bytes or str, UTF-8; None for a missing entry) in
    vocabulary order; bos and unk as the reference's tokenizer.ggml ids."""

    def __init__(self, vocab, bos: int = 1, unk: int = 0):
        self.lib = load()
        enc = [v.encode() if isinstance(v, str) else v for v in vocab]
        arr = (C.c_char_p * len(enc))(*enc)
        self.h = self.lib.holo_tokenizer_create(arr, len(enc), int(bos), int(unk))
        if not self.h:
            raise RuntimeError("holo_tokenizer_create failed")
        self.vocab_size = len(enc)

    def encode(self, text, add_bos: bool = False, max_tokens: int | None = None) -> np.ndarray:
        """Token ids of text (str or bytes; the reference stops at the first
        NUL byte), at most max_tokens (default: one per byte, plus BOS)."""
        b = text.encode() if isinstance(text, str) else bytes(text)
        cap = len(b) + 1 if max_tokens is None else int(max_tokens)
        out = np.zeros(max(cap, 1), np.int32)
        n = self.lib.holo_tokenize(self.h, b, out.ctypes.data_as(C.POINTER(C.c_int)), cap, int(add_bos))
        if n < 0:
            raise RuntimeError("holo_tokenize: bad arguments")
        return out[:n].copy()

    def close(self):
        if getattr(self, "h", None):
            self.lib.holo_tokenizer_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 -- interpreter shutdown may have unloaded the library
            pass


class Device:
    """Thin owner of the library on the current GPU; raises on library errors."""

    def __init__(self, rank: int = 0, world: int = 1):
        self.lib = load()
        if self.lib.cuda_init_rank(rank, world) != 0:
            raise RuntimeError("cuda_init_rank failed: no usable CUDA device")
        self.lib.cuda_clear_status()

    def check(self, what: str = ""):
        st = self.lib.cuda_last_status()
        if st != 0:
            msg = self.lib.cuda_last_status_string().decode(errors="replace")
            self.lib.cuda_clear_status()
            raise RuntimeError(f"holo status {st} ({msg}) {what}")

    # -- memory -------------------------------------------------------------
    def alloc(self, nbytes: int) -> int:
        p = self.lib.cuda_malloc(max(int(nbytes), 1))
        if not p:
            raise MemoryError(f"cuda_malloc({nbytes}) failed")
        return p

    def free(self, p: int):
        if p:
            self.lib.cuda_free(p)

    def upload(self, arr: np.ndarray) -> int:
        arr = np.ascontiguousarray(arr)
        p = self.alloc(arr.nbytes)
        self.lib.cuda_memcpy_h2d(p, arr.ctypes.data, arr.nbytes)
        return p

    def download(self, p: int, shape, dtype) -> np.ndarray:
        out = np.empty(shape, dtype=dtype)
        self.lib.cuda_memcpy_d2h(out.ctypes.data, p, out.nbytes)
        return out

    def upload_quant(self, blocks: np.ndarray, gtype: int, rows: int, cols: int) -> int:
        blocks = np.ascontiguousarray(blocks)
        assert blocks.nbytes == rows * row_bytes(gtype, cols)
        p = self.lib.cuda_upload_quant(blocks.ctypes.data, gtype, rows, cols)
        if not p:
            self.check("cuda_upload_quant")
            raise RuntimeError("cuda_upload_quant returned NULL")
        return p

    def sync(self):
        self.lib.cuda_sync()
