"""Seeded synthetic GGUF blocks and activations (the benchmark configurations).

The reference publishes no weights or datasets for this path; inputs are
drawn with the shapes and value distributions of the benchmark configs:

* Q8_0 : d = fp16(|N(0, 0.02)| / 127) per block, qs ~ U{-127..127}
* Q4_0 : d as Q8_0, nibbles ~ U{0..15} (value = d * (nib - 8))
* Q4_K : d, dmin ~ fp16(|N(0, 0.02)| / 127) per super-block, eight 6-bit
         scales and eight 6-bit mins ~ U{0..63} packed so the 6-bit unpack of
         src/ai/quant.c:290-297 returns them, nibbles ~ U{0..15}
* x    : N(0, 1) float32

One numpy PCG64 generator per call, seeded by ``seed``; draw order: block
scales (d, then dmin for Q4_K), then 6-bit scale/min codes (Q4_K), then the
quants.  fp16 rounding is round-to-nearest-even from float64.
"""
from __future__ import annotations

import numpy as np

from . import BLOCK_BYTES, BLOCK_ELEMS, F16, Q4_0, Q4_K, Q6_K, Q8_0


def _rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def _scales(rng, n):
    return (np.abs(rng.normal(0.0, 0.02, size=n)) / 127.0).astype(np.float16)


def pack_q4k_scales(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """[n,8] 6-bit scales and mins -> [n,12] bytes in the quant.c:290-297 packing."""
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    out = np.empty((sc.shape[0], 12), np.uint8)
    out[:, 0:4] = sc[:, 0:4] | ((sc[:, 4:8] & 3) << 6)
    out[:, 4:8] = mn[:, 0:4] | ((mn[:, 4:8] & 3) << 6)
    out[:, 8:12] = (sc[:, 4:8] >> 2) | ((mn[:, 4:8] >> 2) << 4)
    return out


def quant_matrix(gtype: int, rows: int, cols: int, seed: int) -> np.ndarray:
    """rows x cols matrix as GGUF blocks, uint8 array [rows * row_bytes]."""
    rng = _rng(seed)
    nb = rows * cols // BLOCK_ELEMS[gtype]
    out = np.empty((nb, BLOCK_BYTES[gtype]), np.uint8)
    if gtype == Q8_0:
        d = _scales(rng, nb)
        qs = rng.integers(-127, 128, size=(nb, 32), dtype=np.int8)
        out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
        out[:, 2:] = qs.view(np.uint8)
    elif gtype == Q4_0:
        d = _scales(rng, nb)
        nib = rng.integers(0, 16, size=(nb, 32), dtype=np.uint8)
        out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
        out[:, 2:] = nib[:, :16] | (nib[:, 16:] << 4)
    elif gtype == Q4_K:
        d = _scales(rng, nb)
        dmin = _scales(rng, nb)
        codes = rng.integers(0, 64, size=(nb, 16), dtype=np.uint8)
        nib = rng.integers(0, 16, size=(nb, 8, 32), dtype=np.uint8)
        out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
        out[:, 2:4] = dmin.view(np.uint8).reshape(nb, 2)
        out[:, 4:16] = pack_q4k_scales(codes[:, :8], codes[:, 8:])
        out[:, 16:] = (nib[:, :, :16] | (nib[:, :, 16:] << 4)).reshape(nb, 128)
    elif gtype == Q6_K:
        # ql, qh uniform bytes (6-bit codes uniform in 0..63), int8 scales
        # uniform in [-64, 63], d as above
        d = _scales(rng, nb)
        out[:, 0:192] = rng.integers(0, 256, size=(nb, 192), dtype=np.uint8)
        out[:, 192:208] = rng.integers(-64, 64, size=(nb, 16), dtype=np.int8).view(np.uint8)
        out[:, 208:210] = d.view(np.uint8).reshape(nb, 2)
    else:
        raise ValueError(f"no generator for type {gtype}")
    return out.reshape(-1)


def activation(n: int, seed: int) -> np.ndarray:
    return _rng(seed + 0x5EED).standard_normal(n, dtype=np.float32)


def f16_matrix(rows: int, cols: int, seed: int, std: float = 0.02) -> np.ndarray:
    return _rng(seed).normal(0.0, std, size=(rows, cols)).astype(np.float16)


# ---------------------------------------------------------------------------
# round-to-nearest quantizers for model weights (the build's own; the
# reference has no f32 -> Q8_0/Q4_0/Q4_K quantizer)
# ---------------------------------------------------------------------------
def quantize(w: np.ndarray, gtype: int) -> np.ndarray:
    """float32 [rows, cols] -> GGUF blocks (uint8 [rows * row_bytes])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    if gtype == Q8_0:
        b = w.reshape(-1, 32)
        amax = np.abs(b).max(axis=1)
        d = (amax / 127.0).astype(np.float16)
        df = d.astype(np.float32)
        inv = np.where(df > 0, 1.0 / np.where(df > 0, df, 1), 0).astype(np.float32)
        q = np.clip(np.rint(b * inv[:, None]), -127, 127).astype(np.int8)
        out = np.empty((b.shape[0], 34), np.uint8)
        out[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
        out[:, 2:] = q.view(np.uint8)
        return out.reshape(-1)
    if gtype == Q4_0:
        b = w.reshape(-1, 32)
        idx = np.abs(b).argmax(axis=1)
        mx = b[np.arange(b.shape[0]), idx]
        d = (mx / -8.0).astype(np.float16)
        df = d.astype(np.float32)
        inv = np.where(df != 0, 1.0 / np.where(df != 0, df, 1), 0).astype(np.float32)
        q = np.clip(np.rint(b * inv[:, None] + 8.0), 0, 15).astype(np.uint8)
        out = np.empty((b.shape[0], 18), np.uint8)
        out[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
        out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
        return out.reshape(-1)
    if gtype == Q4_K:
        b = w.reshape(-1, 8, 32)
        lo = np.minimum(b.min(axis=2), 0.0)
        hi = b.max(axis=2)
        scale = (hi - lo) / 15.0
        mins = -lo
        d = (scale.max(axis=1) / 63.0).astype(np.float16)
        dmin = (mins.max(axis=1) / 63.0).astype(np.float16)
        df, dmf = d.astype(np.float32), dmin.astype(np.float32)
        sc = np.clip(np.rint(scale / np.where(df > 0, df, 1)[:, None]), 0, 63).astype(np.uint8)
        mn = np.clip(np.rint(mins / np.where(dmf > 0, dmf, 1)[:, None]), 0, 63).astype(np.uint8)
        eff_s = df[:, None] * sc.astype(np.float32)
        eff_m = dmf[:, None] * mn.astype(np.float32)
        q = np.rint((b + eff_m[:, :, None]) / np.where(eff_s > 0, eff_s, 1)[:, :, None])
        q = np.clip(q, 0, 15).astype(np.uint8)
        out = np.empty((b.shape[0], 144), np.uint8)
        out[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
        out[:, 2:4] = dmin.view(np.uint8).reshape(-1, 2)
        out[:, 4:16] = pack_q4k_scales(sc, mn)
        out[:, 16:] = (q[:, :, :16] | (q[:, :, 16:] << 4)).reshape(-1, 128)
        return out.reshape(-1)
    if gtype == F16:
        return w.astype(np.float16).view(np.uint8).reshape(-1)
    raise ValueError(f"no quantizer for type {gtype}")


# ---------------------------------------------------------------------------
# random-init Llama-shape models (weights N(0, std) quantized round-to-nearest)
# ---------------------------------------------------------------------------
def llama_weights(cfg: dict, seed: int, std: float = 0.02) -> dict:
    """Host arrays of a random-init model of shape cfg (keys of
    holo_b200.model.ModelDesc): GGUF blocks of cfg['layer_type'] for the seven
    layer matrices, fp16 (emb_type 1) or fp32 token embeddings, output
    matrix of cfg['out_type'], RMSNorm weights 1.0."""
    rng = _rng(seed)
    dim, hd, nh, nkv, ffn, V = (cfg[k] for k in ("dim", "head_dim", "n_heads", "n_kv_heads", "ffn_dim", "vocab"))
    q_dim, kv_dim = nh * hd, nkv * hd
    lt, ot = cfg["layer_type"], cfg["out_type"]

    def mat(rows, cols, t):
        return quantize(rng.normal(0.0, std, size=(rows, cols)).astype(np.float32), t)

    layers = []
    for _ in range(cfg["n_layers"]):
        layers.append({
            "attn_norm": np.ones(dim, np.float32), "ffn_norm": np.ones(dim, np.float32),
            "wq": mat(q_dim, dim, lt), "wk": mat(kv_dim, dim, lt), "wv": mat(kv_dim, dim, lt),
            "wo": mat(dim, q_dim, lt), "w1": mat(ffn, dim, lt), "w2": mat(dim, ffn, lt), "w3": mat(ffn, dim, lt),
        })
    emb = rng.normal(0.0, std, size=(V, dim)).astype(np.float32)
    if cfg.get("emb_type", 1) == 1:
        emb = emb.astype(np.float16)
    return {"layers": layers, "tok_emb": np.ascontiguousarray(emb), "final_norm": np.ones(dim, np.float32),
            "output": mat(V, dim, ot)}
