"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; everything else runs on CPU.

The oracle (oracle/) is the checker here and only here: tests compare the
CUDA library, called through its C ABI, against it.
"""
import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
for p in (ROOT / "google-classic_b200", ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

import holo_b200 as hb  # noqa: E402
import holo_oracle  # noqa: E402

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")


@pytest.fixture(scope="session")
def oracle():
    return holo_oracle.Oracle()


@pytest.fixture(scope="session")
def reference():
    try:
        return holo_oracle.Reference()
    except RuntimeError as e:  # neither prebuilt nor buildable here
        pytest.skip(str(e))


@pytest.fixture(scope="session")
def lib():
    return hb.load()


@pytest.fixture(scope="session")
def dev():
    d = hb.Device(0, 1)
    yield d


def rel_err(y, r):
    """max |y - r| / max |r|: the norm-wise relative error of the parity bar."""
    y = np.asarray(y, np.float64)
    r = np.asarray(r, np.float64)
    return float(np.abs(y - r).max() / max(np.abs(r).max(), 1e-30))


def typed_weights(cfg, seed):
    """synth.llama_weights for cfg, with every matrix in the type cfg gives it:
    per-layer wv / w2 types (holo_b200.model.layer_types), Q6_K anywhere
    (seeded random blocks, synth.quant_matrix: there is no Q6_K quantizer
    here), and a quantized token-embedding table when emb_type is a block
    type.  Other roles: N(0, 0.02) quantized round-to-nearest."""
    from holo_b200 import synth
    from holo_b200.model import layer_types
    carrier = dict(cfg, emb_type=1 if cfg.get("emb_type", 1) == 1 else 0)
    for k in ("layer_type", "out_type"):
        if carrier[k] == hb.Q6_K:
            carrier[k] = hb.Q4_K
    w = synth.llama_weights(carrier, seed)
    rng = np.random.default_rng(seed + 1)

    def mat(t, rows, cols, s):
        if t == hb.Q6_K:
            return synth.quant_matrix(t, rows, cols, s)
        return synth.quantize(rng.normal(0, 0.02, (rows, cols)).astype(np.float32), t)

    dim, ffn, V = cfg["dim"], cfg["ffn_dim"], cfg["vocab"]
    q_dim, kv_dim = cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"]
    lt = cfg["layer_type"]
    for l, (L, (tv, t2)) in enumerate(zip(w["layers"], layer_types(cfg))):
        shapes = {"wq": (q_dim, dim, lt), "wk": (kv_dim, dim, lt), "wv": (kv_dim, dim, tv),
                  "wo": (dim, q_dim, lt), "w1": (ffn, dim, lt), "w2": (dim, ffn, t2), "w3": (ffn, dim, lt)}
        for i, (name, (r, c, t)) in enumerate(shapes.items()):
            if t != carrier["layer_type"]:
                L[name] = mat(t, r, c, seed * 100 + l * 10 + i)
    if cfg["out_type"] != carrier["out_type"]:
        w["output"] = mat(cfg["out_type"], V, dim, seed * 100 + 99)
    et = cfg.get("emb_type", 1)
    if et not in (0, 1):
        w["tok_emb"] = mat(et, V, dim, seed * 100 + 98)
    return w
