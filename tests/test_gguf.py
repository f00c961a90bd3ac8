"""GGUF files (holo_b200/gguf.py) against the reference's own parser
(src/ai/gguf.c, compiled into oracle/_ref): a model written with the
reference's tensor names and metadata keys reads back byte for byte, the
same bytes the reference's loader would hand to upload_tensor, and the same
configuration; files whose general.alignment exceeds 32 -- which the
reference's loader misplaces, since it always rounds the data section to 32
(gguf.c:354-356) -- read correctly.  CPU only; the GPU test loads such a file
into the decode engine."""
import numpy as np
import pytest

import holo_b200 as hb
from holo_b200 import gguf, synth

CFG = dict(n_layers=2, dim=256, n_heads=4, n_kv_heads=2, head_dim=64, ffn_dim=512, vocab=300, max_seq=96,
           rope_base=500000.0, eps=1e-5, layer_type=hb.Q4_K, emb_type=1, out_type=hb.Q8_0)


@pytest.fixture(scope="module")
def weights():
    return synth.llama_weights(CFG, seed=5)


def source_bytes(w):
    """name -> the bytes written for it"""
    out = {"token_embd.weight": w["tok_emb"], "output_norm.weight": w["final_norm"], "output.weight": w["output"]}
    for l, L in enumerate(w["layers"]):
        for k, n in gguf.LAYER_TENSORS.items():
            out[f"blk.{l}.{n}.weight"] = L[k]
    return {k: np.ascontiguousarray(v).view(np.uint8).reshape(-1) for k, v in out.items()}


@pytest.mark.parametrize("alignment", [32, 64, 256])
def test_roundtrip(tmp_path, weights, alignment):
    path = tmp_path / f"m{alignment}.gguf"
    gguf.write_model(path, CFG, weights, alignment=alignment)
    with gguf.GGUFFile(path) as g:
        assert g.alignment == alignment and g.data_offset % alignment == 0
        for name, want in source_bytes(weights).items():
            got = np.ascontiguousarray(g.tensor(name)).view(np.uint8).reshape(-1)
            assert np.array_equal(got, want), name
            assert g.tensors[name][2] % alignment == 0
        got = gguf.model_config(g)
        # the metadata holds float32 values (as the reference reads them, gguf_get_float)
        assert np.float32(got.pop("eps")) == np.float32(CFG["eps"])
        assert got == {k: v for k, v in CFG.items() if k != "eps"}


def test_reference_parser_reads_the_same(tmp_path, weights, reference):
    path = tmp_path / "m.gguf"
    gguf.write_model(path, CFG, weights)
    src = source_bytes(weights)
    with gguf.GGUFFile(path) as g:
        for name in g.tensors:
            ref, t = reference.gguf_tensor(path, name, 1 << 22)
            ours = np.ascontiguousarray(g.tensor(name)).view(np.uint8).reshape(-1)
            assert t == g.tensors[name][1] and np.array_equal(ref, ours) and np.array_equal(ref, src[name]), name
    for key, v in (("block_count", 2), ("embedding_length", 256), ("attention.head_count", 4),
                   ("attention.head_count_kv", 2), ("attention.key_length", 64), ("feed_forward_length", 512),
                   ("context_length", 96)):
        assert reference.gguf_int(path, f"llama.{key}") == v, key
    assert reference.gguf_float(path, "llama.rope.freq_base") == 500000.0
    assert np.float32(reference.gguf_float(path, "llama.attention.layer_norm_rms_epsilon")) == np.float32(1e-5)


def test_large_alignment_is_where_the_reference_misplaces_data(tmp_path, weights):
    """With general.alignment 256 the data section starts on a multiple of
    256; rounding the header end to 32, as gguf.c:354-356 does, lands
    elsewhere whenever the two differ, and the first tensor's bytes there are
    not the tensor (reading the map at that offset, not calling the reference,
    whose reads could run past the end of the file)."""
    path = tmp_path / "m256.gguf"
    gguf.write_model(path, CFG, weights, alignment=256)
    with gguf.GGUFFile(path) as g:
        ref_offset = (g._pos + 31) // 32 * 32
        assert g.data_offset % 256 == 0 and ref_offset != g.data_offset   # this file's header ends off 256
        name = "token_embd.weight"
        n = gguf.tensor_nbytes(g.tensors[name][1], g.tensors[name][0])
        wrong = np.frombuffer(g._mm, np.uint8, count=n, offset=ref_offset + g.tensors[name][2])
        assert not np.array_equal(wrong, source_bytes(weights)[name])


def test_tied_output_and_mixed_types(tmp_path, weights):
    # no output.weight: the output matrix is the token embedding (llm.c:380-384)
    cfg = dict(CFG, emb_type=1)
    path = tmp_path / "tied.gguf"
    meta = {"general.architecture": "llama", "llama.block_count": 2, "llama.embedding_length": 256,
            "llama.attention.head_count": 4, "llama.attention.head_count_kv": 2, "llama.feed_forward_length": 512,
            "llama.context_length": 96}
    t = {"token_embd.weight": (hb.F16, (256, 300), weights["tok_emb"]),
         "output_norm.weight": (hb.F32, (256,), weights["final_norm"])}
    shapes = {"wq": (256, 256), "wk": (256, 128), "wv": (256, 128), "wo": (256, 256), "w1": (256, 512),
              "w2": (512, 256), "w3": (256, 512)}
    for l, L in enumerate(weights["layers"]):
        for k, n in gguf.LAYER_TENSORS.items():
            t[f"blk.{l}.{n}.weight"] = (hb.F32, (256,), L[k]) if k.endswith("norm") else (hb.Q4_K, shapes[k], L[k])
    gguf.write(path, meta, t)
    with gguf.GGUFFile(path) as g:
        c = gguf.model_config(g)
        assert c["out_type"] == hb.F16 and c["head_dim"] == 64 and c["rope_base"] == 10000.0
        w = gguf.model_weights(g, c)
        assert np.array_equal(w["output"], weights["tok_emb"])
    # a layer's ffn_down (or attn_v) of another type: per-layer types, as the
    # reference binds them (llm.c:445-507)
    t["blk.1.ffn_down.weight"] = (hb.Q8_0, (512, 256), synth.quant_matrix(hb.Q8_0, 256, 512, 1))
    gguf.write(path, meta, t)
    with gguf.GGUFFile(path) as g:
        c = gguf.model_config(g)
        assert c["w2_types"] == [hb.Q4_K, hb.Q8_0] and c["wv_types"] == [hb.Q4_K, hb.Q4_K]
    # one of the five matrices that share the reference's g_weight_type in
    # another type: rejected (llm_forward would read it as g_weight_type)
    t["blk.1.ffn_up.weight"] = (hb.Q8_0, (256, 512), synth.quant_matrix(hb.Q8_0, 512, 256, 2))
    gguf.write(path, meta, t)
    with gguf.GGUFFile(path) as g, pytest.raises(ValueError, match="several types"):
        gguf.model_config(g)


def test_rejects_bad_files(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGML" + b"\0" * 60)
    with pytest.raises(ValueError, match="not a GGUF"):
        gguf.GGUFFile(p)
    gguf.write(p, {"x": 1}, {"t": (hb.F32, (8,), np.zeros(8, np.float32))})
    data = p.read_bytes()
    p.write_bytes(data[:-16])   # tensor data cut short
    with gguf.GGUFFile(p) as g, pytest.raises(ValueError, match="past the end"):
        g.tensor("t")


def test_metadata_arrays_roundtrip(tmp_path, reference):
    """Arrays of strings, float32 and int32 (the tokenizer.ggml.* kinds):
    written, read back here (strings also as raw bytes) and by the
    reference's parser (gguf_get_array, gguf.c:479-487)."""
    toks = ["a", "▁b", "中", "", "<0x0A>"]
    meta = {"general.architecture": "llama", "tokenizer.ggml.tokens": toks,
            "tokenizer.ggml.scores": [0.5, -1.25, 3.0, 0.0, -0.5], "tokenizer.ggml.token_type": [1, 2, 3, 1, 6]}
    path = tmp_path / "arr.gguf"
    gguf.write(path, meta, {"t": (hb.F32, (8,), np.zeros(8, np.float32))})
    with gguf.GGUFFile(path) as g:
        assert g.meta["tokenizer.ggml.tokens"] == toks
        assert g.string_array("tokenizer.ggml.tokens") == [t.encode() for t in toks]
        assert g.meta["tokenizer.ggml.scores"] == [0.5, -1.25, 3.0, 0.0, -0.5]
        assert g.meta["tokenizer.ggml.token_type"] == [1, 2, 3, 1, 6]
        assert g.string_array("tokenizer.ggml.scores") is None and g.string_array("absent") is None
        assert np.array_equal(g.tensor("t"), np.zeros(8, np.float32))   # data section still found
    assert reference.gguf_tokens(path) == [t.encode() for t in toks]
    for key in ("tokenizer.ggml.scores", "tokenizer.ggml.token_type"):
        assert reference.lib.href_gguf_array_len(str(path).encode(), key.encode()) == 5
