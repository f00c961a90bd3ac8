"""Host logic of the sharded decode engine, on CPU: the row shards that
holo_model_create assigns (holo_model_shard), the argument checks of a
sharded holo_model_create, and the handle exchange of connect_peers across
two gloo ranks (tests/shard_worker.py host)."""
import json
import os
import socket
import subprocess
import sys

import pytest

import holo_b200 as hb
from holo_b200.model import LLAMA2_7B, LLAMA3_70B, Model, shard_ranges
from conftest import ROOT

sys.path.insert(0, str(ROOT / "tests"))
from shard_worker import CFG, CFG4, tiles  # noqa: E402


@pytest.mark.parametrize("cfg", [CFG, CFG4, LLAMA2_7B, LLAMA3_70B], ids=["test", "test4", "7b", "70b"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shards_tile_every_matrix(cfg, world):
    if cfg["n_kv_heads"] % world:
        with pytest.raises(ValueError):
            shard_ranges(cfg, world, 0)
        return
    parts = [shard_ranges(cfg, world, r) for r in range(world)]
    for key, n, unit in (("heads", cfg["n_heads"], 1), ("kv_heads", cfg["n_kv_heads"], 1), ("dim", cfg["dim"], 1),
                         ("ffn", cfg["ffn_dim"], 16), ("vocab", cfg["vocab"], 1)):
        assert tiles([p[key] for p in parts], n, unit), (key, [p[key] for p in parts])
    g = cfg["n_heads"] // cfg["n_kv_heads"]
    for p in parts:   # whole GQA groups per rank
        assert p["heads"] == (p["kv_heads"][0] * g, p["kv_heads"][1] * g)


@pytest.mark.parametrize("world,rank,change", [
    (3, 0, {}),                        # 32 heads over 3
    (9, 0, {}),                        # more ranks than supported
    (2, 2, {}),                        # rank out of range
    (2, -1, {}),
    (2, 0, {"head_dim": 64, "n_heads": 8, "n_kv_heads": 8}),   # the step kernel serves head_dim 128
    (8, 0, {"ffn_dim": 112}),          # fewer 16-row bands than ranks
])
def test_create_rejects_bad_sharding(lib, world, rank, change):
    lib.cuda_clear_status()
    cfg = dict(LLAMA2_7B, **change)
    with pytest.raises(RuntimeError, match="sharding"):
        Model(cfg, world=world, rank=rank)
    lib.cuda_clear_status()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_exchange_handles_and_agree_on_shards(tmp_path):
    env = dict(os.environ, OMP_NUM_THREADS="1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={free_port()}", str(ROOT / "tests" / "shard_worker.py"),
           "host", str(tmp_path)]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=240)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    for r in range(2):
        res = json.loads((tmp_path / f"host_{r}.json").read_text())
        assert res and all(res.values()), (r, res)


@pytest.mark.parametrize("cfg", [LLAMA2_7B, LLAMA3_70B], ids=["7b", "70b"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_prompt_pass_slices_are_whole_float4s(cfg, world):
    """Sharded prompt passes exchange each rank's column slice with 16-byte
    peer stores, so every slice's offset and width must be a multiple of 4
    floats (holo_model_create falls back to one position a step otherwise):
    true for the bench models at every world size."""
    hd = cfg["head_dim"]
    for r in range(world):
        p = shard_ranges(cfg, world, r)
        for first, count in ((p["heads"][0] * hd, p["heads"][1] * hd), p["dim"], p["ffn"]):
            assert first % 4 == 0 and count % 4 == 0, (world, r, p)
