"""One rank of the sharded-decode tests, run under torch.distributed.run by
test_shard_host.py (gloo, CPU) and test_shard_gpu.py (one GPU per rank).

  python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
      --master-port P tests/shard_worker.py {host|gpu} OUT_DIR

host: every rank computes its row shard through the library (holo_model_shard)
      and exchanges comm handles of a stand-in model through connect_peers;
      the ranks check that the shards tile every matrix and that every rank
      received every handle in rank order.
gpu:  every rank builds its shard of the test model (cfg_for(N)), connects the peers and
      runs the decode calls (generate's prompt and one holo_model_prefill in
      sharded row passes), then a 32-head model (CFG_SPLIT) over a 176-position
      stream; rank 0 writes the logits and token streams to OUT_DIR/gpu.npz
      for the parent test to compare with the reference and one GPU.
timeout: failure detection without a fault: both ranks connect, then rank 1
      stays alive but skips the step; rank 0's step waits for rank 1's slices,
      gives up after its bound and reports HOLO_E_TIMEOUT; rank 0 then clears
      the status and checks that its device still computes (a matvec against
      the oracle) before the ranks meet on the host and exit.
"""
import datetime
import json
import os
import pathlib
import sys

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "google-classic_b200"))

import holo_b200 as hb  # noqa: E402
from holo_b200.model import (LLAMA2_7B, LLAMA3_70B, Model, SamplerDesc, connect_peers,  # noqa: E402
                             shard_ranges)

# the decode test model (GQA, SwiGLU, Q4_K layers, fp16 embeddings, Q8_0 output)
CFG = dict(n_layers=2, dim=512, n_heads=4, n_kv_heads=2, head_dim=128, ffn_dim=768, vocab=1000, max_seq=160,
           rope_base=10000.0, eps=1e-5, layer_type=hb.Q4_K, emb_type=1, out_type=hb.Q8_0)
# four KV heads, for four ranks (one KV head and its GQA pair of query heads each)
CFG4 = dict(CFG, dim=1024, n_heads=8, n_kv_heads=4, ffn_dim=1536)
# eight KV heads, for eight ranks (one query and one KV head each)
CFG8 = dict(CFG4, n_kv_heads=8)
# the 7B's 32 heads of 128 (8 KV heads): a head's positions are cut into
# several attention splits once the stream is long, and the cut must not
# depend on the world size
CFG_SPLIT = dict(n_layers=2, dim=4096, n_heads=32, n_kv_heads=8, head_dim=128, ffn_dim=1024, vocab=1024,
                 max_seq=192, rope_base=10000.0, eps=1e-5, layer_type=hb.Q4_K, emb_type=1, out_type=hb.Q8_0)
PROMPT_SEED, N_PROMPT, N_GREEDY, N_SAMPLED, N_ROWS = 21, 24, 48, 32, 20
SPLIT_SEED, N_SPLIT_PROMPT, N_SPLIT_GREEDY = 12, 16, 160


def cfg_for(world):
    """the gpu-mode model for a world size: CFG on two ranks, CFG4 on four, CFG8 on eight"""
    return CFG if world <= 2 else CFG4 if world <= 4 else CFG8


def split_prompt():
    return np.random.default_rng(SPLIT_SEED).integers(0, CFG_SPLIT["vocab"], size=N_SPLIT_PROMPT).astype(np.int32)


def split_long_prompt():
    return np.random.default_rng(SPLIT_SEED + 1).integers(0, CFG_SPLIT["vocab"], size=100).astype(np.int32)


class StandInModel:
    """comm_handle / open_peers of a model, without a device."""

    def __init__(self, world, rank):
        self.world, self.rank, self.opened = world, rank, None

    def comm_handle(self):
        return bytes([self.rank]) * hb.COMM_HANDLE_BYTES

    def open_peers(self, handles):
        self.opened = handles


def tiles(parts, n, unit=1):
    """parts: (first, count) per rank, in rank order: contiguous, covering [0, n)."""
    pos = 0
    for first, count in parts:
        if first != pos or count <= 0 or first % unit or count % unit:
            return False
        pos += count
    return pos == n


def run_host(rank, world, out):
    import torch.distributed as dist
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    res = {}
    for name, cfg in (("test", CFG), ("7b", LLAMA2_7B), ("70b", LLAMA3_70B)):
        if cfg["n_kv_heads"] % world:
            continue
        mine = shard_ranges(cfg, world, rank)
        every = [None] * world
        dist.all_gather_object(every, mine)
        res[name] = all(tiles([e[k] for e in every], n, u) for k, n, u in
                        (("heads", cfg["n_heads"], 1), ("kv_heads", cfg["n_kv_heads"], 1), ("dim", cfg["dim"], 1),
                         ("ffn", cfg["ffn_dim"], 16), ("vocab", cfg["vocab"], 1)))
        # GQA groups stay whole: the rank's KV heads serve exactly its query heads
        h, kv = mine["heads"], mine["kv_heads"]
        g = cfg["n_heads"] // cfg["n_kv_heads"]
        res[name + "_gqa"] = h[0] == kv[0] * g and h[1] == kv[1] * g
    m = StandInModel(world, rank)
    connect_peers(m)
    res["handles"] = m.opened == [bytes([r]) * hb.COMM_HANDLE_BYTES for r in range(world)]
    dist.barrier()
    dist.destroy_process_group()
    (pathlib.Path(out) / f"host_{rank}.json").write_text(json.dumps(res))


def run_gpu(rank, world, out):
    import torch
    import torch.distributed as dist
    from holo_b200 import synth
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    hb.Device(local, world)
    cfg = cfg_for(world)
    w = synth.llama_weights(cfg, seed=11)
    prompt = np.random.default_rng(PROMPT_SEED).integers(0, cfg["vocab"], size=N_PROMPT).astype(np.int32)
    res = {}
    try:
        for tag, act, kv16 in (("f32", hb.ACT_F32, False), ("q8", hb.ACT_Q8, True)):
            m = Model(cfg, act_mode=act, kv_f16=kv16, world=world, rank=rank)
            m.set_weights(w)
            connect_peers(m)
            res[f"{tag}_logits"] = np.stack([m.forward(t) for t in prompt])
            res[f"{tag}_greedy"] = m.generate(prompt[:16], N_GREEDY, SamplerDesc(0.0, 0.95, 40, 1.1, 64), seed=5)
            res[f"{tag}_sampled"] = m.generate(prompt[:16], N_SAMPLED, SamplerDesc(0.8, 0.95, 40, 1.1, 64), seed=7)
            if act == hb.ACT_Q8:   # a sharded prompt pass, then steps that read its cache
                m.reset()
                m.prefill(prompt[:N_ROWS], want_logits=False)
                res["q8_rows_logits"] = np.stack([m.forward(t) for t in prompt[N_ROWS:]])
            dist.barrier()
            m.close()
        # 32 heads, a 176-position stream: several attention splits a head
        from holo_b200.model import synthetic_model
        m = synthetic_model(CFG_SPLIT, seed=SPLIT_SEED, act_mode=hb.ACT_Q8, kv_f16=True, world=world, rank=rank)
        connect_peers(m)
        sp = split_prompt()
        res["split_greedy"] = m.generate(sp, N_SPLIT_GREEDY, SamplerDesc(0.0, 0.95, 40, 1.1, 64), seed=5)
        m.reset()
        res["split_logits"] = np.stack([m.forward(t) for t in np.concatenate([sp, res["split_greedy"]])])
        # a 100-row prompt pass (tensor-core matmuls whose K split is planned
        # for the whole matrices), then one step reading its cache
        m.reset()
        lp = split_long_prompt()
        m.prefill(lp[:-1], want_logits=False)
        res["split_rows_logits"] = m.forward(int(lp[-1]))
        dist.barrier()
        m.close()
        # every rank computed the same logits and tokens
        for k in sorted(res):
            every = [None] * world
            dist.all_gather_object(every, res[k])
            res[k + "_ranks_equal"] = np.array(all(np.array_equal(e, every[0]) for e in every))
    finally:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        np.savez(pathlib.Path(out) / "gpu.npz", **res)


def run_timeout(rank, world, out):
    import time
    import torch
    import torch.distributed as dist
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    # gloo: the host-side meeting after the failure needs no GPU collective
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    from holo_b200 import synth
    dev = hb.Device(local, world)
    w = synth.llama_weights(CFG, seed=11)
    m = Model(CFG, act_mode=hb.ACT_Q8, kv_f16=True, world=world, rank=rank)
    m.set_weights(w)
    connect_peers(m)
    res = {}
    if rank == 0:
        t0 = time.perf_counter()
        try:
            m.forward(5)
            res["raised"], res["message"] = False, ""
        except RuntimeError as e:   # the status the step recorded, cleared by the raise
            res["raised"], res["message"] = True, str(e)
        res["seconds"] = time.perf_counter() - t0
        m.lib.cuda_clear_status()
        # the context still computes: a matvec against the restatement
        sys.path.insert(0, str(ROOT / "oracle"))
        import holo_oracle
        Wq = synth.quant_matrix(hb.Q4_K, 64, 512, 3)
        x = synth.activation(512, 3)
        Wd, xd, yd = dev.upload_quant(Wq, hb.Q4_K, 64, 512), dev.upload(x), dev.alloc(4 * 64)
        dev.lib.cuda_matvec(yd, Wd, xd, 64, 512, hb.Q4_K, hb.ACT_Q8, None)
        y = dev.download(yd, (64,), np.float32)
        dev.check("matvec after the time-out")
        r = holo_oracle.Oracle().matvec_q8(hb.Q4_K, Wq, x, 64, 512)
        res["after_rel_err"] = float(np.abs(y - r).max() / np.abs(r).max())
        (pathlib.Path(out) / "timeout.json").write_text(json.dumps(res))
    # rank 1 never launched the step; both meet here (rank 1 keeps its memory
    # mapped until rank 0's kernels are over)
    dist.barrier()
    m.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    mode, out = sys.argv[1], sys.argv[2]
    r, n = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    {"host": run_host, "gpu": run_gpu, "timeout": run_timeout}[mode](r, n, out)
