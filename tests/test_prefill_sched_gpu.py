"""The tensor-core batched matmul's two schedules (csrc/prefill.cu): the tile
grid (pf_mma_kernel: one CTA per 128-row weight tile x token tile x K split)
and the persistent token-range schedule (pf_seg_kernel: the same work cut
into pieces of up to 256 tokens of one weight tile, spread evenly over the
SMs).  Each output element is the same K chunks accumulated in one TMEM
accumulator in the same order under both, so the results must be
bit-identical -- a sharded prompt pass (other row tiles, so other pieces)
relies on that to match one GPU -- and within the restatement's bar (1e-3
norm-wise, test_prefill_gpu).  The schedule is fixed per process
(HOLO_PREFILL_SCHED=tiles / seg), so each runs in a child process.
Cases: 1.5 waves of tiles (M 512), a W1/W3-like 172-tile grid at M 127,
K splits (few row tiles) with pieces crossing split boundaries, a partial
last row tile, ragged token counts, Q4_0 and Q8_0.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

import holo_b200 as hb
from holo_b200 import synth
from conftest import ROOT, rel_err

pytestmark = pytest.mark.gpu

CASES = [(hb.Q4_K, 512, 14336, 1024), (hb.Q4_K, 127, 22016, 512), (hb.Q4_K, 300, 4096, 4096),
         (hb.Q4_K, 256, 512, 4096), (hb.Q4_K, 200, 4000, 1024), (hb.Q4_0, 389, 2816, 768),
         (hb.Q8_0, 160, 3072, 640)]

CHILD = r"""
import json, sys
import numpy as np
sys.path[:0] = [sys.argv[1] + '/google-classic_b200', sys.argv[1] + '/tests']
import holo_b200 as hb
from holo_b200 import synth
cases, out = json.loads(sys.argv[2]), sys.argv[3]
dev = hb.Device(0, 1)
res = {}
for i, (gt, M, N, K) in enumerate(cases):
    W = synth.quant_matrix(gt, N, K, seed=M + N + K)
    X = np.random.default_rng(M * 3 + K).standard_normal((M, K), dtype=np.float32)
    Wd = dev.upload_quant(W, gt, N, K)
    Xd, Yd = dev.upload(X), dev.alloc(4 * M * N)
    assert dev.lib.cuda_matmul_quant_batched(Yd, Wd, Xd, M, N, K) == hb.HOLO_OK
    dev.check("matmul")
    res[str(i)] = dev.download(Yd, (M, N), np.float32)
    for p in (Wd, Xd, Yd):
        dev.free(p)
np.savez(out, **res)
"""


def _run(tmp_path, mode):
    out = tmp_path / f"y_{mode}.npz"
    env = dict(os.environ, HOLO_PREFILL_SCHED=mode)
    p = subprocess.run([sys.executable, "-c", CHILD, str(ROOT), json.dumps(CASES), str(out)], env=env,
                       capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-3000:]
    return dict(np.load(out))


@pytest.fixture(scope="module")
def both(tmp_path_factory):
    tmp = tmp_path_factory.mktemp("sched")
    return _run(tmp, "tiles"), _run(tmp, "seg")


def test_schedules_bit_identical(dev, both):
    tiles, seg = both
    for i, (gt, M, N, K) in enumerate(CASES):
        a, b = tiles[str(i)], seg[str(i)]
        diff = int(np.count_nonzero(a.view(np.uint32) != b.view(np.uint32)))
        print(f"type {gt} M={M} N={N} K={K}: elements differing between the schedules {diff}")
        assert diff == 0


@pytest.mark.parametrize("i", [2, 4, 5, 6])
def test_token_range_schedule_matches_restatement(dev, oracle, both, i):
    gt, M, N, K = CASES[i]
    Y = both[1][str(i)]
    W = synth.quant_matrix(gt, N, K, seed=M + N + K)
    X = np.random.default_rng(M * 3 + K).standard_normal((M, K), dtype=np.float32)
    rows = sorted({0, 1, M // 2, M - 1})
    R = np.stack([oracle.matvec_q8(gt, W, X[m], N, K, threads=8) for m in rows])
    err = rel_err(Y[rows], R)
    print(f"token-range schedule type {gt} M={M} N={N} K={K}: norm-wise rel err {err:.3e}")
    assert np.isfinite(Y).all() and err <= 1e-3
