"""Multi-GPU host logic (cpu_model_b200.shard) on CPU: world_size-2 gloo
process groups run the real exchanges (all-gather of column shards,
all_to_all_single dispatch/return of MoE routes); the per-rank compute is the
CPU oracle, so the sharded results can be compared with the single-process
oracle."""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import oracle
from cpu_model_b200 import shard, synth

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import shard_workers  # noqa: E402


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_row_shards_cover_and_balance():
    for n, w in ((11008, 8), (4096, 3), (5, 8), (1, 2)):
        sh = shard.row_shards(n, w)
        assert sh[0][0] == 0 and sh[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(sh, sh[1:]))
        sizes = [hi - lo for lo, hi in sh]
        assert max(sizes) - min(sizes) <= 1
    assert [shard.expert_owner(e, 8, 4) for e in range(8)] == [0, 0, 1, 1, 2, 2, 3, 3]


@pytest.mark.parametrize("fmt", [4, 8])
def test_column_sharded_pair_gloo(tmp_path, fmt):
    """Column shards + all-gather reproduce the single-process pair exactly
    (each output row is computed by one rank with the full K)."""
    b, d, f = 3, 128, 224        # f not a multiple of the world size's shard
    mp.spawn(shard_workers.pair_worker, args=(2, free_port(), fmt, b, d, f, str(tmp_path)), nprocs=2, join=True)
    wu, su = synth.weights(fmt, f, d, -7, -3, 1)
    wd, sd = synth.weights(fmt, d, f, -7, -3, 2)
    x = synth.normal((b, d), 3)
    xq, xs = oracle.quantize_x(x)
    h = oracle.gemv(fmt, xq, xs, wu, su, f, d)
    hq, hs = oracle.quantize_x(h)
    ref = oracle.gemv(fmt, hq, hs, wd, sd, d, f)
    for r in range(2):
        assert np.array_equal(np.load(os.path.join(str(tmp_path), "pair_%d.npy" % r)), ref)


@pytest.mark.parametrize("fmt", [4, 8])
def test_moe_expert_parallel_gloo(tmp_path, fmt):
    """Experts split over 2 ranks, routes exchanged with all_to_all_single:
    every rank's tokens get the single-process oracle MoE result."""
    t, d, f, e, k = 10, 128, 256, 4, 2
    mp.spawn(shard_workers.moe_worker, args=(2, free_port(), fmt, t, d, f, e, k, str(tmp_path)), nprocs=2,
             join=True)
    experts = shard_workers.moe_experts(fmt, e, d, f)
    for r in range(2):
        x = synth.normal((t, d), 100 + r)
        logits = synth.normal((t, e), 200 + r)
        ref = oracle.moe(fmt, x, logits, d, f, k, experts)
        y = np.load(os.path.join(str(tmp_path), "moe_%d.npy" % r))
        assert np.linalg.norm(ref) > 0
        err = np.linalg.norm(y.astype(np.float64) - ref) / np.linalg.norm(ref)
        assert err <= 1e-6
