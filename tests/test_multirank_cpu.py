"""Host logic of the multi-GPU paths on CPU ranks (gloo), world size 2.

* Vocabulary sharding of the entropy stage: each rank computes per-row partials of its
  half of the vocabulary, the partials are all-gathered, every rank combines them; the
  result must equal the single-shard statistics (entropy within 1e-5, argmax and the
  commit selection exact), as the CUDA partials / combine kernels do across GPUs.
* Data-parallel timing: the step time reported is the maximum over ranks.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, ws, port, q):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    from oracle.sampler import (combine_partials, row_stats, select_by_entropy_with_distance,
                                shard_partials)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws,
                            timeout=datetime.timedelta(seconds=60))
    try:
        rng = np.random.default_rng(11)
        rows, V = 24, 4096
        x = (rng.standard_normal((rows, V)) * 2.5).astype(np.float32)
        x[np.arange(rows), rng.integers(0, V, rows)] += 30.0  # confident rows too
        x[3, 100] = x[3, 3000] = 80.0                          # a cross-shard tie
        Vr = V // ws
        m, S, T, am = shard_partials(x[:, rank * Vr:(rank + 1) * Vr], rank * Vr, 0.0)
        mine = torch.tensor(np.stack([m, S, T, am.astype(np.float64)], axis=1))
        got = [torch.empty_like(mine) for _ in range(ws)]
        dist.all_gather(got, mine)
        parts = [(g[:, 0].numpy(), g[:, 1].numpy(), g[:, 2].numpy(), g[:, 3].numpy().astype(np.int64))
                 for g in got]
        H, amax, mp_ = combine_partials(parts)
        H0, am0, mp0 = row_stats(x, 0.0)
        ok = bool(np.abs(H - H0).max() <= 1e-5 and (amax == am0).all() and
                  np.allclose(mp_, mp0, rtol=1e-6))
        sel = select_by_entropy_with_distance(H.tolist(), list(range(rows)), 0.8, 0.05, 8)
        sel0 = select_by_entropy_with_distance(H0.tolist(), list(range(rows)), 0.8, 0.05, 8)
        ok = ok and sel == sel0
        # max-over-ranks step time
        t = torch.tensor([1.0 + rank])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ok = ok and float(t) == float(ws)
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_vocab_sharded_combine_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: True, 1: True}
