"""Host logic of the multi-GPU paths on CPU ranks (gloo), world size 2.

* Vocabulary sharding of the entropy stage: each rank computes per-row partials of its
  half of the vocabulary, the partials are all-gathered, every rank combines them; the
  result must equal the single-shard statistics (entropy within 1e-5, argmax and the
  commit selection exact), as the CUDA partials / combine kernels do across GPUs.
* Data-parallel timing: the step time reported is the maximum over ranks.
* The vocabulary-sharded decode step (padded row gather, shard LM head, partials gather,
  combine of the rank's own rows, lock-step stop on the gathered live counts) reproduces
  the unsharded oracle decode.
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


def _sharded_decode_worker(rank, ws, port, q):
    """The vocabulary-sharded streaming decode as the library runs it (decode.cu,
    sharded_select), restated over gloo with the oracle: each rank decodes its own
    prompts; per step the final-normed mask rows, padded to the largest window
    capacity of any rank, and a header (live sequences, mask rows) are all-gathered;
    every rank projects all rows onto its LM-head rows and reduces them to partials; the
    partials are all-gathered and each rank combines its own rows and applies the commit
    rule; the ranks step until the gathered live counts are all zero."""
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "tests")]
    from model_configs import c1_config
    from oracle.decoder import OracleDecoder, compute_block_reorder
    from oracle.model import OracleModel, random_weights
    from oracle.sampler import (SamplingParams, combine_partials, effective_cap,
                                select_by_entropy_with_distance, shard_partials,
                                update_running_entropy)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws,
                            timeout=datetime.timedelta(seconds=120))
    try:
        cfg = c1_config()
        om = OracleModel(cfg, random_weights(cfg, seed=0, std=0.02), "f32")
        mask, V, H = cfg.mask_token_id, cfg.vocab_size, cfg.hidden_size
        lo, hi = rank * V // ws, (rank + 1) * V // ws
        W = om.w["lm_head.weight"][lo:hi]
        tau, lam, cap, n_new = 9.0, 0.01, 3, 20
        win = 12 if rank == 0 else 8
        prompts = np.random.default_rng(300 + rank).integers(1, 4095, size=(2 - rank, 16))
        runs = []
        for p in prompts:
            runs.append(dict(cache=om.prefill_cache(p), clen=len(p), win=[mask] * win,
                             wpos=list(range(len(p), len(p) + win)), next=len(p) + win, out=[],
                             done=False, running=np.float32(tau)))
        # agree on the padded rows per rank (sharded_begin)
        caps = [torch.zeros(1, dtype=torch.int64) for _ in range(ws)]
        dist.all_gather(caps, torch.tensor([len(runs) * win]))
        rmax = max(int(c) for c in caps)
        steps = 0
        while True:
            live = [r for r in runs if not r["done"] and len(r["out"]) < n_new and r["win"]]
            rows, meta = [], []
            for r in live:
                nc = 0
                while nc < len(r["win"]) and r["win"][nc] != mask:
                    nc += 1
                ml = [i for i, t in enumerate(r["win"]) if t == mask]
                ro = compute_block_reorder(r["win"], ml, 0)
                rpos = [r["wpos"][i] for i in ro.block_permutation]
                h, new = om.forward_with_positions(ro.reordered_block, rpos, r["cache"],
                                                   return_hidden=True)
                nc = min(nc, n_new - len(r["out"]))
                keep = r["clen"] + nc
                r["cache"] = [(k[:, :keep], v[:, :keep]) for k, v in new]
                r["clen"] = keep
                rows.append(h[ro.num_filled:])
                meta.append((r, nc, ml))
                if nc:  # commit, drain (EOS ends the sequence), refill
                    toks = r["win"][:nc]
                    del r["win"][:nc], r["wpos"][:nc]
                    if cfg.eos_token_id in toks:
                        r["out"] += toks[:toks.index(cfg.eos_token_id) + 1]
                        r["done"] = True
                        continue
                    r["out"] += toks
                    for _ in range(nc):
                        if len(r["out"]) + len(r["win"]) >= n_new:
                            break
                        r["win"].append(mask)
                        r["wpos"].append(r["next"])
                        r["next"] += 1
            mine = np.zeros((rmax, H), np.float32)
            rr = sum(x.shape[0] for x in rows)
            if rr:
                mine[:rr] = np.concatenate(rows)
            hid = [torch.zeros(rmax, H) for _ in range(ws)]
            hdr = [torch.zeros(2, dtype=torch.int64) for _ in range(ws)]
            dist.all_gather(hid, torch.from_numpy(mine))
            dist.all_gather(hdr, torch.tensor([len(live), rr]))
            allrows = torch.cat(hid).numpy()
            m, S, T, am = shard_partials(allrows @ W.T, lo, 0.0)
            part = torch.from_numpy(np.stack([m, S, T, am.astype(np.float64)], axis=1))
            parts = [torch.zeros_like(part) for _ in range(ws)]
            dist.all_gather(parts, part)
            own = slice(rank * rmax, rank * rmax + rr)
            Hh, amax, _ = combine_partials([(p[own, 0].numpy(), p[own, 1].numpy(), p[own, 2].numpy(),
                                             p[own, 3].numpy().astype(np.int64)) for p in parts])
            off = 0
            for r, nc, ml in meta:
                k = len(ml)
                Hs, toks = Hh[off:off + k], amax[off:off + k]
                off += k
                if k == 0 or r["done"]:
                    continue
                r["running"] = update_running_entropy(r["running"], Hs)
                eff = effective_cap(r["running"], tau, cap)
                for s in select_by_entropy_with_distance(list(Hs), ml, tau, lam, eff):
                    post = max(ml[s] - nc, 0)
                    if post < len(r["win"]):
                        r["win"][post] = int(toks[s])
            steps += 1
            if sum(int(h[0]) for h in hdr) == 0:
                break
        dec = OracleDecoder(om, mask, cfg.eos_token_id)
        ok = True
        for p, r in zip(prompts, runs):
            ref, _ = dec.generate_streaming(p.tolist(), n_new, win, SamplingParams(
                temperature=0.0, entropy_threshold=tau, distance_penalty=lam,
                max_tokens_per_step=cap))
            ok = ok and r["out"] == ref[len(p):]
        q.put((rank, (ok, steps)))
    finally:
        dist.destroy_process_group()


def test_vocab_sharded_decode_protocol_two_ranks():
    """Two gloo ranks with unequal windows and sequence counts reproduce the unsharded
    oracle decode of their own prompts and stop after the same step."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_decode_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res[0][0] and res[1][0], res
    assert res[0][1] == res[1][1]
