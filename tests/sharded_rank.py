"""One rank of the vocabulary-sharded decode tests (run as its own process, one GPU each).

    python tests/sharded_rank.py CASE RANK NRANKS UID_HEX OUT_JSON

The rank holds LM-head rows [rank * V / nranks, (rank + 1) * V / nranks), joins the NCCL
communicator through wedlm_comm_init and decodes its own sequences with the streaming
loop; the LM head and the entropy pass run sharded over all ranks.  Cases:
  c1     fp32 parity model; rank r decodes 2 - r prompts (the ranks' windows differ, so the
         gathered buffers carry padding rows); the ids go to OUT_JSON for the oracle check.
  bf16   1-layer bf16 model; the ids of the sharded decode and of a whole-vocabulary
         context on the same GPU go to OUT_JSON.
  leave  both ranks run one sharded step; then rank 1 exits between steps and rank 0's
         next step must end with WEDLM_ERR_TIMEOUT within the communicator timeout.
  sample       fp32 parity model at T > 0 (multinomial and nucleus), seeded per rank; the
               ids go to OUT_JSON for the oracle check.
  sample_bf16  1-layer bf16 model at T > 0 (multinomial and nucleus); the ids of the
               sharded decode and of a whole-vocabulary context with the same seed.
  mismatch     rank 0 asks for T = 0 and rank 1 for T > 0: both ranks' decode_begin must
               refuse with WEDLM_ERR_INVALID_ARG, and a matching decode must then run.
"""
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "wedlm-rs_b200"), os.path.dirname(os.path.abspath(__file__))):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402,F401  (loads the process's NCCL before the library does)

from oracle.model import random_weights  # noqa: E402
from model_configs import c1_config, long_ctx_bf16_config, to_model_config  # noqa: E402

C1_PARAMS = (9.0, 0.01, 3)  # tau, lambda, cap: the threshold branch commits several per step


def params(tau, lam, cap):
    from wedlm_b200 import SamplingParams
    return SamplingParams(temperature=0.0, entropy_threshold=tau, distance_penalty=lam,
                          max_tokens_per_step=cap)


# (temperature, top_p) of the T > 0 cases
SAMPLE_MODES = {"multinomial": (0.8, 1.0), "nucleus": (1.0, 0.7)}


def sample_params(T, top_p, tau, lam, cap):
    from wedlm_b200 import SamplingParams
    return SamplingParams(temperature=T, top_p=top_p, entropy_threshold=tau,
                          distance_penalty=lam, max_tokens_per_step=cap)


def c1_prompts(rank):
    rng = np.random.default_rng(100 + rank)
    return rng.integers(1, 4095, size=(2 - rank, 16))


def bf16_prompts(rank):
    rng = np.random.default_rng(200 + rank)
    return rng.integers(0, 2046, size=(1, 40))


def shard_ctx(cfg, w, rank, nranks, max_seqs, max_ctx, block):
    from wedlm_b200 import Context
    mc = to_model_config(cfg, max_block_tokens=block)
    V = cfg.vocab_size
    mc.vocab_shard_begin, mc.vocab_shard_end = rank * V // nranks, (rank + 1) * V // nranks
    ctx = Context(mc, max_seqs=max_seqs, max_ctx=max_ctx)
    ctx.load_weights(w)
    return ctx


def main():
    case, rank, nranks, uid_hex, out = sys.argv[1:6]
    rank, nranks = int(rank), int(nranks)
    uid = bytes.fromhex(uid_hex)
    res = {"rank": rank}
    if case == "c1":
        cfg = c1_config()
        w = random_weights(cfg, seed=0, std=0.02)
        ctx = shard_ctx(cfg, w, rank, nranks, 2, 256, 32)
        ctx.comm_init(uid, rank, nranks, timeout_ms=60000)
        win = 12 if rank == 0 else 8
        outs, steps = ctx.generate_streaming_batch(c1_prompts(rank), 24, win, params(*C1_PARAMS))
        res["ids"] = [list(map(int, o)) for o in outs]
        res["steps"] = [int(s) for s in steps]
        res["window"] = win
        ctx.close()
    elif case == "bf16":
        from wedlm_b200 import Context
        cfg = long_ctx_bf16_config()
        w = random_weights(cfg, seed=3, std=0.02)
        ctx = shard_ctx(cfg, w, rank, nranks, 1, 512, 32)
        ctx.comm_init(uid, rank, nranks, timeout_ms=60000)
        prm = params(0.8, 0.05, 8)
        outs, _ = ctx.generate_streaming_batch(bf16_prompts(rank), 32, 16, prm)
        res["ids"] = [list(map(int, o)) for o in outs]
        ctx.close()
        full = Context(to_model_config(cfg, max_block_tokens=32), max_seqs=1, max_ctx=512)
        full.load_weights(w)
        outs, _ = full.generate_streaming_batch(bf16_prompts(rank), 32, 16, prm)
        res["ids_whole_vocab"] = [list(map(int, o)) for o in outs]
        full.close()
    elif case == "leave":
        from wedlm_b200 import WedlmError
        cfg = c1_config()
        w = random_weights(cfg, seed=0, std=0.02)
        ctx = shard_ctx(cfg, w, rank, nranks, 1, 256, 32)
        ctx.comm_init(uid, rank, nranks, timeout_ms=3000)
        ctx.decode_begin([0], c1_prompts(1), 24, 8, params(0.8, 0.05, 8))
        res["live_after_first_step"] = ctx.decode_step(1)
        if rank == 1:
            # leave between steps: nothing of this rank is in flight
            with open(out, "w") as f:
                json.dump(res, f)
            os._exit(0)
        t0 = time.time()
        try:
            ctx.decode_step(1)
            res["code"] = 0
        except WedlmError as e:
            res["code"] = e.code
            res["message"] = str(e)
        res["seconds"] = time.time() - t0
        ctx.decode_end()
        # the context still runs work that needs no communicator
        ctx.check_device_error()
        res["context_usable"] = True
        ctx.close()
    elif case == "sample":
        cfg = c1_config()
        w = random_weights(cfg, seed=0, std=0.02)
        ctx = shard_ctx(cfg, w, rank, nranks, 2, 256, 32)
        ctx.comm_init(uid, rank, nranks, timeout_ms=60000)
        win = 12 if rank == 0 else 8
        res["window"] = win
        for name, (T, top_p) in SAMPLE_MODES.items():
            ctx.set_sampling_seed(77 + rank)
            outs, steps = ctx.generate_streaming_batch(c1_prompts(rank), 24, win,
                                                       sample_params(T, top_p, *C1_PARAMS))
            res[name] = {"ids": [list(map(int, o)) for o in outs],
                         "steps": [int(x) for x in steps]}
        ctx.check_device_error()
        ctx.close()
    elif case == "sample_bf16":
        from wedlm_b200 import Context
        cfg = long_ctx_bf16_config()
        w = random_weights(cfg, seed=3, std=0.02)
        ctx = shard_ctx(cfg, w, rank, nranks, 1, 512, 32)
        ctx.comm_init(uid, rank, nranks, timeout_ms=60000)
        full = Context(to_model_config(cfg, max_block_tokens=32), max_seqs=1, max_ctx=512)
        full.load_weights(w)
        for name, (T, top_p) in SAMPLE_MODES.items():
            prm = sample_params(T, top_p, 0.8, 0.05, 8)
            ids = []
            for c in (ctx, full):
                c.set_sampling_seed(31 + rank)
                outs, _ = c.generate_streaming_batch(bf16_prompts(rank), 32, 16, prm)
                ids.append([list(map(int, o)) for o in outs])
            res[name] = {"ids": ids[0], "ids_whole_vocab": ids[1]}
        ctx.close()
        full.close()
    elif case == "mismatch":
        from wedlm_b200 import WedlmError
        cfg = c1_config()
        w = random_weights(cfg, seed=0, std=0.02)
        ctx = shard_ctx(cfg, w, rank, nranks, 1, 256, 32)
        ctx.comm_init(uid, rank, nranks, timeout_ms=30000)
        try:
            ctx.decode_begin([0], c1_prompts(1), 8, 8,
                             sample_params(0.7 * rank, 1.0, 0.8, 0.05, 8))
            res["code"] = 0
        except WedlmError as e:
            res["code"] = e.code
            res["message"] = str(e)
        outs, _ = ctx.generate_streaming_batch(c1_prompts(1), 8, 8, params(0.8, 0.05, 8))
        res["after"] = [list(map(int, o)) for o in outs]
        ctx.close()
    else:
        raise SystemExit(f"unknown case {case}")
    with open(out, "w") as f:
        json.dump(res, f)


if __name__ == "__main__":
    main()
