"""Vocabulary-sharded LM head + entropy pass inside the streaming decode (NCCL between
ranks, one process per GPU), through wedlm_comm_init and the decode loops.

One GPU: a one-rank communicator runs the whole sharded step (gathers of one rank,
the LM head over the gathered rows, per-row partials, combine, and at T > 0 the phased
split-vocabulary sampler) and must give the same ids as the unsharded decode, greedy,
multinomial and nucleus; a context holding a vocabulary shard refuses to decode
without a communicator; a communicator whose second rank never joins fails its init
with WEDLM_ERR_TIMEOUT (a host-side failure: nothing runs on the GPU).
Two GPUs (skipped with fewer): the fp32 parity model decoded by two ranks holding the
two halves of the LM head gives the oracle's ids exactly, greedy and at T > 0
(multinomial and nucleus, seeded); the bf16 model gives the ids of a whole-vocabulary
context, greedy and at T > 0; ranks that ask for different temperatures are refused
together at decode_begin; a rank that leaves between steps makes the other rank's
next step end with an error (WEDLM_ERR_TIMEOUT, or WEDLM_ERR_IO when NCCL notices the
closed connection first).  NVLS is off in every multi-rank child.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle.decoder import OracleDecoder
from oracle.model import OracleModel, random_weights
from oracle.sampler import SamplingParams as OSP
from model_configs import c1_config, long_ctx_bf16_config, to_model_config
import sharded_rank

HERE = os.path.dirname(os.path.abspath(__file__))
ERR_INVALID_ARG, ERR_TIMEOUT, ERR_IO, ERR_STATE = -1, -4, -6, -7


def _params(tau, lam, cap):
    from wedlm_b200 import SamplingParams
    return SamplingParams(temperature=0.0, entropy_threshold=tau, distance_penalty=lam,
                          max_tokens_per_step=cap)


@pytest.mark.parametrize("mode", ["greedy", "multinomial", "nucleus"])
@pytest.mark.parametrize("which", ["c1", "bf16"])
def test_one_rank_communicator_matches_unsharded(which, mode):
    from wedlm_b200 import Context, comm_unique_id
    T, top_p = (0.0, 1.0) if mode == "greedy" else sharded_rank.SAMPLE_MODES[mode]
    if which == "c1":
        cfg, n, win, seed = c1_config(), 24, 12, 0
        prm = sharded_rank.sample_params(T, top_p, 9.0, 0.01, 3)
        prompts = np.random.default_rng(7).integers(1, 4095, size=(2, 16))
    else:
        cfg, n, win, seed = long_ctx_bf16_config(), 32, 16, 3
        prm = sharded_rank.sample_params(T, top_p, 0.8, 0.05, 8)
        prompts = np.random.default_rng(8).integers(0, 2046, size=(2, 40))
    w = random_weights(cfg, seed=seed, std=0.02)
    outs = []
    for comm in (False, True):
        ctx = Context(to_model_config(cfg, max_block_tokens=32), max_seqs=2, max_ctx=512)
        try:
            ctx.load_weights(w)
            ctx.set_sampling_seed(4321)
            if comm:
                ctx.comm_init(comm_unique_id(), 0, 1, timeout_ms=30000)
            outs.append(ctx.generate_streaming_batch(prompts, n, win, prm))
            ctx.check_device_error()
        finally:
            ctx.close()
    (a, sa), (b, sb) = outs
    assert [list(x) for x in a] == [list(x) for x in b]
    assert list(sa) == list(sb)


def test_vocab_shard_without_communicator_is_refused():
    from wedlm_b200 import Context, WedlmError
    cfg = c1_config()
    mc = to_model_config(cfg, max_block_tokens=32)
    mc.vocab_shard_begin, mc.vocab_shard_end = 0, cfg.vocab_size // 2
    ctx = Context(mc, max_seqs=1, max_ctx=128)
    try:
        ctx.load_weights(random_weights(cfg, seed=0, std=0.02))
        with pytest.raises(WedlmError) as e:
            ctx.generate_streaming([1, 2, 3], 4, 4, _params(0.8, 0.05, 8))
        assert e.value.code == ERR_STATE
        with pytest.raises(WedlmError) as e:
            ctx.generate_block([1, 2, 3], 4, _params(0.8, 0.05, 8))
        assert e.value.code == ERR_STATE
    finally:
        ctx.close()


_NEVER_JOINS = r"""
import sys, time
sys.path[:0] = {paths!r}
import torch
from wedlm_b200 import Context, WedlmError, comm_unique_id
from oracle.model import random_weights
from model_configs import c1_config, to_model_config
cfg = c1_config()
ctx = Context(to_model_config(cfg, max_block_tokens=32), max_seqs=1, max_ctx=128)
ctx.load_weights(random_weights(cfg, seed=0, std=0.02))
t0 = time.time()
try:
    ctx.comm_init(comm_unique_id(), 0, 2, timeout_ms=2000)
    print("RESULT ok")
except WedlmError as e:
    print("RESULT", e.code, round(time.time() - t0, 2))
ctx.generate_streaming([1, 2, 3], 4, 4, __import__("wedlm_b200").SamplingParams(
    temperature=0.0, entropy_threshold=0.8, distance_penalty=0.05, max_tokens_per_step=8))
print("USABLE")
ctx.close()
"""


def test_init_times_out_when_a_rank_never_joins():
    root = os.path.dirname(HERE)
    code = _NEVER_JOINS.format(paths=[root, os.path.join(root, "wedlm-rs_b200"), HERE])
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=180)
    lines = [l for l in r.stdout.splitlines() if l.startswith(("RESULT", "USABLE"))]
    assert r.returncode == 0, r.stderr[-2000:]
    res = lines[0].split()
    assert int(res[1]) == ERR_TIMEOUT and float(res[2]) < 30, lines
    assert lines[-1] == "USABLE"


def _two_gpus():
    return torch.cuda.device_count() >= 2


def _run_ranks(case, tmp_path, nranks=2, timeout=300):
    from wedlm_b200 import comm_unique_id
    uid = comm_unique_id().hex()
    procs, outs = [], []
    for r in range(nranks):
        out = str(tmp_path / f"{case}_{r}.json")
        env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(r), NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen([sys.executable, os.path.join(HERE, "sharded_rank.py"), case,
                                       str(r), str(nranks), uid, out], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
        outs.append(out)
    logs = []
    for p in procs:
        try:
            logs.append(p.communicate(timeout=timeout)[0])
        except subprocess.TimeoutExpired:
            p.kill()
            logs.append(p.communicate()[0])
    for p, log in zip(procs, logs):
        assert p.returncode == 0, log[-3000:]
    res = []
    for o in outs:
        with open(o) as f:
            res.append(json.load(f))
    return res


@pytest.mark.skipif(not _two_gpus(), reason="needs 2 GPUs")
def test_two_ranks_fp32_match_oracle(tmp_path):
    res = _run_ranks("c1", tmp_path)
    cfg = c1_config()
    om = OracleModel(cfg, random_weights(cfg, seed=0, std=0.02), "f32")
    dec = OracleDecoder(om, cfg.mask_token_id, cfg.eos_token_id)
    tau, lam, cap = sharded_rank.C1_PARAMS
    for r in res:
        prompts = sharded_rank.c1_prompts(r["rank"])
        assert len(r["ids"]) == len(prompts)
        for b, p in enumerate(prompts):
            ref, rst = dec.generate_streaming(p.tolist(), 24, r["window"],
                                              OSP(temperature=0.0, entropy_threshold=tau,
                                                  distance_penalty=lam, max_tokens_per_step=cap))
            assert r["ids"][b] == ref[len(p):], (r["rank"], b)
            assert r["steps"][b] == rst.steps


@pytest.mark.skipif(not _two_gpus(), reason="needs 2 GPUs")
def test_two_ranks_bf16_match_whole_vocabulary(tmp_path):
    for r in _run_ranks("bf16", tmp_path):
        assert r["ids"] == r["ids_whole_vocab"], r["rank"]


@pytest.mark.skipif(not _two_gpus(), reason="needs 2 GPUs")
def test_rank_leaving_between_steps_times_out(tmp_path):
    res = {r["rank"]: r for r in _run_ranks("leave", tmp_path)}
    assert res[1]["live_after_first_step"] > 0
    # the communicator timeout, or NCCL noticing the closed connection first
    assert res[0]["code"] in (ERR_TIMEOUT, ERR_IO), res[0]
    assert res[0]["seconds"] < 60 and res[0]["context_usable"]


@pytest.mark.skipif(not _two_gpus(), reason="needs 2 GPUs")
def test_two_ranks_fp32_sampling_match_oracle(tmp_path):
    """T > 0 over the split vocabulary: sequence b of rank r draws with rank r's seed and
    key b, as a one-sequence oracle decoder with that seed and seq_index b does."""
    res = _run_ranks("sample", tmp_path)
    cfg = c1_config()
    om = OracleModel(cfg, random_weights(cfg, seed=0, std=0.02), "f32")
    tau, lam, cap = sharded_rank.C1_PARAMS
    for r in res:
        prompts = sharded_rank.c1_prompts(r["rank"])
        for name, (T, top_p) in sharded_rank.SAMPLE_MODES.items():
            got = r[name]
            assert len(got["ids"]) == len(prompts)
            for b, p in enumerate(prompts):
                dec = OracleDecoder(om, cfg.mask_token_id, cfg.eos_token_id,
                                    seed=77 + r["rank"], seq_index=b)
                ref, rst = dec.generate_streaming(
                    p.tolist(), 24, r["window"],
                    OSP(temperature=T, top_p=top_p, entropy_threshold=tau,
                        distance_penalty=lam, max_tokens_per_step=cap))
                assert got["ids"][b] == ref[len(p):], (r["rank"], name, b)
                assert got["steps"][b] == rst.steps


@pytest.mark.skipif(not _two_gpus(), reason="needs 2 GPUs")
def test_two_ranks_bf16_sampling_match_whole_vocabulary(tmp_path):
    for r in _run_ranks("sample_bf16", tmp_path):
        for name in sharded_rank.SAMPLE_MODES:
            assert r[name]["ids"] == r[name]["ids_whole_vocab"], (r["rank"], name)


@pytest.mark.skipif(not _two_gpus(), reason="needs 2 GPUs")
def test_ranks_disagreeing_on_temperature_are_refused(tmp_path):
    res = _run_ranks("mismatch", tmp_path)
    for r in res:
        assert r["code"] == ERR_INVALID_ARG, r
        assert len(r["after"][0]) == 8
