"""The device-resident streaming loop against the host loop.

The decode session runs its per-step bookkeeping (wedlm.rs:380-573: loop head,
commit-before-predict, reordering, commit, drain with the EOS rule, refill, fill of the
picked slots, statistics) in two device kernels around the forward and the selection,
and replays the step as one CUDA graph.  WEDLM_DEVICE_LOOP=0 selects the host loop and
WEDLM_STEP_GRAPH=0 the device loop without the graph.  All three must give the same
committed ids, statistics, live counts per step, step counts and committed cache
lengths, bit for bit: greedy and seeded T > 0 (multinomial and nucleus), f32 and bf16,
several sequences ending at different steps (an EOS id the decode produces), a window
wider than max_new, max_new = 0, and decode_step over several steps at a time.  The f32
cases are also checked against the oracle decoder.
"""
import contextlib
import dataclasses
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle.decoder import OracleDecoder
from oracle.model import OracleModel, random_weights
from oracle.sampler import SamplingParams as OSP
from model_configs import c1_config, long_ctx_bf16_config, to_model_config

MODES = {"host": {"WEDLM_DEVICE_LOOP": "0"},
         "device": {"WEDLM_DEVICE_LOOP": "1", "WEDLM_STEP_GRAPH": "0"},
         "graph": {"WEDLM_DEVICE_LOOP": "1", "WEDLM_STEP_GRAPH": "1"}}
PARAMS = {"greedy_cap": (0.0, 1.0, 9.0, 0.01, 3), "greedy": (0.0, 1.0, 0.8, 0.05, 8),
          "multinomial": (0.8, 1.0, 0.8, 0.05, 8), "nucleus": (1.0, 0.7, 9.0, 0.01, 3)}


@contextlib.contextmanager
def env(kv):
    old = {k: os.environ.get(k) for k in kv}
    os.environ.update(kv)
    try:
        yield
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def sp(T, top_p, tau, lam, cap):
    from wedlm_b200 import SamplingParams
    return SamplingParams(temperature=T, top_p=top_p, entropy_threshold=tau,
                          distance_penalty=lam, max_tokens_per_step=cap)


def run(ctx, mode, prompts, max_new, window, prm, seed=11, chunk=1):
    """decode_begin / decode_step(chunk) until no sequence is live / results."""
    B = len(prompts)
    with env(MODES[mode]):
        ctx.set_sampling_seed(seed)
        l0 = ctx.launch_count()
        ctx.decode_begin(list(range(B)), prompts, max_new, window, prm)
        lives = []
        while True:
            live = ctx.decode_step(chunk)
            lives.append(live)
            if live == 0:
                break
        res = [ctx.decode_result(b) for b in range(B)]
        steps, _, _ = ctx.decode_io_bytes()
        ctx.decode_end()
        launches = ctx.launch_count() - l0
    lens = [ctx.cache_len(b) for b in range(B)]
    return {"res": res, "lives": lives, "steps": steps, "lens": lens, "launches": launches}


def c1_ctx(cfg, w, max_seqs=3):
    from wedlm_b200 import Context
    ctx = Context(to_model_config(cfg, max_block_tokens=32), max_seqs=max_seqs, max_ctx=256)
    ctx.load_weights(w)
    return ctx


@pytest.fixture(scope="module")
def c1_eos():
    """The f32 parity model with an EOS id that sequence 0 produces early, so that the
    three sequences of a batch end at different steps."""
    base = c1_config()
    w = random_weights(base, seed=0, std=0.02)
    prompts = np.random.default_rng(41).integers(1, 4095, size=(3, 16))
    free = dataclasses.replace(base, eos_token_id=4094)
    ctx = c1_ctx(free, w)
    try:
        with env(MODES["host"]):
            outs, _ = ctx.generate_streaming_batch(prompts, 24, 12, sp(*PARAMS["greedy_cap"]))
    finally:
        ctx.close()
    eos = int([t for t in outs[0] if t != free.mask_token_id][4])
    cfg = dataclasses.replace(base, eos_token_id=eos)
    ctx = c1_ctx(cfg, w)
    yield cfg, w, ctx, prompts
    ctx.close()


@pytest.mark.parametrize("pname", list(PARAMS))
def test_c1_device_loop_matches_host_loop_and_oracle(c1_eos, pname):
    cfg, w, ctx, prompts = c1_eos
    prm = sp(*PARAMS[pname])
    got = {m: run(ctx, m, prompts, 24, 12, prm) for m in MODES}
    for m in ("device", "graph"):
        for k in ("res", "lives", "steps", "lens"):
            assert got[m][k] == got["host"][k], (m, k)
    # the graph replays the eager step's launches
    assert got["graph"]["launches"] == got["device"]["launches"]
    # sequences end at different steps (EOS) in the greedy runs
    if pname.startswith("greedy"):
        assert any(r[0] and r[0][-1] == cfg.eos_token_id for r in got["host"]["res"])
    om = OracleModel(cfg, w, "f32")
    T, top_p, tau, lam, cap = PARAMS[pname]
    for b, p in enumerate(prompts):
        dec = OracleDecoder(om, cfg.mask_token_id, cfg.eos_token_id, seed=11, seq_index=b)
        ref, rst = dec.generate_streaming(p.tolist(), 24, 12,
                                          OSP(temperature=T, top_p=top_p, entropy_threshold=tau,
                                              distance_penalty=lam, max_tokens_per_step=cap))
        ids, st = got["graph"]["res"][b]
        assert ids == ref[len(p):], (pname, b)
        assert st["steps"] == rst.steps and st["tokens_generated"] == rst.tokens_generated


@pytest.mark.parametrize("max_new,window", [(5, 12), (0, 8), (1, 4)])
def test_c1_device_loop_edges(c1_eos, max_new, window):
    """A window wider than max_new, nothing to generate, one token."""
    cfg, w, ctx, prompts = c1_eos
    prm = sp(*PARAMS["greedy"])
    got = {m: run(ctx, m, prompts, max_new, window, prm) for m in MODES}
    for m in ("device", "graph"):
        for k in ("res", "lives", "steps", "lens"):
            assert got[m][k] == got["host"][k], (m, k, max_new, window)
    assert all(len(r[0]) <= max_new for r in got["graph"]["res"])


def test_c1_decode_step_chunks(c1_eos):
    """decode_step(n) with n > 1 (steps enqueued back to back, two in flight) ends in the
    same state as one step per call."""
    cfg, w, ctx, prompts = c1_eos
    prm = sp(*PARAMS["greedy_cap"])
    one = run(ctx, "graph", prompts, 24, 12, prm, chunk=1)
    for chunk in (3, 1 << 20):
        many = run(ctx, "graph", prompts, 24, 12, prm, chunk=chunk)
        assert many["res"] == one["res"] and many["steps"] == one["steps"]
        assert many["lens"] == one["lens"] and many["lives"][-1] == 0


@pytest.mark.parametrize("pname", ["greedy", "multinomial", "nucleus"])
def test_bf16_device_loop_matches_host_loop(pname):
    from wedlm_b200 import Context
    cfg = long_ctx_bf16_config()
    ctx = Context(to_model_config(cfg, max_block_tokens=32), max_seqs=2, max_ctx=512)
    try:
        ctx.load_weights(random_weights(cfg, seed=3, std=0.02))
        prompts = np.random.default_rng(42).integers(0, 2046, size=(2, 40))
        prm = sp(*PARAMS[pname])
        got = {m: run(ctx, m, prompts, 32, 16, prm) for m in MODES}
        ctx.check_device_error()
    finally:
        ctx.close()
    for m in ("device", "graph"):
        for k in ("res", "lives", "steps", "lens"):
            assert got[m][k] == got["host"][k], (m, k)
