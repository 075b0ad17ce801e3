"""The allocation-free entropy-select entry point against the allocating one.

wedlm_entropy_select_noalloc runs the same kernels as wedlm_entropy_select with its
scratch in a static device array.  Two calls in a row (the second reusing the
scratch the first left behind) must reproduce the allocating entry point: argmax,
selection and counts exactly, entropy and max-prob within 1e-6 absolute.  Calls
beyond the static limits must fail with WEDLM_ERR_INVALID_ARG before launching.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ERR_INVALID_ARG = -1


@pytest.fixture(scope="module")
def ctx():
    from wedlm_b200 import Context
    c = Context(None)
    yield c
    c.close()


def case(rows_per_seq, V, dtype, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    rows = sum(rows_per_seq)
    x = torch.randn(rows, V, generator=g) * 2.5
    x[torch.arange(rows), torch.randint(0, V, (rows,), generator=g)] += 8.0
    logits = x.to(dtype).cuda()
    seq_rows = np.concatenate([[0], np.cumsum(rows_per_seq)]).astype(np.int32)
    mask_pos = np.concatenate([np.sort(np.random.default_rng(seed + b).choice(
        4 * n + 1, size=n, replace=False)) for b, n in enumerate(rows_per_seq)]).astype(np.int32)
    caps = np.array([max(1, n // 3) for n in rows_per_seq], dtype=np.int32)
    dev = lambda a: torch.from_numpy(a).cuda()
    return logits, dev(seq_rows), dev(mask_pos), dev(caps)


def outputs(rows, nseq):
    return {"H": torch.empty(rows, dtype=torch.float32, device="cuda"),
            "argmax": torch.empty(rows, dtype=torch.int32, device="cuda"),
            "maxprob": torch.empty(rows, dtype=torch.float32, device="cuda"),
            "selected": torch.empty(max(rows, 1), dtype=torch.int32, device="cuda"),
            "n_selected": torch.empty(nseq, dtype=torch.int32, device="cuda")}


def compare(a, b, seq_rows):
    assert torch.equal(a["argmax"], b["argmax"])
    assert torch.equal(a["n_selected"], b["n_selected"])
    torch.testing.assert_close(a["H"], b["H"], rtol=0, atol=1e-6)
    torch.testing.assert_close(a["maxprob"], b["maxprob"], rtol=0, atol=1e-6)
    sr = seq_rows.cpu().numpy()
    for s in range(len(sr) - 1):
        n = int(a["n_selected"][s])
        assert torch.equal(a["selected"][sr[s]:sr[s] + n], b["selected"][sr[s]:sr[s] + n])


@pytest.mark.parametrize("rows_per_seq,V,dtype,T,tau,lam", [
    ([32, 32, 32], 151936, torch.bfloat16, 0.0, 0.8, 0.05),
    ([7, 1, 0, 90], 32000, torch.float32, 0.7, 2.0, 0.02),
    ([600, 700], 4096, torch.bfloat16, 1.3, 7.5, 0.0),
])
def test_two_calls_match_allocating_entry(ctx, rows_per_seq, V, dtype, T, tau, lam):
    cases = [case(rows_per_seq, V, dtype, seed) for seed in (1, 2)]
    rows, nseq = sum(rows_per_seq), len(rows_per_seq)
    for logits, sr, mp, cp in cases:  # back to back, no synchronisation in between
        got = ctx.entropy_select_noalloc(logits, T, tau, lam, sr, mp, cp, outputs(rows, nseq))
        want = ctx.entropy_select(logits, T, tau, lam, sr, mp, cp)
        torch.cuda.synchronize()
        compare(got, want, sr)


def test_no_device_memory_taken_per_call(ctx):
    logits, sr, mp, cp = case([48, 48], 151936, torch.bfloat16, 3)
    outs = [outputs(96, 2) for _ in range(3)]
    ctx.entropy_select_noalloc(logits, 0.0, 0.8, 0.05, sr, mp, cp, outs[0])
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    ctx.entropy_select_noalloc(logits, 0.0, 0.8, 0.05, sr, mp, cp, outs[1])
    ctx.entropy_select_noalloc(logits, 0.0, 0.8, 0.05, sr, mp, cp, outs[2])
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    compare(outs[1], outs[0], sr)
    compare(outs[2], outs[0], sr)


def test_empty_row_set(ctx):
    """No mask rows at all: both entry points report zero selections per sequence (the
    plan must not divide by the row count) and the static scratch stays usable."""
    logits, sr, mp, cp = case([0, 0], 151936, torch.bfloat16, 5)
    got = outputs(0, 2)
    got["n_selected"].fill_(7)
    ctx.entropy_select_noalloc(logits, 0.0, 0.8, 0.05, sr, mp, cp, got)
    want = ctx.entropy_select(logits, 0.0, 0.8, 0.05, sr, mp, cp)
    torch.cuda.synchronize()
    assert got["n_selected"].tolist() == [0, 0] and want["n_selected"].tolist() == [0, 0]
    logits, sr, mp, cp = case([40, 56], 151936, torch.bfloat16, 6)
    after = ctx.entropy_select_noalloc(logits, 0.0, 0.8, 0.05, sr, mp, cp, outputs(96, 2))
    compare(after, ctx.entropy_select(logits, 0.0, 0.8, 0.05, sr, mp, cp), sr)


@pytest.mark.parametrize("rows_per_seq,V", [
    ([4097], 16),          # rows above 4096
    ([1] * 1025, 16),      # nseq above 1024
])
def test_rejects_sizes_beyond_static_scratch(ctx, rows_per_seq, V):
    from wedlm_b200._lib import WedlmError
    logits, sr, mp, cp = case(rows_per_seq, V, torch.bfloat16, 4)
    out = outputs(sum(rows_per_seq), len(rows_per_seq))
    with pytest.raises(WedlmError) as ei:
        ctx.entropy_select_noalloc(logits, 0.0, 0.8, 0.05, sr, mp, cp, out)
    assert ei.value.code == ERR_INVALID_ARG
    assert "static entropy scratch" in str(ei.value)
