"""Parity of the fused entropy-select kernel (through the C ABI) with the oracle.

Tolerances: entropy 1e-3 absolute (bf16 logits; the parity bar), 2e-5 relative
for f32 logits; max-prob 1e-4 relative; argmax and the committed selection bit-exact.
The selection is checked twice: the oracle's rule applied to the kernel's own
entropies must reproduce the kernel's selection exactly, and the oracle's rule on
the oracle's entropies must agree wherever the decision margin exceeds 1e-3.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle.model import bf16_bits_to_f32, f32_to_bf16_bits
from oracle.sampler import row_stats, select_by_entropy_with_distance


@pytest.fixture(scope="module")
def ctx():
    from wedlm_b200 import Context
    c = Context(None)
    yield c
    c.close()


def c2_logits(rows, V, seed, sigma=2.5, spike=(8.0, 1.0)):
    """Config-2 style rows: N(0, sigma^2) plus one N(mu, s) spike at a seeded column."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, V), dtype=np.float32) * np.float32(sigma)
    cols = rng.integers(0, V, size=rows)
    x[np.arange(rows), cols] += rng.normal(spike[0], spike[1], size=rows).astype(np.float32)
    return x


def to_dev(x, dtype):
    if dtype == "bf16":
        b = f32_to_bf16_bits(x)
        t = torch.from_numpy(b.view(np.int16)).cuda().view(torch.bfloat16)
        return t, bf16_bits_to_f32(b)
    return torch.from_numpy(np.ascontiguousarray(x)).cuda(), x


def run(ctx, logits_t, T, tau, lam, seq_rows, mask_pos, caps):
    sr = torch.tensor(seq_rows, dtype=torch.int32, device="cuda")
    mp = torch.tensor(mask_pos, dtype=torch.int32, device="cuda")
    cp = torch.tensor(caps, dtype=torch.int32, device="cuda")
    out = ctx.entropy_select(logits_t, T, tau, lam, sr, mp, cp)
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in out.items()}


def check_against_oracle(out, xf, T, tau, lam, seq_rows, mask_pos, caps, h_atol):
    H, am, mp = row_stats(xf, T)
    assert np.abs(out["H"] - H).max() <= h_atol, np.abs(out["H"] - H).max()
    assert (out["argmax"] == am).all()
    assert np.allclose(out["maxprob"], mp, rtol=1e-4, atol=1e-9)
    for b in range(len(seq_rows) - 1):
        r0, r1 = seq_rows[b], seq_rows[b + 1]
        n = int(out["n_selected"][b])
        got = out["selected"][r0:r0 + n].tolist()
        mine = select_by_entropy_with_distance(out["H"][r0:r1].tolist(), mask_pos[r0:r1], tau, lam,
                                               caps[b])
        assert got == mine, (b, got, mine)
        ref = select_by_entropy_with_distance(H[r0:r1].tolist(), mask_pos[r0:r1], tau, lam, caps[b])
        if r1 > r0:
            lm = min(mask_pos[r0:r1])
            adj = H[r0:r1] + np.float32(lam) * (np.asarray(mask_pos[r0:r1]) - lm)
            margin = np.abs(adj - tau).min()
            srt = np.sort(adj)
            gap = srt[1] - srt[0] if len(srt) > 1 else 1.0
            if margin > h_atol and gap > 2 * h_atol:
                assert ref == got, (b, ref, got)


@pytest.mark.parametrize("rows", [96, 300])
def test_c2_bf16_full_vocab(ctx, rows):
    V = 151936
    x = c2_logits(rows, V, seed=rows)
    t, xf = to_dev(x, "bf16")
    seq_rows = [0, rows]
    mask_pos = list(range(rows))
    out = run(ctx, t, 0.0, 0.8, 0.05, seq_rows, mask_pos, [8])
    check_against_oracle(out, xf, 0.0, 0.8, 0.05, seq_rows, mask_pos, [8], 1e-3)
    # entropy far above tau on every row -> the fallback commits exactly one slot: the
    # first minimum of H + lambda * distance
    assert out["n_selected"][0] == 1


def test_threshold_and_cap_branches(ctx):
    V, rows = 4096, 24
    rng = np.random.default_rng(7)
    x = rng.standard_normal((rows, V), dtype=np.float32) * 0.5
    confident = [1, 2, 5, 7, 11, 13, 17, 20]
    for r in confident:
        x[r, rng.integers(0, V)] = 30.0
    t, xf = to_dev(x, "bf16")
    mask_pos = rng.permutation(40)[:rows].tolist()
    for cap in (0, 1, 3, 8, 30):
        out = run(ctx, t, 0.0, 0.8, 0.01, [0, rows], mask_pos, [cap])
        check_against_oracle(out, xf, 0.0, 0.8, 0.01, [0, rows], mask_pos, [cap], 1e-3)
        assert out["n_selected"][0] == max(min(cap, 8), 1)


def test_multiple_sequences_and_empty(ctx):
    V = 8192
    sizes = [5, 0, 17, 1, 96, 0, 33]
    seq_rows = np.concatenate([[0], np.cumsum(sizes)]).tolist()
    rows = seq_rows[-1]
    x = c2_logits(rows, V, seed=11, sigma=1.0, spike=(14.0, 1.0))
    t, xf = to_dev(x, "bf16")
    rng = np.random.default_rng(5)
    mask_pos = []
    for s in sizes:
        mask_pos += sorted(rng.permutation(128)[:s].tolist(), key=lambda _: rng.random())
    caps = [8, 8, 3, 1, 16, 4, 2]
    for rep in range(2):  # the self-resetting counters must work on a second launch
        out = run(ctx, t, 0.0, 2.0, 0.05, seq_rows, mask_pos, caps)
        check_against_oracle(out, xf, 0.0, 2.0, 0.05, seq_rows, mask_pos, caps, 1e-3)
    assert out["n_selected"][1] == 0 and out["n_selected"][5] == 0


def test_empty_row_set(ctx):
    """No rows: the selection counts are zeroed and the partials entry point is a no-op
    (the split plan must not divide by the row count)."""
    t = torch.empty(0, 151936, dtype=torch.bfloat16, device="cuda")
    sr = torch.tensor([0, 0, 0], dtype=torch.int32, device="cuda")
    mp = torch.empty(0, dtype=torch.int32, device="cuda")
    cp = torch.tensor([8, 8], dtype=torch.int32, device="cuda")
    out = ctx.entropy_select(t, 0.0, 0.8, 0.05, sr, mp, cp)
    parts = ctx.entropy_partials(t, 0, 0.0)
    torch.cuda.synchronize()
    assert out["n_selected"].tolist() == [0, 0] and parts.shape == (0, 4)


def test_ties_resolve_to_last_index(ctx):
    V = 5000
    x = np.zeros((3, V), np.float32)
    x[0, [3, 1000, 4999]] = 5.0
    x[1, :] = 1.0            # all equal -> last column
    x[2, [0, 7]] = 2.0
    t, xf = to_dev(x, "bf16")
    out = run(ctx, t, 0.0, 0.5, 0.0, [0, 3], [0, 1, 2], [2])
    assert out["argmax"].tolist() == [4999, V - 1, 7]
    assert abs(out["H"][1] - np.log(V)) < 1e-3


@pytest.mark.parametrize("T", [0.0, 1.0, 0.5, 1.7])
def test_f32_logits_temperature(ctx, T):
    V, rows = 4096, 16
    x = c2_logits(rows, V, seed=3, sigma=1.5, spike=(6.0, 1.0))
    t, xf = to_dev(x, "f32")
    out = run(ctx, t, T, 0.8, 0.05, [0, rows], list(range(rows)), [8])
    H, _, _ = row_stats(xf, T)
    assert np.allclose(out["H"], H, rtol=2e-5, atol=2e-5)
    check_against_oracle(out, xf, T, 0.8, 0.05, [0, rows], list(range(rows)), [8], 1e-4)


@pytest.mark.parametrize("V,ld", [(4099, 4099), (4099, 4104), (17, 17), (151936, 151944)])
def test_ragged_widths_and_strides(ctx, V, ld):
    rows = 7
    x = c2_logits(rows, ld, seed=V, sigma=2.0)
    x[:, V:] = 1e9  # padding columns beyond V must be ignored
    t, _ = to_dev(x, "bf16")
    tv = t[:, :V]
    xf = bf16_bits_to_f32(f32_to_bf16_bits(x[:, :V]))
    out = run(ctx, tv, 0.0, 0.8, 0.05, [0, rows], list(range(rows)), [8])
    check_against_oracle(out, xf, 0.0, 0.8, 0.05, [0, rows], list(range(rows)), [8], 1e-3)


def test_vocab_shard_partials_combine(ctx):
    V, rows, n = 151936, 96, 4
    x = c2_logits(rows, V, seed=21)
    t, xf = to_dev(x, "bf16")
    w = V // n
    parts = torch.stack([ctx.entropy_partials(t[:, r * w:(r + 1) * w], r * w, 0.0) for r in range(n)])
    sr = torch.tensor([0, 50, rows], dtype=torch.int32, device="cuda")
    mp = torch.tensor(list(range(50)) + list(range(46)), dtype=torch.int32, device="cuda")
    cp = torch.tensor([8, 8], dtype=torch.int32, device="cuda")
    comb = ctx.entropy_combine(parts, 0.8, 0.05, sr, mp, cp)
    full = ctx.entropy_select(t, 0.0, 0.8, 0.05, sr, mp, cp)
    torch.cuda.synchronize()
    assert torch.allclose(comb["H"], full["H"], atol=1e-5)
    assert torch.equal(comb["argmax"], full["argmax"])
    H, am, _ = row_stats(xf, 0.0)
    assert np.abs(comb["H"].cpu().numpy() - H).max() < 1e-3
    assert (comb["argmax"].cpu().numpy() == am).all()
    assert torch.equal(comb["n_selected"], full["n_selected"])
