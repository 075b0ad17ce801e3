"""Block attention on the tensor cores (wedlm_kernel_attention_prepare / _run) against a
plain PyTorch fp32 reference of the same op.

Reference: softmax(Q K^T / sqrt(128) + mask) V with GQA (src/model/attention.rs:188-221);
every cached key visible, window key j visible to window query i iff rank[j] <= rank[i].
The 8B attention shape (32 query / 8 KV heads, head_dim 128) with a 96-row window and
prefixes of 512, 2048 and 8192 cached tokens follows the block-attention workload
(N(0,1) inputs, ranks = a seeded permutation of the window positions, i.e. causal over
explicit positions); further cases cover the reference's index mask, ragged windows,
other GQA groups and an empty prefix.

Tolerance: the kernel rounds the probabilities to bf16 before the PV product and the
output to bf16, about 2^-9 relative each, so the bound is 1% of the largest reference
output plus 1e-3 on the maximum error, and 1% of the mean |reference| on the mean error.
"""
import math

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    from wedlm_b200 import Context
    c = Context(None)
    yield c
    c.close()


def inputs(L, S, nh, nkv, seed, rank_kind):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(S, nh, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(L + S, nkv, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(L + S, nkv, 128, generator=g).to(torch.bfloat16)
    if rank_kind == "positions":
        rank = (L + torch.randperm(S, generator=g)).to(torch.int32)
    else:
        rank = None
    return q.cuda(), k.cuda(), v.cuda(), (rank.cuda() if rank is not None else None)


def reference(q, k, v, L, rank):
    S, nh, d = q.shape
    group = nh // k.shape[1]
    qf, kf, vf = q.float(), k.float(), v.float()
    kf = kf.repeat_interleave(group, dim=1)
    vf = vf.repeat_interleave(group, dim=1)
    scores = torch.einsum("shd,thd->hst", qf, kf) / math.sqrt(d)
    r = rank.long() if rank is not None else torch.arange(S, device=q.device)
    vis = torch.ones(S, L + S, dtype=torch.bool, device=q.device)
    vis[:, L:] = r[None, :] <= r[:, None]
    scores = scores.masked_fill(~vis[None], float("-inf"))
    p = torch.softmax(scores, dim=-1)
    return torch.einsum("hst,thd->shd", p, vf).reshape(S, nh * d)


def check(out, ref):
    err = (out.float() - ref).abs()
    assert err.max().item() <= 1e-2 * ref.abs().max().item() + 1e-3, (err.max().item(),
                                                                     ref.abs().max().item())
    assert err.mean().item() <= 1e-2 * ref.abs().mean().item(), (err.mean().item(),
                                                                 ref.abs().mean().item())


@pytest.mark.parametrize("L", [512, 2048, 8192])
def test_block_attention_8b_shape_positions(ctx, L):
    q, k, v, rank = inputs(L, 96, 32, 8, seed=L, rank_kind="positions")
    ctx.attention_prepare(q, k, v, L, rank)
    out = ctx.attention_run()
    torch.cuda.synchronize()
    ctx.check_device_error()
    check(out, reference(q, k, v, L, rank))


@pytest.mark.parametrize("L,S,nh,nkv", [
    (0, 96, 32, 8),      # no prefix: window only, index-causal
    (100, 17, 32, 8),    # ragged window, prefix not a page multiple
    (700, 200, 32, 8),   # window of several query tiles
    (300, 96, 8, 8),     # no GQA sharing
    (1000, 40, 16, 2),   # group 8
])
def test_block_attention_index_mask(ctx, L, S, nh, nkv):
    q, k, v, rank = inputs(L, S, nh, nkv, seed=L + S, rank_kind="index")
    ctx.attention_prepare(q, k, v, L, None)
    out = ctx.attention_run()
    torch.cuda.synchronize()
    ctx.check_device_error()
    check(out, reference(q, k, v, L, None))


def test_block_attention_repeatable(ctx):
    q, k, v, rank = inputs(2048, 96, 32, 8, seed=5, rank_kind="positions")
    ctx.attention_prepare(q, k, v, 2048, rank)
    a = ctx.attention_run()
    b = ctx.attention_run()
    torch.cuda.synchronize()
    assert torch.equal(a, b)
