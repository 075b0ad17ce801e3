"""The projection GEMMs (tcgen05 bf16 path and f32 CUDA-core path) against a plain
PyTorch fp32 reference of the same op, through ``wedlm_kernel_gemm``.

Tolerance (bf16): |y - ref| <= 2^-7 |ref| + 2e-2 * rms(ref) per element (bf16 output
rounding plus f32-accumulation order); f32 path: 1e-4 relative to rms(ref).
"""
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    from wedlm_b200 import Context
    c = Context(None)
    yield c
    c.close()


def bf(x):
    return x.to(torch.bfloat16)


def rand(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(*shape, generator=g, device="cuda") * scale


def check_close(y, ref, rtol=2 ** -7):
    y, ref = y.float(), ref.float()
    rms = ref.pow(2).mean().sqrt().item()
    bad = (y - ref).abs() > (ref.abs() * rtol + 2e-2 * rms)
    assert not bad.any(), ((y - ref).abs().max().item(), rms, bad.sum().item())


SHAPES = [(96, 6144, 4096), (96, 4096, 4096), (96, 4096, 12288), (96, 151936, 4096),
          (1, 1000, 128), (17, 384, 64), (200, 1280, 512), (300, 640, 256), (768, 2048, 1024),
          (1000, 1280, 512), (1536, 4096, 4096),
          (6144, 4096, 1024), (6144, 6144, 512)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_store_bf16(ctx, M, N, K):
    X = bf(rand(M, K, seed=1))
    W = bf(rand(N, K, scale=K ** -0.5, seed=2))
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ctx.gemm(X, W, out, ctx.EPI_STORE)
    ctx.check_device_error()
    check_close(out, X.float() @ W.float().T)
    # packed weight tiles (1-D bulk-copy path) give the same result bit for bit
    outp = torch.empty_like(out)
    ctx.gemm(X, ctx.pack_weight(W), outp, ctx.EPI_STORE, N=N)
    ctx.check_device_error()
    assert torch.equal(out, outp)


@pytest.mark.parametrize("M,N,K", [(96, 151936, 4096), (33, 640, 256)])
def test_store_f32(ctx, M, N, K):
    X = bf(rand(M, K, seed=3))
    W = bf(rand(N, K, scale=K ** -0.5, seed=4))
    out = torch.empty(M, N, dtype=torch.float32, device="cuda")
    ctx.gemm(X, W, out, ctx.EPI_STORE_F32)
    ctx.check_device_error()
    ref = X.float() @ W.float().T
    assert (out - ref).abs().max().item() < 1e-3 * ref.abs().max().item()


@pytest.mark.parametrize("M,N,K", [(96, 4096, 4096), (96, 4096, 12288), (50, 256, 768),
                                   (1024, 4096, 4096), (6144, 4096, 512)])
def test_residual(ctx, M, N, K):
    X = bf(rand(M, K, seed=5))
    W = bf(rand(N, K, scale=K ** -0.5, seed=6))
    R = bf(rand(M, N, seed=7))
    out = R.clone()
    ctx.gemm(X, W, out, ctx.EPI_RESIDUAL, resid=out)  # in place, as the decode step does
    ctx.check_device_error()
    ref = R.float() + bf(X.float() @ W.float().T).float()
    check_close(out, ref)


@pytest.mark.parametrize("M,N,K", [(96, 12288, 4096), (20, 768, 256), (300, 512, 512),
                                   (640, 768, 256), (1024, 12288, 4096), (6144, 12288, 512)])
def test_swiglu(ctx, M, N, K):
    X = bf(rand(M, K, seed=8))
    Wg = bf(rand(N, K, scale=K ** -0.5, seed=9))
    Wu = bf(rand(N, K, scale=K ** -0.5, seed=10))
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ctx.gemm(X, Wg, out, ctx.EPI_SWIGLU, W2=Wu)
    ctx.check_device_error()
    outp = torch.empty_like(out)
    ctx.gemm(X, ctx.pack_weight(Wg), outp, ctx.EPI_SWIGLU, W2=ctx.pack_weight(Wu), N=N)
    assert torch.equal(out, outp)
    # unrounded f32 reference: the kernel rounds gate, up, silu and the product to bf16
    # as the reference does (three roundings of 2^-9 each), hence rtol 2^-6
    g = X.float() @ Wg.float().T
    u = X.float() @ Wu.float().T
    ref = g / (1 + torch.exp(-g)) * u
    check_close(out, ref, rtol=2 ** -6)


def test_repeat_calls_deterministic(ctx):
    X = bf(rand(96, 4096, seed=11))
    W = bf(rand(4096, 4096, scale=4096 ** -0.5, seed=12))
    a = torch.empty(96, 4096, dtype=torch.bfloat16, device="cuda")
    b = torch.empty_like(a)
    ctx.gemm(X, W, a)
    ctx.gemm(X, W, b)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("epi", [0, 2, 3])
def test_f32_path(ctx, epi):
    M, N, K = 16, 256, 256
    X, W, W2 = rand(M, K, seed=13), rand(N, K, scale=K ** -0.5, seed=14), rand(N, K, scale=K ** -0.5, seed=15)
    R = rand(M, N, seed=16)
    out = R.clone() if epi == 2 else torch.empty(M, N, device="cuda")
    ctx.gemm(X, W, out, epi, W2=W2 if epi == 3 else None, resid=out if epi == 2 else None)
    y = X @ W.T
    ref = {0: y, 2: R + y, 3: (y / (1 + torch.exp(-y))) * (X @ W2.T)}[epi]
    torch.cuda.synchronize()
    assert (out - ref).abs().max().item() < 1e-4 * ref.pow(2).mean().sqrt().item() + 1e-6
