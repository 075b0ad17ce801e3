"""The bounded device-side wait gives up, reports and leaves the context usable.

Every tcgen05 kernel (GEMM, attention) waits on mbarriers through one helper that gives
up after a time limit, records the wait site in the context's error word and lets the
kernel return.  wedlm_kernel_wait_probe waits with that helper on an mbarrier phase that
nothing completes (no arrival, no copy in flight) with a 1 ms limit.  The test checks the
wait ends near its limit, the host sees WEDLM_ERR_TIMEOUT with the site code, the error
word is cleared by the check, and the context still runs a kernel correctly afterwards.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ERR_TIMEOUT = -4


def test_bounded_wait_gives_up_and_reports():
    from wedlm_b200 import Context, WedlmError
    from oracle.sampler import row_stats
    with Context(None) as ctx:
        ctx.check_device_error()  # clean start
        for limit_us in (1000, 3000):
            out = ctx.wait_probe(limit_us * 1000)
            with pytest.raises(WedlmError) as ei:
                ctx.check_device_error()
            assert ei.value.code == ERR_TIMEOUT, ei.value
            assert "code 1" in str(ei.value)
            ok, waited_us = out.cpu().tolist()
            assert ok == 0
            assert limit_us <= waited_us < limit_us + 200_000, waited_us
            ctx.check_device_error()  # the check cleared the word
        # the context (and the GPU) still work: an entropy-select after the probe
        rng = np.random.default_rng(0)
        x = rng.standard_normal((4, 4096), dtype=np.float32)
        t = torch.from_numpy(x).cuda()
        r = ctx.entropy_select(t, 0.0, 0.8, 0.05,
                               torch.tensor([0, 4], dtype=torch.int32, device="cuda"),
                               torch.arange(4, dtype=torch.int32, device="cuda"),
                               torch.tensor([2], dtype=torch.int32, device="cuda"))
        torch.cuda.synchronize()
        H, am, _ = row_stats(x, 0.0)
        assert np.abs(r["H"].cpu().numpy() - H).max() < 1e-4
        assert (r["argmax"].cpu().numpy() == am).all()
        ctx.check_device_error()


def test_probe_rejects_bad_limits():
    from wedlm_b200 import Context, WedlmError
    with Context(None) as ctx:
        for bad in (0, -5, 3_000_000_000):
            with pytest.raises(WedlmError):
                ctx.wait_probe(bad)
