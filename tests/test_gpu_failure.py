"""Failure detection on the GPU without a GPU fault: a kernel whose bounded wait can never succeed
(an mbarrier nothing arrives on) gives up after its poll limit, records the timeout code, and the
call returns B2D_ETIMEOUT; the same context then runs real work correctly."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(b2d, ctx):
    with pytest.raises(b2d.B2DError) as exc:
        ctx.selftest_wait_timeout(1 << 12)
    assert exc.value.status == -6 and "device-side wait expired" in str(exc.value)
    # the status word was cleared and the stream is healthy: a GEMM on the same context is exact
    a = torch.randn(256, 128, device="cuda").half()
    b = torch.randn(256, 128, device="cuda").half()
    out = torch.empty(256, 256, device="cuda")
    ctx.gemm(a.data_ptr(), b.data_ptr(), 256, 256, 128, epilogue=0, bn=256, out=out.data_ptr(), ldo=256)
    ctx.sync()
    ref = a.float() @ b.float().t()
    assert float((out - ref).norm() / ref.norm()) < 1e-5
    # and the self-test reports again (not a sticky error)
    with pytest.raises(b2d.B2DError):
        ctx.selftest_wait_timeout(1 << 12)
    ctx.sync()


def test_selftest_rejects_bad_limits(b2d, ctx):
    with pytest.raises(b2d.B2DError) as exc:
        ctx.selftest_wait_timeout(0)
    assert exc.value.status == -1
