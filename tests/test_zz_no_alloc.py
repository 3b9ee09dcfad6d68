"""GPU test of b2d_gemm_splitk_noalloc, the entry point for callers that cannot
allocate device memory (hosts that pass only buffers from their own pool, or
that forbid cudaMalloc while serving).  It keeps its split-K partials in a fixed
device array inside the library, so the call allocates nothing.

Checked through the C ABI against b2d_gemm (the existing fp32-epilogue GEMM)
with the GEMM tests' tolerance (rel-L2 1e-5), on two calls in a row, plus the
rejection of sizes beyond the fixed array.  This file is named to be collected
last; it passes alone in a fresh process and after the other tests.
"""
import ctypes as C

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-5


def _noalloc(b2d, a, b, m, n, k, splits, bn, bias, out, bf16=False):
    err = C.create_string_buffer(256)
    st = b2d.lib().b2d_gemm_splitk_noalloc(int(bf16), C.c_void_p(a.data_ptr()), C.c_void_p(b.data_ptr()), m, n, k,
                                           splits, bn, C.c_void_p(bias.data_ptr() if bias is not None else None),
                                           C.c_void_p(out.data_ptr()), n,
                                           C.c_void_p(torch.cuda.current_stream().cuda_stream), err, 256)
    return st, err.value.decode()


@pytest.mark.parametrize("bf16", [False, True])
def test_noalloc_matches_gemm_twice(b2d, ctx, bf16):
    dt = torch.bfloat16 if bf16 else torch.float16
    g = torch.Generator(device="cuda").manual_seed(17)
    shapes = [(2048, 64, 1536, 8, 64), (300, 512, 1024, 4, 256)]  # the head's final projection, then a ragged one
    for m, n, k, splits, bn in shapes:
        a = torch.randn(m, k, device="cuda", generator=g).to(dt)
        b = (torch.randn(n, k, device="cuda", generator=g) * 0.05).to(dt)
        bias = torch.randn(n, device="cuda", generator=g)
        ref = torch.empty(m, n, device="cuda")
        ctx.gemm(a.data_ptr(), b.data_ptr(), m, n, k, bf16=bf16, epilogue=b2d.EPI_F32, bn=bn,
                 bias=bias.data_ptr(), out=ref.data_ptr(), ldo=n,
                 stream=torch.cuda.current_stream().cuda_stream)
        for _ in range(2):  # the shared array keeps the previous call's contents; results must not depend on it
            out = torch.full((m, n), float("nan"), device="cuda")
            st, msg = _noalloc(b2d, a, b, m, n, k, splits, bn, bias, out, bf16)
            assert st == 0, msg
            torch.cuda.synchronize()
            err = float((out - ref).norm() / ref.norm())
            assert err < TOL, err


def test_noalloc_rejects_oversize(b2d, ctx):
    m, n, k = 4096, 4096, 1024
    a = torch.zeros(m, k, device="cuda", dtype=torch.float16)
    b = torch.zeros(n, k, device="cuda", dtype=torch.float16)
    out = torch.zeros(m, n, device="cuda")
    st, msg = _noalloc(b2d, a, b, m, n, k, 2, 256, None, out)  # 2 * 4096 * 4096 floats > 8 Mi floats
    assert st == -1 and "exceeds the fixed scratch" in msg


def test_noalloc_reports_an_expired_wait(b2d, ctx):
    """A bounded device-side wait that expires is reported by b2d_gemm_splitk_noalloc_status (B2D_ETIMEOUT, then
    cleared), not swallowed; the test drives the library's own bounded wait to its limit, with no GPU fault."""
    L = b2d.lib()
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    err = C.create_string_buffer(256)
    assert L.b2d_gemm_splitk_noalloc_status(s, err, 256) == 0, err.value
    assert L.b2d_gemm_splitk_noalloc_selftest_timeout(1 << 12, s, err, 256) == 0, err.value
    assert L.b2d_gemm_splitk_noalloc_status(s, err, 256) == -6
    assert b"device-side wait expired" in err.value
    assert L.b2d_gemm_splitk_noalloc_status(s, err, 256) == 0  # cleared after it was reported
    # the next call on the shared array is exact again
    m, n, k = 256, 256, 512
    a = torch.randn(m, k, device="cuda").half()
    b = torch.randn(n, k, device="cuda").half()
    out = torch.empty(m, n, device="cuda")
    st, msg = _noalloc(b2d, a, b, m, n, k, 2, 256, None, out)
    assert st == 0, msg
    assert L.b2d_gemm_splitk_noalloc_status(s, err, 256) == 0
    ref = a.float() @ b.float().t()
    assert float((out - ref).norm() / ref.norm()) < TOL
