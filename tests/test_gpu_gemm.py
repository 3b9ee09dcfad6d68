"""GPU parity of the kernel-level entry points against plain fp32 references:
the tcgen05 GEMM (all epilogues, ragged M) and the Q8_0 dequantiser (bit-exact)."""
import numpy as np
import pytest

from oracle import q8
from tests.helpers import golden

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _ref(a, b, bias=None):
    y = a.float() @ b.float().T
    return y + bias if bias is not None else y


SHAPES = [(1, 256, 64), (100, 256, 128), (128, 512, 1536), (300, 1536, 1536), (2048, 256, 4608)]


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_f32_epilogue(ctx, bf16, m, n, k):
    dt = torch.bfloat16 if bf16 else torch.float16
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n + k)
    a = torch.randn(m, k, device="cuda", generator=g).to(dt)
    b = (torch.randn(n, k, device="cuda", generator=g) * 0.05).to(dt)
    bias = torch.randn(n, device="cuda", generator=g)
    out = torch.full((m, n), float("nan"), device="cuda")
    ctx.gemm(a.data_ptr(), b.data_ptr(), m, n, k, bf16=bf16, epilogue=0, bn=256, bias=bias.data_ptr(),
             out=out.data_ptr(), ldo=n)
    torch.cuda.synchronize()
    ref = _ref(a, b, bias)
    err = (out - ref).norm() / ref.norm()
    assert err < 1e-5, float(err)


@pytest.mark.parametrize("bn", [64, 128, 256])
def test_gemm_tile_widths_and_ct_output(ctx, bn):
    m, n, k = 333, 768, 512
    a = torch.randn(m, k, device="cuda").half()
    b = (torch.randn(n, k, device="cuda") * 0.05).half()
    out = torch.zeros(m, n, device="cuda", dtype=torch.float16)
    ctx.gemm(a.data_ptr(), b.data_ptr(), m, n, k, epilogue=1, bn=bn, out=out.data_ptr(), ldo=n)
    torch.cuda.synchronize()
    ref = _ref(a, b)
    assert ((out.float() - ref).norm() / ref.norm()) < 2e-3


def test_gemm_swiglu_epilogue(ctx):
    m, f, k = 257, 512, 256
    a = torch.randn(m, k, device="cuda").half()
    w_act = (torch.randn(f, k, device="cuda") * 0.05).half()
    w_lin = (torch.randn(f, k, device="cuda") * 0.05).half()
    # interleave 128-row blocks: [act 0..127 | lin 0..127 | act 128..255 | ...]
    w = torch.cat([torch.cat([w_act[i:i + 128], w_lin[i:i + 128]]) for i in range(0, f, 128)])
    out = torch.zeros(m, f, device="cuda", dtype=torch.float16)
    ctx.gemm(a.data_ptr(), w.data_ptr(), m, 2 * f, k, epilogue=2, bn=256, out=out.data_ptr(), ldo=f)
    torch.cuda.synchronize()
    ref = torch.nn.functional.silu(_ref(a, w_act)) * _ref(a, w_lin)
    assert ((out.float() - ref).norm() / ref.norm()) < 3e-3


def test_gemm_gated_residual_epilogue(ctx):
    m, n, k = 190, 512, 1024
    a = torch.randn(m, k, device="cuda").half()
    b = (torch.randn(n, k, device="cuda") * 0.05).half()
    gate_full = torch.randn(m, 3 * n, device="cuda")
    x0 = torch.randn(m, n, device="cuda")
    x = x0.clone()
    gate = gate_full[:, n:2 * n]
    ctx.gemm(a.data_ptr(), b.data_ptr(), m, n, k, epilogue=3, bn=256, resid=x.data_ptr(), ldr=n,
             gate=gate.data_ptr(), ldg=3 * n)
    torch.cuda.synchronize()
    ref = x0 + gate * _ref(a, b)
    assert ((x - ref).norm() / ref.norm()) < 1e-5


def test_gemm_rejects_bad_k(ctx, b2d):
    a = torch.zeros(8, 96, device="cuda").half()
    with pytest.raises(b2d.B2DError):
        ctx.gemm(a.data_ptr(), a.data_ptr(), 8, 8, 96, out=a.data_ptr(), ldo=8)


def test_q8_0_dequant_bit_exact(ctx):
    g = golden("q8_kat")
    qb = torch.from_numpy(g["q8"].data.copy()).cuda()
    rows, k = g["x"].dims
    out = torch.zeros(rows, k, device="cuda")
    ctx.q8_0_dequantize(qb.data_ptr(), rows, k, out.data_ptr())
    torch.cuda.synchronize()
    ref = g["dequant"].array()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("m,n,k", [(2048, 512, 1536), (300, 1536, 1024), (129, 256, 64)])
def test_pair_gemm_all_epilogues(ctx, bf16, m, n, k):
    """The 2-SM (cta_group::2, 256 x 256 pair tile) kernel, selected with bn = 512."""
    dt = torch.bfloat16 if bf16 else torch.float16
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn(m, k, device="cuda", generator=g).to(dt)
    b = (torch.randn(n, k, device="cuda", generator=g) * 0.05).to(dt)
    bias = torch.randn(n, device="cuda", generator=g)
    ref = _ref(a, b, bias)
    out = torch.full((m, n), float("nan"), device="cuda")
    ctx.gemm(a.data_ptr(), b.data_ptr(), m, n, k, bf16=bf16, epilogue=0, bn=512, bias=bias.data_ptr(),
             out=out.data_ptr(), ldo=n)
    torch.cuda.synchronize()
    assert float((out - ref).norm() / ref.norm()) < 1e-5
    outc = torch.zeros(m, n, device="cuda", dtype=dt)
    ctx.gemm(a.data_ptr(), b.data_ptr(), m, n, k, bf16=bf16, epilogue=1, bn=512, bias=bias.data_ptr(),
             out=outc.data_ptr(), ldo=n)
    torch.cuda.synchronize()
    assert float((outc.float() - ref).norm() / ref.norm()) < (1e-2 if bf16 else 2e-3)
    x0 = torch.randn(m, n, device="cuda", generator=g)
    gate = torch.randn(m, n, device="cuda", generator=g)
    x = x0.clone()
    ctx.gemm(a.data_ptr(), b.data_ptr(), m, n, k, bf16=bf16, epilogue=3, bn=512, bias=bias.data_ptr(),
             resid=x.data_ptr(), ldr=n, gate=gate.data_ptr(), ldg=n)
    torch.cuda.synchronize()
    want = x0 + gate * ref
    assert float((x - want).norm() / want.norm()) < 1e-5
    x = x0.clone()  # no gate: x += acc + bias
    ctx.gemm(a.data_ptr(), b.data_ptr(), m, n, k, bf16=bf16, epilogue=3, bn=512, bias=bias.data_ptr(),
             resid=x.data_ptr(), ldr=n)
    torch.cuda.synchronize()
    want = x0 + ref
    assert float((x - want).norm() / want.norm()) < 1e-5
    f = n // 2
    sw = torch.zeros(m, f, device="cuda", dtype=dt)
    ctx.gemm(a.data_ptr(), b.data_ptr(), m, n, k, bf16=bf16, epilogue=2, bn=512, bias=bias.data_ptr(),
             out=sw.data_ptr(), ldo=f)
    torch.cuda.synchronize()
    idx_a = torch.cat([torch.arange(i, i + 128) for i in range(0, n, 256)]).cuda()
    want_sw = torch.nn.functional.silu(ref[:, idx_a]) * ref[:, idx_a + 128]
    assert float((sw.float() - want_sw).norm() / want_sw.norm()) < (1e-2 if bf16 else 3e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("m,n,k", [(2050, 1536, 1536), (300, 576, 1024), (129, 192, 64)])
def test_pair192_gemm_epilogues(ctx, bf16, m, n, k):
    """The 2-SM pair kernel with 256 x 192 tiles (96 B rows per CTA), selected with bn = 384."""
    dt = torch.bfloat16 if bf16 else torch.float16
    g = torch.Generator(device="cuda").manual_seed(m + n + k + 7)
    a = torch.randn(m, k, device="cuda", generator=g).to(dt)
    b = (torch.randn(n, k, device="cuda", generator=g) * 0.05).to(dt)
    bias = torch.randn(n, device="cuda", generator=g)
    ref = _ref(a, b, bias)
    out = torch.full((m, n), float("nan"), device="cuda")
    ctx.gemm(a.data_ptr(), b.data_ptr(), m, n, k, bf16=bf16, epilogue=0, bn=384, bias=bias.data_ptr(),
             out=out.data_ptr(), ldo=n)
    torch.cuda.synchronize()
    assert float((out - ref).norm() / ref.norm()) < 1e-5
    outc = torch.zeros(m, n, device="cuda", dtype=dt)
    ctx.gemm(a.data_ptr(), b.data_ptr(), m, n, k, bf16=bf16, epilogue=1, bn=384, bias=bias.data_ptr(),
             out=outc.data_ptr(), ldo=n)
    torch.cuda.synchronize()
    assert float((outc.float() - ref).norm() / ref.norm()) < (1e-2 if bf16 else 2e-3)
    x0 = torch.randn(m, n, device="cuda", generator=g)
    gate = torch.randn(m, n, device="cuda", generator=g)
    x = x0.clone()
    ctx.gemm(a.data_ptr(), b.data_ptr(), m, n, k, bf16=bf16, epilogue=3, bn=384, bias=bias.data_ptr(),
             resid=x.data_ptr(), ldr=n, gate=gate.data_ptr(), ldg=n)
    torch.cuda.synchronize()
    want = x0 + gate * ref
    assert float((x - want).norm() / want.norm()) < 1e-5
    x = x0.clone()  # no gate: x += acc + bias
    ctx.gemm(a.data_ptr(), b.data_ptr(), m, n, k, bf16=bf16, epilogue=3, bn=384, bias=bias.data_ptr(),
             resid=x.data_ptr(), ldr=n)
    torch.cuda.synchronize()
    want = x0 + ref
    assert float((x - want).norm() / want.norm()) < 1e-5
