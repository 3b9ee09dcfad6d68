"""GPU parity of the weight-streaming GEMM (the VibeVoice head's projections when a call has at most 128 rows)
through the C ABI, against a torch fp32 reference of the same operands:

* 16-bit weights (fp16 / bf16) and Q8_0 weights expanded to fp16(q * d) inside the main loop; the Q8_0 case is
  compared with the fp16 rounding of dequantize_row_q8_0's values (tests/golden/q8_kat.b2db pins that
  dequantisation bit for bit in the GEMM tests);
* every epilogue (fp32, 16-bit, SwiGLU pairs, gated residual), row counts 1..128, the planned launch and
  explicit K splits of 2..8 CTAs per column tile (partial sums added on chip across the cluster, rows split
  unevenly among its CTAs) -- results must be identical across launches (fixed summation order).
Tolerance: rel-L2 1e-5 for fp32 outputs (fp32 accumulation of exactly representable products), 4e-3 for 16-bit
outputs (one fp16 / bf16 rounding)."""
import numpy as np
import pytest

from oracle import q8

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

F16, Q8_0, BF16 = 1, 8, 30


def _weights(n, k, wtype, g):
    w = torch.randn(n, k, generator=g) * 0.05
    if wtype == Q8_0:
        blocks = q8.quantize_q8_0(w.numpy().astype(np.float32))
        deq = torch.from_numpy(q8.dequantize_q8_0(blocks, k)).half().float()  # fp16(q * d)
        return torch.from_numpy(np.frombuffer(blocks.tobytes(), np.uint8).copy()).cuda(), deq.cuda()
    dt = torch.bfloat16 if wtype == BF16 else torch.float16
    wd = w.to(dt).cuda()
    return wd, wd.float()


def _rel(a, b):
    return float((a.float() - b).norm() / b.norm())


@pytest.mark.parametrize("wtype", [F16, Q8_0, BF16])
@pytest.mark.parametrize("m,n,k,bn,split", [(128, 1536, 4608, 0, 1), (37, 21504, 1536, 0, 1), (1, 256, 64, 0, 1),
                                            (128, 384, 1536, 128, 3), (100, 3584, 3584, 0, 1),
                                            (128, 1536, 4608, 64, 6), (64, 1536, 4608, 128, 8),
                                            (5, 768, 1024, 192, 2), (128, 512, 256, 256, 4)])
def test_stream_f32_and_residual(b2d, ctx, wtype, m, n, k, bn, split):
    g = torch.Generator().manual_seed(m * 7 + n + k)
    bf16 = wtype == BF16
    w, wref = _weights(n, k, wtype, g)
    dt = torch.bfloat16 if bf16 else torch.float16
    a = torch.randn(m, k, generator=g).to(dt).cuda()
    bias = torch.randn(n, generator=g).cuda()
    ref = a.float() @ wref.t() + bias
    out = torch.full((m, n), float("nan"), device="cuda")
    outs = []
    for _ in range(2):
        ctx.gemm_stream(a.data_ptr(), w.data_ptr(), m, n, k, w_type=wtype, bf16=bf16, epilogue=b2d.EPI_F32, bn=bn,
                        split=split, bias=bias.data_ptr(), out=out.data_ptr(), ldo=n)
        ctx.sync()
        outs.append(out.clone())
    assert _rel(outs[0], ref) < 1e-5
    assert torch.equal(outs[0], outs[1])
    # gated residual: x += gate * (acc + bias)
    x0 = torch.randn(m, n, generator=g).cuda()
    gate = torch.randn(m, n, generator=g).cuda()
    x = x0.clone()
    ctx.gemm_stream(a.data_ptr(), w.data_ptr(), m, n, k, w_type=wtype, bf16=bf16, epilogue=b2d.EPI_RESID, bn=bn,
                    split=split, bias=bias.data_ptr(), resid=x.data_ptr(), ldr=n, gate=gate.data_ptr(), ldg=n)
    ctx.sync()
    assert _rel(x - x0, gate * ref) < 1e-5


@pytest.mark.parametrize("wtype", [F16, Q8_0])
@pytest.mark.parametrize("m,f,h,split", [(128, 4608, 1536, 0), (9, 768, 256, 0), (64, 10752, 3584, 0),
                                         (128, 4608, 1536, 4)])
def test_stream_swiglu(b2d, ctx, wtype, m, f, h, split):
    """[gate | up] interleaved per 128 rows, as the head stores gate_proj / up_proj."""
    g = torch.Generator().manual_seed(f + m)
    w, wref = _weights(2 * f, h, wtype, g)
    a = torch.randn(m, h, generator=g).half().cuda()
    acc = a.float() @ wref.t()
    blocks = acc.view(m, 2 * f // 256, 2, 128)
    ref = (torch.nn.functional.silu(blocks[:, :, 0]) * blocks[:, :, 1]).reshape(m, f)
    out = torch.empty(m, f, dtype=torch.float16, device="cuda")
    ctx.gemm_stream(a.data_ptr(), w.data_ptr(), m, 2 * f, h, w_type=wtype, epilogue=b2d.EPI_SWIGLU,
                    bn=256 if split else 0, split=max(split, 1), out=out.data_ptr(), ldo=f)
    ctx.sync()
    assert _rel(out, ref) < 4e-3


def test_stream_ct_output(b2d, ctx):
    g = torch.Generator().manual_seed(5)
    w, wref = _weights(1024, 512, F16, g)
    a = torch.randn(77, 512, generator=g).half().cuda()
    out = torch.empty(77, 1024, dtype=torch.float16, device="cuda")
    ctx.gemm_stream(a.data_ptr(), w.data_ptr(), 77, 1024, 512, w_type=F16, epilogue=b2d.EPI_CT, bn=128, split=2,
                    out=out.data_ptr(), ldo=1024)
    ctx.sync()
    assert _rel(out, a.float() @ wref.t()) < 4e-3


def test_stream_rejects_bad_requests(b2d, ctx):
    a = torch.zeros(129, 64, dtype=torch.float16, device="cuda")
    w = torch.zeros(256, 64, dtype=torch.float16, device="cuda")
    out = torch.zeros(129, 256, device="cuda")
    with pytest.raises(b2d.B2DError):  # more than 128 rows
        ctx.gemm_stream(a.data_ptr(), w.data_ptr(), 129, 256, 64, w_type=F16, out=out.data_ptr(), ldo=256)
    with pytest.raises(b2d.B2DError):  # N not a multiple of the tile
        ctx.gemm_stream(a.data_ptr(), w.data_ptr(), 4, 200, 64, w_type=F16, bn=64, out=out.data_ptr(), ldo=256)
