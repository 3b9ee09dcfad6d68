"""GPU parity of the Stable Audio Oobleck VAE decoder (OobleckAutoencoderRuntime::decode) through the C ABI:
every conv of the decoder (in-conv, transposed-conv upsampling with its crop, dilated residual units, out-conv)
runs as an implicit GEMM on the tensor cores with fp16 operands and fp32 accumulation, and the snake activations
and residual adds are fused into the GEMM epilogues.  Compared with the reference's own CPU output
(tests/golden/oobleck_*.b2db) and the numpy restatement (oracle/oobleck.py); tolerance rel-L2 1e-2 (fp16 operand
rounding through 12-17 convs; the reference computes in fp32)."""
import numpy as np
import pytest

from oracle import synth
from tests.helpers import golden, rel_l2, weight_specs

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def make(b2d, ctx, cfg):
    return b2d.OobleckDecoder(ctx, cfg.latent_dim, cfg.channels, cfg.c_mults, cfg.strides, cfg.audio_channels,
                              weights=weight_specs(synth.oobleck_weights(cfg)))


@pytest.mark.parametrize("name", ["oobleck_tiny", "oobleck_tiny_b2_odd", "oobleck_sao_shape_1x16"])
def test_oobleck_decode_matches_reference(b2d, ctx, name):
    from oracle import oobleck
    cfg = synth.OOBLECK_CONFIGS[name]
    dec = make(b2d, ctx, cfg)
    lat = synth.oobleck_inputs(cfg)["latents"].array()
    out = dec.decode(lat)
    ref = golden(name)["audio"].array()
    exact = oobleck.OobleckDecoder(synth.oobleck_weights(cfg), cfg).decode(lat)
    assert out.shape == ref.shape and np.isfinite(out).all()
    err, err_exact = rel_l2(out, ref), rel_l2(out, exact)
    print("%s: vs ref %.3g, vs restatement %.3g" % (name, err, err_exact))
    assert err < 1e-2 and err_exact < 1e-2
    assert np.array_equal(out, dec.decode(lat))
    # device API on the same inputs
    d_lat = torch.from_numpy(lat).cuda()
    d_out = torch.empty(out.shape, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    dec.decode_device(d_lat, d_out, stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(d_out.cpu().numpy(), out)
