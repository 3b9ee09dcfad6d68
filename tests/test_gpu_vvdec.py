"""GPU parity of the VibeVoice acoustic sigma-VAE decoder (VibeVoiceTokenizerWeightsRuntime::decode_acoustic)
through the C ABI: the causal stem / head convs, the transposed-conv upsamplers (right trim) and the FFN linears
run on the tensor cores (implicit-GEMM conv kernel, fp16 operands, fp32 accumulation and residual stream), with
GELU and the layer-scale residual fused into the epilogues; RMSNorm and the depthwise mixer are row kernels.
Compared with the reference's own CPU output (tests/golden/vvdec_*.b2db) and the numpy restatement
(oracle/vvdec.py); tolerance rel-L2 1e-2 (fp16 operand rounding; the reference computes in fp32)."""
import numpy as np
import pytest

from oracle import synth
from tests.helpers import golden, rel_l2, weight_specs

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _check(b2d, ctx, name):
    from oracle import vvdec
    cfg = synth.VVDEC_CONFIGS[name]
    w = synth.vvdec_weights(cfg)
    dec = b2d.VibeVoiceAcousticDecoder(ctx, cfg.vae_dim, cfg.n_filters, cfg.ratios, cfg.depths, cfg.disable_last_norm,
                                       cfg.eps, weights=weight_specs({k: v for k, v in w.items()
                                                                      if k.startswith("model.acoustic_tokenizer.decoder")}))
    lat = synth.vvdec_inputs(cfg)["latents"].array()
    out = dec.decode(lat)
    ref = golden(name)["samples"].array()
    exact = vvdec.AcousticDecoder(w, cfg).decode(lat)
    assert out.shape == ref.shape and np.isfinite(out).all()
    err, err_exact = rel_l2(out, ref), rel_l2(out, exact)
    print("%s: vs ref %.3g, vs restatement %.3g" % (name, err, err_exact))
    assert err < 1e-2 and err_exact < 1e-2
    d_lat = torch.from_numpy(lat).cuda()
    d_out = torch.empty(out.shape, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    dec.decode_device(d_lat, d_out, stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(d_out.cpu().numpy(), out)


@pytest.mark.parametrize("name", ["vvdec_tiny", "vvdec_tiny_norm"])
def test_vvdec_decode_matches_reference(b2d, ctx, name):
    _check(b2d, ctx, name)


# The 32-channel stage of the released decoders runs zero-padded to a 64-column tile (RMS means over the true
# channel count).
def test_vvdec_decode_32_channel_stage_matches_reference(b2d, ctx):
    _check(b2d, ctx, "vvdec_tiny_c32")
