"""The drop-in build on the GPU: audio.cpp's own harness and call sites (sample_vibevoice_speech_latents with a
VibeVoiceDiffusionHeadWeightsRuntime, VibeVoiceDiffusionHeadWeightsRuntime::predict, FoundationRfDitRuntime::
prepare / sample), compiled from the reference's unmodified headers and linked with audio.cpp_b200/dropin/ in
place of the reference's diffusion_head.cpp, diffusion_sampler.cpp and foundation/rf_dit.cpp
(oracle/_ref/b2d_ref_dropin, built by oracle/ref/Makefile's `dropin` target).  The reference's call sites must
then reproduce the reference's own CPU latents within the GPU parity tolerances, bit for bit what this
library's Python API returns for the same request, and honour the weight storage type (quantize-on-load)."""
import numpy as np
import pytest

from oracle import ref_runner, synth
from tests.helpers import golden, rel_l2, weight_specs

pytestmark = pytest.mark.gpu

EXE = ref_runner.dropin_binary()
needs_dropin = pytest.mark.skipif(EXE is None, reason="drop-in harness not built (make -C oracle/ref dropin)")


def _api_head(b2d, ctx, cfg, w):
    return b2d.VibeVoiceDiffusionHead(ctx, cfg.hidden, cfg.layers, cfg.ffn_ratio, weights=weight_specs(w))


@needs_dropin
@pytest.mark.parametrize("name", ["tiny_q8", "tiny_bf16", "small_q8_ragged", "vv15_q8_1024"])
def test_reference_sampler_call_site_runs_on_the_gpu(b2d, ctx, name):
    cfg = synth.HEAD_CONFIGS[name]
    w, inp = synth.head_weights(cfg), synth.head_inputs(cfg)
    out = ref_runner.run("vv", inp, w, threads=1, exe=EXE)["latents"].array()
    g = golden("head_" + name)
    ref, exact = g["latents"].array(), g["exact_latents"].array()
    err, spread = rel_l2(out, ref), rel_l2(exact, ref)
    print("%s through the reference's call site: vs ref %.3g (spread %.3g)" % (name, err, spread))
    assert err < max(1e-2, 1.5 * spread)
    mine = _api_head(b2d, ctx, cfg, w).sample(inp["positive_condition"].array(), inp["negative_condition"].array(),
                                              inp["initial_speech"].array(), cfg.steps, cfg.cfg)
    assert np.array_equal(out, mine)


@needs_dropin
@pytest.mark.parametrize("name", ["tiny_f16", "tiny_bf16"])
def test_storage_type_q8_0_quantizes_on_load(b2d, ctx, name):
    cfg = synth.HEAD_CONFIGS[name]
    w, inp = synth.head_weights(cfg), synth.head_inputs(cfg)
    inp["storage_type"] = synth.B.i64(b2d.STORAGE_Q8_0)
    out = ref_runner.run("vv", inp, w, threads=1, exe=EXE)["latents"].array()
    ref = golden("head_%s_as_q8" % name)["latents"].array()
    err = rel_l2(out, ref)
    print("%s stored as Q8_0: vs ref %.3g" % (name, err))
    assert err < 1e-2
    # the same conversion through the Python API gives the same bytes and so the same latents
    conv = [(n, *b2d.convert_tensor(t, d, p, b2d.STORAGE_Q8_0)) for n, t, d, p in weight_specs(w)]
    head = b2d.VibeVoiceDiffusionHead(ctx, cfg.hidden, cfg.layers, cfg.ffn_ratio,
                                      weights=[(n, t, d, p) for (n, t, p), (_, _, d, _) in
                                               zip(conv, weight_specs(w))])
    mine = head.sample(inp["positive_condition"].array(), inp["negative_condition"].array(),
                       inp["initial_speech"].array(), cfg.steps, cfg.cfg)
    assert np.array_equal(out, mine)


@needs_dropin
def test_reference_predict_call_site(b2d, ctx):
    cfg = synth.HEAD_CONFIGS["tiny_q8"]
    w = synth.head_weights(cfg)
    rng = np.random.default_rng(4)
    frames = 7
    inp = cfg.scalars()
    inp["noisy"] = synth.B.f32(rng.standard_normal((frames, 64)).astype(np.float32))
    inp["condition"] = synth.B.f32(rng.standard_normal((frames, cfg.hidden)).astype(np.float32))
    inp["timestep"] = synth.B.f32(np.float32(421.0))
    out = ref_runner.run("vvpredict", inp, w, threads=1, exe=EXE)["prediction"].array()
    ref = ref_runner.run("vvpredict", inp, w, threads=1)["prediction"].array() if ref_runner.available() else None
    mine = _api_head(b2d, ctx, cfg, w).predict(inp["noisy"].array(), 421.0, inp["condition"].array())
    assert np.array_equal(out, mine)
    if ref is not None:
        assert rel_l2(out, ref) < 1e-2


@needs_dropin
@pytest.mark.parametrize("name", ["tiny_bf16", "tiny_f16_3msde", "tiny_q8_b2_noapg"])
def test_reference_dit_call_site_runs_on_the_gpu(b2d, ctx, name):
    cfg = synth.DIT_CONFIGS[name]
    w, inp = synth.dit_weights(cfg), synth.dit_inputs(cfg)
    res = ref_runner.run("dit", inp, w, threads=1, exe=EXE)
    out = res["latents"].array()
    g = golden("dit_" + name)
    ref, exact = g["latents"].array(), g["exact_latents"].array()
    err, spread = rel_l2(out, ref), rel_l2(exact, ref)
    print("%s through the reference's call site: vs ref %.3g (spread %.3g)" % (name, err, spread))
    assert err < max(2e-2, 1.5 * spread)
    from oracle import philox
    draws = cfg.steps - 1 if cfg.sampler == "dpmpp-3m-sde" else 0
    n = cfg.batch * cfg.io_channels * cfg.latent_tokens
    assert int(res["rng_offset_out"].array()[0]) == draws * philox.offset_blocks(n, cfg.rng_sms, cfg.rng_max_threads)
