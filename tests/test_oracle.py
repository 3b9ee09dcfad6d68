"""CPU tests: the numpy oracle against the reference's golden vectors (tests/golden,
produced by the reference's own ggml CPU implementation via make_golden.py)."""
import numpy as np
import pytest

from oracle import bundle as B
from oracle import q8, synth
from oracle import vibevoice as V
from tests.golden.make_golden import digest
from tests.helpers import golden, rel_l2


def test_bundle_roundtrip(tmp_path):
    d = {"a": B.f32(np.arange(6, dtype=np.float32).reshape(2, 3)), "b": B.i64([1, 2, 3]),
         "c": B.Tensor(B.Q8_0, (1, 32), np.arange(34, dtype=np.uint8))}
    p = str(tmp_path / "x.b2db")
    B.write(p, d)
    r = B.read(p)
    assert r["a"].dims == (2, 3) and np.array_equal(r["a"].array(), d["a"].array())
    assert np.array_equal(r["b"].data, [1, 2, 3])
    assert r["c"].dtype == B.Q8_0 and np.array_equal(r["c"].data, d["c"].data)


def test_q8_0_bit_exact_vs_reference():
    g = golden("q8_kat")
    x = g["x"].array()
    mine = q8.quantize_q8_0(x)
    assert np.array_equal(mine.reshape(-1), g["q8"].data), "Q8_0 bytes differ from quantize_row_q8_0_ref"
    deq = q8.dequantize_q8_0(mine, x.shape[1])
    assert np.array_equal(deq.view(np.uint32), g["dequant"].array().view(np.uint32)), "dequant not bit-exact"


def test_q8_0_zero_block_and_ties():
    x = np.zeros((1, 64), np.float32)
    x[0, 32:] = np.linspace(-1, 1, 32)
    b = q8.quantize_q8_0(x).reshape(2, 34)
    assert b[0, 0] == 0 and b[0, 1] == 0 and not b[0, 2:].any()
    q, d = q8.split_q8_0(q8.quantize_q8_0(x), 64)
    assert q[0, 63] == 127 and q[0, 32] == -127


def test_bf16_rounding_matches_ggml():
    x = np.array([1.0, 1.00390625, 1.01171875, -3.5, np.float32(1e-40), np.inf, np.nan], np.float32)
    bits = q8.to_bf16_bits(x)
    assert bits[0] == 0x3F80 and bits[1] == 0x3F80  # tie to even
    assert bits[2] == 0x3F82
    assert bits[5] == 0x7F80 and (bits[6] & 0x40)


@pytest.mark.parametrize("steps", [1, 2, 3, 5, 10, 20, 50, 100])
def test_scheduler_port_vs_reference(steps):
    g = golden("sched_%d" % steps)
    s = V.Scheduler(1000)
    s.set_timesteps(steps)
    assert [float(t) for t in s.timesteps] == list(g["timesteps"].data)
    outs = g["model_outputs"].array()
    trace = s.run([outs[i] for i in range(steps)], g["sample"].array())
    ref = g["trace"].array()
    # The restatement rounds in its own order, so it drifts from the reference's fp32 arithmetic by a few 1e-8
    # of the state's scale per step: measured max |port - ref| / max |ref| per step 4.1e-7 (20 steps), 8.7e-7
    # (50), 1.7e-6 (100).  Bound: 5e-6 of the step's scale.
    for i in range(steps):
        err = float(np.max(np.abs(np.asarray(trace[i], np.float64) - ref[i])) / np.max(np.abs(ref[i])))
        assert err < 5e-6, "step %d: %.3g" % (i, err)


HEAD_TOL = {  # rel-L2 of the port vs the reference's ggml CPU run (fp32-accumulate build)
    "tiny_f16": 2e-4, "tiny_q8": 5e-5, "tiny_bf16": 1e-3, "small_q8_ragged": 5e-3,
    "one_frame_f16": 2e-4, "one_step_q8": 1e-5,
}


@pytest.mark.parametrize("name", sorted(HEAD_TOL))
def test_head_port_vs_reference(name):
    cfg = synth.HEAD_CONFIGS[name]
    w, inp = synth.head_weights(cfg), synth.head_inputs(cfg)
    g = golden("head_" + name)
    assert np.array_equal(digest(w, inp), g["input_sha256"].data), "synthetic generator drifted"
    head = V.Head(w, cfg)
    mine = V.sample_speech_latents(head, cfg, inp["positive_condition"].array(),
                                   inp["negative_condition"].array(), inp["initial_speech"].array())
    assert rel_l2(mine, g["latents"].array()) < HEAD_TOL[name]


# Known answers of generate_torch_cuda_randn (tests/unittests/test_torch_random.cpp:33-100 of audio.cpp).
KAT_F32_1234 = [-1.61649048, 0.56845516, -0.510224819, -0.911339402, -1.15551639, -0.22615087, -1.2891326, 1.065382,
                -0.7166605, -0.533334374, 0.207757875, -0.979843318, 0.744693458, -0.239484429, 0.27371496,
                0.092008315]
KAT_F32_1234_AT = {16: -0.803610802, 17: -1.6377064, 31: -0.300402969, 32: -0.251393795, 63: -0.924830973,
                   64: 0.799798131, 127: -0.167921364, 128: -0.322486848, 255: -1.76037288, 256: 0.534284174,
                   299: -0.986868858}
KAT_BF16_5678 = [-0.65625, -0.5625, 0.384765625, -0.151367188, 0.7421875, 0.244140625, 0.609375, 0.00321960449,
                 -0.46875, 0.306640625, -0.225585938, -0.9140625, 0.7734375, 0.120117188, 0.52734375, -0.5078125]
KAT_BF16_1234_AT = {16: -0.8046875, 17: -1.640625, 31: -0.30078125, 32: -0.251953125, 63: -0.92578125,
                    64: 0.80078125, 127: -0.16796875, 128: -0.322265625, 255: -1.7578125, 256: 0.53515625,
                    299: -0.98828125}


def test_philox_randn_known_answers():
    from oracle import philox
    np.testing.assert_allclose(philox.torch_cuda_randn(16, 1234), KAT_F32_1234, rtol=0, atol=2e-6)
    full = philox.torch_cuda_randn(300, 1234)
    for i, v in KAT_F32_1234_AT.items():
        assert abs(full[i] - v) <= 2e-6, i
    assert np.array_equal(philox.torch_cuda_randn(16, 5678, bf16=True), np.float32(KAT_BF16_5678))
    fb = philox.torch_cuda_randn(300, 1234, bf16=True)
    for i, v in KAT_BF16_1234_AT.items():
        assert fb[i] == np.float32(v), i
    # start index slices the full stream (test_start_index_matches_full_generation_slice)
    assert np.array_equal(philox.torch_cuda_randn(32, 1234, start=128), full[128:160])


def test_philox_tensor_iterator_layout():
    from oracle import philox
    # stride = 256 * min(blocks, SMs * threads / 256); each call advances ceil(n / (4 * stride))
    assert philox.iterator_stride(1000, 1, 256) == 256
    assert philox.offset_blocks(1000, 1, 256) == 1
    assert philox.offset_blocks(1025, 1, 256) == 2
    n = 64 * 3 * 1024
    st = philox.iterator_stride(n, 148, 2048)
    assert st == 256 * min((n + 255) // 256, 148 * 8)
    a = philox.tensor_iterator_randn(n, 5, 3, 148, 2048)
    # element seq < stride with loop 0, component 0 is Philox(counter=(offset, 0, seq, 0)).x through Box-Muller
    x, y, _, _ = philox.philox4x32_10(np.uint64(3), 0, np.arange(4, dtype=np.uint64), 0, 5)
    assert np.array_equal(a[:4], philox.box_muller(x, y)[0])


@pytest.mark.parametrize("name", ["sa3_tiny_f32", "sa3_tiny_f32_diff_b2", "sa3_tiny_f32_euler_nocfg",
                                  "sa3_tiny_bf16_diff", "sa3_mid_bf16_diff_b2", "sa3_mid_q8_euler"])
def test_sa3_port_vs_reference(name):
    """The Stable Audio 3 DiT restatement (oracle/sa3.py) against StableAudioRfDitRuntime::sample run by the
    reference's own CPU build: with fp32 weights the arithmetic is the same up to summation order (1e-5); with
    bf16 weights the reference requantises activations, and the fp32-activation restatement sits within
    max(2e-3, 1.5 x) of that spread as stored in the fixture."""
    from oracle import sa3, synth
    cfg = synth.SA3_CONFIGS[name]
    w, inp = synth.sa3_weights(cfg), synth.sa3_inputs(cfg)
    g = golden(name)
    assert np.array_equal(digest(w, inp), g["input_sha256"].data), "synthetic generator drifted"
    ref = g["latents"].array()
    mine = sa3.sample(sa3.Sa3Dit(w, cfg, act="ggml" if cfg.wtype != synth.F32 else "exact"), cfg, inp)
    err = float(np.linalg.norm(mine - ref) / np.linalg.norm(ref))
    if cfg.wtype == synth.F32:
        assert err < 1e-5, err
    else:
        spread = float(np.linalg.norm(g["exact_latents"].array() - ref) / np.linalg.norm(ref))
        assert err < max(2e-3, 1.5 * spread), (err, spread)
    # pingpong draws one TensorIterator Philox block per step; the reference's offset out-parameter agrees
    from oracle import philox
    draws = cfg.steps if cfg.sampler == "pingpong" else 0
    n = cfg.batch * cfg.io_channels * cfg.latent_tokens
    assert int(g["rng_offset_out"].data[0]) == draws * philox.offset_blocks(n, cfg.rng_sms, cfg.rng_max_threads)


@pytest.mark.parametrize("name", ["oobleck_tiny", "oobleck_tiny_b2_odd"])
def test_oobleck_port_vs_reference(name):
    """The Oobleck VAE decoder restatement (oracle/oobleck.py) against OobleckAutoencoderRuntime::decode run by the
    reference's own CPU build (fp32 weights: same arithmetic up to summation order)."""
    from oracle import oobleck, synth
    cfg = synth.OOBLECK_CONFIGS[name]
    w, inp = synth.oobleck_weights(cfg), synth.oobleck_inputs(cfg)
    g = golden(name)
    assert np.array_equal(digest(w, inp), g["input_sha256"].data), "synthetic generator drifted"
    ref = g["audio"].array()
    mine = oobleck.OobleckDecoder(w, cfg).decode(inp["latents"].array())
    assert mine.shape == ref.shape
    err = float(np.linalg.norm(mine - ref) / np.linalg.norm(ref))
    assert err < 1e-5, err


@pytest.mark.parametrize("name", ["vvdec_tiny", "vvdec_tiny_norm", "vvdec_tiny_c32"])
def test_vvdec_port_vs_reference(name):
    """The VibeVoice acoustic decoder restatement (oracle/vvdec.py) against
    VibeVoiceTokenizerWeightsRuntime::decode_acoustic run by the reference's own CPU build (fp32 weights)."""
    from oracle import synth, vvdec
    cfg = synth.VVDEC_CONFIGS[name]
    w, inp = synth.vvdec_weights(cfg), synth.vvdec_inputs(cfg)
    g = golden(name)
    assert np.array_equal(digest(w, inp), g["input_sha256"].data), "synthetic generator drifted"
    ref = g["samples"].array()
    mine = vvdec.AcousticDecoder(w, cfg).decode(inp["latents"].array())
    assert mine.shape == ref.shape
    err = float(np.linalg.norm(mine - ref) / np.linalg.norm(ref))
    assert err < 1e-5, err


@pytest.mark.parametrize("name", ["saocond_tiny", "saocond_tiny_b1_noneg"])
def test_saocond_port_vs_reference(name):
    """The SAO 1.0 conditioner restatement (oracle/saocond.py: T5-base encoder with relative position buckets and
    padding mask, number conditioners, cross / global assembly) against FoundationConditionerRuntime::encode run by
    the reference's own CPU build (fp32 weights)."""
    from oracle import saocond, synth
    cfg = synth.SAOCOND_CONFIGS[name]
    w, inp = synth.saocond_weights(cfg), synth.saocond_inputs(cfg)
    g = golden(name)
    assert np.array_equal(digest(w, inp), g["input_sha256"].data), "synthetic generator drifted"
    c = saocond.Conditioner(w, cfg)
    secs = inp["normalized_seconds"].array()
    cross, cmask, glob = c.encode_one(inp["input_ids"].array(), inp["attention_mask"].array(), secs)
    rel = lambda a, b: float(np.linalg.norm(a - b) / np.linalg.norm(b))  # noqa: E731
    assert rel(cross, g["cross_positive"].array()) < 1e-5
    assert rel(glob, g["global"].array()) < 1e-5
    assert np.array_equal(cmask, g["cross_mask"].array())
    if cfg.has_negative:
        neg, _, _ = c.encode_one(inp["negative_ids"].array(), inp["negative_mask"].array(), secs)
        assert rel(neg, g["cross_negative"].array()) < 1e-5
    # the bucket table's known values (T5's bidirectional scheme): 0 on the diagonal, 16 + d for small k > q
    b = saocond.relative_buckets(40)
    assert b[5, 5] == 0 and b[5, 6] == 17 and b[6, 5] == 1 and b.max() <= 31


@pytest.mark.parametrize("name", ["vvlm_tiny", "vvlm_tiny_mha_long"])
def test_vvlm_port_vs_reference(name):
    """The VibeVoice LM restatement (oracle/vvlm.py: Qwen2.5 layers with GQA, NEOX RoPE base 1e6, causal attention,
    SwiGLU MLP, tied lm_head) against VibeVoiceDecoderWeightsRuntime's prefill + cached steps run by the reference's
    own CPU build (fp32 weights): logits and last hidden of the prefill's last position and of every step."""
    from oracle import synth, vvlm
    cfg = synth.VVLM_CONFIGS[name]
    w, inp = synth.vvlm_weights(cfg), synth.vvlm_inputs(cfg)
    g = golden(name)
    assert np.array_equal(digest(w, inp), g["input_sha256"].data), "synthetic generator drifted"
    logits, hidden = vvlm.LanguageModel(w, cfg).run(inp["prefill_ids"].array(), inp["step_ids"].array())
    rel = lambda a, b: float(np.linalg.norm(a - b) / np.linalg.norm(b))  # noqa: E731
    assert rel(logits, g["logits"].array()) < 1e-5
    assert rel(hidden, g["last_hidden"].array()) < 1e-5
