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


@pytest.mark.parametrize("steps", [1, 2, 10, 20])
def test_scheduler_port_vs_reference(steps):
    g = golden("sched_%d" % steps)
    s = V.Scheduler(1000)
    s.set_timesteps(steps)
    assert [float(t) for t in s.timesteps] == list(g["timesteps"].data)
    outs = g["model_outputs"].array()
    trace = s.run([outs[i] for i in range(steps)], g["sample"].array())
    ref = g["trace"].array()
    for i in range(steps):
        np.testing.assert_allclose(trace[i], ref[i], rtol=2e-6, atol=2e-6)


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
