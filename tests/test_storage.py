"""Weight storage-type selection and quantize-on-load (host code of the C ABI, no GPU):
b2d_storage_resolve follows the reference weight store's rules (backend_weight_store.h:237-290) and
b2d_tensor_convert produces the reference's bytes (tensor_source.cpp:150-200): Q8_0 against the bytes the
reference's own ggml_quantize_chunk wrote into tests/golden/q8_kat.b2db, F16 against IEEE round-to-nearest-even
(numpy), BF16 against the oracle's restatement of ggml's rounding."""
import numpy as np
import pytest

from oracle import q8
from tests.helpers import golden

F32, F16, Q8_0, BF16 = 0, 1, 8, 30


def _conv(b2d, gtype, dims, payload, storage):
    return b2d.convert_tensor(gtype, dims, payload, storage)


def test_resolve_rules(b2d):
    w = np.zeros((64, 96), np.float16)
    assert _conv(b2d, F16, (64, 96), w, b2d.STORAGE_NATIVE)[0] == F16
    assert _conv(b2d, F16, (64, 96), w, b2d.STORAGE_Q8_0)[0] == Q8_0
    assert _conv(b2d, F16, (64, 96), w, b2d.STORAGE_BF16)[0] == BF16
    # quantized targets fall back to F32 for 1-D tensors and rows that are not whole 32-blocks
    assert _conv(b2d, F16, (96,), np.zeros(96, np.float16), b2d.STORAGE_Q8_0)[0] == F32
    assert _conv(b2d, F16, (4, 48), np.zeros((4, 48), np.float16), b2d.STORAGE_Q8_0)[0] == F32
    with pytest.raises(b2d.B2DError):  # Q4_K and the like are not on this path
        _conv(b2d, F16, (64, 96), w, 10)


def test_q8_0_matches_reference_bytes(b2d):
    g = golden("q8_kat")
    x = g["x"].array().astype(np.float32)
    t, out = _conv(b2d, F32, x.shape, x, b2d.STORAGE_Q8_0)
    assert t == Q8_0
    ref = np.frombuffer(g["q8"].data.tobytes(), np.uint8)
    assert np.array_equal(out, ref)


def test_q8_0_matches_restatement_from_16_bit_sources(b2d):
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((40, 256)) * 0.05).astype(np.float32)
    w[3, :32] = 0.0
    w16 = w.astype(np.float16)
    _, out = _conv(b2d, F16, w16.shape, w16, b2d.STORAGE_Q8_0)
    assert np.array_equal(out, q8.quantize_q8_0(w16.astype(np.float32)).reshape(-1))
    bf = q8.to_bf16_bits(w)
    _, out = _conv(b2d, BF16, w.shape, bf, b2d.STORAGE_Q8_0)
    assert np.array_equal(out, q8.quantize_q8_0(q8.from_bf16_bits(bf).reshape(w.shape)).reshape(-1))


def test_f16_round_to_nearest_even(b2d):
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.standard_normal(4096).astype(np.float32) * s for s in (1e-6, 1e-3, 1.0, 1e3, 7e4)])
    edge = np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e9, -1e9, np.inf, -np.inf, 2.0 ** -24, 2.0 ** -25,
                     1.5 * 2.0 ** -25, 2.0 ** -14, 2.0 ** -14 * (1 - 2 ** -11), 1.0 + 2.0 ** -11,
                     1.0 + 3 * 2.0 ** -11], np.float32)
    x = np.concatenate([x, edge]).reshape(1, -1)
    _, out = _conv(b2d, F32, x.shape, x, b2d.STORAGE_F16)
    with np.errstate(over="ignore"):  # the large inputs overflow to infinity, as they must
        ref = x.astype(np.float16)
    assert np.array_equal(out.view(np.uint16), ref.view(np.uint16).reshape(-1))
    nan = np.array([[np.nan, 1.0]], np.float32)
    _, out = _conv(b2d, F32, nan.shape, nan, b2d.STORAGE_F16)
    assert np.isnan(out.view(np.float16)[0]) and out.view(np.float16)[1] == 1.0


def test_bf16_rounding_and_round_trips(b2d):
    rng = np.random.default_rng(6)
    x = (rng.standard_normal((16, 64)) * 3).astype(np.float32)
    _, out = _conv(b2d, F32, x.shape, x, b2d.STORAGE_BF16)
    assert np.array_equal(out.view(np.uint16), q8.to_bf16_bits(x).reshape(-1))
    # Q8_0 -> F16 decodes q * d then rounds once; Q8_0 -> Q8_0 keeps the bytes
    blocks = q8.quantize_q8_0(x)
    _, out = _conv(b2d, Q8_0, x.shape, blocks, b2d.STORAGE_F16)
    assert np.array_equal(out.view(np.float16), q8.dequantize_q8_0(blocks, 64).astype(np.float16).reshape(-1))
    _, out = _conv(b2d, Q8_0, x.shape, blocks, b2d.STORAGE_NATIVE)
    assert np.array_equal(out, blocks.reshape(-1))
