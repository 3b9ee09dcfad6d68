"""GPU parity of the Stable Audio Open 1.0 conditioner (FoundationConditionerRuntime::encode_one) through the C ABI:
T5-base on the tensor-core GEMMs (fp16 operands, fp32 accumulation and residual stream), T5 attention with the
bucketed relative-position bias and padding mask, the seconds number embeddings and the cross / global assembly on
the device.  Compared with the reference's own CPU output (tests/golden/saocond_*.b2db) and the numpy restatement
(oracle/saocond.py); tolerance rel-L2 1e-2, the cross mask exactly."""
import numpy as np
import pytest

from oracle import synth
from tests.helpers import golden, rel_l2, weight_specs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["saocond_tiny", "saocond_tiny_b1_noneg"])
def test_saocond_encode_matches_reference(b2d, ctx, name):
    cfg = synth.SAOCOND_CONFIGS[name]
    w, inp = synth.saocond_weights(cfg), synth.saocond_inputs(cfg)
    cond = b2d.StableAudioConditioner(ctx, cfg.hidden, cfg.layers, cfg.heads, cfg.head_dim, cfg.intermediate,
                                      cfg.vocab, cfg.prompt_max_length, cfg.eps, weights=weight_specs(w))
    g = golden(name)
    secs = inp["normalized_seconds"].array()
    cross, cmask, glob = cond.encode_one(inp["input_ids"].array(), inp["attention_mask"].array(), secs)
    err_c, err_g = rel_l2(cross, g["cross_positive"].array()), rel_l2(glob, g["global"].array())
    print("%s: cross %.3g, global %.3g" % (name, err_c, err_g))
    assert np.isfinite(cross).all() and err_c < 1e-2 and err_g < 1e-3
    assert np.array_equal(cmask, g["cross_mask"].array())
    if cfg.has_negative:
        neg, _, _ = cond.encode_one(inp["negative_ids"].array(), inp["negative_mask"].array(), secs)
        assert rel_l2(neg, g["cross_negative"].array()) < 1e-2
        # encode (the reference's public entry) runs both batches and returns the same values
        both = cond.encode(inp["input_ids"].array(), inp["attention_mask"].array(), secs,
                           inp["negative_ids"].array(), inp["negative_mask"].array())
        assert rel_l2(both["positive"][0], cross) < 1e-6 and rel_l2(both["negative"][0], neg) < 1e-6
