"""Independent contexts on different devices in one process, used from two host threads at once.

The C ABI promises that a b2d_ctx is bound to one device and that contexts on different devices may run
concurrently (audio.cpp's launcher would drive one runtime per GPU from its own thread).  Each thread loads the
same tiny head and DiT, samples repeatedly, and must reproduce the single-device results bit for bit; kernel
attributes (dynamic shared-memory limits) are per device, so the second device must not depend on the first
having configured them.  Needs two GPUs; skipped on a one-GPU box."""
import threading

import numpy as np
import pytest

from oracle import synth
from tests.helpers import weight_specs

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _sample_head(b2d, dev, reps, out, errors):
    try:
        cfg = synth.HEAD_CONFIGS["small_q8_ragged"]
        ctx = b2d.Context(dev)
        head = b2d.VibeVoiceDiffusionHead(ctx, cfg.hidden, cfg.layers, cfg.ffn_ratio,
                                          weights=weight_specs(synth.head_weights(cfg)))
        inp = synth.head_inputs(cfg)
        args = [inp[k].array() for k in ("positive_condition", "negative_condition", "initial_speech")]
        dcfg = synth.DIT_CONFIGS["tiny_bf16"]
        dit = b2d.StableAudioDiT(ctx, dcfg.embed_dim, dcfg.depth, dcfg.num_heads, dcfg.cond_token_dim,
                                 dcfg.global_cond_dim, dcfg.io_channels, dcfg.prompt_max_length,
                                 weights=weight_specs(synth.dit_weights(dcfg)))
        dinp = synth.dit_inputs(dcfg)
        dargs = [dinp[k].array() for k in ("noise", "padding_mask", "cross_positive", "cross_negative", "global")]
        res = []
        for _ in range(reps):
            res.append((head.sample(*args, cfg.steps, cfg.cfg),
                        dit.sample(*dargs, steps=dcfg.steps, cfg_scale=dcfg.cfg, apg_scale=dcfg.apg)))
        out[dev] = res
        ctx.close()
    except Exception as e:  # reported by the main thread
        errors.append((dev, repr(e)))


def test_two_devices_two_threads(b2d):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    # reference results: device 0 alone
    solo, errors = {}, []
    _sample_head(b2d, 0, 1, solo, errors)
    assert not errors, errors
    out = {}
    threads = [threading.Thread(target=_sample_head, args=(b2d, d, 3, out, errors)) for d in (1, 0)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=600)
    assert not errors, errors
    for dev in (0, 1):
        for head_out, dit_out in out[dev]:
            assert np.array_equal(head_out, solo[0][0][0])
            assert np.array_equal(dit_out, solo[0][0][1])
