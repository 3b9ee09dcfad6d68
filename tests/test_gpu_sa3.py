"""GPU parity of the Stable Audio 3 rectified-flow DiT path (StableAudioRfDitRuntime::sample) through the
C ABI: whole pingpong / euler sampling runs against the reference's own ggml CPU outputs
(tests/golden/sa3_*.b2db, made by oracle/ref's harness) and the fp32-activation numpy restatement
(oracle/sa3.py).  Covers memory tokens, local-add conditioning, per-head qk-RMSNorm + RoPE, differential
attention, the 6-way adaLN gates, APG-CFG with a masked negative prompt, ragged padding masks, the
per-step TensorIterator Philox noise and the rng_offset_blocks out-parameter.

Latent tolerance (rel-L2): max(2e-2, 1.5 x spread), spread = the reference's distance to the same
arithmetic without its activation rounding; the device path computes with fp16 (f32 weights) or bf16
operands and fp32 accumulation.
"""
import numpy as np
import pytest

from oracle import synth
from tests.helpers import golden, rel_l2, weight_specs

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

_models = {}


def make(b2d, ctx, name):
    if name not in _models:
        cfg = synth.SA3_CONFIGS[name]
        _models.clear()
        _models[name] = (cfg, b2d.StableAudio3DiT(
            ctx, cfg.embed_dim, cfg.depth, cfg.num_heads, cfg.cond_dim, cfg.global_cond_dim, cfg.local_add_cond_dim,
            cfg.num_memory_tokens, cfg.prompt_max_length, cfg.differential, cfg.io_channels,
            weights=weight_specs(synth.sa3_weights(cfg))))
    return _models[name]


def run(cfg, model, inp, **kw):
    a = {k: inp[k].array() for k in ("noise", "padding_mask", "schedule", "cross_positive", "cross_negative",
                                      "negative_mask", "global", "local_add")}
    return model.sample(a["noise"], a["padding_mask"], a["schedule"], a["cross_positive"], a["cross_negative"],
                        a["negative_mask"], a["global"], a["local_add"], cfg_scale=cfg.cfg, apg_scale=cfg.apg,
                        sampler=cfg.sampler, seed=cfg.seed, rng_offset=0, rng_policy=(cfg.rng_sms, cfg.rng_max_threads),
                        **kw)


@pytest.mark.parametrize("name", ["sa3_tiny_f32", "sa3_tiny_f32_diff_b2", "sa3_tiny_f32_euler_nocfg",
                                  "sa3_tiny_bf16_diff", "sa3_mid_bf16_diff_b2", "sa3_mid_q8_euler"])
def test_sa3_sample_matches_reference(b2d, ctx, name):
    cfg, model = make(b2d, ctx, name)
    inp = synth.sa3_inputs(cfg)
    out = run(cfg, model, inp)
    g = golden(name)
    ref, exact = g["latents"].array(), g["exact_latents"].array()
    assert np.isfinite(out).all()
    spread = rel_l2(exact, ref)
    err, err_exact = rel_l2(out, ref), rel_l2(out, exact)
    print("%s: vs ref %.3g (spread %.3g), vs exact %.3g" % (name, err, spread, err_exact))
    assert err < max(2e-2, 1.5 * spread), "rel-L2 %.3g vs reference (spread %.3g)" % (err, spread)
    assert err_exact < max(2e-2, 1.5 * spread), "rel-L2 %.3g vs exact oracle (spread %.3g)" % (err_exact, spread)
    # the graph replays deterministically, and the Philox offset advances once per pingpong step
    assert np.array_equal(out, run(cfg, model, inp))
    expect = int(g["rng_offset_out"].data[0]) if cfg.sampler == "pingpong" else 0
    assert model.rng_offset_blocks == expect


def test_sa3_device_api_and_errors(b2d, ctx):
    cfg, model = make(b2d, ctx, "sa3_tiny_f32")
    inp = synth.sa3_inputs(cfg)
    host = run(cfg, model, inp)
    keys = ("noise", "padding_mask", "schedule", "cross_positive", "cross_negative", "negative_mask", "global",
            "local_add")
    dev = [torch.from_numpy(np.ascontiguousarray(inp[k].array())).cuda() for k in keys]
    out = torch.empty(dev[0].shape, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    model.sample_device(*dev, out, cfg_scale=cfg.cfg, apg_scale=cfg.apg, sampler=cfg.sampler, seed=cfg.seed,
                        rng_policy=(cfg.rng_sms, cfg.rng_max_threads), stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), host)
    with pytest.raises(b2d.B2DError, match="pingpong or euler"):
        model.sample(*[inp[k].array() for k in keys], sampler="bogus")


def test_sa3_no_negative_prompt_and_rng_offset(b2d, ctx):
    """cross_negative = NULL (the unconditional half sees zeros, make_cross_conditioning with has_negative false)
    and a non-zero starting Philox offset, against the fp32-activation restatement run on the same request."""
    from oracle import bundle as B
    from oracle import sa3
    cfg, model = make(b2d, ctx, "sa3_tiny_f32")
    inp = dict(synth.sa3_inputs(cfg))
    inp["has_negative"] = B.i64(0)
    inp["rng_offset"] = B.i64(37)
    exact = sa3.sample(sa3.Sa3Dit(synth.sa3_weights(cfg), cfg, act="exact"), cfg, inp)
    a = {k: inp[k].array() for k in ("noise", "padding_mask", "schedule", "cross_positive", "global", "local_add")}
    out = model.sample(a["noise"], a["padding_mask"], a["schedule"], a["cross_positive"], None, None, a["global"],
                       a["local_add"], cfg_scale=cfg.cfg, apg_scale=cfg.apg, sampler=cfg.sampler, seed=cfg.seed,
                       rng_offset=37, rng_policy=(cfg.rng_sms, cfg.rng_max_threads))
    err = rel_l2(out, exact)
    print("no negative, offset 37: vs exact %.3g" % err)
    assert err < 2e-3, err
    from oracle import philox
    n = cfg.batch * cfg.io_channels * cfg.latent_tokens
    assert model.rng_offset_blocks == 37 + cfg.steps * philox.offset_blocks(n, cfg.rng_sms, cfg.rng_max_threads)


def test_sa3_prompt_shards_reproduce_the_batched_call(b2d, ctx):
    """Data-parallel shards of one batched pingpong request (one prompt each, rng_batch = (first, total)) draw
    their slices of the batched call's TensorIterator noise and reproduce its latents (up to GEMM accumulation
    order), and the batched call itself matches the reference."""
    cfg, model = make(b2d, ctx, "sa3_tiny_f32_diff_b2")
    inp = synth.sa3_inputs(cfg)
    keys = ("noise", "padding_mask", "schedule", "cross_positive", "cross_negative", "negative_mask", "global",
            "local_add")
    full = {k: inp[k].array() for k in keys}
    kw = dict(cfg_scale=cfg.cfg, apg_scale=cfg.apg, sampler=cfg.sampler, seed=cfg.seed,
              rng_policy=(cfg.rng_sms, cfg.rng_max_threads))
    batched = model.sample(*[full[k] for k in keys], **kw)
    offset_batched = model.rng_offset_blocks
    parts = []
    for b in range(cfg.batch):
        parts.append(model.sample(*[full[k][b:b + 1] for k in keys], rng_batch=(b, cfg.batch), **kw))
        assert model.rng_offset_blocks == offset_batched
    sharded = np.concatenate(parts)
    err = rel_l2(sharded, batched)
    print("shards vs batched %.3g" % err)
    assert err < 1e-3, err
    assert rel_l2(batched, golden("sa3_tiny_f32_diff_b2")["latents"].array()) < 2e-2
    # without the batch slice each one-prompt call draws its own (different) noise stream
    alone = model.sample(*[full[k][1:2] for k in keys], **kw)
    assert rel_l2(alone, batched[1:2]) > 1e-2
