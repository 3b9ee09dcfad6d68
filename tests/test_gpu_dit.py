"""GPU parity of the Stable Audio Open 1.0 DiT path through the C ABI:
* the flash-attention kernel against a torch fp32 softmax(QK^T/8)V (self-attention
  shape, and the cross-attention shape with 130 keys and repeated KV heads);
* whole DPM++ 2M sampling runs against the reference's own ggml CPU outputs
  (tests/golden/dit_*.b2db) and the fp32-activation numpy restatement.

Latent tolerance (rel-L2): vs the reference max(2e-2, 1.5 x spread) where spread is
the reference's distance to the same arithmetic without its activation rounding;
vs the fp32-activation restatement max(2e-2 (bf16 operands) / 1e-2 (fp16 operands), 1.5 x spread):
from sigma_max = 100 a 2-step run amplifies bf16 activation rounding to ~3.4 % in the reference itself.
"""
import os

import numpy as np
import pytest

from oracle import bundle as B
from oracle import synth
from tests.helpers import GOLDEN, golden, rel_l2, weight_specs

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _attn_ref(q, k, v, rep):
    # q [S, Lq, H, 64], k/v [S, Lk, KVH, 64]
    k = k.float().repeat_interleave(rep, dim=2)
    v = v.float().repeat_interleave(rep, dim=2)
    s = torch.einsum("sqhd,skhd->shqk", q.float(), k) / 8.0
    return torch.einsum("shqk,skhd->sqhd", torch.softmax(s, dim=-1), v)


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("lq,lk,heads,rep,nseq", [(1025, 1025, 4, 1, 2), (1025, 130, 4, 2, 2), (37, 16, 2, 1, 3),
                                                  (200, 64, 3, 3, 1)])
def test_attention_kernel(ctx, bf16, lq, lk, heads, rep, nseq):
    dt = torch.bfloat16 if bf16 else torch.float16
    g = torch.Generator(device="cuda").manual_seed(lq + lk)
    q = torch.randn(nseq, lq, heads, 64, device="cuda", generator=g).to(dt)
    k = torch.randn(nseq, lk, heads // rep, 64, device="cuda", generator=g).to(dt)
    v = torch.randn(nseq, lk, heads // rep, 64, device="cuda", generator=g).to(dt)
    o = torch.zeros(nseq, lq, heads, 64, device="cuda", dtype=dt)
    ctx.attention(q.data_ptr(), heads * 64, lq * heads * 64, k.data_ptr(), v.data_ptr(), (heads // rep) * 64,
                  lk * (heads // rep) * 64, o.data_ptr(), heads * 64, lq * heads * 64, lq, lk, heads, rep, nseq,
                  bf16=bf16)
    torch.cuda.synchronize()
    ref = _attn_ref(q, k, v, rep)
    err = float((o.float() - ref).norm() / ref.norm())
    assert err < (1e-2 if bf16 else 2e-3), err


_dits = {}


def make_dit(b2d, ctx, name):
    """The configuration and a loaded model; consecutive configurations with the same weights share the model."""
    cfg = synth.DIT_CONFIGS[name]
    key = (cfg.embed_dim, cfg.depth, cfg.num_heads, cfg.cond_token_dim, cfg.global_cond_dim, cfg.io_channels,
           cfg.prompt_max_length, cfg.wtype, cfg.wseed)
    if key not in _dits:
        w = synth.dit_weights(cfg)
        _dits.clear()
        _dits[key] = b2d.StableAudioDiT(ctx, cfg.embed_dim, cfg.depth, cfg.num_heads, cfg.cond_token_dim,
                                        cfg.global_cond_dim, cfg.io_channels, cfg.prompt_max_length,
                                        weights=weight_specs(w))
    return cfg, _dits[key]


# Multi-step C3 runs at full size.  The trajectory of the random-init SAO-1.0 DiT at CFG 7 is stiff: the
# reference's own two arithmetics (BF16 weights, whose matmuls round activations to bf16, and the same weight
# values as F32, fixture *_f32w) are 0.41 apart after 10 steps and 0.066 after 100, and the fp32-activation
# restatement is 0.81 from both after 10 steps.  Per-element rel-L2 is therefore held at 1.5x the distance
# measured on a B200 (gpu vs reference; gpu vs the restatement where the fixture has it), as a regression bound.
STIFF_TOL = {  # name: (vs reference, vs exact restatement or None)
    "sao_bf16_1x1024_10steps": (1.2, 0.53),  # measured 0.80 / 0.356
    "sao_bf16_1x1024": (1.26, 0.163),         # measured 0.84 / 0.108 (100 steps, APG 1)
    "sao_bf16_1x1024_noapg": (1.5, None),     # measured 1.008 (100 steps, plain CFG)
}


def check_fresh_graph_reference(name, out, g, tol_exact):
    """Compares with the reference run one fresh graph per model evaluation (fixture dit_<name>_fresh), where that
    fixture exists.  The stock reference runtime recomputes with stale RoPE positions after its first graph call
    (rf_dit.cpp:928-932 writes them once; ggml-alloc.c:692, 803-815 lends a consumed input's memory to later nodes),
    so its multi-step latents are not its own algorithm; the fresh-graph run is.  Bound: the one the restatement
    bound implies (triangle inequality), ||out - fresh|| <= tol_exact ||exact|| + ||exact - fresh||."""
    path = os.path.join(GOLDEN, "dit_%s_fresh.b2db" % name)
    if tol_exact is None or not os.path.exists(path):
        return None
    fresh = B.read(path)["latents"].array().astype(np.float64)
    exact = g["exact_latents"].array().astype(np.float64)
    bound = (tol_exact * np.linalg.norm(exact) + np.linalg.norm(exact - fresh)) / np.linalg.norm(fresh)
    err = rel_l2(out, fresh)
    assert err < bound, "rel-L2 %.3g vs the fresh-graph reference (bound %.3g)" % (err, bound)
    return err


def run(cfg, dit, inp):
    return dit.sample(inp["noise"].array(), inp["padding_mask"].array(), inp["cross_positive"].array(),
                      inp["cross_negative"].array(), inp["global"].array(), steps=cfg.steps,
                      sigma_min=cfg.sigma_min, sigma_max=cfg.sigma_max, rho=cfg.rho, cfg_scale=cfg.cfg,
                      apg_scale=cfg.apg, sampler=cfg.sampler, schedule=inp["schedule"].array(), seed=cfg.seed,
                      rng_offset=0, rng_policy=(cfg.rng_sms, cfg.rng_max_threads))


@pytest.mark.parametrize("name", ["tiny_bf16", "tiny_q8_b2_noapg", "tiny_f16_ragged", "sao_bf16_1x1024_2steps",
                                  "sao_bf16_1x1024_10steps", "sao_bf16_1x1024", "sao_bf16_1x1024_noapg",
                                  "sao_q8_1x1024_2steps", "tiny_bf16_vddim", "tiny_f16_3msde",
                                  "sao_q8_16x64_2steps", "sao_q8_16x1024_2steps"])
def test_dit_sample_matches_reference(b2d, ctx, name):
    cfg, dit = make_dit(b2d, ctx, name)
    inp = synth.dit_inputs(cfg)
    out = run(cfg, dit, inp)
    g = golden("dit_" + name)
    ref = g["latents"].array()
    assert np.isfinite(out).all()
    err = rel_l2(out, ref)
    if name in STIFF_TOL:
        tol_ref, tol_exact = STIFF_TOL[name]
        line = "%s: vs ref %.3g" % (name, err)
        assert err < tol_ref, "rel-L2 %.3g vs reference" % err
        if tol_exact is not None:
            err_exact = rel_l2(out, g["exact_latents"].array())
            line += ", vs exact %.3g" % err_exact
            assert err_exact < tol_exact, "rel-L2 %.3g vs exact restatement" % err_exact
            err_fresh = check_fresh_graph_reference(name, out, g, tol_exact)
            if err_fresh is not None:
                line += ", vs fresh-graph reference %.3g" % err_fresh
        print(line)
    elif "exact_latents" in g:
        exact = g["exact_latents"].array()
        spread = rel_l2(exact, ref)
        err_exact = rel_l2(out, exact)
        print("%s: vs ref %.3g (spread %.3g), vs exact %.3g" % (name, err, spread, err_exact))
        assert err < max(2e-2, 1.5 * spread), "rel-L2 %.3g vs reference (spread %.3g)" % (err, spread)
        assert err_exact < max(2e-2 if cfg.wtype == synth.BF16 else 1e-2, 1.5 * spread), \
            "rel-L2 %.3g vs exact oracle (spread %.3g)" % (err_exact, spread)
    else:
        raise AssertionError("fixture %s has no restatement and no stiff-trajectory bound" % name)
    out2 = run(cfg, dit, inp)
    assert np.array_equal(out, out2)
    # rng_offset_blocks out-parameter: one TensorIterator draw per step with a non-zero next sigma
    from oracle import philox
    draws = cfg.steps - 1 if cfg.sampler == "dpmpp-3m-sde" else 0
    n = cfg.batch * cfg.io_channels * cfg.latent_tokens
    assert dit.rng_offset_blocks == draws * philox.offset_blocks(n, cfg.rng_sms, cfg.rng_max_threads)


# Known answers of generate_torch_cuda_randn / the TensorIterator form
# (tests/unittests/test_torch_random.cpp:33-100 of audio.cpp) are pinned against the oracle on CPU
# in test_oracle.py; here the device generator must equal that oracle bit for bit.
@pytest.mark.parametrize("layout,count,seed,offset,sms,mt,bf16", [
    (0, 4099, 1234, 0, 1, 256, False), (0, 1000, 5678, 0, 1, 256, True),
    (1, 65 * 64 * 3, 42, 0, 148, 2048, False), (1, 5000, 7, 13, 1, 256, False), (1, 1 << 20, 99, 5, 148, 2048, True)])
def test_torch_randn_matches_oracle(ctx, layout, count, seed, offset, sms, mt, bf16):
    from oracle import philox
    out = torch.empty(count, dtype=torch.float32, device="cuda")
    ctx.torch_randn(out.data_ptr(), count, seed, offset, layout, sms, mt, bf16,
                    stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    if layout == 0:
        ref = philox.torch_cuda_randn(count, seed, bf16=bf16, start=offset)
    else:
        ref = philox.tensor_iterator_randn(count, seed, offset, sms, mt, bf16=bf16)
    # log / sin / cos of the device math library versus libm: a few fp32 ulp, which after bf16 rounding
    # can flip a value that sits on a rounding boundary by one bf16 ulp (2^-7 relative)
    if bf16:
        diff = got != ref
        assert diff.mean() < 1e-4
        ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref[diff]), 1e-30))) - 7)
        assert (np.abs(got[diff] - ref[diff]) <= ulp).all()
    else:
        np.testing.assert_allclose(got, ref, rtol=2e-6, atol=2e-6)
    assert abs(float(got.mean())) < 0.1 and abs(float(got.std()) - 1.0) < 0.1


def test_dit_without_cfg_and_device_api(b2d, ctx):
    cfg, dit = make_dit(b2d, ctx, "tiny_bf16")
    inp = synth.dit_inputs(cfg)
    host = dit.sample(inp["noise"].array(), inp["padding_mask"].array(), inp["cross_positive"].array(), None,
                      inp["global"].array(), steps=3, cfg_scale=1.0)
    assert np.isfinite(host).all()
    from oracle import dit as D
    cfg1 = synth.DitConfig(**{**cfg.__dict__, "steps": 3, "cfg": 1.0})
    ref = D.sample_dpmpp_2m(D.Dit(synth.dit_weights(cfg), cfg1, act="exact"), cfg1, inp)
    assert rel_l2(host, ref) < 2e-2
    dev = [torch.from_numpy(inp[k].array().copy()).cuda() for k in ("noise", "padding_mask", "cross_positive",
                                                                    "global")]
    out = torch.empty_like(dev[0])
    dit.sample_device(dev[0], dev[1], dev[2], None, dev[3], out, steps=3, cfg_scale=1.0,
                      stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ctx.sync()
    assert np.array_equal(out.cpu().numpy(), host)


def test_dit_prompt_shards_reproduce_the_batched_3m_sde_call(b2d, ctx):
    """Data-parallel shards of one batched DPM++ 3M SDE request (rng_batch = (first, total)) draw their slices
    of the batched call's TensorIterator noise and reproduce its latents (up to GEMM accumulation order)."""
    cfg, dit = make_dit(b2d, ctx, "tiny_f16_3msde")
    inp = synth.dit_inputs(cfg)
    keys = ("noise", "padding_mask", "cross_positive", "cross_negative", "global")
    full = {k: inp[k].array() for k in keys}
    kw = dict(steps=cfg.steps, sigma_min=cfg.sigma_min, sigma_max=cfg.sigma_max, rho=cfg.rho, cfg_scale=cfg.cfg,
              apg_scale=cfg.apg, sampler=cfg.sampler, seed=cfg.seed, rng_policy=(cfg.rng_sms, cfg.rng_max_threads))
    batched = dit.sample(*[full[k] for k in keys], **kw)
    off = dit.rng_offset_blocks
    parts = []
    for b in range(cfg.batch):
        parts.append(dit.sample(*[full[k][b:b + 1] for k in keys], rng_batch=(b, cfg.batch), **kw))
        assert dit.rng_offset_blocks == off
    err = rel_l2(np.concatenate(parts), batched)
    print("shards vs batched %.3g" % err)
    assert err < 1e-3, err
    with pytest.raises(b2d.B2DError, match="outside a batch"):
        dit.sample(*[full[k][1:2] for k in keys], rng_batch=(2, cfg.batch), **kw)
