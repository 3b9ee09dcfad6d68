"""GPU parity of the VibeVoice language model (Qwen2.5 decoder) through the C ABI: prefill of the prompt's
embeddings, then cached single-position steps, with the projections on the tensor-core GEMMs (fp16 operands, fp32
accumulation and residual stream), NEOX RoPE + KV append, causal GQA attention against the fp32 KV cache and SwiGLU.
Logits and final-norm hidden state of the prefill's last position and of every step are compared with the
reference's own CPU output (tests/golden/vvlm_*.b2db) and the numpy restatement (oracle/vvlm.py); tolerance
rel-L2 1e-2."""
import numpy as np
import pytest

from oracle import synth
from tests.helpers import golden, rel_l2, weight_specs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["vvlm_tiny", "vvlm_tiny_mha_long"])
def test_vvlm_prefill_and_steps_match_reference(b2d, ctx, name):
    cfg = synth.VVLM_CONFIGS[name]
    w, inp = synth.vvlm_weights(cfg), synth.vvlm_inputs(cfg)
    lm = b2d.VibeVoiceLanguageModel(ctx, cfg.hidden, cfg.intermediate, cfg.heads, cfg.kv_heads, cfg.head_dim,
                                    cfg.layers, cfg.vocab, cfg.max_positions, cfg.eps, cfg.rope_theta,
                                    weights=weight_specs(w))
    table = w["model.language_model.embed_tokens.weight"].array()
    logits, hidden = [], []
    lg, hd = lm.prefill(table[inp["prefill_ids"].array()])
    logits.append(lg)
    hidden.append(hd)
    for i in inp["step_ids"].array():
        lg, hd = lm.step(table[i])
        logits.append(lg)
        hidden.append(hd)
    g = golden(name)
    err_l = rel_l2(np.stack(logits), g["logits"].array())
    err_h = rel_l2(np.stack(hidden), g["last_hidden"].array())
    print("%s: logits %.3g, hidden %.3g" % (name, err_l, err_h))
    assert err_l < 1e-2 and err_h < 1e-2


def test_vvlm_device_buffers_match_host_buffers(b2d, ctx):
    """prefill_device / step_device (device embeddings in, device logits and hidden out, no host round trip) give
    the host entry points' values."""
    import torch
    cfg = synth.VVLM_CONFIGS["vvlm_tiny"]
    w, inp = synth.vvlm_weights(cfg), synth.vvlm_inputs(cfg)
    lm = b2d.VibeVoiceLanguageModel(ctx, cfg.hidden, cfg.intermediate, cfg.heads, cfg.kv_heads, cfg.head_dim,
                                    cfg.layers, cfg.vocab, cfg.max_positions, cfg.eps, cfg.rope_theta,
                                    weights=weight_specs(w))
    table = w["model.language_model.embed_tokens.weight"].array()
    host = [lm.prefill(table[inp["prefill_ids"].array()])]
    host += [lm.step(table[i]) for i in inp["step_ids"].array()]
    dev = torch.device("cuda", ctx.device)
    lg = torch.empty(cfg.vocab, dtype=torch.float32, device=dev)
    hd = torch.empty(cfg.hidden, dtype=torch.float32, device=dev)
    got = []
    e = torch.from_numpy(np.ascontiguousarray(table[inp["prefill_ids"].array()], np.float32)).to(dev)
    lm.prefill_device(e, lg, hd)
    ctx.sync()
    got.append((lg.cpu().numpy(), hd.cpu().numpy()))
    for i in inp["step_ids"].array():
        e = torch.from_numpy(np.ascontiguousarray(table[i], np.float32)).to(dev)
        lm.step_device(e, lg, hd)
        ctx.sync()
        got.append((lg.cpu().numpy(), hd.cpu().numpy()))
    for (hl, hh), (gl, gh) in zip(host, got):
        assert rel_l2(gl, hl) < 1e-6 and rel_l2(gh, hh) < 1e-6


def test_lm_hidden_state_feeds_the_head_on_device(b2d, ctx):
    """The generator's per-token hand-off with every buffer on the GPU: the LM's cached step writes its last hidden
    state to device memory and the diffusion head samples that token's latent from it as the positive condition
    (src/models/vibevoice/generator.cpp:590-608).  Same latents as the host-buffer chain."""
    import torch
    lcfg = synth.VVLmConfig(hidden=256, intermediate=512, heads=4, kv_heads=2, head_dim=64, layers=1, prefill=5,
                            steps=3, wseed=51, seed=52)
    hcfg = synth.HeadConfig(hidden=256, wtype=synth.F16, frames=1, steps=5)
    w, inp = synth.vvlm_weights(lcfg), synth.vvlm_inputs(lcfg)
    lm = b2d.VibeVoiceLanguageModel(ctx, lcfg.hidden, lcfg.intermediate, lcfg.heads, lcfg.kv_heads, lcfg.head_dim,
                                    lcfg.layers, lcfg.vocab, lcfg.max_positions, lcfg.eps, lcfg.rope_theta,
                                    weights=weight_specs(w))
    head = b2d.VibeVoiceDiffusionHead(ctx, hcfg.hidden, hcfg.layers, hcfg.ffn_ratio,
                                      weights=weight_specs(synth.head_weights(hcfg)))
    table = w["model.language_model.embed_tokens.weight"].array()
    ids = inp["step_ids"].array()
    neg = np.zeros((1, hcfg.hidden), np.float32)
    x0 = np.random.default_rng(7).standard_normal((len(ids), 2, 64)).astype(np.float32)
    # host buffers
    lm.prefill(table[inp["prefill_ids"].array()])
    host = []
    for j, i in enumerate(ids):
        _, hd = lm.step(table[i])
        host.append(head.sample(hd[None, :].copy(), neg, x0[j], hcfg.steps, hcfg.cfg))
    # device buffers
    dev = torch.device("cuda", ctx.device)
    lg = torch.empty(lcfg.vocab, dtype=torch.float32, device=dev)
    hd = torch.empty(1, lcfg.hidden, dtype=torch.float32, device=dev)
    neg_d = torch.zeros(1, hcfg.hidden, dtype=torch.float32, device=dev)
    x0_d = torch.from_numpy(x0).to(dev)
    out = torch.empty(len(ids), 1, 64, dtype=torch.float32, device=dev)
    lm.prefill_device(torch.from_numpy(np.ascontiguousarray(table[inp["prefill_ids"].array()])).to(dev), lg, hd)
    for j, i in enumerate(ids):
        lm.step_device(torch.from_numpy(np.ascontiguousarray(table[i])).to(dev), lg, hd)
        head.sample_device(hd, neg_d, x0_d[j], hcfg.steps, hcfg.cfg, out[j])
    ctx.sync()
    got = out.cpu().numpy()
    for j in range(len(ids)):
        assert rel_l2(got[j], host[j]) < 1e-6, j
