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
