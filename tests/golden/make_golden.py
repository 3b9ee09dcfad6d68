"""Generates the golden fixtures in this directory by running the reference's
own CPU implementation (oracle/_ref/b2d_ref_v4: audio.cpp's unmodified hot-path
sources + vendored ggml CPU backend, AVX-512 build with fp32 dot-product
accumulation) on the seeded synthetic configurations of oracle/synth.py.

Each fixture <name>.b2db holds the reference outputs plus ``input_sha256``
(a digest of the weight and input bundles) so a test can detect drift in the
synthetic generator before comparing.  Run from the repo root:

    python tests/golden/make_golden.py [names...]

It needs oracle/_ref built (make -C oracle/ref REF=<audio.cpp> VARIANT=v4).
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
os.environ.setdefault("B2D_REF_VARIANT", "v4")

from oracle import bundle as B  # noqa: E402
from oracle import dit, oobleck, ref_runner, sa3, saocond, synth, vibevoice, vvdec, vvlm  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))

HEAD_GOLDENS = ["tiny_f16", "tiny_q8", "tiny_bf16", "small_q8_ragged", "one_frame_f16", "one_step_q8",
                "vv15_f16_64", "vv15_q8_1024", "vv7_q8_32_3steps", "vv7_q8_1024"]
DIT_GOLDENS = ["tiny_bf16", "tiny_q8_b2_noapg", "tiny_f16_ragged", "tiny_bf16_vddim", "tiny_f16_3msde",
               "sao_bf16_1x1024_2steps", "sao_q8_1x1024_2steps", "sao_q8_16x64_2steps",
               "sao_q8_16x1024_2steps", "sao_bf16_1x1024", "sao_bf16_1x1024_noapg"]
SA3_GOLDENS = [n for n in synth.SA3_CONFIGS if "bench" not in n]
OOBLECK_GOLDENS = [n for n in synth.OOBLECK_CONFIGS if "bench" not in n]
VVDEC_GOLDENS = [n for n in synth.VVDEC_CONFIGS if "bench" not in n]
SAOCOND_GOLDENS = list(synth.SAOCOND_CONFIGS)
VVLM_GOLDENS = list(synth.VVLM_CONFIGS)


def digest(*bundles) -> np.ndarray:
    h = hashlib.sha256()
    for b in bundles:
        for name in sorted(b):
            t = b[name]
            h.update(name.encode())
            h.update(bytes([t.dtype]))
            h.update(np.asarray(t.dims, np.int64).tobytes())
            h.update(t.data.tobytes())
    return np.frombuffer(h.digest(), dtype=np.uint8).copy()


def head_golden(name: str) -> None:
    cfg = synth.HEAD_CONFIGS[name]
    w, inp = synth.head_weights(cfg), synth.head_inputs(cfg)
    out = ref_runner.run("vv", inp, w)
    # The reference requantises activations (Q8_0 blocks / fp16 / bf16) before every CPU matmul;
    # "exact_latents" is the numpy restatement with fp32 activations, i.e. the graph's arithmetic
    # without that rounding.  Their distance is the reference's own quantisation spread.
    head = vibevoice.Head(w, cfg, act="exact")
    exact = vibevoice.sample_speech_latents(head, cfg, inp["positive_condition"].array(),
                                            inp["negative_condition"].array(), inp["initial_speech"].array())
    fixture = {"latents": out["latents"], "exact_latents": B.f32(exact),
               "input_sha256": B.Tensor(B.U8, (32,), digest(w, inp))}
    B.write(os.path.join(HERE, "head_%s.b2db" % name), fixture)
    print("head", name, "ok", out["latents"].dims)


def head_storage_golden(name: str, storage: int, tag: str) -> None:
    """The head loaded with a weight storage type (quantize-on-load in the reference's weight store)."""
    cfg = synth.HEAD_CONFIGS[name]
    w, inp = synth.head_weights(cfg), synth.head_inputs(cfg)
    inp["storage_type"] = B.i64(storage)
    out = ref_runner.run("vv", inp, w)
    B.write(os.path.join(HERE, "head_%s_as_%s.b2db" % (name, tag)),
            {"latents": out["latents"], "input_sha256": B.Tensor(B.U8, (32,), digest(w, inp))})
    print("head", name, "as", tag, "ok")


def sched_golden() -> None:
    rng = np.random.default_rng(7)
    for steps in (1, 2, 10, 20, 3, 5, 50, 100):
        n = 96
        sample = rng.standard_normal(n).astype(np.float32)
        outs = rng.standard_normal((steps, n)).astype(np.float32)
        inp = synth.HeadConfig(steps=steps).scalars()
        inp.update({"sample": B.f32(sample), "model_outputs": B.f32(outs)})
        out = ref_runner.run("vvsched", inp)
        B.write(os.path.join(HERE, "sched_%d.b2db" % steps),
                {"sample": B.f32(sample), "model_outputs": B.f32(outs), "trace": out["trace"],
                 "timesteps": out["timesteps"]})
        print("sched", steps, "ok")


def q8_golden() -> None:
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((16, 256)) * 0.05).astype(np.float32)
    x[0, :32] = 0.0                      # all-zero block (d = 0)
    x[1, :32] = np.linspace(-1, 1, 32)   # exact ties around +-0.5 after scaling
    x[2, 7] = 40.0                       # outlier dominating its block
    x[3, :] = -x[3, :]
    out = ref_runner.run("q8", {"x": B.f32(x)})
    B.write(os.path.join(HERE, "q8_kat.b2db"), {"x": B.f32(x), "q8": out["q8"], "dequant": out["dequant"]})
    print("q8 ok")


# Full-length runs whose fp32-activation restatement is left out: the fixture holds the reference's latents
# only (the 100-step restatement of sao_bf16_1x1024 takes about 1.7 h of numpy on 8 cores).
NO_EXACT = {"sao_bf16_1x1024_noapg"}


def dit_golden(name: str) -> None:
    cfg = synth.DIT_CONFIGS[name]
    w, inp = synth.dit_weights(cfg), synth.dit_inputs(cfg)
    out = ref_runner.run("dit", inp, w, timeout=4 * 3600)
    fixture = {"latents": out["latents"], "input_sha256": B.Tensor(B.U8, (32,), digest(w, inp))}
    if name not in NO_EXACT:
        fixture["exact_latents"] = B.f32(dit.sample(dit.Dit(w, cfg, act="exact"), cfg, inp))  # fp32 activations
    B.write(os.path.join(HERE, "dit_%s.b2db" % name), fixture)
    print("dit", name, "ok", out["latents"].dims)


def dit_f32_golden(name: str) -> None:
    """The same seeded BF16 weights handed to the reference as F32 tensors (exact values): the reference then
    computes without rounding activations to bf16 before its matmuls.  Its distance to the BF16 run is the
    reference's own activation-rounding spread at full length, which the stiff CFG-7 trajectory amplifies."""
    cfg = synth.DIT_CONFIGS[name]
    w, inp = synth.dit_weights(cfg), synth.dit_inputs(cfg)
    w32 = {n: (B.Tensor(B.F32, t.dims, synth.decode_weight(t).reshape(-1).astype(np.float32))
               if t.dtype == B.BF16 else t) for n, t in w.items()}
    out = ref_runner.run("dit", inp, w32, timeout=6 * 3600)
    B.write(os.path.join(HERE, "dit_%s_f32w.b2db" % name),
            {"latents": out["latents"], "input_sha256": B.Tensor(B.U8, (32,), digest(w32, inp))})
    print("dit", name, "as f32 ok")


def dit_fresh_golden(name: str) -> None:
    """The reference's DPM++ 2M trajectory with a fresh FoundationRfDitRuntime for every model evaluation (harness
    command ``dit_fresh``).  The stock runtime computes its first graph call correctly and later calls with stale
    RoPE positions (written once when the graph is built, rf_dit.cpp:928-932, while ggml's allocator lends an
    input's memory to later nodes, ggml-alloc.c:692, 803-815), so its multi-step latents drift from its own
    algorithm; this fixture holds the reference's arithmetic (BF16 weights, bf16-rounded activations) without that
    drift."""
    cfg = synth.DIT_CONFIGS[name]
    w, inp = synth.dit_weights(cfg), synth.dit_inputs(cfg)
    out = ref_runner.run("dit_fresh", inp, w, timeout=6 * 3600)
    B.write(os.path.join(HERE, "dit_%s_fresh.b2db" % name),
            {"latents": out["latents"], "input_sha256": B.Tensor(B.U8, (32,), digest(w, inp))})
    print("dit", name, "fresh-graph ok")


def sa3_golden(name: str) -> None:
    """Stable Audio 3 DiT (StableAudioRfDitRuntime::sample) on a tiny seeded configuration."""
    cfg = synth.SA3_CONFIGS[name]
    w, inp = synth.sa3_weights(cfg), synth.sa3_inputs(cfg)
    out = ref_runner.run("sa3", inp, w)
    exact = sa3.sample(sa3.Sa3Dit(w, cfg, act="exact"), cfg, inp)
    B.write(os.path.join(HERE, "%s.b2db" % name),
            {"latents": out["latents"], "exact_latents": B.f32(exact), "rng_offset_out": out["rng_offset_out"],
             "input_sha256": B.Tensor(B.U8, (32,), digest(w, inp))})
    print("sa3", name, "ok", out["latents"].dims)


def oobleck_golden(name: str) -> None:
    """Stable Audio Oobleck VAE decode (OobleckAutoencoderRuntime::decode) on a tiny seeded configuration."""
    cfg = synth.OOBLECK_CONFIGS[name]
    w, inp = synth.oobleck_weights(cfg), synth.oobleck_inputs(cfg)
    out = ref_runner.run("oobleck", inp, w)
    B.write(os.path.join(HERE, "%s.b2db" % name),
            {"audio": out["audio"], "input_sha256": B.Tensor(B.U8, (32,), digest(w, inp))})
    print("oobleck", name, "ok", out["audio"].dims)


def vvdec_golden(name: str) -> None:
    """VibeVoice acoustic sigma-VAE decode (VibeVoiceTokenizerWeightsRuntime::decode_acoustic), tiny config."""
    cfg = synth.VVDEC_CONFIGS[name]
    w, inp = synth.vvdec_weights(cfg), synth.vvdec_inputs(cfg)
    out = ref_runner.run("vvdec", inp, w)
    B.write(os.path.join(HERE, "%s.b2db" % name),
            {"samples": out["samples"], "input_sha256": B.Tensor(B.U8, (32,), digest(w, inp))})
    print("vvdec", name, "ok", out["samples"].dims)


def saocond_golden(name: str) -> None:
    """SAO 1.0 conditioner (FoundationConditionerRuntime::encode: T5-base + number conditioners), tiny config."""
    cfg = synth.SAOCOND_CONFIGS[name]
    w, inp = synth.saocond_weights(cfg), synth.saocond_inputs(cfg)
    out = ref_runner.run("saocond", inp, w)
    keep = {k: v for k, v in out.items() if k != "wall_ms"}
    keep["input_sha256"] = B.Tensor(B.U8, (32,), digest(w, inp))
    B.write(os.path.join(HERE, "%s.b2db" % name), keep)
    print("saocond", name, "ok", out["cross_positive"].dims)


def vvlm_golden(name: str) -> None:
    """VibeVoice Qwen2.5 LM: prefill + cached steps (VibeVoiceDecoderWeightsRuntime), tiny config."""
    cfg = synth.VVLM_CONFIGS[name]
    w, inp = synth.vvlm_weights(cfg), synth.vvlm_inputs(cfg)
    out = ref_runner.run("vvlm", inp, w)
    B.write(os.path.join(HERE, "%s.b2db" % name),
            {"logits": out["logits"], "last_hidden": out["last_hidden"],
             "input_sha256": B.Tensor(B.U8, (32,), digest(w, inp))})
    print("vvlm", name, "ok", out["logits"].dims)


def main(argv) -> None:
    names = argv or (["q8", "sched"] + ["head:" + n for n in HEAD_GOLDENS] + ["dit:" + n for n in DIT_GOLDENS] +
                     ["sa3:" + n for n in SA3_GOLDENS] + ["oobleck:" + n for n in OOBLECK_GOLDENS] +
                     ["vvdec:" + n for n in VVDEC_GOLDENS] + ["saocond:" + n for n in SAOCOND_GOLDENS] +
                     ["vvlm:" + n for n in VVLM_GOLDENS])
    for n in names:
        if n == "q8":
            q8_golden()
        elif n == "sched":
            sched_golden()
        elif n.startswith("headq8:"):  # storage type Q8_0 (assets::TensorStorageType::Q8_0 = 13)
            head_storage_golden(n[7:], 13, "q8")
        elif n.startswith("head:"):
            head_golden(n[5:])
        elif n.startswith("ditfresh:"):
            dit_fresh_golden(n[9:])
        elif n.startswith("ditf32:"):
            dit_f32_golden(n[7:])
        elif n.startswith("dit:"):
            dit_golden(n[4:])
        elif n.startswith("sa3:"):
            sa3_golden(n[4:])
        elif n.startswith("oobleck:"):
            oobleck_golden(n[8:])
        elif n.startswith("vvdec:"):
            vvdec_golden(n[6:])
        elif n.startswith("saocond:"):
            saocond_golden(n[8:])
        elif n.startswith("vvlm:"):
            vvlm_golden(n[5:])
        else:
            raise SystemExit("unknown fixture " + n)


if __name__ == "__main__":
    main(sys.argv[1:])
