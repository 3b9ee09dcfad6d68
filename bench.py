"""Benchmark of the diffusion denoising hot path on B200.

Workload (the headline configuration, C2): VibeVoice-1.5B diffusion head, Q8_0 weights
(random N(0, 0.02), seeded), 1024 frames per call with CFG pairs (2048 head
rows), conditions N(0,1) [1024, 1536], null condition zeros, x_T N(0,1),
10-step DPM-Solver++(2M), CFG 1.3.  One "step" = one whole sampling call
(sample_vibevoice_speech_latents).  Metric: latent frames/s (CFG rows not
counted), whole job over all ranks.  N GPUs: one process per GPU, each samples
its own 1024 frames (weak scaling, no collective on the data path).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "latent frames/sec (VibeVoice diffusion head)"
UNIT = "frames/s"
T_START = time.time()
WORKLOAD = "vv15_q8_1024"
C1_WORKLOAD = "vv15_f16_64"


def load_package():
    if "audiocpp_b200" in sys.modules:
        return sys.modules["audiocpp_b200"]
    spec = importlib.util.spec_from_file_location("audiocpp_b200", os.path.join(ROOT, "audio.cpp_b200", "__init__.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules["audiocpp_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def config_json(cfg, n, extra=None):
    d = {"workload": WORKLOAD, "model": "VibeVoice-1.5B diffusion head (random-init)", "weights": cfg.wtype,
         "frames_per_rank": cfg.frames, "head_rows_per_rank": 2 * cfg.frames, "hidden": cfg.hidden,
         "layers": cfg.layers, "ffn": cfg.ffn, "latent": cfg.latent, "dpm_steps": cfg.steps, "cfg_scale": cfg.cfg,
         "global_batch_frames": cfg.frames * n, "parallelism": "dp%d (independent frames per GPU)" % n,
         "l2": "flushed (256 MiB write) before every timed call"}
    if extra:
        d.update(extra)
    return d


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _wait_for(path, limit_s):
    t0 = time.time()
    while not os.path.exists(path):
        if time.time() - t0 > limit_s:
            return False
        time.sleep(0.2)
    return True


def log(msg):
    """Progress on stderr (stdout carries only the JSON line)."""
    print("[bench rank %s %.0fs] %s" % (os.environ.get("RANK", "0"), time.time() - T_START, msg), file=sys.stderr,
          flush=True)


def node_shared(fn, cfg, wait_s=600.0):
    """fn(cfg) computed once per node: with several ranks, local rank 0 synthesises the seeded weights and the
    other ranks of the node read its pickle (the DiT's 1.1 GB of Q8_0 weights take about a minute of numpy per
    synthesis, which eight ranks would otherwise repeat side by side).  The hand-off is through files only (the
    file appears by an atomic rename; each reader leaves a marker; the writer removes both once every local rank
    has read), so it does not depend on when a device-side barrier returns.  Every rank must pass the same
    `cfg`; should a rank not find the file within `wait_s` seconds it synthesises the weights itself (and the writer
    stops waiting for it), so a mismatch costs time, never a hang.  Outside the timed region."""
    world, _, local = dist_setup()
    log("weights: %s" % fn.__name__)
    if world == 1:
        return fn(cfg)
    import pickle
    import tempfile
    import zlib
    nlocal = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    tag = "%s_%08x" % (fn.__name__, zlib.crc32(repr(cfg).encode()))
    path = os.path.join(tempfile.gettempdir(), "b2d_bench_%d_%s.pkl" % (os.getppid(), tag))
    if local == 0:
        val = fn(cfg)
        with open(path + ".tmp", "wb") as f:
            pickle.dump(val, f, protocol=5)
        os.replace(path + ".tmp", path)
        if all(_wait_for("%s.read%d" % (path, r), wait_s) for r in range(1, nlocal)):
            for r in range(1, nlocal):
                os.remove("%s.read%d" % (path, r))
            os.remove(path)
        else:
            print("bench: a local rank did not read %s; left in place" % path, file=sys.stderr, flush=True)
        return val
    if not _wait_for(path, wait_s):
        print("bench: %s did not appear; synthesising on this rank" % path, file=sys.stderr, flush=True)
        return fn(cfg)
    with open(path, "rb") as f:
        val = pickle.load(f)
    open("%s.read%d" % (path, local), "w").close()
    return val


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    def __init__(self, device: int):
        self.device, self.samples, self.proc = device, [], None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), "--query-gpu=" + q,
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 7:
                self.samples.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[3 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": float(self.samples[0][1]),
                "reasons": reasons, "samples": len(self.samples)}


def run_cpu_reference(cfg, frames, reps, threads):
    """The reference's own CPU implementation (oracle/_ref) on `frames` frames of the workload."""
    from oracle import ref_runner, synth
    sub = synth.HeadConfig(**{**cfg.__dict__, "frames": frames})
    inp = synth.head_inputs(sub)
    w = synth.head_weights(sub)
    out = ref_runner.run("vv", inp, w, threads=threads, reps=reps)
    ms = out["wall_ms"].data
    return ms, ref_runner.variant()


def bench_reference(args):
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    from oracle import ref_runner, synth
    cfg = synth.HEAD_CONFIGS[WORKLOAD]
    threads = os.cpu_count() or 1
    frames = cfg.frames  # the full 1024-frame call (same weights, inputs, 10 steps, CFG) -- about 7 s on 16 cores
    if not ref_runner.available():
        print(json.dumps({"impl": "reference", "unavailable": "reference CPU build (oracle/_ref) not present"}))
        return
    ms, variant = run_cpu_reference(cfg, frames, args.warmup + args.steps, threads)
    timed = np.array(ms[args.warmup:], np.float64)
    value = frames / (timed.mean() / 1e3)
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": float(timed.mean()), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32 graph, Q8_0 weights (ggml CPU)", "data": "synthetic",
            "impl": "reference",
            "config": config_json(cfg, 1),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference",
                             "sample": "%d frames x %d DPM steps x CFG per call, audio.cpp ggml CPU build (%s)" % (
                                 frames, cfg.steps, variant)},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def bench_ggml_cuda(args):
    """GPU comparison point: the reference's own ggml-cuda backend (oracle/ref/Makefile VARIANT=cuda, compiled for
    sm_100a from the vendored sources) running the reference's stock sampling entry points on the C2 and C1 head workloads
    and the C3 DiT workload, timed by the harness around each whole sampling call (host inputs in, host latents
    out, the runtime and its device weights built before the first call).  One JSON line, rank 0 only."""
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    from oracle import bundle as B
    from oracle import ref_runner, synth
    exe = ref_runner.cuda_binary()
    if exe is None:
        print(json.dumps({"impl": "reference-ggml-cuda", "unavailable": "oracle/_ref/b2d_ref_cuda not built"}))
        return
    env = {"B2D_REF_BACKEND": "cuda"}
    golden_dir = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tests", "golden")

    def rel_to_golden(name, lat):
        path = os.path.join(golden_dir, name + ".b2db")
        if not os.path.exists(path):
            return None
        ref = B.read(path)["latents"].array().astype(np.float64).ravel()
        return float(np.linalg.norm(lat.astype(np.float64).ravel() - ref) / np.linalg.norm(ref))

    line = {"impl": "reference-ggml-cuda", "n_gpus": 1, "backend": "audio.cpp vendored ggml-cuda, sm_100a"}
    reps = args.warmup + args.steps
    for key, workload in (("head", WORKLOAD), ("c1", C1_WORKLOAD)):
        cfg = synth.HEAD_CONFIGS[workload]
        try:
            o = ref_runner.run("vv", synth.head_inputs(cfg), synth.head_weights(cfg), reps=reps, exe=exe,
                               env=env, timeout=900)
            ms = float(np.median(np.asarray(o["wall_ms"].data[args.warmup:], np.float64)))
            line[key] = {"workload": workload, "metric": METRIC, "value": round(cfg.frames / (ms / 1e3), 1),
                         "unit": UNIT, "ms_per_call": round(ms, 3), "calls_timed": args.steps,
                         "rel_l2_vs_reference_cpu": rel_to_golden("head_" + workload, o["latents"].array())}
        except Exception as e:  # the reference's failure is reported, not raised
            line[key] = {"unavailable": str(e).splitlines()[0][:300]}
    dcfg = synth.DIT_CONFIGS[DIT_WORKLOAD]
    try:
        calls = max(1, args.dit_steps)
        o = ref_runner.run("dit", synth.dit_inputs(dcfg), synth.dit_weights(dcfg), reps=1 + calls,
                           exe=exe, env=env, timeout=1800)
        ms = float(np.median(np.asarray(o["wall_ms"].data[1:], np.float64)))
        line["dit"] = {"workload": DIT_WORKLOAD, "metric": "sequence-steps/s (SAO DiT, CFG rows counted)",
                       "value": round(2 * dcfg.batch * dcfg.steps / (ms / 1e3), 3), "unit": "seq-steps/s",
                       "ms_per_call": round(ms, 2), "calls_timed": calls,
                       "rel_l2_vs_reference_cpu": rel_to_golden("dit_" + DIT_WORKLOAD, o["latents"].array())}
    except Exception as e:
        line["dit"] = {"unavailable": str(e).splitlines()[0][:300]}
    print(json.dumps(line))


def gemm_roofline(b2d, ctx, torch, cfg, peaks):
    """Times the dominant kernel (FFN gate/up GEMM + SwiGLU epilogue, 2048 x 9216 x 1536) with CUDA events."""
    M, K, N = 2 * cfg.frames, cfg.hidden, 2 * cfg.ffn
    a = torch.randn(M, K, device="cuda").half()
    w = (torch.randn(N, K, device="cuda") * 0.02).half()
    out = torch.empty(M, N // 2, device="cuda", dtype=torch.float16)
    st = torch.cuda.current_stream()
    # bn=512: the 2-SM (cta_group::2) 256 x 256 pair-tile kernel the head runs for this GEMM
    launch = lambda: ctx.gemm(a.data_ptr(), w.data_ptr(), M, N, K, epilogue=b2d.EPI_SWIGLU, bn=512,
                              out=out.data_ptr(), ldo=N // 2, stream=st.cuda_stream)
    for _ in range(5):
        launch()
    torch.cuda.synchronize()
    reps = 50
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        launch()
    e1.record(st)
    torch.cuda.synchronize()
    dt = e0.elapsed_time(e1) / reps / 1e3
    flops = 2.0 * M * N * K
    achieved = flops / dt / 1e12
    peak = peaks.get("bf16_tflops", 1590.0)
    return {"kernel": "gemm_tc2_kernel<SWIGLU,half> 2-SM (FFN gate/up, %dx%dx%d)" % (M, N, K), "bound": "tensor",
            "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
            "peak_source": "MEASURED_PEAKS.json bf16_tflops (burst, cuBLAS)" if "bf16_tflops" in peaks
            else "fallback 1590", "launch_us": round(dt * 1e6, 2), "flop_per_launch": flops,
            # dram__bytes_read.sum + dram__bytes_write.sum of one launch of this GEMM shape (ncu, 1-SM kernel):
            # = the algorithmic A + B bytes, no re-reads
            "traffic": 34637056 + 26368, "traffic_unit": "bytes/launch"}


DIT_WORKLOAD = "sao_bf16_1x1024"
# dram__bytes_read.sum + dram__bytes_write.sum of one out-projection launch of that GEMM (ncu, one launch;
# on the C3 workload): A 6.3 MB + W 4.7 MB + residual 12.6 MB read, i.e. no re-reads
RESID_TRAFFIC_DIT = 23680000


def gemm_time(b2d, ctx, torch, M, N, K, epilogue, bn=256, bf16=False, reps=30):
    """Average device time of one tcgen05 GEMM launch (CUDA events on the launching stream)."""
    dt = torch.bfloat16 if bf16 else torch.float16
    a = torch.randn(M, K, device="cuda").to(dt)
    w = (torch.randn(N, K, device="cuda") * 0.02).to(dt)
    out = torch.zeros(M, N, device="cuda")
    bias = torch.zeros(N, device="cuda")
    st = torch.cuda.current_stream()
    ldo = N // 2 if epilogue == b2d.EPI_SWIGLU else N
    if epilogue == b2d.EPI_RESID:  # x[M, N] += acc + bias, fp32 residual stream read and written in place
        launch = lambda: ctx.gemm(a.data_ptr(), w.data_ptr(), M, N, K, bf16=bf16, epilogue=epilogue, bn=bn,
                                  bias=bias.data_ptr(), resid=out.data_ptr(), ldr=N, stream=st.cuda_stream)
    else:
        launch = lambda: ctx.gemm(a.data_ptr(), w.data_ptr(), M, N, K, bf16=bf16, epilogue=epilogue, bn=bn,
                                  out=out.data_ptr(), ldo=ldo, stream=st.cuda_stream)
    for _ in range(3):
        launch()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        launch()
    e1.record(st)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps / 1e3


def bench_dit(args, torch, b2d, ctx, world, rank, timed, peaks):
    """C3: Stable-Audio-Open-1.0 DiT, BF16, 1 prompt + CFG (2 sequences) x 1024 frames, 100-step DPM++ 2M,
    CFG 7, APG 1.  Per rank its own prompt (weak scaling).  Metric: sequence-steps/s over all ranks."""
    from oracle import synth
    cfg = synth.DIT_CONFIGS[DIT_WORKLOAD]
    w = node_shared(synth.dit_weights, cfg)  # the same weights on every rank
    cfg = synth.DitConfig(**{**cfg.__dict__, "prompt_seeds": (rank,)})
    if args.dit_dpm_steps:  # profiling only: shorter schedules (the reported config says so)
        cfg = synth.DitConfig(**{**cfg.__dict__, "steps": args.dit_dpm_steps})
    gt = {0: 0, 1: 1, 3: 8, 2: 30}
    dit = b2d.StableAudioDiT(ctx, cfg.embed_dim, cfg.depth, cfg.num_heads, cfg.cond_token_dim, cfg.global_cond_dim,
                             cfg.io_channels, cfg.prompt_max_length,
                             weights=[(n, gt[t.dtype], t.dims, t.data) for n, t in w.items()])
    del w
    inp = synth.dit_inputs(cfg)
    keys = ("noise", "padding_mask", "cross_positive", "cross_negative", "global")
    dev = [torch.from_numpy(inp[k].array().copy()).cuda() for k in keys]
    host = [torch.from_numpy(inp[k].array().copy()).pin_memory() for k in keys]
    out_dev = torch.empty_like(dev[0])
    out_host = torch.empty(dev[0].shape).pin_memory()
    st = torch.cuda.current_stream()
    kw = dict(steps=cfg.steps, sigma_min=cfg.sigma_min, sigma_max=cfg.sigma_max, rho=cfg.rho, cfg_scale=cfg.cfg,
              apg_scale=cfg.apg, stream=st.cuda_stream)
    calls, warm = max(1, min(args.steps, args.dit_steps)), max(1, min(args.warmup, args.dit_warmup))
    ms = timed(lambda: dit.sample_device(*dev, out_dev, **kw), calls, warm)
    ctx.sync(st.cuda_stream)
    ms_e2e = timed(lambda: dit.sample(*host, out=out_host, **kw), calls, 1)
    seq_steps = 2 * cfg.batch * cfg.steps * world
    res = {"metric": "denoise sequence-steps/sec (DiT)", "value": round(seq_steps / (ms / 1e3), 2),
           "unit": "seq-steps/s", "ms_per_call": round(ms, 2), "timed_calls": calls, "warmup_calls": warm,
           "prompt_steps_per_s": round(seq_steps / 2 / (ms / 1e3), 2),
           "config": {"workload": DIT_WORKLOAD, "model": "Stable-Audio-Open-1.0-shaped DiT (random-init)",
                      "weights": cfg.wtype, "sequences_per_rank": 2 * cfg.batch, "tokens": cfg.latent_tokens + 1,
                      "dpm_steps": cfg.steps, "cfg_scale": cfg.cfg, "apg_scale": cfg.apg, "n_gpus": world},
           "dtype": "bf16 tensor-core operands, fp32 accumulate",
           "e2e": {"value": round(seq_steps / (ms_e2e / 1e3), 2), "unit": "seq-steps/s",
                   "h2d_bytes_per_step": sum(t.numel() * 4 for t in host), "d2h_bytes_per_step": out_host.numel() * 4,
                   "api": "b2d_dit_sample (host buffers, pinned)"},
           "gpu_launches_per_call": 14 + cfg.steps * (4 + cfg.depth * 11) + 2 * cfg.steps,
           "whole_call_tflops": round(2 * cfg.batch * cfg.steps * 2.264e12 / (ms / 1e3) / 1e12, 1)}
    assert np.isfinite(out_host.numpy()).all()
    if rank == 0:
        R = 2 * cfg.batch * (cfg.latent_tokens + 1)
        # The dominant kernel of the DiT step (largest device-time share in the launch list): the gated-residual GEMM
        # gemm_tc_kernel<192, RESID>, launched three times per layer -- self-attention out (K = d), cross-attention
        # out (K = d) and FF out (K = 4d), each x += acc + b on the fp32 residual stream.  Reported over those three
        # launches: their FLOPs / their summed event time.
        d = cfg.embed_dim
        t_o = gemm_time(b2d, ctx, torch, R, d, d, b2d.EPI_RESID, bn=192, bf16=True)
        t_f = gemm_time(b2d, ctx, torch, R, d, 4 * d, b2d.EPI_RESID, bn=192, bf16=True)
        fl = 2.0 * R * d * d * 2 + 2.0 * R * d * 4 * d
        t = 2 * t_o + t_f
        peak = peaks.get("bf16_tflops", 1590.0)
        res["roofline"] = {"kernel": "gemm_tc_kernel<192,RESID,bf16> (out-proj %dx%dx%d x2, FF-out %dx%dx%d)"
                                     % (R, d, d, R, d, 4 * d),
                           "bound": "tensor", "achieved": round(fl / t / 1e12, 1), "peak": peak,
                           "unit": "TFLOP/s", "frac": round(fl / t / 1e12 / peak, 4),
                           "launch_us": {"out_proj": round(t_o * 1e6, 2), "ff_out": round(t_f * 1e6, 2)},
                           "flop_per_layer": fl,
                           "traffic": RESID_TRAFFIC_DIT,
                           "traffic_unit": "bytes per out-projection launch (ncu); algorithmic 23.6 MB"}
        t_ff = gemm_time(b2d, ctx, torch, R, 8 * d, d, b2d.EPI_SWIGLU, bn=512, bf16=True)
        fl_ff = 2.0 * R * 8 * d * d
        res["ffn_in_gemm"] = {"kernel": "gemm_tc2_kernel<SWIGLU,bf16> 2-SM (FFN in, %dx%dx%d)" % (R, 8 * d, d),
                              "achieved": round(fl_ff / t_ff / 1e12, 1), "unit": "TFLOP/s",
                              "frac": round(fl_ff / t_ff / 1e12 / peak, 4)}
        if not args.no_cpu_baseline and world == 1:
            from oracle import ref_runner
            if ref_runner.available():
                c1 = synth.DitConfig(**{**cfg.__dict__, "steps": 1})
                o = ref_runner.run("dit", synth.dit_inputs(c1), synth.dit_weights(c1), reps=1)
                cms = float(o["wall_ms"].data[0])
                res["cpu_baseline"] = {"value": round(2 * cfg.batch / (cms / 1e3), 4), "unit": "seq-steps/s",
                                       "cores": os.cpu_count(), "kind": "reference",
                                       "sample": "1 DPM++ step of the 2-sequence C3 workload, audio.cpp ggml CPU (%s)"
                                                 % ref_runner.variant()}
    return res


SA3_WORKLOAD = "sa3_bench_bf16"


def bench_sa3(args, torch, b2d, ctx, world, rank, timed):
    """Stable Audio 3 DiT (the first row after the head and the SAO DiT): BF16, 1 prompt + CFG (2 sequences)
    x (64 memory + 2584 latent) tokens, 8 pingpong steps, CFG 7, APG 1.  Per rank its own prompt (weak
    scaling).  Metric: sequence-steps/s over all ranks."""
    from oracle import synth
    cfg = synth.SA3_CONFIGS[SA3_WORKLOAD]
    if args.small:  # profiling only: a shape an ncu capture finishes (the reported config says so)
        cfg = synth.Sa3Config(**{**cfg.__dict__, "latent_tokens": 448, "steps": 2})
    w = node_shared(synth.sa3_weights, cfg)  # the same weights on every rank
    cfg = synth.Sa3Config(**{**cfg.__dict__, "prompt_seeds": (rank,)})
    gt = {0: 0, 1: 1, 3: 8, 2: 30}
    model = b2d.StableAudio3DiT(ctx, cfg.embed_dim, cfg.depth, cfg.num_heads, cfg.cond_dim, cfg.global_cond_dim,
                                cfg.local_add_cond_dim, cfg.num_memory_tokens, cfg.prompt_max_length,
                                cfg.differential, cfg.io_channels,
                                weights=[(n, gt[t.dtype], t.dims, t.data) for n, t in w.items()])
    if rank != 0 or args.no_cpu_baseline:
        del w
    inp = synth.sa3_inputs(cfg)
    keys = ("noise", "padding_mask", "schedule", "cross_positive", "cross_negative", "negative_mask", "global",
            "local_add")
    dev = [torch.from_numpy(inp[k].array().copy()).cuda() for k in keys]
    host = [torch.from_numpy(inp[k].array().copy()).pin_memory() for k in keys]
    out_dev = torch.empty_like(dev[0])
    out_host = torch.empty(dev[0].shape).pin_memory()
    st = torch.cuda.current_stream()
    kw = dict(cfg_scale=cfg.cfg, apg_scale=cfg.apg, sampler=cfg.sampler, seed=cfg.seed,
              rng_policy=(cfg.rng_sms, cfg.rng_max_threads), stream=st.cuda_stream)
    calls, warm = max(1, min(args.steps, 5)), max(3, min(args.warmup, 3))
    ms = timed(lambda: model.sample_device(*dev, out_dev, **kw), calls, warm)
    ctx.sync(st.cuda_stream)
    ms_e2e = timed(lambda: model.sample(*host, out=out_host, **kw), calls, 1)
    seq_steps = 2 * cfg.batch * cfg.steps * world
    L1 = cfg.num_memory_tokens + cfg.latent_tokens
    d = cfg.embed_dim
    # per sequence-step: projections 2 L1 d (3d + d + d + d + 8d + 4d) + attention 4 L1 (L1 + P1) d; local-add and
    # the cross K/V are step-invariant and computed once per call
    fl = 2 * L1 * d * 18 * d + 4 * L1 * (L1 + cfg.prompt_max_length + 1) * d
    res = {"metric": "denoise sequence-steps/sec (SA3 DiT)", "value": round(seq_steps / (ms / 1e3), 2),
           "unit": "seq-steps/s", "ms_per_call": round(ms, 2), "timed_calls": calls, "warmup_calls": warm,
           "config": {"workload": SA3_WORKLOAD + ("_small" if args.small else ""),
                      "model": "Stable-Audio-3-layout DiT at SAO-1.0 transformer size (random-init)",
                      "weights": cfg.wtype, "sequences_per_rank": 2 * cfg.batch, "tokens": L1,
                      "steps": cfg.steps, "sampler": cfg.sampler, "cfg_scale": cfg.cfg, "apg_scale": cfg.apg,
                      "differential_attention": cfg.differential, "n_gpus": world},
           "dtype": "bf16 tensor-core operands, fp32 accumulate",
           "e2e": {"value": round(seq_steps / (ms_e2e / 1e3), 2), "unit": "seq-steps/s",
                   "h2d_bytes_per_step": sum(t.numel() * 4 for t in host), "d2h_bytes_per_step": out_host.numel() * 4,
                   "api": "b2d_sa3_sample (host buffers, pinned)"},
           "gpu_launches_per_call": 18 + 5 * cfg.depth + cfg.steps * (7 + 14 * cfg.depth),
           "whole_call_tflops": round(seq_steps / world * cfg.depth * fl / (ms / 1e3) / 1e12, 1)}
    assert np.isfinite(out_host.numpy()).all()
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        from oracle import ref_runner
        if ref_runner.available():
            c1 = synth.Sa3Config(**{**cfg.__dict__, "steps": 1})
            o = ref_runner.run("sa3", synth.sa3_inputs(c1), w, reps=1)
            cms = float(o["wall_ms"].data[0])
            res["cpu_baseline"] = {"value": round(2 * cfg.batch / (cms / 1e3), 4), "unit": "seq-steps/s",
                                   "cores": os.cpu_count(), "kind": "reference",
                                   "sample": "1 pingpong step of the 2-sequence SA3 workload, audio.cpp ggml CPU (%s)"
                                             % ref_runner.variant()}
    return res


OOBLECK_WORKLOAD = "oobleck_bench_sao_1x1024"


def bench_oobleck(args, torch, b2d, ctx, world, rank, timed):
    """Oobleck VAE decode at the SAO-1.0 shape: 1024 latents -> 2,097,152 stereo frames per rank (weak scaling).
    Metric: decoded audio frames/s over all ranks."""
    from oracle import synth
    cfg = synth.OOBLECK_CONFIGS[OOBLECK_WORKLOAD]
    if args.small:  # profiling only: 128 latents (262,144 frames), activations still larger than L2
        cfg = synth.OobleckConfig(**{**cfg.__dict__, "latent_tokens": 128})
    w = node_shared(synth.oobleck_weights, cfg)
    dec = b2d.OobleckDecoder(ctx, cfg.latent_dim, cfg.channels, cfg.c_mults, cfg.strides, cfg.audio_channels,
                             weights=[(n, 0, t.dims, t.data) for n, t in w.items()])
    lat = synth.oobleck_inputs(synth.OobleckConfig(**{**cfg.__dict__, "seed": cfg.seed + rank}))["latents"].array()
    frames = cfg.latent_tokens * int(np.prod(cfg.strides))
    d_lat = torch.from_numpy(lat.copy()).cuda()
    d_out = torch.empty((cfg.batch, frames, cfg.audio_channels), dtype=torch.float32, device="cuda")
    h_lat = torch.from_numpy(lat.copy()).pin_memory()
    h_out = torch.empty((cfg.batch, frames, cfg.audio_channels)).pin_memory()
    st = torch.cuda.current_stream()
    calls, warm = max(1, min(args.steps, 5)), 3
    ms = timed(lambda: dec.decode_device(d_lat, d_out, stream=st.cuda_stream), calls, warm)
    ctx.sync(st.cuda_stream)
    ms_e2e = timed(lambda: dec.decode(h_lat, out=h_out, stream=st.cuda_stream), calls, 1)
    # algorithmic FLOPs: 2 x output rows x Cout x taps x Cin per conv (transposed conv: 2 taps x s phases)
    ch = [cfg.channels * m for m in (1,) + tuple(cfg.c_mults)]
    L, fl = cfg.latent_tokens, 2.0 * cfg.latent_tokens * ch[-1] * 7 * cfg.latent_dim
    for blk in range(len(cfg.strides), 0, -1):
        s, cin, cout = cfg.strides[blk - 1], ch[blk], ch[blk - 1]
        fl += 2.0 * L * s * cout * 2 * cin
        L *= s
        fl += 3 * (2.0 * L * cout * 7 * cout + 2.0 * L * cout * cout)
    fl += 2.0 * L * cfg.audio_channels * 7 * ch[0]
    fl *= cfg.batch
    total = frames * cfg.batch * world
    res = {"metric": "decoded audio frames/sec (Oobleck VAE)", "value": round(total / (ms / 1e3), 1),
           "unit": "frames/s", "ms_per_call": round(ms, 3), "timed_calls": calls, "warmup_calls": warm,
           "realtime_factor_44k1": round(total / (ms / 1e3) / 44100.0, 1),
           "config": {"workload": OOBLECK_WORKLOAD + ("_small" if args.small else ""), "model": "Stable-Audio-Open-1.0-shaped Oobleck decoder (random-init)",
                      "latent_tokens": cfg.latent_tokens, "frames": frames, "channels": ch, "strides": cfg.strides,
                      "n_gpus": world},
           "dtype": "fp16 tensor-core operands, fp32 accumulate and residual stream",
           "e2e": {"value": round(total / (ms_e2e / 1e3), 1), "unit": "frames/s",
                   "h2d_bytes_per_step": h_lat.numel() * 4, "d2h_bytes_per_step": h_out.numel() * 4,
                   "api": "b2d_oobleck_decode (host buffers, pinned)"},
           "gpu_launches_per_call": 4 + 7 * len(cfg.strides),
           "whole_call_tflops": round(fl / (ms / 1e3) / 1e12, 1)}
    assert np.isfinite(h_out.numpy()).all()
    if rank == 0 and not args.no_cpu_baseline and world == 1:
        from oracle import ref_runner
        if ref_runner.available():
            c1 = synth.OobleckConfig(**{**cfg.__dict__, "latent_tokens": 16})
            o = ref_runner.run("oobleck", synth.oobleck_inputs(c1), w, reps=1)
            cms = float(o["wall_ms"].data[0])
            f1 = 16 * int(np.prod(cfg.strides))
            res["cpu_baseline"] = {"value": round(f1 / (cms / 1e3), 1), "unit": "frames/s",
                                   "cores": os.cpu_count(), "kind": "reference",
                                   "sample": "16 of the 1024 latents (%d frames), audio.cpp ggml CPU (%s)"
                                             % (f1, ref_runner.variant())}
    return res


def _parallel_module():
    spec = importlib.util.spec_from_file_location("b2d_parallel", os.path.join(ROOT, "audio.cpp_b200", "parallel.py"))
    par = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(par)
    return par


GT = {0: 0, 1: 1, 3: 8, 2: 30}  # bundle dtype -> ggml type id


def head_weight_bytes_per_step(cfg, bytes_per_weight=2.0):
    """Weights one denoising step must stream: every layer's adaLN [3H, H], gate/up [F, H], down [H, F], the final
    adaLN [2H, H], final linear [64, H] and noisy_images_proj [H, 64] (cond_proj and the timestep MLP are once per
    call), at the resident operand width."""
    H, F, L = cfg.hidden, cfg.ffn, cfg.latent
    return bytes_per_weight * (cfg.layers * (3 * H * H + 3 * F * H) + 2 * H * H + 2 * L * H)


def bench_c1(args, torch, b2d, ctx, world, rank, timed, peaks):
    """C1: VibeVoice-1.5B head, F16 weights, 64 frames (128 head rows), 10 steps, CFG 1.3.  Weight streaming:
    judged on weight bytes per call against the measured HBM copy bandwidth.  Per rank its own 64 frames."""
    from oracle import synth
    cfg = synth.HEAD_CONFIGS[C1_WORKLOAD]
    w = node_shared(synth.head_weights, cfg)
    inp = synth.head_inputs(synth.HeadConfig(**{**cfg.__dict__, "cseed": 1 + 100 * rank, "xseed": 2 + 100 * rank}))
    head = b2d.VibeVoiceDiffusionHead(ctx, cfg.hidden, cfg.layers, cfg.ffn_ratio,
                                      weights=[(n, GT[t.dtype], t.dims, t.data) for n, t in w.items()])
    del w
    keys = ("positive_condition", "negative_condition", "initial_speech")
    dev = [torch.from_numpy(inp[k].array().copy()).cuda() for k in keys]
    host = [torch.from_numpy(inp[k].array().copy()).pin_memory() for k in keys]
    out_dev = torch.empty(cfg.frames, 64, device="cuda")
    out_host = torch.empty(cfg.frames, 64).pin_memory()
    st = torch.cuda.current_stream()
    ms = timed(lambda: head.sample_device(*dev, cfg.steps, cfg.cfg, out_dev, stream=st.cuda_stream), 20, 5)
    ctx.sync(st.cuda_stream)
    ms_e2e = timed(lambda: head.sample(*host, cfg.steps, cfg.cfg, out=out_host, stream=st.cuda_stream), 20, 3)
    assert np.isfinite(out_host.numpy()).all()
    wbytes = head_weight_bytes_per_step(cfg) * cfg.steps + 2.0 * (cfg.hidden * cfg.hidden + cfg.hidden * 256 +
                                                                  cfg.hidden * cfg.hidden)
    peak = peaks.get("hbm_gbs", 6650.0)
    ach = wbytes / (ms / 1e3) / 1e9
    frames = cfg.frames * world
    res = {"metric": "latent frames/sec (VibeVoice diffusion head, C1 weight streaming)",
           "value": round(frames / (ms / 1e3), 1), "unit": "frames/s", "ms_per_call": round(ms, 4),
           "timed_calls": 20, "warmup_calls": 5,
           "config": {"workload": C1_WORKLOAD, "model": "VibeVoice-1.5B diffusion head (random-init)",
                      "weights": "f16", "frames_per_rank": cfg.frames, "head_rows_per_rank": 2 * cfg.frames,
                      "dpm_steps": cfg.steps, "cfg_scale": cfg.cfg, "n_gpus": world},
           "dtype": "f16 tensor-core operands, fp32 accumulate",
           "e2e": {"value": round(frames / (ms_e2e / 1e3), 1), "unit": "frames/s",
                   "h2d_bytes_per_step": sum(t.numel() * 4 for t in host), "d2h_bytes_per_step": out_host.numel() * 4,
                   "api": "b2d_vv_sample (host buffers, pinned)"},
           "roofline": {"kernel": "whole sampling call (weight stream)", "bound": "hbm", "achieved": round(ach, 1),
                        "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
                        "algorithmic_bytes_per_call": wbytes,
                        "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback 6650"}}
    return res


def bench_c5(args, torch, b2d, ctx, world, rank, timed, peaks):
    """C5: VibeVoice-7B-shaped head (H 3584), Q8_0, 8192 frames split over the ranks (strong scaling: the job is
    fixed), 10 steps, CFG 1.3, plus the final gather of all latents to every rank inside the timed region."""
    from oracle import synth
    par = _parallel_module()
    cfg = synth.HEAD_CONFIGS["vv7_q8_8192"]
    w = node_shared(synth.head_weights, cfg)
    head = b2d.VibeVoiceDiffusionHead(ctx, cfg.hidden, cfg.layers, cfg.ffn_ratio,
                                      weights=[(n, GT[t.dtype], t.dims, t.data) for n, t in w.items()])
    del w
    inp = synth.head_inputs(cfg)
    pos, neg, init, (lo, hi) = par.shard_head_inputs(inp["positive_condition"].array(),
                                                     inp["negative_condition"].array(),
                                                     inp["initial_speech"].array(), world, rank)
    del inp
    n = hi - lo
    dev = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (pos, neg, init)]
    host = [torch.from_numpy(np.ascontiguousarray(a)).pin_memory() for a in (pos, neg, init)]
    out_dev = torch.empty(n, 64, device="cuda")
    out_host = torch.empty(n, 64).pin_memory()
    st = torch.cuda.current_stream()

    def job():
        head.sample_device(*dev, cfg.steps, cfg.cfg, out_dev, stream=st.cuda_stream)
        return par.gather_rows(out_dev, cfg.frames, world)

    def job_e2e():
        return head.sample(*host, cfg.steps, cfg.cfg, out=out_host, stream=st.cuda_stream)

    calls = 5
    ms = timed(job, calls, 2)
    ctx.sync(st.cuda_stream)
    ms_e2e = timed(job_e2e, calls, 1)
    full = job()
    assert full.shape == (cfg.frames, 64) and bool(torch.isfinite(full).all())
    fl = 2.0 * cfg.frames * cfg.steps * (100 * cfg.hidden ** 2 + 256 * cfg.hidden)
    peak = peaks.get("bf16_tflops", 1590.0)
    tf = fl / (ms / 1e3) / 1e12 / world
    return {"metric": "latent frames/sec (VibeVoice-7B head, C5 strong scaling)",
            "value": round(cfg.frames / (ms / 1e3), 1), "unit": "frames/s", "ms_per_call": round(ms, 3),
            "timed_calls": calls, "warmup_calls": 2, "scaling": "strong",
            "config": {"workload": "vv7_q8_8192", "model": "VibeVoice-7B-shaped diffusion head (random-init)",
                       "weights": "q8_0", "hidden": cfg.hidden, "global_frames": cfg.frames,
                       "frames_per_rank": n, "dpm_steps": cfg.steps, "cfg_scale": cfg.cfg, "n_gpus": world,
                       "parallelism": "dp%d (frames sharded, CFG pairs kept per rank; one all_gather timed)" % world},
            "dtype": "f16 tensor-core operands (Q8_0 dequantised), fp32 accumulate",
            "e2e": {"value": round(cfg.frames / (ms_e2e / 1e3), 1), "unit": "frames/s",
                    "h2d_bytes_per_step": sum(t.numel() * 4 for t in host), "d2h_bytes_per_step": n * 64 * 4,
                    "api": "b2d_vv_sample (host buffers, pinned), each rank its shard (no gather)"},
            "per_gpu_tflops": round(tf, 1), "per_gpu_frac_of_bf16_peak": round(tf / peak, 4)}


def bench_c4(args, torch, b2d, ctx, world, rank, timed, peaks):
    """C4: SAO-1.0 DiT, Q8_0, 16 prompts (seeds 0-15) + CFG = 32 sequences x 1025 tokens, 100 DPM++ 2M steps,
    prompts split over the ranks (strong scaling), plus the final gather of all latents inside the timed region."""
    from oracle import synth
    par = _parallel_module()
    cfg = synth.DIT_CONFIGS["sao_q8_16x1024"]
    if args.dit_dpm_steps:
        cfg = synth.DitConfig(**{**cfg.__dict__, "steps": args.dit_dpm_steps})
    w = node_shared(synth.dit_weights, cfg)
    dit = b2d.StableAudioDiT(ctx, cfg.embed_dim, cfg.depth, cfg.num_heads, cfg.cond_token_dim, cfg.global_cond_dim,
                             cfg.io_channels, cfg.prompt_max_length,
                             weights=[(n, GT[t.dtype], t.dims, t.data) for n, t in w.items()])
    del w
    inp = synth.dit_inputs(cfg)
    keys = ("noise", "padding_mask", "cross_positive", "cross_negative", "global")
    local, (lo, hi) = par.shard_prompts([inp[k].array() for k in keys], cfg.batch, world, rank)
    dev = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in local]
    host = [torch.from_numpy(np.ascontiguousarray(a)).pin_memory() for a in local]
    out_dev = torch.empty_like(dev[0])
    out_host = torch.empty(dev[0].shape).pin_memory()
    st = torch.cuda.current_stream()
    kw = dict(steps=cfg.steps, sigma_min=cfg.sigma_min, sigma_max=cfg.sigma_max, rho=cfg.rho, cfg_scale=cfg.cfg,
              apg_scale=cfg.apg, stream=st.cuda_stream)

    def job():
        dit.sample_device(*dev, out_dev, **kw)
        return par.gather_rows(out_dev, cfg.batch, world)

    def job_e2e():
        return dit.sample(*host, out=out_host, **kw)

    ms = timed(job, 1, 1)
    ctx.sync(st.cuda_stream)
    ms_e2e = timed(job_e2e, 1, 0)
    full = job()
    assert tuple(full.shape) == (cfg.batch, 64, cfg.latent_tokens) and bool(torch.isfinite(full).all())
    seq_steps = 2 * cfg.batch * cfg.steps
    peak = peaks.get("bf16_tflops", 1590.0)
    tf = seq_steps * 2.264e12 / (ms / 1e3) / 1e12 / world
    return {"metric": "denoise sequence-steps/sec (DiT, C4 strong scaling)",
            "value": round(seq_steps / (ms / 1e3), 2), "unit": "seq-steps/s", "ms_per_call": round(ms, 2),
            "timed_calls": 1, "warmup_calls": 1, "scaling": "strong",
            "prompt_steps_per_s": round(seq_steps / 2 / (ms / 1e3), 2),
            "config": {"workload": "sao_q8_16x1024" + ("_%dsteps" % cfg.steps if args.dit_dpm_steps else ""),
                       "model": "Stable-Audio-Open-1.0-shaped DiT (random-init)", "weights": "q8_0",
                       "prompts": cfg.batch, "prompts_per_rank": hi - lo, "tokens": cfg.latent_tokens + 1,
                       "dpm_steps": cfg.steps, "cfg_scale": cfg.cfg, "apg_scale": cfg.apg, "n_gpus": world,
                       "parallelism": "dp%d (prompt pairs sharded; one all_gather timed)" % world},
            "dtype": "f16 tensor-core operands (Q8_0 dequantised), fp32 accumulate",
            "e2e": {"value": round(seq_steps / (ms_e2e / 1e3), 2), "unit": "seq-steps/s",
                    "h2d_bytes_per_step": sum(t.numel() * 4 for t in host), "d2h_bytes_per_step": out_host.numel() * 4,
                    "api": "b2d_dit_sample (host buffers, pinned), each rank its shard (no gather)"},
            "per_gpu_tflops": round(tf, 1), "per_gpu_frac_of_bf16_peak": round(tf / peak, 4)}


def make_timer(torch, args, world, st):
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda")

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def timed(call, steps, warmup):
        for _ in range(warmup):
            call()
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        total = 0.0
        for _ in range(steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            call()
            e1.record(st)
            e1.synchronize()
            total += e0.elapsed_time(e1)
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        return max_over_ranks(total / steps)
    return timed


def bench_dit_only(args, torch, b2d, world, rank, local):
    """--workload dit / sa3: time only that DiT (used for profiling); prints its result as the line."""
    ctx = b2d.Context(local)
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        peaks = {}
    st = torch.cuda.current_stream()
    with ClockSampler(local) as clk:
        timer = make_timer(torch, args, world, st)
        if args.workload == "sa3":
            res = bench_sa3(args, torch, b2d, ctx, world, rank, timer)
        elif args.workload == "c1":
            res = bench_c1(args, torch, b2d, ctx, world, rank, timer, peaks)
        elif args.workload == "c4":
            res = bench_c4(args, torch, b2d, ctx, world, rank, timer, peaks)
        elif args.workload == "c5":
            res = bench_c5(args, torch, b2d, ctx, world, rank, timer, peaks)
        elif args.workload == "oobleck":
            res = bench_oobleck(args, torch, b2d, ctx, world, rank, timer)
        else:
            res = bench_dit(args, torch, b2d, ctx, world, rank, timer, peaks)
    if rank == 0:
        res.update({"n_gpus": world, "steps": res["timed_calls"], "warmup": res["warmup_calls"],
                    "higher_is_better": True, "scaling": res.get("scaling", "weak"), "vs_baseline": None,
                    "data": "synthetic (seeded random weights and inputs)", "clocks": clk.summary()})
        print(json.dumps(res))
    ctx.close()
    if world > 1:
        torch.distributed.destroy_process_group()


def bench_ours(args):
    import torch
    world, rank, local = dist_setup()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    b2d = load_package()
    from oracle import synth  # seeded synthetic weights/inputs (no checkpoints here)
    cfg = synth.HEAD_CONFIGS[WORKLOAD]
    if args.workload in ("dit", "sa3", "oobleck", "c1", "c4", "c5"):
        return bench_dit_only(args, torch, b2d, world, rank, local)
    w = node_shared(synth.head_weights, cfg)
    inp = synth.head_inputs(synth.HeadConfig(**{**cfg.__dict__, "cseed": 1 + 100 * rank, "xseed": 2 + 100 * rank}))
    gt = {0: 0, 1: 1, 3: 8, 2: 30}
    ctx = b2d.Context(local)
    head = b2d.VibeVoiceDiffusionHead(ctx, cfg.hidden, cfg.layers, cfg.ffn_ratio,
                                      weights=[(n, gt[t.dtype], t.dims, t.data) for n, t in w.items()])
    del w
    st = torch.cuda.current_stream()
    dev = [torch.from_numpy(inp[k].array().copy()).cuda() for k in ("positive_condition", "negative_condition",
                                                                    "initial_speech")]
    host = [torch.from_numpy(inp[k].array().copy()).pin_memory() for k in ("positive_condition",
                                                                            "negative_condition", "initial_speech")]
    out_dev = torch.empty(cfg.frames, 64, device="cuda")
    out_host = torch.empty(cfg.frames, 64).pin_memory()
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda")

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def timed(call, steps=None, warmup=None):
        steps = args.steps if steps is None else steps
        for _ in range(args.warmup if warmup is None else warmup):
            call()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        total = 0.0
        for _ in range(steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            call()
            e1.record(st)
            e1.synchronize()
            total += e0.elapsed_time(e1)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(total / steps)

    dev_call = lambda: head.sample_device(*dev, cfg.steps, cfg.cfg, out_dev, stream=st.cuda_stream)
    host_call = lambda: head.sample(*host, cfg.steps, cfg.cfg, out=out_host, stream=st.cuda_stream)
    with ClockSampler(local) as clk:
        ms = timed(dev_call)
    ctx.sync(st.cuda_stream)
    ms_e2e = timed(host_call)
    assert np.isfinite(out_host.numpy()).all()
    # the one collective of the data-parallel path: gather every rank's latents (outside the timed steps)
    gather_ms = 0.0
    if world > 1:
        import importlib.util
        spec = importlib.util.spec_from_file_location("b2d_parallel", os.path.join(ROOT, "audio.cpp_b200", "parallel.py"))
        par = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(par)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.distributed.barrier()
        g0.record(st)
        full = par.gather_rows(out_dev, cfg.frames * world, world)
        g1.record(st)
        torch.cuda.synchronize()
        gather_ms = max_over_ranks(g0.elapsed_time(g1))
        assert full.shape[0] == cfg.frames * world

    frames_total = cfg.frames * world
    value = frames_total / (ms / 1e3)
    e2e = frames_total / (ms_e2e / 1e3)
    h2d = sum(t.numel() * 4 for t in host)
    d2h = out_host.numel() * 4
    launches_per_call = 5 + cfg.steps * (3 * cfg.layers + 6)

    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        peaks = {}
    dit_res = None
    if args.workload in ("all", "dit"):
        dit_res = bench_dit(args, torch, b2d, ctx, world, rank, timed, peaks)
    extra = {}
    if args.workload == "all":
        extra["sa3"] = bench_sa3(args, torch, b2d, ctx, world, rank, timed)
        extra["oobleck"] = bench_oobleck(args, torch, b2d, ctx, world, rank, timed)
        extra["c1"] = bench_c1(args, torch, b2d, ctx, world, rank, timed, peaks)
        extra["c5"] = bench_c5(args, torch, b2d, ctx, world, rank, timed, peaks)
        if not args.no_c4:
            extra["c4"] = bench_c4(args, torch, b2d, ctx, world, rank, timed, peaks)
    if rank == 0:
        roof = gemm_roofline(b2d, ctx, torch, cfg, peaks)
        flops_call = 2.0 * cfg.frames * cfg.steps * (100 * cfg.hidden ** 2 + 256 * cfg.hidden)
        line = {"metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f16 tensor-core operands (Q8_0 dequantised), fp32 accumulate",
                "data": "synthetic (seeded random weights and inputs)",
                "config": config_json(cfg, world),
                "e2e": {"value": round(e2e, 1), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                        "ms_per_step": round(ms_e2e, 4), "api": "b2d_vv_sample (host buffers, pinned)"},
                "gpu_launches": launches_per_call * args.steps,
                "final_gather_ms": round(gather_ms, 4),
                "roofline": roof,
                "whole_call_tflops": round(flops_call / (ms / 1e3) / 1e12, 1),
                "clocks": clk.summary()}
        if not args.no_cpu_baseline and world == 1:
            frames = cfg.frames  # the whole 1024-frame call, as the GPU arm runs it
            cms, variant = run_cpu_reference(cfg, frames, 4, os.cpu_count() or 1)
            v = frames / (float(np.median(cms[1:])) / 1e3)
            line["cpu_baseline"] = {"value": round(v, 2), "unit": UNIT, "cores": os.cpu_count(), "kind": "reference",
                                    "sample": "the full %d-frame call, 10 DPM steps + CFG, audio.cpp ggml CPU (%s), "
                                              "1 warm-up + median of 3 timed calls" % (frames, variant)}
        if dit_res is not None:
            line["dit"] = dit_res
        line.update(extra)
        print(json.dumps(line))
    ctx.close()
    if world > 1:
        torch.distributed.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="all", choices=["all", "head", "dit", "sa3", "oobleck", "c1", "c4", "c5"],
                    help="all = head line (C2) with the C3 DiT, SA3, Oobleck, C1, C5 and C4 results attached; "
                         "head = VibeVoice head only; dit / sa3 / oobleck / c1 / c4 / c5 = only that workload")
    ap.add_argument("--no-c4", action="store_true", help="leave the C4 leg (16-prompt Q8_0 DiT) out of 'all'")
    ap.add_argument("--dit-steps", type=int, default=3, help="timed DiT sampling calls (each 100 DPM++ steps)")
    ap.add_argument("--dit-dpm-steps", type=int, default=0,
                    help="profiling only: DPM++ steps per DiT call instead of the workload's 100")
    ap.add_argument("--dit-warmup", type=int, default=1)
    ap.add_argument("--small", action="store_true",
                    help="profiling only: smaller SA3 / Oobleck shapes that an ncu capture can finish")
    ap.add_argument("--gpu-baseline", action="store_true",
                    help="time the reference's own ggml-cuda backend (oracle/_ref/b2d_ref_cuda) on C2 and C3 instead")
    args = ap.parse_args()
    if args.gpu_baseline:
        bench_ggml_cuda(args)
    elif args.impl == "reference":
        bench_reference(args)
    else:
        bench_ours(args)


if __name__ == "__main__":
    main()
