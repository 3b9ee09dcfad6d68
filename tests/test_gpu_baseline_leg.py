"""CPU tests of bench.py's reference ggml-cuda comparison leg (--gpu-baseline): without the CUDA build it prints
one 'unavailable' line and exits cleanly; the harness's backend switch is an environment variable that leaves the
CPU variants' default untouched."""
import importlib.util
import io
import json
import os
import contextlib
import types

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("b2d_bench_gpu_baseline", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_gpu_baseline_unavailable_without_cuda_build(monkeypatch):
    from oracle import ref_runner
    monkeypatch.setattr(ref_runner, "cuda_binary", lambda: None)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        monkeypatch.delenv(k, raising=False)
    bench = _bench()
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        bench.bench_ggml_cuda(types.SimpleNamespace(warmup=1, steps=1, dit_steps=1))
    line = json.loads(buf.getvalue().strip().splitlines()[-1])
    assert line["impl"] == "reference-ggml-cuda" and "unavailable" in line


def test_harness_backend_switch_defaults_to_cpu():
    src = open(os.path.join(ROOT, "oracle", "ref", "harness.cpp")).read()
    assert "engine::core::BackendType::Cpu" in src and src.count("ref_backend()") >= 8
    assert 'getenv("B2D_REF_BACKEND")' in src
