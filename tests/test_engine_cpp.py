"""Runs the C++ tests of the audio.cpp-facing classes (audio.cpp_b200/host/test_engine.cpp):
the scheduler against the reference vectors on CPU, and the head / DiT / SA3 runtimes on the GPU."""
import os
import subprocess

import pytest

from oracle import bundle as B
from oracle import synth
from tests.helpers import GOLDEN

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "audio.cpp_b200", "test_engine")


def _run(*args):
    if not os.path.exists(EXE):
        pytest.fail("audio.cpp_b200/test_engine is not built (python audio.cpp_b200/build.py)")
    p = subprocess.run([EXE, *args], capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stdout + p.stderr
    return p.stdout


def test_cpp_scheduler_vs_reference():
    _run("sched", GOLDEN)


@pytest.mark.gpu
def test_cpp_head_runtime(tmp_path):
    cfg = synth.HEAD_CONFIGS["tiny_q8"]
    B.write(str(tmp_path / "w.b2db"), synth.head_weights(cfg))
    B.write(str(tmp_path / "in.b2db"), synth.head_inputs(cfg))
    print(_run("head", str(tmp_path / "w.b2db"), str(tmp_path / "in.b2db"), os.path.join(GOLDEN, "head_tiny_q8.b2db")))


@pytest.mark.gpu
def test_cpp_dit_runtime(tmp_path):
    cfg = synth.DIT_CONFIGS["tiny_bf16"]
    B.write(str(tmp_path / "w.b2db"), synth.dit_weights(cfg))
    B.write(str(tmp_path / "in.b2db"), synth.dit_inputs(cfg))
    print(_run("dit", str(tmp_path / "w.b2db"), str(tmp_path / "in.b2db"), os.path.join(GOLDEN, "dit_tiny_bf16.b2db")))


@pytest.mark.gpu
def test_cpp_sa3_runtime(tmp_path):
    cfg = synth.SA3_CONFIGS["sa3_tiny_f32_diff_b2"]
    B.write(str(tmp_path / "w.b2db"), synth.sa3_weights(cfg))
    B.write(str(tmp_path / "in.b2db"), synth.sa3_inputs(cfg))
    print(_run("sa3", str(tmp_path / "w.b2db"), str(tmp_path / "in.b2db"),
               os.path.join(GOLDEN, "sa3_tiny_f32_diff_b2.b2db")))
