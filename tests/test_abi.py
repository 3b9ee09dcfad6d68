"""CPU tests of the C ABI library: it loads, exports every symbol include/b200diff.h
declares, and its host-only scheduler matches the reference golden vectors."""
import os
import re

import numpy as np
import pytest

from oracle import vibevoice as V
from tests.helpers import golden

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "b200diff.h")).read()
    return sorted(set(re.findall(r"B2D_API\s+[\w\s\*]+?\b(b2d_\w+)\s*\(", src)))


def test_header_and_library_agree(b2d):
    names = declared_symbols()
    assert len(names) >= 10
    L = b2d.lib()
    for n in names:
        assert hasattr(L, n), "library does not export %s" % n
    assert sorted(b2d.EXPORTED) == names
    assert "sm_100a" in b2d.version()


def test_create_without_gpu_fails_cleanly(b2d):
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    with pytest.raises(b2d.B2DError):
        b2d.Context(0)


@pytest.mark.parametrize("steps", [1, 2, 3, 5, 10, 20, 50, 100])
def test_schedule_matches_reference(b2d, steps):
    g = golden("sched_%d" % steps)
    sched = b2d.vv_schedule(1000, steps)
    assert [float(s.timestep) for s in sched] == list(g["timesteps"].data)
    # apply the coefficients exactly as the device kernel does
    outs, x = g["model_outputs"].array(), g["sample"].array().astype(np.float32)
    prev = None
    ref = g["trace"].array()
    for i, s in enumerate(sched):
        conv = (np.float32(s.alpha_s) * x - np.float32(s.sigma_s) * outs[i]).astype(np.float32)
        if s.order == 1:
            x = (np.float32(s.sample_coeff) * x + np.float32(s.d0_coeff) * conv).astype(np.float32)
        else:
            d1 = (np.float32(s.inv_r0) * (conv - prev)).astype(np.float32)
            x = (np.float32(s.sample_coeff) * x + np.float32(s.d0_coeff) * conv
                 + np.float32(0.5) * np.float32(s.d0_coeff) * d1).astype(np.float32)
        prev = conv
        np.testing.assert_allclose(x, ref[i], rtol=1e-6, atol=1e-6)
    assert sched[0].order == 1 and sched[-1].order == 1
    assert all(s.order == 2 for s in sched[1:-1])
    assert sched[-1].sigma_next == 0.0


def test_schedule_equals_port_coefficients(b2d):
    s = V.Scheduler(1000)
    s.set_timesteps(10)
    lib = b2d.vv_schedule(1000, 10)
    for i, c in enumerate(lib):
        sc, d0, inv = s.coefficients(i, c.order)
        assert np.isclose(c.sample_coeff, sc, rtol=1e-6) and np.isclose(c.d0_coeff, d0, rtol=1e-6)


def test_schedule_rejects_bad_counts(b2d):
    with pytest.raises(b2d.B2DError):
        b2d.vv_schedule(1000, 0)
