"""Runs the reference's own CPU implementation (oracle/_ref/b2d_ref_<isa>, built by
oracle/ref/Makefile from audio.cpp's sources) on B2DB bundles (TEST ORACLE / CPU baseline).

The binary is picked by the host's ISA (or forced with B2D_REF_VARIANT): ``spr`` (AMX + AVX-512 BF16/VNNI),
``v4`` (AVX-512) or ``v3`` (AVX2/FMA/F16C), the first one whose CPU flags are
all present.  ``available()`` is False when none is built.
"""
from __future__ import annotations

import os
import subprocess
import tempfile
from typing import Dict, Optional

from . import bundle as B

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

_REQUIRED = {
    "spr": {"amx_tile", "amx_int8", "amx_bf16", "avx512f", "avx512bw", "avx512vl", "avx512_vnni", "avx512_bf16",
            "avx512_fp16", "avx_vnni"},
    "v4": {"avx512f", "avx512bw", "avx512vl", "avx512dq", "avx512cd", "avx2", "fma", "f16c"},
    "v3": {"avx2", "fma", "f16c", "bmi2"},
}


def _cpu_flags() -> set:
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.startswith("flags"):
                    return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


def binary() -> Optional[str]:
    flags = _cpu_flags()
    forced = os.environ.get("B2D_REF_VARIANT")
    for variant in ((forced,) if forced else ("spr", "v4", "v3")):
        path = os.path.join(REF_DIR, "b2d_ref_" + variant)
        if os.path.exists(path) and _REQUIRED[variant] <= flags:
            return path
    return None


def available() -> bool:
    return binary() is not None


def variant() -> Optional[str]:
    b = binary()
    return None if b is None else os.path.basename(b).split("_")[-1]


def dropin_binary() -> Optional[str]:
    """The harness linked with the B200 drop-in translation units instead of the reference's diffusion head,
    sampler and foundation DiT (oracle/ref/Makefile target ``dropin``); needs a B200 to run."""
    path = os.path.join(REF_DIR, "b2d_ref_dropin")
    return path if os.path.exists(path) else None


def cuda_binary() -> Optional[str]:
    """The harness built with the vendored ggml-cuda backend for sm_100a (oracle/ref/Makefile VARIANT=cuda): the
    reference's own GPU code path, run with B2D_REF_BACKEND=cuda as a timing comparison point."""
    path = os.path.join(REF_DIR, "b2d_ref_cuda")
    return path if os.path.exists(path) else None


def run(cmd: str, inputs: Dict[str, B.Tensor], weights: Optional[Dict[str, B.Tensor]] = None,
        threads: int = 0, reps: int = 1, weights_path: Optional[str] = None, timeout: float = 3600,
        exe: Optional[str] = None, env: Optional[Dict[str, str]] = None) -> Dict[str, B.Tensor]:
    exe = exe or binary()
    if exe is None:
        raise RuntimeError("reference CPU build not found under oracle/_ref (run oracle/ref/Makefile)")
    threads = threads or os.cpu_count() or 1
    with tempfile.TemporaryDirectory(prefix="b2dref") as tmp:
        inp, out = os.path.join(tmp, "in.b2db"), os.path.join(tmp, "out.b2db")
        B.write(inp, inputs)
        args = [exe, cmd]
        if cmd in ("vvpredict", "vv", "dit", "dit_fresh", "sa3", "oobleck", "vvdec", "saocond", "vvlm"):
            if weights_path is None:
                weights_path = os.path.join(tmp, "w.b2db")
                B.write(weights_path, weights)
            args += [weights_path, inp, out, str(threads)]
            if cmd != "vvpredict":
                args.append(str(reps))
        else:
            args += [inp, out]
        proc = subprocess.run(args, capture_output=True, text=True, timeout=timeout,
                              env=None if env is None else {**os.environ, **env})
        if proc.returncode != 0:
            raise RuntimeError("reference harness failed (%d): %s" % (proc.returncode, proc.stderr[-2000:]))
        return B.read(out)
