"""CPU oracle for the diffusion hot path (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy, the reference's CPU algorithm for the
VibeVoice diffusion head + DPM-Solver++ sampler and the Stable Audio Open 1.0
foundation DiT + DPM++ 2M sampler, and wraps the reference's own CPU build
(``oracle/ref`` -> ``oracle/_ref/b2d_ref_*``) that pins the restatement.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
and ``--impl reference`` legs may import it, and only as the checker / CPU
baseline.  The product path (``audio.cpp_b200``) never imports or calls it.
"""
