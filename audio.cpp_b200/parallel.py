"""Data-parallel sharding for the diffusion hot path: one process per GPU, independent
frames (VibeVoice head) or prompts (DiT) per rank, no collective on the step path,
one gather of the final latents.

audio.cpp itself has no multi-GPU code; this follows the only scale-out it has --
batching independent generations -- across ranks:
* head: frame b's positive / negative condition rows and its initial-speech rows b and
  B + b stay on one rank, because CFG combines them (diffusion_sampler.cpp:35-56);
* DiT: a prompt's cond / uncond sequences stay on one rank, because APG reduces over
  both (rf_dit.cpp:988-1028).
The gather uses torch.distributed (NCCL on GPUs, gloo in the CPU tests).
"""
from __future__ import annotations

from typing import Tuple

import numpy as np


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [lo, hi) share of n units for `rank`; the first n % world ranks get one extra."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("invalid rank %d of %d" % (rank, world))
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard_head_inputs(pos: np.ndarray, neg: np.ndarray, init: np.ndarray, world: int, rank: int):
    """Frames [lo, hi) of a head request: pos/neg [B, H], init [2B, 64] (cond rows then uncond rows)."""
    B = pos.shape[0]
    lo, hi = shard_range(B, world, rank)
    init_local = np.concatenate([init[lo:hi], init[B + lo:B + hi]])
    return pos[lo:hi], neg[lo:hi], init_local, (lo, hi)


def shard_prompts(arrays, batch: int, world: int, rank: int):
    """Prompts [lo, hi) of per-prompt arrays (leading dim = batch)."""
    lo, hi = shard_range(batch, world, rank)
    return [a[lo:hi] for a in arrays], (lo, hi)


def shard_prompts_rng(arrays, batch: int, world: int, rank: int):
    """Prompts [lo, hi) of one batched DiT request, plus the ``rng_batch=(lo, batch)`` slice that makes this
    shard's per-step noise (DPM++ 3M SDE, SA3 pingpong) the batched call's own draw: torch's TensorIterator
    Philox layout depends on the total element count, so a shard that sampled on its own would draw a
    different stream (b2d_dit_request / b2d_sa3_request ``rng_batch_total`` / ``rng_batch_first``)."""
    local, (lo, hi) = shard_prompts(arrays, batch, world, rank)
    return local, (lo, hi), (lo, batch)


def gather_rows(local, n_total: int, world: int):
    """All ranks' row blocks (contiguous shard_range order) -> the full [n_total, ...] tensor on every rank.

    `local` is a torch tensor on this rank's device; shards may differ in length by one, so each
    is padded to the largest share for the collective and trimmed afterwards."""
    import torch
    import torch.distributed as dist
    if world == 1:
        return local
    counts = [shard_range(n_total, world, r) for r in range(world)]
    cap = max(hi - lo for lo, hi in counts)
    pad = torch.zeros((cap,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[:local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad)
    return torch.cat([parts[r][:hi - lo] for r, (lo, hi) in enumerate(counts)])
