"""CPU tests of the multi-GPU host logic (audio.cpp_b200/parallel.py) with world_size-2
gloo process groups: sharding keeps CFG pairs together, the final gather restores the
global order, and a rank that fails before the gather is reported on the host."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp



def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_range_partitions():
    par = _parallel()
    for n in (0, 1, 7, 8, 1024, 8193):
        for world in (1, 2, 3, 8):
            spans = [par.shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            assert max(h - l for l, h in spans) - min(h - l for l, h in spans) <= 1
    with pytest.raises(ValueError):
        par.shard_range(4, 2, 2)


def _parallel():
    import importlib.util
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("b2d_parallel", os.path.join(root, "audio.cpp_b200", "parallel.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_head_shard_keeps_cfg_pairs():
    par = _parallel()
    B, H = 7, 4
    pos = np.arange(B * H, dtype=np.float32).reshape(B, H)
    neg = -pos
    init = np.arange(2 * B * 64, dtype=np.float32).reshape(2 * B, 64)
    for rank in range(3):
        p, n, i, (lo, hi) = par.shard_head_inputs(pos, neg, init, 3, rank)
        assert np.array_equal(p, pos[lo:hi]) and np.array_equal(n, neg[lo:hi])
        assert np.array_equal(i[:hi - lo], init[lo:hi]) and np.array_equal(i[hi - lo:], init[B + lo:B + hi])


def _worker(rank, world, port, n_total, fail_rank, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import torch.distributed as dist
    par = _parallel()
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        lo, hi = par.shard_range(n_total, world, rank)
        if rank == fail_rank:
            raise RuntimeError("injected failure on rank %d" % rank)
        # stand-in for this rank's sampled latents: row r = r (global index) in every column
        local = torch.arange(lo, hi, dtype=torch.float32)[:, None].repeat(1, 64)
        full = par.gather_rows(local, n_total, world)
        q.put((rank, "ok", full[:, 0].tolist()))
    except Exception as e:  # reported to the parent on the host, never through a device fault
        q.put((rank, "error", str(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _spawn(n_total, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n_total, fail_rank, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    return sorted(res)


@pytest.mark.parametrize("n_total", [8, 9])
def test_gather_restores_order_gloo(n_total):
    res = _spawn(n_total)
    for rank, status, rows in res:
        assert status == "ok", rows
        assert rows == list(range(n_total))


def test_failed_rank_is_reported_on_host():
    res = dict((r, (s, m)) for r, s, m in _spawn(8, fail_rank=1))
    assert res[1][0] == "error" and "injected failure" in res[1][1]
    # the surviving rank's gather ends with an error (peer gone / timeout), not a hang
    assert res[0][0] == "error"


def test_prompt_shards_carry_the_batched_noise_slice():
    """Each rank's rng_batch slice starts at its first prompt and names the whole batch, and the slices tile the
    batch in rank order (the device side, shards == the batched call, is test_gpu_dit / test_gpu_sa3's)."""
    par = _parallel()
    batch, T = 5, 7
    noise = np.arange(batch * 64 * T, dtype=np.float32).reshape(batch, 64, T)
    for world in (1, 2, 3):
        covered = []
        for rank in range(world):
            (local,), (lo, hi), (first, total) = par.shard_prompts_rng([noise], batch, world, rank)
            assert first == lo and total == batch and local.shape[0] == hi - lo
            assert np.array_equal(local, noise[lo:hi])
            covered += list(range(lo, hi))
        assert covered == list(range(batch))


def _shared_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    import importlib.util
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("b2d_bench", os.path.join(root, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import synth
        cfg = synth.HEAD_CONFIGS["tiny_q8"]
        calls = []

        def make(c):
            calls.append(rank)
            return synth.head_weights(c)

        w = bench.node_shared(make, cfg)
        ref = synth.head_weights(cfg)
        same = sorted(w) == sorted(ref) and all(np.array_equal(w[k].data, ref[k].data) for k in ref)
        q.put((rank, same, len(calls)))
    finally:
        dist.destroy_process_group()


def test_bench_weights_synthesised_once_per_node():
    """bench.py's ranks on one node share one synthesis of the seeded weights: only local rank 0 runs it and
    every rank ends with the same bytes."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shared_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == [(0, True, 1), (1, True, 0)]


def _mismatch_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    import importlib.util
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    spec = importlib.util.spec_from_file_location("b2d_bench", os.path.join(root, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    from oracle import synth
    cfg = synth.HEAD_CONFIGS["tiny_q8" if rank == 0 else "tiny_f16"]  # ranks disagree: no shared file
    w = bench.node_shared(synth.head_weights, cfg, wait_s=2.0)
    ref = synth.head_weights(cfg)
    q.put((rank, all(np.array_equal(w[k].data, ref[k].data) for k in ref)))


def test_bench_weight_sharing_never_hangs_on_a_mismatch():
    """Ranks that pass different configs each end with their own weights after the wait limit, not a hang."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_mismatch_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == [(0, True), (1, True)]
    import glob
    import tempfile
    for f in glob.glob(os.path.join(tempfile.gettempdir(), "b2d_bench_%d_*" % os.getpid())):
        os.remove(f)  # the writer leaves its file when a reader never came
