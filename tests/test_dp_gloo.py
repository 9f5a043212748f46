"""Multi-rank host logic on CPU (gloo, world size 2): sharding, the timing
max-reduction, and a rank that fails before the barrier.  No GPU involved."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from inspark_proper_format_b200.dp import RankContext, shard_range, weak_scaling_throughput


def test_shard_range_covers_exactly():
    for total in (0, 1, 7, 64, 128, 1001):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_weak_scaling_throughput():
    assert weak_scaling_throughput(10.0, 4, 2.0) == 20.0
    with pytest.raises(ValueError):
        weak_scaling_throughput(1.0, 1, 0.0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    try:
        ctx = RankContext.from_env(backend="gloo").init(timeout_s=10.0)
        if rank == fail_rank:
            raise RuntimeError("injected failure before the barrier")
        from oracle import fir as ofir
        b, c, t = 6, 3, 64
        x = np.random.default_rng(0).standard_normal((b, c, t)).astype(np.float32) * 0.5
        lo, hi = shard_range(b, world, rank)
        up, down = ofir.bigvgan_filters()
        a = np.linspace(0.5, 2.0, c).astype(np.float32)
        y = ofir.alias_free_snake(x[lo:hi], up, down, a, ofir.snake_inverse_beta(a))
        ctx.barrier()
        slowest = ctx.max_over_ranks(float(rank + 1))
        ctx.close()
        q.put((rank, "ok", lo, hi, y, slowest))
    except Exception as e:  # reported to the parent, never hangs
        q.put((rank, "error", repr(e), None, None, None))


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(results, key=lambda r: r[0])


def test_two_ranks_shard_and_reduce():
    res = _run(2)
    assert all(r[1] == "ok" for r in res), res
    from oracle import fir as ofir
    b, c, t = 6, 3, 64
    x = np.random.default_rng(0).standard_normal((b, c, t)).astype(np.float32) * 0.5
    up, down = ofir.bigvgan_filters()
    a = np.linspace(0.5, 2.0, c).astype(np.float32)
    full = ofir.alias_free_snake(x, up, down, a, ofir.snake_inverse_beta(a))
    stitched = np.concatenate([r[4] for r in res])
    np.testing.assert_array_equal(stitched, full)            # no data exchange needed
    assert all(r[5] == 2.0 for r in res)                      # max over ranks


def test_failed_rank_surfaces_as_error_not_hang():
    res = _run(2, fail_rank=1)
    assert res[1][1] == "error" and "injected" in res[1][2]
    assert res[0][1] == "error"                               # the survivor's barrier times out / errors


def _calib_worker(rank, world, port, q):
    """The bench's split of config 2: contiguous utterances per rank, the static scale
    calibrated as the max over the ranks' shard maxima, then each rank quantizes its rows."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    try:
        from oracle import normquant as onq
        from oracle.formats import bf16_round
        ctx = RankContext.from_env(backend="gloo").init(timeout_s=20.0)
        utts, frames, k = 8, 12, 64
        g = np.random.default_rng(1)
        x = bf16_round(g.standard_normal((utts * frames, k)).astype(np.float32) * 3)
        gamma = (g.random(k) * 0.2 + 0.9).astype(np.float32)
        u0, u1 = shard_range(utts, world, rank)
        y = onq.rms_norm_gptfast(x[u0 * frames:u1 * frames], gamma, 1e-6, True)
        scale = ctx.max_over_ranks(float(np.abs(y).max())) / 448.0
        codes = onq.quant_e4m3_static(y, np.float32(scale))
        ctx.close()
        q.put((rank, "ok", codes, scale))
    except Exception as e:  # reported to the parent, never hangs
        q.put((rank, "error", repr(e), None))


def test_contiguous_split_with_shared_calibration_equals_one_gpu():
    from oracle import normquant as onq
    from oracle.formats import bf16_round
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_calib_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=120) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert all(r[1] == "ok" for r in res), res
    g = np.random.default_rng(1)
    x = bf16_round(g.standard_normal((8 * 12, 64)).astype(np.float32) * 3)
    gamma = (g.random(64) * 0.2 + 0.9).astype(np.float32)
    y = onq.rms_norm_gptfast(x, gamma, 1e-6, True)
    full = onq.quant_e4m3_static(y, np.float32(float(np.abs(y).max()) / 448.0))
    assert res[0][3] == res[1][3]                                  # one scale on every rank
    np.testing.assert_array_equal(np.concatenate([r[2] for r in res]), full)


def test_strong_scaling_throughput():
    from inspark_proper_format_b200.dp import strong_scaling_throughput
    assert strong_scaling_throughput(10.0, 2.0) == 5.0
    with pytest.raises(ValueError):
        strong_scaling_throughput(1.0, 0.0)
