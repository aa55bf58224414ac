"""The multi-GPU host logic on CPU ranks (gloo, world size 2): row sharding,
the max-over-ranks timing reduction, the checksum gather, the whole-job output
verification against the oracle (with a planted mismatch), and a rank that
drops out being detected by the others instead of hanging them.  The
per-shard compute is the oracle (CPU), so the test covers the partitioning
and the collectives, not the kernels."""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _shard_worker(rank, world, port, q):
    sys.path.insert(0, str(ROOT))
    import bench
    from oracle.pyoracle import Oracle
    _init(rank, world, port)
    rows, n = 37, 256
    a, b = bench.shard(rows, rank, world)
    rng = np.random.default_rng(0)
    g = rng.normal(0, 2, (rows, n)).astype(np.float32)
    u = rng.normal(0, 2, (rows, n)).astype(np.float32)
    codes, scales = Oracle(nthreads=1).swiglu_q8(g[a:b], u[a:b])
    chk = bench.output_checksum(torch.from_numpy(codes), torch.from_numpy(scales))
    allchk = bench.gather_checksums(chk, world)
    tmax = bench.max_over_ranks(float(rank + 1), world, device="cpu")
    tsum = bench.sum_over_ranks(float(b - a), world, device="cpu")
    # whole-tensor reference on every rank, then split like the shards
    full_c, full_s = Oracle(nthreads=1).swiglu_q8(g, u)
    ref = [bench.output_checksum(torch.from_numpy(full_c[x:y]), torch.from_numpy(full_s[x:y])).tolist()
           for x, y in (bench.shard(rows, r, world) for r in range(world))]
    q.put((rank, allchk == ref, tmax, tsum))
    dist.destroy_process_group()


def _verify_worker(rank, world, port, q):
    """Each rank's shard of a small SwiGLU -> Q8 job, made by the oracle on the
    generator's inputs (the CPU stand-in for the kernel), through
    bench.verify_outputs; then once more with one code changed on rank 1."""
    sys.path.insert(0, str(ROOT))
    import bench
    from oracle.pyoracle import Oracle
    _init(rank, world, port)
    rows, n = 37, 256
    a, b = bench.shard(rows, rank, world)
    orc = Oracle(nthreads=1)
    g = orc.fill_normal(b - a, n, a, bench.SEED_GATE, 0.0, 2.0)
    u = orc.fill_normal(b - a, n, a, bench.SEED_UP, 0.0, 2.0)
    codes, scales = orc.swiglu_q8(g, u)
    good = bench.verify_outputs(torch.from_numpy(codes), torch.from_numpy(scales), rank, world, rows, n)
    if rank == 1:
        codes[3, 17] = codes[3, 17] + 1 if codes[3, 17] < 127 else 126
    bad = bench.verify_outputs(torch.from_numpy(codes), torch.from_numpy(scales), rank, world, rows, n)
    q.put((rank, good, bad))
    dist.destroy_process_group()


def _dropout_worker(rank, world, port, q):
    _init(rank, world, port, timeout_s=10)
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()  # flush the message before the abrupt exit
        os._exit(0)  # leaves between steps, nothing in flight
    try:
        t = torch.ones(1)
        dist.all_reduce(t)
        q.put((rank, "no error"))
    except Exception as e:  # the peer is gone: the collective must fail, not hang
        q.put((rank, f"error: {type(e).__name__}"))


def _run(fn, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = []
    for _ in range(world):
        out.append(q.get(timeout=timeout))
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return sorted(out)


def test_shards_cover_rows_exactly():
    sys.path.insert(0, str(ROOT))
    import bench
    for rows in (1, 7, 16384):
        for world in (1, 2, 3, 4, 8):
            spans = [bench.shard(rows, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == rows
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def test_two_rank_shard_gather_matches_single():
    res = _run(_shard_worker)
    for rank, ok, tmax, tsum in res:
        assert ok, f"rank {rank}: gathered shard checksums differ from the single-rank split"
        assert tmax == 2.0  # max over ranks of (rank + 1)
        assert tsum == 37.0  # shards cover all rows


def test_rank_dropout_is_detected():
    res = dict(_run(_dropout_worker, timeout=90))
    assert res[1] == "left"
    assert res[0].startswith("error"), res[0]


def test_two_rank_verification_against_oracle():
    res = _run(_verify_worker)
    for rank, good, bad in res:
        assert good["mismatches"] == 0 and bad["mismatches"] == 1, (rank, good, bad)
    r0 = res[0]
    assert r0[1]["codes"] == 37 * 256 and r0[1]["scales"] == 37 * 4 and r0[1]["rows"] == 37
    assert r0[2]["code_mismatches"] == 1 and r0[2]["scale_mismatches"] == 0
