"""Launches on several streams and inside CUDA graphs keep their order and
results: a layer's chain of kernels captured into a CUDA graph and replayed
gives the bits of the same chain run eagerly, and the end-to-end pattern of the
bench (row chunks over three streams, each chunk's host-to-device copies, kernel
and device-to-host copies on its stream) gives the bits of one whole-tensor
launch.  Both with launch overlap on, the library's default."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def layer_chain(v7g, r, d, w, o, codes, scales, y, wq, ws, stream=None):
    """add + RMSNorm -> RMSNorm -> Q8 -> Q8 GEMV -> add, each consuming the previous output."""
    v7g.fused_add_rmsnorm_rows(o, r, d, w, 1e-6, stream=stream)
    v7g.rmsnorm_quantize_rows(codes, scales, o, w, 1e-6, stream=stream)
    v7g.q8_gemv(y, codes[:4], scales[:4], wq, ws, stream=stream)
    v7g.add_inplace(r, o, stream=stream)


def test_graph_capture_replays_chain(cuda):
    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(5)
    rows, n, dout = 512, 2048, 1024
    r0 = torch.from_numpy(rng.standard_normal((rows, n), dtype=np.float32)).cuda()
    d = torch.from_numpy((0.5 * rng.standard_normal((rows, n))).astype(np.float32)).cuda()
    w = torch.from_numpy((1 + 0.1 * rng.standard_normal(n)).astype(np.float32)).cuda()
    wq = torch.from_numpy(rng.integers(-127, 128, (dout, n), dtype=np.int8)).cuda()
    ws = torch.from_numpy((0.001 + 0.01 * rng.random((dout, n // 64))).astype(np.float32)).cuda()
    r = r0.clone()
    o = torch.empty_like(r)
    codes = torch.empty(rows, n, dtype=torch.int8, device=r.device)
    scales = torch.empty(rows, n // 64, device=r.device)
    y = torch.empty(4, dout, device=r.device)

    # eager reference: two rounds
    for _ in range(2):
        layer_chain(v7g, r, d, w, o, codes, scales, y, wq, ws)
    torch.cuda.synchronize()
    want = [t.cpu().clone() for t in (r, o, codes, scales, y)]

    # the same two rounds from a captured graph (the eager run above did each
    # entry's one-time set-up, outside the capture)
    r.copy_(r0)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        layer_chain(v7g, r, d, w, o, codes, scales, y, wq, ws, stream=side)
    r.copy_(r0)  # capture does not execute
    torch.cuda.synchronize()
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    got = [t.cpu() for t in (r, o, codes, scales, y)]
    for a, b in zip(want, got):
        assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))
    del graph


def test_chunked_streams_match_single_launch(cuda):
    import v7multiplikator_b200 as v7g
    rows, n = 4096, 12288
    g = torch.empty(rows, n, device="cuda")
    u = torch.empty(rows, n, device="cuda")
    v7g.fill_normal(g, seed=21, mean=0.0, std=2.0)
    v7g.fill_normal(u, seed=22, mean=0.0, std=2.0)
    codes = torch.empty(rows, n, dtype=torch.int8, device="cuda")
    scales = torch.empty(rows, n // 64, device="cuda")
    v7g.swiglu_q8_rows(codes, scales, g, u)
    torch.cuda.synchronize()
    want_c, want_s = codes.cpu(), scales.cpu()

    hg = g.cpu().pin_memory()
    hu = u.cpu().pin_memory()
    hc = torch.empty(rows, n, dtype=torch.int8).pin_memory()
    hs = torch.empty(rows, n // 64).pin_memory()
    dg, du = torch.empty_like(g), torch.empty_like(u)
    dc, ds = torch.empty_like(codes), torch.empty_like(scales)
    streams = [torch.cuda.Stream() for _ in range(3)]
    cur = torch.cuda.current_stream()
    for rep in range(2):
        for s in streams:
            s.wait_stream(cur)
        for i, a in enumerate(range(0, rows, 256)):
            b = a + 256
            s = streams[i % 3]
            with torch.cuda.stream(s):
                dg[a:b].copy_(hg[a:b], non_blocking=True)
                du[a:b].copy_(hu[a:b], non_blocking=True)
                v7g.swiglu_q8_rows(dc[a:b], ds[a:b], dg[a:b], du[a:b], stream=s)
                hc[a:b].copy_(dc[a:b], non_blocking=True)
                hs[a:b].copy_(ds[a:b], non_blocking=True)
        for s in streams:
            cur.wait_stream(s)
        torch.cuda.synchronize()
        assert torch.equal(hc, want_c)
        assert torch.equal(hs.view(torch.int32), want_s.view(torch.int32))
        hc.zero_()
        hs.zero_()


def test_host_threads_on_own_streams(cuda):
    """Batched entries called from several host threads at once, each on its
    own stream (ctypes releases the interpreter lock during the call), give the
    results of one thread: the per-device one-time set-up and the launch path
    are safe to enter concurrently."""
    import threading

    import v7multiplikator_b200 as v7g
    rng = np.random.default_rng(9)
    n, dout, rows = 4096, 2048, 256
    wq = torch.from_numpy(rng.integers(-127, 128, (dout, n), dtype=np.int8)).cuda()
    ws = torch.from_numpy((0.001 + 0.01 * rng.random((dout, n // 64))).astype(np.float32)).cuda()
    w = torch.from_numpy((1 + 0.1 * rng.standard_normal(n)).astype(np.float32)).cuda()
    xs = [torch.from_numpy(rng.standard_normal((rows, n), dtype=np.float32)).cuda() for _ in range(4)]

    def work(x, stream):
        codes = torch.empty(rows, n, dtype=torch.int8, device="cuda")
        scales = torch.empty(rows, n // 64, device="cuda")
        y = torch.empty(2, dout, device="cuda")
        for _ in range(10):
            v7g.rmsnorm_quantize_rows(codes, scales, x, w, 1e-6, stream=stream)
            v7g.q8_gemv(y, codes[:2], scales[:2], wq, ws, stream=stream)
            v7g.q8_fused_gemv(y[1:], x[:1], wq, ws, stream=stream)
        stream.synchronize()
        return codes.cpu(), scales.cpu(), y.cpu()

    torch.cuda.synchronize()
    want = [work(x, torch.cuda.current_stream()) for x in xs]
    got = [None] * len(xs)
    errors = []

    def run(i):
        try:
            got[i] = work(xs[i], torch.cuda.Stream())
        except Exception as e:  # reported below
            errors.append(e)

    threads = [threading.Thread(target=run, args=(i,)) for i in range(len(xs))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    for a, b in zip(want, got):
        for ta, tb in zip(a, b):
            assert torch.equal(ta.view(torch.uint8), tb.view(torch.uint8))
