"""Tensor-parallel shards on the GPU.

* One GPU: a shard handle (yskn_b200_matrix_create_shard: rows [r0, r1), columns
  [c0, c1) cut from the whole tensor's code stream) gives exactly the whole tensor's
  int64 sums restricted to those rows, with the activation groups outside [c0, c1)
  dropped (oracle sums with those integer scales set to zero), for both file layouts.
* Two GPUs (skipped with fewer): yskn_b200/tp.py over NCCL, row-parallel with the
  MAX and int64 SUM all-reduces and column-parallel with the row gather, bit-identical
  to the one-GPU operator.
"""
import os
import socket

import numpy as np
import pytest

import fixtures
import oracle as O

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


@pytest.mark.parametrize("layout,bits", [("warp", 6), ("row", 8), ("warp", 4)])
def test_shard_sums_are_the_restricted_whole_sums(cuda, layout, bits):
    import torch
    import yskn_b200
    rows, cols = 1536, 2048
    words, lut16, sc16 = fixtures.model_matrix(rows, cols, bits, 77)  # random bits: valid in either layout
    si = O.signs("mulberry32_7919_13", 7, 0, cols)
    so = O.signs("mulberry32_7919_13", 7, cols, rows)
    dw = _dev(words.view(np.int32))
    M = 3
    rnd = fixtures.FixtureRandom(9)
    act = rnd.take(M * cols).astype(np.uint8).view(np.int8).reshape(M, cols).copy()
    A = (rnd.take(M * (cols // 512)) % 100000).astype(np.int32).reshape(M, -1)
    lut8, _ = O.quantize_weight_table(lut16, sc16)
    for r0, r1, c0, c1 in [(512, 1536, 512, 1536), (0, 512, 0, 2048), (1024, 1536, 1536, 2048)]:
        m = yskn_b200.Matrix(dw, layout, rows, rows, cols, bits, lut16, sc16, si, so, shard=(r0, r1, c0, c1))
        out = torch.empty((M, r1 - r0), dtype=torch.int64, device="cuda")
        yskn_b200.weighted_sums([m], _dev(act[:, c0:c1]), _dev(A[:, c0 // 512:c1 // 512]), [out])
        Am = A.copy()
        Am[:, :c0 // 512] = 0
        Am[:, c1 // 512:] = 0
        ref = O.fast_weighted_sums(words, layout, rows, cols, bits, lut8, act, Am)[:, r0:r1]
        assert np.array_equal(out.cpu().numpy(), ref)


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    import yskn_b200
    from yskn_b200 import tp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    try:
        M, cols = 2, 4096
        x = fixtures.normal(5, M * cols).reshape(M, cols)
        words, lut16, sc16 = fixtures.model_matrix(2048, cols, 8, 11)
        si = O.signs("mulberry32_7919_13", 7, 0, cols)
        so = O.signs("mulberry32_7919_13", 7, cols, 2048)
        dw = _dev(words.view(np.int32))
        rp = tp.RowParallelLinear(dw, "warp", 2048, 2048, cols, 8, lut16, sc16, si, so)
        y = torch.empty((M, 2048), dtype=torch.float32, device="cuda")
        rp(_dev(x[:, rp.col_begin:rp.col_end]), y)
        cp = tp.ColumnParallelLinear(dw, "warp", 2048, 2048, cols, 8, lut16, sc16, si, so)
        yl = torch.empty((M, cp.rows), dtype=torch.float32, device="cuda")
        cp(_dev(x), yl)
        yc = tp.gather_rows(yl, cp.ranges)
        torch.cuda.synchronize()
        assert yskn_b200.status() == 0
        q.put((rank, y.cpu().numpy(), yc.cpu().numpy()))
    finally:
        dist.destroy_process_group()


def test_tp_two_gpus_bit_identical(cuda):
    import torch
    import torch.multiprocessing as mp
    import yskn_b200
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    M, cols = 2, 4096
    x = fixtures.normal(5, M * cols).reshape(M, cols)
    words, lut16, sc16 = fixtures.model_matrix(2048, cols, 8, 11)
    si = O.signs("mulberry32_7919_13", 7, 0, cols)
    so = O.signs("mulberry32_7919_13", 7, cols, 2048)
    m = yskn_b200.Matrix(_dev(words.view(np.int32)), "warp", 2048, 2048, cols, 8, lut16, sc16, si, so)
    work = torch.empty(yskn_b200.linear_work_bytes([m], M), dtype=torch.uint8, device="cuda")
    y1 = torch.empty((M, 2048), dtype=torch.float32, device="cuda")
    yskn_b200.linear([m], _dev(x), work, [y1])
    ref = y1.cpu().numpy()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, y, yc in results:
        assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))
        assert np.array_equal(yc.view(np.uint32), ref.view(np.uint32))


def _rowpar_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    import yskn_b200
    from yskn_b200 import tp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    try:
        out = {}
        ex = tp.make_exchange(2048)
        mats = {}
        for name, (rows, cols, seed) in _ROWPAR_SHAPES.items():
            words, lut16, sc16 = fixtures.model_matrix(rows, cols, 8, seed)
            si = O.signs("mulberry32_7919_13", 7, 0, cols)
            so = O.signs("mulberry32_7919_13", 7, cols, rows)
            mats[name] = tp.RowParallelLinear(_dev(words.view(np.int32)), "warp", rows, rows, cols, 8, lut16, sc16,
                                              si, so, exchange=ex)
        # Interleaved calls, three rounds: the exchange cycles through its epochs and both slots.
        for rnd in range(3):
            for name, (rows, cols, seed) in _ROWPAR_SHAPES.items():
                M = 1 + (rnd + len(name)) % 3
                x = fixtures.normal(seed + 100 * rnd, M * cols).reshape(M, cols)
                rp = mats[name]
                y = torch.empty((M, rows), dtype=torch.float32, device="cuda")
                rp(_dev(x[:, rp.col_begin:rp.col_end]), y)
                out[(name, rnd)] = y.cpu().numpy()
        # The same calls captured in a CUDA graph and replayed twice.
        st = torch.cuda.Stream()
        xs, ys = {}, {}
        for name, (rows, cols, seed) in _ROWPAR_SHAPES.items():
            x = fixtures.normal(seed + 999, cols).reshape(1, cols)
            rp = mats[name]
            xs[name] = _dev(x[:, rp.col_begin:rp.col_end])
            ys[name] = torch.empty((1, rows), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for name in _ROWPAR_SHAPES:
                mats[name](xs[name], ys[name], stream=st)
        for rep in range(2):
            for y in ys.values():
                y.zero_()
            torch.cuda.synchronize()
            g.replay()
            torch.cuda.synchronize()
            for name in _ROWPAR_SHAPES:
                out[(name, "graph%d" % rep)] = ys[name].cpu().numpy()
        del g
        assert yskn_b200.status() == 0
        torch.cuda.synchronize()
        dist.barrier()  # no rank has kernels in flight before the areas are unmapped
        ex.close()
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


_ROWPAR_SHAPES = {"o": (1024, 3072, 21), "down": (2048, 4096, 23)}


def test_tp_rowpar_one_launch_two_gpus_bit_identical(cuda):
    """yskn_b200_linear_rowpar on 2 GPUs (row maxima and int64 block sums exchanged over
    NVLink inside the kernel) gives the one-GPU operator's bits, for interleaved
    matrices, M = 1..3, repeated rounds and CUDA-graph replays."""
    import torch
    import torch.multiprocessing as mp
    import yskn_b200
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ref = {}
    for name, (rows, cols, seed) in _ROWPAR_SHAPES.items():
        words, lut16, sc16 = fixtures.model_matrix(rows, cols, 8, seed)
        si = O.signs("mulberry32_7919_13", 7, 0, cols)
        so = O.signs("mulberry32_7919_13", 7, cols, rows)
        m = yskn_b200.Matrix(_dev(words.view(np.int32)), "warp", rows, rows, cols, 8, lut16, sc16, si, so)
        cases = [(rnd, 1 + (rnd + len(name)) % 3, seed + 100 * rnd) for rnd in range(3)]
        cases += [("graph0", 1, seed + 999), ("graph1", 1, seed + 999)]
        for key, M, xseed in cases:
            x = fixtures.normal(xseed, M * cols).reshape(M, cols)
            work = torch.empty(yskn_b200.linear_work_bytes([m], M), dtype=torch.uint8, device="cuda")
            y = torch.empty((M, rows), dtype=torch.float32, device="cuda")
            yskn_b200.linear([m], _dev(x), work, [y])
            ref[(name, key)] = y.cpu().numpy()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rowpar_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, out in results:
        assert set(out) == set(ref)
        for k, y in out.items():
            assert np.array_equal(y.view(np.uint32), ref[k].view(np.uint32)), k


def test_rowpar_wait_for_a_peer_that_never_arrives_times_out(cuda):
    """A row-parallel launch whose peer never runs (world 2, rank 0 alone on one GPU; the
    peer's exchange area is valid memory that no kernel serves) gives up within a short
    wait limit and reports YSKN_ETIMEDOUT; the device stays usable afterwards."""
    import time
    import torch
    import yskn_b200
    rows, cols = 2048, 4096
    words, lut16, sc16 = fixtures.model_matrix(rows, cols, 8, 23)
    si = O.signs("mulberry32_7919_13", 7, 0, cols)
    so = O.signs("mulberry32_7919_13", 7, cols, rows)
    dw = _dev(words.view(np.int32))
    shard = yskn_b200.Matrix(dw, "warp", rows, rows, cols, 8, lut16, sc16, si, so, shard=(0, rows, 0, cols // 2))
    ex0 = yskn_b200.TpExchange(2, 0, rows)
    ex1 = yskn_b200.TpExchange(2, 1, rows)  # the absent peer's area: never connected, never launched
    ex0.connect_peers([None, ex1.area])
    ex0.set_wait(0.002)
    x = _dev(fixtures.normal(5, cols // 2).reshape(1, cols // 2))
    y = torch.empty((1, rows), dtype=torch.float32, device="cuda")
    assert yskn_b200.status() == 0
    t0 = time.time()
    yskn_b200.linear_rowpar(ex0, shard, x, y)
    rc = yskn_b200.status()
    elapsed = time.time() - t0
    assert rc == yskn_b200.ETIMEDOUT
    assert elapsed < 2.0, elapsed  # two 2 ms limits, not one limit per polled word
    # The context still works: a plain operator call is correct.
    m = yskn_b200.Matrix(dw, "warp", rows, rows, cols, 8, lut16, sc16, si, so)
    xf = fixtures.normal(6, cols).reshape(1, cols)
    work = torch.empty(yskn_b200.linear_work_bytes([m], 1), dtype=torch.uint8, device="cuda")
    yskn_b200.linear([m], _dev(xf), work, [y])
    ref = O.linear(words, "warp", rows, cols, 8, lut16, sc16, xf, si, so)
    assert yskn_b200.status() == 0
    assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    ex0.close()
    ex1.close()
