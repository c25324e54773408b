"""Tensor-parallel host logic (yskn_b200/tp.py) on gloo ranks, world size 2, on CPU.

The CUDA library cannot run here, so the ranks pass tp.py a CPU stand-in for its
compute backend built on the oracle (this file only; the product's backend is the
CUDA library and has no fallback). What is under test is tp.py itself: the 512-block
splits, the shard geometry, the all-reduce MAX of the row maxima followed by the
rescale, the exact int64 all-reduce SUM, the replicated restore and the row gather.
The bar: every rank's output equals the one-process oracle result bit for bit.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import fixtures
import oracle as O
from yskn_b200 import tp


def test_split_blocks_follow_512_blocks():
    assert tp.split_blocks(17408, 8) == [(0, 2560), (2560, 5120), (5120, 7168), (7168, 9216), (9216, 11264),
                                         (11264, 13312), (13312, 15360), (15360, 17408)]
    assert tp.split_blocks(1024, 4) == [(0, 512), (512, 1024), (1024, 1024), (1024, 1024)]
    assert tp.split_blocks(1000, 2) == [(0, 512), (512, 1000)]
    for extent, world in [(6144, 8), (12288, 8), (5120, 3), (151936, 8)]:
        r = tp.split_blocks(extent, world)
        assert r[0][0] == 0 and r[-1][1] == extent
        assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
        assert all(b % 512 == 0 for b, _ in r)


class _Mat:
    """A shard of a row-layout tensor, held as oracle inputs."""

    def __init__(self, words, layout, rows, phys, cols, bits, lut16, sc16, s_in, s_out=None, shard=None):
        assert layout == "row"
        r0, r1, c0, c1 = shard or (0, phys, 0, cols)
        w = np.asarray(words, np.uint32).reshape(phys, cols // 256, 4 * bits)
        self.words = np.ascontiguousarray(w[r0:r1, c0 // 256:c1 // 256]).ravel()
        self.rows, self.physical_rows, self.cols, self.bits = min(rows, r1) - r0, r1 - r0, c1 - c0, bits
        self.lut8, self.tau = O.quantize_weight_table(lut16, np.asarray(sc16)[r0:r1])
        self.lut16, self.sc16 = lut16, np.asarray(sc16)[r0:r1]
        self.signs_in_ptr = np.asarray(s_in, np.int8)[c0:c1]
        self.s_out = None if s_out is None else np.asarray(s_out, np.int8)[r0:r1]
        self.has_rotation = s_out is not None


class _OracleOps:
    Matrix = _Mat

    @staticmethod
    def quantize(x, signs, act, alpha, scales, rq, stream=None):
        a, al, A, r = O.quantize_activation(x.numpy(), signs)
        act.copy_(torch.from_numpy(a))
        alpha.copy_(torch.from_numpy(al))
        scales.copy_(torch.from_numpy(A))
        rq.copy_(torch.from_numpy(r))

    @staticmethod
    def rescale(alpha, row_max, scales, rq, stream=None):
        al = alpha.numpy().astype(np.float32)
        mx = row_max.numpy().astype(np.float32)
        with np.errstate(divide="ignore"):
            mult = np.where(mx > 0, np.float32(16777216.0) / mx, np.float32(0)).astype(np.float32)
        scales.copy_(torch.from_numpy(np.rint(al * mult[:, None]).astype(np.int32)))
        rq.copy_(torch.from_numpy((mx * np.float32(2.0 ** -24)).astype(np.float32)))

    @staticmethod
    def weighted_sums(mats, act, scales, outs, stream=None):
        for m, o in zip(mats, outs):
            o.copy_(torch.from_numpy(O.fast_weighted_sums(m.words, "row", m.physical_rows, m.cols, m.bits, m.lut8,
                                                          act.numpy(), scales.numpy(), threads=1)))

    @staticmethod
    def restore(ws, rq, inv_rms, m, rotate, n_rows, clear, y, stream=None):
        ir = None if inv_rms is None else inv_rms.numpy()
        y.copy_(torch.from_numpy(O.restore(ws.numpy(), rq.numpy(), m.tau, m.s_out if rotate else None, ir, n_rows)))

    @staticmethod
    def linear_work_bytes(mats, M):
        return 1

    @staticmethod
    def linear(mats, x, work, ys, inv_rms=None, stream=None):
        for m, y in zip(mats, ys):
            ir = None if inv_rms is None else inv_rms.numpy()
            y.copy_(torch.from_numpy(O.linear(m.words, "row", m.physical_rows, m.cols, m.bits, m.lut16, m.sc16,
                                              x.numpy(), m.signs_in_ptr, m.s_out, ir, m.rows)))


def _tensor(rows, cols, seed, rotated):
    words, lut16, sc16 = fixtures.model_matrix(rows, cols, 8, seed)
    si = O.signs("mulberry32_7919_13", 7, 0, cols)
    so = O.signs("mulberry32_7919_13", 7, cols, rows) if rotated else None
    return words, lut16, sc16, si, so


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        M = 3
        x = fixtures.normal(41, M * 2048).reshape(M, 2048)
        inv_rms = np.array([1.0, 0.5, 2.0], np.float32)
        # Row-parallel: 1024 x 2048 with an output rotation, 4 column groups -> 2 per rank.
        w, l16, s16, si, so = _tensor(1024, 2048, 3, True)
        rp = tp.RowParallelLinear(w, "row", 1024, 1024, 2048, 8, l16, s16, si, so, ops=_OracleOps)
        y = torch.empty((M, 1024), dtype=torch.float32)
        rp(torch.from_numpy(np.ascontiguousarray(x[:, rp.col_begin:rp.col_end])), y,
           inv_rms=torch.from_numpy(inv_rms))
        np.save(os.path.join(out_dir, "row_%d.npy" % rank), y.numpy())
        # Column-parallel: 1000 rows (1024 physical, 2 blocks) without rotation -> one block per rank.
        w2, l2, s2, si2, _ = _tensor(1024, 2048, 5, False)
        cp = tp.ColumnParallelLinear(w2, "row", 1000, 1024, 2048, 8, l2, s2, si2, None, ops=_OracleOps)
        yl = torch.empty((M, cp.rows), dtype=torch.float32)
        cp(torch.from_numpy(x), yl)
        full = tp.gather_rows(yl, [(r0, min(r1, 1000)) for r0, r1 in cp.ranges])
        np.save(os.path.join(out_dir, "col_%d.npy" % rank), full.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(300)
def test_tp_world2_matches_one_process(tmp_path):
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    M = 3
    x = fixtures.normal(41, M * 2048).reshape(M, 2048)
    inv_rms = np.array([1.0, 0.5, 2.0], np.float32)
    w, l16, s16, si, so = _tensor(1024, 2048, 3, True)
    ref = O.linear(w, "row", 1024, 2048, 8, l16, s16, x, si, so, inv_rms)
    w2, l2, s2, si2, _ = _tensor(1024, 2048, 5, False)
    ref2 = O.linear(w2, "row", 1024, 2048, 8, l2, s2, x, si2, None, None, 1000)
    for r in range(2):
        assert np.array_equal(np.load(tmp_path / ("row_%d.npy" % r)).view(np.uint32), ref.view(np.uint32))
        assert np.array_equal(np.load(tmp_path / ("col_%d.npy" % r)).view(np.uint32), ref2.view(np.uint32))


class _FakeExchange:
    """Stand-in for yskn_b200.TpExchange: a recognisable handle per rank; connect records
    what it was given."""

    def __init__(self, world, rank, rows):
        self.world, self.rank, self.rows = world, rank, rows
        self.ipc_handle = bytes([rank + 1]) * 64
        self.handles = None

    def connect(self, handles):
        self.handles = list(handles)


class _ExchangeOps(_OracleOps):
    TpExchange = _FakeExchange
    rowpar_calls = []

    @staticmethod
    def linear_rowpar(exchange, mat, x_local, y, inv_rms=None, stream=None):
        _ExchangeOps.rowpar_calls.append((exchange.rank, tuple(x_local.shape)))
        y.fill_(1.0)


def _exchange_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ex = tp.make_exchange(5000, ops=_ExchangeOps)
        # every rank holds every rank's handle, in rank order; the area is whole 512-blocks
        assert ex.handles == [bytes([r + 1]) * 64 for r in range(world)]
        assert (ex.world, ex.rank, ex.rows) == (world, rank, 5120)
        w, l16, s16, si, so = _tensor(1024, 2048, 3, True)
        rp = tp.RowParallelLinear(w, "row", 1024, 1024, 2048, 8, l16, s16, si, so, ops=_ExchangeOps, exchange=ex)
        x = fixtures.normal(41, 17 * 2048).reshape(17, 2048)
        xl = torch.from_numpy(np.ascontiguousarray(x[:, rp.col_begin:rp.col_end]))
        y = torch.zeros((2, 1024), dtype=torch.float32)
        rp(xl[:2], y)  # M <= 16 with a rotation: the one-launch operator
        assert _ExchangeOps.rowpar_calls == [(rank, (2, 1024))] and float(y.min()) == 1.0
        y17 = torch.empty((17, 1024), dtype=torch.float32)
        rp(xl, y17)  # M = 17: the NCCL path, which matches one process
        ref = O.linear(w, "row", 1024, 2048, 8, l16, s16, x, si, so, None)
        assert np.array_equal(y17.numpy().view(np.uint32), ref.view(np.uint32))
        assert len(_ExchangeOps.rowpar_calls) == 1
        np.save(os.path.join(out_dir, "ok_%d.npy" % rank), np.ones(1))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_tp_exchange_plumbing_world2(tmp_path):
    """make_exchange swaps the ranks' handles through the process group and connects
    each rank with all of them in rank order; RowParallelLinear takes the one-launch
    operator for M <= 16 and the NCCL path beyond."""
    mp.spawn(_exchange_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        assert (tmp_path / ("ok_%d.npy" % r)).exists()
