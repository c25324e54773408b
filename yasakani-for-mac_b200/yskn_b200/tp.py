"""Tensor parallelism of the compressed linear operator: one process per GPU,
torch.distributed (NCCL over NVLink) for the exchanges, the CUDA library for all
arithmetic.

The split follows the format's 512-blocks (docs/FORMAT.md: output rotations act on
512-row blocks, activation groups are 512 columns):

* Column-parallel projections (gate/up, q/k/v, the Gated-DeltaNet input projections)
  give each rank whole 512-row blocks of physical rows. Each rank quantises the
  (replicated) input itself and restores and rotates its own rows: no collective.
  A projection with fewer blocks than ranks is replicated.
* Row-parallel projections (down, o_proj, out_proj) give each rank whole 512-column
  groups and take that rank's slice of the input. Two exchanges make the result
  bit-identical to one GPU:
    1. all-reduce MAX of each activation row's largest group scale (M floats): the
       integer group scales A_g = rne(alpha_g * 2^24 / max) are defined over the whole
       row (crates/yskn-ref/src/compressed_linear.rs:113-128), and
       yskn_b200_rescale puts every rank on that grid;
    2. all-reduce SUM of the int64 weighted sums (exact and associative).
  Every rank then restores (+ output H512) the whole output row.

`ops` is the compute backend: the `yskn_b200` module (the CUDA library) unless a
test substitutes a CPU stand-in to exercise this host logic on gloo ranks.
"""
import torch
import torch.distributed as dist

import yskn_b200 as _cuda_ops


def split_blocks(extent, world, block=512):
    """Contiguous balanced split of ceil(extent / block) blocks over `world` ranks:
    [(begin, end)] in elements per rank (ends clipped to `extent`)."""
    nb = -(-extent // block)
    base, rem = divmod(nb, world)
    out, b = [], 0
    for r in range(world):
        n = base + (1 if r < rem else 0)
        out.append((min(b * block, extent), min((b + n) * block, extent)))
        b += n
    return out


def _rank_world(group):
    return dist.get_rank(group), dist.get_world_size(group)


class ColumnParallelLinear:
    """Physical rows [row_begin, row_end) of a tensor on this rank (whole 512-row blocks)."""

    def __init__(self, d_codes, layout, rows, physical_rows, cols, bits, lut16, scale16, signs_in, signs_out=None,
                 group=None, ops=None):
        self.ops = ops or _cuda_ops
        rank, world = _rank_world(group)
        ranges = split_blocks(physical_rows, world)
        if any(r0 >= min(r1, rows) for r0, r1 in ranges):  # fewer real blocks than ranks: replicate
            ranges = [(0, physical_rows)] * world
        self.ranges = ranges
        self.row_begin, self.row_end = ranges[rank]
        self.mat = self.ops.Matrix(d_codes, layout, rows, physical_rows, cols, bits, lut16, scale16, signs_in,
                                   signs_out, shard=(self.row_begin, self.row_end, 0, cols))
        self.rows = self.mat.rows  # logical rows of this shard
        self._work = {}

    def __call__(self, x, y, inv_rms=None, stream=None):
        """x: f32 [M][cols] (the whole input, replicated); y: f32 [M][self.rows]."""
        M = x.shape[0]
        if M not in self._work:
            self._work[M] = torch.empty(self.ops.linear_work_bytes([self.mat], M), dtype=torch.uint8,
                                        device=x.device)
        self.ops.linear([self.mat], x, self._work[M], [y], inv_rms=inv_rms, stream=stream)
        return y


def make_exchange(max_physical_rows, group=None, ops=None):
    """This rank's exchange area of the one-launch row-parallel operator
    (yskn_b200_linear_rowpar), connected to every peer's: the CUDA IPC handles travel
    once through the process group (all_gather_object), the data then moves GPU to GPU
    over NVLink without NCCL. Sized for matrices of up to max_physical_rows rows."""
    ops = ops or _cuda_ops
    rank, world = _rank_world(group)
    rows = -(-max_physical_rows // 512) * 512
    ex = ops.TpExchange(world, rank, rows)
    handles = [None] * world
    dist.all_gather_object(handles, ex.ipc_handle, group=group)
    ex.connect(handles)
    dist.barrier(group=group)  # every rank mapped before anyone sends
    return ex


class RowParallelLinear:
    """Columns [col_begin, col_end) of a tensor on this rank (whole 512-column groups).

    With `exchange` (make_exchange) a call with M <= 16 rows on a matrix with an output
    rotation is one launch per rank (yskn_b200_linear_rowpar: the row maxima and the
    int64 block sums travel over NVLink inside the kernel); otherwise the NCCL path
    below (quantise, all-reduce MAX, rescale, sums, all-reduce SUM, restore)."""

    def __init__(self, d_codes, layout, rows, physical_rows, cols, bits, lut16, scale16, signs_in, signs_out=None,
                 group=None, ops=None, exchange=None):
        self.ops = ops or _cuda_ops
        self.group = group
        self.exchange = exchange
        rank, world = _rank_world(group)
        self.ranges = split_blocks(cols, world)
        self.col_begin, self.col_end = self.ranges[rank]
        if self.col_begin >= self.col_end:
            raise ValueError("row-parallel split leaves a rank without a 512-column group")
        self.mat = self.ops.Matrix(d_codes, layout, rows, physical_rows, cols, bits, lut16, scale16, signs_in,
                                   signs_out, shard=(0, physical_rows, self.col_begin, self.col_end))
        self.rows, self.physical_rows = rows, physical_rows
        self._buf = {}

    def _buffers(self, M, device):
        if M not in self._buf:
            kc = self.col_end - self.col_begin
            G = kc // 512
            self._buf[M] = dict(
                act=torch.empty((M, kc), dtype=torch.int8, device=device),
                alpha=torch.empty((M, G), dtype=torch.float32, device=device),
                scales=torch.empty((M, G), dtype=torch.int32, device=device),
                rq=torch.empty(M, dtype=torch.float32, device=device),
                ws=torch.empty((M, self.physical_rows), dtype=torch.int64, device=device))
        return self._buf[M]

    def __call__(self, x_local, y, inv_rms=None, stream=None):
        """x_local: f32 [M][col_end - col_begin] (this rank's slice of the input);
        y: f32 [M][rows], the whole output, identical on every rank."""
        M = x_local.shape[0]
        ops = self.ops
        if self.exchange is not None and M <= 16 and self.mat.has_rotation:
            ops.linear_rowpar(self.exchange, self.mat, x_local, y, inv_rms=inv_rms, stream=stream)
            return y
        b = self._buffers(M, x_local.device)
        ops.quantize(x_local, self.mat.signs_in_ptr, b["act"], b["alpha"], b["scales"], b["rq"], stream=stream)
        row_max = b["alpha"].amax(dim=1)
        dist.all_reduce(row_max, op=dist.ReduceOp.MAX, group=self.group)
        ops.rescale(b["alpha"], row_max, b["scales"], b["rq"], stream=stream)
        ops.weighted_sums([self.mat], b["act"], b["scales"], [b["ws"]], stream=stream)
        dist.all_reduce(b["ws"], op=dist.ReduceOp.SUM, group=self.group)
        ops.restore(b["ws"], b["rq"], inv_rms, self.mat, self.mat.has_rotation, self.rows, False, y, stream=stream)
        return y


def gather_rows(y_local, ranges, group=None):
    """All-gather the column-parallel outputs [M][rows of each rank] into [M][total rows]
    (shards padded to the largest for the collective)."""
    M = y_local.shape[0]
    width = max(r1 - r0 for r0, r1 in ranges)
    pad = torch.zeros((M, width), dtype=y_local.dtype, device=y_local.device)
    pad[:, :y_local.shape[1]] = y_local
    parts = [torch.empty_like(pad) for _ in ranges]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([p[:, :r1 - r0] for p, (r0, r1) in zip(parts, ranges)], dim=1)
