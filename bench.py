"""Benchmark of the compressed-integer linear path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--bits 8|6]

Workload (the reference's headline configuration): one hybrid layer's full linear set at batch-1
decode, hidden 5120 -- attention q/k/v/o, Gated-DeltaNet in_proj_qkv/in_proj_z/
out_proj, MLP gate/up/down -- on synthetic 27B-shape compressed weights (random
code words, seeded N(0,1) value table, row scales ~0.02; bits=8 is the format's
4-bit width, bits=6 the lowest). One step = the six operator calls of the layer
(q/k/v, o, qkv/z, out, gate/up, down; matrices sharing an input go in one call), each
from its input as the producer hands it over (int8 rows and group scales: the quantiser
runs in the producing kernel) -> exact int64 weighted sums -> restore + output H512 (one
launch per call at M=1, yskn_b200_linear_q8), captured in one CUDA graph. The metric is HBM throughput of the compressed weights:
algorithmic bytes per step / step time. Codes per step (243.8 MB at bits=8) exceed
the 126 MB L2, so no L2 flush is needed between steps.

With --gpus N > 1 (torchrun, one rank per GPU) every rank streams the linear set of
its own layer (independent matrices, as the layers of a model held on different GPUs;
no collective on the data path): the value is all ranks' bytes over the max-over-ranks
step time (weak scaling). The same line carries, measured on all ranks:
* `layer_tp`: one layer's set tensor-parallel (yskn_b200/tp.py): q/k/v, qkv/z and gate/up
  column-parallel over whole 512-row blocks (k/v replicated at 4 and 8 GPUs), o/out/down
  row-parallel over 512-column groups, each one launch per rank that exchanges the row
  maxima and the exact int64 block sums over NVLink (yskn_b200_linear_rowpar); the
  whole layer's bytes over the step time (strong scaling; `--layer-tp` makes it the line);
* `decode_27b`: the 27B-shape decode pass tensor-parallel (yskn_b200/tp_stack.py), one
  token stream over all ranks, tokens bit-identical to one GPU.

`--impl reference` times the CPU path instead: the C restatement (oracle/) of the
reference's CPU engine (crates/yskn-engine kernel + pool, crates/yskn-ref quantiser
and restore), on all host threads, rank 0 only.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "yasakani-for-mac_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import numpy as np  # noqa: E402

# (name, rows, cols); the reference model's shapes, docs/spec/01_MODEL_ARCHITECTURE.md:101-131
LAYER = [("q_proj", 12288, 5120), ("k_proj", 1024, 5120), ("v_proj", 1024, 5120), ("o_proj", 5120, 6144),
         ("in_proj_qkv", 10240, 5120), ("in_proj_z", 6144, 5120), ("out_proj", 5120, 6144),
         ("gate_proj", 17408, 5120), ("up_proj", 17408, 5120), ("down_proj", 5120, 17408)]
ROW_PARALLEL = {"o_proj", "out_proj", "down_proj"}
CALLS = [["q_proj", "k_proj", "v_proj"], ["o_proj"], ["in_proj_qkv", "in_proj_z"], ["out_proj"],
         ["gate_proj", "up_proj"], ["down_proj"]]
# DRAM bytes (read + write) of the six operator launches of one step (int8 inputs), summed
# over one ncu capture of this workload (bits 8, M 1: dram__bytes_read.sum +
# dram__bytes_write.sum); a static capture, not measured in the run (the line says so in
# roofline.traffic_source). None where no capture exists.
GEMV_TRAFFIC = {(8, 1): 248_117_248}
METRIC = "compressed GEMV HBM TB/s (one hybrid layer's linear set, batch-1 decode)"
UNIT = "TB/s"


def measured_peaks():
    """MEASURED_PEAKS.json (the pool's measured copy bandwidth and GEMM peaks), or {}."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


HBM_FALLBACK_GBS = 6650.0  # an earlier copy-bandwidth measurement on this pool, used without the file


def make_weights(bits, seed0=1000, signs=None):
    """The layer set's synthetic matrices. `signs(rule, seed, offset, n)` makes the sign
    streams: the library's host helper for the B200 arm, the oracle's for the CPU arm (so
    the reference arm never loads the product library)."""
    from yskn_b200 import synthetic
    if signs is None:
        import yskn_b200 as Y
        signs = Y.signs
    out = {}
    for i, (name, rows, cols) in enumerate(LAYER):
        words, lut16, sc16 = synthetic.model_matrix(rows, cols, bits, seed0 + 17 * i)
        out[name] = dict(rows=rows, cols=cols, words=words, lut16=lut16, sc16=sc16,
                         s_in=signs("mulberry32_7919_13", 7, 0, cols),
                         s_out=signs("mulberry32_7919_13", 7, cols, rows))
    return out


def make_inputs(M):
    from yskn_b200 import synthetic
    return [synthetic.normal(500 + j, M * LAYER_COLS[c[0]]).reshape(M, LAYER_COLS[c[0]]) for j, c in enumerate(CALLS)]


LAYER_COLS = {n: c for n, _, c in LAYER}
LAYER_ROWS = {n: r for n, r, _ in LAYER}


def algorithmic_bytes(bits, M):
    """Minimum bytes one step must move: codes + int8 table + f32 row scales + output signs
    per matrix, its f32 output; int8 input rows + f32 group scales per call."""
    total = 0
    for name, rows, cols in LAYER:
        total += rows * cols * bits // 16 + 8192 + 4 * rows + rows + 4 * M * rows
    for c in CALLS:
        total += M * LAYER_COLS[c[0]] + 4 * M * (LAYER_COLS[c[0]] // 512)
    return total


def gemv_bytes(rows, cols, bits, M):
    """Algorithmic bytes of one weighted-sums launch: codes + int8 table + int8
    activations + int32 group scales + int64 sums."""
    return rows * cols * bits // 16 + 8192 + M * cols + 4 * M * (cols // 512) + 8 * M * rows


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.proc, self.lines = index, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.index)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=lambda: self.lines.extend(iter(self.proc.stdout.readline, "")))
            self.thread.daemon = True
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clocks not sampled"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_inputs(W, xs):
    """Each call's int8 input, integer group scales and row quanta (the quantiser, run once
    outside the timed steps, as the GPU arm's inputs come quantised from their producer)."""
    import oracle as O
    out = []
    for c, x in zip(CALLS, xs):
        act, _, A, rq = O.quantize_activation(x, W[c[0]]["s_in"])
        out.append((act, A, rq))
    return out


def cpu_layer_step(W, qs, fraction=1.0, threads=None):
    """The CPU path for one step (the reference's CPU engine restated in C): threaded
    weighted sums from the quantised inputs (first `fraction` of each matrix's rows),
    restore."""
    import oracle as O
    nbytes = 0
    for c, (act, A, rq) in zip(CALLS, qs):
        for name in c:
            w = W[name]
            rows = max(32, int(w["rows"] * fraction) // 32 * 32)
            ws = O.fast_weighted_sums(w["words"], "warp", w["rows"], w["cols"], w["bits"], w["lut8"], act, A,
                                      rows=rows, threads=threads)
            if rows == w["rows"]:
                O.restore(ws, rq, w["tau"], w["s_out"])
            nbytes += rows * w["cols"] * w["bits"] // 16
    return nbytes


def prepare_cpu(W, bits):
    import oracle as O
    for w in W.values():
        w["lut8"], w["tau"] = O.quantize_weight_table(w["lut16"], w["sc16"])
        w["bits"] = bits


def run_reference(args, rank, world):
    if rank != 0:
        return
    import oracle as O
    W = make_weights(args.bits, signs=O.signs)
    prepare_cpu(W, args.bits)
    xs = cpu_inputs(W, make_inputs(1))
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    cpu_layer_step(W, xs, 1.0, threads)
    t_full = time.perf_counter() - t0
    budget = 90.0
    fraction = min(1.0, budget / max(1e-9, (args.steps + args.warmup) * t_full))
    for _ in range(args.warmup):
        cpu_layer_step(W, xs, fraction, threads)
    t0 = time.perf_counter()
    nbytes = 0
    for _ in range(args.steps):
        nbytes += cpu_layer_step(W, xs, fraction, threads)
    dt = time.perf_counter() - t0
    value = nbytes / dt / 1e12
    sample = ("each step: all 10 matrices of the layer set, first %.1f%% of rows (codes %.1f MB), threaded "
              "int64 sums from the quantised inputs%s" % (100 * fraction, nbytes / args.steps / 1e6,
                                         " + restore" if fraction >= 1.0 else ""))
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "i8", "data": "synthetic",
            "config": config(args),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    return line


def config(args):
    if args.gpus > 1 and args.layer_tp:
        par = "tp%d (column-parallel q/k/v, qkv/z, gate/up; row-parallel o, out, down)" % args.gpus
    elif args.gpus > 1:
        par = "layers%d: each rank streams its own layer's linear set (independent matrices), no collective" % args.gpus
    else:
        par = "single"
    return {"workload": "one hybrid layer's full linear set (q,k,v,o; GDN in_proj_qkv,in_proj_z,out_proj; "
                        "gate,up,down), batch-1 decode, hidden 5120",
            "bits": args.bits, "bits_per_weight": args.bits / 2, "M": 1,
            "codes_mb_per_step": sum(r * c * args.bits // 16 for _, r, c in LAYER) / 1e6,
            "l2": "inputs larger than L2: every step streams all codes (>126 MB); no flush",
            "parallelism": par}


def run_b200(args, rank, world, local_rank):
    import torch
    import yskn_b200 as Y
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    from yskn_b200 import tp
    tp_mode = world > 1 and args.layer_tp
    # N > 1 without tensor parallelism: every rank its own layer's matrices (another seed)
    W = make_weights(args.bits, seed0=1000 + (0 if tp_mode else 7919 * rank))
    # N > 1: tensor parallelism over whole 512-blocks (yskn_b200/tp.py). Column-parallel
    # projections keep whole 512-row blocks per rank (replicated when there are fewer
    # blocks than ranks: k/v at 4 and 8 GPUs); o/out/down are row-parallel, one launch
    # per rank and call with their exchange over NVLink (yskn_b200_linear_rowpar).
    mats, rowpar = {}, {}
    exchange = None
    if tp_mode:
        exchange = tp.make_exchange(max(r for n, r, _ in LAYER if n in ROW_PARALLEL))
    for name, w in W.items():
        dw = torch.from_numpy(w["words"].view(np.int32)).to(dev)
        args_m = (dw, "warp", w["rows"], w["rows"], w["cols"], args.bits, w["lut16"], w["sc16"], w["s_in"],
                  w["s_out"])
        if tp_mode and name in ROW_PARALLEL:
            rowpar[name] = tp.RowParallelLinear(*args_m, exchange=exchange)
            mats[name] = rowpar[name].mat
        else:
            shard = None
            if tp_mode:
                ranges = tp.split_blocks(w["rows"], world)
                r0, r1 = ranges[rank] if all(a < b for a, b in ranges) else (0, w["rows"])
                shard = (r0, r1, 0, w["cols"])
            mats[name] = Y.Matrix(*args_m, shard=shard)
        del dw
    M = 1
    xs_full = make_inputs(M)
    # Each call's input as its producer hands it over: int8 rows and per-group scales (the
    # quantiser runs in the producing kernel; yskn_b200_quantize here, once, untimed).
    # Row-parallel calls take this rank's column slice (their integer grid is set in the
    # launch from every rank's group scales).
    q_host = []
    for x, c in zip(xs_full, CALLS):
        kc = x.shape[1]
        act = torch.empty((M, kc), dtype=torch.int8, device=dev)
        alpha = torch.empty((M, kc // 512), dtype=torch.float32, device=dev)
        sgn = torch.from_numpy(np.ascontiguousarray(W[c[0]]["s_in"])).to(dev)
        Y.quantize(torch.from_numpy(x).to(dev), sgn.data_ptr(), act, alpha,
                   torch.empty((M, kc // 512), dtype=torch.int32, device=dev),
                   torch.empty(M, dtype=torch.float32, device=dev))
        a, al = act.cpu().numpy(), alpha.cpu().numpy()
        if c[0] in rowpar:
            c0, c1 = rowpar[c[0]].col_begin, rowpar[c[0]].col_end
            a, al = a[:, c0:c1], al[:, c0 // 512:c1 // 512]
        q_host += [np.ascontiguousarray(a).view(np.uint8), np.ascontiguousarray(al).view(np.uint8)]
    # A step's inputs (and its outputs) are views of one buffer, 256-byte aligned, so the
    # end-to-end step moves each direction with a single copy.
    def packed(shapes, dtype=torch.float32, **kw):
        offs, o = [], 0
        for s in shapes:
            offs.append(o)
            o += -(-int(np.prod(s)) // 256) * 256
        buf = torch.empty(o, dtype=dtype, **kw)
        return buf, [buf[a:a + int(np.prod(s))].view(*s) for a, s in zip(offs, shapes)]

    x_all, xb = packed([q.shape for q in q_host], dtype=torch.uint8, device=dev)
    for v, q in zip(xb, q_host):
        v.copy_(torch.from_numpy(q))
    xs = [(xb[2 * j].view(torch.int8), xb[2 * j + 1].view(torch.float32)) for j in range(len(CALLS))]
    out_shapes = [(M, mats[n].rows) for c in CALLS for n in c]
    y_all, y_flat = packed(out_shapes, device=dev)
    ys, k = [], 0
    for c in CALLS:
        ys.append(y_flat[k:k + len(c)])
        k += len(c)
    group = [[mats[n] for n in c] for c in CALLS]
    stream = torch.cuda.Stream(dev)

    def call(j, bx=None, by=None):  # the operator from int8 input: sums + restore (+ H512) in one launch
        c, (act, alpha), y = CALLS[j], (bx or xs)[j], (by or ys)[j]
        if c[0] in rowpar:
            Y.linear_rowpar_q8(exchange, rowpar[c[0]].mat, act, alpha, y[0], stream=stream)
        else:
            Y.linear_q8(group[j], act, alpha, y, stream=stream)

    def step(bx=None, by=None):
        for j in range(len(CALLS)):
            call(j, bx, by)

    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize()
    Y.check(Y.status(stream), "status")
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            graph.replay()
    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    ids = [v.strip() for v in visible.split(",") if v.strip()]
    sampler = ClockSampler(ids[local_rank] if local_rank < len(ids) else str(local_rank))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with sampler:
        barrier()
        e0.record(stream)
        torch.cuda.nvtx.range_push("timed")  # an ncu capture can select the timed launches by this range
        with torch.cuda.stream(stream):
            for _ in range(args.steps):
                graph.replay()
        torch.cuda.nvtx.range_pop()
        e1.record(stream)
        barrier()
        ms = e0.elapsed_time(e1)
        # Per call (informative): each of the step's launches captured alone in a graph
        # with events on the launching stream, replayed in step order (device time, no
        # host gaps; each figure holds one graph launch's latency).
        reps = max(20, min(200, args.steps))
        gemv_ms = [0.0] * len(CALLS)
        graphs = []
        for j in range(len(CALLS)):
            gg = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gg, stream=stream):
                call(j)
            graphs.append(gg)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in CALLS]
        with torch.cuda.stream(stream):
            for r in range(reps + 3):
                for j, gg in enumerate(graphs):
                    ev[j][0].record(stream)
                    gg.replay()
                    ev[j][1].record(stream)
                stream.synchronize()
                if r >= 3:
                    for j in range(len(CALLS)):
                        gemv_ms[j] += ev[j][0].elapsed_time(ev[j][1]) / reps
        # End to end through the public API, every step: its int8 inputs and group scales
        # copied in from pinned host memory, the six operator calls, its f32 outputs copied
        # back to pinned host memory. Steps run as a serving loop pipelines them: two device
        # buffer sets; a step's inputs go in on one copy stream while the step before it
        # computes, and its outputs come back on another while the step after it computes
        # (each copy ordered against the computations that use its buffer). Every step moves
        # its own bytes both ways; PIPE steps per graph, the first input and the last output
        # of each graph exposed.
        PIPE = 8
        xh_all, xh = packed([q.shape for q in q_host], dtype=torch.uint8, pin_memory=True)
        for v, q in zip(xh, q_host):
            v.copy_(torch.from_numpy(q))
        yh = [packed(out_shapes, pin_memory=True)[0] for _ in range(2)]
        x_all2, xb2 = packed([q.shape for q in q_host], dtype=torch.uint8, device=dev)
        xs2 = [(xb2[2 * j].view(torch.int8), xb2[2 * j + 1].view(torch.float32)) for j in range(len(CALLS))]
        y_all2, y_flat2 = packed(out_shapes, device=dev)
        ys2, k = [], 0
        for c in CALLS:
            ys2.append(y_flat2[k:k + len(c)])
            k += len(c)
        bufs = [(x_all, xs, y_all, ys), (x_all2, xs2, y_all2, ys2)]
        c_in, c_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        e2e_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(e2e_graph, stream=stream):
            fork = torch.cuda.Event()
            fork.record(stream)
            c_in.wait_event(fork)
            c_out.wait_event(fork)
            computed, returned = [], []
            for kk in range(PIPE):
                xa, bx, ya, by = bufs[kk % 2]
                if kk >= 2:
                    c_in.wait_event(computed[kk - 2])  # the step two back has read this input buffer
                with torch.cuda.stream(c_in):
                    xa.copy_(xh_all, non_blocking=True)
                arrived = torch.cuda.Event()
                arrived.record(c_in)
                stream.wait_event(arrived)
                if kk >= 2:
                    stream.wait_event(returned[kk - 2])  # its outputs have gone out of this buffer
                step(bx, by)
                computed.append(torch.cuda.Event())
                computed[-1].record(stream)
                c_out.wait_event(computed[-1])
                with torch.cuda.stream(c_out):
                    yh[kk % 2].copy_(ya, non_blocking=True)
                returned.append(torch.cuda.Event())
                returned[-1].record(c_out)
            stream.wait_event(returned[-1])
        e2e_replays = max(2, -(-max(10, min(args.steps, 500)) // PIPE))
        e2e_steps = e2e_replays * PIPE
        barrier()
        e2 = torch.cuda.Event(enable_timing=True)
        e3 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e2e_graph.replay()
            stream.synchronize()
            e2.record(stream)
            for _ in range(e2e_replays):
                e2e_graph.replay()
            e3.record(stream)
        barrier()
        e2e_ms = e2.elapsed_time(e3)
        # the pipelined steps computed what the plain step computes
        for (_, _, ya, _), yhb in zip(bufs, yh):
            if not torch.equal(yhb.view(torch.int32), y_all.view(torch.int32).cpu()):
                raise RuntimeError("pipelined end-to-end step: outputs differ from the timed step's")
    Y.check(Y.status(stream), "status")
    torch.cuda.synchronize()
    del graph, graphs, e2e_graph  # graphs holding NCCL calls go before the process group
    if exchange is not None:  # unmapped only once no rank has kernels in flight
        torch.distributed.barrier()
        exchange.close()
    t = torch.tensor([ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms, e2e_ms = t.tolist()
    # This rank's algorithmic bytes per step (its shards: codes, table, row scales, signs,
    # f32 input slice, f32 outputs), and its copies.
    if not tp_mode:
        gemv_local = algorithmic_bytes(args.bits, M)
    else:
        gemv_local = 0
        for c in CALLS:
            kc = mats[c[0]].cols
            gemv_local += M * kc + 4 * M * (kc // 512)
            for n in c:
                m = mats[n]
                out_rows = LAYER_ROWS[n] if n in rowpar else m.rows
                gemv_local += m.physical_rows * kc * args.bits // 16 + 8192 + 5 * m.physical_rows + 4 * M * out_rows
    h2d_local = x_all.numel()  # the copies as issued (inputs + alignment padding)
    d2h_local = 4 * y_all.numel()
    tot = torch.tensor([h2d_local, d2h_local], dtype=torch.int64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(tot)
    h2d, d2h = tot.tolist()
    # N > 1: the tensor-parallel layer set and decode pass, measured on every rank.
    layer_tp = decode = None
    if world > 1 and not tp_mode and not args.no_configs:
        import copy
        a = copy.copy(args)
        a.layer_tp, a.skip_stack, a.no_configs, a.skip_cpu = True, True, True, True
        a.steps = min(args.steps, 100)
        r = run_b200(a, rank, world, local_rank)
        layer_tp = _summary(r, us_per_call_alone=r["us_per_call_alone"]) if r else None
    if not args.skip_stack and not tp_mode:
        from yskn_b200 import stack as S
        sms, se2e, _ = measure_stack(dev, 64, 4096, args.bits, 20, 3, world)
        tb = S.token_bytes(64, S.VOCAB, 4096, args.bits)
        peak_d = measured_peaks().get("hbm_gbs", HBM_FALLBACK_GBS)
        decode = {"metric": STACK_METRIC, "value": 20 / (sms * 1e-3), "unit": "tok/s", "ms_per_token": sms / 20,
                  "e2e_tok_s": 20 / (se2e * 1e-3), "tokens": 20, "warmup": 3,
                  "hbm_frac": tb / (sms / 20 * 1e-3) / 1e9 / (peak_d * world), "bytes_per_token": tb,
                  "scaling": "strong" if world > 1 else "single",
                  "config": "64 layers (48 GDN + 16 attention, KV cache 4096 rows), vocab 151936, bits=%d, "
                            "seeded random weights, one CUDA graph per token%s" % (
                                args.bits, "; tensor-parallel over %d GPUs (yskn_b200/tp_stack.py)" % world
                                if world > 1 else "")}
    if rank != 0:
        return
    step_bytes = algorithmic_bytes(args.bits, M)
    jobs = 1 if tp_mode else world  # layer sets per step over all ranks
    value = jobs * step_bytes * args.steps / (ms * 1e-3) / 1e12
    e2e_value = jobs * step_bytes * e2e_steps / (e2e_ms * 1e-3) / 1e12
    peaks = measured_peaks()
    peak = peaks.get("hbm_gbs", HBM_FALLBACK_GBS)
    # The timed region is the dominant kernel's launches back to back (six fused
    # trellis_sums_kernel launches per step and rank, nothing else: the row-parallel exchange
    # runs inside them), so its average launch duration is the timed region's device
    # time / launches (inter-launch gaps in); per GPU, against one GPU's HBM peak.
    achieved = gemv_local * args.steps / (ms * 1e-3) / 1e9
    # CPU baseline (rank 0, N=1 only): the oracle port on a bounded sample.
    cpu = None
    if world == 1 and not args.skip_cpu:
        prepare_cpu(W, args.bits)
        threads = os.cpu_count() or 1
        t0 = time.perf_counter()
        n = 0
        nbytes = 0
        qs = cpu_inputs(W, xs_full)
        while time.perf_counter() - t0 < 10.0 or n < 2:
            nbytes += cpu_layer_step(W, qs, 1.0, threads)
            n += 1
        dt = time.perf_counter() - t0
        cpu = {"value": nbytes / dt / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": "%d full layer-set steps (threaded int64 sums from the quantised inputs + restore), "
                         "%.1f s" % (n, dt)}
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if tp_mode else "weak",
            "vs_baseline": None, "dtype": "i8", "data": "synthetic", "config": config(args),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": GEMV_TRAFFIC.get((args.bits, M)) if not tp_mode else None,
                         "traffic_source": "static ncu capture of this workload (not measured in this run)"
                         if GEMV_TRAFFIC.get((args.bits, M)) and not tp_mode else None,
                         "kernel": "trellis_sums_kernel (fused operator from int8 input: weighted sums + restore; the 6 "
                                   "launches of each step, timed over the timed region)" + (
                                       "; rank 0's shards, row-parallel calls exchanging over NVLink in-kernel"
                                       if tp_mode else "; per rank" if world > 1 else ""),
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback"},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            # One fused launch (quantise + sums + restore) per operator call at M=1, on
            # every rank (row-parallel calls included: their exchange is in the kernel).
            "gpu_launches": args.steps * len(CALLS),
            "clocks": sampler.summary(),
            "step_bytes": step_bytes, "us_per_call_alone": [round(1e3 * x, 2) for x in gemv_ms],
            "decode_27b": decode}
    if world > 1 and not tp_mode:
        line["layer_tp"] = layer_tp
    if world == 1 and not args.no_configs:
        line["configs"] = other_configs(args, rank, world, local_rank)
    return line


def _summary(line, **extra):
    """The figures of a sub-measurement that the default line carries."""
    keep = ("metric", "value", "unit", "ms_per_step", "roofline", "e2e", "config", "gpu_launches", "clocks")
    out = {k: line[k] for k in keep if k in line}
    out.update(extra)
    return out


def other_configs(args, rank, world, local_rank):
    """The path's other configurations, measured in the same run at N=1 so the default
    line records every one (each with its own roofline; no CPU baselines here, the
    dedicated --workload runs carry those): config 2 at the format's lowest width
    (bits 6), config 3 at M=4096 (tcgen05 GEMM) and M=8 (verify), config 4 at 32k and 2k."""
    import copy
    import torch
    out = {}

    def sub(name, fn, **kw):
        a = copy.copy(args)
        a.skip_cpu, a.skip_stack, a.no_configs = True, True, True
        a.steps = min(args.steps, 50)
        for k, v in kw.items():
            setattr(a, k, v)
        try:
            out[name] = _summary(fn(a, rank, world, local_rank))
        except Exception as e:  # a sub-measurement that fails is reported, not hidden
            out[name] = {"error": "%s: %s" % (type(e).__name__, e)}
        torch.cuda.synchronize()
        torch.cuda.empty_cache()

    if args.bits != 6:
        sub("linear_bits6", run_b200, bits=6)
    sub("gemm_4096", run_gemm, gemm_m=4096)
    sub("verify_8", run_gemm, gemm_m=8)
    sub("kv4_32k", run_kv, ctx=32768)
    sub("kv4_2k", run_kv, ctx=2048)
    return out


# --------------------------------------------------------------------- KV attention
# --workload kv4: config 4 of the path (24 query / 4 KV heads, head dim 256, packed
# 4-bit rows, one decode token). One step = the attention of the model's 16 attention
# layers (every fourth of 64), each layer with its own cache of `--ctx` rows, so the
# step streams 16 x 1056 x ctx bytes of cache (> L2 from ctx 8192; smaller contexts
# rotate over as many cache copies as exceed L2).
KV_QH, KV_KVH, KV_LAYERS = 24, 4, 16
KV_METRIC = "KV4 decode attention cache GB/s (24 q / 4 KV heads, 16 attention layers, one token)"


def kv_layer_bytes(ctx, M):
    """Algorithmic bytes of one layer: packed rows + row scales of both sides, both
    codebooks, value means, bf16 queries and gates in, bf16 outputs."""
    return KV_KVH * 2 * ctx * (128 + 4) + 2 * KV_KVH * 512 + KV_KVH * 1024 + 3 * M * KV_QH * 512


def kv_config(args, copies):
    return {"workload": "KV4 decode attention (config 4): 24 query / 4 KV heads, head dim 256, packed 4-bit "
                        "trellis rows, M=1, %d attention layers per step" % KV_LAYERS,
            "ctx": args.ctx, "splits": "one wave over the SMs" if args.kv_splits < 0 else args.kv_splits,
            "cache_mb_per_step": KV_LAYERS * 1056 * args.ctx / 1e6, "distinct_caches": copies,
            "l2": "the step's caches exceed L2 (126 MB); no flush",
            "parallelism": "KV heads over %d GPUs" % args.gpus if args.gpus > 1 else "single"}


def kv_host_inputs(ctx, layer):
    from yskn_b200 import synthetic
    kw, ks, vw, vs = synthetic.kv_cache(KV_KVH, ctx, 9000 + 13 * layer)
    book = np.tile(synthetic.kv_codebook_bf16(), (KV_KVH, 1))
    vmean = (synthetic.normal(7000 + layer, KV_KVH * 256) * np.float32(0.05)).reshape(KV_KVH, 256)
    bf = lambda x: ((x.view(np.uint32).astype(np.uint64) + 0x7FFF + ((x.view(np.uint32) >> 16) & 1)) >> 16)  # noqa
    q = bf(synthetic.normal(7100 + layer, KV_QH * 256)).astype(np.uint16).reshape(1, KV_QH, 256)
    gate = bf(synthetic.normal(7200 + layer, KV_QH * 256)).astype(np.uint16).reshape(1, KV_QH, 256)
    return kw, ks, vw, vs, book, vmean, q, gate


def cpu_kv_sample(args, seconds=10.0):
    """The oracle's attention (oracle/kv_oracle.c) on the host: whole query heads of one
    layer, as many as fit in `seconds`, each KV head's rows decoded once for its six
    query heads. Returns (GB/s of cache rows, query heads done, seconds)."""
    import kv
    kw, ks, vw, vs, book, vmean, q, _ = kv_host_inputs(args.ctx, 0)
    t0 = time.perf_counter()
    done, nbytes = 0, 0
    dec = {}
    while time.perf_counter() - t0 < seconds or done == 0:
        j = done % KV_QH
        h = j // (KV_QH // KV_KVH)
        if h not in dec:
            dec[h] = (kv.decode_packed_rows(kw[h], 4, book[h]), kv.decode_packed_rows(vw[h], 4, book[h]))
        qf = (q[0, j].astype(np.uint32) << 16).view(np.float32)
        kv.attend_head(qf, dec[h][0], ks[h], dec[h][1], vs[h], vmean[h], args.ctx, 31 if args.ctx < 4096 else 42)
        nbytes += 2 * args.ctx * 132 * (1.0 / (KV_QH // KV_KVH))  # a KV head's rows serve 6 query heads
        done += 1
    dt = time.perf_counter() - t0
    return nbytes / dt / 1e9, done, dt


def run_kv(args, rank, world, local_rank):
    import torch
    import yskn_b200 as Y
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    M = 1
    copies = max(KV_LAYERS, int(np.ceil(400e6 / (1056 * args.ctx))))  # cache copies: together > L2
    heads = [h for h in range(KV_KVH) if h % world == rank]  # KV heads of this rank (N > 1)
    nh = len(heads)
    layers = []
    for layer in range(copies):
        kw, ks, vw, vs, book, vmean, q, gate = kv_host_inputs(args.ctx, layer)
        qsel = np.concatenate([q[:, h * 6:(h + 1) * 6] for h in heads], axis=1) if nh else q[:, :0]
        gsel = np.concatenate([gate[:, h * 6:(h + 1) * 6] for h in heads], axis=1) if nh else gate[:, :0]
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
        layers.append(dict(kw=t(kw[heads].view(np.int32)), ks=t(ks[heads]), vw=t(vw[heads].view(np.int32)),
                           vs=t(vs[heads]), kb=t(book[heads].view(np.int16)), vb=t(book[heads].view(np.int16)),
                           vm=t(vmean[heads]), q=t(qsel.view(np.int16)), gate=t(gsel.view(np.int16)),
                           out=torch.empty((M, 6 * nh, 256), dtype=torch.int16, device=dev),
                           work=torch.empty(max(16, Y.kv4_attention_work_bytes(M, max(1, 6 * nh), args.ctx,
                                                                               args.kv_splits)),
                                            dtype=torch.uint8, device=dev)))
    stream = torch.cuda.Stream(dev)
    steps_per_graph = max(1, copies // KV_LAYERS)

    def step(layer_set):
        if not nh:
            return
        for L in layer_set:
            Y.kv4_attention(L["q"], L["kw"], L["ks"], L["vw"], L["vs"], L["kb"], L["vb"], args.ctx, L["work"],
                            L["out"], gate=L["gate"], v_mean=L["vm"], n_splits=args.kv_splits, stream=stream)

    # One graph = `steps_per_graph` steps of 16 layers over distinct caches.
    with torch.cuda.stream(stream):
        step(layers)
    torch.cuda.synchronize()
    Y.check(Y.status(stream), "status")
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step(layers[:steps_per_graph * KV_LAYERS])
    replays = max(1, -(-args.steps // steps_per_graph))
    steps = replays * steps_per_graph

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            graph.replay()
    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    ids = [v.strip() for v in visible.split(",") if v.strip()]
    sampler = ClockSampler(ids[local_rank] if local_rank < len(ids) else str(local_rank))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with sampler:
        barrier()
        e0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(replays):
                graph.replay()
        e1.record(stream)
        barrier()
        ms = e0.elapsed_time(e1)
        # End to end, every step: that step's 16 layers' queries and gates in from pinned
        # host memory (one copy), the attention, the gated outputs back (one copy); the
        # graph runs `steps_per_graph` such steps over the distinct caches.
        used = layers[:steps_per_graph * KV_LAYERS]
        per_step = []
        for s0 in range(0, len(used), KV_LAYERS):
            group = used[s0:s0 + KV_LAYERS]
            qg = torch.cat([torch.cat([L["q"].reshape(-1), L["gate"].reshape(-1)]) for L in group])
            outs = torch.cat([L["out"].reshape(-1) for L in group])
            o = 0
            for L in group:
                n = L["q"].numel()
                L["q"], L["gate"] = qg[o:o + n].view_as(L["q"]), qg[o + n:o + 2 * n].view_as(L["gate"])
                o += 2 * n
            o = 0
            for L in group:
                n = L["out"].numel()
                L["out"] = outs[o:o + n].view_as(L["out"])
                o += n
            per_step.append((group, qg, qg.cpu().pin_memory(), outs, torch.empty_like(outs, device="cpu").pin_memory()))
        e2e_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(e2e_graph, stream=stream):
            for group, qg, qg_host, outs, out_host in per_step:
                qg.copy_(qg_host, non_blocking=True)
                step(group)
                out_host.copy_(outs, non_blocking=True)
        e2e_replays = max(1, -(-max(10, min(args.steps, 200)) // steps_per_graph))
        barrier()
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e2e_graph.replay()
            stream.synchronize()
            e2.record(stream)
            for _ in range(e2e_replays):
                e2e_graph.replay()
            e3.record(stream)
        barrier()
        e2e_ms = e2.elapsed_time(e3)
    Y.check(Y.status(stream), "status")
    torch.cuda.synchronize()
    del graph, e2e_graph
    h2d, d2h = 2 * per_step[0][1].numel(), 2 * per_step[0][3].numel()
    t = torch.tensor([ms / steps, e2e_ms / (e2e_replays * steps_per_graph), h2d, d2h], dtype=torch.float64,
                     device=dev)
    if world > 1:
        mx = t[:2].clone()
        torch.distributed.all_reduce(mx, op=torch.distributed.ReduceOp.MAX)
        tot = t[2:].clone()
        torch.distributed.all_reduce(tot)
        t = torch.cat([mx, tot])
    ms_step, e2e_ms_step, h2d, d2h = t.tolist()
    if rank != 0:
        return
    step_bytes = KV_LAYERS * kv_layer_bytes(args.ctx, M)
    value = step_bytes / (ms_step * 1e-3) / 1e9
    peaks = measured_peaks()
    peak = peaks.get("hbm_gbs", HBM_FALLBACK_GBS)
    cpu = None
    if world == 1 and not args.skip_cpu:
        v, done, dt = cpu_kv_sample(args)
        cpu = {"value": v, "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": "%d query heads of one layer at ctx %d (oracle attention, 1 thread), %.1f s" %
                         (done, args.ctx, dt)}
    line = {"metric": KV_METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": kv_config(args, copies),
            "roofline": {"bound": "hbm", "achieved": value, "peak": peak, "unit": "GB/s", "frac": value / peak,
                         "traffic": None,
                         "kernel": "kv4_attention_kernel (splits, combine, inverse rotation and gate in one "
                                   "launch; the step's 16 launches, device time)",
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback"},
            "cpu_baseline": cpu,
            "e2e": {"value": step_bytes / (e2e_ms_step * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": steps * KV_LAYERS,
            "clocks": sampler.summary(), "step_bytes": step_bytes}
    return line


def run_reference_kv(args, rank, world):
    if rank != 0:
        return
    budget = max(5.0, min(60.0, 90.0 / max(1, args.steps + args.warmup)))
    for _ in range(args.warmup):
        cpu_kv_sample(args, 1.0)
    vals = [cpu_kv_sample(args, budget) for _ in range(max(1, min(args.steps, 3)))]
    value = float(np.median([v for v, _, _ in vals]))
    done = sum(d for _, d, _ in vals)
    sample = "%d query heads of one layer at ctx %d over %d samples (oracle attention, 1 thread)" % (
        done, args.ctx, len(vals))
    line = {"impl": "reference", "metric": KV_METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": kv_config(args, KV_LAYERS),
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": 1, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    return line


# ------------------------------------------------------------------------------ GEMM
# --workload gemm: config 3 of the path: the operator y = W x for M = --gemm-m tokens
# (4096: prefill, 8: speculative verify) on one 17408 x 5120 bits=8 matrix; M >= 64 runs
# the tcgen05 GEMM (predecode + kind::i8 MMA), smaller M the decode GEMV.
GEMM_N, GEMM_K = 17408, 5120
I8_PEAK_TOPS = 4375.8  # own tcgen05 kind::i8 dense peak on this pool (peak/i8_peak.cu microbenchmark)


def gemm_config(args):
    return {"workload": "prefill / verify operator (config 3): y = W x, W 17408 x 5120 bits=8 (4 b/w), M=%d" %
                        args.gemm_m, "M": args.gemm_m, "N": GEMM_N, "K": GEMM_K, "bits": 8,
            "path": "tcgen05 kind::i8 GEMM" if args.gemm_m >= 64 else "decode GEMV",
            "l2": "codes 44.6 MB + predecoded int8 89 MB + activations per step (> L2 at M=4096); "
                  "the M=8 step streams the 44.6 MB of codes",
            "parallelism": "single"}


def run_gemm(args, rank, world, local_rank):
    import torch
    import yskn_b200 as Y
    from yskn_b200 import synthetic
    if world > 1:
        raise SystemExit("--workload gemm runs on one GPU")
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    M, N, K = args.gemm_m, GEMM_N, GEMM_K
    words, lut16, sc16 = synthetic.model_matrix(N, K, 8, 4242)
    si = Y.signs("mulberry32_7919_13", 7, 0, K)
    so = Y.signs("mulberry32_7919_13", 7, K, N)
    dw = torch.from_numpy(words.view(np.int32)).to(dev)
    mat = Y.Matrix(dw, "warp", N, N, K, 8, lut16, sc16, si, so)
    del dw
    x_host = torch.from_numpy(synthetic.normal(77, M * K).reshape(M, K)).pin_memory()
    x = x_host.to(dev)
    y = torch.empty((M, N), dtype=torch.float32, device=dev)
    y_host = torch.empty((M, N), dtype=torch.float32).pin_memory()
    work = torch.empty(Y.linear_work_bytes([mat], M), dtype=torch.uint8, device=dev)
    act = torch.empty((M, K), dtype=torch.int8, device=dev)
    alpha = torch.empty((M, K // 512), dtype=torch.float32, device=dev)
    scales = torch.empty((M, K // 512), dtype=torch.int32, device=dev)
    rq = torch.empty(M, dtype=torch.float32, device=dev)
    ws = torch.empty((M, N), dtype=torch.int64, device=dev)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        Y.linear([mat], x, work, [y], stream=stream)
        Y.quantize(x, mat.signs_in_ptr, act, alpha, scales, rq, stream=stream)
        Y.weighted_sums([mat], act, scales, [ws], stream=stream)
    torch.cuda.synchronize()
    Y.check(Y.status(stream), "status")

    def timed(fn, reps):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            fn()
        with torch.cuda.stream(stream):
            for _ in range(max(3, args.warmup)):
                g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            e1.record(stream)
            torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) / reps

    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    ids = [v.strip() for v in visible.split(",") if v.strip()]
    sampler = ClockSampler(ids[local_rank] if local_rank < len(ids) else str(local_rank))
    with sampler:
        ms = timed(lambda: Y.linear([mat], x, work, [y], stream=stream), args.steps)
        sums_ms = timed(lambda: Y.weighted_sums([mat], act, scales, [ws], stream=stream), args.steps)

        def e2e():
            x.copy_(x_host, non_blocking=True)
            Y.linear([mat], x, work, [y], stream=stream)
            y_host.copy_(y, non_blocking=True)
        e2e_ms = timed(e2e, max(5, min(args.steps, 50)))
    Y.check(Y.status(stream), "status")
    ops = 2.0 * M * N * K
    value = ops / (ms * 1e-3) / 1e12
    achieved = ops / (sums_ms * 1e-3) / 1e12
    cpu = None
    if not args.skip_cpu:
        import oracle as O
        lut8, _ = O.quantize_weight_table(lut16, sc16)
        act8, _, A, _ = O.quantize_activation(x_host.numpy()[:min(M, 64)], si)
        threads = os.cpu_count() or 1
        t0 = time.perf_counter()
        rows_done = 0
        while time.perf_counter() - t0 < 10.0 or rows_done == 0:
            O.fast_weighted_sums(words, "warp", N, K, 8, lut8, act8, A, rows=2048, threads=threads)
            rows_done += 2048
        dt = time.perf_counter() - t0
        cpu = {"value": 2.0 * act8.shape[0] * rows_done * K / dt / 1e12, "unit": "TOPS", "cores": threads,
               "kind": "port", "sample": "%d tokens x %d weight rows x 5120 (threaded int64 sums), %.1f s" %
                                        (act8.shape[0], rows_done, dt)}
    tensor = M >= 64
    hbm_peak = measured_peaks().get("hbm_gbs", HBM_FALLBACK_GBS)
    line = {"metric": "compressed linear TOPS (config 3, M=%d)" % M, "value": value, "unit": "TOPS", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "i8", "data": "synthetic", "config": gemm_config(args),
            "roofline": ({"bound": "tensor", "achieved": achieved, "peak": I8_PEAK_TOPS, "unit": "TOPS",
                          "frac": achieved / I8_PEAK_TOPS, "traffic": None,
                          "kernel": "trellis_predecode_kernel + trellis_mma_kernel (weighted sums), device time",
                          "peak_source": "own tcgen05 kind::i8 microbenchmark (peak/i8_peak.cu) on this pool"}
                         if tensor else
                         {"bound": "hbm", "achieved": (N * K / 2 + 8192 + M * K + 8 * M * N) / (sums_ms * 1e-3) / 1e9,
                          "peak": hbm_peak, "unit": "GB/s", "traffic": None, "kernel": "trellis_sums_kernel (weighted sums)",
                          "frac": (N * K / 2 + 8192 + M * K + 8 * M * N) / (sums_ms * 1e-3) / 1e9 / hbm_peak,
                          "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in measured_peaks() else "fallback"}),
            "cpu_baseline": cpu,
            "e2e": {"value": ops / (e2e_ms * 1e-3) / 1e12, "unit": "TOPS", "h2d_bytes_per_step": 4 * M * K,
                    "d2h_bytes_per_step": 4 * M * N},
            "gpu_launches": args.steps * (4 if tensor else 1), "clocks": sampler.summary(),
            "weighted_sums_ms": sums_ms}
    return line


def run_reference_gemm(args, rank, world):
    """The reference's CPU path (the oracle's C restatement of the threaded engine kernel)
    on a bounded sample of the config-3 operator, on all host threads."""
    if rank != 0:
        return
    import oracle as O
    from yskn_b200 import synthetic
    words, lut16, sc16 = synthetic.model_matrix(GEMM_N, GEMM_K, 8, 4242)
    si = O.signs("mulberry32_7919_13", 7, 0, GEMM_K)
    lut8, _ = O.quantize_weight_table(lut16, sc16)
    m = min(args.gemm_m, 64)
    act8, _, A, _ = O.quantize_activation(synthetic.normal(77, m * GEMM_K).reshape(m, GEMM_K), si)
    threads = os.cpu_count() or 1
    budget = max(2.0, min(30.0, 90.0 / max(1, args.steps + args.warmup)))
    for _ in range(args.warmup):
        O.fast_weighted_sums(words, "warp", GEMM_N, GEMM_K, 8, lut8, act8, A, rows=512, threads=threads)
    vals = []
    for _ in range(max(1, min(args.steps, 3))):
        t0, rows = time.perf_counter(), 0
        while time.perf_counter() - t0 < budget or rows == 0:
            O.fast_weighted_sums(words, "warp", GEMM_N, GEMM_K, 8, lut8, act8, A, rows=2048, threads=threads)
            rows += 2048
        vals.append(2.0 * m * rows * GEMM_K / (time.perf_counter() - t0) / 1e12)
    value = float(np.median(vals))
    line = {"impl": "reference", "metric": "compressed linear TOPS (config 3, M=%d)" % args.gemm_m, "value": value,
            "unit": "TOPS", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "i8", "data": "synthetic",
            "config": gemm_config(args),
            "cpu_baseline": {"value": value, "unit": "TOPS", "cores": threads, "kind": "port",
                             "sample": "%d tokens x 2048-row blocks of the 17408 x 5120 matrix, %d samples of "
                                       "%.0f s (threaded int64 sums)" % (m, len(vals), budget)},
            "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    return line


STACK_METRIC = "27B-shape decode tok/s (64-layer hybrid stack, batch 1)"


def stack_config(args):
    return {"workload": "config 5: %d-layer hybrid stack (every 4th layer attention 24q/4kv x 256 with a 4-bit KV "
                        "cache of %d rows, the rest Gated DeltaNet 16/48 heads x 128), hidden 5120, MLP 17408, vocab "
                        "151936, bits=%d body and head, batch 1, greedy token fed back on the device" %
                        (args.layers, args.stack_ctx, args.bits),
            "global_batch": 1,
            "parallelism": "tp%d (yskn_b200/tp_stack.py)" % int(os.environ.get("WORLD_SIZE", "1"))
            if int(os.environ.get("WORLD_SIZE", "1")) > 1 else "1 GPU",
            "l2": "weights of one token (~13 GB) far exceed L2"}


def measure_stack(dev, layers, ctx, bits, steps, warmup, world=1, seed=1, sampler=None):
    """Times the decode pass (yskn_b200/stack.py; N > 1 tensor-parallel, yskn_b200/
    tp_stack.py, every rank) replayed as one CUDA graph per token: returns (device ms for
    `steps` tokens, max over ranks; e2e ms with the host's 4-byte token in and out per
    token; launches per token of one rank)."""
    import torch
    import yskn_b200 as Y
    from yskn_b200 import stack as S
    if world > 1:
        from yskn_b200.tp_stack import TPStack
        st = TPStack(dev, layers=layers, ctx=ctx, bits=bits, seed=seed)
    else:
        st = S.Stack(dev, layers=layers, ctx=ctx, bits=bits, seed=seed)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        st.decode(stream)  # eager once: per-device set-up happens outside capture
    torch.cuda.synchronize()
    Y.check(Y.status(stream), "status")
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        st.decode(stream)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    with torch.cuda.stream(stream):
        for _ in range(max(3, warmup)):
            graph.replay()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    import contextlib
    with sampler if sampler is not None else contextlib.nullcontext():
        with torch.cuda.stream(stream):
            e0.record(stream)
            torch.cuda.nvtx.range_push("timed")
            for _ in range(steps):
                graph.replay()
            torch.cuda.nvtx.range_pop()
            e1.record(stream)
        barrier()
    ms = e0.elapsed_time(e1)
    # end to end: the host supplies each token (4 bytes from pinned memory) and reads the
    # next one back (4 bytes) before the following step, as a chat loop does
    tok_in = torch.zeros(1, dtype=torch.int32).pin_memory()
    tok_out = torch.zeros(1, dtype=torch.int32).pin_memory()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e2.record(stream)
        for _ in range(steps):
            st.token.copy_(tok_in, non_blocking=True)
            graph.replay()
            tok_out.copy_(st.token, non_blocking=True)
            stream.synchronize()
            tok_in.copy_(tok_out)
        e3.record(stream)
    barrier()
    e2e_ms = e2.elapsed_time(e3)
    Y.check(Y.status(stream), "status")
    launches = st.launches_per_token()
    del graph  # holds an NCCL call at N > 1: released before the exchange and the process group
    if world > 1:
        st.close()
        t = torch.tensor([ms, e2e_ms], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, e2e_ms = t.tolist()
    del st
    torch.cuda.empty_cache()
    return ms, e2e_ms, launches


def run_reference_stack(args, rank, world):
    """CPU arm of --workload stack: the operator port on the host cores over the layer set,
    its code bytes per second divided by one token's bytes (linears only, an upper bound
    on a CPU decode rate; the mixers, attention and head are not timed). Rank 0 only."""
    from yskn_b200 import stack as S
    if rank != 0:
        return
    import oracle as O
    W = make_weights(args.bits, signs=O.signs)
    prepare_cpu(W, args.bits)
    xs = cpu_inputs(W, make_inputs(1))
    threads = os.cpu_count() or 1
    tb = S.token_bytes(args.layers, S.VOCAB, args.stack_ctx, args.bits)
    for _ in range(max(1, min(args.warmup, 3))):
        cpu_layer_step(W, xs, 1.0, threads)
    t0 = time.perf_counter()
    n, nbytes = 0, 0
    while n < args.steps and (time.perf_counter() - t0 < 60.0 or n < 1):
        nbytes += cpu_layer_step(W, xs, 1.0, threads)
        n += 1
    dt = time.perf_counter() - t0
    value = (nbytes / dt) / tb
    sample = ("%d full layer-set steps of the CPU operator port (%.1f s), code bytes/s divided by one token's "
              "bytes (linears only)" % (n, dt))
    return ({"impl": "reference", "metric": STACK_METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
                      "steps": n, "warmup": args.warmup, "ms_per_step": 1e3 / value, "higher_is_better": True,
                      "scaling": "weak", "vs_baseline": None, "dtype": "i8", "data": "synthetic",
                      "config": stack_config(args),
                      "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                                       "sample": sample},
                      "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})


def run_stack(args, rank, world, local_rank):
    """The whole decode pass per token as one CUDA graph (yskn_b200/stack.py). N > 1 runs it
    tensor-parallel (yskn_b200/tp_stack.py): one token stream over all ranks, value =
    tokens/s of that stream (strong scaling)."""
    import torch
    from yskn_b200 import stack as S
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    ids = [v.strip() for v in visible.split(",") if v.strip()]
    sampler = ClockSampler(ids[local_rank] if local_rank < len(ids) else str(local_rank))
    ms, e2e_ms, launches = measure_stack(dev, args.layers, args.stack_ctx, args.bits, args.steps, args.warmup,
                                         world, 1, sampler)
    if rank != 0:
        return
    value = args.steps / (ms * 1e-3)
    e2e_value = args.steps / (e2e_ms * 1e-3)
    tb = S.token_bytes(args.layers, S.VOCAB, args.stack_ctx, args.bits)
    peaks = measured_peaks()
    peak = peaks.get("hbm_gbs", HBM_FALLBACK_GBS)
    achieved = tb / (ms / args.steps * 1e-3) / 1e9 / world  # per GPU (each streams 1/N of the weights)
    cpu = None
    if world == 1 and not args.skip_cpu:
        W = make_weights(args.bits)
        prepare_cpu(W, args.bits)
        xs = cpu_inputs(W, make_inputs(1))
        threads = os.cpu_count() or 1
        t0 = time.perf_counter()
        n, nbytes = 0, 0
        while time.perf_counter() - t0 < 10.0 or n < 1:
            nbytes += cpu_layer_step(W, xs, 1.0, threads)
            n += 1
        dt = time.perf_counter() - t0
        cpu = {"value": (nbytes / dt) / tb, "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": "%d full layer-set steps of the CPU operator port (%.1f s), its code bytes/s divided by "
                         "one token's bytes (linear operators only; no mixer, attention or head work)" % (n, dt)}
    line = {"metric": STACK_METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None, "dtype": "i8", "data": "synthetic (seeded random codes and weights)",
            "config": stack_config(args),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "bytes_per_token": tb,
                         "kernel": "the whole decode pass (all kernels of one token), algorithmic bytes per token",
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback"},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4},
            "gpu_launches": args.steps * launches,
            "clocks": sampler.summary()}
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--bits", type=int, default=8, choices=[6, 8])
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-stack", action="store_true", help="linear: leave out the 27B-shape decode pass")
    ap.add_argument("--workload", default="linear", choices=["linear", "kv4", "gemm", "stack"])
    ap.add_argument("--layers", type=int, default=64, help="stack: layers (every fourth attention)")
    ap.add_argument("--stack-ctx", type=int, default=4096, help="stack: KV cache rows per attention layer")
    ap.add_argument("--gemm-m", type=int, default=4096, help="gemm: activation rows (4096 prefill, 8 verify)")
    ap.add_argument("--ctx", type=int, default=32768, help="kv4: cache rows per layer")
    ap.add_argument("--kv-splits", type=int, default=-1, help="kv4: 0 reference schedule, -1 one wave over the SMs")
    ap.add_argument("--no-configs", action="store_true", help="linear: leave out the other configurations' figures")
    ap.add_argument("--layer-tp", action="store_true",
                    help="linear, N > 1: one layer's set tensor-parallel (strong scaling) instead of a set per rank")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = {"kv4": run_reference_kv, "gemm": run_reference_gemm, "stack": run_reference_stack}.get(
            args.workload, run_reference)(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    if world > 1:
        import datetime
        import torch
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local_rank))
    try:
        line = {"kv4": run_kv, "gemm": run_gemm, "stack": run_stack}.get(args.workload, run_b200)(args, rank, world,
                                                                                                     local_rank)
        if line is not None and rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
